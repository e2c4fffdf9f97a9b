"""DDIS loss and mergeable metric states."""
