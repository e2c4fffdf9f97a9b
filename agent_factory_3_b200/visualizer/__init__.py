"""Self-contained HTML viewer of rollout groups (CPU string generation, no graphics API)."""
from .app import create_groups_viewer

__all__ = ["create_groups_viewer"]
