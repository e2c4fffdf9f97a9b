"""Self-contained HTML viewer of rollout groups (CPU string generation, no graphics API):
``create_groups_viewer(group_results, title=...)``; ``load_saved_batch`` reads a batch saved by
``RolloutSaver`` back for re-rendering (``python -m agent_factory_3_b200.visualizer``)."""
from .app import create_groups_viewer, load_saved_batch

__all__ = ["create_groups_viewer", "load_saved_batch"]
