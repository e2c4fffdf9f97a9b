"""Module path of the reference's collator (trainer/data/data_collator_with_packing.py); the
implementation is ``trainer.data.collator``."""
from .collator import DataCollatorWithPacking, shift_completion_mask

__all__ = ["DataCollatorWithPacking", "shift_completion_mask"]
