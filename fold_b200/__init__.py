"""FOLD drafter attention on B200: position-free far memory with local order.

Drop-in for the reference package `fold` (fold/__init__.py): the same exports, backed by the
sm_100a CUDA library libfold_b200.so (see include/fold_b200.h).
"""
from .attention import FoldError, install, use_full_draft_storage

__all__ = ["FoldError", "install", "use_full_draft_storage"]
