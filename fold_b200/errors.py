"""Error type of the FOLD path (fold/attention.py:40 of the reference)."""


class FoldError(ValueError):
    """An unsupported setup, a bad argument, or a failure reported by the CUDA library."""


# Bits of the device error word the kernels OR into (include/fold_b200.h).
DEVERR_APPEND_RANGE = 1
DEVERR_ROPE_RANGE = 2
DEVERR_TIMEOUT = 4
DEVERR_CAPACITY = 8
DEVERR_BLOCK_TABLE = 16

DEVERR_NAMES = {
    DEVERR_APPEND_RANGE: "append/gather position outside the side cache",
    DEVERR_ROPE_RANGE: "rotation offset beyond the rope table",
    DEVERR_TIMEOUT: "a pipeline wait of the far read gave up",
    DEVERR_CAPACITY: "far_len exceeds the side cache capacity",
    DEVERR_BLOCK_TABLE: "a window-read block-table entry outside the paged cache",
}


def describe_device_error(word: int) -> str:
    return "; ".join(msg for bit, msg in DEVERR_NAMES.items() if word & bit) or "none"
