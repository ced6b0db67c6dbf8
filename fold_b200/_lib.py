"""ctypes binding of libfold_b200.so, the C-ABI declared in include/fold_b200.h.

The library is loaded on first use and never replaced by a Python or PyTorch fallback: if it is
missing, every kernel call raises FoldError.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .errors import FoldError

LIB_PATH = Path(__file__).resolve().with_name("libfold_b200.so")

_i32, _i64, _f32, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> argument types (every entry point returns int status unless listed in _RESTYPES)
SIGNATURES = {
    "fold_status_string": [_i32],
    "fold_last_error": [],
    "fold_version": [],
    "fold_num_sms": [],
    "fold_append": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i64, _i32, _vp, _vp],
    "fold_gather": [_vp, _i32, _i32, _i32, _i64, _vp, _i32, _vp, _vp, _vp, _vp],
    "fold_append_fp8": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _vp, _vp, _i64,
                        _i32, _vp, _vp],
    "fold_far_read_fp8": [_vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _vp, _vp, _vp,
                          _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp],
    "fold_far_query": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i32, _i32, _i32,
                       _i32, _i32, _vp, _vp],
    "fold_rerope_query": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32,
                          _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp],
    "fold_far_read": [_vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _vp, _i64, _i64, _vp,
                      _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp],
    "fold_far_read_default_splits": [_i32, _i32, _i32, _i32],
    "fold_far_read_kernel_for": [_i32, _i32, _i32, _i32],
    "fold_far_read_select_kernel": [_i32],
    "fold_merge": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _vp,
                   _i64, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp],
    "fold_combine": [_vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _vp],
    "fold_allgather_partials": [_vp, _vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _vp],
    "fold_window_read": [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i64, _i64, _i64, _vp, _i32, _i32, _i32,
                         _i32, _f32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp],
    "fold_step_read": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _vp,
                       _vp, _vp, _vp, _i64, _i32, _i64, _i64, _i64, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _i32, _vp,
                       _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _f32, _vp, _vp],
    "fold_merge_partials": [_vp, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _i32, _i32, _i32,
                            _i32, _f32, _vp],
    "fold_exchange_create": [_i32, _i32, _i64, _i32, ctypes.POINTER(ctypes.c_void_p), _vp],
    "fold_exchange_open": [_vp, _vp],
    "fold_exchange_destroy": [_vp],
    "fold_exchange_merge": [_vp, _vp, _vp, _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i32,
                            _i32, _i32, _i32, _i32, _f32, _vp, _vp],
    "fold_far_read_exchange": [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _vp, _vp,
                               _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                               _i32, _i32, _f32, _f32, _vp, _vp],
    "fold_far_read_merge_static": [_vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _vp, _i64,
                                   _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                   _i32, _f32, _f32, _vp, _vp],
}
_RESTYPES = {"fold_status_string": ctypes.c_char_p, "fold_last_error": ctypes.c_char_p}

_lock = threading.Lock()
_lib = None


def load():
    """The loaded library (raises FoldError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise FoldError(f"the FOLD CUDA library is missing ({LIB_PATH}); build it with "
                                "`python -m fold_b200.build`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, _i32)
            _lib = lib
    return _lib


_fns = {}


def call(name: str, *args) -> None:
    """Calls an entry point and raises FoldError on a non-zero status."""
    fn = _fns.get(name)
    if fn is None:
        fn = _fns[name] = getattr(load(), name)
    status = fn(*args)
    if status:
        lib = load()
        msg = lib.fold_last_error().decode(errors="replace")
        kind = lib.fold_status_string(status).decode()
        raise FoldError(f"{name}: {kind}: {msg}")


def num_sms() -> int:
    return int(load().fold_num_sms())


def default_splits(hkv: int, hd: int, n: int, hq: int) -> int:
    return int(load().fold_far_read_default_splits(hkv, hd, n, hq))


def far_read_kernel_for(hd: int, n: int, hq: int, hkv: int) -> int:
    return int(load().fold_far_read_kernel_for(hd, n, hq, hkv))
