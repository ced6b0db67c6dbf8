"""The C-ABI library loads without a GPU and exports every entry point include/fold_b200.h
declares; the Python binding declares the same set. No kernel is launched."""
import ctypes
import re
from pathlib import Path

import pytest

from fold_b200 import _lib
from fold_b200.errors import FoldError

HEADER = Path(__file__).resolve().parents[1] / "include" / "fold_b200.h"


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fold_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    for required in ("fold_append", "fold_far_query", "fold_far_read", "fold_merge", "fold_combine",
                     "fold_rerope_query", "fold_gather"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_lib.SIGNATURES) == declared()


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.fold_version() >= 1
    assert lib.fold_status_string(0) == b"ok"
    assert lib.fold_status_string(3) == b"misaligned pointer or stride"


def test_argument_errors_are_reported_without_a_gpu():
    # invalid sizes are rejected before any CUDA call
    with pytest.raises(FoldError, match="far read"):
        _lib.call("fold_far_read", None, 0, 0, None, None, None, 0, 0, None, 0, 0, 0, None, None, 0, 0, None, None,
                  1, 1, 1, 1, 128, 1, 1, 1, 1.0, None, None)
    with pytest.raises(FoldError, match="merge"):
        _lib.call("fold_merge", None, 0, 0, None, 0, 0, None, 0, 0, 0, 0, None, 0, 0, 0, 1, None, 0, 0, None, None,
                  1, 1, 128, 1, 1, 0.5, None)
    # an empty append is a no-op that needs no device
    _lib.call("fold_append", None, 0, 0, None, 0, 0, None, None, 0, None, 2, 1, 128, 0, 0, None, None)


def test_kernel_selection_validates():
    from fold_b200 import kernels
    with pytest.raises(FoldError):
        kernels.select_far_read_kernel("fastest")
    with pytest.raises(FoldError, match="far read kernel"):
        _lib.call("fold_far_read_select_kernel", 7)
    kernels.select_far_read_kernel("tc")
    kernels.select_far_read_kernel("auto")


def test_exchange_rejects_bad_arguments_without_a_gpu():
    import ctypes
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(64)
    with pytest.raises(FoldError, match="world"):
        _lib.call("fold_exchange_create", 9, 0, 64, 1, ctypes.byref(ptr), ctypes.cast(buf, ctypes.c_void_p))
    with pytest.raises(FoldError, match="world"):
        _lib.call("fold_exchange_create", 2, 2, 64, 1, ctypes.byref(ptr), ctypes.cast(buf, ctypes.c_void_p))
    with pytest.raises(FoldError, match="multiple of 4"):
        _lib.call("fold_exchange_create", 2, 0, 62, 1, ctypes.byref(ptr), ctypes.cast(buf, ctypes.c_void_p))
    with pytest.raises(FoldError, match="null pointer"):
        _lib.call("fold_exchange_merge", None, None, None, 1, None, 0, 0, None, 0, 0, None, 0, 0, None, None, 1, 1,
                  128, 1, 1, 0.5, None, None)
    _lib.call("fold_exchange_destroy", None)  # destroying nothing is a no-op


_CTYPES = {"void*": ctypes.c_void_p, "const void*": ctypes.c_void_p, "int*": ctypes.c_void_p,
           "const int*": ctypes.c_void_p, "float*": ctypes.c_void_p, "const float*": ctypes.c_void_p,
           "const int64_t*": ctypes.c_void_p, "void**": None, "int64_t": ctypes.c_int64, "int": ctypes.c_int,
           "float": ctypes.c_float}


def test_binding_argument_types_match_header():
    """Every ctypes argument list has the header's arity and types, position by position."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, params in re.findall(r"\b(fold_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        sig = _lib.SIGNATURES[name]
        assert len(params) == len(sig), name
        for p, t in zip(params, sig):
            kind = re.sub(r"\s+", " ", p.rsplit(" ", 1)[0].replace(" *", "*")).strip()
            if p.split()[-1].startswith("*"):
                kind += "*"
            want = _CTYPES[kind]
            if want is None:  # void** out-parameter
                assert t is not ctypes.c_int and t is not ctypes.c_float, (name, p)
            else:
                assert t is want, (name, p, t)


def test_far_read_kernel_choice_per_shape():
    from fold_b200 import kernels
    kernels.select_far_read_kernel("auto")
    try:
        # mma.sync tiles up to 48 query rows per KV head, tcgen05 tiles past that
        assert _lib.far_read_kernel_for(128, 8, 32, 8) == 0      # 32 rows
        assert _lib.far_read_kernel_for(256, 8, 16, 8) == 0      # 16 rows
        assert _lib.far_read_kernel_for(128, 12, 32, 8) == 0     # 48 rows
        assert _lib.far_read_kernel_for(128, 16, 32, 8) == 1     # 64 rows
        assert kernels.far_read_uses_tcgen05(128, 16, 32, 8)
        assert _lib.far_read_kernel_for(128, 8, 32, 5) == -1     # hq not a multiple of hkv
        assert _lib.far_read_kernel_for(128, 0, 32, 8) == -1
        kernels.select_far_read_kernel("mma")
        assert _lib.far_read_kernel_for(128, 16, 32, 8) == 0
        kernels.select_far_read_kernel("tc")
        assert _lib.far_read_kernel_for(128, 8, 32, 8) == 1
    finally:
        kernels.select_far_read_kernel("auto")


# Stand-in addresses that pass the alignment checks; every case below fails validation before
# any CUDA call, so nothing is dereferenced.
_P = 1 << 20


def _window_args(**kw):
    a = dict(q=_P, qst=4096, qsh=128, qsl=_P, seq=_P, kc=_P, vc=_P, num_blocks=64, block_size=16, sb=32768,
             sh=2048, ss=128, bt=_P, bt_len=8, wl=2063, wr=15, causal=1, scale=0.088, o=_P, lse=_P, splits=18,
             n=8, hq=32, hkv=8, hd=128, err=None, stream=None)
    a.update(kw)
    return list(a.values())


def test_window_read_rejects_bad_arguments_without_a_gpu():
    with pytest.raises(FoldError, match="window read: null pointer"):
        _lib.call("fold_window_read", *_window_args(bt=None))
    with pytest.raises(FoldError, match="head size"):
        _lib.call("fold_window_read", *_window_args(hd=64))
    with pytest.raises(FoldError, match="block size"):
        _lib.call("fold_window_read", *_window_args(block_size=8))
    with pytest.raises(FoldError, match="16-byte aligned"):
        _lib.call("fold_window_read", *_window_args(ss=100))
    with pytest.raises(FoldError, match="bad sizes"):
        _lib.call("fold_window_read", *_window_args(hkv=5))
    with pytest.raises(FoldError, match="at most 64"):
        _lib.call("fold_window_read", *_window_args(n=32))


def test_step_read_requires_a_plan_word():
    with pytest.raises(FoldError, match="step read: null plan"):
        # every pointer null and every size zero: the plan word is checked first
        args = [None if t is ctypes.c_void_p else 0 for t in _lib.SIGNATURES["fold_step_read"]]
        _lib.call("fold_step_read", *args)


def test_merge_partials_rejects_bad_arguments_without_a_gpu():
    base = [_P, _P, 18, _P, _P, 18, None, _P, 4096, 128, _P, _P, 8, 32, 128, 2048, 16, 0.5, None]
    with pytest.raises(FoldError, match="same slot count"):
        args = list(base)
        args[5], args[6] = 17, _P
        _lib.call("fold_merge_partials", *args)
    with pytest.raises(FoldError, match="head size"):
        args = list(base)
        args[14] = 130
        _lib.call("fold_merge_partials", *args)
    with pytest.raises(FoldError, match="null pointer"):
        args = list(base)
        args[3] = None
        _lib.call("fold_merge_partials", *args)
    with pytest.raises(FoldError, match="element pairs"):
        args = list(base)
        args[8] = 4095
        _lib.call("fold_merge_partials", *args)
