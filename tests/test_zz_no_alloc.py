"""The far read + merge entry point that allocates nothing (fold_far_read_merge_static).

It serves callers that cannot allocate device memory while they run the draft step, such as an
engine that plans all device buffers ahead of time and hands the attention plugin only the
step's tensors. Its split partials live in a static scratch array of the library, so this test
calls it through the C-ABI twice in a row (the second call reuses the scratch the first one
left behind) and checks each result against the regular entry points (fold_far_read with
caller-allocated partials, then fold_merge). This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from fold_b200 import _lib, kernels
from fold_b200.errors import FoldError
from fold_b200.rope import rope_table
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, lengths, side_from

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def make_step(seed, n, hq, hkv, hd, far_keys, window):
    rng = np.random.default_rng(seed)
    hist = far_keys + window
    L = hist + n
    side = side_from(rng.standard_normal((L, hkv, hd)), rng.standard_normal((L, hkv, hd)), -(-L // 256) + 1)
    q = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    o_l = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    lse_l = torch.from_numpy((rng.standard_normal((hq, n)) + 4).astype(np.float32)).cuda()
    table = rope_table(torch.from_numpy(fo.inv_freq(500000.0, hd)).cuda(), hist + window + 2 * n + 1, "cuda")
    qsl, seq = lengths(n, hist)
    return dict(side=side, q=q, o_l=o_l, lse_l=lse_l, table=table, qsl=qsl, seq=seq, n=n, hq=hq, hkv=hkv, hd=hd,
                window=window, scale=2.0 * hd ** -0.5, L=L)


def static_buffers(s):
    """The caller's own buffers of a call: output, far_len and the device error word."""
    return (torch.full((s["n"], s["hq"], s["hd"]), float("nan"), device="cuda", dtype=torch.bfloat16),
            torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda"))


def static_call(s, splits, bufs=None):
    out, far_len, err = bufs or static_buffers(s)
    q, o_l, lse_l, table, side = s["q"], s["o_l"], s["lse_l"], s["table"], s["side"]
    _lib.call("fold_far_read_merge_static", q.data_ptr(), q.stride(0), q.stride(1), s["qsl"].data_ptr(),
              s["seq"].data_ptr(), table.data_ptr(), table.shape[0], table.shape[1], side.data_ptr(), side.shape[0],
              0, s["L"], far_len.data_ptr(), o_l.data_ptr(), o_l.stride(0), o_l.stride(1), lse_l.data_ptr(),
              lse_l.stride(0), lse_l.stride(1), out.data_ptr(), out.stride(0), out.stride(1), splits, s["n"], s["hq"],
              s["hkv"], s["hd"], s["window"], s["n"], s["window"] + s["n"], s["scale"], 0.5, err.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return out, far_len, err


def regular_call(s, splits):
    n, hq, hd = s["n"], s["hq"], s["hd"]
    o_part = torch.empty((splits, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((splits, hq, n), device="cuda", dtype=torch.float32)
    kernels.far_read(s["q"], s["qsl"], s["seq"], s["side"], o_part, lse_part, window=s["window"], block=n,
                     far_distance=s["window"] + n, softmax_scale=s["scale"], table=s["table"], capacity=s["L"])
    out = torch.empty((n, hq, hd), device="cuda", dtype=torch.bfloat16)
    kernels.merge(s["o_l"], s["lse_l"], o_part, lse_part, out, s["qsl"], s["seq"], window=s["window"], block=n,
                  alpha=2.0)
    return out


def test_static_scratch_matches_regular_path_on_two_calls():
    # first call: 128K-context-like head layout, many splits; second call: a different step with
    # fewer splits and a shorter memory, which must not see the first call's partials
    first = make_step(1, 10, 32, 8, 128, 20000, 2048)
    second = make_step(2, 8, 16, 8, 256, 3000, 512)
    for s, splits in ((first, 18), (second, 5)):
        got, far_len, err = static_call(s, splits)
        want = regular_call(s, splits)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, "the static path recorded a device error"
        assert int(far_len.item()) == s["L"] - s["n"] - s["window"]
        assert torch.isfinite(got.float()).all()
        assert (got.float() - want.float()).abs().max().item() <= OUT_ATOL


def test_static_call_allocates_no_device_memory():
    """The property the entry point exists for: once the library is loaded on the device, a call
    changes neither the device's free memory nor the torch allocator's counters."""
    s = make_step(4, 10, 32, 8, 128, 20000, 2048)
    static_call(s, 18)  # first use on the device: loads the library's module (and its static array)
    bufs = static_buffers(s)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    stats0 = torch.cuda.memory_stats()
    static_call(s, 18, bufs)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    stats1 = torch.cuda.memory_stats()
    assert int(bufs[2].item()) == 0
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    for key in ("allocation.all.allocated", "segment.all.allocated", "reserved_bytes.all.allocated"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key


def test_static_scratch_rejects_oversize_requests():
    s = make_step(3, 10, 32, 8, 128, 1000, 256)
    with pytest.raises(FoldError, match="exceeds the static scratch"):
        static_call(s, 1000)  # 1000 * 10 * 32 * 129 floats > 4 Mi
