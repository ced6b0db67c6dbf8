"""The fp8 side cache, the far memory's storage-format option (e4m3 K and V^T with per-KV-head
scales, half the bytes per key of the bf16 side cache).

* fold_append_fp8 is bit-exact against the oracle's quantisation (the float32 product of the bf16
  value and the reciprocal scale, rounded to e4m3) and layout.
* fold_far_read_fp8 meets the output bar (max-abs 2e-2) and the LSE bar (1e-3 relative) against
  the oracle's far read over the dequantised keys and values: what the cache stores.
* Against the unquantised (bf16) memory it is an approximation: the accuracy study at the 128K
  Llama shape with x8 outlier channels prints its error and bounds the mean error and the LSE.
* FoldWorkspace(side_format="fp8") runs the FOLD forward on it.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from fold_b200 import kernels
from fold_b200.attention import FoldAttention, FoldWorkspace
from fold_b200.rope import rope_table
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, lengths, lse_close, paged_from, randn_kv, to64

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

HD = 128


def head_scales(x):
    """Per-KV-head scale amax / 448 (float32), the calibration that uses the whole e4m3 range."""
    return (np.abs(x).max(axis=(0, 2)) / 448.0).astype(np.float32)


def side8_bits(side8):
    return side8.cpu().numpy()


def f16_round(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)


def test_append_fp8_bit_exact():
    rng = np.random.default_rng(8)
    hkv, max_len = 3, 700
    pages = fo.side_pages(max_len)
    side8 = torch.zeros(kernels.fp8_side_shape(pages, hkv), device="cuda", dtype=torch.uint8)
    ref = np.zeros(tuple(side8.shape), dtype=np.uint8)
    ks = np.array([0.01, 0.05, 0.003], dtype=np.float32)
    vs = np.array([0.02, 0.004, 0.03], dtype=np.float32)
    ks_t, vs_t = torch.from_numpy(ks).cuda(), torch.from_numpy(vs).cuda()
    # a prefill chunk across page halves and pages, a step with one rejected slot, an overwrite,
    # single positions at page edges
    calls = [(np.arange(0, 300), None), (np.arange(300, 310), [4]), (np.arange(100, 520), None),
             (np.array([699, 127, 128, 255, 256]), None)]
    for pos, invalid in calls:
        m = pos.size
        slots = pos.copy()
        if invalid:
            slots[invalid] = -1
        fused = bf16_tensor(randn_kv(rng, (m, 2, hkv, HD), 2) * 3)
        k, v = fused[:, 0], fused[:, 1]
        kernels.append_fp8(k, v, torch.from_numpy(pos).cuda(), torch.from_numpy(slots).cuda(), side8, ks_t, vs_t)
        fo.append_fp8(ref, to64(k), to64(v), pos, slots, ks, vs)
    torch.cuda.synchronize()
    assert np.array_equal(side8_bits(side8), ref)


def run_far_fp8(n, hq, hkv, far_keys, *, splits, window=64, outliers=0, seed=0, extra=0):
    """fold_far_read_fp8 over a cache filled by fold_append_fp8; returns the device (o, lse) after
    the split combine, the oracle's over the dequantised cache, and the oracle's over the bf16
    keys and values the cache was filled from."""
    rng = np.random.default_rng(seed)
    B = n
    hist = far_keys + window + B - n if far_keys > 0 else window // 2
    L = max(far_keys + extra, 1)
    k = fo.bf16_round(randn_kv(rng, (L, hkv, HD), outliers))
    v = fo.bf16_round(randn_kv(rng, (L, hkv, HD), outliers))
    ks, vs = head_scales(k), head_scales(v)
    pages = -(-L // 256) + 1
    side8 = torch.zeros(kernels.fp8_side_shape(pages, hkv), device="cuda", dtype=torch.uint8)
    ks_t, vs_t = torch.from_numpy(ks).cuda(), torch.from_numpy(vs).cuda()
    for a in range(0, L, 16384):
        b = min(L, a + 16384)
        pos = torch.arange(a, b, device="cuda")
        kernels.append_fp8(bf16_tensor(k[a:b]), bf16_tensor(v[a:b]), pos, pos, side8, ks_t, vs_t)
    q = bf16_tensor(rng.standard_normal((n, hq, HD), dtype=np.float32))
    f = fo.inv_freq(500000.0, HD)
    table = rope_table(torch.from_numpy(f).cuda(), hist + 2 * window + 2 * B + 1, "cuda")
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((splits, n, hq, HD), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((splits, hq, n), device="cuda", dtype=torch.float32)
    far_len = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    scale = HD ** -0.5 * 2.0
    kernels.far_read_fp8(q, qsl, seq, side8, ks_t, vs_t, o_part, lse_part, window=window, block=B,
                         far_distance=window + B, softmax_scale=scale, table=table, far_len=far_len,
                         capacity=L + 10 ** 6, err=err)
    o_d, lse_d = kernels.combine(o_part, lse_part)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(far_len.item()) == fo.far_len(hist, window, B, n)
    lim = fo.far_row_limits(hist, window, B, n)
    qf = f16_round(fo.far_query(to64(q), hist, f, window + B))  # the kernel's f16 far query
    kd, vd = fo.fp8_side_view_kv(side8_bits(side8), L, ks, vs)
    o_w, lse_w = fo.far_read(qf, kd, vd, lim, scale)
    o_b, lse_b = fo.far_read(fo.far_query(to64(q), hist, f, window + B), k, v, lim, scale)
    return to64(o_d), to64(lse_d), (o_w, lse_w), (o_b, lse_b)


FP8_CASES = [
    # n, hq, hkv, far_keys, splits
    (10, 32, 8, 1000, 5),
    (10, 32, 8, 1, 3),
    (10, 32, 8, 129, 4),
    (8, 32, 8, 5000, 18),
    (1, 4, 1, 700, 7),
    (3, 8, 1, 4097, 16),
    (2, 64, 2, 2049, 11),
]


@pytest.mark.parametrize("n,hq,hkv,far_keys,splits", FP8_CASES)
def test_far_read_fp8_matches_oracle_on_the_stored_values(n, hq, hkv, far_keys, splits):
    o_d, lse_d, (o_w, lse_w), _ = run_far_fp8(n, hq, hkv, far_keys, splits=splits, extra=300, seed=far_keys)
    assert np.abs(o_d - o_w).max() <= OUT_ATOL
    lse_close(lse_d, lse_w)


def test_far_read_fp8_accuracy_study_llama_128k():
    """The 128K Llama shape (129024 far keys) with x8 outlier channels on K and V."""
    o_d, lse_d, (o_w, lse_w), (o_b, lse_b) = run_far_fp8(10, 32, 8, 129024, splits=18, window=2048, outliers=4,
                                                         seed=1)
    err_stored = np.abs(o_d - o_w).max()
    err_bf16 = np.abs(o_d - o_b)
    lse_rel = np.abs(lse_d - lse_b) / np.maximum(np.abs(lse_b), 1.0)
    print(f"fp8 side cache, 128K Llama shape: max-abs vs the stored values {err_stored:.5f}; vs the bf16 memory "
          f"max-abs {err_bf16.max():.4f}, mean-abs {err_bf16.mean():.5f}, LSE max relative {lse_rel.max():.4f}")
    assert err_stored <= OUT_ATOL
    lse_close(lse_d, lse_w)
    # the storage's own error (3 mantissa bits): bounded on average, not per element
    assert err_bf16.mean() <= 0.05 and lse_rel.max() <= 0.05


def test_fold_forward_with_fp8_side_cache():
    """FoldWorkspace(side_format="fp8"): append through the workspace, then the FOLD forward (the
    bf16 window read of the paged cache, the fp8 far read, the merge) against the oracle with the
    dequantised memory."""
    rng = np.random.default_rng(21)
    n, hq, hkv, W, t = 10, 32, 8, 256, 3000
    f = fo.inv_freq(1e6, HD)
    keys = fo.bf16_round(rng.standard_normal((t + n, hkv, HD), dtype=np.float32))
    vals = fo.bf16_round(rng.standard_normal((t + n, hkv, HD), dtype=np.float32))
    q = rng.standard_normal((n, hq, HD), dtype=np.float32)
    k_roped = fo.bf16_round(fo.rotate(keys, np.arange(t + n), f))
    q_roped = fo.bf16_round(fo.rotate(q, np.arange(t, t + n), f))
    kv_cache, table = paged_from(k_roped, vals, 16, rng)
    ks, vs = head_scales(keys[:t]), head_scales(vals[:t])
    dummy = torch.zeros((1, hkv, 16, 2 * HD), device="cuda", dtype=torch.bfloat16)
    ws = FoldWorkspace(dummy, W, n, t + n, inv_freq=torch.from_numpy(f).cuda(), far_distance=W + n, num_heads=hq,
                       side_format="fp8", k_scale=torch.from_numpy(ks), v_scale=torch.from_numpy(vs))
    pos = torch.arange(t, device="cuda")
    ws.append(bf16_tensor(keys[:t]), bf16_tensor(vals[:t]), pos, pos)
    assert ws.side.dtype == torch.uint8 and ws.side.numel() == ws.side_pages * hkv * 256 * HD * 2
    original = SimpleNamespace(head_size=HD, scale=HD ** -0.5, num_heads=hq, sliding_window=(-1, -1),
                               vllm_flash_attn_version=4)
    meta = SimpleNamespace(num_actual_tokens=n, query_start_loc=torch.tensor([0, n], dtype=torch.int32, device="cuda"),
                           seq_lens=torch.tensor([t + n], dtype=torch.int32, device="cuda"), max_query_len=n,
                           max_seq_len=t + n, block_table=table, use_cascade=False, causal=True)
    output = torch.empty((n, hq * HD), device="cuda", dtype=torch.bfloat16)
    out = FoldAttention(original, ws).forward(None, bf16_tensor(q_roped), None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    ws.check()
    o_l, lse_l = fo.local_read(q_roped, k_roped, vals, t, W, n, original.scale)
    kd, vd = fo.fp8_side_view_kv(side8_bits(ws.side), t, ks, vs)
    lim = fo.far_row_limits(t, W, n, n)
    qf = f16_round(fo.far_query(q_roped, t, f, W + n))
    o_f, lse_f = fo.far_read(qf, kd[:int(lim.max())], vd[:int(lim.max())], lim, original.scale * 2.0)
    want = fo.merge(o_l, lse_l, o_f, lse_f, t, W, n, 2.0)
    assert np.abs(to64(out).reshape(want.shape) - want).max() <= OUT_ATOL
