"""Parity of the window (exact-position) read over a paged cache, and of the merge of two sets of
split partials, with the CPU oracle (float64), called through the C-ABI.

The cache is vLLM's FlashAttention layout kv[num_blocks, Hkv, block_size, 2D] with shuffled
blocks; every slot that holds no context entry is NaN. Bars: output max-abs 2e-2, LSE within
1e-3 relative.
"""
import numpy as np
import pytest
import torch

from fold_b200 import kernels
from fold_b200.errors import DEVERR_BLOCK_TABLE
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, lengths, lse_close, paged_from, side_from, to64

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

# n, hq, hkv, hd, hist, (left, right), causal, block_size, splits
CASES = [
    (10, 32, 8, 128, 6000, (2057, 9), False, 16, 16),   # FOLD window of a Llama-3.1-8B drafter, W 2048
    (10, 32, 8, 128, 1000, (2057, 9), False, 32, 16),   # the window reaches past the first entry
    (1, 32, 8, 128, 3001, (2057, 9), False, 16, 5),     # one row
    (8, 32, 8, 128, 4099, (2047, 0), True, 256, 16),    # native causal sliding window
    (16, 16, 4, 256, 5000, (4111, 15), False, 64, 16),  # hd 256, 64 rows per KV head
    (8, 16, 8, 256, 4500, (4095, 0), True, 16, 37),     # hd 256, 16 rows per KV head
    (3, 4, 2, 128, 777, (-1, -1), True, 16, 3),         # unbounded window: causal full attention
    (5, 8, 8, 128, 100, (20, 2), False, 48, 1),         # short odd window, block size 48, one split
]


def window_case(n, hq, hkv, hd, hist, bs, seed):
    rng = np.random.default_rng(seed)
    seq = hist + n
    q = fo.bf16_round(rng.standard_normal((n, hq, hd)))
    k = fo.bf16_round(rng.standard_normal((seq, hkv, hd)))
    v = fo.bf16_round(rng.standard_normal((seq, hkv, hd)))
    kv, table = paged_from(k, v, bs, rng)
    return q, k, v, kv, table


@pytest.mark.parametrize("n,hq,hkv,hd,hist,ws,causal,bs,splits", CASES)
def test_window_read_matches_oracle(n, hq, hkv, hd, hist, ws, causal, bs, splits):
    q, k, v, kv, table = window_case(n, hq, hkv, hd, hist, bs, seed=hist + n)
    scale = hd ** -0.5
    want_o, want_lse = fo.window_read(q, k, v, hist, ws[0], ws[1], causal, scale)
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((splits, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((splits, hq, n), device="cuda", dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kc, vc = kernels.paged_planes(kv, hd)
    kernels.window_read(bf16_tensor(q), qsl, seq, kc, vc, table, o_part, lse_part, window_size=ws, causal=causal,
                        softmax_scale=scale, err=err)
    o, lse = kernels.combine(o_part, lse_part)
    out = torch.empty((n, hq, hd), device="cuda", dtype=torch.bfloat16)
    kernels.merge_partials(o_part, lse_part, None, None, out, qsl, seq, window=1, block=1, alpha=1.0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.abs(to64(o) - want_o).max() <= OUT_ATOL
    lse_close(to64(lse), want_lse)
    got = to64(out)
    assert np.isfinite(got).all()
    assert np.abs(got - want_o).max() <= OUT_ATOL


def test_window_read_separate_planes_and_strided_query():
    """K and V in separate planes laid out [num_blocks, block_size, Hkv, D] (vLLM's other
    FlashAttention layout, seen through a permuted view) and a query with a token stride."""
    n, hq, hkv, hd, hist, bs = 10, 32, 8, 128, 2500, 16
    q, k, v, kv, table = window_case(n, hq, hkv, hd, hist, bs, seed=11)
    nb = kv.shape[0]
    kplane = kv[..., :hd].permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)  # strides of [nb, bs, hkv, hd]
    vplane = kv[..., hd:].permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    assert kplane.shape == (nb, hkv, bs, hd) and kplane.stride(2) == hkv * hd
    qbuf = torch.zeros((n, hq + 4, hd), device="cuda", dtype=torch.bfloat16)
    qbuf[:, :hq] = bf16_tensor(q)
    scale = hd ** -0.5
    ws = (2057, 9)
    want_o, want_lse = fo.window_read(q, k, v, hist, ws[0], ws[1], False, scale)
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((16, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((16, hq, n), device="cuda", dtype=torch.float32)
    kernels.window_read(qbuf[:, :hq], qsl, seq, kplane, vplane, table, o_part, lse_part, window_size=ws, causal=False,
                        softmax_scale=scale)
    o, lse = kernels.combine(o_part, lse_part)
    torch.cuda.synchronize()
    assert np.abs(to64(o) - want_o).max() <= OUT_ATOL
    lse_close(to64(lse), want_lse)


def test_window_read_flags_bad_block_table_entries():
    n, hq, hkv, hd, hist, bs = 4, 8, 2, 128, 300, 16
    q, k, v, kv, table = window_case(n, hq, hkv, hd, hist, bs, seed=3)
    table[0, 2] = kv.shape[0] + 5  # outside the cache: read from block 0 instead and flagged
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((4, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((4, hq, n), device="cuda", dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kc, vc = kernels.paged_planes(kv, hd)
    kernels.window_read(bf16_tensor(q), qsl, seq, kc, vc, table, o_part, lse_part, window_size=(-1, -1), causal=True,
                        softmax_scale=0.1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & DEVERR_BLOCK_TABLE


@pytest.mark.parametrize("hist", [1500, 2047, 2048, 9000])
def test_merge_partials_matches_oracle_fold_step(hist):
    """Window read + far read as split partials, merged in one kernel: the oracle's FOLD step
    (window read, far read at alpha, merge; fold/attention.py:162-172)."""
    n, hq, hkv, hd, W, alpha = 10, 32, 8, 128, 2048, 2.0
    B = n
    rng = np.random.default_rng(hist)
    seq = hist + n
    f = fo.inv_freq(500000.0, hd)
    q = fo.bf16_round(rng.standard_normal((n, hq, hd)))
    k_raw = fo.bf16_round(rng.standard_normal((seq, hkv, hd)))
    v = fo.bf16_round(rng.standard_normal((seq, hkv, hd)))
    k_roped = fo.bf16_round(fo.rotate(k_raw, np.arange(seq), f))
    scale = hd ** -0.5
    o_l, lse_l = fo.local_read(q, k_roped, v, hist, W, B, scale)
    qf = fo.far_query(q, hist, f, W + B)
    lim = fo.far_row_limits(hist, W, B, n)
    L = max(int(lim.max()), 1)
    o_f, lse_f = fo.far_read(qf, k_raw[:L], v[:L], lim, scale * alpha)
    want = fo.merge(o_l, lse_l, o_f, lse_f, hist, W, B, alpha)

    kv, table = paged_from(k_roped, v, 16, rng)
    qd = bf16_tensor(q)
    qsl, seq_t = lengths(n, hist)
    wo = torch.empty((16, n, hq, hd), device="cuda", dtype=torch.float32)
    wl = torch.empty((16, hq, n), device="cuda", dtype=torch.float32)
    kc, vc = kernels.paged_planes(kv, hd)
    kernels.window_read(qd, qsl, seq_t, kc, vc, table, wo, wl, window_size=(W + B - 1, B - 1), causal=False,
                        softmax_scale=scale)
    pages = fo.side_pages(seq)
    side = side_from(k_raw, v, pages)
    table_rows = 1 << 16
    from fold_b200.rope import rope_table
    tab = rope_table(torch.from_numpy(f), table_rows, "cuda")
    fo_p = torch.empty((37, n, hq, hd), device="cuda", dtype=torch.float32)
    fl_p = torch.empty((37, hq, n), device="cuda", dtype=torch.float32)
    kernels.far_read(qd, qsl, seq_t, side, fo_p, fl_p, window=W, block=B, far_distance=W + B,
                     softmax_scale=scale * alpha, table=tab)
    out = torch.empty((n, hq, hd), device="cuda", dtype=torch.bfloat16)
    kernels.merge_partials(wo, wl, fo_p, fl_p, out, qsl, seq_t, window=W, block=B, alpha=alpha)
    torch.cuda.synchronize()
    assert np.abs(to64(out) - want).max() <= OUT_ATOL
    # the same step as one launch of both reads (the blocks split per step) and the merge of the
    # slots the step used
    S = kernels.default_splits(hkv)
    far = (torch.empty((S, n, hq, hd), device="cuda"), torch.empty((S, hq, n), device="cuda"))
    win = (torch.empty((S, n, hq, hd), device="cuda"), torch.empty((S, hq, n), device="cuda"))
    plan = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.step_read(qd, qd, qsl, seq_t, side, far, kc, vc, table, win, plan, window=W, block=B, far_distance=W + B,
                      softmax_scale=scale, alpha=alpha, window_size=(W + B - 1, B - 1), causal=False, table=tab)
    out2 = torch.empty_like(out)
    kernels.merge_partials(win[0], win[1], far[0], far[1], out2, qsl, seq_t, window=W, block=B, alpha=alpha,
                           plan=plan)
    torch.cuda.synchronize()
    assert 1 <= int(plan[0].item()) < S
    assert np.abs(to64(out2) - want).max() <= OUT_ATOL


@pytest.mark.parametrize("hd,hq,hkv,n,hist", [(128, 32, 8, 10, 20000), (128, 32, 8, 10, 131062),
                                              (128, 32, 8, 8, 32760), (256, 16, 8, 8, 9000),
                                              (128, 32, 8, 10, 1500)])  # last: no far key at all
def test_step_read_equals_separate_reads(hd, hq, hkv, n, hist, far_kernel):
    """The one-launch step read: w of each KV head's S blocks (plan[0] = w) write bit for bit the
    partials of fold_window_read with w splits; all S blocks write far slots, which together hold
    the far read: combined, they equal the combine of fold_far_read's S partials (to float32
    rounding of a different split of the keys). A second launch writes the same bits. Shapes whose
    far read takes the tcgen05 kernel are refused."""
    from fold_b200.errors import FoldError

    rng = np.random.default_rng(hd + hist)
    W, B, alpha = 2048, n, 2.0
    seq = hist + n
    f = fo.inv_freq(500000.0, hd)
    qd = bf16_tensor(rng.standard_normal((n, hq, hd)))
    k_raw = rng.standard_normal((seq, hkv, hd), dtype=np.float32)
    v = rng.standard_normal((seq, hkv, hd), dtype=np.float32)
    kv, table = paged_from(k_raw, v, 16, rng)
    side = side_from(k_raw, v, fo.side_pages(seq))
    from fold_b200.rope import rope_table
    tab = rope_table(torch.from_numpy(f), 1 << 18, "cuda")
    qsl, seq_t = lengths(n, hist)
    kc, vc = kernels.paged_planes(kv, hd)
    scale = hd ** -0.5
    ws = (W + B - 1, B - 1)

    def bufs(s):
        return (torch.full((s, n, hq, hd), float("nan"), device="cuda"),
                torch.full((s, hq, n), float("nan"), device="cuda"))

    S = kernels.default_splits(hkv)
    far_a, win_a = bufs(S), bufs(S)
    plan = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = dict(window=W, block=B, far_distance=W + B, softmax_scale=scale, alpha=alpha, window_size=ws,
                causal=False, table=tab)
    if kernels.far_read_uses_tcgen05(hd, n, hq, hkv):
        with pytest.raises(FoldError, match="tcgen05"):
            kernels.step_read(qd, qd, qsl, seq_t, side, far_a, kc, vc, table, win_a, plan, **args)
        return
    far_b = bufs(S)
    kernels.far_read(qd, qsl, seq_t, side, far_b[0], far_b[1], window=W, block=B, far_distance=W + B,
                     softmax_scale=scale * alpha, table=tab)
    o_b, l_b = kernels.combine(far_b[0], far_b[1])
    first = None
    for launch in range(2):
        kernels.step_read(qd, qd, qsl, seq_t, side, far_a, kc, vc, table, win_a, plan, **args)
        torch.cuda.synchronize()
        w = int(plan[0].item())
        assert 1 <= w < S
        if first is None:
            first = far_a[0].clone()
        else:
            assert torch.equal(far_a[0], first), "a second launch wrote other far partials"
        win_b = bufs(w)
        kernels.window_read(qd, qsl, seq_t, kc, vc, table, win_b[0], win_b[1], window_size=ws, causal=False,
                            softmax_scale=scale)
        o_a, l_a = kernels.combine(far_a[0], far_a[1])
        torch.cuda.synchronize()
        assert torch.equal(win_a[0][:w], win_b[0]) and torch.equal(win_a[1][:w], win_b[1])
        assert np.abs(to64(o_a) - to64(o_b)).max() <= 5e-3
        lse_close(to64(l_a), to64(l_b), rtol=1e-4)
