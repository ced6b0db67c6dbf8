"""Parity of the CUDA kernels with the CPU oracle, called through the C-ABI (fold_b200.kernels).

append/gather: bit-exact. far query: within one bf16 ulp of the oracle's table rotation.
far read + merge: output max-abs 2e-2 against the float64 oracle (absolute, on every channel,
the x8 outlier channels included), LSE within 1e-3 relative. The full-length cases of the three
long-context shapes (129,024 far keys at head_dim 128; 258,048 at head_dim 256 with 64 and 16
query rows per KV head) print their measured max-abs error.
"""
import numpy as np
import pytest
import torch

from fold_b200 import kernels
from fold_b200.rope import rope_table
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, lengths, lse_close, randn_kv, side_from, to64

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


# ------------------------------------------------------------------------------------- append
@pytest.mark.parametrize("hd,hkv", [(128, 8), (256, 4), (64, 2)])
def test_append_bit_exact(hd, hkv):
    rng = np.random.default_rng(hd + hkv)
    max_len = 1000
    pages = fo.side_pages(max_len)
    side = torch.zeros((pages, hkv, 256, 2 * hd), device="cuda", dtype=torch.bfloat16)
    ref = np.zeros(side.shape, dtype=np.uint16)
    calls = [(np.arange(0, 600), None), (np.arange(600, 610), [3]), (np.arange(250, 700), None),
             (np.array([999, 5, 77]), None), (np.arange(610, 611), [0])]
    for pos, invalid in calls:
        m = pos.size
        slots = pos.copy()
        if invalid:
            slots[invalid] = -1
        # K and V as strided views of a fused buffer, the way the drafter produces them
        fused = bf16_tensor(rng.standard_normal((m, 2, hkv, hd), dtype=np.float32))
        k, v = fused[:, 0], fused[:, 1]
        kernels.append(k, v, torch.from_numpy(pos).cuda(), torch.from_numpy(slots).cuda(), side)
        fo.append(ref, bits(k).reshape(m, hkv, hd), bits(v).reshape(m, hkv, hd), pos, slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(side), ref)


def test_append_sharded_skips_foreign_positions_and_gather_round_trips():
    rng = np.random.default_rng(5)
    hkv, hd = 2, 128
    pos_lo, held = 512, 512
    pages = held // 256 + 1
    side = torch.zeros((pages, hkv, 256, 2 * hd), device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = np.arange(300, 1300)
    k = bf16_tensor(rng.standard_normal((pos.size, hkv, hd), dtype=np.float32))
    v = bf16_tensor(rng.standard_normal((pos.size, hkv, hd), dtype=np.float32))
    p = torch.from_numpy(pos).cuda()
    kernels.append(k, v, p, p, side, pos_lo=pos_lo, skip_foreign=True, err=err)
    mine = (pos >= pos_lo) & (pos < pos_lo + held)
    kg, vg = kernels.gather(side, p[torch.from_numpy(mine).cuda()], pos_lo=pos_lo, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(kg, k[torch.from_numpy(mine).cuda()])
    assert torch.equal(vg, v[torch.from_numpy(mine).cuda()])
    # an unsharded cache flags positions beyond its capacity instead of writing them
    kernels.append(k[:3], v[:3], torch.tensor([0, 5000, 1], device="cuda"), torch.zeros(3, device="cuda",
                   dtype=torch.int64), side, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1


def test_append_rejects_positions_shorter_than_the_rows():
    """Every K/V row needs its position and slot: shorter arrays are refused (the kernel would
    read past them), longer ones are cut to the rows."""
    from fold_b200.errors import FoldError
    side = torch.zeros((3, 2, 256, 256), device="cuda", dtype=torch.bfloat16)
    k = torch.randn((8, 2, 128), device="cuda").to(torch.bfloat16)
    pos = torch.arange(8, device="cuda")
    with pytest.raises(FoldError, match="one entry per K/V row"):
        kernels.append(k, k, pos[:7], pos, side)
    with pytest.raises(FoldError, match="one entry per K/V row"):
        kernels.append(k, k, pos, pos[:5], side)
    kernels.append(k, k, torch.arange(12, device="cuda"), torch.arange(12, device="cuda"), side)
    kg, _ = kernels.gather(side, pos)
    torch.cuda.synchronize()
    assert torch.equal(kg, k)


# ---------------------------------------------------------------------------------- far query
@pytest.mark.parametrize("n,hq,hd,rot,hist,D", [(10, 32, 128, 128, 131062, 2058), (8, 4, 128, 64, 100000, 2056),
                                               (4, 4, 64, 64, 30, 44), (3, 2, 256, 256, 262000, 4112)])
def test_far_query_matches_oracle(n, hq, hd, rot, hist, D):
    rng = np.random.default_rng(n * hq)
    q = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    f = fo.inv_freq(500000.0, rot)
    inv = torch.from_numpy(f).cuda()
    qsl, seq = lengths(n, hist)
    far_len = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    table = rope_table(inv, abs(D - hist) + 1, "cuda")
    qf = kernels.far_query(q, qsl, seq, inv, far_len, far_distance=D, window=D - n, block=n, table=table)
    torch.cuda.synchronize()
    assert int(far_len.item()) == fo.far_len(hist, D - n, n, n)
    want = fo.far_query(to64(q), hist, f, D)
    got = to64(qf)
    # one bf16 rounding of a float32 rotation with an exact table
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max() + 1e-6
    ulp = np.abs(got - fo.bf16_round(want)) / np.maximum(np.abs(want), 1e-30)
    assert (got == fo.bf16_round(want)).mean() > 0.98, ulp.max()


def test_rerope_matches_oracle():
    rng = np.random.default_rng(9)
    n, hq, hd, hist, D = 8, 4, 128, 70000, 2056
    q = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    f = fo.inv_freq(1e6, hd)
    inv = torch.from_numpy(f).cuda()
    qsl, seq = lengths(n, hist)
    far_len = torch.zeros(1, dtype=torch.int32, device="cuda")
    qs, qf = kernels.rerope_queries(q, qsl, seq, inv, far_len, far_distance=D, window=D - n, block=n, constant=True,
                                    logn_ref=4096)
    torch.cuda.synchronize()
    ws, wf = fo.rerope_queries(to64(q), hist, f, D, 4096)
    assert np.abs(to64(qs) - ws).max() <= 2 ** -7 * np.abs(ws).max()
    assert np.abs(to64(qf) - wf).max() <= 2 ** -7 * np.abs(wf).max() + 1e-3


# ----------------------------------------------------------------------------------- far read
def run_far(n, hq, hkv, hd, far_keys, *, splits, window=64, extra=0, outliers=0, seed=0, rot=None, pos_lo=0,
            held=None, qlen=None):
    """Far read over a side cache whose first `far_keys + extra` positions are filled; returns
    (device o/lse after combine, oracle o/lse)."""
    rng = np.random.default_rng(seed)
    B = n
    hist = far_keys + window + B - n if far_keys > 0 else window // 2  # far_len = hist - W - B + n
    rot = rot or hd
    L = max(far_keys + extra, 1)
    k = randn_kv(rng, (L, hkv, hd), outliers)
    v = randn_kv(rng, (L, hkv, hd), outliers)
    kb, vb = fo.bf16_round(k), fo.bf16_round(v)
    held = L if held is None else held
    pages = -(-held // 256) + 1
    local = slice(pos_lo, pos_lo + held)
    side = side_from(kb[local], vb[local], pages)
    q = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    f = fo.inv_freq(500000.0, rot)
    table = rope_table(torch.from_numpy(f).cuda(), hist + 2 * window + 2 * B + 1, "cuda")
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((splits, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((splits, hq, n), device="cuda", dtype=torch.float32)
    far_len = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qf = torch.empty_like(q)
    scale = hd ** -0.5 * 2.0
    kernels.far_read(q, qsl, seq, side, o_part, lse_part, window=window, block=B, far_distance=window + B,
                     softmax_scale=scale, table=table, far_len=far_len, qf=qf, pos_lo=pos_lo, capacity=L + 10 ** 6,
                     err=err)
    o_d, lse_d = kernels.combine(o_part, lse_part)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(far_len.item()) == fo.far_len(hist, window, B, n)
    # oracle: the device's own bf16 far query (checked separately above) against the exact keys
    lim = fo.far_row_limits(hist, window, B, n)
    lim = np.minimum(lim, pos_lo + held)
    kf, vf = kb[local], vb[local]
    o_w, lse_w = fo.far_read(to64(qf), kf, vf, lim, scale, key_lo=pos_lo)
    return to64(o_d), to64(lse_d), o_w, lse_w, dict(o_part=o_part, lse_part=lse_part, qf=qf, q=q, hist=hist)


def out_close(o_d, o_w, what=""):
    """The output bar: max-abs 2e-2, absolute, over every channel (outlier channels included)."""
    err = float(np.abs(o_d - o_w).max())
    print(f"{what} output max-abs error {err:.5f} (bar {OUT_ATOL})")
    assert err <= OUT_ATOL, f"max error {err}"


def run_far_device(n, hq, hkv, hd, far_keys, *, splits, window, seed, outliers=0, theta=1e6):
    """Far read of a full-length side cache generated on the device (seeded torch generator), the
    oracle computed per KV head from the same bf16 keys and values. Returns (device o, lse,
    oracle o, lse)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    L = far_keys
    k = torch.randn((L, hkv, hd), device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn((L, hkv, hd), device="cuda", generator=gen).to(torch.bfloat16)
    if outliers:
        ch = torch.randperm(hd, generator=torch.Generator().manual_seed(seed))[:outliers].cuda()
        k[..., ch] *= 8
        v[..., ch] *= 8
    pages = -(-L // 256) + 1
    side = torch.zeros((pages, hkv, 256, 2 * hd), device="cuda", dtype=torch.bfloat16)
    full = L // 256
    side[:full] = torch.cat((k[:full * 256], v[:full * 256]), -1).view(full, 256, hkv, 2 * hd).transpose(1, 2)
    if L > full * 256:
        side[full, :, :L - full * 256] = torch.cat((k[full * 256:], v[full * 256:]), -1).transpose(0, 1)
    q = torch.randn((n, hq, hd), device="cuda", generator=gen).to(torch.bfloat16)
    B = n
    hist = far_keys + window  # far_len = hist - W - B + n = far_keys
    f = fo.inv_freq(theta, hd)
    table = rope_table(torch.from_numpy(f).cuda(), hist + 2 * window + 2 * B + 1, "cuda")
    qsl, seq = lengths(n, hist)
    o_part = torch.empty((splits, n, hq, hd), device="cuda", dtype=torch.float32)
    lse_part = torch.empty((splits, hq, n), device="cuda", dtype=torch.float32)
    far_len = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qf = torch.empty_like(q)
    scale = hd ** -0.5 * 2.0
    kernels.far_read(q, qsl, seq, side, o_part, lse_part, window=window, block=B, far_distance=window + B,
                     softmax_scale=scale, table=table, far_len=far_len, qf=qf, capacity=L, err=err)
    o_d, lse_d = kernels.combine(o_part, lse_part)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(far_len.item()) == far_keys
    lim = fo.far_row_limits(hist, window, B, n)
    g = hq // hkv
    qf64 = to64(qf)
    o_w, lse_w = np.zeros((n, hq, hd)), np.zeros((hq, n))
    for h in range(hkv):  # one KV head at a time keeps the float64 copies at a few hundred MB
        kh, vh = to64(k[:, h:h + 1]), to64(v[:, h:h + 1])
        oh, lh = fo.far_read(qf64[:, h * g:(h + 1) * g], kh, vh, lim, scale)
        o_w[:, h * g:(h + 1) * g], lse_w[h * g:(h + 1) * g] = oh, lh
    return to64(o_d), to64(lse_d), o_w, lse_w


FAR_CASES = [
    # n, hq, hkv, hd, far_keys, splits
    (10, 32, 8, 128, 1000, 5),
    (10, 32, 8, 128, 1, 3),
    (10, 32, 8, 128, 63, 2),
    (10, 32, 8, 128, 129, 4),
    (10, 32, 8, 128, 256, 1),
    (8, 32, 8, 128, 5000, 18),
    (1, 4, 1, 128, 700, 7),
    (3, 8, 1, 128, 4097, 16),
    (16, 16, 4, 256, 3000, 9),
    (8, 16, 8, 256, 2000, 4),
    (5, 10, 5, 256, 333, 2),
    (7, 56, 7, 128, 1500, 6),
    (2, 64, 2, 128, 2049, 11),
]


@pytest.mark.parametrize("n,hq,hkv,hd,far_keys,splits", FAR_CASES)
def test_far_read_matches_oracle(n, hq, hkv, hd, far_keys, splits, far_kernel):
    o_d, lse_d, o_w, lse_w, x = run_far(n, hq, hkv, hd, far_keys, splits=splits, extra=300, seed=far_keys)
    assert np.abs(o_d - o_w).max() <= OUT_ATOL
    lse_close(lse_d, lse_w)


def test_far_read_no_far_keys_gives_empty_rows(far_kernel):
    o_d, lse_d, o_w, lse_w, _ = run_far(10, 32, 8, 128, 0, splits=4, extra=50)
    assert np.all(np.isneginf(lse_d)) and np.all(o_d == 0)


def test_far_read_outliers_partial_rotary(far_kernel):
    o_d, lse_d, o_w, lse_w, x = run_far(10, 32, 8, 128, 3000, splits=8, outliers=4, rot=64, extra=200)
    out_close(o_d, o_w, f"{far_kernel} 3000 keys, x8 outliers, rotary 64:")
    lse_close(lse_d, lse_w)


def test_far_read_shard_of_cache(far_kernel):
    """A shard holding positions [512, 1536) of a 4000-key far memory."""
    o_d, lse_d, o_w, lse_w, _ = run_far(10, 32, 8, 128, 4000, splits=6, pos_lo=512, held=1024, extra=0)
    assert np.abs(o_d - o_w).max() <= OUT_ATOL
    lse_close(lse_d, lse_w)


def test_far_read_full_context_llama_shape(far_kernel):
    """Llama-3.1-8B drafter shape at 131072 context (129024 far keys), outlier channels x8."""
    o_d, lse_d, o_w, lse_w, x = run_far(10, 32, 8, 128, 129024, splits=18, window=2048, outliers=4, seed=1)
    out_close(o_d, o_w, f"{far_kernel} 128K Llama shape (129024 keys, x8 outliers):")
    lse_close(lse_d, lse_w)


@pytest.mark.parametrize("n,hq,hkv,splits", [(16, 16, 4, 37), (8, 16, 8, 18)])
def test_far_read_full_context_hd256(n, hq, hkv, splits, far_kernel):
    """The 262144-context head_dim-256 shapes: 258048 far keys; 16/4 heads with a 16-token block
    (64 query rows per KV head) and 16/8 heads with an 8-token block (16 rows)."""
    o_d, lse_d, o_w, lse_w = run_far_device(n, hq, hkv, 256, 258048, splits=splits, window=4096, seed=n + hkv)
    out_close(o_d, o_w, f"{far_kernel} 262K hd 256, {hq}/{hkv} heads, block {n}:")
    lse_close(lse_d, lse_w)


def test_far_read_full_context_llama_shape_device_generated(far_kernel):
    """The 128K Llama shape again with device-generated inputs and the x8 outlier channels on K
    and V (a second seed)."""
    o_d, lse_d, o_w, lse_w = run_far_device(10, 32, 8, 128, 129024, splits=18, window=2048, seed=7, outliers=4,
                                            theta=5e5)
    out_close(o_d, o_w, f"{far_kernel} 128K Llama shape (device inputs, x8 outliers):")
    lse_close(lse_d, lse_w)


# -------------------------------------------------------------------------------------- merge
@pytest.mark.parametrize("hd,splits", [(128, 18), (256, 3), (64, 1)])
def test_merge_with_partials_matches_oracle(hd, splits):
    rng = np.random.default_rng(hd)
    n, hq, W, B, alpha = 6, 8, 60, 6, 2.0
    hist = 63  # rows 0..1 have no memory, 2..5 do
    o_l = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    lse_l = torch.from_numpy((rng.standard_normal((hq, n)) * 3 + 5).astype(np.float32)).cuda()
    o_p = torch.from_numpy(rng.standard_normal((splits, n, hq, hd)).astype(np.float32)).cuda()
    lse_np = (rng.standard_normal((splits, hq, n)) * 4 + 9).astype(np.float32)
    lse_np[0, 0, :] = -np.inf  # an empty split
    lse_p = torch.from_numpy(lse_np).cuda()
    out = torch.zeros((n, hq, hd), device="cuda", dtype=torch.bfloat16)
    qsl, seq = lengths(n, hist)
    kernels.merge(o_l, lse_l, o_p, lse_p, out, qsl, seq, window=W, block=B, alpha=alpha)
    torch.cuda.synchronize()
    o_f, lse_f = fo.combine(to64(o_p), lse_np)
    want = fo.merge(to64(o_l), to64(lse_l), o_f, lse_f, hist, W, B, alpha)
    assert np.abs(to64(out) - want).max() <= 2 ** -7 * np.abs(want).max() + 1e-5


def test_merge_reference_form_bf16_single_far():
    """The reference's own call shape: o_f bf16 [n, Hq, D], lse_f [Hq, n] (a transposed view)."""
    rng = np.random.default_rng(3)
    n, hq, hd, W, B = 10, 8, 128, 2048, 10
    hist = 9000
    o_l = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    o_f = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
    lse_l = torch.from_numpy(rng.standard_normal((n, hq)).astype(np.float32)).cuda().t()
    lse_f = torch.from_numpy((rng.standard_normal((hq, n)) * 5 + 7).astype(np.float32)).cuda()
    out = torch.empty((n, hq * hd), device="cuda", dtype=torch.bfloat16)
    qsl, seq = lengths(n, hist)
    kernels.merge(o_l, lse_l, o_f, lse_f, out.view(n, hq, hd), qsl, seq, window=W, block=B, alpha=2.0)
    torch.cuda.synchronize()
    want = fo.merge(to64(o_l), to64(lse_l), to64(o_f), to64(lse_f), hist, W, B, 2.0)
    assert np.abs(to64(out).reshape(n, hq, hd) - want).max() <= 2 ** -7 * np.abs(want).max() + 1e-5


def test_combine_matches_oracle():
    rng = np.random.default_rng(11)
    s, n, hq, hd = 7, 5, 4, 128
    o_p = rng.standard_normal((s, n, hq, hd)).astype(np.float32)
    lse = (rng.standard_normal((s, hq, n)) * 3).astype(np.float32)
    lse[2] = -np.inf
    lse[:, 1, 3] = -np.inf  # a row without any mass
    o_d, l_d = kernels.combine(torch.from_numpy(o_p).cuda(), torch.from_numpy(lse).cuda())
    torch.cuda.synchronize()
    o_w, l_w = fo.combine(o_p, lse)
    assert np.abs(to64(o_d) - o_w).max() <= 1e-5
    lse_close(to64(l_d), l_w, rtol=1e-5)
