"""The CPU oracle checked against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). Nothing here needs a GPU."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import fold_oracle as fo

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / name))


BLOCK_CASES = sorted(p.name for p in GOLDEN.glob("fold_block_*.npz") if "config1" not in p.name
                     and "regen" not in p.name)
REGEN_CASES = sorted(p.name for p in GOLDEN.glob("fold_block_regen_*.npz"))


@pytest.mark.parametrize("name", REGEN_CASES)
def test_regenerated_cases_match_reference(name):
    from tests.helpers import golden_block_case
    g = golden_block_case(name)
    out = fo.fold_block(g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"], window=g["window"],
                        alpha=g["alpha"], inv_freq=g["inv_freq"], scale=g["scale"])
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-11)


@pytest.mark.parametrize("name", BLOCK_CASES)
def test_fold_block_matches_reference(name):
    g = load(name)
    out = fo.fold_block(g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"], window=int(g["window"]),
                        alpha=float(g["alpha"]), inv_freq=g["inv_freq"], scale=float(g["scale"]))
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", BLOCK_CASES)
def test_fold_step_from_gpu_buffers_matches_reference(name):
    """The composite the GPU path computes (RoPE'd query and cache, un-rotated side cache, local
    read + far query + far read + merge) equals fold_block."""
    g = load(name)
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    W, alpha, f, scale = int(g["window"]), float(g["alpha"]), g["inv_freq"], float(g["scale"])
    t, B = kc.shape[0], q.shape[0]
    keys = np.concatenate((kc, kb)).astype(np.float64)
    vals = np.concatenate((vc, vb)).astype(np.float64)
    k_roped = fo.rotate(keys, np.arange(t + B), f)
    q_roped = fo.rotate(q, np.arange(t, t + B), f)
    pages = fo.side_pages(t + B)
    side = np.zeros((pages, kc.shape[1], fo.SIDE_BLOCK, 2 * kc.shape[2]))
    fo.append(side, keys, vals, np.arange(t + B), np.arange(t + B))
    out, parts = fo.fold_step(q_roped, k_roped, vals, side, t, window=W, block=B, alpha=alpha, scale=scale,
                              inv_freq=f, round_qf=False)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-10)
    # the parts decompose the reference the same way (Eq. 3, 4)
    ref_out, zn, zf, on, of = fo.fold_block(q, kc, vc, kb, vb, window=W, alpha=alpha, inv_freq=f, scale=scale,
                                            return_parts=True)
    np.testing.assert_allclose(parts["lse_l"], zn.T, rtol=0, atol=1e-10)
    has = np.isfinite(zf)
    np.testing.assert_allclose((parts["lse_f"] / alpha).T[has], zf[has], rtol=0, atol=1e-10)


def test_config1_inputs_regenerate_and_match():
    g = load("fold_block_config1.npz")
    rng = np.random.default_rng(int(g["seed"]))
    t, B, hq, hkv, d = (int(g[k]) for k in ("t", "B", "hq", "hkv", "d"))
    q = rng.standard_normal((B, hq, d), dtype=np.float32)
    kc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    kb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    vb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    h = hashlib.sha256()
    for a in (q, kc, vc, kb, vb):
        h.update(a.tobytes())
    assert h.hexdigest() == str(g["inputs_sha256"])
    f = fo.inv_freq(float(g["theta"]), d)
    out = fo.fold_block(q, kc, vc, kb, vb, window=int(g["window"]), alpha=float(g["alpha"]), inv_freq=f,
                        scale=float(g["scale"]))
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-11)


QUERY_CASES = sorted(p.name for p in GOLDEN.glob("far_query_*.npz"))


def ulp_diff_bf16(a_bits, b_bits):
    """Distance in bfloat16 units in the last place between two bit patterns."""
    def key(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))


@pytest.mark.parametrize("name", QUERY_CASES)
def test_far_query_matches_reference_kernel(name):
    g = load(name)
    q = fo.bits_to_f64(g["q"])
    hist, n = int(g["hist"]), int(g["qlen"])
    assert fo.far_len(hist, g["window"], g["block"], n) == int(g["far_len"])
    D = int(g["far_distance"])
    # the reference kernel's float32 arithmetic, restated, reproduces its output bit for bit
    # (the golden vectors come from Triton's CPU interpreter, which truncates to bfloat16)
    q32 = fo.far_query_f32angle(q, hist, g["inv_freq"], D)
    assert np.array_equal(fo.bf16_trunc_bits(q32), g["qf"])
    # the float64 rotation (fold/reference.py's arithmetic) differs from it only by the float32
    # angle error |D - H| * max(inv_freq) * 2^-24 rad per element, times |q|
    qf = fo.far_query(q, hist, g["inv_freq"], D)
    err = abs(D - hist) * float(np.max(g["inv_freq"])) * 2.0 ** -24 * 2 * np.abs(q).max()
    ref = fo.bits_to_f64(g["qf"])
    assert np.abs(qf - ref).max() <= err + 2.0 ** -7 * np.abs(ref).max()
    # the device's table form (float64 table, float32 arithmetic) tracks the float64 rotation
    table = fo.rope_table(g["inv_freq"], abs(D - hist) + 1)
    qt = fo.far_query_table(q, hist, table, D)
    assert np.abs(qt - qf).max() <= 1e-5 * np.abs(q).max()


@pytest.mark.parametrize("name", QUERY_CASES)
def test_rerope_matches_reference_kernel(name):
    g = load(name)
    q = fo.bits_to_f64(g["q"])
    hist = int(g["hist"])
    assert fo.far_len(hist, g["window"], g["block"], int(g["qlen"])) == int(g["rerope_far_len"])
    D = int(g["far_distance"])
    qs, qf = fo.rerope_queries(q, hist, g["inv_freq"], D, int(g["logn_ref"]))
    assert ulp_diff_bf16(fo.bf16_trunc_bits(qs), g["rerope_qs"]).max() <= 1
    ref = fo.bits_to_f64(g["rerope_qf"])
    err = (abs(D - hist) + q.shape[0]) * float(np.max(g["inv_freq"])) * 2.0 ** -24 * 2 * np.abs(qs).max()
    assert np.abs(qf - ref).max() <= err + 2.0 ** -7 * np.abs(ref).max() + 1e-6


MERGE_CASES = sorted(p.name for p in GOLDEN.glob("merge_*.npz"))


@pytest.mark.parametrize("name", MERGE_CASES)
def test_merge_matches_reference_kernel(name):
    g = load(name)
    out = fo.merge(fo.bits_to_f64(g["o_l"]), g["lse_l"], fo.bits_to_f64(g["o_f"]), g["lse_f"], int(g["hist"]),
                   int(g["window"]), int(g["block"]), float(g["alpha"]))
    # float64 here, float32 in the reference kernel, truncated to bfloat16 by the interpreter
    d = ulp_diff_bf16(fo.bf16_trunc_bits(out), g["out"])
    assert d.max() <= 1
    assert (d == 0).mean() > 0.99


def test_append_matches_reference_scatter():
    g = load("append_scatter.npz")
    L, nkv, hd, pages = int(g["L"]), int(g["nkv"]), int(g["hd"]), int(g["pages"])
    sides = [np.zeros((pages, nkv, fo.SIDE_BLOCK, 2 * hd), dtype=np.uint16) for _ in range(L)]
    dummy_rows = []
    for c in range(int(g["ncalls"])):
        pos, slots = g[f"c{c}_pos"], g[f"c{c}_slots"]
        k, v = g[f"c{c}_k"], g[f"c{c}_v"]
        for li in range(L):
            fo.append(sides[li], k[li], v[li], pos, slots)
        dummy_rows += [(c, i) for i in np.nonzero(slots < 0)[0]]
    for li, key in enumerate(("side0", "side1")):
        ref = g[key]
        mine = sides[li]
        # the dummy slot received several rows in one call: its content depends on write order
        mask = np.ones(mine.shape[:3], dtype=bool)
        mask[pages - 1, :, fo.SIDE_BLOCK - 1] = False
        assert np.array_equal(mine[mask], ref[mask])
        cands = [np.concatenate((g[f"c{c}_k"][li][i], g[f"c{c}_v"][li][i]), -1) for c, i in dummy_rows]
        assert any(np.array_equal(ref[pages - 1, :, fo.SIDE_BLOCK - 1], x) for x in cands)


def test_combine_of_chunks_equals_single_read():
    rng = np.random.default_rng(7)
    n, hq, hkv, d, L = 5, 8, 2, 32, 700
    qf = rng.standard_normal((n, hq, d))
    k = rng.standard_normal((L, hkv, d))
    v = rng.standard_normal((L, hkv, d))
    lim = np.array([0, 1, 300, 699, 700])
    o, lse = fo.far_read(qf, k, v, lim, 0.3)
    cuts = [0, 64, 65, 300, 512, 700]
    parts = [fo.far_read(qf, k[a:b], v[a:b], lim, 0.3, key_lo=a) for a, b in zip(cuts[:-1], cuts[1:])]
    oc, lc = fo.combine(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    np.testing.assert_allclose(oc, o, atol=1e-12)
    np.testing.assert_array_equal(np.isinf(lc), np.isinf(lse))
    fin = np.isfinite(lse)
    np.testing.assert_allclose(lc[fin], lse[fin], atol=1e-12)
    assert np.all(o[0] == 0) and np.all(np.isneginf(lse[:, 0]))


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], dtype=np.float32)
    np.testing.assert_array_equal(fo.bf16_round(x), [1.0, 1.0, 1.0 + 2 ** -6, -2.5, 0.0])


def test_window_read_follows_flash_attention_window_rules():
    """fo.window_read against a per-row loop over FlashAttention's bottom-right window rule
    (key j < seq visible to row r at p = H + r iff p - left <= j <= p + right, and j <= p when
    causal; a negative bound is unbounded), for the FOLD window, a native causal sliding window,
    the unbounded causal case and a row with no key."""
    rng = np.random.default_rng(3)
    n, hq, hkv, d, hist = 4, 4, 2, 16, 37
    seq = hist + n
    q = rng.standard_normal((n, hq, d))
    k = rng.standard_normal((seq, hkv, d))
    v = rng.standard_normal((seq, hkv, d))
    g = hq // hkv
    for left, right, causal in [(9 + n - 1, n - 1, False), (5, 0, True), (-1, -1, True), (-1, 2, False)]:
        o, lse = fo.window_read(q, k, v, hist, left, right, causal, 0.3)
        for r in range(n):
            p = hist + r
            js = [j for j in range(seq) if (left < 0 or p - j <= left) and (right < 0 or j - p <= right)
                  and (not causal or j <= p)]
            for h in range(hq):
                s = np.array([0.3 * q[r, h] @ k[j, h // g] for j in js])
                m = s.max()
                w = np.exp(s - m)
                assert abs(lse[h, r] - (m + np.log(w.sum()))) < 1e-12
                assert np.allclose(o[r, h], (w[:, None] * v[js, h // g]).sum(0) / w.sum(), atol=1e-12)
    o1, l1 = fo.window_read(q, k, v, hist, 9 + n - 1, n - 1, False, 0.3)
    o2, l2 = fo.local_read(q, k, v, hist, 9, n, 0.3)
    assert np.array_equal(o1, o2) and np.array_equal(l1, l2)
    # rows whose window holds no cached key are empty: o = 0, lse = -inf
    o, lse = fo.window_read(q, k, v, hist, 0, 0, False, 0.3, keys_len=hist)
    assert np.all(o == 0) and np.all(np.isneginf(lse))
