"""Shared fixtures of the tests: seeded inputs, golden cases, device/oracle conversions,
tolerances."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import torch

from oracle import fold_oracle as fo

# Parity bar: attention output max-abs 2e-2 in bf16 against the float64 oracle; LSE within 1e-3
# relative (absolute floor 1e-3 for LSEs near zero).
OUT_ATOL = 2e-2
LSE_RTOL = 1e-3


def bf16_tensor(a, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=device, dtype=torch.bfloat16)


def to64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def randn_kv(rng, shape, outliers=0, scale=8.0):
    """N(0,1) values; `outliers` channels per head (last axis) scaled by `scale`."""
    x = rng.standard_normal(shape, dtype=np.float32)
    if outliers:
        ch = rng.choice(shape[-1], size=outliers, replace=False)
        x[..., ch] *= scale
    return x


def lse_close(got, want, rtol=LSE_RTOL):
    got, want = np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64)
    inf_g, inf_w = np.isneginf(got), np.isneginf(want)
    assert np.array_equal(inf_g, inf_w), "empty rows differ"
    fin = ~inf_w
    err = np.abs(got[fin] - want[fin])
    bound = rtol * np.maximum(np.abs(want[fin]), 1.0)
    assert np.all(err <= bound), f"max lse error {err.max() if err.size else 0}"


def lengths(n, hist, device="cuda"):
    qsl = torch.tensor([0, n], dtype=torch.int32, device=device)
    seq = torch.tensor([hist + n], dtype=torch.int32, device=device)
    return qsl, seq


def side_from(k, v, pages, device="cuda"):
    """A side cache holding K, V [L, Hkv, D] at positions 0..L-1 (bf16, host-built)."""
    L, hkv, d = k.shape
    side = np.zeros((pages, hkv, fo.SIDE_BLOCK, 2 * d), dtype=np.float32)
    pos = np.arange(L)
    side[pos // fo.SIDE_BLOCK, :, pos % fo.SIDE_BLOCK, :d] = k
    side[pos // fo.SIDE_BLOCK, :, pos % fo.SIDE_BLOCK, d:] = v
    return bf16_tensor(side.reshape(pages, hkv, fo.SIDE_BLOCK, 2 * d), device)


def paged_from(k, v, block_size, rng, spare_blocks=3, fill=np.nan, device="cuda"):
    """vLLM's FlashAttention cache kv[num_blocks, Hkv, block_size, 2D] (bf16) holding K, V
    [L, Hkv, D] at positions 0..L-1 in shuffled blocks; every other slot holds `fill` (NaN by
    default: the window read must neither use nor be poisoned by it). Returns kv and the block
    table int32 [1, blocks + 2] (the trailing entries are 0, as vLLM pads)."""
    L, hkv, d = k.shape
    nbl = -(-L // block_size)
    nb = nbl + spare_blocks
    perm = rng.permutation(nb)[:nbl]
    kv = np.full((nb, hkv, block_size, 2 * d), fill, dtype=np.float32)
    pos = np.arange(L)
    blk, off = perm[pos // block_size], pos % block_size
    kv[blk, :, off, :d] = k
    kv[blk, :, off, d:] = v
    table = np.zeros((1, nbl + 2), dtype=np.int32)
    table[0, :nbl] = perm
    return bf16_tensor(kv, device), torch.from_numpy(table).to(device)


def torch_local_read(q, kv_cache, meta, original, *, window_size, causal, num_splits):
    """float32 torch window read over a contiguous [seq, 2, Hkv, D] cache (test stand-in for the
    FlashAttention read; FlashAttention semantics: bottom-right aligned window)."""
    k, v = kv_cache[:, 0].float(), kv_cache[:, 1].float()
    n, hq, d = q.shape
    seq = int(meta.seq_lens[0])
    hkv = k.shape[1]
    g = hq // hkv
    left, right = window_size
    p = seq - n + torch.arange(n, device=q.device)
    j = torch.arange(seq, device=q.device)
    dist = p[:, None] - j[None, :]
    mask = torch.ones_like(dist, dtype=torch.bool)
    if left >= 0:
        mask &= dist <= left
    if right >= 0:
        mask &= -dist <= right
    if causal:
        mask &= dist >= 0
    kk = k[:seq].repeat_interleave(g, dim=1)  # [seq, hq, d]
    vv = v[:seq].repeat_interleave(g, dim=1)
    s = torch.einsum("nhd,jhd->hnj", q.float(), kk) * original.scale
    s = s.masked_fill(~mask[None], float("-inf"))
    lse = torch.logsumexp(s, -1)  # [hq, n]
    o = torch.einsum("hnj,jhd->nhd", torch.softmax(s, -1), vv)
    return o.to(q.dtype), lse.float().contiguous()


GOLDEN = Path(__file__).resolve().parent / "golden"


def block_inputs(seed, t, B, hq, hkv, d):
    """The generator of tests/golden/make_golden.py: q, k_ctx, v_ctx, k_blk, v_blk float32 N(0, 1)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, hq, d), dtype=np.float32)
    kc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    kb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    vb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    return q, kc, vc, kb, vb


def golden_block_case(name):
    """A fold_block golden case: dict with q, k_ctx, v_ctx, k_blk, v_blk, inv_freq, window, alpha,
    scale and the reference output `out` (inputs regenerated and hash-checked when not stored)."""
    g = dict(np.load(GOLDEN / name))
    if "q" not in g:
        t, B, hq, hkv, d = (int(g[k]) for k in ("t", "B", "hq", "hkv", "d"))
        q, kc, vc, kb, vb = block_inputs(int(g["seed"]), t, B, hq, hkv, d)
        h = hashlib.sha256()
        for a in (q, kc, vc, kb, vb):
            h.update(a.tobytes())
        assert h.hexdigest() == str(g["inputs_sha256"]), "input generator drifted"
        rot = int(g["rot"]) if "rot" in g else d
        g.update(q=q, k_ctx=kc, v_ctx=vc, k_blk=kb, v_blk=vb, inv_freq=fo.inv_freq(float(g["theta"]), rot))
    g["window"], g["alpha"], g["scale"] = int(g["window"]), float(g["alpha"]), float(g["scale"])
    return g


def golden_block_names(min_hd=0):
    out = []
    for p in sorted(GOLDEN.glob("fold_block_*.npz")):
        with np.load(p) as z:
            d = int(z["d"]) if "d" in z else int(z["q"].shape[-1])
        if d >= min_hd:
            out.append(p.name)
    return out
