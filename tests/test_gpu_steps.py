"""Many draft steps through the public layer API, against the oracle (the Qwen3-8B drafter shape:
32 query / 8 KV heads, head_dim 128, RoPE theta 1e6, block 8, window 2048, alpha 2, context
32768, 200 draft steps accepting 1-8 tokens each, drawn from the seed).

Each step follows the reference's draft loop (fold/attention.py:133-173 for the read,
:233-265 for the commit of accepted tokens):
  1. the block's draft K/V (RoPE'd at H .. H+B-1) are written into the drafter's paged cache;
  2. FoldAttention.forward reads: the window read of the paged cache, the rotated far read of the
     side cache, the merge (the step read in one launch when the shape allows it);
  3. the accepted tokens' committed K/V replace the draft entries in the paged cache, and their
     un-rotated keys and values are appended to the side cache with FoldWorkspace.append.
Every 25th step (and the last) the output is compared with the oracle's FOLD step on the
accumulated context, and far_len with fold/kernels.py:29-30. After the last step every committed
position of the side cache is gathered back and compared bit for bit."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from fold_b200 import kernels
from fold_b200.attention import FoldAttention, FoldWorkspace
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, to64

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

HQ, HKV, HD, B, W, ALPHA, THETA, CTX, STEPS, BS = 32, 8, 128, 8, 2048, 2.0, 1e6, 32768, 200, 16


class PagedCache:
    """The drafter's paged cache kv[blocks, Hkv, BS, 2 * HD] (shuffled blocks) with a host mirror
    of the RoPE'd keys and values at every position, for the oracle."""

    def __init__(self, length, rng):
        nbl = -(-length // BS)
        self.perm = rng.permutation(nbl)
        self.kv = torch.full((nbl, HKV, BS, 2 * HD), float("nan"), device="cuda", dtype=torch.bfloat16)
        self.table = torch.from_numpy(self.perm.astype(np.int32))[None].cuda()
        self.k = np.zeros((length, HKV, HD))  # bf16 values, float64
        self.v = np.zeros((length, HKV, HD))

    def write(self, pos, k_roped, v):
        kb, vb = fo.bf16_round(k_roped), fo.bf16_round(v)
        self.k[pos], self.v[pos] = kb, vb
        p = torch.from_numpy(pos).cuda()
        blk = torch.from_numpy(self.perm[pos // BS]).cuda()
        off = p % BS
        self.kv[blk, :, off, :HD] = bf16_tensor(kb)
        self.kv[blk, :, off, HD:] = bf16_tensor(vb)


def test_two_hundred_draft_steps_match_oracle():
    rng = np.random.default_rng(2026)
    f = fo.inv_freq(THETA, HD)
    acc = rng.integers(1, B + 1, size=STEPS)
    H0 = CTX - B
    length = H0 + int(acc.sum()) + B
    # committed K (before RoPE) and V of every position, and the draft K/V of each step's block
    k_raw = fo.bf16_round(rng.standard_normal((length, HKV, HD), dtype=np.float32))
    v_raw = fo.bf16_round(rng.standard_normal((length, HKV, HD), dtype=np.float32))
    cache = PagedCache(length, rng)
    cache.write(np.arange(H0), fo.rotate(k_raw[:H0], np.arange(H0), f), v_raw[:H0])

    dummy = torch.zeros((1, HKV, 16, 2 * HD), device="cuda", dtype=torch.bfloat16)
    inv = torch.from_numpy(f).cuda()
    ws = FoldWorkspace(dummy, W, B, length, inv_freq=inv, far_distance=W + B, alpha=ALPHA, num_heads=HQ)
    # the prefill: committed context appended in chunks, as precompute_and_store_context_kv does
    for a in range(0, H0, 8192):
        b = min(H0, a + 8192)
        pos = torch.arange(a, b, device="cuda")
        ws.append(bf16_tensor(k_raw[a:b]), bf16_tensor(v_raw[a:b]), pos, pos)
    original = SimpleNamespace(head_size=HD, scale=HD ** -0.5, num_heads=HQ, sliding_window=(-1, -1),
                               vllm_flash_attn_version=4)
    layer = FoldAttention(original, ws)
    output = torch.empty((B, HQ * HD), device="cuda", dtype=torch.bfloat16)
    qsl = torch.tensor([0, B], dtype=torch.int32, device="cuda")
    H = H0
    checked = []
    for i in range(STEPS):
        blk = np.arange(H, H + B)
        k_draft = rng.standard_normal((B, HKV, HD), dtype=np.float32)
        v_draft = rng.standard_normal((B, HKV, HD), dtype=np.float32)
        cache.write(blk, fo.rotate(k_draft, blk, f), v_draft)
        q_roped = fo.bf16_round(fo.rotate(rng.standard_normal((B, HQ, HD), dtype=np.float32), blk, f))
        meta = SimpleNamespace(num_actual_tokens=B, query_start_loc=qsl,
                               seq_lens=torch.tensor([H + B], dtype=torch.int32, device="cuda"), max_query_len=B,
                               max_seq_len=H + B, block_table=cache.table, use_cascade=False, causal=True)
        out = layer.forward(None, bf16_tensor(q_roped), None, None, cache.kv, meta, output)
        if i % 25 == 0 or i == STEPS - 1:
            torch.cuda.synchronize()
            ws.check()
            assert int(ws.far_len.item()) == fo.far_len(H, W, B, B)
            o_l, lse_l = fo.local_read(q_roped, cache.k, cache.v, H, W, B, original.scale)
            qf = fo.far_query(q_roped, H, f, W + B)
            lim = fo.far_row_limits(H, W, B, B)
            o_f, lse_f = fo.far_read(qf, k_raw[:int(lim.max())], v_raw[:int(lim.max())], lim,
                                     original.scale * ALPHA)
            want = fo.merge(o_l, lse_l, o_f, lse_f, H, W, B, ALPHA)
            err = np.abs(to64(out).reshape(B, HQ, HD) - want).max()
            checked.append((i, H, err))
            assert err <= OUT_ATOL, f"step {i} (H = {H}): max error {err}"
        # commit the accepted tokens: the paged cache gets their K/V, the side cache their raw K, V
        a = int(acc[i])
        com = np.arange(H, H + a)
        cache.write(com, fo.rotate(k_raw[com], com, f), v_raw[com])
        p = torch.from_numpy(com).cuda()
        ws.append(bf16_tensor(k_raw[com]), bf16_tensor(v_raw[com]), p, p)
        H += a
    torch.cuda.synchronize()
    ws.check()
    print("checked steps (step, H, max error):", [(i, h, round(float(e), 5)) for i, h, e in checked])
    # the side cache holds every committed position, bit for bit
    pos = torch.arange(H, device="cuda")
    kg, vg = kernels.gather(ws.side, pos, err=ws.err)
    torch.cuda.synchronize()
    ws.check()
    assert np.array_equal(fo.bf16_bits(k_raw[:H]), kg.cpu().view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(fo.bf16_bits(v_raw[:H]), vg.cpu().view(torch.int16).numpy().view(np.uint16))
