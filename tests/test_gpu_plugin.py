"""The wrapped context-K/V path of the install (fold/attention.py:227-267) on the GPU.

The reference clones the normalised keys, lets vLLM's rotary op rotate them in place, then
scatters the clone into the side cache. This package appends the un-rotated keys before the rotary
op runs (one kernel, no clone). The test drives the wrapper with the stand-in drafter of
tests/standins.py and a rotary op that really changes the keys in place, over the same calls as
tests/golden/append_scatter.npz (recorded from the reference's wrapper), and requires the side
caches of both layers to equal the reference's bit for bit, and the KV-cache update to receive
the rotated keys."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from fold_b200 import attention
from fold_b200.attention import FoldWorkspace
from oracle import fold_oracle as fo
from tests.helpers import GOLDEN
from tests.standins import Inner

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).cuda()


def test_wrapped_context_kv_appends_before_the_in_place_rotary(monkeypatch):
    import vllm._custom_ops as ops

    g = np.load(GOLDEN / "append_scatter.npz")
    L, nkv, hd, max_len, pages = int(g["L"]), int(g["nkv"]), int(g["hd"]), int(g["max_len"]), int(g["pages"])
    rotated = []

    def rotary_in_place(positions, key, query, head_size, cos_sin, is_neox):
        key.neg_()  # stands for the rotation: any in-place change of the keys
        rotated.append(int(positions.numel()))

    monkeypatch.setattr(ops, "rotary_embedding", rotary_in_place)
    cache = torch.zeros((4, nkv, 16, 2 * hd), device="cuda", dtype=torch.bfloat16)
    workspaces = {i: FoldWorkspace(cache, 32, 4, max_len, inv_freq=torch.ones(hd // 2, device="cuda"),
                                   far_distance=36) for i in range(L)}
    assert workspaces[0].side_pages == pages
    updates = []

    def kv_update(attn, k, v, kv_cache, slots):
        updates.append((bits(k), bits(v), slots.cpu().numpy()))

    attn_layers = [SimpleNamespace(impl=SimpleNamespace(do_kv_cache_update=kv_update), kv_cache=None)
                   for _ in range(L)]
    inner = Inner([], attn_layers, nkv=nkv, hd=hd, rope_device="cuda")
    attention._wrap_context_kv(inner, workspaces)
    for c in range(int(g["ncalls"])):
        pos, slots = g[f"c{c}_pos"], g[f"c{c}_slots"]
        k, v = from_bits(g[f"c{c}_k"]), from_bits(g[f"c{c}_v"])  # [L, m, nkv, hd]
        inner.next_kv = (k.clone(), v)
        m = pos.size
        inner.precompute_and_store_context_kv(torch.zeros((m, 8), device="cuda"), torch.from_numpy(pos).cuda(),
                                              torch.from_numpy(slots).cuda())
        torch.cuda.synchronize()
        # the KV cache of each layer received the rotated (here: negated) keys and the raw values
        for li in range(L):
            uk, uv, us = updates[-L + li]
            assert np.array_equal(uk, bits(-k[li])) and np.array_equal(uv, g[f"c{c}_v"][li])
            assert np.array_equal(us, slots)
    assert len(rotated) == int(g["ncalls"])
    for li, key in enumerate(("side0", "side1")):
        ref, mine = g[key], bits(workspaces[li].side)
        # the dummy slot received several rows in one call: its content depends on write order
        mask = np.ones(mine.shape[:3], dtype=bool)
        mask[pages - 1, :, fo.SIDE_BLOCK - 1] = False
        assert np.array_equal(mine[mask], ref[mask])
