"""Generate the golden vectors of tests/golden/ from the reference implementation itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <checkout of the reference>
    (or FOLD_REFERENCE=<checkout> python tests/golden/make_golden.py)

What it runs, all on the CPU:
  * fold.reference.fold_block (fold/reference.py:21-53) on seeded inputs;
  * fold.kernels.far_query / merge / rerope_queries (fold/kernels.py:111-142) through Triton's
    CPU interpreter (TRITON_INTERPRET=1), i.e. the reference's own kernels;
  * the side-cache scatter of fold.attention._wrap_context_kv (fold/attention.py:233-265) with
    a stand-in drafter object whose projections return fixed tensors and whose vLLM rotary op
    is a no-op (the side cache stores keys before RoPE, fold/attention.py:240);
  * the plugin surface: fold.attention.install, use_full_draft_storage and FoldWorkspace
    (fold/attention.py:44-73,270-375) and fold.rope.drafter_rope (fold/rope.py:14-28) on the
    stand-in drafters of tests/standins.py, recording each report or error (plugin_surface.json).

Inputs come from numpy's default_rng so that they regenerate bit for bit on any machine; each
file stores the inputs it needs (small cases) or their sha256 (the full config-1 case).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402

HERE = Path(__file__).resolve().parent


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def block_inputs(seed, t, B, hq, hkv, d):
    """Unrotated q [B, hq, d], k/v ctx [t, hkv, d], k/v blk [B, hkv, d], float32 N(0, 1)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, hq, d), dtype=np.float32)
    kc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((t, hkv, d), dtype=np.float32)
    kb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    vb = rng.standard_normal((B, hkv, d), dtype=np.float32)
    return q, kc, vc, kb, vb


def inv_freq(theta, rot):
    i = np.arange(0, rot, 2, dtype=np.float64)
    return (1.0 / (theta ** (i / rot))).astype(np.float32)


def run_fold_block(torch, ref, q, kc, vc, kb, vb, *, window, alpha, freq, scale):
    g = q.shape[1] // kc.shape[1]
    T = lambda a: torch.from_numpy(np.repeat(a, g, axis=1))  # noqa: E731 (GQA expanded, fold/reference.py:24)
    out = ref.fold_block(torch.from_numpy(q), T(kc), T(vc), T(kb), T(vb), window=window, alpha=alpha,
                         inv_freq=torch.from_numpy(freq), scale=scale)
    return out.numpy()


# (name, seed, t, B, W, hq, hkv, d, rot, theta, alpha)
BLOCK_CASES = [
    ("tiny_nofar", 1, 20, 4, 16, 4, 2, 32, 32, 10000.0, 2.0),       # t < W + B: no row has memory
    ("tiny_edge", 2, 21, 4, 16, 4, 2, 32, 32, 10000.0, 2.0),        # only the last row has one far key
    ("small_mixed", 3, 70, 6, 60, 4, 2, 32, 32, 10000.0, 2.0),      # rows 0..2 without memory, 3..5 with
    ("small_partial_rot", 4, 300, 5, 64, 6, 3, 64, 32, 500000.0, 2.0),  # rotary on half the head
    ("small_alpha1", 5, 257, 8, 100, 8, 2, 64, 64, 1e6, 1.0),
    ("small_alpha3", 6, 513, 3, 128, 2, 1, 128, 128, 500000.0, 3.0),
]


# Larger cases stored as (seed, shapes, sha256 of the inputs, output): the inputs regenerate from
# numpy's default_rng. (name, seed, t, B, W, hq, hkv, d, rot, theta, alpha)
REGEN_CASES = [
    ("gqa4_h128", 41, 1500, 10, 256, 8, 2, 128, 128, 500000.0, 2.0),
    ("gqa2_h256", 42, 900, 8, 128, 4, 2, 256, 256, 1e6, 2.0),
    ("gqa4_h256_tail", 43, 300, 16, 280, 8, 2, 256, 256, 1e6, 2.0),   # only the last rows reach memory
    ("qwen3_like", 44, 3000, 8, 512, 32, 8, 128, 128, 1e6, 2.0),
    ("partial_rot_h128", 45, 700, 5, 100, 4, 1, 128, 64, 500000.0, 3.0),
]


def gen_fold_block(torch, ref, full):
    for name, seed, t, B, W, hq, hkv, d, rot, theta, alpha in BLOCK_CASES:
        q, kc, vc, kb, vb = block_inputs(seed, t, B, hq, hkv, d)
        f = inv_freq(theta, rot)
        scale = d ** -0.5
        out = run_fold_block(torch, ref, q, kc, vc, kb, vb, window=W, alpha=alpha, freq=f, scale=scale)
        np.savez_compressed(HERE / f"fold_block_{name}.npz", q=q, k_ctx=kc, v_ctx=vc, k_blk=kb, v_blk=vb,
                            inv_freq=f, window=W, alpha=alpha, scale=scale, out=out)
        print("fold_block", name, out.shape)
    for name, seed, t, B, W, hq, hkv, d, rot, theta, alpha in REGEN_CASES:
        q, kc, vc, kb, vb = block_inputs(seed, t, B, hq, hkv, d)
        f = inv_freq(theta, rot)
        scale = d ** -0.5
        out = run_fold_block(torch, ref, q, kc, vc, kb, vb, window=W, alpha=alpha, freq=f, scale=scale)
        np.savez_compressed(HERE / f"fold_block_regen_{name}.npz", seed=seed, t=t, B=B, hq=hq, hkv=hkv, d=d,
                            rot=rot, theta=theta, window=W, alpha=alpha, scale=scale,
                            inputs_sha256=sha(q, kc, vc, kb, vb), out=out)
        print("fold_block regen", name, out.shape)
    if full:
        # config 1: batch 1, 32 q / 8 kv heads, hd 128, B 10, t 8192, W 2048, alpha 2, theta 5e5, seed 0
        q, kc, vc, kb, vb = block_inputs(0, 8192, 10, 32, 8, 128)
        f = inv_freq(500000.0, 128)
        scale = 128 ** -0.5
        out = run_fold_block(torch, ref, q, kc, vc, kb, vb, window=2048, alpha=2.0, freq=f, scale=scale)
        np.savez_compressed(HERE / "fold_block_config1.npz", seed=0, t=8192, B=10, hq=32, hkv=8, d=128,
                            theta=500000.0, window=2048, alpha=2.0, scale=scale,
                            inputs_sha256=sha(q, kc, vc, kb, vb), out=out)
        print("fold_block config1", out.shape)


def bf16(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def bits(torch, t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


# (name, seed, n, hq, d, rot, theta, hist, W, B, D)
QUERY_CASES = [
    ("neg_delta", 11, 10, 8, 64, 64, 500000.0, 5000, 2048, 10, 2058),
    ("pos_delta", 12, 4, 4, 64, 64, 10000.0, 30, 40, 4, 44),
    ("partial_rot", 13, 8, 4, 128, 64, 1e6, 100000, 2048, 8, 2056),
    ("big_hist", 14, 10, 8, 128, 128, 500000.0, 131062, 2048, 10, 2058),
    ("short_block", 15, 3, 2, 32, 32, 10000.0, 700, 64, 8, 72),  # qlen < B
]


def gen_queries(torch, kernels):
    for name, seed, n, hq, d, rot, theta, hist, W, B, D in QUERY_CASES:
        rng = np.random.default_rng(seed)
        q = bf16(torch, rng.standard_normal((n, hq, d), dtype=np.float32))
        f = torch.from_numpy(inv_freq(theta, rot))
        qsl = torch.tensor([0, n], dtype=torch.int32)
        seq = torch.tensor([hist + n], dtype=torch.int32)
        fl = torch.zeros(1, dtype=torch.int32)
        qf = kernels.far_query(q, qsl, seq, f, fl, far_distance=D, window=W, block=B)
        fl2 = torch.zeros(1, dtype=torch.int32)
        qs, qr = kernels.rerope_queries(q, qsl, seq, f, fl2, far_distance=D, window=W, block=B,
                                        constant=True, logn_ref=4096)
        np.savez_compressed(HERE / f"far_query_{name}.npz", q=bits(torch, q), inv_freq=f.numpy(), hist=hist,
                            qlen=n, window=W, block=B, far_distance=D, qf=bits(torch, qf),
                            far_len=int(fl.item()), rerope_qs=bits(torch, qs), rerope_qf=bits(torch, qr),
                            rerope_far_len=int(fl2.item()), logn_ref=4096)
        print("far_query", name, int(fl.item()))


# (name, seed, n, hq, d, hist, W, B, alpha)
MERGE_CASES = [
    ("all_far", 21, 10, 8, 128, 9000, 2048, 10, 2.0),
    ("mixed", 22, 6, 4, 64, 70, 60, 6, 2.0),      # rows 0..2 without memory
    ("none_far", 23, 4, 4, 64, 10, 60, 4, 2.0),
    ("alpha3", 24, 8, 4, 256, 5000, 1024, 8, 3.0),
]


def gen_merge(torch, kernels):
    for name, seed, n, hq, d, hist, W, B, alpha in MERGE_CASES:
        rng = np.random.default_rng(seed)
        ol = bf16(torch, rng.standard_normal((n, hq, d), dtype=np.float32))
        of = bf16(torch, rng.standard_normal((n, hq, d), dtype=np.float32))
        ll = torch.from_numpy((rng.standard_normal((hq, n)) * 3 + 5).astype(np.float32))
        lf = torch.from_numpy((rng.standard_normal((hq, n)) * 6 + 10).astype(np.float32))
        out = torch.zeros((n, hq, d), dtype=torch.bfloat16)
        qsl = torch.tensor([0, n], dtype=torch.int32)
        seq = torch.tensor([hist + n], dtype=torch.int32)
        kernels.merge(ol, ll, of, lf, out, qsl, seq, window=W, block=B, alpha=alpha)
        np.savez_compressed(HERE / f"merge_{name}.npz", o_l=bits(torch, ol), lse_l=ll.numpy(), o_f=bits(torch, of),
                            lse_f=lf.numpy(), hist=hist, window=W, block=B, alpha=alpha, out=bits(torch, out))
        print("merge", name)


class _Impl:
    def do_kv_cache_update(self, attn, k, v, cache, slots):
        pass


class _Layer:
    def __init__(self):
        self.impl = _Impl()
        self.kv_cache = None


class _Inner:
    """Stand-in for the drafter model of fold/attention.py:233-265. _project_context_kv returns
    the next prepared (K, V) pair; the key norm is the identity."""

    def __init__(self, torch, L, nkv, hd):
        self._num_attn_layers, self._num_kv_heads, self._head_dim = L, nkv, hd
        self._kv_size = nkv * hd
        self._rope_cos_sin_cache = torch.zeros(8, hd, dtype=torch.bfloat16)
        self._rope_head_size, self._rope_is_neox = hd, True
        self._attn_layers = [_Layer() for _ in range(L)]
        self.next_kv = None

    def _project_context_kv(self, states, num_ctx, L, nkv, hd):
        return self.next_kv

    def _normalize_context_k(self, k):
        return k


def gen_append(torch, attention):
    import vllm._custom_ops as ops

    ops.rotary_embedding = lambda *a, **k: None  # the side cache keeps keys before RoPE
    rng = np.random.default_rng(31)
    L, nkv, hd, max_len = 2, 2, 64, 600
    cache = torch.zeros((4, nkv, 16, 2 * hd), dtype=torch.bfloat16)
    ws = {i: attention.FoldWorkspace(cache, 32, 4, max_len, inv_freq=torch.ones(hd // 2), far_distance=36)
          for i in range(L)}
    inner = _Inner(torch, L, nkv, hd)
    attention._wrap_context_kv(inner, ws)
    calls = []
    # (positions, slots): a prefill chunk, a ragged step, a step with two rejected (invalid) slots,
    # a chunk that crosses page boundaries and overwrites earlier positions
    plan = [
        (np.arange(0, 300), np.arange(0, 300)),
        (np.arange(300, 307), np.arange(300, 307)),
        (np.arange(307, 317), np.array([307, 308, 309, -1, 311, 312, 313, 314, -1, 316])),
        (np.arange(250, 520), np.arange(250, 520)),
        (np.array([599]), np.array([599])),
    ]
    for pos, slots in plan:
        m = pos.size
        k = rng.standard_normal((L, m, nkv, hd), dtype=np.float32)
        v = rng.standard_normal((L, m, nkv, hd), dtype=np.float32)
        inner.next_kv = (bf16(torch, k), bf16(torch, v))
        inner.wrapped_args = None
        inner.precompute_and_store_context_kv(torch.zeros((m, 8)), torch.from_numpy(pos.astype(np.int64)),
                                              torch.from_numpy(slots.astype(np.int64)))
        calls.append(dict(pos=pos.astype(np.int64), slots=slots.astype(np.int64),
                          k=bits(torch, inner.next_kv[0]), v=bits(torch, inner.next_kv[1])))
    out = {}
    for i, c in enumerate(calls):
        for key, val in c.items():
            out[f"c{i}_{key}"] = val
    np.savez_compressed(HERE / "append_scatter.npz", L=L, nkv=nkv, hd=hd, max_len=max_len, ncalls=len(calls),
                        pages=ws[0].side_pages, side0=bits(torch, ws[0].side), side1=bits(torch, ws[1].side), **out)
    print("append pages", ws[0].side_pages)


def _outcome(fn):
    """{"value": fn()} or {"error": exception class name, "message": its text}."""
    try:
        return {"value": fn()}
    except Exception as e:  # noqa: BLE001 - the error itself is the recorded outcome
        return {"error": type(e).__name__, "message": str(e)}


def gen_plugin_surface(torch, attention, rope):
    """The reference's install / use_full_draft_storage / FoldWorkspace / drafter_rope on the
    stand-in drafters of tests/standins.py: every report, every layer's wrapper and workspace
    geometry, every error."""
    import json

    sys.path.insert(0, str(HERE.parents[1]))
    from tests import standins as si

    out = {}
    for name, (scn, kwargs) in si.INSTALL_SCENARIOS.items():
        def run(scn=scn, kwargs=kwargs):
            spec = si.build_speculator(scn)
            rep = attention.install(spec, **kwargs)
            again = attention.install(spec, **kwargs)
            got = si.report_of(spec, rep)
            got["idempotent"] = again is rep
            return got
        out[name] = _outcome(run)
    for name, scn in si.STORAGE_SCENARIOS.items():
        def run(scn=scn):
            spec = si.build_speculator(scn)
            res = attention.use_full_draft_storage(spec)
            again = attention.use_full_draft_storage(spec)
            ctx = spec.vllm_config.compilation_config.static_forward_context
            return {"result": dict(res), "idempotent": again is res,
                    "specs": {k: layer.get_kv_cache_spec("cfg") for k, layer in ctx.items()}}
        out[name] = _outcome(run)
    for name, kwargs in si.ROPE_SCENARIOS.items():
        def run(kwargs=kwargs):
            r = rope.drafter_rope(si.make_rotary(**kwargs))
            return {"inv_freq": [float(x) for x in r.inv_freq.tolist()], "rotary_dim": r.rotary_dim,
                    "head_dim": r.head_dim, "dtype": str(r.inv_freq.dtype)}
        out[name] = _outcome(run)
    for name, (w, b, max_len, mode, shape) in si.WORKSPACE_SCENARIOS.items():
        def run(w=w, b=b, max_len=max_len, mode=mode, shape=shape):
            ws = attention.FoldWorkspace(torch.zeros(shape, dtype=torch.bfloat16), w, b, max_len,
                                         inv_freq=torch.ones(shape[-1] // 4 if len(shape) == 4 else 1),
                                         far_distance=0, mode=mode)
            return {"side_shape": list(ws.side.shape), "side_pages": ws.side_pages, "far_distance": ws.far_distance,
                    "local_splits": ws.local_splits, "window": ws.window, "block": ws.block}
        out[name] = _outcome(run)
    (HERE / "plugin_surface.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("plugin surface cases", len(out))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reference", default=os.environ.get("FOLD_REFERENCE"),
                   help="checkout of the reference (or set FOLD_REFERENCE)")
    p.add_argument("--no-full", action="store_true", help="skip the config-1 case (about 10 s)")
    p.add_argument("--only", choices=["plugin"], help="regenerate only one group of vectors")
    args = p.parse_args()
    if not args.reference:
        p.error("give --reference <checkout> or set FOLD_REFERENCE")
    sys.path.insert(0, args.reference)
    import torch
    from fold import attention, kernels
    from fold import reference as ref
    from fold import rope

    torch.set_num_threads(os.cpu_count() or 1)
    if args.only != "plugin":
        gen_fold_block(torch, ref, not args.no_full)
        gen_queries(torch, kernels)
        gen_merge(torch, kernels)
        gen_append(torch, attention)
    gen_plugin_surface(torch, attention, rope)


if __name__ == "__main__":
    main()
