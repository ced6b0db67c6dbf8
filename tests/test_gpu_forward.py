"""The FOLD forward (FoldAttention.forward with the reference's signature) and the side-cache
append path, on the GPU, against the reference's own fold_block outputs (tests/golden).

Every kernel of the step is the CUDA library: the window read over a paged cache in vLLM's
FlashAttention layout (shuffled blocks, NaN in every unused slot), the rotated far read, the merge
of both split sets and the append. One test replaces the window read through the `local_read`
hook with a float32 torch read."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from fold_b200.attention import FoldAttention, FoldWorkspace, SlidingFoldAttention
from oracle import fold_oracle as fo
from tests.helpers import OUT_ATOL, bf16_tensor, golden_block_case, golden_block_names, paged_from, torch_local_read

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def build_step(g, device="cuda", sliding=False, paged=True, block_size=16):
    """Buffers of one draft step for a golden case: RoPE'd query and drafter cache (paged, or
    [seq, 2, hkv, d] for the torch read), side cache filled through the append kernel (keys before
    RoPE), fake vLLM layer and metadata."""
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    t, B = kc.shape[0], q.shape[0]
    hq, hkv, d = q.shape[1], kc.shape[1], q.shape[2]
    f = g["inv_freq"]
    keys = np.concatenate((kc, kb))
    vals = np.concatenate((vc, vb))
    k_roped = fo.rotate(keys, np.arange(t + B), f)
    q_roped = fo.rotate(q, np.arange(t, t + B), f)
    table = None
    if paged:
        kv_cache, table = paged_from(k_roped, vals, block_size, np.random.default_rng(t), device=device)
    else:
        kv_cache = torch.stack((bf16_tensor(k_roped, device), bf16_tensor(vals, device)), dim=1)  # [seq, 2, hkv, d]
    dummy_cache = torch.zeros((1, hkv, 16, 2 * d), device=device, dtype=torch.bfloat16)
    W = g["window"]
    inv = torch.from_numpy(f).to(device)
    native = W + B - 1  # a sliding layer whose native causal window equals the FOLD window
    ws = FoldWorkspace(dummy_cache, native + 1 - B if sliding else W, B, t + B, inv_freq=inv, far_distance=W + B,
                       alpha=g["alpha"], num_heads=hq)
    pos = torch.arange(t, device=device)
    ws.append(bf16_tensor(kc, device), bf16_tensor(vc, device), pos, pos)
    original = SimpleNamespace(head_size=d, scale=g["scale"], num_heads=hq, sliding_window=(native, 0),
                               vllm_flash_attn_version=4)
    meta = SimpleNamespace(num_actual_tokens=B, query_start_loc=torch.tensor([0, B], dtype=torch.int32, device=device),
                           seq_lens=torch.tensor([t + B], dtype=torch.int32, device=device), max_query_len=B,
                           max_seq_len=t + B, block_table=table, use_cascade=False, causal=True)
    query = bf16_tensor(q_roped, device)
    output = torch.empty((B, hq * d), device=device, dtype=torch.bfloat16)
    return ws, original, meta, query, kv_cache, output


CASES = golden_block_names(min_hd=128)


@pytest.mark.parametrize("name", CASES)
def test_fold_forward_matches_reference(name, far_kernel):
    g = golden_block_case(name)
    ws, original, meta, query, kv_cache, output = build_step(g)
    layer = FoldAttention(original, ws)
    out = layer.forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    ws.check()
    got = out.float().cpu().numpy().reshape(g["out"].shape)
    assert np.abs(got - g["out"]).max() <= OUT_ATOL


@pytest.mark.parametrize("block_size", [32, 256])
def test_fold_forward_block_sizes(block_size):
    g = golden_block_case(CASES[-1])
    ws, original, meta, query, kv_cache, output = build_step(g, block_size=block_size)
    out = FoldAttention(original, ws).forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    ws.check()
    assert np.abs(out.float().cpu().numpy().reshape(g["out"].shape) - g["out"]).max() <= OUT_ATOL


def test_local_read_hook_replaces_the_window_read():
    g = golden_block_case(CASES[0])
    ws, original, meta, query, kv_cache, output = build_step(g, paged=False)
    out = FoldAttention(original, ws, local_read=torch_local_read).forward(None, query, None, None, kv_cache, meta,
                                                                            output)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy().reshape(g["out"].shape) - g["out"]).max() <= OUT_ATOL


@pytest.mark.parametrize("name", CASES[:3])
def test_sliding_fold_forward_matches_reference(name):
    """sliding_layers="fold": native causal window (W + B - 1, 0) as the local branch."""
    g = golden_block_case(name)
    ws, original, meta, query, kv_cache, output = build_step(g, sliding=True)
    layer = SlidingFoldAttention(original, ws)
    out = layer.forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    # with the native window W + B - 1 the native read sees the same near set as FOLD, except the
    # block entries after each row (causal): compare against the oracle of that split
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    t, B = kc.shape[0], q.shape[0]
    f = g["inv_freq"]
    keys = np.concatenate((kc, kb)).astype(np.float64)
    vals = np.concatenate((vc, vb)).astype(np.float64)
    k_roped = fo.bf16_round(fo.rotate(keys, np.arange(t + B), f))
    q_roped = fo.bf16_round(fo.rotate(q, np.arange(t, t + B), f))
    W = g["window"]
    o_l, lse_l = fo.local_read(q_roped, k_roped, fo.bf16_round(vals), t, W + B - 1, 1, g["scale"])
    qf = fo.far_query(q_roped, t, f, W + B)
    lim = fo.far_row_limits(t, W, B, B)
    o_f, lse_f = fo.far_read(qf, fo.bf16_round(keys[:t]), fo.bf16_round(vals[:t]), lim, g["scale"] * g["alpha"])
    want = fo.merge(o_l, lse_l, o_f, lse_f, t, W, B, g["alpha"])
    got = out.float().cpu().numpy().reshape(want.shape)
    assert np.abs(got - want).max() <= OUT_ATOL


def test_window_mode_and_empty_step():
    g = golden_block_case(CASES[0])
    ws, original, meta, query, kv_cache, output = build_step(g)
    ws.mode = "window"
    layer = FoldAttention(original, ws)
    out = layer.forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    t, B = kc.shape[0], q.shape[0]
    f = g["inv_freq"]
    k_roped = fo.bf16_round(fo.rotate(np.concatenate((kc, kb)), np.arange(t + B), f))
    q_roped = fo.bf16_round(fo.rotate(q, np.arange(t, t + B), f))
    o_l, _ = fo.local_read(q_roped, k_roped, fo.bf16_round(np.concatenate((vc, vb))), t, ws.window, B, g["scale"])
    assert np.abs(out.float().cpu().numpy().reshape(o_l.shape) - o_l).max() <= OUT_ATOL
    meta.num_actual_tokens = 0
    assert torch.count_nonzero(layer.forward(None, query, None, None, kv_cache, meta, output)) == 0


def test_native_window_layer_matches_oracle():
    """sliding_layers="window": the plain native causal read, no memory (fold/attention.py:98-123)."""
    from fold_b200.attention import NativeWindowAttention
    g = golden_block_case(CASES[0])
    ws, original, meta, query, kv_cache, output = build_step(g)
    native = 300
    original.sliding_window = (native, 0)
    layer = NativeWindowAttention(original, block=query.shape[0], device=query.device)
    out = layer.forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    layer.check()
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    t, B = kc.shape[0], q.shape[0]
    f = g["inv_freq"]
    k_roped = fo.bf16_round(fo.rotate(np.concatenate((kc, kb)), np.arange(t + B), f))
    q_roped = fo.bf16_round(fo.rotate(q, np.arange(t, t + B), f))
    want, _ = fo.window_read(q_roped, k_roped, fo.bf16_round(np.concatenate((vc, vb))), t, native, 0, True,
                             g["scale"])
    assert np.abs(out.float().cpu().numpy().reshape(want.shape) - want).max() <= OUT_ATOL


# ---------------------------------------------------------------- ReRoPE mode (fold-mode=rerope)
RE_CASE = "fold_block_regen_qwen3_like.npz"  # t = 3000: the log-n scale is above 1 for ref 256
LOGN_REF = 256


def rerope_inputs(g):
    q, kc, vc, kb, vb = g["q"], g["k_ctx"], g["v_ctx"], g["k_blk"], g["v_blk"]
    t, B = kc.shape[0], q.shape[0]
    f = g["inv_freq"]
    keys = np.concatenate((kc, kb)).astype(np.float64)
    vals = np.concatenate((vc, vb)).astype(np.float64)
    k_roped = fo.bf16_round(fo.rotate(keys, np.arange(t + B), f))
    q_roped = fo.bf16_round(fo.rotate(q, np.arange(t, t + B), f))
    return t, B, f, keys, vals, k_roped, q_roped


def test_logn_scale_rows_kernel_matches_oracle():
    """logn_scale_rows (fold/attention.py:76-83) as the query-scale path of the rerope kernel."""
    from fold_b200.attention import logn_scale_rows
    rng = np.random.default_rng(12)
    n, hq, hd = 10, 8, 128
    for hist in (0, 100, 5000, 131062):
        q = bf16_tensor(rng.standard_normal((n, hq, hd), dtype=np.float32))
        qsl = torch.tensor([0, n], dtype=torch.int32, device="cuda")
        seq = torch.tensor([hist + n], dtype=torch.int32, device="cuda")
        got = logn_scale_rows(q, qsl, seq, 4096).float().cpu().numpy()
        want = fo.logn_scale_rows(q.float().cpu().numpy(), hist, 4096)
        assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
        assert (got == fo.bf16_round(want)).mean() > 0.98


def test_fold_forward_rerope_mode_matches_oracle():
    """FoldAttention in rerope mode (fold/attention.py:158-160): the window read of the log-n
    scaled query, the far read of that query rotated to the constant distance D."""
    g = golden_block_case(RE_CASE)
    ws, original, meta, query, kv_cache, output = build_step(g)
    ws.mode, ws.logn_ref = "rerope", LOGN_REF
    out = FoldAttention(original, ws).forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    ws.check()
    t, B, f, keys, vals, k_roped, q_roped = rerope_inputs(g)
    W, alpha, scale = g["window"], g["alpha"], g["scale"]
    qs, qf = fo.rerope_queries(q_roped, t, f, W + B, LOGN_REF)
    o_l, lse_l = fo.local_read(fo.bf16_round(qs), k_roped, fo.bf16_round(vals), t, W, B, scale)
    lim = fo.far_row_limits(t, W, B, B)
    o_f, lse_f = fo.far_read(fo.bf16_round(qf), fo.bf16_round(keys[:t]), fo.bf16_round(vals[:t]), lim, scale * alpha)
    want = fo.merge(o_l, lse_l, o_f, lse_f, t, W, B, alpha)
    assert np.abs(out.float().cpu().numpy().reshape(want.shape) - want).max() <= OUT_ATOL


def test_sliding_fold_forward_rerope_mode_matches_oracle():
    """SlidingFoldAttention in rerope mode (fold/attention.py:203-207): the native causal read of
    the log-n scaled query, the far read of that query rotated to the constant distance."""
    g = golden_block_case(RE_CASE)
    ws, original, meta, query, kv_cache, output = build_step(g, sliding=True)
    ws.mode, ws.logn_ref = "rerope", LOGN_REF
    out = SlidingFoldAttention(original, ws).forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    ws.check()
    t, B, f, keys, vals, k_roped, q_roped = rerope_inputs(g)
    W, alpha, scale = g["window"], g["alpha"], g["scale"]
    qn = fo.bf16_round(fo.logn_scale_rows(q_roped, t, LOGN_REF))
    _, qf = fo.rerope_queries(qn, t, f, W + B, 0)
    o_l, lse_l = fo.window_read(qn, k_roped, fo.bf16_round(vals), t, W + B - 1, 0, True, scale)
    lim = fo.far_row_limits(t, W, B, B)
    o_f, lse_f = fo.far_read(fo.bf16_round(qf), fo.bf16_round(keys[:t]), fo.bf16_round(vals[:t]), lim, scale * alpha)
    want = fo.merge(o_l, lse_l, o_f, lse_f, t, W, B, alpha)
    assert np.abs(out.float().cpu().numpy().reshape(want.shape) - want).max() <= OUT_ATOL


def test_native_window_layer_with_logn_scale_matches_oracle():
    """NativeWindowAttention with logn_ref (fold/attention.py:113-115)."""
    from fold_b200.attention import NativeWindowAttention
    g = golden_block_case(RE_CASE)
    ws, original, meta, query, kv_cache, output = build_step(g)
    native = 300
    original.sliding_window = (native, 0)
    layer = NativeWindowAttention(original, LOGN_REF, block=query.shape[0], device=query.device)
    out = layer.forward(None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    layer.check()
    t, B, f, keys, vals, k_roped, q_roped = rerope_inputs(g)
    qn = fo.bf16_round(fo.logn_scale_rows(q_roped, t, LOGN_REF))
    want, _ = fo.window_read(qn, k_roped, fo.bf16_round(vals), t, native, 0, True, g["scale"])
    assert np.abs(out.float().cpu().numpy().reshape(want.shape) - want).max() <= OUT_ATOL
