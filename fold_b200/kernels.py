"""Python face of the CUDA kernels, with the reference's kernel API (fold/kernels.py:111-142).

far_query, rerope_queries and merge keep the reference's names, arguments and results. far_read,
append, gather and combine are the new entry points that replace the FlashAttention read of the
side cache and its torch scatter. All of them run on the current CUDA stream, read the step
lengths on the device (graph-capturable) and raise FoldError when the library reports an error.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from .errors import FoldError
from .rope import rope_table

SIDE_BLOCK = 256  # positions per side-cache page (fold/attention.py:48)
DEFAULT_TABLE_ROWS = 1 << 18


def _p(t):
    return None if t is None else t.data_ptr()


# The raw handle of the current stream without building a torch.cuda.Stream object (~0.2 us
# instead of ~2 us per call); the public accessor where this torch build lacks it.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise FoldError("FOLD kernels take CUDA tensors (there is no CPU path)")


def _check_lengths(qsl, seq_lens):
    if qsl.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise FoldError("query_start_loc and seq_lens must be int32")


def _table_for(inv_freq, device, rows):
    return rope_table(inv_freq, rows, device)


def far_query(q, qsl, seq_lens, inv_freq, far_len, *, far_distance, window, block, table=None):
    """q [n, Hq, D] -> far query [n, Hq, D] rotated by (D - H) * inv_freq. Writes far_len[0].
    (fold/kernels.py:111-119). `table` is an optional prebuilt rope table."""
    _require_cuda(q, qsl, seq_lens, far_len)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    if table is None:
        table = _table_for(inv_freq, q.device, DEFAULT_TABLE_ROWS + int(far_distance) + 1)
    qf = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    _lib.call("fold_far_query", _p(q), q.stride(0), q.stride(1), _p(qf), qf.stride(0), qf.stride(1), _p(qsl),
              _p(seq_lens), _p(table), table.shape[0], table.shape[1], _p(far_len), n, hq, d, int(window), int(block),
              int(far_distance), None, _stream(q))
    return qf


def rerope_queries(q, qsl, seq_lens, inv_freq, far_len, *, far_distance, window, block, constant, logn_ref,
                   table=None):
    """q [n, Hq, D] -> (window query, far query) for the ReRoPE baseline. Writes far_len[0].
    (fold/kernels.py:122-132)."""
    _require_cuda(q, qsl, seq_lens, far_len)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    if table is None:
        table = _table_for(inv_freq, q.device, DEFAULT_TABLE_ROWS + int(far_distance) + n + 1)
    qs = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    qf = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    inv_log_ref = (1.0 / math.log(logn_ref)) if logn_ref else 0.0
    _lib.call("fold_rerope_query", _p(q), q.stride(0), q.stride(1), _p(qs), qs.stride(0), qs.stride(1), _p(qf),
              qf.stride(0), qf.stride(1), _p(qsl), _p(seq_lens), _p(table), table.shape[0], table.shape[1],
              _p(far_len), n, hq, d, int(window), int(block), int(far_distance), int(bool(constant)),
              float(inv_log_ref), None, _stream(q))
    return qs, qf


def logn_scale(q, qsl, seq_lens, logn_ref):
    """q [n, Hq, D] -> q * max(1, log(H + r + 1) / log(logn_ref)) for row r at position H + r,
    the ReRoPE query scale of fold/attention.py:76-83 (the query-scale path of fold_rerope_query;
    the step lengths are read on the device)."""
    _require_cuda(q, qsl, seq_lens)
    _check_lengths(qsl, seq_lens)
    if not logn_ref or logn_ref <= 1:
        raise FoldError("logn_scale: logn_ref must be greater than 1")
    n, hq, d = q.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    qs = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    if n == 0:
        return qs
    if q.dtype != torch.bfloat16:
        raise FoldError("logn_scale: q must be bfloat16")
    _lib.call("fold_rerope_query", _p(q), q.stride(0), q.stride(1), _p(qs), qs.stride(0), qs.stride(1), None, 0, 0,
              _p(qsl), _p(seq_lens), None, 0, 0, None, n, hq, d, 0, 1, 0, 0, 1.0 / math.log(logn_ref), None,
              _stream(q))
    return qs


def merge(out_l, lse_l, out_f, lse_f, out, qsl, seq_lens, *, window, block, alpha):
    """Writes the mass-weighted merge into out [n, Hq, D] (fold/kernels.py:135-142).

    out_l [n, Hq, D] bf16, lse_l [Hq, n]. The far side is either one read, out_f [n, Hq, D]
    (bf16 or float32) with lse_f [Hq, n], or the split partials of far_read, out_f
    [S, n, Hq, D] float32 with lse_f [S, Hq, n], which are combined on the fly."""
    _require_cuda(out_l, lse_l, out_f, lse_f, out, qsl, seq_lens)
    _check_lengths(qsl, seq_lens)
    n, hq, d = out_l.shape
    if out_f.dim() == 3:
        of_s, (of_t, of_h), splits = 0, out_f.stride()[:2], 1
        lf_s, lf_h, lf_t = 0, lse_f.stride(0), lse_f.stride(1)
    else:
        splits = out_f.shape[0]
        of_s, of_t, of_h = out_f.stride()[:3]
        lf_s, lf_h, lf_t = lse_f.stride()
    if out_f.stride(-1) != 1 or out_l.stride(-1) != 1 or out.stride(-1) != 1:
        raise FoldError("merge: the head dimension must be contiguous")
    if out_l.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise FoldError("merge: out_l and out must be bfloat16")
    if out_f.dtype not in (torch.bfloat16, torch.float32) or lse_l.dtype != torch.float32 or lse_f.dtype != torch.float32:
        raise FoldError("merge: out_f must be bf16/float32 and the LSEs float32")
    _lib.call("fold_merge", _p(out_l), out_l.stride(0), out_l.stride(1), _p(lse_l), lse_l.stride(0), lse_l.stride(1),
              _p(out_f), int(out_f.dtype == torch.bfloat16), of_s, of_t, of_h, _p(lse_f), lf_s, lf_h, lf_t, splits,
              _p(out), out.stride(0), out.stride(1), _p(qsl), _p(seq_lens), n, hq, d, int(window), int(block),
              1.0 / float(alpha), _stream(out))


def _check_partials(o_part, lse_part, n, hq, d, what):
    splits = o_part.shape[0]
    if o_part.shape != (splits, n, hq, d) or lse_part.shape != (splits, hq, n) or not o_part.is_contiguous() \
            or not lse_part.is_contiguous() or o_part.dtype != torch.float32 or lse_part.dtype != torch.float32:
        raise FoldError(f"{what}: partials must be contiguous float32 [S, n, Hq, D] and [S, Hq, n]")
    return splits


def _side_args(q, side, table, rot_dim, pos_lo, capacity, far_len):
    """(q, C-ABI arguments from the rope table to far_len) of a far read of `side`."""
    n, hq, d = q.shape
    pages = side.shape[0]
    if side.dtype != torch.bfloat16 or q.dtype != torch.bfloat16:
        raise FoldError("far_read: q and the side cache must be bfloat16")
    if not side.is_contiguous() or side.shape[2] != SIDE_BLOCK or side.shape[3] != 2 * d:
        raise FoldError("far_read: side cache must be a contiguous [pages, Hkv, 256, 2 * head_dim] tensor")
    if q.stride(-1) != 1:
        q = q.contiguous()
    if capacity is None:
        capacity = int(pos_lo) + (pages - 1) * SIDE_BLOCK
    if table is not None and rot_dim is None:
        rot_dim = table.shape[1]
    return q, (_p(table), 0 if table is None else table.shape[0], 0 if table is None else int(rot_dim), _p(side),
               pages, int(pos_lo), int(capacity), _p(far_len))


def _paged_args(q, k_cache, v_cache, block_table, window_size, causal):
    """(q, C-ABI arguments from the cache planes to `causal`) of a window read."""
    n, hq, d = q.shape
    nb, hkv, bs, dk = k_cache.shape
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise FoldError("window_read: q and the cache must be bfloat16")
    if v_cache.shape != k_cache.shape or dk != d or k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1:
        raise FoldError("window_read: K and V planes must be [num_blocks, Hkv, block_size, head_dim] views with "
                        "equal strides and a contiguous head dimension")
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise FoldError("window_read: block_table must be int32 with contiguous rows")
    if q.stride(-1) != 1:
        q = q.contiguous()
    left, right = (int(w) for w in window_size)
    st_block, st_head, st_slot = k_cache.stride()[:3]
    return q, (_p(k_cache), _p(v_cache), nb, bs, st_block, st_head, st_slot, _p(block_table), block_table.shape[-1],
               left, right, int(bool(causal)))


def far_read(q, qsl, seq_lens, side, o_part, lse_part, *, window, block, far_distance, softmax_scale,
             table=None, rot_dim=None, far_len=None, qf=None, pos_lo=0, capacity=None, err=None):
    """Split-KV read of the side cache with the far-query rotation fused in.

    q [n, Hq, D] bf16, RoPE'd at positions H + r (or already the far query when table is None);
    side [pages, Hkv, 256, 2D] bf16; o_part [S, n, Hq, D] and lse_part [S, Hq, n] float32 receive
    one normalised partial per split. The cache holds positions [pos_lo, pos_lo + (pages-1)*256);
    capacity (default: that range's end) bounds far_len for the capacity check."""
    _require_cuda(q, qsl, seq_lens, side, o_part, lse_part, table, far_len, qf, err)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q.shape
    splits = _check_partials(o_part, lse_part, n, hq, d, "far_read")
    q, side_args = _side_args(q, side, table, rot_dim, pos_lo, capacity, far_len)
    _lib.call("fold_far_read", _p(q), q.stride(0), q.stride(1), _p(qsl), _p(seq_lens), *side_args, _p(qf),
              0 if qf is None else qf.stride(0), 0 if qf is None else qf.stride(1), _p(o_part), _p(lse_part), splits,
              n, hq, side.shape[1], d, int(window), int(block), int(far_distance), float(softmax_scale), _p(err),
              _stream(q))


def far_read_exchange(exchange, q, qsl, seq_lens, side, o_part, lse_part, out_l, lse_l, out, *, window, block,
                      far_distance, softmax_scale, alpha, table=None, rot_dim=None, far_len=None, pos_lo=0,
                      capacity=None, err=None):
    """far_read followed, in the same cooperative launch, by the exchange of the ranks' partials
    and the merge with the window read (out_l [n, Hq, D] bf16, lse_l [Hq, n]) into out [n, Hq, D]
    bf16; `exchange` is the handle of an open exchange (shard.PeerExchange; one rank: the far
    read and the merge in one launch). o_part/lse_part are the far read's split buffers (scratch).
    The far softmax scale is alpha * softmax_scale."""
    _require_cuda(q, qsl, seq_lens, side, o_part, lse_part, out_l, lse_l, out, table, far_len, err)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q.shape
    splits = _check_partials(o_part, lse_part, n, hq, d, "far_read_exchange")
    if tuple(out_l.shape) != (n, hq, d) or tuple(out.shape) != (n, hq, d):
        raise FoldError("far_read_exchange: q, out_l and out shapes differ")
    if out_l.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or lse_l.dtype != torch.float32:
        raise FoldError("far_read_exchange: out_l and out must be bfloat16 and lse_l float32")
    if out_l.stride(-1) != 1 or out.stride(-1) != 1:
        raise FoldError("far_read_exchange: the head dimension must be contiguous")
    q, side_args = _side_args(q, side, table, rot_dim, pos_lo, capacity, far_len)
    _lib.call("fold_far_read_exchange", exchange, _p(q), q.stride(0), q.stride(1), _p(qsl), _p(seq_lens), *side_args,
              _p(o_part), _p(lse_part), splits, _p(out_l), out_l.stride(0), out_l.stride(1), _p(lse_l),
              lse_l.stride(0), lse_l.stride(1), _p(out), out.stride(0), out.stride(1), n, hq, side.shape[1], d,
              int(window), int(block), int(far_distance), float(softmax_scale) * float(alpha), 1.0 / float(alpha),
              _p(err), _stream(q))


def paged_planes(kv_cache, head_dim):
    """K and V planes [num_blocks, Hkv, block_size, D] of vLLM's FlashAttention cache
    kv_cache[num_blocks, Hkv, block_size, 2 * D] (views, no copy)."""
    return kv_cache[..., :head_dim], kv_cache[..., head_dim:]


def window_read(q, qsl, seq_lens, k_cache, v_cache, block_table, o_part, lse_part, *, window_size, causal,
                softmax_scale, err=None):
    """Exact-position window read of a paged cache into split partials (the FlashAttention window
    read of fold/attention.py:148-151,163 and :211-215).

    q [n, Hq, D] bf16 (RoPE'd); k_cache, v_cache [num_blocks, Hkv, block_size, D] bf16 planes with
    equal strides (paged_planes of vLLM's cache); block_table int32 [1, max_blocks] or
    [max_blocks]; window_size (left, right) as FlashAttention's (-1: unbounded). o_part
    [S, n, Hq, D] and lse_part [S, Hq, n] float32 receive one partial per split."""
    _require_cuda(q, qsl, seq_lens, k_cache, v_cache, block_table, o_part, lse_part, err)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q.shape
    splits = _check_partials(o_part, lse_part, n, hq, d, "window_read")
    q, paged = _paged_args(q, k_cache, v_cache, block_table, window_size, causal)
    _lib.call("fold_window_read", _p(q), q.stride(0), q.stride(1), _p(qsl), _p(seq_lens), *paged, float(softmax_scale),
              _p(o_part), _p(lse_part), splits, n, hq, k_cache.shape[1], d, _p(err), _stream(q))


def step_read(q_far, q_win, qsl, seq_lens, side, far_parts, k_cache, v_cache, block_table, window_parts, plan, *,
              window, block, far_distance, softmax_scale, alpha, window_size, causal, table=None, rot_dim=None,
              far_len=None, pos_lo=0, capacity=None, err=None):
    """The far read (as far_read, of q_far) and the window read (as window_read, of q_win) of one
    draft step in one launch: the S blocks of each KV head share the two reads, split per step
    from the device-side lengths. far_parts and window_parts are (o, lse) buffers of S slots each;
    the step stores its split (window blocks) in plan (int32 [1], device), which merge_partials
    reads. The far softmax scale is alpha * softmax_scale, the window's softmax_scale. Not for
    shapes whose far read takes the tcgen05 kernel (far_read_uses_tcgen05)."""
    (fo_, fl_), (wo_, wl_) = far_parts, window_parts
    _require_cuda(q_far, q_win, qsl, seq_lens, side, fo_, fl_, k_cache, v_cache, block_table, wo_, wl_, plan, table,
                  far_len, err)
    _check_lengths(qsl, seq_lens)
    n, hq, d = q_far.shape
    if q_win.shape != q_far.shape:
        raise FoldError("step_read: the far and window queries must have the same shape")
    splits = _check_partials(fo_, fl_, n, hq, d, "step_read")
    if _check_partials(wo_, wl_, n, hq, d, "step_read") != splits:
        raise FoldError("step_read: the far and window partials must have the same number of slots")
    if plan.dtype != torch.int32 or plan.numel() < 1:
        raise FoldError("step_read: plan must be an int32 tensor of at least one element")
    q_far, side_args = _side_args(q_far, side, table, rot_dim, pos_lo, capacity, far_len)
    q_win, paged = _paged_args(q_win, k_cache, v_cache, block_table, window_size, causal)
    _lib.call("fold_step_read", _p(q_far), q_far.stride(0), q_far.stride(1), _p(q_win), q_win.stride(0),
              q_win.stride(1), _p(qsl), _p(seq_lens), *side_args, _p(fo_), _p(fl_), *paged, _p(wo_), _p(wl_),
              splits, _p(plan), n, hq, side.shape[1], d, int(window), int(block), int(far_distance),
              float(softmax_scale) * float(alpha), float(softmax_scale), _p(err), _stream(q_far))


def merge_partials(o_wpart, lse_wpart, o_fpart, lse_fpart, out, qsl, seq_lens, *, window, block, alpha, plan=None):
    """Writes into out [n, Hq, D] bf16 the alpha-weighted merge (fold/kernels.py:135-142) of the
    window read's split partials (o_wpart [Sw, n, Hq, D], lse_wpart [Sw, Hq, n]) with the far
    read's (o_fpart [Sf, n, Hq, D], lse_fpart [Sf, Hq, n]); with o_fpart None the combined window
    read alone. With `plan` (step_read's device word) only the slots that step used are read."""
    _require_cuda(o_wpart, lse_wpart, o_fpart, lse_fpart, out, qsl, seq_lens, plan)
    _check_lengths(qsl, seq_lens)
    sw, n, hq, d = o_wpart.shape
    sf = 0 if o_fpart is None else o_fpart.shape[0]
    for o, l, s in ((o_wpart, lse_wpart, sw), (o_fpart, lse_fpart, sf)):
        if o is None:
            continue
        if o.shape != (s, n, hq, d) or l.shape != (s, hq, n) or o.dtype != torch.float32 \
                or l.dtype != torch.float32 or not o.is_contiguous() or not l.is_contiguous():
            raise FoldError("merge_partials: partials must be contiguous float32 [S, n, Hq, D] and [S, Hq, n]")
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1 or out.shape != (n, hq, d):
        raise FoldError("merge_partials: out must be bfloat16 [n, Hq, D] with a contiguous head dimension")
    if plan is not None and (plan.dtype != torch.int32 or sf != sw):
        raise FoldError("merge_partials: a step plan is int32, with both partial sets of the same slot count")
    _lib.call("fold_merge_partials", _p(o_wpart), _p(lse_wpart), sw, _p(o_fpart), _p(lse_fpart), sf, _p(plan),
              _p(out), out.stride(0), out.stride(1), _p(qsl), _p(seq_lens), n, hq, d, int(window), int(block),
              1.0 / float(alpha), _stream(out))


def append(k, v, positions, slots, side, *, pos_lo=0, skip_foreign=False, err=None):
    """Writes K [ctx, Hkv, D] (before RoPE) and V [ctx, Hkv, D] of committed entries into the
    side cache at their positions (fold/attention.py:260-265); rows with slot < 0 go to the
    dummy slot. positions and slots are int64 (int32 inputs are widened)."""
    _require_cuda(k, v, positions, slots, side, err)
    ctx = k.shape[0]
    if ctx == 0:
        return
    pages, hkv, _, d2 = side.shape
    if k.dtype != side.dtype or v.dtype != side.dtype or side.dtype != torch.bfloat16:
        raise FoldError("append: K, V and the side cache must be bfloat16")
    if k.shape[1:] != (hkv, d2 // 2) or v.shape[1:] != (hkv, d2 // 2) or v.shape[0] < ctx:
        raise FoldError("append: K/V must be [ctx, Hkv, head_dim] matching the side cache")
    if k.stride(-1) != 1 or v.stride(-1) != 1:
        raise FoldError("append: the head dimension of K and V must be contiguous")
    if positions.dim() != 1 or slots.dim() != 1 or positions.shape[0] < ctx or slots.shape[0] < ctx:
        raise FoldError("append: positions and slots need one entry per K/V row")
    if positions.shape[0] != ctx or positions.dtype != torch.int64 or not positions.is_contiguous():
        positions = positions[:ctx].to(torch.int64).contiguous()
    if slots.shape[0] != ctx or slots.dtype != torch.int64 or not slots.is_contiguous():
        slots = slots[:ctx].to(torch.int64).contiguous()
    _lib.call("fold_append", _p(k), k.stride(0), k.stride(1), _p(v), v.stride(0), v.stride(1), _p(positions),
              _p(slots), ctx, _p(side), pages, hkv, d2 // 2, int(pos_lo), int(bool(skip_foreign)), _p(err),
              _stream(side))


FP8_HEAD_DIM = 128  # the fp8 side cache's head size


def fp8_side_shape(pages: int, hkv: int):
    """Shape of an fp8 side cache of `pages` pages (uint8; layout in include/fold_b200.h)."""
    return (int(pages), int(hkv), 2, 2, 128, 128)


def _check_fp8_side(side8, k_scale, v_scale):
    if side8.dtype != torch.uint8 or side8.dim() != 6 or tuple(side8.shape[2:]) != (2, 2, 128, 128) \
            or not side8.is_contiguous():
        raise FoldError("fp8 side cache: a contiguous uint8 [pages, Hkv, 2, 2, 128, 128] tensor")
    hkv = side8.shape[1]
    for s in (k_scale, v_scale):
        if s.dtype != torch.float32 or s.numel() != hkv or not s.is_contiguous():
            raise FoldError("fp8 side cache: k_scale and v_scale are contiguous float32 [Hkv]")


def append_fp8(k, v, positions, slots, side8, k_scale, v_scale, *, pos_lo=0, skip_foreign=False, err=None):
    """Quantising append into an fp8 side cache: K [ctx, Hkv, 128] (before RoPE) and V, bf16, are
    divided by the per-head scales and rounded to e4m3 (fold_append_fp8)."""
    _require_cuda(k, v, positions, slots, side8, k_scale, v_scale, err)
    ctx = k.shape[0]
    if ctx == 0:
        return
    _check_fp8_side(side8, k_scale, v_scale)
    hkv = side8.shape[1]
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise FoldError("append_fp8: K and V must be bfloat16")
    if k.shape[1:] != (hkv, FP8_HEAD_DIM) or v.shape[1:] != (hkv, FP8_HEAD_DIM) or v.shape[0] < ctx:
        raise FoldError("append_fp8: K/V must be [ctx, Hkv, 128] matching the side cache")
    if k.stride(-1) != 1 or v.stride(-1) != 1:
        raise FoldError("append_fp8: the head dimension of K and V must be contiguous")
    if positions.dim() != 1 or slots.dim() != 1 or positions.shape[0] < ctx or slots.shape[0] < ctx:
        raise FoldError("append_fp8: positions and slots need one entry per K/V row")
    positions = positions[:ctx].to(torch.int64).contiguous()
    slots = slots[:ctx].to(torch.int64).contiguous()
    _lib.call("fold_append_fp8", _p(k), k.stride(0), k.stride(1), _p(v), v.stride(0), v.stride(1), _p(positions),
              _p(slots), ctx, _p(side8), side8.shape[0], hkv, FP8_HEAD_DIM, _p(k_scale), _p(v_scale), int(pos_lo),
              int(bool(skip_foreign)), _p(err), _stream(side8))


def far_read_fp8(q, qsl, seq_lens, side8, k_scale, v_scale, o_part, lse_part, *, window, block, far_distance,
                 softmax_scale, table=None, rot_dim=None, far_len=None, pos_lo=0, capacity=None, err=None):
    """far_read of an fp8 side cache (fold_far_read_fp8): the same split partials, with K and V
    the e4m3 values times their per-head scales."""
    _require_cuda(q, qsl, seq_lens, side8, k_scale, v_scale, o_part, lse_part, table, far_len, err)
    _check_lengths(qsl, seq_lens)
    _check_fp8_side(side8, k_scale, v_scale)
    n, hq, d = q.shape
    if d != FP8_HEAD_DIM or q.dtype != torch.bfloat16:
        raise FoldError("far_read_fp8: q must be bfloat16 with head size 128")
    splits = _check_partials(o_part, lse_part, n, hq, d, "far_read_fp8")
    if q.stride(-1) != 1:
        q = q.contiguous()
    pages = side8.shape[0]
    if capacity is None:
        capacity = int(pos_lo) + (pages - 1) * SIDE_BLOCK
    if table is not None and rot_dim is None:
        rot_dim = table.shape[1]
    _lib.call("fold_far_read_fp8", _p(q), q.stride(0), q.stride(1), _p(qsl), _p(seq_lens), _p(table),
              0 if table is None else table.shape[0], 0 if table is None else int(rot_dim), _p(side8), pages,
              int(pos_lo), int(capacity), _p(far_len), _p(k_scale), _p(v_scale), _p(o_part), _p(lse_part), splits, n,
              hq, side8.shape[1], d, int(window), int(block), int(far_distance), float(softmax_scale), _p(err),
              _stream(q))


def gather(side, positions, *, pos_lo=0, err=None):
    """K, V [m, Hkv, D] of the given absolute positions of a side cache."""
    _require_cuda(side, positions, err)
    pages, hkv, _, d2 = side.shape
    positions = positions.to(torch.int64).contiguous()
    m = positions.numel()
    k = torch.empty((m, hkv, d2 // 2), device=side.device, dtype=side.dtype)
    v = torch.empty_like(k)
    _lib.call("fold_gather", _p(side), pages, hkv, d2 // 2, int(pos_lo), _p(positions), m, _p(k), _p(v), _p(err),
              _stream(side))
    return k, v


def combine(o_part, lse_part, o_out=None, lse_out=None):
    """Log-sum-exp combine of S partials [S, n, Hq, D] / [S, Hq, n] into one (float32)."""
    _require_cuda(o_part, lse_part)
    s, n, hq, d = o_part.shape
    if o_out is None:
        o_out = torch.empty((n, hq, d), device=o_part.device, dtype=torch.float32)
    if lse_out is None:
        lse_out = torch.empty((hq, n), device=o_part.device, dtype=torch.float32)
    _lib.call("fold_combine", _p(o_part.contiguous()), _p(lse_part.contiguous()), s, _p(o_out), _p(lse_out), n, hq, d,
              _stream(o_part))
    return o_out, lse_out


def allgather_partials(comm, o_part, lse_part, send, recv):
    """The NCCL step of the sharded far read (fold_allgather_partials): this rank's split partials
    o_part [S, n, Hq, D] / lse_part [S, Hq, n] are combined into `send` (one record of n*Hq*D +
    Hq*n floats: o then lse) and every rank's record is all-gathered into recv [world * record]
    with ncclAllGather on the communicator `comm` (an ncclComm_t address). Returns the gathered
    (o [world, n, Hq, D], lse [world, Hq, n]) views of recv, ready for merge()."""
    _require_cuda(o_part, lse_part, send, recv)
    s, n, hq, d = o_part.shape
    _check_partials(o_part, lse_part, n, hq, d, "allgather_partials")
    per = n * hq * d + hq * n
    if send.dtype != torch.float32 or recv.dtype != torch.float32 or not send.is_contiguous() \
            or not recv.is_contiguous() or send.numel() < per or recv.numel() % per or recv.numel() < per:
        raise FoldError("allgather_partials: send holds one record and recv whole records (float32, contiguous)")
    if not comm:
        raise FoldError("allgather_partials: no NCCL communicator")
    _lib.call("fold_allgather_partials", int(comm), _p(o_part), _p(lse_part), s, _p(send), _p(recv), n, hq, d,
              _stream(o_part))
    world = recv.numel() // per
    b = recv.view(world, per)
    return b[:, : n * hq * d].view(world, n, hq, d), b[:, n * hq * d:].view(world, hq, n)


FAR_READ_KERNELS = {"auto": -1, "mma": 0, "tc": 1}


def select_far_read_kernel(kernel: str = "auto") -> None:
    """Choose the far-read kernel for later calls: "mma" (mma.sync tiles), "tc" (tcgen05 tiles with
    TMEM accumulators) or "auto" (per shape)."""
    if kernel not in FAR_READ_KERNELS:
        raise FoldError(f"far-read kernel must be one of {sorted(FAR_READ_KERNELS)}")
    _lib.call("fold_far_read_select_kernel", FAR_READ_KERNELS[kernel])


def far_read_uses_tcgen05(hd, n, hq, hkv) -> bool:
    """Whether the far read of this shape takes the tcgen05 kernel (no one-launch step read then)."""
    return _lib.far_read_kernel_for(hd, n, hq, hkv) == 1


def default_splits(hkv):
    """Split count per KV head that fills the device with one CTA per SM."""
    return _lib.default_splits(hkv, 0, 0, 0)
