"""FOLD attention for vLLM drafters, on the B200 kernels of this package.

Drop-in for fold/attention.py of the reference: the same public names (FoldError, FoldWorkspace,
FoldAttention, SlidingFoldAttention, NativeWindowAttention, install, use_full_draft_storage), the
same forward signature and options (window, alpha, mode, sliding_layers, logn_ref,
local_splits), the same side-cache tensor and report. What changes is the work behind them:

  * the far-memory read and the far-query rotation are one CUDA kernel (kernels.far_read) that
    writes split partials, instead of far_query plus a FlashAttention call over the side cache;
  * the merge combines those partials with the window read in one kernel (kernels.merge);
  * the side-cache append is one 16-byte-vector kernel per layer (kernels.append), issued before
    the keys are rotated, so no copy of the un-rotated keys is needed;
  * the window (exact-position) read of the drafter's paged cache is the same split-read kernel in
    its paged mode (kernels.window_read), instead of a FlashAttention call; the merge combines its
    split partials with the far read's (kernels.merge_partials).

No FlashAttention call is left on the step. A layer may still be given a `local_read` callable
returning (o, lse) in FlashAttention's layout, which then replaces the window read.

Geometry of a draft step with block B at positions H .. H+B-1 (H = seq_len - qlen): context
entries with p - j < D = W + B are read at their true distances by the window read; older ones
are memory entries, read from the side cache with the query rotated to the shared distance D + r.
"""
from __future__ import annotations

import copy
from types import MethodType
from typing import Any, Callable, Optional

import torch

from . import kernels
from .errors import FoldError, describe_device_error
from .rope import drafter_rope, rope_table

SUPPORTED_DRAFTERS = ("DFlashQwen3ForCausalLM", "Qwen3DSparkForCausalLM", "Gemma4DSparkForCausalLM")
MODES = ("fold", "window", "rerope")

__all__ = ["FoldError", "FoldWorkspace", "FoldAttention", "SlidingFoldAttention", "NativeWindowAttention",
           "install", "use_full_draft_storage", "logn_scale_rows", "SUPPORTED_DRAFTERS", "MODES"]


class FoldWorkspace:
    """Per-layer state: the side cache of un-rotated keys and values, the device-side far
    length, the rope table and the split partials of the far read.

    Same constructor as the reference (fold/attention.py:50-73). The side cache keeps its layout
    side[pages, Hkv, 256, 2 * head_dim] with pages = ceil(max_model_len / 256) + 1, the last page
    holding the dummy slot. Extra keyword arguments: num_heads (query heads, to size the partials
    up front; else they are sized on first use), splits (far-read splits; default one CTA per SM),
    a shard of a sequence-partitioned cache (pos_lo = first position held, shard_len = positions
    held), and the storage format of the side cache: side_format "bf16" (the reference's, the
    cache dtype) or "fp8" (e4m3 K and V^T at half the bytes per key, head size 128; k_scale and
    v_scale are the per-KV-head dequantisation scales, a float or one per head: a stored value
    is round(x / scale))."""

    side_block = kernels.SIDE_BLOCK

    def __init__(self, cache, window, block, max_model_len, *, inv_freq, far_distance, alpha=2.0, mode="fold",
                 logn_ref=0, num_heads: Optional[int] = None, splits: Optional[int] = None, pos_lo: int = 0,
                 shard_len: Optional[int] = None, side_format: str = "bf16", k_scale=1.0, v_scale=1.0):
        if window < 1 or block < 1:
            raise FoldError("window and block size must be positive")
        if cache.ndim != 4 or cache.shape[-1] % 2:
            raise FoldError("expected a FlashAttention cache [pages, Hkv, block, 2 * head_dim]")
        if cache.shape[0] < 1 or cache.shape[2] % 16:
            raise FoldError("FlashAttention needs allocated pages and a page size divisible by 16")
        if mode not in MODES:
            raise FoldError(f"mode must be one of {MODES}")
        if pos_lo % self.side_block:
            raise FoldError("a shard must start on a side-cache page boundary")
        if side_format not in ("bf16", "fp8"):
            raise FoldError('side_format must be "bf16" or "fp8"')
        if side_format == "fp8" and cache.shape[-1] != 2 * kernels.FP8_HEAD_DIM:
            raise FoldError("the fp8 side cache needs head size 128")
        self.window, self.block, self.max_model_len = int(window), int(block), int(max_model_len)
        self.mode, self.alpha, self.logn_ref = mode, float(alpha), int(logn_ref)
        _, hkv, _, d2 = cache.shape
        self.num_kv_heads, self.head_dim = int(hkv), int(d2 // 2)
        self.device = cache.device
        self.pos_lo = int(pos_lo)
        self.sharded = shard_len is not None or self.pos_lo > 0
        held = self.max_model_len - self.pos_lo if shard_len is None else int(shard_len)
        # the window ablation keeps no memory; one page beyond the held range holds the dummy slot
        pages = 1 if mode == "window" else (max(held, 0) + self.side_block - 1) // self.side_block + 1
        self.side_pages = pages
        self.side_format = side_format
        if side_format == "fp8":
            self.side = torch.zeros(kernels.fp8_side_shape(pages, hkv), device=cache.device, dtype=torch.uint8)
            self.k_scale, self.v_scale = (torch.as_tensor(x, dtype=torch.float32).to(cache.device).expand(hkv)
                                          .contiguous() for x in (k_scale, v_scale))
        else:
            self.side = torch.zeros((pages, hkv, self.side_block, d2), device=cache.device, dtype=cache.dtype)
        self.side_table = torch.arange(pages, device=cache.device, dtype=torch.int32)[None]
        self.far_len = torch.zeros(1, device=cache.device, dtype=torch.int32)
        self.err = torch.zeros(1, device=cache.device, dtype=torch.int32)
        self.inv_freq = inv_freq.to(device=cache.device, dtype=torch.float32)
        self.far_distance = int(far_distance) or self.window + self.block
        self.local_splits = 16
        self.far_splits = int(splits) if splits else None
        self._table = None
        self._parts = {}
        self._window_parts = {}
        self._step_far, self._step_window = {}, {}
        self.plan = torch.zeros(1, device=cache.device, dtype=torch.int32)  # the step read's split
        if num_heads is not None:  # the buffers the forward of this layer uses, before any graph capture
            hq = int(num_heads)
            if mode != "window" and self.one_launch(self.block, hq):
                self.step_partials(self.block, hq)
            else:
                self.window_partials(self.block, hq)
                if mode != "window":
                    self.partials(self.block, hq)

    # -- derived state ---------------------------------------------------------------------------
    @property
    def capacity(self) -> int:
        """Number of positions the (unsharded) cache addresses."""
        return self.max_model_len

    @property
    def table(self) -> torch.Tensor:
        """Rope table covering every offset |D - H| of this workspace (shared between layers)."""
        if self._table is None:
            rows = max(self.max_model_len, self.far_distance) + self.block + 1
            self._table = rope_table(self.inv_freq, rows, self.device)
        return self._table

    def splits(self) -> int:
        if self.far_splits is None:
            self.far_splits = kernels.default_splits(self.num_kv_heads)
        return self.far_splits

    def partials(self, n: int, num_heads: int):
        """Split partial buffers (o [S, n, Hq, D], lse [S, Hq, n], float32) for n rows."""
        key = (int(n), int(num_heads))
        buf = self._parts.get(key)
        if buf is None:
            s = self.splits()
            buf = (torch.empty((s, n, num_heads, self.head_dim), device=self.device, dtype=torch.float32),
                   torch.empty((s, num_heads, n), device=self.device, dtype=torch.float32))
            self._parts[key] = buf
        return buf

    def window_partials(self, n: int, num_heads: int):
        """Split partial buffers of the window read (local_splits splits) for n rows."""
        return _partial_buffers(self._window_parts, self.local_splits, n, num_heads, self.head_dim, self.device)

    def one_launch(self, n: int, num_heads: int) -> bool:
        """Whether the far and window reads of a step of n rows run as one launch (read_step): for
        an unsharded cache whose far read takes the mma.sync kernel."""
        return (not self.sharded and self.side_format == "bf16"
                and not kernels.far_read_uses_tcgen05(self.head_dim, n, num_heads, self.num_kv_heads))

    def step_partials(self, n: int, num_heads: int):
        """(far, window) split buffers of the one-launch step read: splits() slots each (the
        blocks of a KV head share the two reads, one block per SM in all)."""
        s = max(self.splits(), 2)
        far = _partial_buffers(self._step_far, s, n, num_heads, self.head_dim, self.device)
        win = _partial_buffers(self._step_window, s, n, num_heads, self.head_dim, self.device)
        return far, win

    def check(self) -> None:
        """Raises FoldError if a kernel recorded a device-side error (synchronises)."""
        word = int(self.err.item())
        if word:
            self.err.zero_()
            raise FoldError(f"FOLD device error: {describe_device_error(word)}")

    # -- the two kernels of a step ----------------------------------------------------------------
    def append(self, k, v, positions, slots):
        """Side-cache append of committed entries (keys before RoPE)."""
        if self.side_format == "fp8":
            kernels.append_fp8(k, v, positions, slots, self.side, self.k_scale, self.v_scale, pos_lo=self.pos_lo,
                               skip_foreign=self.sharded, err=self.err)
            return
        kernels.append(k, v, positions, slots, self.side, pos_lo=self.pos_lo, skip_foreign=self.sharded,
                       err=self.err)

    def read_far(self, q, qsl, seq_lens, scale, *, rotate=True):
        """Rotated far read of q [n, Hq, D]; returns the partials (o [S, n, Hq, D], lse [S, Hq, n])."""
        n, hq, _ = q.shape
        o_part, lse_part = self.partials(n, hq)
        if self.side_format == "fp8":
            kernels.far_read_fp8(q, qsl, seq_lens, self.side, self.k_scale, self.v_scale, o_part, lse_part,
                                 window=self.window, block=self.block, far_distance=self.far_distance,
                                 softmax_scale=scale * self.alpha, table=self.table if rotate else None,
                                 far_len=self.far_len, pos_lo=self.pos_lo, capacity=self.capacity, err=self.err)
            return o_part, lse_part
        kernels.far_read(q, qsl, seq_lens, self.side, o_part, lse_part, window=self.window, block=self.block,
                         far_distance=self.far_distance, softmax_scale=scale * self.alpha,
                         table=self.table if rotate else None, far_len=self.far_len, pos_lo=self.pos_lo,
                         capacity=self.capacity, err=self.err)
        return o_part, lse_part

    def read_step(self, q, q_window, qsl, seq_lens, scale, kv_cache, block_table, *, window_size, causal,
                  rotate=True):
        """The far read of q (rotated, as read_far) and the window read of q_window over the
        drafter's paged cache kv_cache [blocks, Hkv, block_size, 2D] in one launch. Returns the
        (far, window) split partials, for kernels.merge_partials with plan=self.plan."""
        n, hq, _ = q.shape
        far, win = self.step_partials(n, hq)
        k, v = kernels.paged_planes(kv_cache, self.head_dim)
        kernels.step_read(q, q_window, qsl, seq_lens, self.side, far, k, v, block_table, win, self.plan,
                          window=self.window,
                          block=self.block, far_distance=self.far_distance, softmax_scale=scale, alpha=self.alpha,
                          window_size=window_size, causal=causal, table=self.table if rotate else None,
                          far_len=self.far_len, pos_lo=self.pos_lo, capacity=self.capacity, err=self.err)
        return far, win


def _partial_buffers(cache: dict, splits: int, n: int, num_heads: int, head_dim: int, device):
    """(o [splits, n, Hq, D], lse [splits, Hq, n]) float32, allocated once per shape."""
    key = (int(splits), int(n), int(num_heads))
    buf = cache.get(key)
    if buf is None:
        buf = (torch.empty((splits, n, num_heads, head_dim), device=device, dtype=torch.float32),
               torch.empty((splits, num_heads, n), device=device, dtype=torch.float32))
        cache[key] = buf
    return buf


def logn_scale_rows(q, query_start_loc, seq_lens, logn_ref):
    """The ReRoPE query scale max(1, log(p + 1) / log(ref)) at the absolute position p = H + r of
    each row r (fold/attention.py:76-83), as one kernel (kernels.logn_scale) that reads H from the
    device-side lengths."""
    return kernels.logn_scale(q, query_start_loc, seq_lens, logn_ref)


LocalRead = Callable[..., Any]


class _Wrapped:
    def __init__(self, original: Any, local_read: Optional[LocalRead] = None):
        self.original = original
        self.local_read = local_read

    def __getattr__(self, name):
        return getattr(self.original, name)

    def _native(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale):
        return self.original.forward(layer, query, key, value, kv_cache, attn_metadata, output=output,
                                     output_scale=output_scale, output_block_scale=output_block_scale)

    @staticmethod
    def _check_meta(meta):
        if meta.use_cascade or not isinstance(meta.causal, bool):
            raise FoldError("cascade attention and dynamic causality are not supported")

    def _fold_read(self, w, q_far, q_win, kv_cache, meta, out, *, window_size, causal, num_splits, rotate):
        """Far read + window read + merge of a FOLD layer into out [n, Hq, D]: one launch for both
        reads when the window read is this package's and the workspace allows it (one_launch)."""
        o, qsl, seq = self.original, meta.query_start_loc, meta.seq_lens
        local = dict(window_size=window_size, causal=causal, num_splits=num_splits, window=w.window,
                     block=w.block, alpha=w.alpha, err=w.err)
        n, hq = out.shape[0], out.shape[1]
        if self.local_read is None and w.one_launch(n, hq):
            far, win = w.read_step(q_far, q_win, qsl, seq, o.scale, kv_cache, meta.block_table,
                                   window_size=window_size, causal=causal, rotate=rotate)
            kernels.merge_partials(win[0], win[1], far[0], far[1], out, qsl, seq, window=w.window, block=w.block,
                                   alpha=w.alpha, plan=w.plan)
            return
        far = w.read_far(q_far, qsl, seq, o.scale, rotate=rotate)
        parts = None if self.local_read is not None else w.window_partials(n, hq)
        self._window_and_merge(q_win, kv_cache, meta, parts, far, out, **local)

    def _window_and_merge(self, q, kv_cache, meta, parts, far, out, *, window_size, causal, num_splits, window,
                          block, alpha, err):
        """The window read of q over the layer's paged cache, merged with the far partials `far`
        ((o, lse) or None) into out [n, Hq, D]. `parts` are the window read's split buffers."""
        o = self.original
        qsl, seq = meta.query_start_loc, meta.seq_lens
        if self.local_read is not None:
            out_l, lse_l = self.local_read(q, kv_cache, meta, o, window_size=window_size, causal=causal,
                                           num_splits=num_splits)
            if far is None:
                out.copy_(out_l.reshape(out.shape))
            else:
                kernels.merge(out_l.view(out.shape), lse_l, far[0], far[1], out, qsl, seq, window=window,
                              block=block, alpha=alpha)
            return
        k, v = kernels.paged_planes(kv_cache, o.head_size)
        kernels.window_read(q, qsl, seq, k, v, meta.block_table, parts[0], parts[1], window_size=window_size,
                            causal=causal, softmax_scale=o.scale, err=err)
        kernels.merge_partials(parts[0], parts[1], None if far is None else far[0], None if far is None else far[1],
                               out, qsl, seq, window=window, block=block, alpha=alpha)


class NativeWindowAttention(_Wrapped):
    """Native sliding-window read, optionally with the ReRoPE query scale (fold/attention.py:98-123):
    the window read kernel over the layer's own window, its splits combined into the output."""

    splits = 16  # num_splits of the reference's read (fold/attention.py:121)

    def __init__(self, original: Any, logn_ref: int = 0, local_read: Optional[LocalRead] = None,
                 block: Optional[int] = None, device=None):
        super().__init__(original, local_read)
        self.logn_ref = int(logn_ref)
        self._parts = {}
        self.err = None
        if block is not None and device is not None and local_read is None:
            self._buffers(int(block), int(original.num_heads), device)  # before any graph capture

    def _buffers(self, n, hq, device):
        if self.err is None:
            self.err = torch.zeros(1, device=device, dtype=torch.int32)
        return _partial_buffers(self._parts, self.splits, n, hq, self.original.head_size, device)

    def check(self) -> None:
        """Raises FoldError if the window read recorded a device-side error (synchronises)."""
        word = int(self.err.item()) if self.err is not None else 0
        if word:
            self.err.zero_()
            raise FoldError(f"FOLD device error: {describe_device_error(word)}")

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if attn_metadata is None:
            return self._native(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                output_block_scale)
        o, meta = self.original, attn_metadata
        n = meta.num_actual_tokens
        if n == 0:
            return output.zero_()
        q = query[:n]
        if self.logn_ref:
            q = logn_scale_rows(q, meta.query_start_loc, meta.seq_lens, self.logn_ref)
        hq = q.shape[1]
        parts = None if self.local_read is not None else self._buffers(n, hq, q.device)
        self._window_and_merge(q, kv_cache, meta, parts, None, output[:n].view(n, hq, o.head_size),
                               window_size=o.sliding_window, causal=meta.causal, num_splits=self.splits, window=1,
                               block=1, alpha=1.0, err=self.err)
        return output


class FoldAttention(_Wrapped):
    """Full-attention drafter layer: window read, rotated far read, merge."""

    def __init__(self, original: Any, workspace: FoldWorkspace, local_read: Optional[LocalRead] = None):
        super().__init__(original, local_read)
        self.workspace = workspace

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if attn_metadata is None:
            return self._native(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                output_block_scale)
        self._check_meta(attn_metadata)
        w, o, meta = self.workspace, self.original, attn_metadata
        n = meta.num_actual_tokens
        if n == 0:
            return output.zero_()
        B = w.block
        qsl, seq = meta.query_start_loc, meta.seq_lens
        q = query[:n]
        hq = q.shape[1]
        out = output[:n].view(n, hq, o.head_size)
        # the window read: non-causal, window [W + B - 1, B - 1] (fold/attention.py:148-151)
        window_size = (w.window + B - 1, B - 1)
        if w.mode == "window":
            parts = None if self.local_read is not None else w.window_partials(n, hq)
            self._window_and_merge(q, kv_cache, meta, parts, None, out, window_size=window_size, causal=False,
                                   num_splits=w.local_splits, window=w.window, block=B, alpha=w.alpha, err=w.err)
            return output
        if q.stride(-1) != 1:
            q = q.contiguous()
        q_far, rotate = q, True
        if w.mode == "rerope":
            q, q_far = kernels.rerope_queries(q, qsl, seq, w.inv_freq, w.far_len, far_distance=w.far_distance,
                                              window=w.window, block=B, constant=True, logn_ref=w.logn_ref,
                                              table=w.table)
            rotate = False
        self._fold_read(w, q_far, q, kv_cache, meta, out, window_size=window_size, causal=False,
                        num_splits=w.local_splits, rotate=rotate)
        return output


class SlidingFoldAttention(_Wrapped):
    """Sliding-window drafter layer: the native window read is the local branch, every older
    entry is read from the far memory. With native window (w, 0) the workspace window is
    w + 1 - B, so the far rule "distance >= window + B" splits exactly at the native window."""

    def __init__(self, original: Any, workspace: FoldWorkspace, local_read: Optional[LocalRead] = None):
        super().__init__(original, local_read)
        if workspace.mode == "window":
            raise FoldError("the Window ablation keeps the native sliding-window read")
        self.workspace = workspace

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if attn_metadata is None:
            return self._native(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                output_block_scale)
        self._check_meta(attn_metadata)
        w, o, meta = self.workspace, self.original, attn_metadata
        n = meta.num_actual_tokens
        if n == 0:
            return output.zero_()
        qsl, seq = meta.query_start_loc, meta.seq_lens
        B = w.block
        qn = logn_scale_rows(query[:n], qsl, seq, w.logn_ref) if w.logn_ref else query[:n]
        qp = qn if qn.stride(-1) == 1 else qn.contiguous()
        q_far, rotate = qp, True
        if w.mode == "rerope":
            _, q_far = kernels.rerope_queries(qp, qsl, seq, w.inv_freq, w.far_len, far_distance=w.far_distance,
                                              window=w.window, block=B, constant=True, logn_ref=0, table=w.table)
            rotate = False
        hq = qn.shape[1]
        # the native causal sliding read is the local branch (fold/attention.py:211-215)
        self._fold_read(w, q_far, qn, kv_cache, meta, output[:n].view(n, hq, o.head_size),
                        window_size=o.sliding_window, causal=meta.causal, num_splits=w.local_splits, rotate=rotate)
        return output


def _wrap_context_kv(inner, workspaces):
    """Replace the drafter's precompute_and_store_context_kv so that the keys (after the key
    norm, before RoPE) and values of every committed context entry are also appended to the side
    cache of each FOLD layer (fold/attention.py:227-267).

    The append runs before the in-place rotary op, so it reads the un-rotated keys directly and
    the reference's copy of them is not needed."""
    from vllm import _custom_ops as ops

    def wrapped(context_states, context_positions, context_slot_mapping=None):
        if not hasattr(inner, "_num_attn_layers"):
            inner._build_fused_kv_buffers()
        num_ctx = context_states.shape[0]
        L, kv, hd, nkv = inner._num_attn_layers, inner._kv_size, inner._head_dim, inner._num_kv_heads
        all_k, all_v = inner._project_context_kv(context_states, num_ctx, L, nkv, hd)
        all_k_normed = inner._normalize_context_k(all_k)
        per_layer = isinstance(context_slot_mapping, (list, tuple))

        def slots_of(i):
            return context_slot_mapping[i] if per_layer else context_slot_mapping

        if context_slot_mapping is not None:
            for i, ws in workspaces.items():
                slots = slots_of(i)
                if slots is None or ws.mode == "window":
                    continue
                ws.append(all_k_normed[i][:num_ctx], all_v[i][:num_ctx], context_positions[:num_ctx],
                          slots[:num_ctx])
        all_k_flat = all_k_normed.view(L * num_ctx, kv)
        cos_sin = inner._rope_cos_sin_cache
        if cos_sin.dtype != all_k_flat.dtype:
            cos_sin = cos_sin.to(dtype=all_k_flat.dtype)
        ops.rotary_embedding(context_positions.repeat(L), all_k_flat, None, inner._rope_head_size, cos_sin,
                             inner._rope_is_neox)
        if context_slot_mapping is None:
            return
        all_k_final = all_k_flat.view(L, num_ctx, nkv, hd)
        for i in range(L):
            slots = slots_of(i)
            if slots is None:
                continue
            attn = inner._attn_layers[i]
            attn.impl.do_kv_cache_update(attn, all_k_final[i], all_v[i], attn.kv_cache, slots)

    inner.precompute_and_store_context_kv = wrapped


def use_full_draft_storage(speculator: Any) -> dict:
    """Give the drafter's sliding-window layers full KV storage so that vLLM keeps their old pages
    (their reads keep the native window). Call after the drafter is loaded and before the KV cache
    is allocated (fold/attention.py:270-299). Idempotent."""
    done = getattr(speculator, "_fold_full_storage", None)
    if done is not None:
        return done
    context = speculator.vllm_config.compilation_config.static_forward_context
    changed = []
    for name in speculator.model.get_draft_kv_cache_layer_names():
        layer = context[name]
        if getattr(layer, "sliding_window", None) is None:
            continue
        cache = getattr(layer, "kv_cache", None)
        if isinstance(cache, torch.Tensor) and cache.numel():
            raise FoldError("full draft storage must be requested before KV allocation")
        bound = layer.get_kv_cache_spec
        if not hasattr(bound, "__func__"):
            raise FoldError("unexpected KV spec override")

        def spec_without_window(this, vllm_config, _spec=bound.__func__):
            view = copy.copy(this)
            view.sliding_window = None
            return _spec(view, vllm_config)

        layer.get_kv_cache_spec = MethodType(spec_without_window, layer)
        changed.append(name)
    speculator._fold_full_storage = {"layers": changed}
    return speculator._fold_full_storage


def _is_flash_attention(impl) -> bool:
    try:
        from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl
    except Exception:  # vLLM without that backend: only the class name can be checked
        return type(impl).__name__ == "FlashAttentionImpl"
    return type(impl) is FlashAttentionImpl


def install(speculator: Any, *, window: int, alpha: float = 2.0, mode: str = "fold", sliding_layers: str = "window",
            logn_ref: int = 0, local_splits: int = 16, local_read: Optional[LocalRead] = None) -> dict:
    """Wrap the attention of every drafter layer (fold/attention.py:302-375). Call after KV
    allocation and before CUDA graph capture. Returns the installation report.

    window          W, the number of recent context entries kept at exact positions
    alpha           concentration factor of the memory
    mode            "fold", "window" (FOLD without memory) or "rerope" (baseline)
    sliding_layers  "window" keeps the native read of sliding-window layers, "fold" lets them
                    read the memory as well
    logn_ref        reference length of the ReRoPE query scale (rerope mode)
    local_splits    split count of the window read
    local_read      optional replacement of the window read: a callable returning (o, lse) in
                    FlashAttention's layout
    """
    previous = getattr(speculator, "_fold_installation", None)
    if previous is not None:
        return previous
    if mode not in MODES or sliding_layers not in ("window", "fold"):
        raise FoldError("invalid mode or sliding_layers")
    if mode == "rerope" and not logn_ref:
        raise FoldError("rerope mode needs logn_ref")
    if mode != "rerope":
        logn_ref = 0
    if type(speculator.model).__name__ not in SUPPORTED_DRAFTERS:
        raise FoldError(f"supported drafters: {SUPPORTED_DRAFTERS}")
    cfg = speculator.vllm_config
    if cfg.scheduler_config.max_num_seqs != 1:
        raise FoldError("batch size 1 only")
    inner = speculator.model.model
    names = set(speculator.model.get_draft_kv_cache_layer_names())
    context = cfg.compilation_config.static_forward_context
    B = int(speculator.num_query_per_req)
    D = window + B
    report = dict(mode=mode, window=window, block=B, far_distance=D, alpha=alpha, logn_ref=logn_ref,
                  sliding_layers=sliding_layers, fold_layers=[], native_window_layers=[], side_cache_bytes=0)
    workspaces = {}

    def make_workspace(layer, dl, w):
        rope = drafter_rope(dl.self_attn.rotary_emb)
        return FoldWorkspace(layer.kv_cache, w, B, speculator.max_model_len, inv_freq=rope.inv_freq, far_distance=D,
                             alpha=alpha, mode=mode, logn_ref=logn_ref, num_heads=int(layer.impl.num_heads))

    for li, dl in enumerate(inner.layers):
        name = dl.self_attn.attn.layer_name
        if name not in names:
            raise FoldError(f"{name} is not a drafter KV layer")
        layer = context[name]
        impl = layer.impl
        if local_read is None and (not _is_flash_attention(impl) or impl.vllm_flash_attn_version not in (3, 4)):
            # the window read takes FlashAttention's paged cache layout and metadata
            raise FoldError(f"{name}: FlashAttention 3 or 4 is required")
        native = int(impl.sliding_window[0])
        if native >= 0:
            if native > window:
                raise FoldError(f"{name}: native window is wider than W")
            if sliding_layers == "fold" and mode != "window":
                if impl.sliding_window[1] != 0 or native + 1 - B < 1:
                    raise FoldError(f"{name}: expected a causal native window wider than the block")
                ws = make_workspace(layer, dl, native + 1 - B)
                layer.impl = SlidingFoldAttention(impl, ws, local_read)
                workspaces[li] = ws
                report["fold_layers"].append(name)
                report["side_cache_bytes"] += ws.side.numel() * ws.side.element_size()
            else:
                layer.impl = NativeWindowAttention(impl, logn_ref, local_read, block=B,
                                                   device=layer.kv_cache.device)
                report["native_window_layers"].append(name)
            continue
        ws = make_workspace(layer, dl, window)
        ws.local_splits = int(local_splits)
        layer.impl = FoldAttention(impl, ws, local_read)
        workspaces[li] = ws
        report["fold_layers"].append(name)
        report["side_cache_bytes"] += ws.side.numel() * ws.side.element_size()
    _wrap_context_kv(inner, workspaces)
    speculator._fold_workspaces = workspaces
    speculator._fold_installation = report
    return report
