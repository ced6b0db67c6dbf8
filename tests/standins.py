"""A stand-in vLLM drafter for the plugin-surface tests and their golden vectors.

fold/attention.py:270-375 (install, use_full_draft_storage) and fold/rope.py:14-28 (drafter_rope)
of the reference touch only a few attributes of vLLM's speculator object: the drafter model's class
name and layer names, the layers' attention impls (a FlashAttentionImpl with its sliding window and
FlashAttention version), their KV caches and KV-spec methods, the rotary modules, and the scheduler
and compilation configs. The classes below provide exactly those, so that the same scenario can be
installed by the reference (tests/golden/make_golden.py records its reports and errors) and by this
package (tests/test_plugin_surface.py compares them).

A scenario is a dict of plain values: `layers` lists each drafter layer as None (full attention) or
its native sliding window (left, right); the other keys set the model class name, the batch limit,
the FlashAttention version, a foreign layer name, and so on.
"""
from __future__ import annotations

from types import SimpleNamespace

HQ, HKV, HD, BLOCK, MAX_LEN, PAGE = 8, 2, 128, 8, 1000, 16


def _rotary_class(name):
    """A rotary module class with the given class name (the reference checks the name)."""

    def compute_inv_freq(self, base):
        import torch

        return 1.0 / (base ** (torch.arange(0, self.rotary_dim, 2, dtype=torch.float) / self.rotary_dim))

    return type(name, (), {"_compute_inv_freq": compute_inv_freq})


def make_rotary(name="RotaryEmbedding", *, base=1e6, rotary_dim=HD, head_size=HD, neox=True, device="cpu"):
    import torch

    r = _rotary_class(name)()
    r.base, r.rotary_dim, r.head_size, r.is_neox_style = base, rotary_dim, head_size, neox
    r.cos_sin_cache = torch.zeros((4, rotary_dim), device=device)
    return r


def _flash_impl(version, window):
    """A FlashAttentionImpl of vLLM without running its constructor (only the attributes that the
    install reads are set)."""
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    impl = FlashAttentionImpl.__new__(FlashAttentionImpl)
    impl.vllm_flash_attn_version = version
    impl.sliding_window = tuple(window) if window is not None else (-1, -1)
    impl.num_heads, impl.num_kv_heads, impl.head_size, impl.scale = HQ, HKV, HD, HD ** -0.5
    return impl


class _OtherImpl:
    """An attention impl that is not FlashAttention."""

    def __init__(self, window):
        self.vllm_flash_attn_version = 3
        self.sliding_window = tuple(window) if window is not None else (-1, -1)
        self.num_heads, self.num_kv_heads, self.head_size, self.scale = HQ, HKV, HD, HD ** -0.5


class AttentionLayer:
    """vLLM's Attention layer as the static forward context holds it."""

    def __init__(self, name, impl, kv_cache, sliding_window):
        self.layer_name = name
        self.impl = impl
        self.kv_cache = kv_cache
        self.sliding_window = sliding_window
        self.spec_calls = []

    def get_kv_cache_spec(self, vllm_config):
        self.spec_calls.append(vllm_config)
        return {"sliding_window": self.sliding_window}


class Inner:
    """The drafter's inner model: its decoder layers, and the context K/V path that the install
    wraps (fold/attention.py:233-267). _project_context_kv returns the next prepared (K, V)."""

    def __init__(self, layers, attn_layers, nkv=HKV, hd=HD, rope_device="cpu"):
        import torch

        self.layers = layers
        self._attn_layers = attn_layers
        self._num_attn_layers, self._num_kv_heads, self._head_dim = len(attn_layers), nkv, hd
        self._kv_size = nkv * hd
        self._rope_cos_sin_cache = torch.zeros((8, hd), dtype=torch.bfloat16, device=rope_device)
        self._rope_head_size, self._rope_is_neox = hd, True
        self.next_kv = None
        self.cache_updates = []

    def _project_context_kv(self, states, num_ctx, L, nkv, hd):
        return self.next_kv

    def _normalize_context_k(self, k):
        return k


def build_speculator(scn: dict, device="cpu"):
    """The stand-in speculator of a scenario (see the module docstring)."""
    import torch

    windows = scn.get("layers", [None, None])
    version = scn.get("fa_version", 3)
    names = [f"drafter.layers.{i}.self_attn.attn" for i in range(len(windows))]
    context, decoder, attn_layers = {}, [], []
    allocated = scn.get("allocated", True)
    for i, (name, win) in enumerate(zip(names, windows)):
        impl = _OtherImpl(win) if scn.get("not_flash") else _flash_impl(version, win)
        cache = (torch.zeros((4, HKV, PAGE, 2 * HD), device=device, dtype=torch.bfloat16) if allocated
                 else torch.empty(0, device=device, dtype=torch.bfloat16))
        layer = AttentionLayer(name, impl, cache, None if win is None else int(win[0]) + 1)
        context[name] = layer
        attn_layers.append(SimpleNamespace(impl=SimpleNamespace(do_kv_cache_update=None), kv_cache=None))
        rot = make_rotary(base=scn.get("theta", 1e6), rotary_dim=scn.get("rotary_dim", HD), device=device)
        attn = SimpleNamespace(layer_name=scn.get("foreign_name") if scn.get("foreign_name") and i == 1 else name)
        decoder.append(SimpleNamespace(self_attn=SimpleNamespace(attn=attn, rotary_emb=rot)))
    if scn.get("override_spec"):
        context[names[-1]].get_kv_cache_spec = lambda cfg: None  # a plain function, not a bound method
    inner = Inner(decoder, attn_layers, rope_device=device)
    model_cls = type(scn.get("model", "DFlashQwen3ForCausalLM"), (), {})
    model = model_cls()
    model.model = inner
    model.get_draft_kv_cache_layer_names = lambda: list(names)
    cfg = SimpleNamespace(scheduler_config=SimpleNamespace(max_num_seqs=scn.get("max_num_seqs", 1)),
                          compilation_config=SimpleNamespace(static_forward_context=context))
    return SimpleNamespace(model=model, vllm_config=cfg, num_query_per_req=BLOCK, max_model_len=MAX_LEN)


SLIDE = (127, 0)  # a causal native window of 128 entries

# name -> (scenario, install keyword arguments)
INSTALL_SCENARIOS = {
    "fold_full": (dict(layers=[None, None, None]), dict(window=256)),
    "fold_alpha3_splits8": (dict(layers=[None, None]), dict(window=300, alpha=3.0, local_splits=8)),
    "fold_fa4": (dict(layers=[None, None], fa_version=4), dict(window=256)),
    "sliding_window": (dict(layers=[None, SLIDE, None, SLIDE]), dict(window=256)),
    "sliding_fold": (dict(layers=[None, SLIDE, None, SLIDE]), dict(window=256, sliding_layers="fold")),
    "window_mode": (dict(layers=[None, SLIDE]), dict(window=256, mode="window", sliding_layers="fold")),
    "rerope": (dict(layers=[None, SLIDE]), dict(window=256, mode="rerope", logn_ref=4096)),
    "rerope_sliding_fold": (dict(layers=[None, SLIDE]), dict(window=256, mode="rerope", logn_ref=4096,
                                                             sliding_layers="fold")),
    "logn_ignored_in_fold": (dict(layers=[None]), dict(window=256, logn_ref=4096)),
    "qwen3_dspark": (dict(layers=[None], model="Qwen3DSparkForCausalLM"), dict(window=128)),
    "gemma4_dspark": (dict(layers=[None], model="Gemma4DSparkForCausalLM"), dict(window=128)),
    # errors
    "err_mode": (dict(layers=[None]), dict(window=256, mode="fast")),
    "err_sliding_layers": (dict(layers=[None]), dict(window=256, sliding_layers="all")),
    "err_rerope_logn": (dict(layers=[None]), dict(window=256, mode="rerope")),
    "err_drafter": (dict(layers=[None], model="LlamaForCausalLM"), dict(window=256)),
    "err_batch": (dict(layers=[None], max_num_seqs=2), dict(window=256)),
    "err_foreign_layer": (dict(layers=[None, None], foreign_name="target.layers.1.self_attn.attn"),
                          dict(window=256)),
    "err_fa2": (dict(layers=[None], fa_version=2), dict(window=256)),
    "err_not_flash": (dict(layers=[None], not_flash=True), dict(window=256)),
    "err_native_wider": (dict(layers=[None, (511, 0)]), dict(window=256)),
    "err_sliding_noncausal": (dict(layers=[None, (127, 3)]), dict(window=256, sliding_layers="fold")),
    "err_sliding_narrow": (dict(layers=[None, (5, 0)]), dict(window=256, sliding_layers="fold")),
    "err_window": (dict(layers=[None]), dict(window=0)),
}

# name -> scenario of use_full_draft_storage (the KV cache not yet allocated)
STORAGE_SCENARIOS = {
    "storage_mixed": dict(layers=[None, SLIDE, None, SLIDE], allocated=False),
    "storage_none_sliding": dict(layers=[None, None], allocated=False),
    "err_storage_allocated": dict(layers=[None, SLIDE], allocated=True),
    "err_storage_override": dict(layers=[None, SLIDE], allocated=False, override_spec=True),
}

# name -> keyword arguments of make_rotary
ROPE_SCENARIOS = {
    "rope_default": dict(),
    "rope_partial": dict(rotary_dim=64, base=5e5),
    "rope_gemma4": dict(name="Gemma4RotaryEmbedding", base=1e4),
    "err_rope_scaled": dict(name="Llama3RotaryEmbedding"),
    "err_rope_gptj": dict(neox=False),
    "err_rope_dims": dict(rotary_dim=256),
}

# name -> (window, block, max_model_len, mode, cache shape): FoldWorkspace constructor checks
WORKSPACE_SCENARIOS = {
    "ws_ok": (64, 8, 1000, "fold", (4, HKV, PAGE, 2 * HD)),
    "ws_window_mode": (64, 8, 1000, "window", (4, HKV, PAGE, 2 * HD)),
    "err_ws_window": (0, 8, 1000, "fold", (4, HKV, PAGE, 2 * HD)),
    "err_ws_block": (64, 0, 1000, "fold", (4, HKV, PAGE, 2 * HD)),
    "err_ws_ndim": (64, 8, 1000, "fold", (4, HKV, 2 * HD)),
    "err_ws_odd": (64, 8, 1000, "fold", (4, HKV, PAGE, 2 * HD + 1)),
    "err_ws_page": (64, 8, 1000, "fold", (4, HKV, 24, 2 * HD)),
    "err_ws_pages": (64, 8, 1000, "fold", (0, HKV, PAGE, 2 * HD)),
    "err_ws_mode": (64, 8, 1000, "sparse", (4, HKV, PAGE, 2 * HD)),
}


def report_of(speculator, report):
    """What an install left behind, as plain values: the report, the impl class of every layer,
    and each FOLD workspace's geometry."""
    ctx = speculator.vllm_config.compilation_config.static_forward_context
    layers = {}
    for name, layer in ctx.items():
        entry = {"impl": type(layer.impl).__name__}
        ws = getattr(layer.impl, "workspace", None)
        if ws is not None:
            entry.update(window=ws.window, block=ws.block, far_distance=ws.far_distance, mode=ws.mode,
                         alpha=ws.alpha, logn_ref=ws.logn_ref, local_splits=ws.local_splits,
                         side_shape=list(ws.side.shape), side_pages=ws.side_pages,
                         side_table=ws.side_table.cpu().tolist(), max_model_len=ws.max_model_len,
                         inv_freq=[float(x) for x in ws.inv_freq.cpu().tolist()])
        if hasattr(layer.impl, "logn_ref") and ws is None:
            entry["logn_ref"] = layer.impl.logn_ref
        layers[name] = entry
    return {"report": dict(report), "layers": layers}
