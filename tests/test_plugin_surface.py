"""The drop-in surface against the reference's own behaviour, on the CPU.

tests/golden/plugin_surface.json holds what the reference's install, use_full_draft_storage,
FoldWorkspace constructor and drafter_rope (fold/attention.py:44-73,270-375, fold/rope.py:14-28)
did on the stand-in drafters of tests/standins.py: each installation report, the wrapper class of
every layer with its workspace geometry, and every error with its message. This file runs this
package's versions on the same stand-ins and requires the same outcome. It also drives the vLLM
plugin hook (fold/vllm_plugin.py:19-46) against vLLM's GPUModelRunner with its model-loading and
graph-capture methods replaced by recorders.

The workspaces live on the CPU here: the install only allocates and binds, it launches no kernel.
"""
import json
import logging
from pathlib import Path

import pytest
import torch

from fold_b200 import attention, rope
from tests import standins as si

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "plugin_surface.json").read_text())


def outcome(fn):
    try:
        return {"value": fn()}
    except Exception as e:  # noqa: BLE001 - the error is the outcome under test
        return {"error": type(e).__name__, "message": str(e)}


def plain(x):
    """JSON round trip (tuples -> lists), as the golden file stores values."""
    return json.loads(json.dumps(x))


def check(name, got):
    want = GOLDEN[name]
    got = plain(got)
    if "error" in want:
        assert got == want, f"{name}: {got} != {want}"
        return
    assert "value" in got, f"{name}: raised {got}"
    assert got["value"] == want["value"], name


@pytest.mark.parametrize("name", sorted(si.INSTALL_SCENARIOS))
def test_install_matches_reference(name):
    scn, kwargs = si.INSTALL_SCENARIOS[name]

    def run():
        spec = si.build_speculator(scn)
        rep = attention.install(spec, **kwargs)
        again = attention.install(spec, **kwargs)
        got = si.report_of(spec, rep)
        got["idempotent"] = again is rep
        return got

    check(name, outcome(run))


def test_install_scenarios_cover_every_error_of_the_reference():
    errors = {v["message"].split(": ", 1)[-1] for v in GOLDEN.values() if v.get("error") == "FoldError"}
    for msg in ("invalid mode or sliding_layers", "rerope mode needs logn_ref", "batch size 1 only",
                "FlashAttention 3 or 4 is required", "native window is wider than W",
                "expected a causal native window wider than the block", "is not a drafter KV layer",
                "full draft storage must be requested before KV allocation", "unexpected KV spec override"):
        assert any(msg in e for e in errors), msg


@pytest.mark.parametrize("name", sorted(si.STORAGE_SCENARIOS))
def test_full_draft_storage_matches_reference(name):
    scn = si.STORAGE_SCENARIOS[name]

    def run():
        spec = si.build_speculator(scn)
        res = attention.use_full_draft_storage(spec)
        again = attention.use_full_draft_storage(spec)
        ctx = spec.vllm_config.compilation_config.static_forward_context
        return {"result": dict(res), "idempotent": again is res,
                "specs": {k: layer.get_kv_cache_spec("cfg") for k, layer in ctx.items()}}

    check(name, outcome(run))


@pytest.mark.parametrize("name", sorted(si.ROPE_SCENARIOS))
def test_drafter_rope_matches_reference(name):
    kwargs = si.ROPE_SCENARIOS[name]

    def run():
        r = rope.drafter_rope(si.make_rotary(**kwargs))
        return {"inv_freq": [float(x) for x in r.inv_freq.tolist()], "rotary_dim": r.rotary_dim,
                "head_dim": r.head_dim, "dtype": str(r.inv_freq.dtype)}

    check(name, outcome(run))


def test_rope_table_rows_are_the_rotation_of_drafter_frequencies():
    r = rope.drafter_rope(si.make_rotary(rotary_dim=64, base=5e5))
    t = rope.table_host(r.inv_freq, 70000)
    f = r.inv_freq.double().numpy()
    for p in (0, 1, 2048, 69999):
        assert abs(t[p, :32] - torch.cos(torch.tensor(p * f)).numpy()).max() < 1e-6
        assert abs(t[p, 32:] - torch.sin(torch.tensor(p * f)).numpy()).max() < 1e-6


@pytest.mark.parametrize("name", sorted(si.WORKSPACE_SCENARIOS))
def test_workspace_checks_match_reference(name):
    w, b, max_len, mode, shape = si.WORKSPACE_SCENARIOS[name]

    def run():
        ws = attention.FoldWorkspace(torch.zeros(shape, dtype=torch.bfloat16), w, b, max_len,
                                     inv_freq=torch.ones(shape[-1] // 4 if len(shape) == 4 else 1), far_distance=0,
                                     mode=mode)
        return {"side_shape": list(ws.side.shape), "side_pages": ws.side_pages, "far_distance": ws.far_distance,
                "local_splits": ws.local_splits, "window": ws.window, "block": ws.block}

    check(name, outcome(run))


def test_install_wraps_the_context_kv_path_and_keeps_forward_signature():
    spec = si.build_speculator(dict(layers=[None, si.SLIDE]))
    inner = spec.model.model
    before = getattr(inner, "precompute_and_store_context_kv", None)
    attention.install(spec, window=256, sliding_layers="fold")
    assert inner.precompute_and_store_context_kv is not before
    ctx = spec.vllm_config.compilation_config.static_forward_context
    for layer in ctx.values():
        impl = layer.impl
        # the reference's wrapper signature (fold/attention.py:133-134)
        import inspect
        params = list(inspect.signature(impl.forward).parameters)
        assert params == ["layer", "query", "key", "value", "kv_cache", "attn_metadata", "output", "output_scale",
                          "output_block_scale"]
        # unknown attributes reach the wrapped FlashAttention impl
        assert impl.vllm_flash_attn_version == 3 and impl.num_kv_heads == si.HKV


# ------------------------------------------------------------------ the vLLM plugin hook
class _Runner:
    """A GPU model runner as the plugin sees it: its speculator, and the two methods it wraps."""

    def __init__(self, speculator):
        self.speculator = speculator
        self.calls = []


@pytest.fixture
def runner_cls(monkeypatch):
    """vLLM's GPUModelRunner with load_model/capture_model replaced by recorders (restored after)."""
    from vllm.v1.worker.gpu.model_runner import GPUModelRunner

    def load_model(self, *args, **kwargs):
        self.calls.append(("load", args, kwargs))

    def capture_model(self, *args, **kwargs):
        self.calls.append(("capture", args, kwargs))
        return 7

    monkeypatch.setattr(GPUModelRunner, "load_model", load_model)
    monkeypatch.setattr(GPUModelRunner, "capture_model", capture_model)
    monkeypatch.setattr(GPUModelRunner, "_fold", False, raising=False)
    return GPUModelRunner


def test_register_without_config_changes_nothing(runner_cls, monkeypatch):
    from fold_b200 import vllm_plugin

    monkeypatch.delenv("FOLD_CONFIG", raising=False)
    load = runner_cls.load_model
    vllm_plugin.register()
    assert runner_cls.load_model is load and not runner_cls._fold


def test_register_installs_fold_at_load_and_capture(runner_cls, monkeypatch, caplog):
    from fold_b200 import vllm_plugin

    monkeypatch.setenv("FOLD_CONFIG", json.dumps({"window": 256, "alpha": 2.0, "sliding_layers": "fold"}))
    vllm_plugin.register()
    assert runner_cls._fold
    wrapped_load, wrapped_capture = runner_cls.load_model, runner_cls.capture_model
    vllm_plugin.register()  # idempotent: no second wrapping
    assert runner_cls.load_model is wrapped_load and runner_cls.capture_model is wrapped_capture

    spec = si.build_speculator(dict(layers=[None, si.SLIDE], allocated=False))
    runner = _Runner(spec)
    runner_cls.load_model(runner, "weights", dummy=True)
    assert runner.calls[0] == ("load", ("weights",), {"dummy": True})
    # full KV storage was requested for the sliding layer before allocation
    assert spec._fold_full_storage == {"layers": ["drafter.layers.1.self_attn.attn"]}
    # the KV cache gets allocated, then capture installs FOLD with FOLD_CONFIG's arguments
    for layer in spec.vllm_config.compilation_config.static_forward_context.values():
        layer.kv_cache = torch.zeros((4, si.HKV, si.PAGE, 2 * si.HD), dtype=torch.bfloat16)
    with caplog.at_level(logging.INFO, logger="vllm.fold"):
        assert runner_cls.capture_model(runner) == 7
    assert runner.calls[1] == ("capture", (), {})
    rep = spec._fold_installation
    assert rep["window"] == 256 and rep["sliding_layers"] == "fold"
    assert rep["fold_layers"] == ["drafter.layers.0.self_attn.attn", "drafter.layers.1.self_attn.attn"]
    assert any("FOLD installed" in r.getMessage() for r in caplog.records)


def test_register_skips_runners_without_a_drafter(runner_cls, monkeypatch):
    from types import SimpleNamespace

    from fold_b200 import vllm_plugin

    monkeypatch.setenv("FOLD_CONFIG", json.dumps({"window": 256}))
    vllm_plugin.register()
    runner = _Runner(SimpleNamespace(model=None))
    runner_cls.load_model(runner)
    assert runner_cls.capture_model(runner) == 7
    assert not hasattr(runner.speculator, "_fold_installation")
