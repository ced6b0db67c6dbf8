"""The benchmark's reference arm runs on the host cores alone: its JSON line carries the keys the
benchmark contract names, and ranks other than 0 exit without work. The GPU arm is exercised on
a B200 only (it refuses to run without one)."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=e, capture_output=True,
                       text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    return [json.loads(line) for line in p.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    lines = run_bench("--impl", "reference", "--config", "3", "--steps", "1", "--warmup", "0")
    assert len(lines) == 1
    d = lines[0]
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["higher_is_better"] is False and d["value"] > 0
    assert d["config"]["workload"] == "qwen3-8b-drafter-32k"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_no_work():
    assert run_bench("--impl", "reference", "--steps", "1", "--warmup", "0",
                     env={"RANK": "1", "WORLD_SIZE": "2"}) == []
