"""The bench's reference arm (`bench.py --impl reference`) on the host: the driver times it beside
the GPU arm every time, so its JSON line must keep the contract (one line, the same metric and
unit as the GPU arm, a `cpu_baseline` that says what was timed, and an `e2e` with no copies).
The arm runs the C restatement of the reference CPU path (oracle/); no GPU is involved."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_reference(*extra):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--warmup", "3", *extra], cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("config", ["llama8b", "smollm", "qwen3moe"])
def test_reference_arm_line(config):
    d = run_reference("--config", config, "--steps", "1")
    import bench

    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_reference_arm_gemv_config_is_marked_unavailable():
    d = run_reference("--config", "gemv-q4_k", "--steps", "1")
    assert d["impl"] == "reference" and d["unavailable"]
