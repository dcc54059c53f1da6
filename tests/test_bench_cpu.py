"""bench.py's output contract on the CPU: the reference arm (the CPU port of the
path, what the driver runs as `bench.py --impl reference`) prints one JSON line
with the contract's keys, and the FlashInfer comparison refuses the token
counts it does not run."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=600):
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True,
                         timeout=timeout, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


def test_reference_arm_json_contract():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "0")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_flashinfer_arm_refuses_below_eight_tokens():
    d = _run("--impl", "flashinfer", "--tokens", "1", timeout=120)
    assert d["impl"] == "flashinfer" and "unavailable" in d
