"""bench.py's output contract: one JSON line with the fields the benchmark driver reads.  The reference arm (the CPU
port, no GPU) runs here; our arm needs a B200 and runs on c1 with few steps."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "e2e", "cpu_baseline"}


def _run(args, timeout):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT, capture_output=True,
                         text=True, timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run(["--impl", "reference", "--workload", "c1", "--steps", "1", "--warmup", "0"], 600)
    assert BASE <= set(d) and d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "TFLOPS" and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["config"]["workload"] == "c1"
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb) and cb["kind"] in ("port", "reference")
    assert cb["value"] == d["value"] and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.gpu
def test_our_arm_line(engine):
    d = _run(["--workload", "c1", "--steps", "3", "--warmup", "3", "--e2e-steps", "2", "--no-cpu-baseline"], 900)
    assert BASE <= set(d) and "impl" not in d
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 3 and d["scaling"] == "strong"
    assert d["gpu_launches"] > 0
    r = d["roofline"]
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(r) and r["frac"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])
    e = d["e2e"]
    assert {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"} <= set(e)
    assert e["h2d_bytes_per_step"] == 2 * 1024 * 1024 * 8 and e["d2h_bytes_per_step"] == 1024 * 1024 * 8
    assert e["value"] > 0 and e["single_call"]["value"] > 0
