"""bench.py's reference arm on CPU: one JSON line with the keys the driver
reads, the requested step and warm-up counts, and the CPU-baseline fields."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*extra):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *extra], cwd=ROOT,
                       capture_output=True, text=True, timeout=600, check=True)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    line = run_bench("--impl", "reference", "--steps", "2", "--warmup", "3")
    for key in ("metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline",
                "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 3
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["config"]["workload"] == "bq-decode-b64"
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_for_a_non_moe_workload_says_unavailable():
    line = run_bench("--impl", "reference", "--workload", "attn-decode-full-b64")
    assert line["impl"] == "reference" and "unavailable" in line
