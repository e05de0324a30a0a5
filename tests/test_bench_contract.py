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


def test_roofline_accounting_constants():
    """The algorithmic bytes and FLOPs the bench divides by (per expert, per
    token, per stage) equal the figures the roofline is defined with: bq expert
    5,964,288 B (gate/up 3,970,560 + down 1,993,728, colsums excluded), bf16
    expert 11,894,784 B, 95,158,272 FLOP per token, 3.898e11 FLOP per 4096-token
    prefill step."""
    sys.path.insert(0, ROOT)
    import bench
    assert bench.BQ_EXPERT_GU_BYTES == 3_970_560 and bench.BQ_EXPERT_DN_BYTES == 1_993_728
    assert bench.BQ_EXPERT_BYTES == 5_964_288 and bench.BF16_EXPERT_BYTES == 11_894_784
    assert bench.FLOP_PER_TOKEN == 95_158_272
    R = 4096 * 8
    p1 = bench.stage_model("bq_phase1_gate_up.tc", "bq", 4096, 128, R)
    p2 = bench.stage_model("bq_phase2_down.tc", "bq", 4096, 128, R)
    assert p1[0] == p2[0] == "tensor"
    assert abs(p1[1] + p2[1] - 4096 * bench.FLOP_PER_TOKEN) < 1.0
    assert abs((p1[1] + p2[1]) - 3.898e11) < 1e8
    # decode phase 1 at b64: the routed experts' gate/up bytes dominate
    bound, b = bench.stage_model("bq_phase1_gate_up", "bq", 64, 126, 512)
    assert bound == "hbm" and 126 * 3_970_560 <= b < 126 * 3_970_560 * 1.01
