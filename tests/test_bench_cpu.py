"""bench.py's reference arm (the CPU dequantise-then-matvec path the oracle restates) keeps the JSON contract on a
machine without a GPU: one line with the metric, the impl tag, the CPU baseline and a zero-copy e2e block."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--layers", "2",
                        "--steps", "2", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "decode-step GEMV HBM GB/s" and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["steps"] == 2 and d["warmup"] == 1                 # whole steps, timed as asked
    assert d["config"]["bytes_per_step"] == 2 * 53567488 + 50406404


def test_cli_lists_the_workloads_and_scale_formats():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120, cwd=ROOT)
    assert r.returncode == 0
    for opt in ("--workload", "--scales", "--impl", "--gpus", "--steps", "--warmup"):
        assert opt in r.stdout


def test_tp_record_reports_the_speedup_over_one_gpu():
    """The default multi-GPU line's `tp` record: the tensor-parallel step beside the same run's one-GPU step."""
    sys.path.insert(0, ROOT)
    import bench
    full = 36 * 53567488 + 50406404
    rec = bench.tp_record(ms_tp=0.9, rank_bytes=full // 2, full_bytes=full, world=2, collective="nccl",
                          ms_one_gpu=0.345)
    assert rec["world"] == 2 and rec["collective"] == "nccl"
    assert abs(rec["speedup_vs_one_gpu"] - round(0.345 / 0.9, 3)) < 1e-9
    assert abs(rec["tok_s"] - round(1e3 / 0.9, 1)) < 1e-9
    assert abs(rec["model_gbs"] - round(full / 0.9e-3 / 1e9, 1)) < 1e-9
    assert 0 < rec["rank_roofline_frac"] < 1 and rec["limit"] and rec["workload"]
