"""Host-side pieces of bench.py that the JSON line depends on (CPU only)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_roofline_inputs():
    sys.path.insert(0, ROOT)
    import bench
    pk = bench.peaks()
    assert pk["source"] in ("measured", "fallback") and pk["hbm_gbs"] > 1000 and pk["bf16_tflops"] > 500
    # roofline.traffic comes from the committed ncu summary of the headline kernel
    assert bench.profile_traffic("fp8_gemm_4096.md") == 36319488.0
    assert bench.profile_traffic("no_such_profile.md") is None
    assert bench.FLOPS == 2.0 * 4096 ** 3


def test_reference_arm_line_on_cpu():
    """--impl reference times the oracle port of the reference FP8 GEMM on the
    host and prints one JSON line with the fields the driver reads."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
