"""bench.py's output contract, checked on the CPU through the reference arm.

The reference arm (`--impl reference`) times the oracle; its line must be the
only thing on stdout, one JSON object with the keys the driver reads.
"""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "tiny",
                          "--steps", "2", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1


def test_prefill_roofline_arithmetic():
    sys.path.insert(0, ROOT)
    import bench
    r = bench.prefill_roofline(gemm_flops=1.0e12, attn_flops=0.5e12, ms=10.0, peak=1500.0, peak_source="test")
    assert abs(r["achieved"] - 150.0) < 1e-9          # 1.5 TFLOP in 10 ms
    assert abs(r["issued"] - (2.0 + 1.5) * 100.0) < 1e-9  # 2 MMAs per GEMM product, 3 per attention product
    assert abs(r["frac"] - 0.1) < 1e-12 and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
