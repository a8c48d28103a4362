"""bench.py's line contract on the CPU: the library arm and the reference arm
share one (metric, config) per configuration and GPU count, and the reference
arm (the reference's own CPU path) prints a complete line."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
import bench  # noqa: E402


def _args(*extra):
    old = sys.argv
    sys.argv = ["bench.py", *extra]
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_line_identity_per_configuration():
    m, c = bench.line_identity(_args(), 1)
    assert m == "INT4 MoE FFN tokens/s (decode, T=64)" and c["tokens"] == 64 and c["parallelism"] == "single GPU"
    m, c = bench.line_identity(_args(), 8)
    assert m.endswith("T=64 per GPU)") and c["parallelism"] == "ep8" and c["experts_per_gpu"] == 16
    m, c = bench.line_identity(_args("--config", "qwen3_30b_a3b_stack48"), 1)
    assert m == "INT4 MoE 48-layer stack tokens/s (decode, T=16)" and c["layers"] == 48
    m, c = bench.line_identity(_args("--config", "glm45_air", "--tokens", "4096"), 1)
    assert m.endswith("T=4096)") and c["hidden"] == 4096 and c["l2"].startswith("rotating")


@pytest.mark.skipif(not os.path.exists(os.path.join(REPO, "oracle", "_ref", "libllmoc_ref.so")),
                    reason="the reference's CPU operators are not built here")
def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    m, c = bench.line_identity(_args(), 1)
    assert d["impl"] == "reference" and d["metric"] == m and d["config"] == c
    assert d["value"] > 0 and d["cpu_baseline"]["kind"] == "reference"
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
