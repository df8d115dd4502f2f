"""tests/verify.py: the reference's scoring contract on B200 (argument handling on
the CPU; one pilot run on the GPU)."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "tests"))
import verify  # noqa: E402


def test_selection_and_exclusive_arguments():
    assert verify.selected_ops(verify.parse_args([])) == verify.OPS
    assert verify.selected_ops(verify.parse_args(["--pilot"])) == ["matmul", "silu", "rmsnorm_matmul"]
    assert verify.selected_ops(verify.parse_args(["--op", "lora"])) == ["lora"]
    with pytest.raises(SystemExit):
        verify.parse_args(["--op", "silu", "--pilot"])
    with pytest.raises(SystemExit):
        verify.parse_args(["--candidate", "x.py"])            # a candidate needs --op
    with pytest.raises(SystemExit):
        verify.parse_args(["--op", "silu", "--candidate", "x.py", "--build-baselines"])
    with pytest.raises(SystemExit):
        verify.parse_args(["--num-cores", "3"])
    assert len(verify.OPS) == 14


def test_gates():
    assert verify.gate_for("silu", False) == 1e-5
    assert verify.gate_for("matmul", False) == 1e-2
    assert verify.gate_for("matmul", True) == 2e-5       # the reference's fp32 gate
    assert verify.gate_for("mamba", True) == 3e-5


def test_work_accounting():
    from oracle import inputs
    d = inputs.nkibench("matmul", 42, M=8, K=16, N=32)
    assert verify.work("matmul", d) == ("tensor", 2.0 * 8 * 16 * 32)
    d = inputs.nkibench("silu", 42, M=4, N=8)
    assert verify.work("silu", d) == ("hbm", 2 * 32 * 4)
    d = inputs.nkibench("bmm", 42, B=2, M=4, K=8, N=16)
    assert verify.work("bmm", d) == ("hbm", (2 * 4 * 8 + 2 * 8 * 16) * 2 + 2 * 4 * 16 * 2)


@pytest.mark.gpu
def test_pilot_run_on_gpu(tmp_path):
    bl = tmp_path / "baselines.json"
    cmd = [sys.executable, str(REPO / "tests" / "verify.py"), "--pilot", "--fast", "--baselines", str(bl)]
    r = subprocess.run(cmd + ["--build-baselines"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert set(json.loads(bl.read_text())) == {"matmul", "silu", "rmsnorm_matmul"}
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert [x["op"] for x in rows] == ["matmul", "silu", "rmsnorm_matmul"]
    assert all(x["passed"] and x["latency_ms"] > 0 and x["speedup"] for x in rows)
    assert "geomean speedup" in r.stdout
    # the reference's own fp32 gate: an fp32 operator, and the contractions with an fp32 path
    for op in ("silu", "matmul", "transpose_matmul", "bmm"):
        r = subprocess.run([sys.executable, str(REPO / "tests" / "verify.py"), "--op", op, "--fast",
                            "--strict-fp32", "--baselines", str(bl)], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
