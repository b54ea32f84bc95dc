"""The sequence-parallel projection exchange benchmark (``bench_tp.py``) runs end to end on two gloo ranks with the
NCCL-path composition (torch matmuls on CPU) and reports its roofline bookkeeping. This checks the wiring only; the
CPU timing is not a measurement (the fused NVLink path needs GPUs)."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_the_tp_bench_runs_on_cpu_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(ROOT / "bench_tp.py"),
           "--device", "cpu", "--tokens", "256", "--hidden", "128", "--qkv-width", "192", "--iters", "2",
           "--warmup", "1"]
    env = {**os.environ, "OMP_NUM_THREADS": "1", "PYTHONPATH": str(ROOT)}
    result = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert result.returncode == 0, result.stderr[-3000:]
    lines = [json.loads(x) for x in result.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, result.stdout
    record = lines[0]
    assert "not a measurement" in record["note"] and "fused" not in record
    work = record["work"]
    assert work["ag_gemm"]["flops"] == 2.0 * 256 * 128 * 96  # all rows x hidden x this rank's QKV width
    assert work["gemm_rs"]["nvlink_bytes_out"] == 1 * 128 * 128 * 2  # the other rank's rows, bf16
    for name in ("ag_gemm", "gemm_rs"):
        assert record["nccl"][name]["ms"] > 0 and work[name]["bound_ms"] > 0
