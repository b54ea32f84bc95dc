"""The sharded-AdamW exchange benchmark (``bench_zero.py``) runs end to end on two gloo ranks: the NCCL-path code of
``ShardedAdamW`` reduce-scatters, steps and all-gathers, and every rank ends with the same parameters. This checks
the wiring only; the CPU timing is not a measurement (the fused NVLink path needs GPUs)."""

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


def test_the_zero_bench_runs_on_cpu_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(ROOT / "bench_zero.py"),
           "--device", "cpu", "--numel", "40000", "--tensors", "3", "--iters", "2", "--warmup", "1"]
    env = {**os.environ, "OMP_NUM_THREADS": "1", "PYTHONPATH": str(ROOT)}
    result = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert result.returncode == 0, result.stderr[-3000:]
    lines = [json.loads(x) for x in result.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, result.stdout
    record = lines[0]
    assert record["replicas_identical"] is True and "not a measurement" in record["note"]
    assert record["numel"] == 3 * 13336  # each tensor rounded up to a multiple of 8 elements
    assert record["nccl"]["total_ms"] > 0
