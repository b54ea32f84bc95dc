"""The multi-GPU benchmark script for benchmark configurations 3 and 4 (``bench_parallel.py``) runs end to end on gloo ranks
with tiny models of the same layouts: sequence-parallel TP+EP, and pipeline x data parallel with the sharded
optimizer. This checks the wiring only; the timing it prints on CPU is not a measurement."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("config,ranks", [("tp-ep", 2), ("pp-zero", 4)])
def test_the_parallel_bench_runs_on_cpu_ranks(config, ranks):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(ROOT / "bench_parallel.py"),
           "--config", config, "--device", "cpu", "--tiny", "--steps", "2", "--warmup", "1"]
    env = {**os.environ, "OMP_NUM_THREADS": "1", "PYTHONPATH": str(ROOT)}
    result = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert result.returncode == 0, result.stderr[-3000:]
    lines = [json.loads(x) for x in result.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, result.stdout
    record = lines[0]
    assert record["value"] > 0 and record["steps"] == 2 and "not a measurement" in record["note"]
    assert record["final_loss"] == pytest.approx(record["final_loss"]) and record["final_loss"] > 0
    if config == "pp-zero":
        assert record["config"]["parallelism"].startswith("pp2 x dp2") and "sharded" in record["config"]["optimizer"]
        assert record["dp_replicas_identical"] is True  # experts are averaged over the replicas like the rest
