"""Failure detection without any GPU fault (gloo ranks on CPU): a rank that dies between steps, and a sharded
checkpoint with a missing or corrupt shard. Survivors must fail with an error, never hang."""

import os
import socket
import time
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dying_worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="10")
    from quantaweave_b200.parallel.groups import ensure_process_group

    ensure_process_group("cpu")
    t = torch.ones(8)
    dist.all_reduce(t)  # step 1 completes everywhere
    if rank == 1:
        os._exit(0)  # this rank disappears between steps, with no collective in flight
    started = time.time()
    try:
        dist.all_reduce(t)  # step 2: the peer is gone
        queue.put((rank, "no error", time.time() - started))
    except Exception as exc:  # noqa: BLE001
        queue.put((rank, type(exc).__name__, time.time() - started))
    queue.close()
    queue.join_thread()  # flush the result before the hard exit (the peer is gone, so no orderly shutdown)
    os._exit(0)


def test_survivor_fails_fast_when_a_rank_dies_between_steps():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome, seconds = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=30)
    assert rank == 0 and outcome != "no error", outcome
    assert seconds < 60, seconds  # bounded by the process-group timeout (10 s here), not a hang


def _resume_worker(rank, world, port, tmp, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="60")
    from pathlib import Path

    from quantaweave_b200.training.trainer import default_args, run_training

    tmp = Path(tmp)
    try:
        common = dict(synthetic_data="uniform", vocab_size=64, sequence_length=16, batch_size=2, hidden_size=32,
                      layers=2, ffn_size=64, attention_heads=4, total_experts=4, active_experts=2, device="cpu",
                      no_power_tracking=True, expert_parallel=True, checkpoint_interval=2, output=tmp / "out",
                      checkpoint_dir=tmp / "ckpt", metrics_file=tmp / f"m{rank}.jsonl")
        run_training(default_args(steps=int(os.environ["QW_TEST_STEPS"]), **common))
        queue.put((rank, "ok", ""))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _launch(tmp, steps):
    os.environ["QW_TEST_STEPS"] = str(steps)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_resume_worker, args=(r, 2, port, str(tmp), queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (status, payload)) for r, status, payload in (queue.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    return results


@pytest.mark.parametrize("damage", ["missing", "corrupt"])
def test_resume_with_a_bad_shard_fails_on_every_rank(tmp_path, damage):
    first = _launch(tmp_path, 2)
    assert all(status == "ok" for status, _ in first.values()), first
    shard = next((tmp_path / "ckpt").rglob("model.rank1.pt"))
    if damage == "missing":
        shard.unlink()
    else:
        shard.write_bytes(shard.read_bytes()[:100])
    second = _launch(tmp_path, 4)
    for rank, (status, payload) in second.items():
        assert status == "error" and "cannot resume from the sharded checkpoint" in payload, (rank, payload[-800:])
