"""Straggler capacity and resharded checkpoints across real gloo ranks (reference tests:
tests/test_future_features.py): a slow rank's expert capacity shrinks while the fast rank's grows, capacity stays put
without the option, the trainer logs per-device imbalance, and a weights-only resharded checkpoint (no optimizer
state) loads on 2 ranks into a model whose logits match the single-process model's."""

import json
from pathlib import Path

import torch

from quantaweave_b200 import QuantaWeaveMoEForCausalLM

from test_parallel_cpu import run_ranks, tiny_config


def _capacity_case(rank, world, adapt):
    from quantaweave_b200.parallel.expert_parallel import DeviceLoadTracker, init_expert_parallel

    ep = init_expert_parallel("cpu", 1)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(tiny_config(capacity_factor=1.0, num_experts=4, top_k=1),
                                      expert_parallel=ep).eval()
    for moe in model.moes():
        moe.simulated_cost_per_row = 2e-3 if rank == 1 else 0.0
    tracker = DeviceLoadTracker(model, ep, strength=0.0, interval=1, adapt_capacity=adapt, capacity_scale_min=0.5,
                                capacity_scale_max=2.0)
    batch = torch.randint(0, 64, (4, 17), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        for step in range(1, 4):
            model(batch, labels=batch)
            metrics = tracker.update(step)
    return [moe.capacity_scale for moe in model.moes()], metrics["time_imbalance"]


def test_straggler_capacity_shrinks_the_slow_rank_and_grows_the_fast_one():
    results = run_ranks(_capacity_case, 2, (True,))
    fast, slow = results[0][0], results[1][0]
    assert all(s < 1.0 for s in slow) and all(f > 1.0 for f in fast), (fast, slow)
    assert all(0.5 <= s <= 2.0 for s in fast + slow) and results[0][1] > 1.0
    fixed = run_ranks(_capacity_case, 2, (False,))
    assert all(s == 1.0 for r in fixed.values() for s in r[0])


def _trainer_metrics_case(rank, world, tmp):
    from test_parallel_cpu import _trainer_case

    return _trainer_case(rank, world, tmp, 4, {"straggler_capacity": True, "device_metrics": True,
                                               "straggler_interval": 1, "simulate_slow_rank": "1:0.001",
                                               "log_interval": 1, "checkpoint_interval": 0})


def test_the_trainer_logs_per_device_imbalance_with_straggler_capacity(tmp_path):
    run_ranks(_trainer_metrics_case, 2, (str(tmp_path),))
    rows = [json.loads(x) for x in (tmp_path / "m0.jsonl").read_text().splitlines()]
    assert rows and all("time_imbalance" in r and "rows_imbalance" in r for r in rows)
    assert max(r["time_imbalance"] for r in rows) > 1.0


def _resharded_case(rank, world, tmp):
    from quantaweave_b200.parallel.checkpoint import load_sharded_checkpoint
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel
    from quantaweave_b200.utils.checkpoint_io import load_checkpoint

    tmp = Path(tmp)
    cfg = tiny_config(capacity_factor=0.0)
    ep = init_expert_parallel("cpu", 1)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).eval()
    optimizer = torch.optim.AdamW(model.parameters())
    step = load_sharded_checkpoint(tmp / "shards", model, optimizer, ep)  # optimizer None in the shard: tolerated
    full = QuantaWeaveMoEForCausalLM(cfg).eval()
    full.load_state_dict(load_checkpoint(tmp / "full" / "model.pt")["model"])
    ids = torch.randint(0, 64, (2, 17), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        got, want = model(ids)["logits"], full(ids)["logits"]
    assert torch.allclose(got, want, atol=1e-5), (got - want).abs().max()
    assert not optimizer.state  # nothing was restored into the optimizer
    return step


def test_a_weights_only_resharded_checkpoint_loads_across_ranks(tmp_path):
    from quantaweave_b200.parallel.checkpoint import reshard_checkpoint
    from quantaweave_b200.training.trainer import save_checkpoint

    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(tiny_config(capacity_factor=0.0))
    save_checkpoint(tmp_path / "full", model, torch.optim.AdamW(model.parameters()), 7, None, torch.device("cpu"))
    info = reshard_checkpoint(tmp_path / "full", tmp_path / "shards", ep_size=2)
    assert info["world_size"] == 2 and (tmp_path / "shards" / "config.json").exists()
    assert run_ranks(_resharded_case, 2, (str(tmp_path),)) == {0: 7, 1: 7}


def _sequence_parallel_capacity_case(rank, world):
    """Under sequence parallelism the tensor-parallel ranks are the expert ranks; a slow rank must still show up as
    slow (its timings are not averaged away over the tensor-parallel group). One controller step is checked: later
    steps route traffic off the slow rank, which then stops being slow."""
    from quantaweave_b200.parallel.expert_parallel import DeviceLoadTracker, init_expert_parallel

    ep = init_expert_parallel("cpu", world, sequence_parallel=True)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(tiny_config(capacity_factor=1.0, num_experts=4, top_k=1),
                                      expert_parallel=ep).eval()
    for moe in model.moes():
        moe.simulated_cost_per_row = 2e-3 if rank == 1 else 0.0
    tracker = DeviceLoadTracker(model, ep, strength=0.5, interval=1, adapt_capacity=True, capacity_scale_min=0.5,
                                capacity_scale_max=2.0)
    batch = torch.randint(0, 64, (4, 17), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        model(batch, labels=batch)
        metrics = tracker.update(1)
    return [moe.capacity_scale for moe in model.moes()], metrics["time_imbalance"], metrics["rank_bias"]


def test_straggler_control_acts_under_sequence_parallelism():
    results = run_ranks(_sequence_parallel_capacity_case, 2)
    fast, slow = results[0][0], results[1][0]
    assert all(s < 1.0 for s in slow) and all(f > 1.0 for f in fast), (fast, slow)
    assert results[0][1] > 1.0
    bias = results[0][2]
    assert bias[1] < bias[0]  # routing is biased away from the slow rank's experts
