"""Multi-process parallelism on CPU (gloo, world 2): expert, tensor and pipeline parallelism, the sharded
optimizer and sharded checkpoints, each compared against single-device training of the same weights."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, queue, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        result = fn(rank, world, *args)
        queue.put((rank, "ok", result))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world=2, args=()):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, queue, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=300)
        if status != "ok":
            for p in procs:
                p.kill()
            raise AssertionError(f"rank {rank} failed:\n{payload}")
        results[rank] = payload
    for p in procs:
        p.join(timeout=60)
    return results


def tiny_config(**kw):
    base = dict(vocab_size=64, hidden_size=32, layers=2, ffn_size=64, num_experts=4, top_k=2, attention_heads=4,
                max_sequence_length=17, capacity_factor=1.25, norm_type="rmsnorm", position_embedding="rope",
                attention_bias=False)
    base.update(kw)
    return QuantaWeaveConfig(**base)


def _batches(world, per_rank=2, seq=17, vocab=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    full = torch.randint(0, vocab, (world * per_rank, seq), generator=g)
    return [full[r * per_rank:(r + 1) * per_rank] for r in range(world)]


# ------------------------------------------------------------------------------------------ expert parallel
def _ep_case(rank, world, tp):
    from quantaweave_b200.parallel.expert_parallel import (clip_grad_norm_parallel, init_expert_parallel,
                                                           sync_gradients)
    from quantaweave_b200.parallel.tensor_parallel import shard_state_dict

    cfg = tiny_config()
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg)
    ep = init_expert_parallel("cpu", tp)
    model = QuantaWeaveMoEForCausalLM(tiny_config(), expert_parallel=ep)
    state = full.state_dict()
    per = cfg.num_experts // ep.world_size
    mine = {}
    for key, value in state.items():
        if ".experts." in key:
            e = int(key.split(".experts.")[1].split(".")[0])
            if ep.rank * per <= e < (ep.rank + 1) * per:
                mine[key.replace(f".experts.{e}.", f".experts.{e - ep.rank * per}.")] = value
        else:
            mine[key] = value
    if ep.tp_size > 1:
        mine = shard_state_dict(mine, ep.tp_rank, ep.tp_size, cfg)
    model.load_state_dict(mine)
    batches = _batches(ep.world_size)
    out = model(batches[ep.rank], labels=batches[ep.rank])
    out["loss"].backward()
    sync_gradients(model, ep)
    norm = clip_grad_norm_parallel(model, ep, 1e9)
    # single-device reference: average of per-slice losses/grads with the same per-slice capacity
    ref_losses = []
    for b in batches:
        o = full(b, labels=b)
        (o["loss"] / len(batches)).backward()
        ref_losses.append(float(o["loss"]))
    ref_norm = torch.sqrt(sum(p.grad.double().pow(2).sum() for p in full.parameters())).item()
    ref_grads = full.state_dict()
    ref_grads = {n: p.grad for n, p in full.named_parameters()}
    router = dict(model.named_parameters())["blocks.0.moe.router.weight"].grad
    w_down = dict(model.named_parameters())["blocks.0.moe.w_down"].grad
    ref_w_down = ref_grads["blocks.0.moe.w_down"][ep.rank * per:(ep.rank + 1) * per]
    assert abs(float(out["loss"]) - ref_losses[ep.rank]) < 1e-4
    assert abs(float(norm) - ref_norm) < 1e-4 * max(1.0, ref_norm)
    assert torch.allclose(router, ref_grads["blocks.0.moe.router.weight"], atol=1e-5)
    if ep.tp_size == 1:
        assert torch.allclose(w_down, ref_w_down, atol=1e-5)
    return float(out["loss"])


def test_expert_parallel_matches_single_device():
    run_ranks(_ep_case, 2, (1,))


def test_tensor_parallel_model_matches_single_device():
    run_ranks(_ep_case, 2, (2,))


def _tp_case(rank, world):
    from quantaweave_b200.models.layers import Attention
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel
    from quantaweave_b200.parallel.tensor_parallel import TensorParallelAttention, shard_state_dict

    cfg = tiny_config(attention_heads=4, kv_heads=2)
    torch.manual_seed(1)
    ref = Attention(cfg)
    ep = init_expert_parallel("cpu", 2)
    tp = TensorParallelAttention(cfg, ep)
    full_state = {f"blocks.0.attention.{k}": v for k, v in ref.state_dict().items()}
    shard = shard_state_dict(full_state, ep.tp_rank, ep.tp_size, cfg)
    tp.load_state_dict({k.replace("blocks.0.attention.", ""): v for k, v in shard.items()}, strict=False)
    x = torch.randn(2, 9, 32, generator=torch.Generator().manual_seed(3))
    y = tp(x)
    y_ref = ref(x)
    assert torch.allclose(y, y_ref, atol=1e-5), (y - y_ref).abs().max()
    y.sum().backward()
    return True


def test_tensor_parallel_gqa_attention_matches():
    run_ranks(_tp_case, 2)


# ------------------------------------------------------------------------------------------ sequence parallel
def _sp_case(rank, world):
    from quantaweave_b200.parallel.expert_parallel import clip_grad_norm_parallel, init_expert_parallel, sync_gradients
    from quantaweave_b200.parallel.tensor_parallel import is_tp_sharded_shared, shard_state_dict

    # unlimited capacity and no aux loss: per-rank routing statistics would otherwise differ from the full batch's
    cfg = tiny_config(attention_heads=4, kv_heads=2, capacity_factor=0.0, router_aux_loss_coef=0.0,
                      attention_bias=True)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg)
    ctx = init_expert_parallel("cpu", world, sequence_parallel=True)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ctx)
    per = cfg.num_experts // world
    state = {}
    full_state = full.state_dict()
    attention = {k: v for k, v in full_state.items() if is_tp_sharded_shared(k)}
    state.update(shard_state_dict(attention, rank, world, cfg))
    for key, value in full_state.items():
        if key in attention:
            continue
        if ".experts." in key:
            e = int(key.split(".experts.")[1].split(".")[0])
            if rank * per <= e < (rank + 1) * per:
                state[key.replace(f".experts.{e}.", f".experts.{e - rank * per}.")] = value
        else:
            state[key] = value
    model.load_state_dict(state)
    batch = torch.randint(0, 64, (2, 17), generator=torch.Generator().manual_seed(5))  # the same batch on every rank
    out = model(batch, labels=batch, return_logits=False)
    out["loss"].backward()
    sync_gradients(model, ctx)
    norm = float(clip_grad_norm_parallel(model, ctx, 1e9))
    loss = out["loss"].detach().clone()
    dist.all_reduce(loss)
    ref = full(batch, labels=batch)
    ref["loss"].backward()
    assert abs(float(loss) / world - float(ref["loss"])) < 1e-5, (float(loss) / world, float(ref["loss"]))
    ref_norm = torch.sqrt(sum(p.grad.double().pow(2).sum() for p in full.parameters())).item()
    assert abs(norm - ref_norm) < 1e-4 * max(1.0, ref_norm), (norm, ref_norm)
    ref_grads = {n: p.grad for n, p in full.named_parameters()}
    qf = cfg.attention_heads / (cfg.attention_heads + 2 * cfg.num_kv_heads)
    from quantaweave_b200.parallel.tensor_parallel import shard_tensor

    for name, p in model.named_parameters():
        expect = ref_grads[name]
        if name.endswith(("w_gate_up", "w_down")):
            expect = expect[rank * per:(rank + 1) * per]
        elif is_tp_sharded_shared(name):
            expect = shard_tensor(name, expect, rank, world, qf)
        assert torch.allclose(p.grad, expect, atol=1e-5, rtol=1e-4), (name, (p.grad - expect).abs().max())
    return float(loss)


def test_sequence_parallel_attention_tp_and_experts_ep_on_the_same_ranks():
    """Orthogonal mapping: attention tensor-parallel and experts expert-parallel over the same 2 ranks, token rows
    sharded between the attention blocks; loss, clip norm and every gradient match the single-process model."""
    run_ranks(_sp_case, 2)


# ------------------------------------------------------------------------------------------ pipeline
def _pp_case(rank, world, schedule, microbatches):
    from quantaweave_b200.parallel.pipeline_parallel import PipelineEngine, clip_grad_norm_pipeline, init_pipeline_parallel

    cfg = tiny_config(layers=3)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg)
    pp = init_pipeline_parallel("cpu", cfg.layers)
    stage_model = QuantaWeaveMoEForCausalLM(tiny_config(layers=3), pipeline=pp)
    state = {}
    for key, value in full.state_dict().items():
        if key.startswith("blocks."):
            idx = int(key.split(".")[1])
            if pp.layer_start <= idx < pp.layer_end:
                state[key.replace(f"blocks.{idx}.", f"blocks.{idx - pp.layer_start}.", 1)] = value
        elif key.startswith(("token_embedding", "position_embedding")) and pp.is_first:
            state[key] = value
        elif key.startswith(("final_norm", "lm_head")) and pp.is_last:
            state[key] = value
    stage_model.load_state_dict(state)
    batch = _batches(1, per_rank=4)[0]
    engine = PipelineEngine(stage_model, pp, microbatches, schedule=schedule)
    result = engine.train_step(batch)
    norm = clip_grad_norm_pipeline(stage_model, pp, 1e9)
    # reference: full model, same micro-batches, summed loss / M
    ref_loss = 0.0
    for i in range(microbatches):
        mb = batch[i * (4 // microbatches):(i + 1) * (4 // microbatches)]
        out = full(mb, labels=mb)
        (out["loss"] / microbatches).backward()
        ref_loss += float(out["loss"]) / microbatches
    ref_norm = torch.sqrt(sum(p.grad.double().pow(2).sum() for p in full.parameters())).item()
    assert abs(result["loss"] - ref_loss) < 1e-4, (result["loss"], ref_loss)
    assert abs(norm - ref_norm) < 1e-4 * max(1, ref_norm)
    return result["loss"]


@pytest.mark.parametrize("schedule,microbatches", [("gpipe", 1), ("gpipe", 2), ("1f1b", 2), ("1f1b", 4)])
def test_pipeline_matches_single_device(schedule, microbatches):
    run_ranks(_pp_case, 2, (schedule, microbatches))


# ------------------------------------------------------------------------------------------ sharded optimizer
def _zero_case(rank, world):
    from quantaweave_b200.parallel.data_parallel import init_data_parallel
    from quantaweave_b200.parallel.sharded_optimizer import ShardedAdamW

    cfg = tiny_config()
    torch.manual_seed(0)
    a = QuantaWeaveMoEForCausalLM(cfg)
    b = QuantaWeaveMoEForCausalLM(cfg)
    b.load_state_dict(a.state_dict())
    dp = init_data_parallel("cpu")
    sharded = ShardedAdamW(a, dp, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, group=None)
    plain = torch.optim.AdamW(b.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    batches = _batches(world)
    for _ in range(2):
        out = a(batches[rank], labels=batches[rank])
        out["loss"].backward()
        dp.sync_gradients(a, sharded)  # under plain data parallelism the experts are replicated and sharded too
        sharded.step()
        sharded.zero_grad()
        out = b(batches[rank], labels=batches[rank])
        out["loss"].backward()
        dp.sync_gradients(b)
        plain.step()
        plain.zero_grad()
    assert not sharded.local  # no expert parallelism: nothing is rank-local
    diffs = [(n, (p - q).abs().max().item()) for (n, p), q in zip(a.named_parameters(), b.parameters())]
    worst = max(d for _, d in diffs)
    assert worst < 1e-5, diffs
    # every replica ends with the same weights, experts included
    for p in a.parameters():
        other = p.detach().clone()
        dist.broadcast(other, 0)
        assert torch.equal(other, p.detach())
    return sharded.state_numel()


def test_sharded_optimizer_matches_adamw_on_replicated_parameters():
    run_ranks(_zero_case, 2)


# ------------------------------------------------------------------------------------------ checkpoints
def test_consolidate_and_reshard_roundtrip(tmp_path):
    from quantaweave_b200.parallel.checkpoint import consolidate_checkpoint, reshard_checkpoint

    cfg = tiny_config()
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg)
    src = tmp_path / "full"
    src.mkdir()
    torch.save({"model": model.state_dict(), "optimizer": None, "step": 3, "extra": {}}, src / "model.pt")
    cfg.save(src / "config.json")
    info = reshard_checkpoint(src, tmp_path / "shards", ep_size=2, tp_size=2)
    assert info["world_size"] == 4
    consolidate_checkpoint(tmp_path / "shards", tmp_path / "merged")
    merged = torch.load(tmp_path / "merged" / "model.pt", weights_only=False)["model"]
    original = model.state_dict()
    assert merged.keys() == original.keys()
    for key in original:
        assert torch.equal(merged[key], original[key]), key


def test_sequence_parallel_reshard_roundtrip(tmp_path):
    """Orthogonal-mapping shards: rank r gets attention slice r and experts [2r, 2r+2) whole; consolidating them
    restores the original checkpoint exactly, and a shard loads into a sequence-parallel model's parameter shapes."""
    from quantaweave_b200.parallel.checkpoint import consolidate_checkpoint, reshard_checkpoint

    cfg = tiny_config(attention_heads=4, kv_heads=2, attention_bias=True)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg)
    src = tmp_path / "full"
    src.mkdir()
    torch.save({"model": model.state_dict(), "optimizer": None, "step": 3, "extra": {}}, src / "model.pt")
    cfg.save(src / "config.json")
    info = reshard_checkpoint(src, tmp_path / "shards", ep_size=2, tp_size=2, sequence_parallel=True)
    assert info["world_size"] == 2 and info["sequence_parallel"]
    shard = torch.load(info["shards"][1], weights_only=False)
    assert shard["layout"]["sequence_parallel"] and shard["layout"]["tp_rank"] == 1
    assert shard["model"]["blocks.0.attention.out_proj.weight"].shape == (32, 16)
    assert shard["model"]["blocks.0.moe.experts.1.down.weight"].shape == (32, 64)  # experts stay whole
    assert torch.equal(shard["model"]["blocks.0.moe.experts.0.down.weight"],
                       model.state_dict()["blocks.0.moe.experts.2.down.weight"])
    consolidate_checkpoint(tmp_path / "shards", tmp_path / "merged")
    merged = torch.load(tmp_path / "merged" / "model.pt", weights_only=False)["model"]
    original = model.state_dict()
    assert merged.keys() == original.keys()
    for key in original:
        assert torch.equal(merged[key], original[key]), key


def _trainer_case(rank, world, tmp, steps, extra=None):
    from pathlib import Path

    from quantaweave_b200.training.trainer import default_args, run_training

    tmp = Path(tmp)
    common = dict(synthetic_data="uniform", vocab_size=64, sequence_length=16, batch_size=2, hidden_size=32, layers=2,
                  ffn_size=64, attention_heads=4, total_experts=4, active_experts=2, device="cpu",
                  no_power_tracking=True, expert_parallel=True, checkpoint_interval=2,
                  output=tmp / "out", checkpoint_dir=tmp / "ckpt", metrics_file=tmp / f"m{rank}.jsonl")
    common.update(extra or {})
    summary = run_training(default_args(steps=steps, **common))
    return summary["steps"], summary.get("final_loss")


def test_sequence_parallel_trainer_checkpoints_resumes_and_consolidates(tmp_path):
    """``--sequence-parallel`` through ``run_training`` on 2 ranks: both ranks report the same loss, the shards carry
    the orthogonal layout, a fresh launch resumes from them, and the consolidated checkpoint loads into a plain
    single-process model."""
    extra = {"tensor_parallel": 2, "sequence_parallel": True, "log_interval": 1}
    first = run_ranks(_trainer_case, 2, (str(tmp_path), 2, extra))
    assert first[0][1] is not None and abs(first[0][1] - first[1][1]) < 1e-6, first
    results = run_ranks(_trainer_case, 2, (str(tmp_path), 4, extra))
    assert results[0][0] == 4
    shard = torch.load(tmp_path / "out" / "shards" / "model.rank1.pt", weights_only=False)
    assert shard["layout"].get("sequence_parallel") and shard["layout"]["tp_rank"] == 1
    merged = torch.load(tmp_path / "out" / "model.pt", weights_only=False)["model"]
    cfg = QuantaWeaveConfig.load(tmp_path / "out" / "config.json")
    QuantaWeaveMoEForCausalLM(cfg).load_state_dict(merged)


def test_expert_parallel_trainer_checkpoints_and_resumes(tmp_path):
    run_ranks(_trainer_case, 2, (str(tmp_path), 2))
    results = run_ranks(_trainer_case, 2, (str(tmp_path), 4))  # a fresh launch resumes from the step-2 shards
    assert results[0][0] == 4
    assert (tmp_path / "out" / "model.pt").exists()
    assert (tmp_path / "out" / "shards" / "model.rank1.pt").exists()


# ------------------------------------------------------------------------------------------ expert-parallel decode
def _ep_decode_case(rank, world):
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel

    cfg = tiny_config(capacity_factor=0.0, max_sequence_length=33, attention_heads=4, kv_heads=2)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg).eval()
    ep = init_expert_parallel("cpu", 1)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).eval()
    per = cfg.num_experts // world
    state = {}
    for key, value in full.state_dict().items():
        if ".experts." in key:
            e = int(key.split(".experts.")[1].split(".")[0])
            if rank * per <= e < (rank + 1) * per:
                state[key.replace(f".experts.{e}.", f".experts.{e - rank * per}.")] = value
        else:
            state[key] = value
    model.load_state_dict(state)
    prompts = torch.randint(0, 64, (2, 5), generator=torch.Generator().manual_seed(9))  # same prompts everywhere
    got = FastDecoder(model, torch.device("cpu"), max_batch=2).generate(prompts, 8)
    want = FastDecoder(full, torch.device("cpu"), max_batch=2).generate(prompts, 8)
    assert torch.equal(got, want), (got, want)
    return got.tolist()


def test_expert_parallel_decode_matches_single_process():
    """Each rank holds half the experts; SPMD decoding with one all-reduce per MoE layer reproduces the
    single-process decoder's greedy tokens on every rank."""
    results = run_ranks(_ep_decode_case, 2)
    assert results[0] == results[1]


# ------------------------------------------------------------------------------------------ straggler control
def _straggler_case(rank, world):
    from quantaweave_b200.parallel.expert_parallel import DeviceLoadTracker, init_expert_parallel

    cfg = tiny_config(capacity_factor=0.0, num_experts=4, top_k=1)
    ep = init_expert_parallel("cpu", 1)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).eval()
    for moe in model.moes():
        moe.simulated_cost_per_row = 1.0 if rank == 1 else 0.0  # rank 1's experts look slow
    tracker = DeviceLoadTracker(model, ep, strength=0.5, rate=0.5, interval=1)
    batch = torch.randint(0, 64, (4, 17), generator=torch.Generator().manual_seed(3))
    history = []
    with torch.no_grad():
        for step in range(1, 9):
            model(batch, labels=batch)
            history.append(tracker.update(step))
    first, last = history[0]["device_rows"], history[-1]["device_rows"]
    assert tracker.rank_bias[:, 1].mean() < 0 < tracker.rank_bias[:, 0].mean()  # slow rank pushed away
    assert last[1] < first[1] and last[0] > first[0], (first, last)
    assert abs(float(tracker.rank_bias.sum())) < 1e-9  # re-centred
    state = tracker.state_dict()
    tracker.load_state_dict(state)
    return last


def test_straggler_routing_moves_traffic_off_a_slow_rank():
    results = run_ranks(_straggler_case, 2)
    assert results[0] == results[1]  # both ranks see the same gathered loads
