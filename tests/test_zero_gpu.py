"""Fused ZeRO optimizer on 2 B200s: the peer-memory reduce-scatter + AdamW + all-gather kernels against the NCCL
path (reduce_scatter / all_gather), same data, same clip, three steps."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import cuda_ready

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ready() or torch.cuda.device_count() < 2, reason="needs 2 B200s")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(rank, mode):
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.ops import ext
    from quantaweave_b200.parallel.expert_parallel import (broadcast_shared_parameters, clip_grad_norm_parallel,
                                                           init_expert_parallel, sync_gradients)
    from quantaweave_b200.parallel.sharded_optimizer import ShardedAdamW
    from quantaweave_b200.training.native import prepare_model

    fused = mode != "nccl"
    os.environ["QW_ZERO_FUSED"] = "1" if fused else "0"
    os.environ["QW_ZERO_OVERLAP"] = "1" if mode == "overlap" else "0"
    torch.cuda.set_device(rank)
    ctx = init_expert_parallel("cuda", 1, transport="nccl")
    cfg = QuantaWeaveConfig(vocab_size=512, hidden_size=256, layers=2, ffn_size=256, num_experts=8, top_k=2,
                            attention_heads=4, max_sequence_length=129, capacity_factor=1.25, norm_type="rmsnorm",
                            position_embedding="rope", attention_bias=False, init_std=0.02)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ctx).cuda()
    prepare_model(model, "bf16")
    broadcast_shared_parameters(model, ctx)
    # small buckets, so the overlapped reduce-scatter runs as several bucket launches during backward
    opt = ShardedAdamW(model, ctx, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, bucket_elems=1 << 16)
    assert opt.fused == fused
    norms, first = [], {}
    for step in range(3):
        g = torch.Generator().manual_seed(100 * step + rank)
        batch = torch.randint(0, cfg.vocab_size, (2, 129), generator=g).cuda()
        if mode == "overlap":
            opt.arm_overlap()
        model(batch, labels=batch, return_logits=False)["loss"].backward()
        sync_gradients(model, ctx, opt)
        if step == 0:
            first["grad"] = {str(k): v["grad"].detach().cpu().clone() for k, v in opt.shards.items()}
        norms.append(float(clip_grad_norm_parallel(model, ctx, 0.5, True, opt)))
        opt.step()
        if step == 0:
            first["master"] = {str(k): v["master"].detach().cpu().clone() for k, v in opt.shards.items()}
        opt.zero_grad()
    torch.cuda.synchronize()
    assert ext().read_status(True) == 0
    shared = {n: p.detach().float().cpu() for n, p in model.named_parameters() if ".experts" not in n
              and not n.endswith(("w_gate_up", "w_down"))}
    return {"norms": norms, "shared": shared, "first": first}


def _worker(rank, world, port, mode, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0")
    try:
        queue.put((rank, "ok", _case(rank, mode)))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(mode):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=600)
        if status != "ok":
            for p in procs:
                p.join(timeout=30)
            raise AssertionError(f"rank {rank} failed:\n{payload}")
        results[rank] = payload
    for p in procs:
        p.join(timeout=60)
    return results


@pytest.mark.parametrize("mode", ["fused", "overlap"])
def test_fused_zero_matches_nccl_zero(mode):
    """``fused``: peer-load reduce-scatter after backward; ``overlap``: the same kernels launched bucket by bucket on
    a side stream while backward runs. Both against the NCCL reduce_scatter / all_gather path."""
    lr, steps = 1e-3, 3
    fused, plain = _run(mode), _run("nccl")
    for rank in (0, 1):
        # step 1, same inputs: the peer-load reduce-scatter is the fp32 sum of two values, exactly what NCCL computes
        for key, value in plain[rank]["first"]["grad"].items():
            assert torch.equal(fused[rank]["first"]["grad"][key], value), key
        # the fp32 masters after one AdamW step differ only by rounding (clip coefficient from an fp32 vs an fp64
        # sum of squares, fused multiply-adds)
        for key, value in plain[rank]["first"]["master"].items():
            diff = (fused[rank]["first"]["master"][key] - value).abs().max().item()
            assert diff <= 1e-6, (key, diff)
        assert abs(fused[rank]["norms"][0] - plain[rank]["norms"][0]) < 1e-6 * plain[rank]["norms"][0]
        # later steps see bf16 parameters that may round one ulp apart, and AdamW turns tiny gradient differences
        # into sign flips of size ~lr, so the trajectories are compared against AdamW's displacement bound
        for a, b in zip(fused[rank]["norms"][1:], plain[rank]["norms"][1:]):
            assert abs(a - b) < 1e-2 * b, (a, b)
        for name, value in plain[rank]["shared"].items():
            d = (fused[rank]["shared"][name] - value).abs()
            bound = 2 * lr * steps + value.abs() * 2.0 ** -7
            assert bool((d <= bound).all()), (name, d.max().item())
            assert d.mean().item() < 0.1 * lr, (name, d.mean().item())
    # the replicated parameters stay identical across ranks
    for name, value in fused[0]["shared"].items():
        assert torch.equal(value, fused[1]["shared"][name]), name
