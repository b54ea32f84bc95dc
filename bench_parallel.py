"""Training tokens/sec for the two multi-GPU benchmark configurations that ``bench.py`` does not cover.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 --master-port P \
        bench_parallel.py --config tp-ep --steps 5 --warmup 3
    python -m torch.distributed.run ... bench_parallel.py --config pp-zero --steps 5 --warmup 3

``tp-ep`` (benchmark configuration 3): the Mixtral-shaped model (vocab 32000, d4096, 32 layers, 32 query / 8 KV heads,
8 experts h14336, top-2, capacity 1.0) with attention tensor-parallel and experts expert-parallel over the SAME
ranks (sequence parallelism: token rows sharded between the attention blocks), activation checkpointing, 4
sequences of 4096 per step, seeded uniform token ids. One data-parallel group, so tokens/step = 4 x 4096.

``pp-zero`` (benchmark configuration 4): vocab 50304, d2048, 24 layers, 16 heads, 16 experts h5632, top-2, as 4 pipeline
stages x 2 data-parallel replicas, GPipe with 8 micro-batches of 4 x 2048 tokens per replica, the sharded AdamW
over the data-parallel group. tokens/step = 8 x 4 x 2048 x 2.

Both time exactly K full steps (forward, backward, gradient sync and clip, optimizer step) with CUDA events
between barriers and report the max over ranks, with nvidia-smi clocks sampled during the timed region, as
``bench.py`` does. ``--device cpu --tiny`` runs the same code on gloo ranks with a small model to check the wiring;
its wall-clock figure is labelled a CPU smoke run and is not a measurement.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys
import time
import traceback

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", choices=("tp-ep", "pp-zero"), required=True)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    p.add_argument("--tiny", action="store_true", help="a small model of the same layout (wiring check)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--layers", type=int, default=0, help="debug override of the layer count (the metric needs the "
                                                           "configuration's own)")
    p.add_argument("--kernel-breakdown", action="store_true",
                   help="after the timed steps, every rank runs one more step under the torch profiler and rank 0 "
                        "prints its per-kernel device time (shares only, to stderr)")
    return p.parse_args()


def _setup(device_kind: str):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world, rank, local = (int(os.environ.get(k, d)) for k, d in (("WORLD_SIZE", 1), ("RANK", 0), ("LOCAL_RANK", 0)))
    if world < 2:
        raise SystemExit("launch with torch.distributed.run on 2 or more ranks")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    timeout = timedelta(seconds=float(os.environ.setdefault("QW_PG_TIMEOUT_S", "300")))
    if device_kind == "cuda":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", timeout=timeout)
    return rank, world, local


class _WallTimer:
    """CPU smoke runs only: wall clock between barriers (never reported as a measurement)."""

    def __enter__(self):
        import torch.distributed as dist

        dist.barrier()
        self.start = time.perf_counter()
        return self

    def __exit__(self, *exc):
        import torch
        import torch.distributed as dist

        dist.barrier()
        elapsed = torch.tensor([time.perf_counter() - self.start], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        self.ms = float(elapsed) * 1e3


def _tp_ep(args, rank, world, device):
    import torch

    from quantaweave_b200 import QuantaWeaveMoEForCausalLM, preset
    from quantaweave_b200.parallel.expert_parallel import (broadcast_shared_parameters, clip_grad_norm_parallel,
                                                           init_expert_parallel, sync_gradients)

    seqs, seq = (4, 4096) if not args.tiny else (2, 64)
    overrides = dict(max_sequence_length=seq + 1)
    if args.tiny:
        overrides.update(vocab_size=256, hidden_size=8 * world, layers=2, attention_heads=world, kv_heads=world,
                         num_experts=world, ffn_size=32)
    if args.layers:
        overrides["layers"] = args.layers
    cfg = preset("mixtral-8x7b", **overrides)
    ep = init_expert_parallel(device.type, tensor_parallel=world, sequence_parallel=True)
    torch.manual_seed(args.seed + rank)
    with torch.device(device):
        model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep)
    model.activation_checkpointing = True
    if device.type == "cuda":
        from quantaweave_b200.training.native import prepare_model

        prepare_model(model, "bf16")
    broadcast_shared_parameters(model, ep)
    model.train()
    opt = _optimizer(model, device)
    gen = torch.Generator().manual_seed(args.seed)  # every rank gets the same sequences (one data-parallel group)
    # seqs x seq token rows (each position predicts the next; the last has no target), so the rows split evenly
    # over the sequence-parallel ranks
    batches = [torch.randint(0, cfg.vocab_size, (seqs, seq), generator=gen).to(device)
               for _ in range(args.warmup + args.steps)]

    def step(batch):
        out = model(batch, labels=batch, return_logits=False)
        out["loss"].backward()
        sync_gradients(model, ep, None)
        clip_grad_norm_parallel(model, ep, 1.0, False, opt)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return out["loss"]

    description = {"model": ("mixtral-8x7b shape (benchmark configuration 3)" if not args.layers else
                             f"DEBUG {args.layers}-layer variant of the mixtral-8x7b shape")
                   if not args.tiny else "tiny tp-ep wiring check",
                   "global_batch": seqs, "seq_len": seq,
                   "parallelism": f"sp: attention tp{world} + experts ep{world} on the same ranks",
                   "activation_checkpointing": True, "ep_transport": ep.transport}
    return step, batches, seqs * seq, description, None


def _pp_zero(args, rank, world, device):
    import torch

    from quantaweave_b200 import QuantaWeaveMoEForCausalLM, preset
    from quantaweave_b200.parallel.pipeline_parallel import PipelineEngine, init_pipeline_parallel
    from quantaweave_b200.parallel.sharded_optimizer import ShardedAdamW

    dp = 2 if world >= 4 else 1
    micro, per_micro, seq = (8, 4, 2048) if not args.tiny else (4, 2, 64)
    overrides = dict(max_sequence_length=seq + 1)
    if args.tiny:
        overrides.update(vocab_size=256, hidden_size=32, layers=2 * (world // dp), attention_heads=4, num_experts=4,
                         ffn_size=32)
    if args.layers:
        overrides["layers"] = args.layers
    cfg = preset("moe-pp-e16", **overrides)
    pp = init_pipeline_parallel(device.type, cfg.layers, data_parallel=dp)
    torch.manual_seed(args.seed + pp.stage)
    with torch.device(device):
        model = QuantaWeaveMoEForCausalLM(cfg, pipeline=pp)
    if device.type == "cuda":
        from quantaweave_b200.training.native import prepare_model

        prepare_model(model, "bf16")
    if pp.dp_size > 1:
        pp.broadcast_parameters(model)
    model.train()
    opt = ShardedAdamW(model, pp, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1) if pp.dp_size > 1 else \
        _optimizer(model, device)
    engine = PipelineEngine(model, pp, micro, contextlib.nullcontext, schedule="gpipe")
    if hasattr(opt, "arm_overlap"):  # the sharded AdamW reduce-scatters bucket by bucket during the last backward
        engine.before_last_backward = opt.arm_overlap
    gen = torch.Generator().manual_seed(args.seed * 1000 + pp.dp_rank)  # each replica its own sequences
    batches = [torch.randint(0, cfg.vocab_size, (micro * per_micro, seq + 1), generator=gen).to(device)
               for _ in range(args.warmup + args.steps)]

    def step(batch):
        result = engine.train_step(batch)
        engine.clip_and_sync(opt, 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return result["loss"]

    description = {"model": ("moe-pp-e16 (benchmark configuration 4)" if not args.layers else
                             f"DEBUG {args.layers}-layer variant of moe-pp-e16") if not args.tiny else
                   "tiny pp-zero wiring check",
                   "global_batch": micro * per_micro * pp.dp_size, "seq_len": seq,
                   "parallelism": f"pp{pp.num_stages} x dp{pp.dp_size}, gpipe, {micro} micro-batches",
                   "optimizer": "sharded AdamW over the data-parallel group" if pp.dp_size > 1 else "AdamW"}
    def replicas_identical() -> bool:
        """Every data-parallel replica of this stage holds the same weights (experts included)."""
        import torch.distributed as dist

        total = torch.stack([p.detach().double().sum() for p in model.parameters()]).sum().reshape(1)
        seen = [torch.zeros_like(total) for _ in range(pp.dp_size)]
        dist.all_gather(seen, total, group=pp.dp_group)
        return all(torch.equal(seen[0], x) for x in seen)

    return step, batches, micro * per_micro * seq * pp.dp_size, description, replicas_identical if pp.dp_size > 1 \
        else None


def _optimizer(model, device):
    import torch

    if device.type == "cuda":
        from quantaweave_b200.optim.adamw import FusedAdamW

        return FusedAdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    return torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)


def main() -> None:
    args = parse()
    rank, world, local = _setup(args.device)
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    device = torch.device("cuda", local) if args.device == "cuda" else torch.device("cpu")
    try:
        build = _tp_ep if args.config == "tp-ep" else _pp_zero
        step, batches, tokens_per_step, description, check = build(args, rank, world, device)
        for i in range(args.warmup):
            step(batches[i])
        if device.type == "cuda":
            from quantaweave_b200.ops.status import check_device_status
            from quantaweave_b200.utils.timing import ClockSampler, DeviceTimer

            torch.cuda.synchronize()
            with ClockSampler(local) as clocks:
                with DeviceTimer() as timer:
                    for i in range(args.steps):
                        loss = step(batches[args.warmup + i])
            check_device_status()
            clock_summary = clocks.summary()
        else:
            with _WallTimer() as timer:
                for i in range(args.steps):
                    loss = step(batches[args.warmup + i])
            clock_summary = None
        ms = timer.ms / args.steps
        record = {"metric": "MoE train tokens/sec", "value": tokens_per_step / (ms / 1e3), "unit": "tokens/s",
                  "n_gpus": world if device.type == "cuda" else 0, "steps": args.steps, "warmup": args.warmup,
                  "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
                  "data": "synthetic: seeded uniform token ids, random-init weights", "config": description,
                  "clocks": clock_summary, "final_loss": float(loss.detach() if hasattr(loss, "detach") else loss),
                  "impl": "native"}
        if device.type == "cpu":
            record.update(dtype="fp32", note="CPU smoke run of the wiring on gloo ranks; not a measurement")
        if device.type == "cuda":
            record["peak_mem_gb"] = round(torch.cuda.max_memory_allocated() / 1e9, 1)
        if callable(check):  # every rank takes part (a collective)
            record["dp_replicas_identical"] = bool(check())
        if rank == 0:
            print(json.dumps(record), flush=True)
        if device.type == "cuda" and args.kernel_breakdown:  # every rank steps (collectives), rank 0 reports
            from bench import kernel_breakdown

            kernel_breakdown(lambda: step(batches[-1]), report=rank == 0)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    try:
        main()
    except Exception:  # noqa: BLE001
        traceback.print_exc()
        sys.exit(1)
