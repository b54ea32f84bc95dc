"""Sharded AdamW (ZeRO over a data-parallel group): the fused NVLink kernels against the NCCL collectives.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port P \
        bench_zero.py --numel 1073741824 --iters 10 --warmup 3

Every rank holds the same replicated bf16 parameters (``--numel`` elements in ``--tensors`` tensors) and a fresh
bf16 gradient for each of them. One iteration is what ``ShardedAdamW`` does after backward:

* ``reduce_gradients``: the gradients are packed into the staging buffer and reduce-scattered, so that each rank
  holds the average of its ``numel / world`` shard in fp32;
* ``step``: AdamW on the shard against the fp32 master, then the updated shard goes back into every rank's
  parameters (the all-gather).

Both implementations of ``parallel/sharded_optimizer.py`` run on the same parameters: ``fused`` (``zero_fused.cu``:
a peer-load reduce-scatter and an AdamW kernel whose stores into every rank's parameter buffer are the all-gather,
both with 16-byte accesses over NVLink) and ``nccl`` (``reduce_scatter_tensor`` / ``all_gather_into_tensor`` of the
fp32 flat buffers, the shape of the reference's owner-reduce / broadcast in ``src/sharded_optimizer.py:52-87``).
The overlap with backward is off here (there is no backward to hide behind); this times the exchange itself.

Timing: CUDA events around each phase on the launching stream, mean over ``--iters`` after ``--warmup``, the max
over ranks. Every buffer is far larger than the 126 MB L2, so nothing is flushed between iterations. Rank 0 prints
one JSON line with both implementations and, for the fused one, the NVLink bytes each rank moves per direction and
the bound they give at 770 GB/s (a measured B200 peer copy), next to the HBM bound at the measured copy bandwidth.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from types import SimpleNamespace

ROOT = os.path.dirname(os.path.abspath(__file__))
NVLINK_GBS = 770.0  # measured peer copy per direction per B200


def _hbm_gbs() -> float:
    """Copy bandwidth of one B200 from the measured-peaks file next to this script, else an earlier measurement."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--numel", type=int, default=1 << 30, help="replicated parameter elements (bf16)")
    p.add_argument("--tensors", type=int, default=16, help="how many parameter tensors they are split into")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda",
                   help="cpu: gloo ranks, the NCCL-path code only, wall clock (a wiring check, not a measurement)")
    return p.parse_args()


def _time(opt, params, grads, iters, warmup, cuda):
    """Mean ms of (reduce_gradients, step) over ``iters`` iterations on this rank: CUDA events on the launching
    stream, or the wall clock on CPU."""
    import time

    import torch

    from quantaweave_b200.utils.timing import barrier

    red, upd = 0.0, 0.0
    for i in range(warmup + iters):
        for p, g in zip(params, grads):
            p.grad = g
        if cuda:
            torch.cuda.synchronize()
        barrier()
        if cuda:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            opt.reduce_gradients()
            e[1].record()
            opt.step()
            e[2].record()
            torch.cuda.synchronize()
            times = (e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2]))
        else:
            t0 = time.perf_counter()
            opt.reduce_gradients()
            t1 = time.perf_counter()
            opt.step()
            t2 = time.perf_counter()
            times = ((t1 - t0) * 1e3, (t2 - t1) * 1e3)
        if i >= warmup:
            red += times[0]
            upd += times[1]
    return red / iters, upd / iters


def _replicas_identical(params, world) -> bool:
    """Collective: every rank's parameters hash to the same checksum after the updates (the all-gather landed)."""
    import torch
    import torch.distributed as dist

    local = torch.stack([p.detach().float().double().sum() for p in params]).sum().reshape(1)
    gathered = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)
    return all(bool(torch.equal(g, gathered[0])) for g in gathered)


def main() -> None:
    args = parse()
    world, rank, local = (int(os.environ.get(k, d)) for k, d in (("WORLD_SIZE", 1), ("RANK", 0), ("LOCAL_RANK", 0)))
    if world < 2:
        raise SystemExit("launch with torch.distributed.run on 2 or more ranks")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    os.environ["QW_ZERO_OVERLAP"] = "0"
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    cuda = args.device == "cuda"
    timeout = timedelta(seconds=float(os.environ.get("QW_PG_TIMEOUT_S", "120")))
    if cuda:
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        dist.init_process_group("nccl", timeout=timeout, device_id=device)
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timeout)
    try:
        from quantaweave_b200.parallel.sharded_optimizer import ShardedAdamW
        from quantaweave_b200.utils.timing import max_over_ranks

        per_tensor = (args.numel // args.tensors + 7) // 8 * 8
        gen = torch.Generator(device=device)
        gen.manual_seed(1234)  # identical parameters on every rank
        model = torch.nn.Module()
        model.weights = torch.nn.ParameterList(
            torch.nn.Parameter(torch.randn(per_tensor, generator=gen, device=device, dtype=torch.bfloat16) * 0.02)
            for _ in range(args.tensors))
        params = list(model.parameters())
        gen.manual_seed(99 + rank)  # each rank's own gradients
        grads = [torch.randn(per_tensor, generator=gen, device=device, dtype=torch.bfloat16) * 1e-3 for _ in params]
        ctx = SimpleNamespace(group=dist.group.WORLD)
        kw = dict(lr=1e-4, betas=(0.9, 0.95), weight_decay=0.1)
        results = {}
        for impl in ("nccl", "fused") if cuda else ("nccl",):
            os.environ["QW_ZERO_FUSED"] = "1" if impl == "fused" else "0"
            opt = ShardedAdamW(model, ctx, **kw)
            assert opt.fused == (impl == "fused")
            red, upd = _time(opt, params, grads, args.iters, args.warmup, cuda)
            red, upd = max_over_ranks(red), max_over_ranks(upd)
            results[impl] = {"reduce_gradients_ms": red, "step_ms": upd, "total_ms": red + upd}
            del opt
            if cuda:
                torch.cuda.synchronize()
        numel = per_tensor * args.tensors
        identical = _replicas_identical(params, world)
        if not cuda:
            if rank == 0:
                print(json.dumps({"metric": "sharded AdamW exchange + update ms", "n_gpus": 0, "numel": numel,
                                  "replicas_identical": identical, **results,
                                  "note": "CPU wiring check on gloo ranks; not a measurement"}), flush=True)
            return
        per = ((numel + world - 1) // world + 7) // 8 * 8
        nv_in = (world - 1) * per * 2  # reduce-scatter: bf16 of this rank's shard from every peer
        nv_out = (world - 1) * per * 2  # all-gather: bf16 of this rank's updated shard into every peer
        # HBM per rank: gradient pack (read + write bf16), the reduce-scatter's local read and fp32 write, AdamW's
        # 28 bytes per shard element, the parameter stores landing in this rank's buffer from every rank
        hbm_reduce = numel * 4 + per * 2 + per * 4
        hbm_step = per * 28 + numel * 2
        f = results["fused"]
        f["nvlink_bytes_in_per_rank"], f["nvlink_bytes_out_per_rank"] = nv_in, nv_out
        hbm = _hbm_gbs()
        f["reduce_bound_ms"] = max(nv_in / NVLINK_GBS / 1e6, hbm_reduce / hbm / 1e6)
        f["step_bound_ms"] = max(nv_out / NVLINK_GBS / 1e6, hbm_step / hbm / 1e6)
        f["fraction_of_bound"] = (f["reduce_bound_ms"] + f["step_bound_ms"]) / f["total_ms"]
        record = {"metric": "sharded AdamW exchange + update ms", "n_gpus": world, "numel": numel,
                  "tensors": args.tensors, "iters": args.iters, "warmup": args.warmup, "dtype": "bf16",
                  "higher_is_better": False, "speedup_fused_vs_nccl": results["nccl"]["total_ms"] / f["total_ms"],
                  "l2": "no flush: every buffer is several GB", "replicas_identical": identical, **results}
        if rank == 0:
            print(json.dumps(record), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
