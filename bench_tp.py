"""Sequence-parallel attention projections over a tensor-parallel group: fused NVLink paths against NCCL collectives.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 --master-port P \
        bench_tp.py --iters 20 --warmup 3

Under sequence parallelism each rank holds ``tokens / world`` token rows between the attention blocks. Around the
attention core two exchanges happen, timed here at the benchmark-configuration-3 shape (Mixtral-shaped: 4 x 4096
tokens, hidden 4096, 32 query / 8 KV heads of 128, so a QKV width of 6144 and an output width of 4096 split over the
ranks):

* ``ag_gemm`` (column-parallel input projection): all-gather the token rows, then ``rows @ W_qkv,r^T``.
  fused: ``FusedTPReducer.all_gather_rows`` stores this rank's rows into every peer's symmetric buffer over NVLink
  (``p2p_broadcast``), then the tcgen05 GEMM; nccl: ``all_gather_into_tensor``, then the same GEMM.
* ``gemm_rs`` (row-parallel output projection): ``o_r @ W_out,r^T`` over all rows, reduce-scattered to this rank's
  rows. fused: ``FusedTPReducer.gemm_reduce_scatter``, whose GEMM epilogue stores each partial output row into its
  owner's staging slot over NVLink, then a fixed-order local sum (``tp_reduce_rows``); nccl: the GEMM, then
  ``reduce_scatter_tensor``.

The reference does the same exchanges as an all-reduce of replicated activations (``src/tensor_parallel.py:72-100``).

Timing: CUDA events on the launching stream around each operation, mean over ``--iters`` after ``--warmup``, the
max over ranks; every operand is tens of MB or more, and a 256 MB buffer is rewritten between iterations so the
L2 starts cold. Rank 0 prints one JSON line: per operation and implementation the time, the NVLink bytes this rank
sends, and the roofline target, the slower of (GEMM FLOPs at the measured bf16 peak) and (NVLink bytes at 770 GB/s,
a measured B200 peer copy per direction).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
NVLINK_GBS = 770.0  # measured peer copy per direction per B200


def _peaks() -> tuple[float, float]:
    """(bf16 TFLOP/s burst, HBM GB/s) from the measured-peaks file next to this script, else earlier measurements."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--tokens", type=int, default=4 * 4096)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--qkv-width", type=int, default=4096 + 2 * 1024, help="query + key + value width, all ranks")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda",
                   help="cpu: gloo ranks, the NCCL composition with torch matmuls (a wiring check, not a measurement)")
    return p.parse_args()


def main() -> None:
    args = parse()
    world, rank, local = (int(os.environ.get(k, d)) for k, d in (("WORLD_SIZE", 1), ("RANK", 0), ("LOCAL_RANK", 0)))
    if world < 2:
        raise SystemExit("launch with torch.distributed.run on 2 or more ranks")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import time
    from datetime import timedelta

    import torch
    import torch.distributed as dist

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
        from quantaweave_b200.parallel.tensor_parallel import (FusedTPReducer, _all_gather_rows,
                                                               _reduce_scatter_rows)
        from quantaweave_b200.utils.timing import barrier, max_over_ranks

        M, H = args.tokens, args.hidden
        if M % world or args.qkv_width % world or H % world:
            raise SystemExit("tokens, hidden and qkv width must divide by the number of ranks")
        rows, n_qkv, k_out = M // world, args.qkv_width // world, H // world
        dtype = torch.bfloat16 if cuda else torch.float32
        gen = torch.Generator(device=device)
        gen.manual_seed(7 + rank)
        x = torch.randn(rows, H, generator=gen, device=device, dtype=dtype)
        o = torch.randn(M, k_out, generator=gen, device=device, dtype=dtype)
        w_qkv = torch.randn(n_qkv, H, generator=gen, device=device, dtype=dtype) * H ** -0.5
        w_out = torch.randn(H, k_out, generator=gen, device=device, dtype=dtype) * k_out ** -0.5
        group = dist.group.WORLD
        flush = torch.empty(64 << 20, device=device, dtype=torch.float32) if cuda else None

        if cuda:
            from quantaweave_b200.ops import ext

            C = ext()

            def gemm(a, w):
                out = torch.empty(a.size(0), w.size(0), device=device, dtype=torch.bfloat16)
                C.linear_fwd(a, w, None, None, out)
                return out
        else:
            def gemm(a, w):
                return a @ w.t()

        impls = {
            "nccl": {
                "ag_gemm": lambda: gemm(_all_gather_rows(x, group), w_qkv),
                "gemm_rs": lambda: _reduce_scatter_rows(gemm(o, w_out), group),
            },
        }
        if cuda:
            reducer = FusedTPReducer.for_group(group, device)
            impls["fused"] = {
                "ag_gemm": lambda: gemm(reducer.all_gather_rows(x), w_qkv),
                "gemm_rs": lambda: reducer.gemm_reduce_scatter(o, w_out, None, False),
            }

        def run(fn):
            total = 0.0
            for i in range(args.warmup + args.iters):
                if cuda:
                    flush.fill_(float(i))
                    torch.cuda.synchronize()
                barrier()
                if cuda:
                    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    start.record()
                    out = fn()
                    end.record()
                    torch.cuda.synchronize()
                    ms = start.elapsed_time(end)
                else:
                    t0 = time.perf_counter()
                    out = fn()
                    ms = (time.perf_counter() - t0) * 1e3
                if i >= args.warmup:
                    total += ms
            return total / args.iters, out

        results, outputs = {}, {}
        for impl, ops in impls.items():
            results[impl] = {}
            for name, fn in ops.items():
                ms, out = run(fn)
                results[impl][name] = {"ms": max_over_ranks(ms)}
                outputs[(impl, name)] = out.float()
        # the two implementations agree (bf16 outputs, fp32 sums in a different order)
        agree = {}
        if "fused" in impls:
            for name in ("ag_gemm", "gemm_rs"):
                a, b = outputs[("fused", name)], outputs[("nccl", name)]
                agree[name] = float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))
        tflops, _ = _peaks()
        work = {
            "ag_gemm": {"flops": 2.0 * M * H * n_qkv, "nvlink_bytes_out": (world - 1) * rows * H * 2},
            "gemm_rs": {"flops": 2.0 * M * k_out * H, "nvlink_bytes_out": (world - 1) * rows * H * 2},
        }
        for name, w in work.items():
            w["bound_ms"] = max(w["flops"] / (tflops * 1e12) * 1e3, w["nvlink_bytes_out"] / (NVLINK_GBS * 1e9) * 1e3)
            for impl in results:
                r = results[impl][name]
                r["fraction_of_bound"] = w["bound_ms"] / r["ms"]
        record = {"metric": "sequence-parallel attention projection exchange ms", "n_gpus": world if cuda else 0,
                  "tokens": M, "hidden": H, "qkv_width": args.qkv_width, "iters": args.iters,
                  "warmup": args.warmup, "dtype": "bf16" if cuda else "fp32", "higher_is_better": False,
                  "peaks": {"bf16_tflops": tflops, "nvlink_gbs_per_direction": NVLINK_GBS},
                  "l2": "256 MB buffer rewritten before every iteration", "work": work, **results,
                  "fused_vs_nccl_max_rel_diff": agree}
        if not cuda:
            record["note"] = "CPU wiring check on gloo ranks; not a measurement"
        if rank == 0:
            print(json.dumps(record), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
