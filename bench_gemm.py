"""tcgen05 GEMM timing at the benchmark configuration 2 shapes, one GPU.

    python bench_gemm.py                      # every case, CUDA-event medians, one JSON line per case
    python bench_gemm.py --case gate_up_balanced --iters 3 --warmup 1     # one case (for a profiler capture)

Cases (H = 1024, F = 2816, 64 experts, 32 x 2048 tokens, top-2):

* ``gate_up_balanced``: grouped gate|up projection with the SwiGLU epilogue, every expert at its capacity
  (2560 rows, 163,840 rows in all);
* ``gate_up_zipf``: the same GEMM with per-expert rows drawn from a Zipf(1.1) over the experts and cut at capacity
  (the load the benchmark's Zipf tokens produce);
* ``down_balanced``: grouped down projection, every expert at capacity;
* ``gate_up_wgrad_balanced`` / ``gate_up_wgrad_zipf``: the gate|up weight gradient, reduced over each expert's rows
  (every expert's [2F x H] block is written, also for experts with few rows);
* ``qkv_fwd``: dense [65536 x 1024] @ [3072 x 1024]^T; ``qkv_wgrad``: its weight gradient (split-K);
* ``lm_head``: dense [16384 x 1024] @ [32000 x 1024]^T (one chunk of the chunked cross-entropy).

Each case reports the median time, TFLOP/s over the useful rows, and the fraction of the measured bf16 peak
(``MEASURED_PEAKS.json`` when present). Inputs are far larger than the 126 MB L2 or re-read identically by every
run, as in training.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

ROOT = os.path.dirname(os.path.abspath(__file__))
H, F, E, CAP = 1024, 2816, 64, 2560


def _peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0  # earlier measurement on this pool (burst cuBLAS bf16)


def _zipf_counts(total_routes: int = 131072, s: float = 1.1):
    weights = [(e + 1) ** -s for e in range(E)]
    norm = sum(weights)
    return [min(CAP, int(total_routes * w / norm)) for w in weights]


def cases(torch, C):
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)

    def grouped(counts, down: bool):
        rows = E * CAP
        offsets = torch.arange(E, device=dev, dtype=torch.int32) * CAP
        cnt = torch.tensor(counts, device=dev, dtype=torch.int32)
        useful = sum(counts)
        if down:
            h = torch.randn(rows, F, device=dev, generator=g).bfloat16()
            w = (torch.randn(E, H, F, device=dev, generator=g) * 0.02).bfloat16()
            y = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
            return (lambda: C.moe_down_fwd(h, w, cnt, offsets, y)), 2.0 * useful * H * F
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        w = (torch.randn(E, 2 * F, H, device=dev, generator=g) * 0.02).bfloat16()
        out = torch.empty(rows, F, device=dev, dtype=torch.bfloat16)
        return (lambda: C.moe_gate_up_fwd(x, w, cnt, offsets, out, None)), 2.0 * useful * 2 * F * H

    def grouped_wgrad(counts):
        rows = E * CAP
        offsets = torch.arange(E, device=dev, dtype=torch.int32) * CAP
        cnt = torch.tensor(counts, device=dev, dtype=torch.int32)
        dgu = torch.randn(rows, 2 * F, device=dev, generator=g).bfloat16()
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        dw = torch.empty(E, 2 * F, H, device=dev, dtype=torch.bfloat16)
        return (lambda: C.moe_wgrad(dgu, x, cnt, offsets, dw, False, 1, 1.0)), 2.0 * sum(counts) * 2 * F * H

    def dense(M, N, K, wgrad=False):
        a = torch.randn(M, K, device=dev, generator=g).bfloat16()
        if wgrad:
            dy = torch.randn(M, N, device=dev, generator=g).bfloat16()
            dw = torch.empty(N, K, device=dev, dtype=torch.bfloat16)
            return (lambda: C.linear_wgrad(dy, a, dw, False)), 2.0 * M * N * K
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        return (lambda: C.linear_fwd(a, w, None, None, out)), 2.0 * M * N * K

    return {
        "gate_up_balanced": lambda: grouped([CAP] * E, False),
        "gate_up_zipf": lambda: grouped(_zipf_counts(), False),
        "down_balanced": lambda: grouped([CAP] * E, True),
        "gate_up_wgrad_balanced": lambda: grouped_wgrad([CAP] * E),
        "gate_up_wgrad_zipf": lambda: grouped_wgrad(_zipf_counts()),
        "qkv_fwd": lambda: dense(65536, 3072, 1024),
        "qkv_wgrad": lambda: dense(65536, 3072, 1024, wgrad=True),
        "lm_head": lambda: dense(16384, 32000, 1024),
    }


def trace_summary(torch, C, run) -> dict:
    """Median per-tile phase lengths (SM clocks) of CTA 0 over one launch: producer streaming time, the issuer's wait
    for a free accumulator, its wait for the first k-block, its k-loop, the epilogue, and the tile period."""
    buf = torch.zeros(64 * 8, dtype=torch.int64, device="cuda")
    C.gemm_trace(buf)
    run()
    torch.cuda.synchronize()
    C.gemm_trace(None)
    t = buf.view(64, 8).cpu().tolist()
    t = [row for row in t if row[3] and row[7]]
    med = lambda xs: statistics.median(xs) if xs else None  # noqa: E731
    return {
        "tiles": len(t),
        "producer": med([r[1] - r[0] for r in t]),
        "acc_wait": med([r[3] - r[2] for r in t]),
        "first_kblock_wait": med([r[4] - r[3] for r in t]),
        "mainloop": med([r[5] - r[3] for r in t]),
        "epilogue": med([r[7] - r[6] for r in t]),
        "epilogue_wait": med([r[6] - r[5] for r in t]),
        "period": med([b[5] - a[5] for a, b in zip(t, t[1:])]),
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--trace", action="store_true",
                    help="also print per-tile SM-clock timestamps of CTA 0 (producer, MMA issuer, epilogue)")
    args = ap.parse_args()
    import torch

    from quantaweave_b200.ops import ext

    C = ext()
    table = cases(torch, C)
    names = list(table) if args.case == "all" else [args.case]
    peak = _peak()
    for name in names:
        run, flops = table[name]()
        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.iters):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            run()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
        ms = statistics.median(times)
        if args.trace:
            print(json.dumps({"case": name, "trace": trace_summary(torch, C, run)}), flush=True)
        tflops = flops / ms / 1e9
        print(json.dumps({"case": name, "ms": round(ms, 4), "tflops": round(tflops, 1),
                          "fraction_of_measured_bf16": round(tflops / peak, 3)}), flush=True)
        if C.read_status(True) != 0:
            raise SystemExit("a kernel reported a device-side error status")


if __name__ == "__main__":
    main()
