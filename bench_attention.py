"""Causal attention kernel timing: forward and backward of ``ops.attention.attention_core`` on one GPU.

    python bench_attention.py --batch 8 --seq 2048 --heads 16 --head-dim 64
    QW_ATTN_BWD=mma python bench_attention.py ...      # the mma.sync backward instead of the tcgen05 one
    QW_ATTN_FWD=mma python bench_attention.py ...      # the mma.sync forward instead of the tcgen05 one

Prints one JSON line: median forward / backward milliseconds over ``--iters`` runs (CUDA events on the launching
stream, after warm-up) and the corresponding TFLOP/s (causal forward = 2 GEMMs over half the S x S scores; backward
counted as 2.5x the forward).
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=0, help="0 = same as --heads")
    ap.add_argument("--head-dim", type=int, default=64)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--trace", action="store_true",
                    help="also print the forward's per-tile timeline (SM clocks) of its first CTA")
    args = ap.parse_args()

    from quantaweave_b200.ops import ext
    from quantaweave_b200.ops.attention import attention_core

    B, S, h, d = args.batch, args.seq, args.heads, args.head_dim
    hkv = args.kv_heads or h
    torch.manual_seed(0)
    qkv = (torch.randn(B * S, (h + 2 * hkv) * d, device="cuda") * 0.5).bfloat16().requires_grad_()
    grad = torch.randn(B * S, h * d, device="cuda").bfloat16()
    for _ in range(args.warmup):
        attention_core(qkv, B, S, h, hkv, d, False, 1e4).backward(grad)
    torch.cuda.synchronize()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    fwd, bwd = [], []
    for _ in range(args.iters):
        events[0].record()
        out = attention_core(qkv, B, S, h, hkv, d, False, 1e4)
        events[1].record()
        out.backward(grad)
        events[2].record()
        torch.cuda.synchronize()
        fwd.append(events[0].elapsed_time(events[1]))
        bwd.append(events[1].elapsed_time(events[2]))
    fwd.sort()
    bwd.sort()
    f_ms, b_ms = fwd[len(fwd) // 2], bwd[len(bwd) // 2]
    flops = 4.0 * B * h * S * S * d / 2
    print(json.dumps({"forward_path": os.environ.get("QW_ATTN_FWD", "tcgen05" if d in (64, 128) else "mma"),
                      "backward_path": os.environ.get("QW_ATTN_BWD", "tcgen05"), "batch": B, "seq": S, "heads": h,
                      "kv_heads": hkv, "head_dim": d, "fwd_ms": round(f_ms, 4), "bwd_ms": round(b_ms, 4),
                      "fwd_tflops": round(flops / f_ms / 1e9, 1), "bwd_tflops": round(2.5 * flops / b_ms / 1e9, 1)}))
    if args.trace:
        buf = torch.zeros(32 * 2 * 8, dtype=torch.int64, device="cuda")
        ext().attn_fwd_trace(buf)
        attention_core(qkv, B, S, h, hkv, d, False, 1e4)
        torch.cuda.synchronize()
        ext().attn_fwd_trace(None)
        t = buf.view(32, 2, 8).cpu().tolist()
        t0 = min(v for tile in t for grp in tile for v in grp if v)
        rows = [[[v - t0 if v else None for v in grp[:6]] for grp in tile] for tile in t if any(tile[0][:6])]
        print(json.dumps({"forward_timeline": "per tile j, per group: [scores ready, probabilities computed, previous "
                                              "PV done, P written, S(j) issued, O(j) issued] in SM clocks",
                          "tiles": rows}))
        buf = torch.zeros(2 * 32 * 16, dtype=torch.int64, device="cuda")
        ext().attn_bwd_trace(buf)
        out = attention_core(qkv, B, S, h, hkv, d, False, 1e4)
        out.backward(grad)
        torch.cuda.synchronize()
        ext().attn_bwd_trace(None)
        for m, name in enumerate(("dkdv", "dq")):
            t = buf.view(2, 32, 16)[m].cpu().tolist()
            t0 = min((v for row in t for v in row if v), default=0)
            print(json.dumps({"backward_timeline": name, "columns": "per tile t: [S/dP issued, scores ready, P/dS "
                                                                    "written (first warp), accumulation issued, P/dS "
                                                                    "written by warps 0-7 of the group] in SM clocks",
                              "tiles": [[v - t0 if v else None for v in row] for row in t if any(row)]}))
    if ext().read_status(True) != 0:
        raise SystemExit("a kernel reported a device-side error status")


if __name__ == "__main__":
    main()
