"""Second headline metric: int4 weight-only MoE decode tokens/sec (benchmark configuration 5) on one B200.

    python bench_decode.py --batch 1 --bits 4
    python bench_decode.py --batch 32 --bits 4
    python bench_decode.py --impl reference --batch 1
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 bench_decode.py --batch 1

Launched on N ranks, the experts are spread expert-parallel over the N GPUs (N must divide 64) and every rank
decodes the same prompts with the native graph-captured step: each rank runs the experts it holds and stores its
per-token partial MoE outputs into every rank's exchange buffer over NVLink (csrc/ep_decode.cu); the reported time is
the max over ranks.

Config 5: the config-2 architecture (vocab 32000, d1024, 16 layers, 16 heads, 64 SwiGLU experts h2816, top-2) with
random-init N(0, 0.02) weights, experts quantised to int4 (group 128, fp16 scales, symmetric) or int8 per-channel;
a 512-token seeded uniform prompt, 256 generated tokens, greedy decoding. Decode time is measured with CUDA events
around the generation loop only (the prefill is timed separately); per-token latency is the p50 over steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
CONFIG = dict(vocab_size=32000, hidden_size=1024, layers=16, attention_heads=16, num_experts=64, ffn_size=2816,
              top_k=2, capacity_factor=1.25, router_aux_loss_coef=0.01)


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--bits", type=int, choices=(4, 8, 16), default=4)
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--new", type=int, default=256)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kernel-breakdown", action="store_true",
                   help="after timing, profile 8 more decode steps and print per-kernel device time per step")
    return p.parse_args()


def kernel_breakdown(step, steps: int = 8) -> None:
    """Device time per decode step of every kernel (torch profiler; shares only, never a reported number)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
    totals: dict = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            t, n = totals.get(e.name[:100], (0.0, 0))
            totals[e.name[:100]] = (t + e.device_time_total, n + 1)
    grand = sum(t for t, _ in totals.values()) or 1.0
    print(f"decode kernel breakdown: {grand / steps:.1f} us of device time per step", file=sys.stderr)
    for name, (t, n) in sorted(totals.items(), key=lambda kv: -kv[1][0])[:25]:
        print(f"  {100 * t / grand:5.1f}%  {t / steps:8.2f} us/step  x{n // steps:<4d} {name}", file=sys.stderr)


def main():
    import torch

    args = parse()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_expert_parallel(args)
    torch.manual_seed(args.seed)
    gen = torch.Generator().manual_seed(args.seed)
    prompts = torch.randint(0, CONFIG["vocab_size"], (args.batch, args.prompt), generator=gen)
    group = 128 if args.bits == 4 else None
    if args.impl == "reference":
        return run_reference(args, prompts, group)
    sys.path.insert(0, ROOT)
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.inference.quantization import quantize_model

    cfg = QuantaWeaveConfig(**CONFIG, max_sequence_length=args.prompt + max(args.new, 8) + 1, norm_type="layernorm",
                            position_embedding="learned", attention_bias=True, init_std=0.02)
    with torch.device("cuda"):
        model = QuantaWeaveMoEForCausalLM(cfg).eval()
    if args.bits != 16:
        quantize_model(model, args.bits, group)
    dec = FastDecoder(model, torch.device("cuda"), max_batch=args.batch)
    prompts = prompts.cuda()
    # warm-up generation (graph already captured at construction)
    dec.generate(prompts, 8)
    torch.cuda.synchronize()
    start, mid = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    dec._prefill(prompts[:, :-1])
    mid.record()
    token = prompts[:, -1]
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.new + 1)]
    events[0].record()
    for i in range(args.new):
        pos = torch.full((args.batch,), args.prompt - 1 + i, dtype=torch.int32, device="cuda")
        token = dec.run_step(token, pos).argmax(-1)
        events[i + 1].record()
    torch.cuda.synchronize()
    step_ms = [events[i].elapsed_time(events[i + 1]) for i in range(args.new)]
    decode_ms = events[0].elapsed_time(events[-1])
    if args.kernel_breakdown:
        pos = torch.full((args.batch,), args.prompt - 1, dtype=torch.int32, device="cuda")
        kernel_breakdown(lambda: dec.run_step(token, pos))
    print(json.dumps({
        "metric": "int4 decode tokens/sec" if args.bits == 4 else f"int{args.bits} decode tokens/sec",
        "value": args.batch * args.new / (decode_ms / 1000.0), "unit": "tokens/s", "n_gpus": 1,
        "batch": args.batch, "prompt": args.prompt, "new_tokens": args.new,
        "p50_token_latency_ms": statistics.median(step_ms), "prefill_ms": start.elapsed_time(mid),
        "higher_is_better": True, "impl": "native", "graph": dec.uses_graph, "weights": f"int{args.bits}"
        + (f" g{group} fp16 scales" if args.bits == 4 else " per-channel" if args.bits == 8 else " bf16"),
        "data": "synthetic seeded uniform prompt, random-init N(0,0.02) weights",
    }))


def run_reference(args, prompts, group):
    import torch

    sys.path.insert(0, ROOT)
    from bench import locate_reference_src

    src, searched = locate_reference_src(ROOT)
    if src is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference modules not found; searched "
                          + "; ".join(searched)}))
        return
    sys.path.insert(0, src)
    from fast_decode import FastDecoder
    from quantization import quantize_model
    from quantweave_moe_model import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM

    if args.batch != 1:
        print(json.dumps({"impl": "reference", "unavailable": "the reference FastDecoder decodes batch 1 only "
                          "(src/fast_decode.py); no batched decode path exists"}))
        return
    cfg = QuantaWeaveConfig(vocab_size=CONFIG["vocab_size"], hidden_size=CONFIG["hidden_size"], layers=CONFIG["layers"],
                            ffn_size=CONFIG["ffn_size"], num_experts=CONFIG["num_experts"], top_k=CONFIG["top_k"],
                            attention_heads=CONFIG["attention_heads"], max_sequence_length=args.prompt + max(args.new, 8) + 1)
    model = QuantaWeaveMoEForCausalLM(cfg)
    with torch.no_grad():
        for _, param in model.named_parameters():
            if param.dim() >= 2:
                param.normal_(0.0, 0.02)
    model = model.cuda().eval()
    if args.bits != 16:
        quantize_model(model, args.bits, group)
    dec = FastDecoder(model, torch.device("cuda"))
    ids = prompts[0].tolist()
    list(dec.stream(ids, 8, temperature=0.0))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dec.feed(ids)
    torch.cuda.synchronize()
    start.record()
    token = int(dec.logits.argmax())
    steps = []
    for _ in range(args.new):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        token = int(dec.append(token).argmax())
        e.record()
        steps.append((s, e))
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    print(json.dumps({
        "metric": f"int{args.bits} decode tokens/sec", "value": args.new / (ms / 1000.0), "unit": "tokens/s",
        "n_gpus": 1, "batch": 1, "prompt": args.prompt, "new_tokens": args.new,
        "p50_token_latency_ms": statistics.median(s.elapsed_time(e) for s, e in steps), "impl": "reference",
        "description": dec.description}))


def run_expert_parallel(args):
    """Decode with the experts sharded over the ranks of one node (``torch.distributed.run``)."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.inference.quantization import quantize_model
    from quantaweave_b200.parallel.expert_parallel import broadcast_shared_parameters, init_expert_parallel

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl", timeout=timedelta(seconds=float(os.environ.get("QW_PG_TIMEOUT_S", "300"))),
                            device_id=torch.device("cuda", local))
    try:
        ep = init_expert_parallel("cuda", 1, transport="nccl")
        group = 128 if args.bits == 4 else None
        prompts = torch.randint(0, CONFIG["vocab_size"], (args.batch, args.prompt),
                                generator=torch.Generator().manual_seed(args.seed))  # the same prompts on every rank
        cfg = QuantaWeaveConfig(**CONFIG, max_sequence_length=args.prompt + max(args.new, 8) + 1,
                                norm_type="layernorm", position_embedding="learned", attention_bias=True,
                                init_std=0.02)
        torch.manual_seed(args.seed + ep.rank)
        with torch.device("cuda"):
            model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).eval()
        broadcast_shared_parameters(model, ep)
        if args.bits != 16:
            quantize_model(model, args.bits, group)  # this rank's experts
        dec = FastDecoder(model, torch.device("cuda"), max_batch=args.batch)
        prompts = prompts.cuda()
        dec.generate(prompts, 8)  # warm-up
        dist.barrier()
        torch.cuda.synchronize()
        start, mid = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        dec._prefill(prompts[:, :-1])
        mid.record()
        token = prompts[:, -1]
        events = [torch.cuda.Event(enable_timing=True) for _ in range(args.new + 1)]
        events[0].record()
        for i in range(args.new):
            pos = torch.full((args.batch,), args.prompt - 1 + i, dtype=torch.int32, device="cuda")
            token = dec.run_step(token, pos).argmax(-1)
            events[i + 1].record()
        torch.cuda.synchronize()
        dist.barrier()
        if args.kernel_breakdown:  # every rank runs the steps (they exchange); rank 0's profile is printed
            pos = torch.full((args.batch,), args.prompt - 1, dtype=torch.int32, device="cuda")
            if ep.rank == 0:
                kernel_breakdown(lambda: dec.run_step(token, pos))
            else:
                for _ in range(8):
                    dec.run_step(token, pos)
            torch.cuda.synchronize()
            dist.barrier()
        timing = torch.tensor([events[0].elapsed_time(events[-1]), start.elapsed_time(mid)], device="cuda")
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
        step_ms = [events[i].elapsed_time(events[i + 1]) for i in range(args.new)]
        if ep.rank == 0:
            decode_ms, prefill_ms = (float(v) for v in timing)
            print(json.dumps({
                "metric": "int4 decode tokens/sec" if args.bits == 4 else f"int{args.bits} decode tokens/sec",
                "value": args.batch * args.new / (decode_ms / 1000.0), "unit": "tokens/s", "n_gpus": ep.world_size,
                "batch": args.batch, "prompt": args.prompt, "new_tokens": args.new,
                "p50_token_latency_ms": statistics.median(step_ms), "prefill_ms": prefill_ms,
                "higher_is_better": True, "impl": "native", "graph": dec.uses_graph,
                "parallelism": f"ep{ep.world_size} (SPMD native graph step; per-token partial MoE outputs exchanged "
                "by NVLink peer stores)" if dec.native else f"ep{ep.world_size} (PyTorch step, all-reduce)",
                "weights": f"int{args.bits}" + (f" g{group} fp16 scales" if args.bits == 4 else
                                                " per-channel" if args.bits == 8 else " bf16"),
                "data": "synthetic seeded uniform prompt, random-init N(0,0.02) weights"}), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
