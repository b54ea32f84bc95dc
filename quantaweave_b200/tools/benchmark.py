"""Benchmark a saved checkpoint: quality, speed, memory, parameter counts and routing health.

Report parity with the reference ``src/benchmark_quantweave_moe.py`` (``run_benchmark`` :81-188 with the same JSON
keys, ``routing_and_compute`` :192-252, ``render_markdown`` :255-303, ``training_stability`` :44-59). On CUDA the
timed pass is measured with CUDA events on the launching stream (device time; the wall clock is reported beside it)
and the model runs the native sm_100a kernels; ``--training-metrics`` folds in the stability of a training log.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import time
from pathlib import Path
from typing import Optional

import torch

from .common import synchronize  # noqa: F401  (the reference exposes it from its benchmark module)


def process_rss_bytes() -> Optional[int]:
    try:
        import psutil

        return psutil.Process(os.getpid()).memory_info().rss
    except ImportError:
        return None


def training_stability(path: Path) -> dict:
    from ..training.metrics import detect_plateau, first_stable_step

    records = [json.loads(line) for line in Path(path).read_text().splitlines() if line.strip()]
    rows = [r for r in records if "loss" in r]
    if not rows:
        return {}
    losses = [r["loss"] for r in rows]
    tail = losses[-min(len(losses), 20):]
    return {
        "logged_steps": len(losses),
        "final_loss": sum(tail) / len(tail),
        "best_loss": min(losses),
        "plateaued": detect_plateau(losses),
        "first_stable_step": first_stable_step([r["step"] for r in rows], losses),
        "mean_tokens_per_second": sum(r.get("tokens_per_second", 0) for r in records) / len(records),
        "total_overflow_routes": sum(r.get("overflow_routes", 0) for r in records),
    }


def histogram(values: list[float], bins: int = 10) -> dict:
    top = max(values) if values and max(values) > 0 else 1.0
    counts = torch.histc(torch.tensor(values, dtype=torch.float32), bins=bins, min=0.0, max=top).tolist()
    return {"edges": [top * i / bins for i in range(bins + 1)], "counts": [int(c) for c in counts]}


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    p.add_argument("--data", type=Path, default=Path("data/smoke/tinystories.jsonl"))
    p.add_argument("--examples", type=int, default=1000)
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    p.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    p.add_argument("--output", type=Path, help="write the report as JSON here, with a Markdown copy next to it")
    p.add_argument("--training-metrics", type=Path, help="the training run's metrics.jsonl, to add loss-stability figures")
    p.add_argument("--no-routing-stats", action="store_true", help="leave out the per-layer routing and expert-time pass")
    from .common import describe_options

    describe_options(p)
    return p


class _Clock:
    """Device-side timing on CUDA (events on the current stream), wall clock elsewhere."""

    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda"
        if self.cuda:
            self.start_event = torch.cuda.Event(enable_timing=True)
            self.end_event = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize()
            self.start_event.record()
        self.wall = time.perf_counter()
        return self

    def __exit__(self, *exc) -> None:
        if self.cuda:
            self.end_event.record()
            torch.cuda.synchronize()
        self.wall = time.perf_counter() - self.wall
        self.seconds = self.start_event.elapsed_time(self.end_event) / 1000.0 if self.cuda else self.wall


def run_benchmark(args) -> dict:
    from ..data.pipeline import WindowDataset, build_corpus, load_tokenizer
    from ..training.trainer import autocast_context, select_device
    from ..utils.hardware import choose_precision, detect, parameter_counts
    from .common import load_model

    for path in (args.checkpoint / "config.json", args.checkpoint / "model.pt", args.data):
        if not Path(path).exists():
            raise FileNotFoundError(f"missing required path: {path}")
    device = select_device(args.device)
    model, payload = load_model(args.checkpoint, device, args.precision, with_payload=True)
    config = model.config
    tokenizer = load_tokenizer(args.checkpoint)
    dataset = WindowDataset(build_corpus([args.data], tokenizer, args.examples), config.max_sequence_length - 1)
    if len(dataset) == 0:
        raise ValueError("benchmark dataset contains no usable sequences")
    batches = [dataset.batch(range(s, min(len(dataset), s + args.batch_size)))
               for s in range(0, len(dataset), args.batch_size)]
    precision = choose_precision(detect(device.type), args.precision)
    counts = parameter_counts(config)
    per_expert = 3 * config.hidden_size * config.ffn_size
    expert_params = config.layers * config.num_experts * per_expert
    total_params = sum(p.numel() for p in model.parameters()) + sum(
        b.numel() for name, b in model.named_buffers() if name.split(".")[-1].startswith(("q_", "qweight")))
    shared = counts["total"] - expert_params
    active = shared + config.layers * config.top_k * per_expert
    param_bytes = sum(t.numel() * t.element_size() for t in list(model.parameters()) + list(model.buffers()))
    expert_elem = 2 if device.type == "cuda" else 4

    loss_sum = aux_sum = 0.0
    tokens = dropped = overflow = routed = 0
    expert_counts = torch.zeros(config.num_experts, dtype=torch.long, device=device)
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats()
    with torch.inference_mode(), _Clock(device) as clock:
        losses, auxes, drops, overs = [], [], [], []
        for batch in batches:
            batch = batch.to(device, non_blocking=True)
            with autocast_context(device, precision):
                out = model(batch, labels=batch, return_logits=False)
            n = batch.size(0) * (batch.size(1) - 1)
            losses.append(out["loss"].float() * n)
            auxes.append(out["router_aux_loss"].float())
            drops.append(out["dropped_routes"])
            overs.append(out["overflow_routes"])
            tokens += n
            routed += batch.numel()
            for idx in out["expert_indices"]:
                expert_counts += torch.bincount(idx.reshape(-1), minlength=config.num_experts)
    loss_sum = float(torch.stack(losses).sum())
    aux_sum = float(torch.stack(auxes).sum())
    dropped = int(torch.stack(drops).sum())
    overflow = int(torch.stack(overs).sum())
    elapsed = clock.seconds
    mean_loss = loss_sum / tokens
    routes = routed * config.layers * config.top_k
    utilization = (expert_counts.double() / routes).cpu().tolist()
    report = {
        "checkpoint": str(args.checkpoint),
        "device": str(device),
        "device_name": torch.cuda.get_device_name(device) if device.type == "cuda" else device.type,
        "precision": precision,
        "tokenizer": tokenizer.kind,
        "examples": len(dataset),
        "tokens": tokens,
        "batches": len(batches),
        "elapsed_seconds": elapsed,
        "wall_seconds": clock.wall,
        "timing": "cuda events (device time)" if device.type == "cuda" else "wall clock",
        "seconds_per_batch": elapsed / len(batches),
        "tokens_per_second": tokens / elapsed,
        "loss": mean_loss,
        "perplexity": math.exp(min(mean_loss, 20)),
        "router_aux_loss": aux_sum / len(batches),
        "dropped_routes": dropped,
        "dropped_route_fraction": dropped / max(1, routes),
        "overflow_routes": overflow,
        "overflow_route_fraction": overflow / max(1, routes),
        "capacity_factor": config.capacity_factor,
        "min_expert_capacity": config.min_expert_capacity,
        "drop_overflow_tokens": config.drop_overflow_tokens,
        "overflow_policy": config.overflow_policy,
        "router_temperature": config.router_temperature,
        "total_parameters": total_params,
        "shared_parameters_estimate": shared,
        "expert_parameters_estimate": expert_params,
        "active_parameters_per_token_estimate": active,
        "active_parameter_ratio": active / counts["total"],
        "num_experts": config.num_experts,
        "active_experts_per_token": config.top_k,
        "inactive_experts_per_token": config.num_experts - config.top_k,
        "expert_utilization_min": min(utilization),
        "expert_utilization_max": max(utilization),
        "expert_utilization_mean": sum(utilization) / len(utilization),
        "expert_utilization_histogram": histogram(utilization),
        "memory": {
            "parameter_bytes": param_bytes,
            "bytes_per_expert": per_expert * config.layers * expert_elem,
            "peak_device_bytes": torch.cuda.max_memory_allocated(device) if device.type == "cuda" else None,
            "process_rss_bytes": process_rss_bytes(),
        },
        "training_step_in_checkpoint": payload.get("step"),
    }
    if not args.no_routing_stats:
        report["routing"], report["expert_compute"] = routing_and_compute(model, batches, device, precision, config)
    if args.training_metrics is not None and Path(args.training_metrics).exists():
        report["training_stability"] = training_stability(args.training_metrics)
    return report


@torch.inference_mode()
def routing_and_compute(model, batches, device, precision, config) -> tuple[dict, dict]:
    """Second pass with router statistics and per-expert timing on (the per-expert loop, slower than the timed pass)."""
    from ..training.trainer import autocast_context

    model.set_collect_stats(True)
    saved_kernels = [moe.kernel for moe in model.moes()]
    for moe in model.moes():
        moe.profile_experts = True
        moe.expert_seconds = [0.0] * moe.num_local_experts
    L, E = config.layers, config.num_experts
    entropy = torch.zeros(L, device=device)
    confidence = torch.zeros(L, device=device)
    conf_hist = torch.zeros(L, 10, device=device)
    assigned = torch.zeros(L, E, dtype=torch.long, device=device)
    load = torch.zeros(L, E, dtype=torch.long, device=device)
    with _Clock(device) as clock:
        for batch in batches:
            with autocast_context(device, precision):
                model(batch.to(device), return_logits=False)
            for layer, stats in enumerate(model.routing_stats()):
                entropy[layer] += stats["entropy_mean"].float()
                confidence[layer] += stats["confidence_mean"].float()
                conf_hist[layer] += stats["confidence_hist"].float()
                assigned[layer] += stats["expert_assigned"].to(device)
                load[layer] += stats["expert_load"].to(device)
    n = len(batches)
    entropy, confidence = (entropy / n).cpu().tolist(), (confidence / n).cpu().tolist()
    conf_hist = (conf_hist / n).cpu()
    assigned, load = assigned.cpu().double(), load.cpu().double()
    per_layer = []
    for layer in range(L):
        share = (load[layer] / load[layer].sum().clamp(min=1)).tolist()
        counts = assigned[layer]
        even = counts.sum() / E
        per_layer.append({
            "utilization": share,
            "utilization_histogram": histogram(share),
            "entropy": entropy[layer],
            "entropy_normalized": entropy[layer] / math.log(E) if E > 1 else 0.0,
            "confidence_mean": confidence[layer],
            "confidence_histogram": conf_hist[layer].tolist(),
            "dead_experts": int((counts == 0).sum()),
            "underused_experts": int((counts < 0.1 * even).sum()),
            "load_cv": float(counts.std(unbiased=False) / counts.mean().clamp(min=1e-9)),
            "drop_rate": float(1 - load[layer].sum() / counts.sum().clamp(min=1)),
        })
    seconds = [sum(moe.expert_seconds[e] for moe in model.moes()) for e in range(model.moes()[0].num_local_experts)]
    for moe, kernel in zip(model.moes(), saved_kernels):
        moe.profile_experts = False
        moe.kernel = kernel
    model.set_collect_stats(False)
    total = sum(seconds)
    routing = {
        "per_layer": per_layer,
        "entropy_mean": sum(x["entropy"] for x in per_layer) / L,
        "confidence_mean": sum(x["confidence_mean"] for x in per_layer) / L,
        "dead_experts_total": sum(x["dead_experts"] for x in per_layer),
    }
    compute = {
        "seconds_per_expert": seconds,
        "moe_seconds_total": total,
        "moe_share_of_forward": total / clock.wall if clock.wall else None,
        "note": "measured on a separate profiled pass (per-expert loop with host timers)",
    }
    return routing, compute


def _megabytes(count) -> str:
    return "n/a" if count is None else f"{count / 1e6:,.1f} MB"


# (section title, [(row label, cell text from the report)]): the two-column summary tables of the report.
_SUMMARY = (
    ("Quality", (
        ("loss", lambda r: f"{r['loss']:.4f}"),
        ("perplexity", lambda r: f"{r['perplexity']:.2f}"),
        ("tokens evaluated", lambda r: f"{r['tokens']:,}"))),
    ("Speed and memory", (
        ("tokens / second", lambda r: f"{r['tokens_per_second']:,.0f}"),
        ("seconds / batch", lambda r: f"{r['seconds_per_batch']:.4f}"),
        ("parameter memory", lambda r: _megabytes(r["memory"]["parameter_bytes"])),
        ("memory per expert (all layers)", lambda r: _megabytes(r["memory"]["bytes_per_expert"])),
        ("peak device memory", lambda r: _megabytes(r["memory"]["peak_device_bytes"])),
        ("process RSS", lambda r: _megabytes(r["memory"]["process_rss_bytes"])))),
    ("Parameters", (
        ("total", lambda r: f"{r['total_parameters']:,}"),
        ("active per token", lambda r: f"{r['active_parameters_per_token_estimate']:,}"),
        ("active / total", lambda r: f"{r['active_parameter_ratio']:.1%}"),
        ("experts (total / active)", lambda r: f"{r['num_experts']} / {r['active_experts_per_token']}"))),
    ("Routing", (
        ("aux (balance) loss", lambda r: f"{r['router_aux_loss']:.4f}"),
        ("overflow routes", lambda r: f"{r['overflow_routes']:,} ({r['overflow_route_fraction']:.2%})"),
        ("dropped routes", lambda r: f"{r['dropped_routes']:,} ({r['dropped_route_fraction']:.2%})"),
        ("capacity factor", lambda r: f"{r['capacity_factor']}"),
        ("expert utilization min / mean / max", lambda r: " / ".join(
            f"{r[f'expert_utilization_{k}']:.4f}" for k in ("min", "mean", "max"))))),
)

_PER_LAYER = ("layer", "entropy (norm.)", "confidence", "load CV", "dead", "underused", "drop rate")


def _table(header, rows) -> list[str]:
    """A Markdown table followed by a blank line."""
    return ["| " + " | ".join(header) + " |", "|" + "---|" * len(header),
            *("| " + " | ".join(str(cell) for cell in row) + " |" for row in rows), ""]


def _layer_cells(index: int, layer: dict) -> tuple:
    return (index, f"{layer['entropy']:.3f} ({layer['entropy_normalized']:.0%})", f"{layer['confidence_mean']:.3f}",
            f"{layer['load_cv']:.3f}", layer["dead_experts"], layer["underused_experts"], f"{layer['drop_rate']:.2%}")


def render_markdown(report: dict) -> str:
    """The benchmark report as Markdown: header bullets, the summary tables of ``_SUMMARY``, then the per-layer
    routing table and the expert-compute line when the routing pass ran, then the training-stability table when a
    metrics file was given."""
    out = [f"# Benchmark: {report['checkpoint']}", "",
           f"- device: {report['device_name']} ({report['device']}), precision {report['precision']}, "
           f"tokenizer {report['tokenizer']}",
           f"- checkpoint step: {report['training_step_in_checkpoint']}", ""]
    for title, rows in _SUMMARY:
        out += [f"## {title}", "", *_table(("metric", "value"), ((label, cell(report)) for label, cell in rows))]
    if "routing" in report:
        out += ["### Per layer", "", *_table(_PER_LAYER, (_layer_cells(i, layer) for i, layer in
                                                          enumerate(report["routing"]["per_layer"])))]
        compute = report["expert_compute"]
        out += [f"MoE layers spent {compute['moe_seconds_total']:.3f}s across experts "
                f"({(compute['moe_share_of_forward'] or 0):.0%} of the profiled pass).", ""]
    if "training_stability" in report:
        out += ["## Training stability", "", *_table(("metric", "value"), report["training_stability"].items())]
    return "\n".join(out)


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    report = run_benchmark(args)
    print(json.dumps(report, indent=2))
    if args.output:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(report, indent=2) + "\n")
        md = args.output.with_suffix(".md")
        md.write_text(render_markdown(report))
        print(f"wrote benchmark report to {args.output} and {md}")


if __name__ == "__main__":
    main()
