"""Hardware detection, precision choice, exact parameter counts and safe-configuration helpers.

Parity with the reference ``src/hardware.py``: ``DeviceInfo``/``detect`` (:21-78), ``choose_precision`` (:80),
``parameter_counts`` from a meta-device model (:95), ``training_state_bytes`` (:111), ``suggest_num_experts``
(:116), ``auto_architecture`` (:183-240), ``find_safe_batch_size`` (:277-347) and ``recommend`` (:350-392).

Differences: ``training_state_bytes`` accounts for this framework's GPU layout (bf16 weights + fp32 master +
bf16 grads + fp32 moments = 16 B/parameter, the same total as the reference's fp32 layout), and the auto-architecture
anchors are this module's own table.
"""

from __future__ import annotations

import argparse
import json
import math
import time
from dataclasses import asdict, dataclass
from typing import Callable, Optional

import torch

from ..config import QuantaWeaveConfig


@dataclass
class DeviceInfo:
    backend: str
    name: str
    count: int
    total_memory_bytes: int
    free_memory_bytes: int
    bf16: bool
    fp16: bool
    runtime: str
    compute_capability: Optional[str] = None

    @property
    def torch_device(self) -> torch.device:
        return torch.device("cuda" if self.backend in {"cuda", "rocm"} else self.backend)


def _host_memory() -> tuple[int, int]:
    try:
        import psutil

        vm = psutil.virtual_memory()
        return vm.total, vm.available
    except ImportError:
        return 0, 0


def detect(requested: str = "auto") -> DeviceInfo:
    if requested == "rocm":
        requested = "cuda"
    if requested in {"auto", "cuda"} and torch.cuda.is_available():
        free, total = torch.cuda.mem_get_info()
        major, minor = torch.cuda.get_device_capability(0)
        return DeviceInfo("cuda", torch.cuda.get_device_name(0), torch.cuda.device_count(), total, free,
                          torch.cuda.is_bf16_supported(), True, f"cuda {torch.version.cuda}", f"{major}.{minor}")
    if requested in {"cuda", "xpu"}:
        raise RuntimeError(f"{requested} was requested but is not available")
    total, free = _host_memory()
    return DeviceInfo("cpu", "cpu", 1, total, free, True, False, f"torch {torch.__version__}")


def choose_precision(info: DeviceInfo, preferred: str = "auto") -> str:
    if preferred == "auto":
        return "fp32" if info.backend == "cpu" else ("bf16" if info.bf16 else "fp16")
    if preferred not in {"bf16", "fp16", "fp32"}:
        raise ValueError("precision must be auto, bf16, fp16 or fp32")
    if preferred == "bf16" and not info.bf16:
        raise ValueError(f"{info.name} does not support bf16")
    if preferred == "fp16" and info.backend == "cpu":
        raise ValueError("fp16 autocast is not supported on CPU; use bf16 or fp32")
    return preferred


def parameter_counts(config: QuantaWeaveConfig) -> dict[str, int]:
    """Exact counts from a meta-device model (no memory is allocated)."""
    from ..models.model import QuantaWeaveMoEForCausalLM

    with torch.device("meta"):
        model = QuantaWeaveMoEForCausalLM(config)
    total = sum(p.numel() for p in model.parameters())
    per_expert = 3 * config.hidden_size * config.ffn_size
    experts = config.layers * config.num_experts * per_expert
    return {"total": total, "experts": experts, "shared": total - experts,
            "active": total - config.layers * (config.num_experts - config.top_k) * per_expert,
            "per_expert": per_expert}


def training_state_bytes(config: QuantaWeaveConfig) -> int:
    return parameter_counts(config)["total"] * 16


def suggest_num_experts(info: DeviceInfo, hidden_size: int, ffn_size: int, layers: int, top_k: int, vocab_size: int,
                        sequence_length: int, memory_fraction: float = 0.5, cap: int = 256) -> int:
    budget = info.total_memory_bytes * memory_fraction
    per_expert = 3 * hidden_size * ffn_size * layers * 16
    shared = (2 * vocab_size * hidden_size + layers * 4 * hidden_size * hidden_size) * 16
    best = top_k
    for experts in range(top_k, cap + 1):
        if shared + experts * per_expert <= budget:
            best = experts
        else:
            break
    del sequence_length
    return best


# (parameter budget, hidden, layers, ffn multiplier x10, heads) anchors, interpolated in log-budget space
_SHAPE_ANCHORS = (
    (2e6, 64, 2, 20, 4),
    (2e7, 256, 4, 20, 4),
    (2e8, 512, 8, 24, 8),
    (2e9, 1024, 16, 27, 16),
    (2e10, 2048, 24, 27, 16),
    (2e11, 4096, 32, 35, 32),
)


def _interpolate_shape(budget: float) -> tuple[int, int, int, int]:
    pts = _SHAPE_ANCHORS
    if budget <= pts[0][0]:
        _, h, l, f, a = pts[0]
        return h, l, h * f // 10, a
    for lo, hi in zip(pts, pts[1:]):
        if budget <= hi[0]:
            t = (math.log(budget) - math.log(lo[0])) / (math.log(hi[0]) - math.log(lo[0]))
            h = int(round((lo[1] + t * (hi[1] - lo[1])) / 64) * 64) or 64
            layers = max(1, int(round(lo[2] + t * (hi[2] - lo[2]))))
            fm = lo[3] + t * (hi[3] - lo[3])
            heads = lo[4] if t < 0.5 else hi[4]
            while h % heads:
                heads //= 2
            return h, layers, int(round(h * fm / 10 / 64) * 64) or 64, max(1, heads)
    _, h, l, f, a = pts[-1]
    return h, l, h * f // 10, a


def auto_architecture(info: DeviceInfo, vocab_size: int, memory_fraction: float = 0.45, quality: str = "balanced") -> dict:
    """Pick a shape whose training state fills about ``memory_fraction`` of device memory."""
    if quality not in {"capacity", "balanced", "dense"}:
        raise ValueError("quality must be capacity, balanced or dense")
    budget_bytes = max(info.total_memory_bytes, 1 << 30) * memory_fraction
    params = budget_bytes / 16
    experts, active = {"capacity": (64, 2), "balanced": (16, 2), "dense": (1, 1)}[quality]
    dense_equiv = params / max(1.0, experts / 4)
    hidden, layers, ffn, heads = _interpolate_shape(dense_equiv)
    config = QuantaWeaveConfig(vocab_size=vocab_size, hidden_size=hidden, layers=layers, ffn_size=ffn,
                               num_experts=experts, top_k=active, attention_heads=heads)
    while training_state_bytes(config) > budget_bytes and config.num_experts > active:
        config.num_experts = max(active, config.num_experts // 2)
    seq = 256 if hidden <= 256 else 512 if hidden <= 1024 else 2048
    return {"hidden_size": hidden, "layers": layers, "ffn_size": ffn, "attention_heads": heads,
            "total_experts": config.num_experts, "active_experts": active, "sequence_length": seq,
            "training_state_fraction_of_budget": training_state_bytes(config) / budget_bytes}


def _is_oom(error: BaseException) -> bool:
    return isinstance(error, torch.OutOfMemoryError) or "out of memory" in str(error).lower()


def find_safe_batch_size(model, device: torch.device, sequence_length: int, autocast: Callable = None,
                         start: int = 1, limit: int = 4096, memory_fraction: float = 0.85, target: float = 0.95,
                         steps: int = 2, peak_fn: Optional[Callable] = None, clock: Callable = time.perf_counter) -> dict:
    """Double the batch with real forward/backward steps (optimizer moments reserved) until OOM or
    ``memory_fraction`` of device memory; return the smallest batch reaching ``target`` of the best throughput."""
    import contextlib

    autocast = autocast or contextlib.nullcontext
    vocab = model.config.vocab_size
    total = torch.cuda.get_device_properties(device).total_memory if device.type == "cuda" else None
    results = []
    batch = start
    reserve = [torch.zeros_like(p, dtype=torch.float32) for p in model.parameters()] if device.type == "cuda" else []
    try:
        while batch <= limit:
            try:
                if device.type == "cuda":
                    torch.cuda.reset_peak_memory_stats(device)
                ids = torch.randint(0, vocab, (batch, sequence_length + 1), device=device)
                began = None
                for i in range(steps):
                    if i == 1:
                        if device.type == "cuda":
                            torch.cuda.synchronize(device)
                        began = clock()
                    with autocast():
                        loss = model(ids, labels=ids, return_logits=False)["loss"]
                    loss.backward()
                    model.zero_grad(set_to_none=True)
                if device.type == "cuda":
                    torch.cuda.synchronize(device)
                elapsed = max(clock() - (began or clock()), 1e-9)
                peak = peak_fn() if peak_fn else (torch.cuda.max_memory_allocated(device) if device.type == "cuda" else 0)
                results.append({"batch_size": batch, "tokens_per_second": batch * sequence_length * max(1, steps - 1) / elapsed,
                                "peak_memory_bytes": peak})
                if total and peak > memory_fraction * total:
                    break
                batch *= 2
            except Exception as error:  # noqa: BLE001
                if not _is_oom(error):
                    raise
                model.zero_grad(set_to_none=True)
                if device.type == "cuda":
                    torch.cuda.empty_cache()
                break
    finally:
        del reserve
    if not results:
        raise RuntimeError("even the smallest batch does not fit on this device")
    best = max(r["tokens_per_second"] for r in results)
    chosen = next(r for r in results if r["tokens_per_second"] >= target * best) if target > 0 else results[-1]
    return {"batch_size": results[-1]["batch_size"], "recommended_batch_size": chosen["batch_size"],
            "tokens_per_second": chosen["tokens_per_second"], "largest_peak_memory_bytes": results[-1]["peak_memory_bytes"],
            "probes": results}


def recommend(info: DeviceInfo, config: QuantaWeaveConfig, sequence_length: int, probe: bool = False,
              preferred_precision: str = "auto") -> dict:
    counts = parameter_counts(config)
    state = counts["total"] * 16
    out = {"device": asdict(info), "precision": choose_precision(info, preferred_precision), "parameters": counts,
           "training_state_bytes": state,
           "fits": info.total_memory_bytes == 0 or state < 0.9 * info.total_memory_bytes,
           "activation_checkpointing": False}
    if probe and info.backend != "cpu":
        from ..models.model import QuantaWeaveMoEForCausalLM

        model = QuantaWeaveMoEForCausalLM(config).to(info.torch_device)
        out["probe"] = find_safe_batch_size(model, info.torch_device, sequence_length)
    return out


def main(argv=None) -> None:
    """CLI with the reference's flags (``src/hardware.py:395-430``): describe the device, optionally pick the shape
    with ``--auto-architecture`` (``--quality``, ``--memory-fraction``), report precision, parameter counts, memory
    fit and a suggested expert count, and with ``--probe`` run real passes to find a safe batch size."""
    parser = argparse.ArgumentParser(description="Describe this machine and size a QuantaWeave model for it")
    parser.add_argument("--device", default="auto", choices=("auto", "cuda", "rocm", "xpu", "cpu"))
    parser.add_argument("--probe", action="store_true", help="run real passes to find a safe batch size")
    parser.add_argument("--auto-architecture", action="store_true",
                        help="pick hidden size, layers, experts and sequence length for this device")
    parser.add_argument("--quality", default="balanced", choices=("capacity", "balanced", "dense"),
                        help="--auto-architecture: favour stored capacity, a balance, or a dense (single-expert) model")
    parser.add_argument("--memory-fraction", type=float, default=0.45,
                        help="--auto-architecture: share of device memory to target")
    parser.add_argument("--precision", default="auto", choices=("auto", "bf16", "fp16", "fp32"))
    parser.add_argument("--hidden-size", type=int, default=256)
    parser.add_argument("--layers", type=int, default=4)
    parser.add_argument("--ffn-size", type=int, default=512)
    parser.add_argument("--total-experts", type=int, default=16)
    parser.add_argument("--active-experts", type=int, default=2)
    parser.add_argument("--attention-heads", type=int, default=4)
    parser.add_argument("--vocab-size", type=int, default=7168)
    parser.add_argument("--sequence-length", type=int, default=128)
    args = parser.parse_args(argv)
    info = detect(args.device)
    if args.auto_architecture:
        shape = auto_architecture(info, args.vocab_size, args.memory_fraction, args.quality)
        args.hidden_size, args.layers, args.ffn_size = shape["hidden_size"], shape["layers"], shape["ffn_size"]
        args.total_experts, args.active_experts = shape["total_experts"], shape["active_experts"]
        args.sequence_length = shape["sequence_length"]
        args.attention_heads = shape.get("attention_heads", args.attention_heads)
    config = QuantaWeaveConfig(vocab_size=args.vocab_size, hidden_size=args.hidden_size, layers=args.layers,
                               ffn_size=args.ffn_size, num_experts=args.total_experts, top_k=args.active_experts,
                               attention_heads=args.attention_heads, max_sequence_length=args.sequence_length + 1)
    report = recommend(info, config, args.sequence_length, args.probe, preferred_precision=args.precision)
    report["suggested_num_experts"] = suggest_num_experts(info, args.hidden_size, args.ffn_size, args.layers,
                                                          args.active_experts, args.vocab_size, args.sequence_length)
    report["shape"] = {"hidden_size": args.hidden_size, "layers": args.layers, "ffn_size": args.ffn_size,
                       "total_experts": args.total_experts, "active_experts": args.active_experts,
                       "sequence_length": args.sequence_length, "attention_heads": args.attention_heads}
    print(json.dumps(report, indent=2, default=str))


if __name__ == "__main__":
    main()
