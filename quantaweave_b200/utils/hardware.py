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


# Depth and FFN width as functions of the model width: (hidden, layers, ffn multiplier), interpolated in log(hidden).
_WIDTH_ANCHORS = ((64, 2, 2.0), (256, 4, 2.0), (512, 8, 2.5), (1024, 16, 2.75), (2048, 24, 2.75), (4096, 32, 3.5),
                  (8192, 48, 3.5))
# quality -> (starting expert count, routed experts per token)
_QUALITIES = {"capacity": (64, 1), "balanced": (16, 2), "dense": (1, 1)}
_MAX_EXPERTS = 256
_MAX_WIDTH = 16384


def _depth_and_ffn(hidden: int) -> tuple[int, int]:
    pts = _WIDTH_ANCHORS
    if hidden <= pts[0][0]:
        layers, mult = pts[0][1], pts[0][2]
    elif hidden >= pts[-1][0]:
        layers, mult = pts[-1][1], pts[-1][2]
    else:
        lo, hi = next((a, b) for a, b in zip(pts, pts[1:]) if hidden <= b[0])
        t = (math.log(hidden) - math.log(lo[0])) / (math.log(hi[0]) - math.log(lo[0]))
        layers, mult = round(lo[1] + t * (hi[1] - lo[1])), lo[2] + t * (hi[2] - lo[2])
    return max(1, int(layers)), max(64, int(round(hidden * mult / 64)) * 64)


def _sequence_length(hidden: int) -> int:
    return 256 if hidden <= 256 else 512 if hidden <= 1024 else 2048


def _linear_counts(vocab: int, hidden: int, ffn: int, seq: int) -> tuple[int, int, int]:
    """(fixed, per layer with one expert, per extra expert per layer) parameter counts, read off three meta-device
    builds: the model's size is affine in the layer count and, per layer, in the expert count."""
    def total(layers: int, experts: int) -> int:
        return parameter_counts(QuantaWeaveConfig(vocab_size=vocab, hidden_size=hidden, layers=layers, ffn_size=ffn,
                                                  num_experts=experts, top_k=1, attention_heads=max(1, hidden // 64),
                                                  max_sequence_length=seq + 1))["total"]

    one = total(1, 1)
    per_layer = total(2, 1) - one
    per_expert = total(1, 2) - one
    return one - per_layer, per_layer, per_expert


def auto_architecture(info: DeviceInfo, vocab_size: int = 7168, memory_fraction: float = 0.45,
                      quality: str = "balanced") -> dict:
    """The largest model whose training state (16 B per parameter) fits ``memory_fraction`` of the device.

    Width sets depth and FFN width (``_WIDTH_ANCHORS``); the widest shape that fits with the quality's starting
    expert count is taken, then the rest of the budget is filled: ``capacity`` and ``balanced`` add experts (up to
    256), ``dense`` widens its single FFN. ``capacity`` routes each token to one of many experts (most parameters,
    fewest active), ``balanced`` to two of a moderate pool, ``dense`` is a plain transformer. A budget below the
    smallest shape still returns that shape when it fits the device; one that fits no device memory at all raises."""
    if quality not in _QUALITIES:
        raise ValueError("quality must be capacity, balanced or dense")
    if not 0 < memory_fraction <= 1:
        raise ValueError("memory_fraction must be in (0, 1]")
    if info.total_memory_bytes <= 0:
        raise ValueError("the device's memory size is unknown; auto-architecture needs it")
    budget = info.total_memory_bytes * memory_fraction
    start_experts, active = _QUALITIES[quality]

    def shape(hidden: int) -> dict:
        layers, ffn = _depth_and_ffn(hidden)
        seq = _sequence_length(hidden)
        fixed, per_layer, per_expert = _linear_counts(vocab_size, hidden, ffn, seq)
        return dict(hidden=hidden, layers=layers, ffn=ffn, seq=seq, fixed=fixed, per_layer=per_layer,
                    per_expert=per_expert)

    def state(sh: dict, experts: int, ffn_extra: int = 0) -> int:
        params = sh["fixed"] + sh["layers"] * (sh["per_layer"] + (experts - 1) * sh["per_expert"])
        params += sh["layers"] * experts * 3 * sh["hidden"] * ffn_extra
        return params * 16

    lo, hi = 1, _MAX_WIDTH // 64  # widths are multiples of 64 (one 64-wide head each)
    best = shape(64)
    if state(best, start_experts) > 0.9 * info.total_memory_bytes:
        raise ValueError(f"no architecture fits this device: even hidden 64 needs {state(best, start_experts):,} "
                         f"bytes of training state, {info.total_memory_bytes:,} available")
    while lo < hi:  # training state grows with width: the widest shape within the budget
        mid = (lo + hi + 1) // 2
        candidate = shape(64 * mid)
        if state(candidate, start_experts) <= budget:
            lo, best = mid, candidate
        else:
            hi = mid - 1
    experts, extra = start_experts, 0
    if quality == "dense":
        while extra < 8 * best["hidden"] and state(best, 1, extra + 64) <= budget:
            extra += 64
    else:
        while experts < _MAX_EXPERTS and state(best, experts + 1) <= budget:
            experts += 1
    hidden, ffn = best["hidden"], best["ffn"] + extra
    config = QuantaWeaveConfig(vocab_size=vocab_size, hidden_size=hidden, layers=best["layers"], ffn_size=ffn,
                               num_experts=experts, top_k=active, attention_heads=max(1, hidden // 64),
                               max_sequence_length=best["seq"] + 1)
    counts = parameter_counts(config)
    state_bytes = counts["total"] * 16
    return {"quality": quality, "memory_fraction": memory_fraction, "vocab_size": vocab_size, "hidden_size": hidden,
            "layers": config.layers, "ffn_size": ffn, "attention_heads": config.attention_heads,
            "total_experts": experts, "active_experts": active, "sequence_length": best["seq"],
            "total_parameters": counts["total"], "active_parameters": counts["active"],
            "training_state_bytes": state_bytes, "training_state_fraction_of_budget": state_bytes / budget}


def _is_oom(error: BaseException) -> bool:
    return isinstance(error, torch.OutOfMemoryError) or "out of memory" in str(error).lower()


def _peak_bytes(device: torch.device) -> Optional[int]:
    """Peak device memory since the last reset; on the host, the process's resident set (None without psutil)."""
    if device.type == "cuda":
        return torch.cuda.max_memory_allocated(device)
    try:
        import psutil

        return psutil.Process().memory_info().rss
    except ImportError:
        return None


def _reset_peak(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)


def find_safe_batch_size(model, device: torch.device, sequence_length: int, autocast: Callable = None,
                         start: int = 1, limit: int = 256, headroom: float = 0.85, target: float = 0.95,
                         optimizer_state_copies: int = 2,
                         steps: int = 2, total_memory: Optional[int] = None, peak_fn: Optional[Callable] = None,
                         clock: Callable = time.perf_counter) -> dict:
    """Double the batch with real forward/backward/clip steps until a step runs out of memory or its peak passes
    ``headroom`` of ``total_memory`` (default: the device's, host memory on CPU).

    The optimizer's state is held for the whole search, so an approved batch still fits once training starts:
    ``optimizer_state_copies`` fp32 copies per trainable parameter (2: the AdamW moments), plus an fp32 master copy
    of every low-precision one. Weights are never
    stepped; gradients are cleared and the module's train/eval mode is restored. Any error other than running out of
    memory propagates. Returns the largest batch that fitted (``batch_size``), the smallest batch whose throughput is
    within ``target`` of the best (``recommended_batch_size``; ``target=0`` picks the largest) and the measured
    ``curve`` of ``{batch_size, tokens_per_second, peak_memory_bytes}``."""
    import contextlib

    autocast = autocast or contextlib.nullcontext
    peak_fn = peak_fn or (lambda: _peak_bytes(device))
    vocab = model.config.vocab_size
    if total_memory is None:
        total_memory = (torch.cuda.get_device_properties(device).total_memory if device.type == "cuda"
                        else _host_memory()[0])
    trainable = [p for p in model.parameters() if p.requires_grad]
    reserve = [torch.zeros_like(p, dtype=torch.float32) for p in trainable for _ in range(optimizer_state_copies)]
    reserve += [torch.zeros_like(p, dtype=torch.float32) for p in trainable if p.dtype != torch.float32]
    was_training = model.training
    model.train()
    curve = []
    batch = start
    try:
        while batch <= limit:
            try:
                _reset_peak(device)
                ids = torch.randint(0, vocab, (batch, sequence_length + 1), device=device)
                began = None
                for i in range(steps):
                    if i == min(1, steps - 1):
                        if device.type == "cuda":
                            torch.cuda.synchronize(device)
                        began = clock()
                    with autocast():
                        loss = model(ids, labels=ids, return_logits=False)["loss"]
                    loss.backward()
                    torch.nn.utils.clip_grad_norm_(trainable, 1.0)
                    model.zero_grad(set_to_none=True)
                if device.type == "cuda":
                    torch.cuda.synchronize(device)
                timed = steps - min(1, steps - 1)
                elapsed = max(clock() - began, 1e-9)
                peak = peak_fn()
                curve.append({"batch_size": batch, "tokens_per_second": batch * sequence_length * timed / elapsed,
                              "peak_memory_bytes": peak})
                if peak is not None and total_memory and peak > headroom * total_memory:
                    curve.pop()  # over the headroom limit: this batch is not safe
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
        model.zero_grad(set_to_none=True)
        model.train(was_training)
    if not curve:
        raise RuntimeError("even batch size 1 does not fit on this device")
    best = max(r["tokens_per_second"] for r in curve)
    chosen = next(r for r in curve if r["tokens_per_second"] >= target * best) if target > 0 else curve[-1]
    return {"batch_size": curve[-1]["batch_size"], "recommended_batch_size": chosen["batch_size"],
            "tokens_per_second": chosen["tokens_per_second"], "peak_memory_bytes": chosen["peak_memory_bytes"],
            "largest_peak_memory_bytes": curve[-1]["peak_memory_bytes"], "curve": curve, "headroom": headroom}


CHECKPOINTING_GAIN = 1.05  # recompute must buy at least 5 % more tokens/s (through a larger batch) to be recommended


def recommend(info: DeviceInfo, config: QuantaWeaveConfig, sequence_length: int, probe: bool = False,
              preferred_precision: str = "auto", autocast: Optional[Callable] = None) -> dict:
    """Precision, parameter counts and whether the training state fits; with ``probe`` (any device) also the batch
    probe run twice, without and with activation checkpointing. Checkpointing is recommended only when its best
    throughput beats the plain model's by ``CHECKPOINTING_GAIN``, or when the plain model does not fit at all; the
    recommended ``batch_size`` is that of the chosen setting."""
    counts = parameter_counts(config)
    state = counts["total"] * 16
    precision = choose_precision(info, preferred_precision)
    memory = info.total_memory_bytes
    out = {"device": asdict(info), "precision": precision, "parameters": counts, "training_state_bytes": state,
           "fits_training_state": memory == 0 or state < 0.8 * memory,
           "max_sequence_length": config.max_sequence_length - 1, "sequence_length": sequence_length,
           # without a measurement: recompute once the training state alone takes 40 % of the device
           "activation_checkpointing_recommended": bool(memory and state > 0.4 * memory)}
    if probe:
        from ..models.model import QuantaWeaveMoEForCausalLM

        device = info.torch_device
        if autocast is None:
            from ..training.trainer import autocast_context

            autocast = lambda: autocast_context(device, precision)  # noqa: E731
        total = memory or None
        results, errors = {}, {}
        for checkpointing in (False, True):
            model = QuantaWeaveMoEForCausalLM(config).to(device)
            model.activation_checkpointing = checkpointing
            try:
                results[checkpointing] = find_safe_batch_size(model, device, sequence_length, autocast,
                                                              total_memory=total)
            except RuntimeError as error:
                errors[checkpointing] = error
            del model
        if not results:
            raise errors[False]
        plain, recompute = results.get(False), results.get(True)
        use = recompute is not None and (plain is None or recompute["tokens_per_second"]
                                         > CHECKPOINTING_GAIN * plain["tokens_per_second"])
        chosen = recompute if use else plain
        out.update(activation_checkpointing_recommended=bool(use), batch_size=chosen["recommended_batch_size"],
                   tokens_per_second=chosen["tokens_per_second"], probe=chosen,
                   probe_without_checkpointing=plain, probe_with_checkpointing=recompute)
    return out


def main(argv=None) -> None:
    """CLI with the reference's flags (``src/hardware.py:395-430``): describe the device, optionally pick the shape
    with ``--auto-architecture`` (``--quality``, ``--memory-fraction``), report precision, parameter counts, memory
    fit and a suggested expert count, and with ``--probe`` run real passes to find a safe batch size."""
    parser = argparse.ArgumentParser(description="Describe this machine and size a QuantaWeave model for it")
    parser.add_argument("--device", default="auto", choices=("auto", "cuda", "rocm", "xpu", "cpu"))
    parser.add_argument("--probe", action="store_true", help="time real training steps to find the largest safe batch")
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
    from ..tools.common import describe_options

    describe_options(parser, {'sequence_length': 'tokens per training sequence', 'device': 'device to describe'})
    args = parser.parse_args(argv)
    info = detect(args.device)
    if args.auto_architecture:
        shape = auto_architecture(info, args.vocab_size, args.memory_fraction, args.quality)
        args.hidden_size, args.layers, args.ffn_size = shape["hidden_size"], shape["layers"], shape["ffn_size"]
        args.total_experts, args.active_experts = shape["total_experts"], shape["active_experts"]
        args.sequence_length = shape["sequence_length"]
        args.attention_heads = shape["attention_heads"]
    config = QuantaWeaveConfig(vocab_size=args.vocab_size, hidden_size=args.hidden_size, layers=args.layers,
                               ffn_size=args.ffn_size, num_experts=args.total_experts, top_k=args.active_experts,
                               attention_heads=args.attention_heads, max_sequence_length=args.sequence_length + 1)
    report = recommend(info, config, args.sequence_length, args.probe, preferred_precision=args.precision)
    report["suggested_num_experts"] = suggest_num_experts(info, args.hidden_size, args.ffn_size, args.layers,
                                                          args.active_experts, args.vocab_size, args.sequence_length)
    if args.auto_architecture:
        report["auto_architecture"] = shape
    report["shape"] = {"hidden_size": args.hidden_size, "layers": args.layers, "ffn_size": args.ffn_size,
                       "total_experts": args.total_experts, "active_experts": args.active_experts,
                       "sequence_length": args.sequence_length, "attention_heads": args.attention_heads}
    print(json.dumps(report, indent=2, default=str))


if __name__ == "__main__":
    main()
