"""Architecture calculator: dense and sparse-MoE specs from size presets, parameter estimates and a manifest.

The public names (``ModelSpec``, ``make_spec``, ``load_presets``, ``billions``, ``main``), the CLI flags, the preset
table and the manifest keys are those of the reference ``src/model_scaling.py`` (:13-158) and its
``configs/architecture_presets.json`` (xs ... xxl; the same numbers, shipped as package data), because sweep files
and manifests written for the reference must keep working.

Estimates are computed from one breakdown (:class:`ParameterBudget`): embeddings ``(1 or 2) * V * H`` (tied or
separate input and output tables), attention ``4 * H^2`` per layer, and ``3 * H * F`` per SwiGLU expert with
``F = round(H * ffn_multiplier)``. A dense model is the one-expert, top-1 case.

B200 addition: :func:`b200_plan` sizes a training job for 180 GB of HBM3e per GPU: bf16 weights + fp32 master + two
fp32 AdamW moments (14 bytes per parameter) plus an activation reserve, the smallest expert-parallel degree (a
divisor of the expert count, at most the 8 GPUs of one NVSwitch node) whose per-GPU share fits, and the training
FLOPs per token.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass
from pathlib import Path
from typing import NamedTuple, Optional

PRESETS_PATH = Path(__file__).resolve().parent.parent / "configs" / "architecture_presets.json"
B200_HBM_BYTES = 180e9
TRAIN_BYTES_PER_PARAM = 2 + 4 + 4 + 4  # bf16 weight, fp32 master, two fp32 moments
MODES = ("dense", "moe")


class ParameterBudget(NamedTuple):
    """Parameter counts of one architecture, by part."""

    embeddings: int
    attention: int
    experts_total: int   # every expert of every layer
    experts_active: int  # the experts one token runs through, over all layers

    @property
    def total(self) -> int:
        return self.embeddings + self.attention + self.experts_total

    @property
    def active(self) -> int:
        return self.embeddings + self.attention + self.experts_active


@dataclass(frozen=True)
class ModelSpec:
    mode: str
    size: str
    hidden_size: int
    layers: int
    num_experts: int
    top_k: int
    vocab_size: int
    ffn_multiplier: float
    tied_embeddings: bool
    capacity_factor: float = 1.25
    min_expert_capacity: int = 4

    # ---- shape ----
    @property
    def ffn_size(self) -> int:
        return round(self.hidden_size * self.ffn_multiplier)

    @property
    def experts(self) -> int:
        """Experts per layer as built (a dense model has one FFN)."""
        return self.num_experts if self.mode == "moe" else 1

    @property
    def active_experts(self) -> int:
        return self.top_k if self.mode == "moe" else 1

    # ---- parameter counts ----
    def budget(self) -> ParameterBudget:
        h = self.hidden_size
        per_expert = 3 * h * self.ffn_size  # gate, up and down projections
        return ParameterBudget(embeddings=(1 if self.tied_embeddings else 2) * self.vocab_size * h,
                               attention=self.layers * 4 * h * h,
                               experts_total=self.layers * self.experts * per_expert,
                               experts_active=self.layers * self.active_experts * per_expert)

    embedding_params = property(lambda self: self.budget().embeddings)
    attention_params = property(lambda self: self.budget().attention)
    expert_params = property(lambda self: self.budget().experts_total)
    active_expert_params = property(lambda self: self.budget().experts_active)
    total_params = property(lambda self: self.budget().total)
    active_params = property(lambda self: self.budget().active)

    def manifest(self) -> dict:
        budget = self.budget()
        identity = {"model_name": f"QuantaWeave-{self.mode}-{self.size}", "model_type": f"quantweave_{self.mode}",
                    "mode": self.mode, "size": self.size}
        shape = {key: getattr(self, key) for key in ("hidden_size", "layers", "ffn_size", "vocab_size",
                                                    "tied_embeddings")}
        routing = {"num_experts": self.experts, "top_k": self.active_experts,
                   "inactive_experts_per_token": max(0, self.experts - self.active_experts),
                   "active_expert_fraction": self.active_experts / self.experts,
                   "capacity_factor": self.capacity_factor, "min_expert_capacity": self.min_expert_capacity}
        return {**identity, **shape, **routing, "estimated_total_params": budget.total,
                "estimated_active_params": budget.active}


def b200_plan(spec: ModelSpec, sequence_length: int = 2048, tokens_per_gpu: int = 16384,
              activation_bytes_per_token_layer: Optional[int] = None) -> dict:
    """Smallest expert-parallel degree (<= 8, dividing the expert count) whose per-GPU training state fits."""
    budget = spec.budget()
    replicated = budget.total - budget.experts_total
    per_token_layer = activation_bytes_per_token_layer or 24 * spec.hidden_size  # bf16 activations for backward
    reserve = tokens_per_gpu * spec.layers * per_token_layer

    def per_gpu(ep: int) -> float:
        return (replicated + budget.experts_total / ep) * TRAIN_BYTES_PER_PARAM + reserve

    fitting = [ep for ep in (1, 2, 4, 8) if spec.experts % ep == 0 and per_gpu(ep) <= 0.9 * B200_HBM_BYTES]
    plan = fitting[0] if fitting else None
    return {"expert_parallel": plan, "fits_on_one_node": plan is not None,
            "bytes_per_gpu_at_plan": None if plan is None else per_gpu(plan),
            "activation_reserve_bytes": reserve,
            "train_flops_per_token": 6 * budget.active + 12 * spec.layers * spec.hidden_size * sequence_length}


def load_presets() -> dict:
    return json.loads(PRESETS_PATH.read_text())


def make_spec(mode: str, size: str, **overrides) -> ModelSpec:
    """The preset ``size`` with any non-None ``overrides`` applied; ``mode`` "dense" forces one expert, top-1."""
    presets = load_presets()
    if size not in presets:
        raise ValueError(f"Unknown size '{size}'. Choose from: {', '.join(presets)}")
    if mode not in MODES:
        raise ValueError("mode must be 'dense' or 'moe'")
    values = dict(presets[size])
    values.update((key, value) for key, value in overrides.items() if value is not None)
    if mode == "dense":
        values["num_experts"] = values["top_k"] = 1
    if values["top_k"] > values["num_experts"]:
        raise ValueError("active experts (top_k) cannot exceed total experts")
    return ModelSpec(mode=mode, size=size, **values)


def billions(value: int) -> float:
    return value / 1e9


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Build a QuantaWeave architecture manifest")
    p.add_argument("--mode", choices=MODES, default="moe")
    p.add_argument("--size", choices=tuple(load_presets()), default="m")
    p.add_argument("--output", type=Path)
    for flag, kind in (("--hidden-size", int), ("--layers", int), ("--num-experts", int), ("--top-k", int)):
        p.add_argument(flag, type=kind)
    p.add_argument("--total-experts", dest="num_experts", type=int, help="alias for --num-experts")
    p.add_argument("--active-experts", dest="top_k", type=int, help="alias for --top-k")
    p.add_argument("--vocab-size", type=int)
    p.add_argument("--ffn-multiplier", type=float)
    p.add_argument("--tied-embeddings", action=argparse.BooleanOptionalAction, default=None)
    p.add_argument("--capacity-factor", type=float, default=1.25)
    p.add_argument("--min-expert-capacity", type=int, default=4)
    p.add_argument("--b200-plan", action="store_true", help="add the per-B200 memory / expert-parallel plan")
    from .common import describe_options

    describe_options(p, {"mode": "dense or mixture-of-experts architecture",
                         "size": "preset size from the architecture table", "output": "write the manifest JSON here",
                         "num_experts": "experts per MoE layer (overrides the preset)",
                         "top_k": "experts per token (overrides the preset)",
                         "ffn_multiplier": "FFN width as a multiple of the model width",
                         "tied_embeddings": "share the input embedding with the LM head"})
    return p


def main(argv=None) -> None:
    p = build_parser()
    args = p.parse_args(argv)
    shape_options = ("hidden_size", "layers", "num_experts", "top_k", "vocab_size", "ffn_multiplier",
                     "tied_embeddings", "capacity_factor", "min_expert_capacity")
    try:
        spec = make_spec(args.mode, args.size, **{name: getattr(args, name) for name in shape_options})
    except ValueError as error:
        p.error(str(error))
    manifest = spec.manifest()
    if args.b200_plan:
        manifest["b200_plan"] = b200_plan(spec)
    print(f"{manifest['model_name']}: total={billions(spec.total_params):.2f}B, "
          f"active/token={billions(spec.active_params):.2f}B")
    if args.output:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(manifest, indent=2) + "\n")
        print(f"wrote {args.output}")


if __name__ == "__main__":
    main()
