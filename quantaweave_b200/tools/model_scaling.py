"""Architecture calculator: dense and sparse-MoE specs from size presets, parameter estimates and a manifest.

Parity with the reference ``src/model_scaling.py`` (``ModelSpec`` :13-84, ``make_spec`` :88-104, CLI :111-158) and
its preset table ``configs/architecture_presets.json`` (xs ... xxl; the same numbers, shipped as package data in
``quantaweave_b200/configs/architecture_presets.json``). Parameter estimates: embeddings ``(1 or 2) * V * H``,
attention ``4 * H^2`` per layer, experts ``3 * H * F`` each (SwiGLU), ``F = round(H * ffn_multiplier)``.

B200 addition: ``b200_plan`` sizes a training job for 180 GB HBM3e per GPU: bf16 weights + fp32 master + two fp32
AdamW moments (14 bytes per parameter) plus an activation reserve, the smallest expert-parallel degree (a divisor of
the expert count, at most 8 GPUs of one NVSwitch node) whose per-GPU share fits, and the per-token FLOPs.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

PRESETS_PATH = Path(__file__).resolve().parent.parent / "configs" / "architecture_presets.json"
B200_HBM_BYTES = 180e9
TRAIN_BYTES_PER_PARAM = 2 + 4 + 4 + 4  # bf16 weight, fp32 master, two fp32 moments


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

    @property
    def ffn_size(self) -> int:
        return round(self.hidden_size * self.ffn_multiplier)

    @property
    def experts(self) -> int:
        return self.num_experts if self.mode == "moe" else 1

    @property
    def active_experts(self) -> int:
        return self.top_k if self.mode == "moe" else 1

    @property
    def embedding_params(self) -> int:
        return (1 if self.tied_embeddings else 2) * self.vocab_size * self.hidden_size

    @property
    def attention_params(self) -> int:
        return self.layers * 4 * self.hidden_size ** 2

    @property
    def expert_params(self) -> int:
        return self.layers * self.experts * 3 * self.hidden_size * self.ffn_size

    @property
    def active_expert_params(self) -> int:
        return self.layers * self.active_experts * 3 * self.hidden_size * self.ffn_size

    @property
    def total_params(self) -> int:
        return self.embedding_params + self.attention_params + self.expert_params

    @property
    def active_params(self) -> int:
        return self.embedding_params + self.attention_params + self.active_expert_params

    def manifest(self) -> dict:
        return {
            "model_name": f"QuantaWeave-{self.mode}-{self.size}",
            "model_type": f"quantweave_{self.mode}",
            "mode": self.mode, "size": self.size, "hidden_size": self.hidden_size, "layers": self.layers,
            "ffn_size": self.ffn_size, "vocab_size": self.vocab_size, "tied_embeddings": self.tied_embeddings,
            "num_experts": self.experts, "top_k": self.active_experts,
            "inactive_experts_per_token": max(0, self.experts - self.active_experts),
            "active_expert_fraction": self.active_experts / self.experts,
            "capacity_factor": self.capacity_factor, "min_expert_capacity": self.min_expert_capacity,
            "estimated_total_params": self.total_params, "estimated_active_params": self.active_params,
        }


def b200_plan(spec: ModelSpec, sequence_length: int = 2048, tokens_per_gpu: int = 16384,
              activation_bytes_per_token_layer: Optional[int] = None) -> dict:
    """Smallest expert-parallel degree (<= 8, dividing the expert count) whose per-GPU training state fits."""
    shared = spec.total_params - spec.expert_params
    act = activation_bytes_per_token_layer or 24 * spec.hidden_size  # bf16 activations kept for backward
    reserve = tokens_per_gpu * spec.layers * act
    plan = None
    for ep in (1, 2, 4, 8):
        if spec.experts % ep:
            continue
        state = (shared + spec.expert_params / ep) * TRAIN_BYTES_PER_PARAM
        if state + reserve <= 0.9 * B200_HBM_BYTES:
            plan = ep
            break
    flops_per_token = 6 * spec.active_params + 12 * spec.layers * spec.hidden_size * sequence_length
    return {"expert_parallel": plan, "fits_on_one_node": plan is not None,
            "bytes_per_gpu_at_plan": None if plan is None else
            (shared + spec.expert_params / plan) * TRAIN_BYTES_PER_PARAM + reserve,
            "activation_reserve_bytes": reserve, "train_flops_per_token": flops_per_token}


def load_presets() -> dict:
    return json.loads(PRESETS_PATH.read_text())


def make_spec(mode: str, size: str, **overrides) -> ModelSpec:
    presets = load_presets()
    if size not in presets:
        raise ValueError(f"Unknown size '{size}'. Choose from: {', '.join(presets)}")
    if mode not in {"dense", "moe"}:
        raise ValueError("mode must be 'dense' or 'moe'")
    values = {**presets[size], **{k: v for k, v in overrides.items() if v is not None}, "mode": mode, "size": size}
    if mode == "dense":
        values.update(num_experts=1, top_k=1)
    if values["top_k"] > values["num_experts"]:
        raise ValueError("active experts (top_k) cannot exceed total experts")
    return ModelSpec(**values)


def billions(value: int) -> float:
    return value / 1e9


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Build a QuantaWeave architecture manifest")
    p.add_argument("--mode", choices=("dense", "moe"), default="moe")
    p.add_argument("--size", choices=tuple(load_presets()), default="m")
    p.add_argument("--output", type=Path)
    p.add_argument("--hidden-size", type=int)
    p.add_argument("--layers", type=int)
    p.add_argument("--num-experts", type=int)
    p.add_argument("--top-k", type=int)
    p.add_argument("--total-experts", dest="num_experts", type=int, help="alias for --num-experts")
    p.add_argument("--active-experts", dest="top_k", type=int, help="alias for --top-k")
    p.add_argument("--vocab-size", type=int)
    p.add_argument("--ffn-multiplier", type=float)
    p.add_argument("--tied-embeddings", action=argparse.BooleanOptionalAction, default=None)
    p.add_argument("--capacity-factor", type=float, default=1.25)
    p.add_argument("--min-expert-capacity", type=int, default=4)
    p.add_argument("--b200-plan", action="store_true", help="add the per-B200 memory / expert-parallel plan")
    from .common import describe_options

    describe_options(p, {'mode': 'dense or mixture-of-experts architecture', 'size': 'preset size from the architecture table', 'output': 'write the manifest JSON here', 'num_experts': 'experts per MoE layer (overrides the preset)', 'top_k': 'experts per token (overrides the preset)', 'ffn_multiplier': 'FFN width as a multiple of the model width', 'tied_embeddings': 'share the input embedding with the LM head'})
    args = p.parse_args(argv)
    try:
        spec = make_spec(args.mode, args.size, hidden_size=args.hidden_size, layers=args.layers,
                         num_experts=args.num_experts, top_k=args.top_k, vocab_size=args.vocab_size,
                         ffn_multiplier=args.ffn_multiplier, tied_embeddings=args.tied_embeddings,
                         capacity_factor=args.capacity_factor, min_expert_capacity=args.min_expert_capacity)
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
