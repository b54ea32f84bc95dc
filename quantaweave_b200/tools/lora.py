"""LoRA adapters over frozen (optionally quantised) expert weights: QLoRA for the MoE.

Behavioural parity with the reference ``src/lora.py`` (``LoRALinear`` :25-51, ``add_lora`` :54-85, adapter save/load
:88-104, ``merge_lora_state`` :107-117): every expert projection gets ``y = base(x) + (alpha/rank) * B(A(x))`` with A
Kaiming-uniform and B zero (the adapter starts as a no-op), the base is frozen, and routers/norms can be unfrozen.

B200 layout: the adapters of one MoE layer are stacked like its experts (``a_gate [E, r, H]``, ``b_gate [E, F, r]``,
``a_up``, ``b_up``, ``a_down [E, r, F]``, ``b_down [E, H, r]``) in one ``ExpertLoRA`` module attached as ``moe.lora``.
Saved adapters and merged state dicts use the reference's per-expert names
(``blocks.{l}.moe.experts.{e}.{gate,up,down}.lora_a / lora_b`` and ``...weight``), so files interchange.
"""

from __future__ import annotations

import math
import re
from pathlib import Path
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..utils.checkpoint_io import load_checkpoint

PROJECTIONS = ("gate", "up", "down")
_ADAPTER_KEY = re.compile(r"^(.*moe\.)experts\.(\d+)\.(gate|up|down)\.lora_(a|b)$")


def _kaiming_uniform(shape, fan_in: int, device) -> Tensor:
    # kaiming_uniform_(a=sqrt(5)) bound: gain sqrt(2 / (1 + 5)) * sqrt(3 / fan_in) = 1 / sqrt(fan_in)
    bound = 1.0 / math.sqrt(fan_in)
    return torch.empty(shape, device=device).uniform_(-bound, bound)


class ExpertLoRA(nn.Module):
    """Stacked low-rank updates of every expert's gate, up and down projections."""

    def __init__(self, experts: int, hidden: int, ffn: int, rank: int, alpha: float, device=None) -> None:
        super().__init__()
        if rank < 1:
            raise ValueError("rank must be positive")
        self.rank, self.scaling = rank, alpha / rank
        dims = {"gate": (hidden, ffn), "up": (hidden, ffn), "down": (ffn, hidden)}
        for name, (n_in, n_out) in dims.items():
            self.register_parameter(f"a_{name}", nn.Parameter(_kaiming_uniform((experts, rank, n_in), n_in, device)))
            self.register_parameter(f"b_{name}", nn.Parameter(torch.zeros(experts, n_out, rank, device=device)))

    def project(self, index: int, name: str, x: Tensor) -> Tensor:
        a, b = getattr(self, f"a_{name}")[index], getattr(self, f"b_{name}")[index]
        return F.linear(F.linear(x, a.to(x.dtype)), b.to(x.dtype)) * self.scaling

    def delta(self, index: int, name: str) -> Tensor:
        a, b = getattr(self, f"a_{name}")[index], getattr(self, f"b_{name}")[index]
        return self.scaling * (b.detach().float() @ a.detach().float())


class LoRALinear(nn.Module):
    """Frozen base layer (``nn.Linear`` or ``QuantizedLinear``) plus a trainable low-rank update."""

    def __init__(self, base: nn.Module, rank: int, alpha: float) -> None:
        super().__init__()
        if rank < 1:
            raise ValueError("rank must be positive")
        self.base = base
        self.in_features, self.out_features = base.in_features, base.out_features
        self.rank, self.scaling = rank, alpha / rank
        ref = next(iter(base.parameters()), None)
        device = (ref if ref is not None else next(iter(base.buffers()))).device
        self.lora_a = nn.Parameter(_kaiming_uniform((rank, self.in_features), self.in_features, device))
        self.lora_b = nn.Parameter(torch.zeros(self.out_features, rank, device=device))

    def base_weight(self) -> Tensor:
        from ..inference.quantization import QuantizedLinear

        return self.base.dequantize() if isinstance(self.base, QuantizedLinear) else self.base.weight

    @property
    def weight(self) -> Tensor:
        """The effective (differentiable in the adapter) weight, for consumers that read ``.weight`` directly."""
        base = self.base_weight()
        return base + (self.scaling * (self.lora_b @ self.lora_a)).to(base.dtype)

    def forward(self, x: Tensor) -> Tensor:
        update = F.linear(F.linear(x, self.lora_a.to(x.dtype)), self.lora_b.to(x.dtype))
        return self.base(x) + update * self.scaling

    def merged_weight(self) -> Tensor:
        return self.base_weight().detach().float() + self.scaling * (self.lora_b.detach().float()
                                                                      @ self.lora_a.detach().float())


def add_lora(model, rank: int = 8, alpha: float = 16.0, include_lm_head: bool = False, train_router: bool = False,
             train_norms: bool = False) -> dict:
    """Freeze the model and attach adapters to every expert projection (and optionally the LM head)."""
    for p in model.parameters():
        p.requires_grad_(False)
    wrapped = 0
    for moe in model.moes():
        if getattr(moe, "lora", None) is not None:
            raise ValueError("model already has LoRA adapters")
        device = (moe.q_gate_up if getattr(moe, "quant", None) is not None else moe.w_gate_up).device
        moe.lora = ExpertLoRA(moe.num_local_experts, moe.hidden_size, moe.ffn_local, rank, alpha, device)
        moe.kernel = "loop"
        wrapped += 3 * moe.num_local_experts
    if include_lm_head:
        if isinstance(model.lm_head, LoRALinear):
            raise ValueError("model already has LoRA adapters")
        model.lm_head = LoRALinear(model.lm_head, rank, alpha)
        wrapped += 1
    extra = []
    for name, p in model.named_parameters():
        is_router = name.endswith("moe.router.weight")
        is_norm = "_norm." in name or name.startswith("final_norm.")
        if (train_router and is_router) or (train_norms and is_norm):
            p.requires_grad_(True)
            extra.append(name)
    from ..inference.quantization import QuantizedLinear

    trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
    quantized = sum(m.in_features * m.out_features for m in model.modules() if isinstance(m, QuantizedLinear))
    for moe in model.moes():
        if getattr(moe, "quant", None) is not None:
            quantized += moe.num_local_experts * 3 * moe.hidden_size * moe.ffn_local
    total = sum(p.numel() for p in model.parameters()) + quantized
    return {"wrapped_layers": wrapped, "rank": rank, "alpha": alpha, "include_lm_head": include_lm_head,
            "extra_trainable": extra, "trainable_parameters": trainable, "total_parameters": total}


def adapter_state(model) -> dict[str, Tensor]:
    """Everything trainable, under the reference's per-expert names."""
    state: dict[str, Tensor] = {}
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        match = re.match(r"^(.*moe\.)lora\.(a|b)_(gate|up|down)$", name)
        if match:
            prefix, ab, proj = match.groups()
            for e in range(p.size(0)):
                state[f"{prefix}experts.{e}.{proj}.lora_{ab}"] = p[e].detach().cpu().clone()
        else:
            state[name] = p.detach().cpu().clone()
    return state


def save_adapter(model, path: Path, info: dict, base_checkpoint: Optional[str] = None) -> None:
    torch.save({"state": adapter_state(model), "info": info, "base_checkpoint": base_checkpoint}, path)


def load_adapter(model, path: Path) -> dict:
    payload = load_checkpoint(path, map_location="cpu")
    params = dict(model.named_parameters())
    unknown = []
    with torch.no_grad():
        for name, tensor in payload["state"].items():
            match = _ADAPTER_KEY.match(name)
            if match:
                prefix, e, proj, ab = match.groups()
                target = params.get(f"{prefix}lora.{ab}_{proj}")
                if target is None or int(e) >= target.size(0):
                    unknown.append(name)
                    continue
                target[int(e)].copy_(tensor.to(target.device))
            elif name in params:
                params[name].copy_(tensor.to(params[name].device))
            else:
                unknown.append(name)
    if unknown:
        raise ValueError(f"adapter does not match this model; unknown tensors: {sorted(unknown)[:3]}")
    return payload["info"]


def merge_lora_state(model) -> dict[str, Tensor]:
    """Full-precision state dict with the keys of an ordinary model: dequantised base + low-rank delta."""
    merged: dict[str, Tensor] = {}
    for key, tensor in model.state_dict().items():
        if ".lora." in key or ".base." in key or key.endswith((".lora_a", ".lora_b", ".qweight", ".scales")):
            continue
        merged[key] = tensor.detach().clone()
    for block_index, moe in enumerate(model.moes()):
        prefix = f"blocks.{block_index}.moe.experts"
        f = moe.ffn_local
        for e in range(moe.num_local_experts):
            wgu, wd = moe.expert_weights(e)
            weights = {"gate": wgu[:f].detach().float(), "up": wgu[f:].detach().float(), "down": wd.detach().float()}
            lora = getattr(moe, "lora", None)
            for proj in PROJECTIONS:
                w = weights[proj] + (lora.delta(e, proj) if lora is not None else 0)
                merged[f"{prefix}.{e}.{proj}.weight"] = w.clone()
    for name, module in model.named_modules():
        if isinstance(module, LoRALinear):
            merged[f"{name}.weight"] = module.merged_weight().clone()
    return merged
