"""Top-k routed mixture of SwiGLU experts.

Semantics follow the reference ``TopKMoE`` (``src/quantweave_moe_model.py:63-272``):

* the router runs in fp32 with autocast disabled: ``softmax(x @ Wr^T / T)``; top-k over the probabilities (or over
  ``logits + expert_bias`` when straggler bias is set, weights still taken from the unbiased probabilities); the k
  weights are renormalised to sum to one;
* capacity is ``max(min_cap, ceil(N*k/E * cf * capacity_scale))`` when capacity is on, else ``N*k``;
* routes are ordered by (expert, descending weight, route index) and those past capacity are skipped (the token keeps
  its residual for that route); ``drop`` reports them as dropped, ``residual`` only as overflow;
* balance loss ``E * sum(mean(probs) * mean(one_hot(top_idx)))``.

Storage differs from the reference on purpose: experts are held as two stacked parameters,
``w_gate_up [E, 2F, H]`` (rows ``[0,F)`` gate, ``[F,2F)`` up) and ``w_down [E, H, F]``, which is the layout the
grouped tcgen05 GEMM reads with one tensor map per operand. State-dict hooks translate to and from the reference's
per-expert keys ``experts.{e}.{gate,up,down}.weight`` so checkpoints stay interchangeable.
"""

from __future__ import annotations

import math
import re
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import QuantaWeaveConfig

_EXPERT_KEY = re.compile(r"^experts\.(\d+)\.(gate|up|down)\.(weight|qweight|scales)$")


class SparseSwiGLU(nn.Module):
    """One SwiGLU expert ``down(silu(gate(x)) * up(x))`` (kept for API parity and for LoRA/quantised experts)."""

    def __init__(self, config: QuantaWeaveConfig, ffn_size: Optional[int] = None) -> None:
        super().__init__()
        ffn_size = ffn_size or config.ffn_size
        self.gate = nn.Linear(config.hidden_size, ffn_size, bias=False)
        self.up = nn.Linear(config.hidden_size, ffn_size, bias=False)
        self.down = nn.Linear(ffn_size, config.hidden_size, bias=False)

    def forward(self, hidden: Tensor) -> Tensor:
        return self.down(F.silu(self.gate(hidden)) * self.up(hidden))


class ExpertView(nn.Module):
    """A read-only per-expert view over the stacked weights (``moe.experts[e].gate.weight`` etc.)."""

    class _Proj:
        def __init__(self, weight: Tensor) -> None:
            self.weight = weight

        def __call__(self, x: Tensor) -> Tensor:
            return F.linear(x, self.weight)

    def __init__(self, moe: "TopKMoE", index: int) -> None:
        super().__init__()
        self._moe = [moe]
        self.index = index

    @property
    def gate(self):
        moe = self._moe[0]
        return self._Proj(moe.w_gate_up[self.index, : moe.ffn_local])

    @property
    def up(self):
        moe = self._moe[0]
        return self._Proj(moe.w_gate_up[self.index, moe.ffn_local :])

    @property
    def down(self):
        return self._Proj(self._moe[0].w_down[self.index])

    def forward(self, x: Tensor) -> Tensor:
        return self.down(F.silu(self.gate(x)) * self.up(x))


class _ExpertList:
    def __init__(self, moe: "TopKMoE") -> None:
        self._moe = moe

    def __len__(self) -> int:
        return self._moe.num_local_experts

    def __getitem__(self, index: int) -> ExpertView:
        if not 0 <= index < len(self):
            raise IndexError(index)
        return ExpertView(self._moe, index)

    def __iter__(self):
        return (self[i] for i in range(len(self)))


class TopKMoE(nn.Module):
    def __init__(self, config: QuantaWeaveConfig, num_local_experts: Optional[int] = None, tensor_parallel=None) -> None:
        super().__init__()
        if config.top_k < 1 or config.top_k > config.num_experts:
            raise ValueError("top_k must be between 1 and num_experts")
        self.tp_size = getattr(tensor_parallel, "tp_size", 1)
        self.tp_group = getattr(tensor_parallel, "tp_group", None) if self.tp_size > 1 else None
        if config.ffn_size % self.tp_size:
            raise ValueError(f"ffn_size {config.ffn_size} must be divisible by the tensor-parallel size {self.tp_size}")
        self.config = config
        self.hidden_size = config.hidden_size
        self.num_experts = config.num_experts
        self.top_k = config.top_k
        self.capacity_factor = config.capacity_factor
        self.min_expert_capacity = config.min_expert_capacity
        self.drop_overflow_tokens = config.drop_overflow_tokens
        self.overflow_policy = config.overflow_policy
        self.router_temperature = config.router_temperature
        self.router = nn.Linear(config.hidden_size, config.num_experts, bias=False)
        self.num_local_experts = num_local_experts or config.num_experts
        self.ffn_local = config.ffn_size // self.tp_size
        e, f, h = self.num_local_experts, self.ffn_local, config.hidden_size
        self.w_gate_up = nn.Parameter(torch.empty(e, 2 * f, h))
        self.w_down = nn.Parameter(torch.empty(e, h, f))
        self.reset_parameters()
        # runtime switches (not parameters, not saved)
        self.collect_stats = False
        self.static_dispatch = False
        self.profile_experts = False
        self.kernel = "auto"                          # "loop" | "native" | "auto"
        self.expert_bias: Optional[Tensor] = None     # straggler-aware routing, selection only
        self.capacity_scale: float = 1.0
        self.simulated_cost_per_row: float = 0.0
        self.recompute_activations = False           # native path: recompute gate/up in backward instead of saving
        self.expert_seconds = [0.0] * self.num_local_experts
        self.last_top_indices: Optional[Tensor] = None
        self.last_stats: dict[str, Tensor] = {}
        self._register_state_dict_hook(_expert_state_dict_hook)
        self._register_load_state_dict_pre_hook(_expert_load_pre_hook, with_module=True)

    # ---- parameters ------------------------------------------------------
    def reset_parameters(self) -> None:
        std = self.config.init_std
        h, f = self.config.hidden_size, self.ffn_local
        with torch.no_grad():
            if std is None:
                # nn.Linear default: U(-1/sqrt(fan_in), 1/sqrt(fan_in)), per expert projection
                self.w_gate_up.uniform_(-1 / math.sqrt(h), 1 / math.sqrt(h))
                self.w_down.uniform_(-1 / math.sqrt(self.config.ffn_size), 1 / math.sqrt(self.config.ffn_size))
            else:
                self.w_gate_up.normal_(0.0, std)
                self.w_down.normal_(0.0, std)
                self.router.weight.normal_(0.0, std)
        del f

    @property
    def experts(self) -> _ExpertList:
        return _ExpertList(self)

    # ---- capacity ------------------------------------------------------------
    def capacity(self, num_tokens: int) -> int:
        if self.capacity_factor > 0 and self.drop_overflow_tokens:
            return max(
                self.min_expert_capacity,
                math.ceil(num_tokens * self.top_k / self.num_experts * self.capacity_factor * self.capacity_scale),
            )
        return num_tokens * self.top_k

    # ---- routing -------------------------------------------------------------
    def route(self, flat_hidden: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        """fp32 router: returns (logits, probs, top_indices, top_weights renormalised)."""
        with torch.autocast(flat_hidden.device.type, enabled=False):
            logits = F.linear(flat_hidden.float(), self.router.weight.float()) / self.router_temperature
            probs = logits.softmax(dim=-1)
        if self.expert_bias is None:
            top_weights, top_indices = probs.topk(self.top_k, dim=-1)
        else:
            top_indices = (logits + self.expert_bias.to(logits)).topk(self.top_k, dim=-1).indices
            top_weights = probs.gather(1, top_indices)
        top_weights = top_weights / top_weights.sum(dim=-1, keepdim=True)
        return logits, probs, top_indices, top_weights

    def forward(self, hidden: Tensor, token_domains: Optional[Tensor] = None, num_domains: int = 0):
        """Returns (output, balance_loss, dropped_routes, overflow_routes, domain_loss)."""
        batch, sequence, width = hidden.shape
        flat = hidden.reshape(-1, width)
        num_tokens = flat.size(0)
        if hidden.is_cuda and (self._native_ok() or self._quantized_native_ok()):
            from ..ops import moe as moe_ops

            self._last_counts = None
            output, probs, top_indices, overflow, kept_counts, dropped = moe_ops.moe_forward(self, flat, self.capacity(num_tokens))
            self.last_top_indices = top_indices.detach()
            if self.collect_stats:
                self._record_stats(probs, top_indices, kept_counts, dropped)
        else:
            _, probs, top_indices, top_weights = self.route(flat)
            self.last_top_indices = top_indices.detach()
            overflow = torch.zeros((), device=hidden.device, dtype=torch.long)
            if self.static_dispatch:
                output = self._static_output(flat, probs, top_indices, top_weights)
            else:
                tokens, weights, kept_counts, overflow, dropped = self.plan(top_indices, top_weights, self.capacity(num_tokens))
                output = self._execute(flat, tokens, weights, kept_counts)
                if self.collect_stats:
                    self._record_stats(probs, top_indices, kept_counts, dropped)
        zero = torch.zeros((), device=hidden.device, dtype=torch.long)
        dropped_routes = overflow if self.overflow_policy == "drop" else zero
        counts = getattr(self, "_last_counts", None) if hidden.is_cuda else None
        balance_loss = self.balance_loss(probs, top_indices, counts)
        domain_loss = probs.new_zeros(())
        if token_domains is not None and num_domains > 1:
            domain_loss = self._domain_loss(probs, token_domains, num_domains)
        return output.reshape(batch, sequence, width), balance_loss, dropped_routes, overflow, domain_loss

    def balance_loss(self, probs: Tensor, top_indices: Tensor, counts: Optional[Tensor] = None) -> Tensor:
        """``E * sum(mean(probs) * share of routes per expert)``; ``counts`` (the router kernel's per-expert route
        counts) avoids a bincount, which synchronises with the host on CUDA."""
        importance = probs.mean(dim=0)
        if counts is None:
            counts = torch.bincount(top_indices.reshape(-1), minlength=self.num_experts)
        assignments = counts.float() / top_indices.numel()
        return self.num_experts * (importance * assignments).sum()

    def _quantized_native_ok(self) -> bool:
        """Quantised experts on many tokens at once (prefill, evaluation): without gradients, the packed weights are
        expanded to bf16 by one kernel and the tcgen05 grouped GEMMs run over all routed rows."""
        if getattr(self, "quant", None) is None or torch.is_grad_enabled() or self.tp_size > 1:
            return False
        if self.kernel == "loop" or self.static_dispatch or self.profile_experts or getattr(self, "lora", None):
            return False
        from ..ops import native_required

        native_required()
        return True

    def _native_ok(self) -> bool:
        if self.kernel == "loop" or self.static_dispatch or self.profile_experts:
            return False
        if getattr(self, "lora", None) is not None or getattr(self, "quant", None) is not None:
            return False  # adapters / quantised bases run the per-expert path (the decoder serves quantised models)
        from ..ops import native_required

        native_required()
        return True

    def plan(self, top_indices: Tensor, top_weights: Tensor, capacity: int):
        """Order routes by (expert, -weight, route) and cut each expert at ``capacity``.

        Returns (token per kept route, weight per kept route, kept count per expert, overflow count,
        (dropped token, dropped expert)).
        """
        route_experts = top_indices.reshape(-1)
        route_weights = top_weights.reshape(-1)
        by_weight = torch.argsort(route_weights, descending=True, stable=True)
        order = by_weight[torch.argsort(route_experts[by_weight], stable=True)]
        counts = torch.bincount(route_experts, minlength=self.num_experts)
        starts = torch.cumsum(counts, dim=0) - counts
        position = torch.arange(order.numel(), device=order.device) - starts[route_experts[order]]
        keep = position < capacity
        kept = order[keep]
        dropped = order[~keep]
        return (
            kept // self.top_k,
            route_weights[kept],
            counts.clamp(max=capacity),
            (~keep).sum(),
            (dropped // self.top_k, route_experts[dropped]),
        )

    def expert_weights(self, index: int) -> tuple[Tensor, Tensor]:
        """(gate|up [2F, H], down [H, F]) of one expert; quantised experts are dequantised on the fly."""
        if getattr(self, "quant", None) is not None:
            from ..inference.quantization import dequantized_expert

            return dequantized_expert(self, index)
        return self.w_gate_up[index], self.w_down[index]

    def expert_forward(self, index: int, x: Tensor) -> Tensor:
        f = self.ffn_local
        lora = getattr(self, "lora", None)
        if getattr(self, "quant", None) is not None or lora is not None:
            wgu, wd = self.expert_weights(index)
            wgu, wd = wgu.to(x.dtype), wd.to(x.dtype)
            gate, up = F.linear(x, wgu[:f]), F.linear(x, wgu[f:])
            if lora is not None:  # low-rank updates of the three projections (gate/up before the activation)
                gate = gate + lora.project(index, "gate", x)
                up = up + lora.project(index, "up", x)
            hidden = F.silu(gate) * up
            out = F.linear(hidden, wd)
            if lora is not None:
                out = out + lora.project(index, "down", hidden)
            return out
        w = self.w_gate_up[index]
        hidden = F.silu(F.linear(x, w[:f])) * F.linear(x, w[f:])
        return F.linear(hidden, self.w_down[index])

    def _execute(self, flat_hidden: Tensor, tokens: Tensor, weights: Tensor, kept_counts: Tensor) -> Tensor:
        output = torch.zeros_like(flat_hidden)
        if tokens.numel() == 0:
            return output
        inputs = self._tp_in(flat_hidden[tokens])
        results = []
        start = 0
        for index, count in enumerate(kept_counts.tolist()):
            if not count:
                continue
            results.append(self._run_expert(index, inputs[start : start + count]))
            start += count
        expert_output = self._tp_out(torch.cat(results)) * weights[:, None]
        output.index_add_(0, tokens, expert_output.to(output.dtype))
        return output

    def _tp_in(self, x: Tensor) -> Tensor:
        if self.tp_group is None:
            return x
        from ..parallel.tensor_parallel import copy_to_tp

        return copy_to_tp(x, self.tp_group)

    def _tp_out(self, x: Tensor) -> Tensor:
        if self.tp_group is None:
            return x
        from ..parallel.tensor_parallel import reduce_from_tp

        return reduce_from_tp(x, self.tp_group)

    def _run_expert(self, index: int, inputs: Tensor) -> Tensor:
        if not self.profile_experts and not self.simulated_cost_per_row:
            return self.expert_forward(index, inputs)
        import time

        if inputs.is_cuda:
            torch.cuda.synchronize()
        started = time.perf_counter()
        result = self.expert_forward(index, inputs)
        if self.simulated_cost_per_row:
            time.sleep(self.simulated_cost_per_row * inputs.size(0))
        if inputs.is_cuda:
            torch.cuda.synchronize()
        self.expert_seconds[index] += time.perf_counter() - started
        return result

    def _static_output(self, flat_hidden: Tensor, probs: Tensor, top_indices: Tensor, top_weights: Tensor) -> Tensor:
        """Capacity-free dense evaluation with no data-dependent control flow (tracing/export)."""
        if self.tp_size > 1:
            raise RuntimeError("static (export) dispatch needs a consolidated, non-tensor-parallel model")
        dense = torch.zeros_like(probs).scatter(1, top_indices, top_weights)
        output = torch.zeros_like(flat_hidden)
        for index in range(self.num_local_experts):
            output = output + self.expert_forward(index, flat_hidden) * dense[:, index : index + 1].to(flat_hidden.dtype)
        return output

    def _domain_loss(self, probs: Tensor, token_domains: Tensor, num_domains: int) -> Tensor:
        """Mean pairwise cosine similarity between the routing profiles of the domains present."""
        membership = F.one_hot(token_domains, num_domains).to(probs.dtype)
        counts = membership.sum(dim=0)
        profiles = (membership.t() @ probs) / counts.clamp(min=1)[:, None]
        profiles = F.normalize(profiles[counts > 0], dim=-1)
        present = profiles.size(0)
        if present < 2:
            return probs.new_zeros(())
        similarity = profiles @ profiles.t()
        return (similarity.sum() - similarity.diagonal().sum()) / (present * (present - 1))

    @torch.no_grad()
    def _record_stats(self, probs: Tensor, top_indices: Tensor, kept_counts: Tensor, dropped) -> None:
        probs = probs.float()
        entropy = -(probs * probs.clamp_min(1e-12).log()).sum(dim=-1)
        top_probability = probs.max(dim=-1).values
        self.last_stats = {
            "expert_load": kept_counts.detach(),
            "expert_assigned": torch.bincount(top_indices.reshape(-1), minlength=self.num_experts),
            "importance": probs.mean(dim=0).detach(),
            "entropy_mean": entropy.mean(),
            "confidence_mean": top_probability.mean(),
            "confidence_hist": torch.histc(top_probability, bins=10, min=0.0, max=1.0),
            "dropped_tokens": dropped[0],
            "dropped_experts": dropped[1],
        }


# ---- checkpoint-format translation -------------------------------------------------------------
def _expert_state_dict_hook(module: TopKMoE, state_dict: dict, prefix: str, local_metadata) -> None:
    """Replace the stacked tensors by the reference's per-expert keys (views, so nothing is copied)."""
    if prefix + "q_gate_up" in state_dict:
        q_gu, s_gu = state_dict.pop(prefix + "q_gate_up"), state_dict.pop(prefix + "s_gate_up")
        q_d, s_d = state_dict.pop(prefix + "q_down"), state_dict.pop(prefix + "s_down")
        f = module.ffn_local
        for e in range(module.num_local_experts):
            state_dict[f"{prefix}experts.{e}.gate.qweight"] = q_gu[e, :f]
            state_dict[f"{prefix}experts.{e}.gate.scales"] = s_gu[e, :f].float()
            state_dict[f"{prefix}experts.{e}.up.qweight"] = q_gu[e, f:]
            state_dict[f"{prefix}experts.{e}.up.scales"] = s_gu[e, f:].float()
            state_dict[f"{prefix}experts.{e}.down.qweight"] = q_d[e]
            state_dict[f"{prefix}experts.{e}.down.scales"] = s_d[e].float()
        return
    gate_up = state_dict.pop(prefix + "w_gate_up", None)
    down = state_dict.pop(prefix + "w_down", None)
    if gate_up is None or down is None:
        return
    f = module.ffn_local
    for e in range(module.num_local_experts):
        state_dict[f"{prefix}experts.{e}.gate.weight"] = gate_up[e, :f]
        state_dict[f"{prefix}experts.{e}.up.weight"] = gate_up[e, f:]
        state_dict[f"{prefix}experts.{e}.down.weight"] = down[e]


def _expert_load_pre_hook(module: TopKMoE, state_dict: dict, prefix: str, local_metadata, strict, missing_keys,
                          unexpected_keys, error_msgs) -> None:
    """Stack ``experts.{e}.{gate,up,down}.weight`` back into ``w_gate_up``/``w_down``."""
    found: dict[tuple[int, str], Tensor] = {}
    quant: dict[tuple[int, str, str], Tensor] = {}
    for key in list(state_dict.keys()):
        if not key.startswith(prefix):
            continue
        match = _EXPERT_KEY.match(key[len(prefix):])
        if match and match.group(3) == "weight":
            found[(int(match.group(1)), match.group(2))] = state_dict.pop(key)
        elif match:
            quant[(int(match.group(1)), match.group(2), match.group(3))] = state_dict.pop(key)
    n = module.num_local_experts
    if quant:
        try:
            state_dict[prefix + "q_gate_up"] = torch.stack(
                [torch.cat([quant[(e, "gate", "qweight")], quant[(e, "up", "qweight")]]) for e in range(n)])
            state_dict[prefix + "s_gate_up"] = torch.stack(
                [torch.cat([quant[(e, "gate", "scales")], quant[(e, "up", "scales")]]) for e in range(n)]).half()
            state_dict[prefix + "q_down"] = torch.stack([quant[(e, "down", "qweight")] for e in range(n)])
            state_dict[prefix + "s_down"] = torch.stack([quant[(e, "down", "scales")] for e in range(n)]).half()
        except KeyError as missing:
            error_msgs.append(f"missing quantized expert tensor {missing} under {prefix}experts")
        return
    if not found:
        return
    try:
        gates = [found[(e, "gate")] for e in range(n)]
        ups = [found[(e, "up")] for e in range(n)]
        downs = [found[(e, "down")] for e in range(n)]
    except KeyError as missing:
        error_msgs.append(f"missing expert weight {missing} under {prefix}experts")
        return
    extra = sorted({e for e, _ in found} - set(range(n)))
    if extra:
        error_msgs.append(f"unexpected experts {extra} under {prefix}experts (module holds {n})")
    state_dict[prefix + "w_gate_up"] = torch.stack([torch.cat([g, u], dim=0) for g, u in zip(gates, ups)])
    state_dict[prefix + "w_down"] = torch.stack(downs)
