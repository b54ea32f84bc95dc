"""Grouped expert GEMMs with the reference's ``moe_kernels`` API, on the tcgen05 grouped GEMM.

The names and behaviour follow ``src/moe_kernels.py`` of the reference (``kernels_available`` :34, ``GroupedPlan``
:92-111, ``grouped_matmul`` :167, ``experts_support_grouped`` :174, ``compute_dtype`` :179, ``grouped_swiglu``
:186-195, ``benchmark`` :198-227): ``grouped_matmul(x, W, plan)`` computes ``Y[rows of e] = X[rows of e] @ W[e]^T``
for rows already sorted by expert, differentiably (``dX = dY @ W[e]``, ``dW[e] = dY[rows of e]^T @ X[rows of e]``).

The B200 kernels (``csrc/gemm.cu``: ``moe_down_fwd``, ``moe_gate_up_dgrad``, ``moe_wgrad``) want every expert's rows
to start on a 128-row boundary with zero rows in between, the layout the model's own MoE path produces directly. A
``GroupedPlan`` therefore also carries the padded offsets and the packed-to-padded row map; ``grouped_matmul``
scatters the packed rows into a zeroed padded buffer, runs the grouped GEMM in bf16 with fp32 accumulation in TMEM
and gathers the rows back. Without the extension, on CPU, or for widths that are not multiples of 8 (the TMA row
alignment) it runs a per-expert loop in the input dtype. The model's MoE layers call the native kernels directly;
this module is the public entry point for code written against the reference's.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor, nn

PAD = 128  # rows per tcgen05 tile


def kernels_available(device: torch.device) -> bool:
    from . import native_available

    return torch.device(device).type == "cuda" and torch.cuda.is_available() and native_available()


class GroupedPlan:
    """Row layout for one set of per-expert row counts (rows sorted by expert)."""

    def __init__(self, counts: Sequence[int], device: torch.device) -> None:
        counts = [int(c) for c in counts]
        starts, ends, padded, row_index, offset, padded_offset = [], [], [], [], 0, 0
        for count in counts:
            starts.append(offset)
            padded.append(padded_offset)
            row_index.extend(range(padded_offset, padded_offset + count))
            offset += count
            ends.append(offset)
            padded_offset += (count + PAD - 1) // PAD * PAD
        as_int = lambda values: torch.tensor(values, dtype=torch.int32, device=device)  # noqa: E731
        self.num_experts = len(counts)
        self.rows = offset
        self.padded_rows = padded_offset
        self.tiles = sum((c + PAD - 1) // PAD for c in counts)
        self.count_list = counts
        self.counts = as_int(counts)
        self.expert_start, self.expert_end = as_int(starts), as_int(ends)
        self.offsets = as_int(padded)
        self.row_index = torch.tensor(row_index, dtype=torch.long, device=device)


def _native(x: Tensor, weight: Tensor) -> bool:
    return (x.is_cuda and kernels_available(x.device) and x.size(1) % 8 == 0 and weight.size(1) % 8 == 0
            and weight.size(1) % 2 == 0)


def _padded(rows: Tensor, plan: GroupedPlan) -> Tensor:
    out = rows.new_zeros(plan.padded_rows, rows.size(1))
    out[plan.row_index] = rows
    return out


def _loop(x: Tensor, weight: Tensor, plan: GroupedPlan, transpose: bool) -> Tensor:
    out = x.new_empty(x.size(0), weight.size(2) if transpose else weight.size(1))
    for e, count in enumerate(plan.count_list):
        start = int(plan.expert_start[e])
        block = x[start:start + count].float()
        w = weight[e].float()
        out[start:start + count] = (block @ w if transpose else block @ w.T).to(out.dtype)
    return out


class _GroupedMatmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, plan: GroupedPlan) -> Tensor:
        ctx.plan = plan
        ctx.native = _native(x, weight)
        ctx.save_for_backward(x, weight)
        if plan.rows == 0:
            return x.new_zeros(0, weight.size(1))
        if not ctx.native:
            return _loop(x, weight, plan, transpose=False)
        from . import ext

        xp = _padded(x.to(torch.bfloat16), plan)
        w = weight.to(torch.bfloat16).contiguous()
        yp = torch.empty(plan.padded_rows, w.size(1), device=x.device, dtype=torch.bfloat16)
        ext().moe_down_fwd(xp, w, plan.counts, plan.offsets, yp)
        return yp[plan.row_index].to(x.dtype)

    @staticmethod
    def backward(ctx, grad: Tensor):
        x, weight = ctx.saved_tensors
        plan = ctx.plan
        grad_x = grad_w = None
        if plan.rows == 0:
            return (x.new_zeros(x.shape) if ctx.needs_input_grad[0] else None,
                    torch.zeros_like(weight) if ctx.needs_input_grad[1] else None, None)
        if not ctx.native:
            if ctx.needs_input_grad[0]:
                grad_x = _loop(grad, weight, plan, transpose=True)
            if ctx.needs_input_grad[1]:
                grad_w = torch.zeros_like(weight)
                for e, count in enumerate(plan.count_list):
                    start = int(plan.expert_start[e])
                    grad_w[e] = (grad[start:start + count].float().T @ x[start:start + count].float()).to(weight.dtype)
            return grad_x, grad_w, None
        from . import ext

        C = ext()
        gp = _padded(grad.to(torch.bfloat16).contiguous(), plan)
        w = weight.to(torch.bfloat16).contiguous()
        if ctx.needs_input_grad[0]:
            dxp = torch.empty(plan.padded_rows, w.size(2), device=grad.device, dtype=torch.bfloat16)
            C.moe_gate_up_dgrad(gp, w, plan.counts, plan.offsets, dxp)  # dX = dY @ W[e] (reduction over W's rows)
            grad_x = dxp[plan.row_index].to(x.dtype)
        if ctx.needs_input_grad[1]:
            xp = _padded(x.to(torch.bfloat16), plan)
            dw = torch.zeros(w.shape, device=grad.device, dtype=torch.float32)  # experts with no rows stay exactly zero
            C.moe_wgrad(gp, xp, plan.counts, plan.offsets, dw, False)
            grad_w = dw.to(weight.dtype)
        return grad_x, grad_w, None


def grouped_matmul(x: Tensor, weight: Tensor, plan: GroupedPlan) -> Tensor:
    """Per-expert ``x @ W[e]^T`` over expert-sorted rows; ``weight`` is ``[E, out, in]``."""
    return _GroupedMatmul.apply(x, weight, plan)


def experts_support_grouped(experts) -> bool:
    """True when every expert is a plain bias-free SwiGLU: ``nn.Linear`` projections (the reference's experts) or the
    views over a ``TopKMoE``'s stacked weights; quantised and LoRA experts are not."""
    from ..models.moe import ExpertView

    for e in experts:
        if isinstance(e, ExpertView):
            moe = e._moe[0]
            if getattr(moe, "quant", None) is not None or getattr(moe, "lora", None) is not None:
                return False
            continue
        for name in ("gate", "up", "down"):
            proj = getattr(e, name, None)
            if not isinstance(proj, nn.Linear) or proj.bias is not None:
                return False
    return True


def compute_dtype(inputs: Tensor) -> torch.dtype:
    device_type = inputs.device.type
    if torch.is_autocast_enabled(device_type):
        return torch.get_autocast_dtype(device_type)
    return inputs.dtype


def grouped_swiglu(inputs: Tensor, experts, counts: Sequence[int], plan: Optional[GroupedPlan] = None) -> Tensor:
    """SwiGLU over expert-sorted rows: ``down(silu(gate(x)) * up(x))`` with each expert's own weights."""
    plan = plan or GroupedPlan(counts, inputs.device)
    dtype = compute_dtype(inputs)
    x = inputs.to(dtype)
    gate = torch.stack([e.gate.weight for e in experts]).to(dtype)
    up = torch.stack([e.up.weight for e in experts]).to(dtype)
    down = torch.stack([e.down.weight for e in experts]).to(dtype)
    hidden = F.silu(grouped_matmul(x, gate, plan)) * grouped_matmul(x, up, plan)
    return grouped_matmul(hidden, down, plan)


def benchmark(experts: int = 32, tokens: int = 8192, hidden: int = 256, ffn: int = 512, top_k: int = 2,
              repeats: int = 20, bf16: bool = False) -> dict:
    """Per-expert loop vs the native grouped MoE path (forward + backward), CUDA-event timed on the current GPU."""
    from ..config import QuantaWeaveConfig
    from ..models.moe import TopKMoE

    if not kernels_available(torch.device("cuda")):
        raise RuntimeError("benchmark needs CUDA and the compiled quantaweave_b200._C extension")
    config = QuantaWeaveConfig(vocab_size=8, hidden_size=hidden, layers=1, ffn_size=ffn, num_experts=experts,
                               top_k=top_k, attention_heads=1, max_sequence_length=tokens, capacity_factor=0)
    result = {}
    for name in ("loop", "native"):
        moe = TopKMoE(config).cuda()
        if name == "native":
            from ..training.native import prepare_model

            prepare_model(moe, "bf16")
        moe.kernel = name
        x = torch.randn(1, tokens, hidden, device="cuda", requires_grad=True)
        context = torch.autocast("cuda", dtype=torch.bfloat16) if bf16 else torch.autocast("cuda", enabled=False)
        for _ in range(3):
            with context:
                out = moe(x)[0]
            out.float().sum().backward()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for _ in range(repeats):
            with context:
                out = moe(x)[0]
            out.float().sum().backward()
        stop.record()
        torch.cuda.synchronize()
        result[name + "_ms"] = start.elapsed_time(stop) / repeats
    result["speedup"] = result["loop_ms"] / result["native_ms"]
    result.update(experts=experts, tokens=tokens, hidden=hidden, ffn=ffn, top_k=top_k, bf16=bf16)
    return result


if __name__ == "__main__":
    import json

    print(json.dumps(benchmark(), indent=2))
