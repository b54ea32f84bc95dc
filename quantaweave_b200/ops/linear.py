"""Dense linear layers on the tcgen05 GEMM: ``y = x @ W^T (+ bias) (+ residual)`` with fused backward GEMMs.

Backward: ``dx = dy @ W`` (B operand read MN-major) and ``dW = dy^T @ x`` (both operands MN-major, the token
dimension is the reduction). Weight gradients leave the GEMM in the parameter's dtype after fp32 accumulation in
TMEM; bias gradients are a column sum.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import ext


def _rows(t: Tensor) -> Tensor:
    t = t.reshape(-1, t.size(-1))
    return t if t.stride(-1) == 1 and t.stride(0) % 8 == 0 else t.contiguous()


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Optional[Tensor], residual: Optional[Tensor]):
        C = ext()
        shape = x.shape
        x2 = _rows(x.to(torch.bfloat16))
        w = weight if weight.dtype == torch.bfloat16 else weight.to(torch.bfloat16)
        out = torch.empty(x2.size(0), w.size(0), device=x.device, dtype=torch.bfloat16)
        res2 = _rows(residual) if residual is not None else None
        C.linear_fwd(x2, w.contiguous(), bias.float() if bias is not None else None, res2, out)
        ctx.save_for_backward(x2, w)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = bias.dtype if bias is not None else None
        ctx.weight_dtype = weight.dtype
        ctx.has_res = residual is not None
        ctx.in_shape = shape
        return out.reshape(*shape[:-1], w.size(0))

    @staticmethod
    def backward(ctx, grad: Tensor):
        C = ext()
        x2, w = ctx.saved_tensors
        g2 = _rows(grad.to(torch.bfloat16))
        dx = dw = db = dres = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(x2.size(0), w.size(1), device=grad.device, dtype=torch.bfloat16)
            C.linear_dgrad(g2, w, dx, False)
            dx = dx.reshape(ctx.in_shape)
        if ctx.needs_input_grad[1]:
            dw = torch.empty(w.size(0), w.size(1), device=grad.device, dtype=ctx.weight_dtype
                             if ctx.weight_dtype in (torch.bfloat16, torch.float32) else torch.float32)
            C.linear_wgrad(g2, x2, dw, False)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = torch.empty(g2.size(1), device=grad.device, dtype=torch.float32)
            part = torch.empty(C.bias_grad_slabs(g2.size(0)), g2.size(1), device=grad.device, dtype=torch.float32)
            C.bias_grad(g2, part, db, False)
            db = db.to(ctx.bias_dtype)
        if ctx.has_res and ctx.needs_input_grad[3]:
            dres = grad
        return dx, dw, db, dres


def linear(x: Tensor, weight: Tensor, bias: Optional[Tensor] = None, residual: Optional[Tensor] = None) -> Tensor:
    """bf16 tcgen05 linear layer; ``residual`` (same shape as the output) is added in the GEMM epilogue."""
    return _LinearFn.apply(x, weight, bias, residual)
