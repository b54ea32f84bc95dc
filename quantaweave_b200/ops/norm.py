"""RMSNorm / LayerNorm kernels with autograd, including the fused ``residual + delta -> norm`` variant."""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import ext


def _flat(x: Tensor) -> Tensor:
    return x.reshape(-1, x.size(-1)).contiguous()


class _NormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Optional[Tensor], eps: float, rms: bool):
        C = ext()
        x2 = _flat(x.to(torch.bfloat16))
        rows = x2.size(0)
        y = torch.empty_like(x2)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        mean = None if rms else torch.empty(rows, device=x.device, dtype=torch.float32)
        C.norm_fwd(x2, None, None, weight.float().contiguous(), None if bias is None else bias.float().contiguous(),
                   y, mean, rstd, eps, rms)
        ctx.save_for_backward(x2, weight, mean if mean is not None else rstd, rstd)
        ctx.rms, ctx.has_bias, ctx.shape = rms, bias is not None, x.shape
        return y.reshape(x.shape)

    @staticmethod
    def backward(ctx, grad: Tensor):
        C = ext()
        x2, weight, mean, rstd = ctx.saved_tensors
        g2 = _flat(grad.to(torch.bfloat16))
        H = x2.size(1)
        blocks = C.norm_bwd_blocks(x2.size(0))
        dx = torch.empty_like(x2)
        dw_part = torch.empty(blocks, H, device=grad.device, dtype=torch.float32)
        db_part = None if ctx.rms else torch.empty(blocks, H, device=grad.device, dtype=torch.float32)
        dw = torch.empty(H, device=grad.device, dtype=torch.float32)
        db = None if ctx.rms else torch.empty(H, device=grad.device, dtype=torch.float32)
        C.norm_bwd(g2, x2, weight.float().contiguous(), None if ctx.rms else mean, rstd, None, dx, dw_part, db_part,
                   dw, db, ctx.rms, False)
        return (dx.reshape(ctx.shape), dw.to(weight.dtype),
                db.to(weight.dtype) if (db is not None and ctx.has_bias) else None, None, None)


def norm(x: Tensor, weight: Tensor, bias: Optional[Tensor], eps: float, kind: str) -> Tensor:
    return _NormFn.apply(x, weight, bias, eps, kind == "rmsnorm")


class _AddNormFn(torch.autograd.Function):
    """``s = x + delta`` (rounded to bf16) and ``y = norm(s)``; returns (s, y)."""

    @staticmethod
    def forward(ctx, x: Tensor, delta: Tensor, weight: Tensor, bias: Optional[Tensor], eps: float, rms: bool):
        C = ext()
        x2, d2 = _flat(x.to(torch.bfloat16)), _flat(delta.to(torch.bfloat16))
        rows = x2.size(0)
        s = torch.empty_like(x2)
        y = torch.empty_like(x2)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        mean = None if rms else torch.empty(rows, device=x.device, dtype=torch.float32)
        C.norm_fwd(x2, d2, s, weight.float().contiguous(), None if bias is None else bias.float().contiguous(), y,
                   mean, rstd, eps, rms)
        ctx.save_for_backward(s, weight, mean if mean is not None else rstd, rstd)
        ctx.rms, ctx.has_bias, ctx.shape = rms, bias is not None, x.shape
        return s.reshape(x.shape), y.reshape(x.shape)

    @staticmethod
    def backward(ctx, grad_s: Tensor, grad_y: Tensor):
        C = ext()
        s, weight, mean, rstd = ctx.saved_tensors
        H = s.size(1)
        gy = _flat(grad_y.to(torch.bfloat16))
        gs = _flat(grad_s.to(torch.bfloat16)) if grad_s is not None else None
        blocks = C.norm_bwd_blocks(s.size(0))
        dx = torch.empty_like(s)
        dw_part = torch.empty(blocks, H, device=s.device, dtype=torch.float32)
        db_part = None if ctx.rms else torch.empty(blocks, H, device=s.device, dtype=torch.float32)
        dw = torch.empty(H, device=s.device, dtype=torch.float32)
        db = None if ctx.rms else torch.empty(H, device=s.device, dtype=torch.float32)
        C.norm_bwd(gy, s, weight.float().contiguous(), None if ctx.rms else mean, rstd, gs, dx, dw_part, db_part, dw,
                   db, ctx.rms, False)
        dx = dx.reshape(ctx.shape)
        return (dx, dx, dw.to(weight.dtype), db.to(weight.dtype) if (db is not None and ctx.has_bias) else None,
                None, None)


def add_norm(x: Tensor, delta: Tensor, weight: Tensor, bias: Optional[Tensor], eps: float, kind: str):
    return _AddNormFn.apply(x, delta, weight, bias, eps, kind == "rmsnorm")
