"""Causal self-attention on the native kernels: tcgen05 QKV GEMM -> in-place RoPE -> flash attention ->
tcgen05 output projection. GQA reads K/V heads in place from the packed QKV rows."""

from __future__ import annotations

import math

import torch
from torch import Tensor

from . import ext
from .linear import linear

_TABLES: dict = {}


def rope_cache(seq: int, head_dim: int, theta: float, device) -> tuple[Tensor, Tensor]:
    key = (seq, head_dim, float(theta), str(device))
    if key not in _TABLES:
        from ..models.layers import rope_tables

        cos, sin = rope_tables(torch.arange(seq, device=device), head_dim, theta)
        _TABLES[key] = (cos.contiguous(), sin.contiguous())
    return _TABLES[key]


class _AttnCore(torch.autograd.Function):
    """qkv [T, (Hq + 2Hkv) * D] (pre-RoPE) -> o [T, Hq * D]."""

    @staticmethod
    def forward(ctx, qkv: Tensor, batch: int, seq: int, hq: int, hkv: int, d: int, rope: bool, theta: float):
        C = ext()
        qkv = qkv.contiguous().clone() if rope else qkv.contiguous()  # RoPE below rotates this copy in place
        if rope:
            cos, sin = rope_cache(seq, d, theta, qkv.device)
            C.rope_apply(qkv, hq + hkv, d, seq, None, cos, sin, False)
        T = qkv.size(0)
        q = qkv[:, : hq * d]
        k = qkv[:, hq * d:(hq + hkv) * d]
        v = qkv[:, (hq + hkv) * d:]
        o = torch.empty(T, hq * d, device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty(batch, hq, seq, device=qkv.device, dtype=torch.float32)
        C.flash_attn_fwd(q, k, v, o, lse, batch, seq, hq, hkv, d, 1.0 / math.sqrt(d))
        ctx.save_for_backward(qkv, o, lse)
        ctx.dims = (batch, seq, hq, hkv, d, rope, theta)
        return o

    @staticmethod
    def backward(ctx, grad_o: Tensor):
        C = ext()
        qkv, o, lse = ctx.saved_tensors
        batch, seq, hq, hkv, d, rope, theta = ctx.dims
        grad_o = grad_o.to(torch.bfloat16).contiguous()
        T = qkv.size(0)
        dqkv = torch.empty_like(qkv)
        delta = torch.empty_like(lse)
        C.flash_attn_bwd(qkv[:, : hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:], o, grad_o, lse, delta,
                         dqkv[:, : hq * d], dqkv[:, hq * d:(hq + hkv) * d], dqkv[:, (hq + hkv) * d:], batch, seq, hq,
                         hkv, d, 1.0 / math.sqrt(d))
        if rope:
            cos, sin = rope_cache(seq, d, theta, qkv.device)
            C.rope_apply(dqkv, hq + hkv, d, seq, None, cos, sin, True)
        del T
        return dqkv, None, None, None, None, None, None, None


def attention_core(qkv: Tensor, batch: int, seq: int, hq: int, hkv: int, d: int, rope: bool, theta: float) -> Tensor:
    return _AttnCore.apply(qkv, batch, seq, hq, hkv, d, rope, theta)


def self_attention(module, x: Tensor, residual: Tensor | None = None) -> Tensor:
    """Forward of ``models.layers.Attention`` on the native path; ``residual`` is fused into the output GEMM."""
    batch, seq, hidden = x.shape
    qkv = linear(x.reshape(-1, hidden), module.in_proj_weight, module.in_proj_bias)
    o = attention_core(qkv, batch, seq, module.heads, module.kv_heads, module.head_dim, module.rope,
                       module.config.rope_theta)
    res = residual.reshape(-1, residual.size(-1)) if residual is not None else None
    out = linear(o, module.out_proj.weight, module.out_proj.bias, res)
    return out.reshape(batch, seq, -1)
