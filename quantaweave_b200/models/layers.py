"""Normalisation, rotary embedding and attention layers.

Parameter names match the reference so that its checkpoints load: the norms expose ``weight``/``bias``
like ``nn.LayerNorm``; attention exposes ``in_proj_weight``/``in_proj_bias``/``out_proj`` like
``nn.MultiheadAttention`` (reference ``src/quantweave_moe_model.py:278-288``, ``src/tensor_parallel.py:75-90``).

Each module has two execution paths selected by the tensor's device:

* CPU (and any non-CUDA device): plain PyTorch fp32 math. This is the oracle every kernel is tested against.
* CUDA: the hand-written sm_100a kernels in ``quantaweave_b200.ops`` (RMSNorm/LayerNorm, RoPE, tcgen05 GEMM,
  flash attention). A CUDA tensor without the compiled extension raises instead of silently falling back.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import QuantaWeaveConfig


def _use_native(x: Tensor) -> bool:
    if not x.is_cuda:
        return False
    from ..ops import native_required

    native_required()
    return True


class Norm(nn.Module):
    """LayerNorm (weight+bias, reference default) or RMSNorm (weight only)."""

    def __init__(self, size: int, kind: str = "layernorm", eps: float = 1e-5) -> None:
        super().__init__()
        self.kind = kind
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(size))
        if kind == "layernorm":
            self.bias = nn.Parameter(torch.zeros(size))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: Tensor) -> Tensor:
        if _use_native(x):
            from ..ops import norm as norm_ops

            return norm_ops.norm(x, self.weight, self.bias, self.eps, self.kind)
        if self.kind == "layernorm":
            return F.layer_norm(x, (x.size(-1),), self.weight, self.bias, self.eps)
        return rms_norm_reference(x, self.weight, self.eps)


def rms_norm_reference(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * weight.float()).to(x.dtype)


def rope_tables(positions: Tensor, head_dim: int, theta: float) -> tuple[Tensor, Tensor]:
    """cos/sin tables ``[len(positions), head_dim/2]`` in fp32 (rotate-half convention)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=positions.device) / head_dim))
    angles = positions.to(torch.float64)[:, None] * inv[None, :]
    return angles.cos().float(), angles.sin().float()


def apply_rope_reference(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """x ``[B, S, heads, D]``; rotate-half RoPE in fp32."""
    half = x.size(-1) // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class Attention(nn.Module):
    """Causal self-attention: fused QKV projection, optional RoPE, MHA or GQA, output projection.

    ``in_proj_weight`` is ``[(Hq + 2*Hkv) * D, hidden]`` (rows: all q heads, then k heads, then v heads),
    identical to ``nn.MultiheadAttention``'s packing when Hkv == Hq. ``tp_size`` > 1 keeps this rank's slice of
    the heads (column-parallel QKV, row-parallel output; the caller reduces the output).
    """

    def __init__(self, config: QuantaWeaveConfig, tp_size: int = 1, tp_rank: int = 0) -> None:
        super().__init__()
        heads, kv_heads, head_dim = config.attention_heads, config.num_kv_heads, config.head_dim
        if heads % tp_size or kv_heads % tp_size:
            raise ValueError(f"attention heads {heads}/{kv_heads} must be divisible by the tensor-parallel size {tp_size}")
        self.config = config
        self.tp_size = tp_size
        self.heads = heads // tp_size
        self.kv_heads = kv_heads // tp_size
        self.head_dim = head_dim
        self.embed_dim = config.hidden_size
        self.rope = config.position_embedding == "rope"
        qkv_rows = (self.heads + 2 * self.kv_heads) * head_dim
        self.in_proj_weight = nn.Parameter(torch.empty(qkv_rows, config.hidden_size))
        if config.attention_bias:
            self.in_proj_bias = nn.Parameter(torch.zeros(qkv_rows))
        else:
            self.register_parameter("in_proj_bias", None)
        self.out_proj = nn.Linear(self.heads * head_dim, config.hidden_size, bias=config.attention_bias)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        std = self.config.init_std
        if std is None:
            # nn.MultiheadAttention's own initialisation (xavier on the packed projection, zero biases)
            full_rows = (self.config.attention_heads + 2 * self.config.num_kv_heads) * self.head_dim
            bound = math.sqrt(6.0 / (full_rows + self.embed_dim))
            nn.init.uniform_(self.in_proj_weight, -bound, bound)
            nn.init.kaiming_uniform_(self.out_proj.weight, a=math.sqrt(5))
        else:
            nn.init.normal_(self.in_proj_weight, std=std)
            nn.init.normal_(self.out_proj.weight, std=std)
        if self.in_proj_bias is not None:
            nn.init.zeros_(self.in_proj_bias)
        if self.out_proj.bias is not None:
            nn.init.zeros_(self.out_proj.bias)

    def qkv(self, x: Tensor, positions: Optional[Tensor] = None) -> tuple[Tensor, Tensor, Tensor]:
        """Projected (and rotated) q ``[B,S,Hq,D]``, k/v ``[B,S,Hkv,D]`` on the oracle path."""
        batch, seq, _ = x.shape
        qkv = F.linear(x, self.in_proj_weight, self.in_proj_bias)
        q_end = self.heads * self.head_dim
        k_end = q_end + self.kv_heads * self.head_dim
        q = qkv[..., :q_end].reshape(batch, seq, self.heads, self.head_dim)
        k = qkv[..., q_end:k_end].reshape(batch, seq, self.kv_heads, self.head_dim)
        v = qkv[..., k_end:].reshape(batch, seq, self.kv_heads, self.head_dim)
        if self.rope:
            if positions is None:
                positions = torch.arange(seq, device=x.device)
            cos, sin = rope_tables(positions, self.head_dim, self.config.rope_theta)
            q = apply_rope_reference(q, cos, sin)
            k = apply_rope_reference(k, cos, sin)
        return q, k, v

    def forward(self, x: Tensor) -> Tensor:
        if _use_native(x):
            from ..ops import attention as attn_ops

            return attn_ops.self_attention(self, x)
        batch, seq, _ = x.shape
        q, k, v = self.qkv(x)
        if self.kv_heads != self.heads:
            repeat = self.heads // self.kv_heads
            k = k.repeat_interleave(repeat, dim=2)
            v = v.repeat_interleave(repeat, dim=2)
        out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        out = out.transpose(1, 2).reshape(batch, seq, self.heads * self.head_dim)
        return self.out_proj(out)
