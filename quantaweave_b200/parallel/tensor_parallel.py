"""Megatron-style tensor parallelism for attention and expert FFNs (reference ``src/tensor_parallel.py``).

``copy_to_tp`` is identity forward / all-reduce backward; ``reduce_from_tp`` is all-reduce forward / identity
backward (:29-56). ``TensorParallelAttention`` keeps this rank's heads (column-parallel QKV, row-parallel output
with a replicated bias) under ``nn.MultiheadAttention`` parameter names (:72-100); GQA is supported by splitting
q, k and v heads separately. Expert FFNs are column-parallel for gate/up and row-parallel for down.
``shard_state_dict`` / ``merge_state_dicts`` slice and merge full checkpoints (:110-149).

On CUDA the attention runs on the native kernels (tcgen05 GEMMs + flash attention); the TP all-reduce is NCCL.
"""

from __future__ import annotations

import math
import re
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import QuantaWeaveConfig


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous().clone()
        dist.all_reduce(grad, group=ctx.group)
        return grad, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, grad):
        return grad, None


def copy_to_tp(x: Tensor, group) -> Tensor:
    return x if group is None else _CopyToTP.apply(x, group)


def reduce_from_tp(x: Tensor, group) -> Tensor:
    return x if group is None else _ReduceFromTP.apply(x, group)


class _RowParallelOutput(nn.Module):
    """Output projection: weight ``[hidden, local_width]`` (row-parallel slice) and a replicated bias."""

    def __init__(self, local_width: int, hidden: int, bias: bool = True) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(hidden, local_width))
        self.bias = nn.Parameter(torch.zeros(hidden)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))


class TensorParallelAttention(nn.Module):
    def __init__(self, config: QuantaWeaveConfig, context) -> None:
        super().__init__()
        tp = context.tp_size
        heads, kv = config.attention_heads, config.num_kv_heads
        if heads % tp or kv % tp:
            raise ValueError(f"attention heads {heads}/{kv} must be divisible by the tensor-parallel size {tp}")
        self.config = config
        self.tp_group = context.tp_group
        self.heads = heads // tp
        self.kv_heads = kv // tp
        self.head_dim = config.head_dim
        self.rope = config.position_embedding == "rope"
        self.local_width = self.heads * self.head_dim
        rows = (self.heads + 2 * self.kv_heads) * self.head_dim
        self.in_proj_weight = nn.Parameter(torch.empty(rows, config.hidden_size))
        self.in_proj_bias = nn.Parameter(torch.zeros(rows)) if config.attention_bias else None
        if config.init_std is None:
            nn.init.xavier_uniform_(self.in_proj_weight)
        else:
            nn.init.normal_(self.in_proj_weight, std=config.init_std)
        self.out_proj = _RowParallelOutput(self.local_width, config.hidden_size, config.attention_bias)
        if config.init_std is not None:
            nn.init.normal_(self.out_proj.weight, std=config.init_std)

    def forward(self, x: Tensor) -> Tensor:
        batch, seq, hidden = x.shape
        x = copy_to_tp(x, self.tp_group)
        if x.is_cuda:
            from ..ops.attention import attention_core
            from ..ops.linear import linear

            qkv = linear(x.reshape(-1, hidden), self.in_proj_weight, self.in_proj_bias)
            o = attention_core(qkv, batch, seq, self.heads, self.kv_heads, self.head_dim, self.rope,
                               self.config.rope_theta)
            partial = linear(o, self.out_proj.weight).reshape(batch, seq, hidden)
        else:
            from ..models.layers import apply_rope_reference, rope_tables

            qkv = F.linear(x, self.in_proj_weight, self.in_proj_bias)
            qe, ke = self.heads * self.head_dim, (self.heads + self.kv_heads) * self.head_dim
            q = qkv[..., :qe].reshape(batch, seq, self.heads, self.head_dim)
            k = qkv[..., qe:ke].reshape(batch, seq, self.kv_heads, self.head_dim)
            v = qkv[..., ke:].reshape(batch, seq, self.kv_heads, self.head_dim)
            if self.rope:
                cos, sin = rope_tables(torch.arange(seq, device=x.device), self.head_dim, self.config.rope_theta)
                q, k = apply_rope_reference(q, cos, sin), apply_rope_reference(k, cos, sin)
            if self.kv_heads != self.heads:
                k = k.repeat_interleave(self.heads // self.kv_heads, dim=2)
                v = v.repeat_interleave(self.heads // self.kv_heads, dim=2)
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
            partial = F.linear(o.transpose(1, 2).reshape(batch, seq, self.local_width), self.out_proj.weight)
        out = reduce_from_tp(partial, self.tp_group)
        return out + self.out_proj.bias.to(out.dtype) if self.out_proj.bias is not None else out


# ---- checkpoint slicing (reference key names) ---------------------------------------------------------
_QKV = re.compile(r"\.attention\.in_proj_(weight|bias)$")
_OUT_WEIGHT = re.compile(r"\.attention\.out_proj\.weight$")
_COLUMN_EXPERT = re.compile(r"\.experts\.\d+\.(gate|up)\.weight$")
_ROW_EXPERT = re.compile(r"\.experts\.\d+\.down\.weight$")


def is_tp_sharded(name: str) -> bool:
    return bool(_QKV.search(name) or _OUT_WEIGHT.search(name) or _COLUMN_EXPERT.search(name) or _ROW_EXPERT.search(name))


def is_tp_sharded_shared(name: str) -> bool:
    """TP-sharded but not an expert: replicated across the expert group, distinct across the TP group."""
    return bool(_QKV.search(name) or _OUT_WEIGHT.search(name))


def _qkv_sizes(total_rows: int, q_fraction: Optional[float]) -> tuple[int, int]:
    if q_fraction is None:
        third = total_rows // 3
        return third, third
    q = int(round(total_rows * q_fraction))
    return q, (total_rows - q) // 2


def shard_tensor(name: str, tensor: Tensor, tp_rank: int, tp_size: int, q_fraction: Optional[float] = None) -> Tensor:
    if _QKV.search(name):
        q_rows, kv_rows = _qkv_sizes(tensor.size(0), q_fraction)
        parts = tensor.split([q_rows, kv_rows, kv_rows], dim=0)
        return torch.cat([p.chunk(tp_size, dim=0)[tp_rank] for p in parts], dim=0).contiguous()
    if _OUT_WEIGHT.search(name) or _ROW_EXPERT.search(name):
        return tensor.chunk(tp_size, dim=1)[tp_rank].contiguous()
    if _COLUMN_EXPERT.search(name):
        return tensor.chunk(tp_size, dim=0)[tp_rank].contiguous()
    return tensor


def shard_state_dict(state: dict, tp_rank: int, tp_size: int, config: Optional[QuantaWeaveConfig] = None) -> dict:
    qf = None
    if config is not None and config.num_kv_heads != config.attention_heads:
        qf = config.attention_heads / (config.attention_heads + 2 * config.num_kv_heads)
    return {name: shard_tensor(name, t, tp_rank, tp_size, qf) for name, t in state.items()}


def merge_tensors(name: str, pieces: list, q_fraction: Optional[float] = None) -> Tensor:
    if _QKV.search(name):
        split = []
        for piece in pieces:
            q_rows, kv_rows = _qkv_sizes(piece.size(0), q_fraction)
            split.append(piece.split([q_rows, kv_rows, kv_rows], dim=0))
        return torch.cat([torch.cat([s[i] for s in split], dim=0) for i in range(3)], dim=0)
    if _OUT_WEIGHT.search(name) or _ROW_EXPERT.search(name):
        return torch.cat(pieces, dim=1)
    if _COLUMN_EXPERT.search(name):
        return torch.cat(pieces, dim=0)
    return pieces[0]


def merge_state_dicts(shards: list, config: Optional[QuantaWeaveConfig] = None) -> dict:
    qf = None
    if config is not None and config.num_kv_heads != config.attention_heads:
        qf = config.attention_heads / (config.attention_heads + 2 * config.num_kv_heads)
    return {name: merge_tensors(name, [s[name] for s in shards], qf) for name in shards[0]}
