"""Megatron-style tensor parallelism for attention and expert FFNs (reference ``src/tensor_parallel.py``).

``copy_to_tp`` is identity forward / all-reduce backward; ``reduce_from_tp`` is all-reduce forward / identity
backward (:29-56). ``TensorParallelAttention`` keeps this rank's heads (column-parallel QKV, row-parallel output
with a replicated bias) under ``nn.MultiheadAttention`` parameter names (:72-100); GQA is supported by splitting
q, k and v heads separately. Expert FFNs are column-parallel for gate/up and row-parallel for down.
``shard_state_dict`` / ``merge_state_dicts`` slice and merge full checkpoints (:110-149).

On CUDA the attention runs on the native kernels (tcgen05 GEMMs + flash attention). Its two all-reduces are fused
into the neighbouring GEMMs over NVLink peer memory (``FusedTPReducer``): the row-parallel output projection's GEMM
stores each partial row straight into the owning rank's staging buffer and a reduction kernel sums the slots and
stores the result into every rank's output buffer (forward); the column-parallel input projection does the same with
its dgrad GEMM (backward). Under sequence parallelism the all-gather of the token rows is done by NVLink peer stores
and the reduce-scatter is fused into the producing GEMM the same way (each rank reduces only its own rows).
``QW_TP_FUSED=0`` keeps NCCL collectives; the expert FFNs' all-reduce stays on NCCL.
"""

from __future__ import annotations

import math
import os
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


def _all_gather_rows(x: Tensor, group) -> Tensor:
    world = dist.get_world_size(group)
    x = x.contiguous()
    out = x.new_empty((x.size(0) * world,) + tuple(x.shape[1:]))
    if x.is_cuda:
        dist.all_gather_into_tensor(out, x, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), x, group=group)
    return out


def _reduce_scatter_rows(x: Tensor, group) -> Tensor:
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    x = x.contiguous()
    if x.is_cuda:
        out = x.new_empty((x.size(0) // world,) + tuple(x.shape[1:]))
        dist.reduce_scatter_tensor(out, x, group=group)
        return out
    summed = x.clone()  # gloo has no reduce-scatter
    dist.all_reduce(summed, group=group)
    return summed.chunk(world)[rank].contiguous()


class _GatherRows(torch.autograd.Function):
    """Sequence parallelism: token rows sharded over the group -> all rows (backward: reduce-scatter)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather_rows(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _reduce_scatter_rows(grad, ctx.group), None


class _ScatterRows(torch.autograd.Function):
    """Sequence parallelism: per-rank partial sums of all rows -> this rank's rows, summed (backward: all-gather)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter_rows(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _all_gather_rows(grad, ctx.group), None


def copy_to_tp(x: Tensor, group) -> Tensor:
    return x if group is None else _CopyToTP.apply(x, group)


def reduce_from_tp(x: Tensor, group) -> Tensor:
    return x if group is None else _ReduceFromTP.apply(x, group)


class FusedTPReducer:
    """All-reduce fused with the producing GEMM over NVLink peer memory (one per (group, device)).

    Buffers come from ``_Channel`` (two parities of symmetric memory, so back-to-back calls never overwrite a slot a
    slower rank is still reading): ``[0, plane)`` is this rank's staging area ``[world][M/world][N]`` and
    ``[plane, 2 plane)`` the reduced ``[M, N]`` output. Per call: GEMM with peer-store epilogue -> ready barrier ->
    ``tp_reduce_bcast`` (fixed-order fp32 sum of the slots + bias, stored into every rank's output) -> done barrier ->
    copy out. Creating one is collective over the group."""

    _instances: dict = {}

    def __init__(self, group, device: torch.device) -> None:
        from .p2p import P2PTransport, _Channel

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.transport = P2PTransport.for_group(group, device)
        self.ready = _Channel(self.transport)
        self.done = _Channel(self.transport)
        self._arrivals = torch.zeros(self.world, dtype=torch.int32, device=device)  # per-destination block counters

    @classmethod
    def for_group(cls, group, device: torch.device) -> "FusedTPReducer":
        key = (id(group), device.index)
        if key not in cls._instances:
            cls._instances[key] = cls(group, device)
        return cls._instances[key]

    @staticmethod
    def usable(x: Tensor, group, width: int) -> bool:
        if group is None or not x.is_cuda or os.environ.get("QW_TP_FUSED", "1") == "0":
            return False
        world = dist.get_world_size(group)
        return world > 1 and x.size(0) % world == 0 and width % 8 == 0

    def gemm_all_reduce(self, a: Tensor, w: Tensor, bias: Optional[Tensor], transposed: bool) -> Tensor:
        """``sum over ranks of (a @ w^T)`` (``a @ w`` when ``transposed``) ``+ bias`` as bf16 ``[M, N]``."""
        from ..ops import ext

        C = ext()
        M = a.size(0)
        N = w.size(1) if transposed else w.size(0)
        rows = M // self.world
        plane = M * N * 2
        self.ready.grow(2 * plane)  # same size on every rank: M and N are replicated across the group
        parity = self.ready.next()
        buf, _, peers = self.ready.bufs[parity]
        if transposed:
            C.linear_dgrad_peer(a, w, peers, rows, self.rank)
        else:
            C.linear_fwd_peer(a, w, peers, rows, self.rank)
        C.ep_signal(self.ready.peer_flags[parity], self.rank, self.ready.epoch)
        self.ready.wait(parity)  # every rank's partial rows have landed in our staging slots
        C.tp_reduce_bcast(buf[:plane].view(torch.bfloat16), self.world, rows, N, bias, peers + plane, self.rank)
        done = self.done.next()
        C.ep_signal(self.done.peer_flags[done], self.rank, self.done.epoch)
        self.done.wait(done)  # every rank's reduced rows have landed in our output buffer
        return buf[plane:2 * plane].view(torch.bfloat16).view(M, N).clone()

    def gemm_reduce_scatter(self, a: Tensor, w: Tensor, bias: Optional[Tensor], transposed: bool) -> Tensor:
        """This rank's rows of ``sum over ranks of (a @ w^T)`` (``a @ w`` when ``transposed``) ``+ bias``: the GEMM
        epilogue stores every partial row into its owner's staging slot over NVLink; after the ready barrier each rank
        sums its own rows over the slots in a fixed rank order. ``[M / world, N]`` bf16."""
        from ..ops import ext

        C = ext()
        M = a.size(0)
        N = w.size(1) if transposed else w.size(0)
        rows = M // self.world
        plane = M * N * 2
        self.ready.grow(plane)
        parity = self.ready.next()
        buf, _, peers = self.ready.bufs[parity]
        if transposed:
            C.linear_dgrad_peer(a, w, peers, rows, self.rank)
        else:
            C.linear_fwd_peer(a, w, peers, rows, self.rank)
        C.ep_signal(self.ready.peer_flags[parity], self.rank, self.ready.epoch)
        self.ready.wait(parity)  # every rank's partial rows of our block have landed
        out = torch.empty(rows, N, device=a.device, dtype=torch.bfloat16)
        C.tp_reduce_rows(buf[:plane].view(torch.bfloat16), self.world, rows, N, bias, out)
        return out

    def all_gather_rows(self, x: Tensor) -> Tensor:
        """``[rows, H]`` of every rank, rank-major ``[world * rows, H]``: each rank stores its rows into every peer's
        buffer with NVLink stores and releases a flag; after the wait the gathered rows are copied out of the
        two-parity buffer (they outlive its next reuse when autograd saves them)."""
        from ..ops import ext

        x = x.contiguous()
        nbytes = x.numel() * x.element_size()
        self.ready.grow(nbytes * self.world)
        parity = self.ready.next()
        buf, _, peers = self.ready.bufs[parity]
        ext().p2p_broadcast(x, peers, self.ready.peer_flags[parity], self.rank, self.ready.epoch, self._arrivals)
        self.ready.wait(parity)
        return buf[:nbytes * self.world].view(x.dtype).view(self.world * x.size(0), *x.shape[1:]).clone()


def _bf16_rows(t: Tensor) -> Tensor:
    t = t.reshape(-1, t.size(-1)).to(torch.bfloat16)
    return t if t.stride(-1) == 1 and t.stride(0) % 8 == 0 else t.contiguous()


def _local_weight_grads(ctx, g2: Tensor, x2: Tensor, w: Tensor):
    from ..ops import ext

    C = ext()
    dw = db = None
    if ctx.needs_input_grad[1]:
        dw = torch.empty(w.size(0), w.size(1), device=g2.device, dtype=ctx.weight_dtype
                         if ctx.weight_dtype in (torch.bfloat16, torch.float32) else torch.float32)
        C.linear_wgrad(g2, x2, dw, False)
    if ctx.bias_dtype is not None and ctx.needs_input_grad[2]:
        db = torch.empty(g2.size(1), device=g2.device, dtype=torch.float32)
        part = torch.empty(C.bias_grad_slabs(g2.size(0)), g2.size(1), device=g2.device, dtype=torch.float32)
        C.bias_grad(g2, part, db, False)
        db = db.to(ctx.bias_dtype)
    return dw, db


class _RowParallelAllReduce(torch.autograd.Function):
    """``sum_r(x_r W_r^T) + b`` with the all-reduce fused into the GEMM; the backward is local (the conjugate of the
    all-reduce is the identity)."""

    @staticmethod
    def forward(ctx, x, weight, bias, reducer):
        x2 = _bf16_rows(x)
        w = weight.to(torch.bfloat16).contiguous()
        out = reducer.gemm_all_reduce(x2, w, bias.float() if bias is not None else None, False)
        ctx.save_for_backward(x2, w)
        ctx.weight_dtype, ctx.bias_dtype = weight.dtype, (bias.dtype if bias is not None else None)
        return out

    @staticmethod
    def backward(ctx, grad):
        from ..ops import ext

        x2, w = ctx.saved_tensors
        g2 = _bf16_rows(grad)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(x2.size(0), w.size(1), device=grad.device, dtype=torch.bfloat16)
            ext().linear_dgrad(g2, w, dx, False)
        dw, db = _local_weight_grads(ctx, g2, x2, w)
        return dx, dw, db, None


class _ColumnParallelInput(torch.autograd.Function):
    """``x W_r^T + b_r`` for a replicated ``x``; the backward all-reduce of ``dx = sum_r dy_r W_r`` is fused into the
    dgrad GEMM."""

    @staticmethod
    def forward(ctx, x, weight, bias, reducer):
        from ..ops import ext

        x2 = _bf16_rows(x)
        w = weight.to(torch.bfloat16).contiguous()
        out = torch.empty(x2.size(0), w.size(0), device=x.device, dtype=torch.bfloat16)
        ext().linear_fwd(x2, w, bias.float() if bias is not None else None, None, out)
        ctx.save_for_backward(x2, w)
        ctx.reducer = reducer
        ctx.weight_dtype, ctx.bias_dtype = weight.dtype, (bias.dtype if bias is not None else None)
        return out

    @staticmethod
    def backward(ctx, grad):
        x2, w = ctx.saved_tensors
        g2 = _bf16_rows(grad)
        dx = ctx.reducer.gemm_all_reduce(g2, w, None, True) if ctx.needs_input_grad[0] else None
        dw, db = _local_weight_grads(ctx, g2, x2, w)
        return dx, dw, db, None


class _SPGatherLinear(torch.autograd.Function):
    """Sequence parallelism, column-parallel input projection: ``(all rows of x) @ W_r^T + b_r`` where each rank holds
    only its token rows of ``x``. The row all-gather is done by NVLink peer stores into symmetric memory (no NCCL);
    in backward the dgrad GEMM stores each partial input-gradient row into its owner's staging slot and every rank
    reduces its own rows — the reduce-scatter is fused into the GEMM."""

    @staticmethod
    def forward(ctx, x, weight, bias, reducer):
        from ..ops import ext

        full = reducer.all_gather_rows(_bf16_rows(x))
        w = weight.to(torch.bfloat16).contiguous()
        out = torch.empty(full.size(0), w.size(0), device=x.device, dtype=torch.bfloat16)
        ext().linear_fwd(full, w, bias.float() if bias is not None else None, None, out)
        ctx.save_for_backward(full, w)
        ctx.reducer = reducer
        ctx.weight_dtype, ctx.bias_dtype = weight.dtype, (bias.dtype if bias is not None else None)
        return out

    @staticmethod
    def backward(ctx, grad):
        full, w = ctx.saved_tensors
        g2 = _bf16_rows(grad)
        dx = ctx.reducer.gemm_reduce_scatter(g2, w, None, True) if ctx.needs_input_grad[0] else None
        dw, db = _local_weight_grads(ctx, g2, full, w)
        return dx, dw, db, None


class _SPLinearScatter(torch.autograd.Function):
    """Sequence parallelism, row-parallel output projection: ``o_r @ W_r^T`` over all rows, reduce-scattered to this
    rank's rows inside the GEMM (peer-store epilogue + fixed-order local reduction); in backward the row gradients
    are all-gathered by NVLink peer stores and the dgrad / wgrad GEMMs run locally."""

    @staticmethod
    def forward(ctx, o, weight, reducer):
        o2 = _bf16_rows(o)
        w = weight.to(torch.bfloat16).contiguous()
        out = reducer.gemm_reduce_scatter(o2, w, None, False)
        ctx.save_for_backward(o2, w)
        ctx.reducer = reducer
        ctx.weight_dtype, ctx.bias_dtype = weight.dtype, None
        return out

    @staticmethod
    def backward(ctx, grad):
        from ..ops import ext

        o2, w = ctx.saved_tensors
        g_full = ctx.reducer.all_gather_rows(_bf16_rows(grad))
        do = None
        if ctx.needs_input_grad[0]:
            do = torch.empty(o2.size(0), w.size(1), device=grad.device, dtype=torch.bfloat16)
            ext().linear_dgrad(g_full, w, do, False)
        dw, _ = _local_weight_grads(ctx, g_full, o2, w)
        return do, dw, None


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
        # sequence parallelism: the input holds this rank's token rows; ``sp_shape`` = (batch, sequence) of the whole
        # batch is set by the model before each forward
        self.sequence_parallel = bool(getattr(context, "sequence_parallel", False))
        self.sp_shape: Optional[tuple] = None
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
        if self.sequence_parallel:
            return self._forward_sequence_parallel(x)
        batch, seq, hidden = x.shape
        if FusedTPReducer.usable(x.reshape(-1, hidden), self.tp_group, hidden):
            from ..ops.attention import attention_core

            reducer = FusedTPReducer.for_group(self.tp_group, x.device)
            qkv = _ColumnParallelInput.apply(x.reshape(-1, hidden), self.in_proj_weight, self.in_proj_bias, reducer)
            o = attention_core(qkv, batch, seq, self.heads, self.kv_heads, self.head_dim, self.rope,
                               self.config.rope_theta)
            out = _RowParallelAllReduce.apply(o, self.out_proj.weight, self.out_proj.bias, reducer)
            return out.reshape(batch, seq, hidden)
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

    def _heads_partial(self, full: Tensor, batch: int, seq: int) -> Tensor:
        """This rank's heads over all rows ``full`` [batch*seq, hidden] -> row-parallel partial output (no bias)."""
        hidden = full.size(-1)
        if full.is_cuda:
            from ..ops.attention import attention_core
            from ..ops.linear import linear

            qkv = linear(full, self.in_proj_weight, self.in_proj_bias)
            o = attention_core(qkv, batch, seq, self.heads, self.kv_heads, self.head_dim, self.rope,
                               self.config.rope_theta)
            return linear(o, self.out_proj.weight)
        from ..models.layers import apply_rope_reference, rope_tables

        qkv = F.linear(full.reshape(batch, seq, hidden), self.in_proj_weight, self.in_proj_bias)
        qe, ke = self.heads * self.head_dim, (self.heads + self.kv_heads) * self.head_dim
        q = qkv[..., :qe].reshape(batch, seq, self.heads, self.head_dim)
        k = qkv[..., qe:ke].reshape(batch, seq, self.kv_heads, self.head_dim)
        v = qkv[..., ke:].reshape(batch, seq, self.kv_heads, self.head_dim)
        if self.rope:
            cos, sin = rope_tables(torch.arange(seq, device=full.device), self.head_dim, self.config.rope_theta)
            q, k = apply_rope_reference(q, cos, sin), apply_rope_reference(k, cos, sin)
        if self.kv_heads != self.heads:
            k = k.repeat_interleave(self.heads // self.kv_heads, dim=2)
            v = v.repeat_interleave(self.heads // self.kv_heads, dim=2)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return F.linear(o.transpose(1, 2).reshape(batch * seq, self.local_width), self.out_proj.weight)

    def _forward_sequence_parallel(self, x: Tensor) -> Tensor:
        """``x``: this rank's token rows (any leading shape, ``rows x hidden``). All-gather the rows, run this rank's
        heads over the whole batch, reduce-scatter the row-parallel output back to this rank's rows."""
        if self.sp_shape is None:
            raise RuntimeError("sequence-parallel attention needs the batch shape (set by the model's forward)")
        batch, seq = self.sp_shape
        shape, hidden = x.shape, x.size(-1)
        rows = x.reshape(-1, hidden)
        if FusedTPReducer.usable(rows, self.tp_group, hidden):
            from ..ops.attention import attention_core

            reducer = FusedTPReducer.for_group(self.tp_group, x.device)
            qkv = _SPGatherLinear.apply(rows, self.in_proj_weight, self.in_proj_bias, reducer)
            o = attention_core(qkv, batch, seq, self.heads, self.kv_heads, self.head_dim, self.rope,
                               self.config.rope_theta)
            out = _SPLinearScatter.apply(o, self.out_proj.weight, reducer)
            if self.out_proj.bias is not None:
                out = out + self.out_proj.bias.to(out.dtype)
            return out.reshape(shape)
        full = _GatherRows.apply(x.reshape(-1, hidden), self.tp_group)
        partial = self._heads_partial(full, batch, seq)
        out = _ScatterRows.apply(partial, self.tp_group)
        if self.out_proj.bias is not None:
            out = out + self.out_proj.bias.to(out.dtype)
        return out.reshape(shape)


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
