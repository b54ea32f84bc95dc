"""The native MoE layer: fp32 router, device-side capacity plan, grouped tcgen05 SwiGLU experts, deterministic
combine, and the full backward. No host synchronisation anywhere in forward or backward.

Forward   logits = x Wr^T (fp32) -> softmax/top-k/renormalise -> plan (capacity, padded segments) -> permute ->
          H = silu(X Wg^T) * (X Wu^T) [grouped GEMM, SwiGLU epilogue, raw gate/up kept or recomputed] ->
          Y = H Wd^T [grouped GEMM] -> out[t] = sum_j w_j Y[row(t,j)]
Backward  dY gathered per route -> A = dY Wd [grouped GEMM; epilogue forms dGU = (w*A) * SwiGLU', w*H and the
          per-route <A, H> partials] -> dWd = dY^T (w*H), dWgu = dGU^T X [grouped weight-gradient GEMMs] ->
          dX = dGU Wgu [grouped GEMM] -> router backward (renormalisation + softmax) -> fp32 router GEMMs.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from . import ext


@dataclass
class RoutingPlan:
    probs: Tensor        # [T, E] fp32
    top_idx: Tensor      # [T, k] int32
    top_w: Tensor        # [T, k] fp32
    counts: Tensor       # [E] int32 routes assigned per expert (before capacity)
    kept: Tensor         # [E] int32 routes kept per expert
    offsets: Tensor      # [E] int32 first padded row of each expert
    meta: Tensor         # [2] int32: total padded rows, overflow routes
    route_row: Tensor    # [T*k] int32 row of each route, -1 when dropped
    max_rows: int        # allocation bound on padded rows


def max_padded_rows(tokens: int, k: int, experts: int, capacity: int) -> int:
    kept_bound = min(tokens * k, experts * capacity)
    return ((kept_bound + 127 * experts) + 127) // 128 * 128


def route(x: Tensor, router_weight: Tensor, k: int, capacity: int, temperature: float,
          expert_bias: Optional[Tensor] = None, slot_rows: int = 0) -> RoutingPlan:
    """Router + capacity plan on the device (no host synchronisation). ``slot_rows`` > 0 lays every expert out at
    a fixed slot ``e * slot_rows`` (the expert-parallel send layout) instead of compact 128-padded segments."""
    C = ext()
    T, H = x.shape
    E = router_weight.size(0)
    dev = x.device
    logits = torch.empty(T, E, device=dev, dtype=torch.float32)
    C.router_logits(x, router_weight.float().contiguous(), logits)
    probs = torch.empty_like(logits)
    top_idx = torch.empty(T, k, device=dev, dtype=torch.int32)
    top_w = torch.empty(T, k, device=dev, dtype=torch.float32)
    counts = torch.empty(E, device=dev, dtype=torch.int32)
    bias = expert_bias.float().contiguous() if expert_bias is not None else None
    C.router_topk(logits, bias, k, temperature, probs, top_idx, top_w, counts)
    kept = torch.empty(E, device=dev, dtype=torch.int32)
    offsets = torch.empty(E, device=dev, dtype=torch.int32)
    uoffsets = torch.empty(E, device=dev, dtype=torch.int32)
    meta = torch.empty(2, device=dev, dtype=torch.int32)
    routes = T * k
    chunks = C.moe_plan_chunks(routes)
    chunk_hist = torch.empty(max(1, chunks), E, device=dev, dtype=torch.int32)
    sorted_routes = torch.empty(max(1, routes), device=dev, dtype=torch.int32)
    route_row = torch.empty(max(1, routes), device=dev, dtype=torch.int32)
    C.moe_plan(top_idx, top_w, counts, capacity, slot_rows, kept, offsets, uoffsets, meta, chunk_hist, sorted_routes,
               route_row)
    rows = E * slot_rows if slot_rows else max_padded_rows(T, k, E, capacity)
    return RoutingPlan(probs, top_idx, top_w, counts, kept, offsets, meta, route_row[:routes], rows)


class _MoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, router_weight: Tensor, w_gate_up: Tensor, w_down: Tensor, capacity: int, k: int,
                temperature: float, expert_bias: Optional[Tensor], recompute: bool):
        C = ext()
        T, H = x.shape
        E, F2, _ = w_gate_up.shape
        F = F2 // 2
        x = x.to(torch.bfloat16).contiguous()
        plan = route(x, router_weight, k, capacity, temperature, expert_bias)
        R = plan.max_rows
        dev = x.device
        x_perm = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        row_token = torch.empty(R, device=dev, dtype=torch.int32)
        row_w = torch.empty(R, device=dev, dtype=torch.float32)
        C.moe_permute(x, k, plan.route_row, plan.top_w, plan.kept, plan.offsets, x_perm, row_token, row_w)
        h = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
        gu = None if recompute else torch.empty(R, F2, device=dev, dtype=torch.bfloat16)
        C.moe_gate_up_fwd(x_perm, w_gate_up, plan.kept, plan.offsets, h, gu)
        y = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        C.moe_down_fwd(h, w_down, plan.kept, plan.offsets, y)
        del h
        out = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        C.moe_combine(y, plan.route_row, plan.top_w, None, k, out)
        saved = [x, router_weight, w_gate_up, w_down, plan.probs, plan.top_idx, plan.top_w, plan.kept, plan.offsets,
                 plan.meta, plan.route_row, row_token, row_w]
        if gu is not None:
            saved.append(gu)
        ctx.save_for_backward(*saved)
        ctx.cfg = (k, temperature, recompute, R, router_weight.dtype)
        ctx.mark_non_differentiable(plan.top_idx, plan.counts, plan.kept, plan.meta, plan.route_row)
        return out, plan.probs, plan.top_idx, plan.counts, plan.kept, plan.meta, plan.route_row

    @staticmethod
    def backward(ctx, d_out, d_probs, *_):
        C = ext()
        k, temperature, recompute, R, rw_dtype = ctx.cfg
        saved = ctx.saved_tensors
        (x, router_weight, w_gate_up, w_down, probs, top_idx, top_w, kept, offsets, meta, route_row, row_token,
         row_w) = saved[:13]
        gu = saved[13] if len(saved) > 13 else None
        T, H = x.shape
        E, F2, _ = w_gate_up.shape
        F = F2 // 2
        dev = x.device
        if d_out is None:
            d_out = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
        d_out = d_out.to(torch.bfloat16).contiguous()
        x_perm = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        C.moe_gather_rows(x, row_token, meta, x_perm)
        if gu is None:  # recompute the raw gate/up activations
            gu = torch.empty(R, F2, device=dev, dtype=torch.bfloat16)
            scratch = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
            C.moe_gate_up_fwd(x_perm, w_gate_up, kept, offsets, scratch, gu)
            del scratch
        dy_perm = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        C.moe_gather_rows(d_out, row_token, meta, dy_perm)
        tiles = C.moe_dw_tiles(F)
        dgu = torch.empty(R, F2, device=dev, dtype=torch.bfloat16)
        hw = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
        partial = torch.empty(R, tiles, device=dev, dtype=torch.float32)
        C.moe_down_bwd(dy_perm, w_down, kept, offsets, gu, row_w, dgu, hw, partial)
        del gu
        d_w_down = torch.empty_like(w_down)
        C.moe_wgrad(dy_perm, hw, kept, offsets, d_w_down, False, 1, 1.0)
        del hw, dy_perm
        d_w_gate_up = torch.empty_like(w_gate_up)
        C.moe_wgrad(dgu, x_perm, kept, offsets, d_w_gate_up, False, 1, 1.0)
        del x_perm
        dx_perm = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        C.moe_gate_up_dgrad(dgu, w_gate_up, kept, offsets, dx_perm)
        del dgu
        d_w = torch.empty(T * k, device=dev, dtype=torch.float32)
        C.moe_route_dw(partial, route_row, d_w)
        del partial
        d_logits = torch.empty_like(probs)
        dp = d_probs.float().contiguous() if d_probs is not None else None
        C.router_backward(probs, top_idx, top_w, d_w, dp, temperature, d_logits)
        rw = router_weight.float().contiguous()
        dx_router = torch.empty(T, H, device=dev, dtype=torch.float32)
        C.router_dx(d_logits, rw, dx_router)
        split = C.router_dw_split(T)
        workspace = torch.empty(max(1, split) * E * H if split > 1 else 1, device=dev, dtype=torch.float32)
        d_router = torch.empty(E, H, device=dev, dtype=torch.float32)
        C.router_dw(d_logits, x, d_router, False, workspace)
        dx = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        C.moe_combine_grad(dx_perm, route_row, dx_router, k, dx)
        return dx, d_router.to(rw_dtype), d_w_gate_up, d_w_down, None, None, None, None, None


def dequantized_stacks(moe) -> tuple[Tensor, Tensor]:
    """bf16 ``w_gate_up [E, 2F, H]`` and ``w_down [E, H, F]`` expanded from a quantised MoE's packed buffers by the
    ``dequant_rows`` kernel (int4 groups or int8 rows with fp16 scales)."""
    C = ext()
    q = moe.quant
    fmt = 2 if q["bits"] == 4 else 1
    E, F2 = moe.q_gate_up.shape[0], moe.q_gate_up.shape[1]
    H = moe.hidden_size
    F = F2 // 2
    w_gate_up = torch.empty(E, F2, H, device=moe.q_gate_up.device, dtype=torch.bfloat16)
    w_down = torch.empty(E, H, F, device=moe.q_down.device, dtype=torch.bfloat16)
    C.dequant_rows(moe.q_gate_up, moe.s_gate_up, H, q["group_in"] if fmt == 2 else H, fmt, w_gate_up)
    C.dequant_rows(moe.q_down, moe.s_down, F, q["group_down"] if fmt == 2 else F, fmt, w_down)
    return w_gate_up, w_down


def moe_forward(moe, flat: Tensor, capacity: int):
    """Native forward of ``models.moe.TopKMoE``; returns (output, probs, top_idx, overflow, kept_counts, dropped).
    Quantised experts (inference only) are expanded to bf16 first."""
    recompute = getattr(moe, "recompute_activations", False)
    if getattr(moe, "quant", None) is not None:
        w_gate_up, w_down = dequantized_stacks(moe)
    else:
        w_gate_up, w_down = moe.w_gate_up, moe.w_down
    out, probs, top_idx, counts, kept, meta, route_row = _MoEFn.apply(
        flat, moe.router.weight, w_gate_up, w_down, int(capacity), moe.top_k, float(moe.router_temperature),
        moe.expert_bias, recompute)
    moe._last_counts = counts
    overflow = meta[1].long()
    dropped = _Dropped(route_row, top_idx, moe.top_k)
    return out.to(flat.dtype), probs, top_idx.long(), overflow, kept, dropped


class _Dropped:
    """Lazily materialised (dropped token ids, dropped expert ids), only built when statistics are collected."""

    def __init__(self, route_row: Tensor, top_idx: Tensor, k: int) -> None:
        self._row, self._idx, self._k = route_row, top_idx, k

    def __getitem__(self, i: int) -> Tensor:
        mask = self._row < 0
        routes = mask.nonzero(as_tuple=True)[0]
        return routes // self._k if i == 0 else self._idx.reshape(-1)[routes].long()


def capacity_for(tokens: int, k: int, experts: int, cf: float, scale: float, min_cap: int, enforce: bool) -> int:
    if cf > 0 and enforce:
        return max(min_cap, math.ceil(tokens * k / experts * cf * scale))
    return tokens * k
