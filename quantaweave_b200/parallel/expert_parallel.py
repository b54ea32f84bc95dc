"""Expert parallelism (optionally with tensor parallelism) on one node.

API and semantics follow the reference ``src/expert_parallel.py``: ranks form a grid
``global_rank = ep_rank * T + tp_rank`` (:69-101); experts are sharded over the expert-parallel group; capacity is
enforced per *source* rank on its local batch (:14); replicated gradients are averaged over the expert group and
expert gradients are scaled by ``1/ep`` (:203-224); clipping uses the true global norm (:227-260); the straggler
controller biases routers away from slow ranks (:280-384).

B200 native path (``_SlotDispatch``): each source rank plans capacity on the device into FIXED slots
(expert ``e`` at rows ``e * slot``, ``slot = roundup(capacity, 128)``), so the dispatch and the combine are even
exchanges whose sizes never need a host synchronisation. The receiving rank sees a ``[source, local expert, slot]``
buffer and runs the grouped tcgen05 SwiGLU GEMMs over ``source x local-expert`` groups (group ``g`` uses expert
``g % local``); weight gradients reduce each expert over the per-source segments inside one GEMM. The exchange
itself is pluggable: NCCL ``all_to_all_single`` (the baseline), the peer-store exchange of ``parallel.p2p``
(``p2p``), or the fused transport (``fused``): the permute kernel stores routed rows, weights and counts straight
into the owners' receive buffers, the expert GEMMs write their outputs into a symmetric return buffer, and the
combine kernel pulls each token's expert rows over NVLink and reduces them (``csrc/ep_fused.cu``).

The CPU (gloo) path keeps the reference's algorithm with uneven differentiable all-to-alls; it is the oracle the
multi-process tests compare against single-device training.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from ..config import QuantaWeaveConfig
from ..models.moe import TopKMoE


@dataclass
class ExpertParallelContext:
    rank: int
    world_size: int
    device: torch.device
    group: Optional[object] = None
    owns_process_group: bool = False
    tp_rank: int = 0
    tp_size: int = 1
    tp_group: Optional[object] = None
    global_rank: int = -1
    global_size: int = -1
    transport: str = "nccl"  # native dispatch: "nccl" (all_to_all), "p2p" (peer-store exchange) or "fused"
    # orthogonal mapping: attention tensor-parallel and experts expert-parallel over the SAME ranks (tp == ep ==
    # world). Activations between the attention blocks are sharded by token rows (sequence parallelism); the
    # experts are not tensor-split.
    sequence_parallel: bool = False

    def __post_init__(self) -> None:
        if self.global_size < 0:
            self.global_size = self.world_size if self.sequence_parallel else self.world_size * self.tp_size
        if self.global_rank < 0:
            self.global_rank = self.rank if self.sequence_parallel else self.rank * self.tp_size + self.tp_rank

    def layout(self) -> dict:
        out = {"kind": "ep", "ep_rank": self.rank, "ep_size": self.world_size, "tp_rank": self.tp_rank,
               "tp_size": self.tp_size}
        if self.sequence_parallel:
            out["sequence_parallel"] = True
        return out

    @property
    def group_root(self) -> int:
        return dist.get_global_rank(self.group, 0) if self.group is not None else 0


def init_expert_parallel(device_arg: str = "auto", tensor_parallel: int = 1,
                         transport: Optional[str] = None, sequence_parallel: bool = False) -> ExpertParallelContext:
    """Join (or create) the process group from torchrun's environment and build the EP x TP grid.

    ``sequence_parallel`` selects the orthogonal mapping instead of the grid: attention tensor-parallel over all
    ranks and experts expert-parallel over the same ranks (``tensor_parallel`` must equal the world size)."""
    from .groups import ensure_process_group

    owns, device = ensure_process_group(device_arg)
    world, rank = dist.get_world_size(), dist.get_rank()
    if sequence_parallel:
        if tensor_parallel != world:
            raise ValueError(f"sequence parallelism maps attention TP and expert EP onto the same ranks: "
                             f"--tensor-parallel must equal the world size {world} (got {tensor_parallel})")
        group = dist.new_group(list(range(world)))
        transport = transport or os.environ.get("QW_EP_TRANSPORT", "auto")
        if transport == "auto":
            transport = "fused" if device.type == "cuda" else "nccl"
        return ExpertParallelContext(rank, world, device, group, owns, rank, world, group, rank, world, transport,
                                     sequence_parallel=True)
    if tensor_parallel < 1 or world % tensor_parallel:
        raise ValueError(f"world size {world} is not divisible by --tensor-parallel {tensor_parallel}")
    ep_size = world // tensor_parallel
    ep_rank, tp_rank = divmod(rank, tensor_parallel)
    ep_group = tp_group = None
    if tensor_parallel > 1:
        for column in range(tensor_parallel):
            g = dist.new_group([row * tensor_parallel + column for row in range(ep_size)])
            ep_group = g if column == tp_rank else ep_group
        for row in range(ep_size):
            g = dist.new_group([row * tensor_parallel + column for column in range(tensor_parallel)])
            tp_group = g if row == ep_rank else tp_group
    transport = transport or os.environ.get("QW_EP_TRANSPORT", "auto")
    if transport == "auto":  # measured on 8 B200s (moe-1b-e64): the fused exchange beats the NCCL all-to-all
        transport = "fused" if device.type == "cuda" else "nccl"
    return ExpertParallelContext(ep_rank, ep_size, device, ep_group, owns, tp_rank, tensor_parallel, tp_group, rank,
                                 world, transport)


# ------------------------------------------------------------------------------------------ reference-style exchange
def _exchange(x: Tensor, send: list, recv: list, group) -> Tensor:
    """Uneven row exchange: ``send[r]`` leading rows of ``x`` go to rank ``r``; ``recv[r]`` rows arrive from it."""
    x = x.contiguous()
    out = x.new_empty((sum(recv), *x.shape[1:]))
    dist.all_to_all_single(out, x, output_split_sizes=recv, input_split_sizes=send, group=group)
    return out


class _AllToAll(torch.autograd.Function):
    """Differentiable :func:`_exchange` (CPU / gloo oracle path): the gradient takes the same route backwards, so the
    backward is the exchange with the two split lists swapped."""

    @staticmethod
    def forward(ctx, x: Tensor, send: list, recv: list, group):
        ctx.route = (recv, send, group)
        return _exchange(x, send, recv, group)

    @staticmethod
    def backward(ctx, grad: Tensor):
        return _exchange(grad, *ctx.route), None, None, None


def _even_exchange(x: Tensor, group) -> Tensor:
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x.contiguous(), group=group)
    return out


# ------------------------------------------------------------------------------------------ native slot dispatch
class _SlotDispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, router_weight: Tensor, w_gate_up: Tensor, w_down: Tensor, moe: "ExpertParallelMoE",
                capacity: int):
        from ..ops import ext
        from ..ops.moe import route

        C = ext()
        ep = moe.context
        world, local = ep.world_size, moe.num_local_experts
        T, H = x.shape
        E = moe.num_experts
        F2 = w_gate_up.size(1)
        F = F2 // 2
        k = moe.top_k
        dev = x.device
        slot = (capacity + 127) // 128 * 128
        x = x.to(torch.bfloat16).contiguous()
        plan = route(x, router_weight, k, capacity, float(moe.router_temperature), moe.expert_bias, slot_rows=slot)
        rows = E * slot
        transport = moe.transport()
        fused = getattr(transport, "dispatch", None) is not None
        store = None
        if fused:  # permute + exchange in one kernel, straight into the owners' persistent layer stores
            store = transport.store_for(id(moe), rows, H, world * local, hold=any(ctx.needs_input_grad[:4]))
            x_recv, w_recv, recv_counts = transport.dispatch(x, plan.route_row, plan.top_w, plan.kept, k, E, local,
                                                             slot, store=store)
            row_token = torch.empty(0, device=dev, dtype=torch.int32)
        else:
            send = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
            row_token = torch.full((rows,), -1, device=dev, dtype=torch.int32)
            row_w = torch.zeros(rows, device=dev, dtype=torch.float32)
            C.moe_permute(x, k, plan.route_row, plan.top_w, plan.kept, plan.offsets, send, row_token, row_w)
            recv_counts = transport.exchange_counts(plan.kept)            # [world * local] (source-major)
            x_recv = transport.exchange(send)                             # [world * local * slot, H]
            w_recv = transport.exchange(row_w)
        offsets = moe.recv_offsets(slot, dev)
        h = torch.empty(rows, F, device=dev, dtype=torch.bfloat16)
        gu = None if moe.recompute_activations else torch.empty(rows, F2, device=dev, dtype=torch.bfloat16)
        C.moe_gate_up_fwd(x_recv, w_gate_up, recv_counts, offsets, h, gu)
        out = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        if fused:  # the down GEMM stores each expert output row into its source rank's return buffer
            y_back, peers = transport.return_buffer(rows, H)
            C.moe_down_fwd_peer(h, w_down, recv_counts, offsets, peers, local * slot, transport.me)
            del h
            transport.publish()
            transport.wait_returned()
            C.moe_combine(y_back, plan.route_row, plan.top_w, None, k, out)
            if moe.tp_size > 1:  # EP x TP grid: each rank's experts hold a slice of F, so the outputs are partial
                dist.all_reduce(out, group=ep.tp_group)
        else:
            y = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
            C.moe_down_fwd(h, w_down, recv_counts, offsets, y)
            del h
            y_back = transport.exchange(y)
            C.moe_combine(y_back, plan.route_row, plan.top_w, None, k, out)
            if moe.tp_size > 1:
                dist.all_reduce(out, group=ep.tp_group)
        saved = [x, router_weight, w_gate_up, w_down, plan.probs, plan.top_idx, plan.top_w, plan.meta, plan.route_row,
                 row_token, recv_counts, offsets, x_recv, w_recv]
        if gu is not None:
            saved.append(gu)
        ctx.save_for_backward(*saved)
        ctx.moe, ctx.slot = moe, slot
        ctx.store = _StoreHold(transport, store) if store is not None and store.held else None
        ctx.mark_non_differentiable(plan.top_idx, plan.counts, plan.kept, plan.meta, plan.route_row)
        return out, plan.probs, plan.top_idx, plan.counts, plan.kept, plan.meta, plan.route_row

    @staticmethod
    def backward(ctx, d_out, d_probs, *_):
        from ..ops import ext

        C = ext()
        moe, slot = ctx.moe, ctx.slot
        saved = ctx.saved_tensors
        (x, router_weight, w_gate_up, w_down, probs, top_idx, top_w, meta, route_row, row_token, recv_counts, offsets,
         x_recv, w_recv) = saved[:14]
        gu = saved[14] if len(saved) > 14 else None
        ep = moe.context
        world, local = ep.world_size, moe.num_local_experts
        T, H = x.shape
        F2 = w_gate_up.size(1)
        F = F2 // 2
        k = moe.top_k
        dev = x.device
        rows = x_recv.size(0)
        transport = moe.transport()
        if d_out is None:
            d_out = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
        d_out = d_out.to(torch.bfloat16).contiguous()
        fused = getattr(transport, "dispatch", None) is not None
        if fused:
            dy_recv, _, _ = transport.dispatch(d_out, route_row, None, None, k, moe.num_experts, local, slot,
                                               pad_counts=recv_counts)
        else:
            dy_send = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
            C.moe_gather_rows(d_out, row_token, meta, dy_send)
            dy_recv = transport.exchange(dy_send)
            del dy_send
        if gu is None:
            gu = torch.empty(rows, F2, device=dev, dtype=torch.bfloat16)
            scratch = torch.empty(rows, F, device=dev, dtype=torch.bfloat16)
            C.moe_gate_up_fwd(x_recv, w_gate_up, recv_counts, offsets, scratch, gu)
            del scratch
        tiles = C.moe_dw_tiles(F)
        dgu = torch.empty(rows, F2, device=dev, dtype=torch.bfloat16)
        hw = torch.empty(rows, F, device=dev, dtype=torch.bfloat16)
        partial = torch.zeros(rows, tiles, device=dev, dtype=torch.float32)
        C.moe_down_bwd(dy_recv, w_down, recv_counts, offsets, gu, w_recv, dgu, hw, partial)
        del gu
        if moe.tp_size > 1:  # <dH, H> per row summed over the F slices of the tensor-parallel row of ranks
            dist.all_reduce(partial, group=ep.tp_group)
        d_w_down = torch.empty_like(w_down)
        C.moe_wgrad(dy_recv, hw, recv_counts, offsets, d_w_down, False, world, 1.0)
        del hw, dy_recv
        d_w_gate_up = torch.empty_like(w_gate_up)
        C.moe_wgrad(dgu, x_recv, recv_counts, offsets, d_w_gate_up, False, world, 1.0)
        if fused:  # the input-gradient GEMM stores each row into its source rank's return buffer
            dx_back, peers = transport.return_buffer(rows, H)
            C.moe_gate_up_dgrad_peer(dgu, w_gate_up, recv_counts, offsets, peers, local * slot, transport.me)
            del dgu
            transport.publish()
            partial_back = transport.exchange(partial)
            transport.wait_returned()
            if ctx.store is not None:
                ctx.store.release()
        else:
            dx_recv = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
            C.moe_gate_up_dgrad(dgu, w_gate_up, recv_counts, offsets, dx_recv)
            del dgu
            dx_back = transport.exchange(dx_recv)
            partial_back = transport.exchange(partial)
        d_w = torch.empty(T * k, device=dev, dtype=torch.float32)
        C.moe_route_dw(partial_back, route_row, d_w)
        d_logits = torch.empty_like(probs)
        dp = d_probs.float().contiguous() if d_probs is not None else None
        C.router_backward(probs, top_idx, top_w, d_w, dp, float(moe.router_temperature), d_logits)
        rw = router_weight.float().contiguous()
        dx_router = torch.empty(T, H, device=dev, dtype=torch.float32)
        C.router_dx(d_logits, rw, dx_router)
        split = C.router_dw_split(T)
        workspace = torch.empty(split * moe.num_experts * H if split > 1 else 1, device=dev, dtype=torch.float32)
        d_router = torch.empty(moe.num_experts, H, device=dev, dtype=torch.float32)
        C.router_dw(d_logits, x, d_router, False, workspace)
        dx = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        if moe.tp_size > 1:  # the expert part of dx is partial over the F slices; the router part is replicated
            C.moe_combine_grad(dx_back, route_row, None, k, dx)
            dist.all_reduce(dx, group=ep.tp_group)
            dx += dx_router.to(torch.bfloat16)
        else:
            C.moe_combine_grad(dx_back, route_row, dx_router, k, dx)
        return dx, d_router.to(router_weight.dtype), d_w_gate_up, d_w_down, None, None


class _StoreHold:
    """Keeps a layer's persistent receive store marked busy until its backward has read it, or until the autograd
    graph holding it is freed without a backward (then the store is free for the next forward)."""

    def __init__(self, transport, store) -> None:
        self.transport, self.store = transport, store

    def release(self) -> None:
        if self.store is not None:
            self.transport.release(self.store)
            self.store = None

    def __del__(self) -> None:
        self.release()


class NcclTransport:
    """Even exchanges over NCCL ``all_to_all_single`` (the baseline the fused P2P transport replaces)."""

    def __init__(self, group) -> None:
        self.group = group

    def exchange_counts(self, kept: Tensor) -> Tensor:
        return _even_exchange(kept, self.group)

    def exchange(self, t: Tensor) -> Tensor:
        return _even_exchange(t, self.group)


class ExpertParallelMoE(TopKMoE):
    def __init__(self, config: QuantaWeaveConfig, context: ExpertParallelContext) -> None:
        if config.num_experts % context.world_size:
            raise ValueError(f"num_experts {config.num_experts} must be divisible by the expert-parallel size "
                             f"{context.world_size}")
        # with sequence parallelism the tensor-parallel ranks are the expert ranks: experts stay whole
        super().__init__(config, num_local_experts=config.num_experts // context.world_size,
                         tensor_parallel=None if context.sequence_parallel else context)
        self.context = context
        self.measure_load = False
        self.load_rows = 0
        self.load_seconds = 0.0
        self._offsets_cache: dict = {}
        self._transport = None

    def transport(self):
        if self._transport is None:
            if self.context.transport == "p2p":
                from .p2p import P2PTransport

                self._transport = P2PTransport.for_group(self.context.group, self.context.device)
            elif self.context.transport == "fused":
                from .p2p import FusedTransport

                self._transport = FusedTransport.for_group(self.context.group, self.context.device)
            else:
                self._transport = NcclTransport(self.context.group)
        return self._transport

    def recv_offsets(self, slot: int, device) -> Tensor:
        key = (slot, str(device))
        if key not in self._offsets_cache:
            groups = self.context.world_size * self.num_local_experts
            self._offsets_cache[key] = torch.arange(groups, device=device, dtype=torch.int32) * slot
        return self._offsets_cache[key]

    def _native_ok(self) -> bool:
        # the single-GPU native MoE would run only this rank's experts with no exchange: the slot dispatch below is
        # the native path here, and every other case takes the reference exchange algorithm (``_execute``)
        return False

    def forward(self, hidden: Tensor, token_domains: Optional[Tensor] = None, num_domains: int = 0):
        if not (hidden.is_cuda and self.kernel != "loop" and not self.static_dispatch
                and not self.profile_experts and not self.simulated_cost_per_row and not self.measure_load):
            return super().forward(hidden, token_domains, num_domains)
        from ..ops import native_required

        native_required()
        batch, seq, width = hidden.shape
        flat = hidden.reshape(-1, width)
        cap = self.capacity(flat.size(0))
        out, probs, top_idx, counts, kept, meta, route_row = _SlotDispatch.apply(
            flat, self.router.weight, self.w_gate_up, self.w_down, self, cap)
        self.last_top_indices = top_idx.detach().long()
        if self.collect_stats:
            from ..ops.moe import _Dropped

            self._record_stats(probs, top_idx.long(), kept, _Dropped(route_row, top_idx, self.top_k))
        overflow = meta[1].long()
        zero = torch.zeros((), device=hidden.device, dtype=torch.long)
        dropped = overflow if self.overflow_policy == "drop" else zero
        balance = self.balance_loss(probs, top_idx, counts)
        domain = probs.new_zeros(())
        if token_domains is not None and num_domains > 1:
            domain = self._domain_loss(probs, token_domains, num_domains)
        return out.reshape(batch, seq, width).to(hidden.dtype), balance, dropped, overflow, domain

    # ---- reference algorithm (CPU / gloo, and the profiling/straggler paths) ----
    def _execute(self, flat_hidden: Tensor, tokens: Tensor, weights: Tensor, kept_counts: Tensor) -> Tensor:
        """Route the kept rows to the ranks that own their experts, run the local experts, route the results back.

        ``kept_counts`` is this rank's ``[world * local]`` per-expert row count in destination-major order, and
        ``tokens`` lists the source row of every kept slot in the same order. The exchanged counts tell every
        received row its local expert (the buffer arrives grouped by source rank, then by expert), so one stable
        sort by expert id gives each expert one contiguous slice.
        """
        ctx, group = self.context, self.context.group
        world, local = ctx.world_size, self.num_local_experts
        recv_counts = torch.empty_like(kept_counts)
        dist.all_to_all_single(recv_counts, kept_counts.contiguous(), group=group)
        send = kept_counts.view(world, local).sum(dim=1).tolist()
        recv = recv_counts.view(world, local).sum(dim=1).tolist()
        received = self._tp_in(_AllToAll.apply(flat_hidden[tokens], send, recv, group))
        expert_of_row = torch.arange(local, device=received.device).repeat(world).repeat_interleave(
            recv_counts.to(received.device))
        order = torch.argsort(expert_of_row, stable=True)
        bounds = [0] + torch.bincount(expert_of_row, minlength=local).cumsum(0).tolist()
        with _LoadClock(self, received):
            grouped = received[order]
            pieces = [self.expert_forward(e, grouped[bounds[e]:bounds[e + 1]]).to(received.dtype)
                      for e in range(local) if bounds[e + 1] > bounds[e]]
            processed = torch.empty_like(received)
            if pieces:
                processed = processed.index_copy(0, order, torch.cat(pieces))
        returned = _AllToAll.apply(self._tp_out(processed), recv, send, group)
        return torch.zeros_like(flat_hidden).index_add_(0, tokens, (returned * weights[:, None]).to(flat_hidden.dtype))

    def _run_expert(self, index: int, inputs: Tensor) -> Tensor:
        return self.expert_forward(index, inputs)



class _LoadClock:
    """Charges the expert work inside the ``with`` block to ``moe.load_seconds`` / ``moe.load_rows`` when the layer
    is measured. The device is synchronised on both sides so the wall clock covers the kernels, and the layer's
    ``simulated_cost_per_row`` (a test hook that makes a rank look slow) is added per row."""

    def __init__(self, moe, rows: Tensor) -> None:
        self.moe, self.rows, self.started = moe, rows, None

    def _sync(self) -> None:
        if self.rows.is_cuda:
            torch.cuda.synchronize(self.rows.device)

    def __enter__(self):
        if self.moe.measure_load:
            self._sync()
            self.started = time.perf_counter()
        return self

    def __exit__(self, *exc) -> None:
        if self.started is None or exc[0] is not None:
            return
        self._sync()
        n = self.rows.size(0)
        self.moe.load_rows += n
        self.moe.load_seconds += time.perf_counter() - self.started + n * self.moe.simulated_cost_per_row


def is_expert_parameter(name: str) -> bool:
    return name.endswith(("moe.w_gate_up", "moe.w_down")) or ".moe.experts." in name


def broadcast_shared_parameters(model, ctx: ExpertParallelContext) -> None:
    """Make replicated tensors identical: tensor-parallel slices across the expert group, everything else across
    the world. Experts stay rank-local."""
    from .tensor_parallel import is_tp_sharded_shared

    for name, param in model.named_parameters():
        if is_expert_parameter(name):
            continue
        if is_tp_sharded_shared(name) and ctx.tp_size > 1:
            if ctx.sequence_parallel:
                continue  # every rank holds a different slice
            if ctx.world_size > 1:
                dist.broadcast(param.data, src=ctx.group_root, group=ctx.group)
        else:
            dist.broadcast(param.data, src=0)
    for _, buf in model.named_buffers():
        dist.broadcast(buf.data, src=0)


def _shared_and_expert(model):
    shared, experts = [], []
    for name, p in model.named_parameters():
        (experts if is_expert_parameter(name) else shared).append(p)
    return shared, experts


def sync_gradients(model, ctx: ExpertParallelContext, sharded_optimizer=None, optimizer=None) -> None:
    """Average replicated gradients over the expert group (one flat all-reduce per dtype); scale expert gradients
    by ``1/ep`` (folded into the fused optimizer when it is given, else applied in place).

    With sequence parallelism every rank's loss covers its own token rows of one shared batch, so each rank's
    autograd already sums every rank's contribution into its attention slices (through the row gathers/scatters)
    and its experts (through the exchange): those are scaled by ``1/world`` like the experts, and only the
    replicated tensors are averaged."""
    from .tensor_parallel import is_tp_sharded_shared

    shared, experts = _shared_and_expert(model)
    if ctx.sequence_parallel:
        slices = [p for n, p in model.named_parameters() if is_tp_sharded_shared(n)]
        ids = {id(p) for p in slices}
        shared = [p for p in shared if id(p) not in ids]
        experts = experts + slices
    if ctx.world_size > 1:
        if sharded_optimizer is not None:
            sharded_optimizer.reduce_gradients()
        else:
            for p in shared:
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
            by_dtype: dict = {}
            for p in shared:
                by_dtype.setdefault(p.grad.dtype, []).append(p)
            for dtype, params in by_dtype.items():
                flat = torch.cat([p.grad.reshape(-1) for p in params])
                if flat.is_cuda:
                    dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=ctx.group)
                else:
                    dist.all_reduce(flat, group=ctx.group)
                    flat /= ctx.world_size
                offset = 0
                for p in params:
                    p.grad.copy_(flat[offset:offset + p.numel()].view_as(p))
                    offset += p.numel()
    scale = 1.0 / ctx.world_size
    fused = optimizer is not None and hasattr(optimizer, "grad_scale")
    for p in experts:
        if p.grad is None:
            continue
        if fused:
            optimizer.grad_scale[p] = scale
        elif ctx.world_size > 1:
            p.grad.mul_(scale)


def clip_grad_norm_parallel(model, ctx: ExpertParallelContext, max_norm: float, sharded: bool = False,
                            optimizer=None):
    """Clip by the true global norm, identically on every rank: replicated tensors once, tensor-parallel slices
    summed over the tensor group, experts summed over the world. With the fused optimizer the norm is computed by
    its kernels and the clip is folded into its step (no host synchronisation)."""
    from .tensor_parallel import is_tp_sharded_shared

    fused = optimizer is not None and hasattr(optimizer, "grad_sumsq")
    replicated, tp_slices, experts = [], [], []
    for name, p in model.named_parameters():
        if p.grad is None:
            continue
        if is_expert_parameter(name):
            experts.append(p)
        elif is_tp_sharded_shared(name) and ctx.tp_size > 1:
            tp_slices.append(p)
        else:
            replicated.append(p)
    device = ctx.device

    def sumsq(params):
        if not params:
            return torch.zeros((), dtype=torch.float64, device=device)
        if fused:
            return optimizer.grad_sumsq(params).to(device)
        return sum(p.grad.detach().double().pow(2).sum() for p in params)

    rep, tps, exp = sumsq(replicated), sumsq(tp_slices), sumsq(experts)
    zero = optimizer if (sharded and hasattr(optimizer, "shard_sumsq")) else None
    if zero is not None:  # replicated gradients now live as averaged shards inside the ZeRO optimizer
        rep = rep + zero.shard_sumsq().to(device)
    if sharded and ctx.world_size > 1:
        rep, tps = rep.clone(), tps.clone()
        dist.all_reduce(rep, group=ctx.group)
        dist.all_reduce(tps, group=ctx.group)
    if ctx.tp_size > 1:
        tps = tps.clone()
        dist.all_reduce(tps, group=ctx.tp_group)
    exp = exp.clone()
    if dist.is_initialized() and ctx.global_size > 1:
        dist.all_reduce(exp)
    total = (rep + tps + exp).sqrt()
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    if fused:
        optimizer.set_clip_coefficient(coef, total)
        return total
    if zero is not None:  # shards are scaled inside the ZeRO step; expert gradients here unless its local
        zero.set_clip_coefficient(coef, total)  # optimizer applies the coefficient itself
        if not hasattr(zero.local_opt, "set_clip_coefficient"):
            for p in experts:
                p.grad.mul_(coef.to(p.grad.dtype))
        return float(total)
    for p in model.parameters():
        if p.grad is not None:
            p.grad.mul_(coef.to(p.grad.dtype))
    return float(total)


def all_reduce_mean(values: list, ctx: ExpertParallelContext) -> list:
    t = torch.tensor(values, dtype=torch.float64, device=ctx.device)
    dist.all_reduce(t, group=ctx.group)
    return (t / ctx.world_size).tolist()


def barrier(ctx=None) -> None:
    from .groups import barrier as _barrier

    _barrier()


def finish(ctx) -> None:
    from .groups import finish as _finish

    _finish(ctx)


# ------------------------------------------------------------------------------------------ straggler control
class DeviceLoadTracker:
    """Per-rank expert time/rows controller (reference ``DeviceLoadTracker``, ``src/expert_parallel.py:280-384``).

    Every ``interval`` steps the per-layer expert seconds and rows each rank accumulated are collected into one
    ``[layers, ranks]`` table (one all-reduce of a rank-slotted slab, after a mean over the tensor-parallel group
    on the EP x TP grid; not under sequence parallelism, where every rank holds different experts).
    The routing bias is an integral controller ``bias_r -= rate * strength * log(t_r / mean)``, clamped to
    ``max_bias`` and re-centred, added to the router logits for selection only. ``adapt_capacity`` additionally sets
    each rank's ``capacity_scale`` to ``clamp(mean / t_r)``. Measuring per-expert time synchronises the device, so
    tracked layers take the reference (per-expert) path.
    """

    def __init__(self, model, ctx: ExpertParallelContext, strength: float = 0.5, max_bias: float = 2.0,
                 rate: float = 0.5, interval: int = 10, adapt_capacity: bool = False,
                 capacity_scale_min: float = 0.5, capacity_scale_max: float = 2.0) -> None:
        self.model, self.ctx, self.interval = model, ctx, interval
        self.strength, self.rate, self.max_bias = strength, rate, max_bias
        self.adapt_capacity = adapt_capacity
        self.capacity_scale_min, self.capacity_scale_max = capacity_scale_min, capacity_scale_max
        self.layers = len(model.moes())
        self.rank_bias = torch.zeros(self.layers, ctx.world_size, dtype=torch.float64)
        self.history: list = []
        for moe in model.moes():
            moe.measure_load = True

    # ---- collection ----
    def _table(self, local: Tensor) -> Tensor:
        """``local[layer, ...]`` of every rank as ``[layer, rank, ...]`` on the host: each rank writes its own slot
        of a zero slab and one sum-all-reduce over the expert-parallel group fills in the others."""
        local = local.to(self.ctx.device, torch.float64)
        # on the EP x TP grid the tensor-parallel ranks share one expert slice and measured the same work, so their
        # figures are averaged; with sequence parallelism the tensor-parallel ranks ARE the expert ranks, each with
        # its own experts, and averaging would erase exactly the differences the controller acts on
        if self.ctx.tp_size > 1 and not self.ctx.sequence_parallel:
            dist.all_reduce(local, group=self.ctx.tp_group)
            local = local / self.ctx.tp_size
        slab = local.new_zeros((self.ctx.world_size, *local.shape))
        slab[self.ctx.rank] = local
        dist.all_reduce(slab, group=self.ctx.group)
        return slab.transpose(0, 1).cpu()

    def _drain(self) -> Tensor:
        moes = self.model.moes()
        local = torch.tensor([[moe.load_seconds, moe.load_rows] for moe in moes], dtype=torch.float64)
        for moe in moes:
            moe.load_seconds, moe.load_rows = 0.0, 0
        return self._table(local)

    # ---- control ----
    @staticmethod
    def _imbalance(per_rank: Tensor) -> float:
        return float(per_rank.max() / per_rank.mean().clamp(min=1e-9))

    def _next_bias(self, seconds: Tensor) -> Tensor:
        """One integral step on the log of each rank's time relative to its layer's mean; only the differences
        between ranks matter, so the result is re-centred per layer."""
        log_ratio = (seconds / seconds.mean(dim=1, keepdim=True).clamp(min=1e-12)).clamp(min=0.05).log()
        bias = (self.rank_bias - self.rate * self.strength * log_ratio).clamp(-self.max_bias, self.max_bias)
        return bias - bias.mean(dim=1, keepdim=True)

    def _capacity_scale(self, seconds: Tensor) -> Tensor:
        mean = seconds.mean(dim=1, keepdim=True).clamp(min=1e-12)
        return (mean / seconds.clamp(min=1e-12)).clamp(self.capacity_scale_min, self.capacity_scale_max)

    def update(self, step: int) -> Optional[dict]:
        if step % self.interval:
            return None
        table = self._drain()
        seconds, rows = table[..., 0], table[..., 1]
        metrics = {"step": step, "device_rows": rows.sum(dim=0).tolist(),
                   "device_seconds": seconds.sum(dim=0).tolist(),
                   "rows_imbalance": self._imbalance(rows.sum(dim=0)),
                   "time_imbalance": self._imbalance(seconds.sum(dim=0))}
        measured = float(seconds.sum()) > 0
        if measured and self.strength > 0:
            self.rank_bias = self._next_bias(seconds)
            self._apply()
        metrics["rank_bias"] = self.rank_bias.mean(dim=0).tolist()
        if measured and self.adapt_capacity:
            scale = self._capacity_scale(seconds)
            for moe, value in zip(self.model.moes(), scale[:, self.ctx.rank].tolist()):
                moe.capacity_scale = value
            metrics["capacity_scale"] = scale.mean(dim=0).tolist()
        self.history.append(metrics)
        return metrics

    def _apply(self) -> None:
        """Expand the per-rank bias to every expert a rank holds (experts are laid out rank-major)."""
        moes = self.model.moes()
        per_expert = self.rank_bias.repeat_interleave(moes[0].num_local_experts, dim=1)
        per_expert = per_expert.to(device=self.ctx.device, dtype=torch.float32)
        for moe, row in zip(moes, per_expert):
            moe.expert_bias = row

    def gather_expert_utilization(self) -> Tensor:
        """``[rank, layer, expert]`` routed-row shares of the last step, as each rank saw them."""
        local = torch.stack([moe.last_stats["expert_load"].double().cpu() for moe in self.model.moes()])
        return self._table(local).transpose(0, 1).contiguous()

    # ---- checkpoint ----
    def state_dict(self) -> dict:
        return {"rank_bias": self.rank_bias.tolist()}

    def load_state_dict(self, state: dict) -> None:
        self.rank_bias = torch.tensor(state["rank_bias"], dtype=torch.float64)
        if bool(self.rank_bias.ne(0).any()):
            self._apply()


def simulated_slow_rank(spec: str) -> tuple[int, float]:
    rank, cost = spec.split(":")
    return int(rank), float(cost)


del math
