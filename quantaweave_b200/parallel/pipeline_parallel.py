"""Pipeline parallelism: GPipe and 1F1B over NCCL point-to-point, with data-parallel replicas (PP x DP).

Behaviour follows the reference ``src/pipeline_parallel.py``: contiguous layer partition with the remainder on the
first stages (:72-82); the first stage owns the embeddings, the last the head; GPipe runs all forwards then the
backwards in reverse, 1F1B warms up ``min(M, S - stage - 1)`` forwards (:213-229); sends are ``isend``s drained at the
end of the step, which avoids the 1F1B send/send deadlock (:123-140); the aux loss is split per stage and
micro-batch (:160-161); loss totals are all-reduced (:202-211).

Differences: activations travel in the compute dtype (bf16 on CUDA) instead of fp32; receives are posted as
``irecv`` before the local work that precedes their use; ranks are laid out ``global = dp_rank * S + stage`` so each
data-parallel replica is a full pipeline, and the replicas average gradients (or reduce-scatter them for the
sharded optimizer) after the pipeline step.
"""

from __future__ import annotations

import contextlib
from collections import deque
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor


@dataclass
class PipelineContext:
    stage: int
    num_stages: int
    device: torch.device
    layer_start: int
    layer_end: int
    owns_process_group: bool = False
    dp_rank: int = 0
    dp_size: int = 1
    dp_group: Optional[object] = None
    pp_group: Optional[object] = None

    @property
    def global_rank(self) -> int:
        return self.dp_rank * self.num_stages + self.stage

    @property
    def global_size(self) -> int:
        return self.num_stages * self.dp_size

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.num_stages - 1

    def peer(self, stage: int) -> int:
        return self.dp_rank * self.num_stages + stage

    def layout(self) -> dict:
        out = {"kind": "pp", "stage": self.stage, "stages": self.num_stages, "layer_start": self.layer_start,
               "layer_end": self.layer_end}
        if self.dp_size > 1:
            out.update(dp_rank=self.dp_rank, dp_size=self.dp_size)
        return out

    def broadcast_parameters(self, model) -> None:
        if self.dp_size > 1:
            root = self.stage  # dp_rank 0 of this stage column
            for p in model.parameters():
                dist.broadcast(p.data, src=root, group=self.dp_group)


def partition_layers(total_layers: int, stages: int) -> list:
    if stages < 1 or total_layers < stages:
        raise ValueError(f"cannot split {total_layers} layers over {stages} pipeline stages")
    base, extra = divmod(total_layers, stages)
    ranges, start = [], 0
    for stage in range(stages):
        size = base + (1 if stage < extra else 0)
        ranges.append((start, start + size))
        start += size
    return ranges


def init_pipeline_parallel(device_arg: str, total_layers: int, data_parallel: int = 1) -> PipelineContext:
    from .groups import ensure_process_group

    owns, device = ensure_process_group(device_arg)
    world, rank = dist.get_world_size(), dist.get_rank()
    if data_parallel < 1 or world % data_parallel:
        raise ValueError(f"world size {world} is not divisible by the pipeline data-parallel size {data_parallel}")
    stages = world // data_parallel
    dp_rank, stage = divmod(rank, stages)
    dp_group = pp_group = None
    if data_parallel > 1:
        for s in range(stages):
            g = dist.new_group([d * stages + s for d in range(data_parallel)])
            dp_group = g if s == stage else dp_group
        for d in range(data_parallel):
            g = dist.new_group([d * stages + s for s in range(stages)])
            pp_group = g if d == dp_rank else pp_group
    start, end = partition_layers(total_layers, stages)[stage]
    return PipelineContext(stage, stages, device, start, end, owns, dp_rank, data_parallel, dp_group, pp_group)


class PipelineEngine:
    def __init__(self, model, ctx: PipelineContext, microbatches: int, autocast: Callable = contextlib.nullcontext,
                 schedule: str = "gpipe") -> None:
        if microbatches < 1:
            raise ValueError("microbatches must be positive")
        if schedule not in ("gpipe", "1f1b"):
            raise ValueError("schedule must be gpipe or 1f1b")
        self.model, self.ctx, self.microbatches, self.autocast, self.schedule = model, ctx, microbatches, autocast, schedule
        self._totals = {"ce": 0.0, "aux": 0.0, "dropped": 0, "overflow": 0}
        self._pending: list = []
        # called right before the step's last micro-batch backward (a sharded optimizer's ``arm_overlap``, so its
        # gradient reduce-scatter runs bucket by bucket during that backward)
        self.before_last_backward: Optional[Callable] = None
        self._backwards = 0

    def _isend(self, tensor: Tensor, stage: int) -> None:
        self._pending.append((dist.isend(tensor, dst=self.ctx.peer(stage)), tensor))

    def _drain(self) -> None:
        for req, _ in self._pending:
            req.wait()
        self._pending = []

    def _act_dtype(self):
        return torch.bfloat16 if self.ctx.device.type == "cuda" else torch.float32

    def _forward_step(self, batch: Tensor, index: int, size: int):
        model, ctx, M = self.model, self.ctx, self.microbatches
        width = model.config.hidden_size
        tokens = batch[index * size:(index + 1) * size].to(ctx.device)
        hidden_in = None
        if ctx.is_first:
            with self.autocast():
                hidden = model.embed(tokens)
        else:
            hidden_in = torch.empty(size, tokens.size(1), width, dtype=self._act_dtype(), device=ctx.device)
            dist.recv(hidden_in, src=ctx.peer(ctx.stage - 1))
            hidden_in.requires_grad_(True)
            hidden = hidden_in
        with self.autocast():
            hidden, balance, dropped, overflow, _ = model.run_blocks(hidden)
        aux = torch.stack(balance).sum()
        aux_term = model.router_aux_loss_coef * aux / model.config.layers / M
        self._totals["aux"] += aux.detach() / M
        self._totals["dropped"] += torch.stack(dropped).sum()
        self._totals["overflow"] += torch.stack(overflow).sum()
        if ctx.is_last:
            with self.autocast():
                if hidden.is_cuda:
                    ce = model.lm_loss(hidden, tokens)
                else:
                    logits = model.head(hidden)
                    ce = F.cross_entropy(logits[:, :-1].reshape(-1, logits.size(-1)).float(), tokens[:, 1:].reshape(-1))
            self._totals["ce"] += ce.detach() / M
            return (hidden_in, ce / M + aux_term, None)
        self._isend(hidden.detach().to(self._act_dtype()).contiguous(), ctx.stage + 1)
        return (hidden_in, hidden, aux_term)

    def _backward_step(self, saved) -> None:
        ctx = self.ctx
        self._backwards += 1
        if self._backwards == self.microbatches and self.before_last_backward is not None:
            self.before_last_backward()
        hidden_in, output, aux_term = saved
        if ctx.is_last:
            output.backward()
        else:
            grad = torch.empty(output.shape, dtype=self._act_dtype(), device=ctx.device)
            dist.recv(grad, src=ctx.peer(ctx.stage + 1))
            torch.autograd.backward([output, aux_term], [grad.to(output.dtype), None])
        if not ctx.is_first:
            self._isend(hidden_in.grad.to(self._act_dtype()).contiguous(), ctx.stage - 1)

    def train_step(self, batch: Tensor) -> dict:
        ctx, M = self.ctx, self.microbatches
        if batch.size(0) % M:
            raise ValueError(f"batch size {batch.size(0)} must be divisible by --microbatches {M}")
        size = batch.size(0) // M
        zero = torch.zeros((), dtype=torch.float64, device=ctx.device)
        self._totals = {"ce": zero.clone(), "aux": zero.clone(), "dropped": zero.clone(), "overflow": zero.clone()}
        self._backwards = 0
        if self.schedule == "1f1b":
            self._run_1f1b(batch, size)
        else:
            self._run_gpipe(batch, size)
        self._drain()
        totals = torch.stack([self._totals["ce"].double(), self._totals["aux"].double(),
                              self._totals["dropped"].double(), self._totals["overflow"].double()])
        dist.all_reduce(totals, group=ctx.pp_group)
        if ctx.dp_size > 1:
            dist.all_reduce(totals, group=ctx.dp_group)
            totals[:2] /= ctx.dp_size
        ce, aux_sum, dropped, overflow = totals.tolist()
        router_aux = aux_sum / self.model.config.layers
        return {"loss": ce + self.model.router_aux_loss_coef * router_aux, "ce_loss": ce, "router_aux_loss": router_aux,
                "dropped_routes": int(dropped), "overflow_routes": int(overflow)}

    def _run_gpipe(self, batch: Tensor, size: int) -> None:
        saved = [self._forward_step(batch, i, size) for i in range(self.microbatches)]
        for i in reversed(range(self.microbatches)):
            self._backward_step(saved[i])

    def _run_1f1b(self, batch: Tensor, size: int) -> None:
        stage, stages, M = self.ctx.stage, self.ctx.num_stages, self.microbatches
        warmup = min(M, stages - stage - 1)
        queue: deque = deque()
        for i in range(warmup):
            queue.append(self._forward_step(batch, i, size))
        for i in range(warmup, M):
            queue.append(self._forward_step(batch, i, size))
            self._backward_step(queue.popleft())
        while queue:
            self._backward_step(queue.popleft())

    def clip_and_sync(self, optimizer, max_norm: float):
        """Average gradients over the data-parallel replicas, then clip by the global norm over all stages."""
        ctx = self.ctx
        if ctx.dp_size > 1:
            if hasattr(optimizer, "reduce_gradients"):
                optimizer.reduce_gradients()
            else:
                from .data_parallel import DataParallelContext

                DataParallelContext(ctx.dp_rank, ctx.dp_size, ctx.device, ctx.dp_group).sync_gradients(self.model)
        return clip_grad_norm_pipeline(self.model, ctx, max_norm, optimizer)


def clip_grad_norm_pipeline(model, ctx: PipelineContext, max_norm: float, optimizer=None):
    """Clip by the norm of the whole model's gradient and return that norm (before clipping).

    Each parameter lives on exactly one stage, so the squared norm of the full gradient is the sum of the stages'
    squared norms: one all-reduce over the pipeline group. With a sharded optimizer the replicas of a stage hold
    disjoint gradient shards; their squared norms are summed over the data-parallel group first, and the clip factor
    is handed to the optimizer, which applies it inside its update."""
    if optimizer is not None and hasattr(optimizer, "shard_sumsq"):
        squared = optimizer.shard_sumsq()
        if ctx.dp_size > 1:
            dist.all_reduce(squared, group=ctx.dp_group)
        grads = []
    else:
        grads = [p.grad for p in model.parameters() if p.grad is not None]
        per_tensor = [torch.linalg.vector_norm(g, dtype=torch.float64) for g in grads]
        squared = (torch.stack(per_tensor).square().sum() if per_tensor
                   else torch.zeros((), dtype=torch.float64, device=ctx.device))
    dist.all_reduce(squared, group=ctx.pp_group)
    norm = squared.sqrt()
    factor = (max_norm / (norm + 1e-6)).clamp(max=1.0)
    if optimizer is not None and hasattr(optimizer, "set_clip_coefficient"):
        optimizer.set_clip_coefficient(factor, norm)
        return float(norm)
    by_dtype: dict = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    for dtype, group in by_dtype.items():
        torch._foreach_mul_(group, factor.to(dtype))
    return float(norm)
