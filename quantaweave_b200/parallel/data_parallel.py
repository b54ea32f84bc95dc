"""Plain data parallelism: every rank holds the whole model (experts included) and a disjoint slice of each
global batch; gradients are averaged with one flat all-reduce per dtype (or reduce-scattered by ``ShardedAdamW``).
Not present in the reference (its DP exists only inside the expert-parallel group); added for dense scaling and for
the pipeline's data-parallel replicas.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DataParallelContext:
    rank: int
    world_size: int
    device: torch.device
    group: Optional[object] = None
    owns_process_group: bool = False

    @property
    def global_rank(self) -> int:
        return self.rank

    @property
    def global_size(self) -> int:
        return self.world_size

    def layout(self) -> dict:
        return {"kind": "dp", "dp_rank": self.rank, "dp_size": self.world_size}

    def broadcast_parameters(self, model) -> None:
        for p in model.parameters():
            dist.broadcast(p.data, src=0, group=self.group)

    def sync_gradients(self, model, sharded_optimizer=None) -> None:
        if sharded_optimizer is not None:
            sharded_optimizer.reduce_gradients()
            return
        params = [p for p in model.parameters()]
        for p in params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        by_dtype: dict = {}
        for p in params:
            by_dtype.setdefault(p.grad.dtype, []).append(p)
        for dtype, group in by_dtype.items():
            flat = torch.cat([p.grad.reshape(-1) for p in group])
            dist.all_reduce(flat, group=self.group)
            flat /= self.world_size
            offset = 0
            for p in group:
                p.grad.copy_(flat[offset:offset + p.numel()].view_as(p))
                offset += p.numel()

    def clip_grad_norm(self, model, optimizer, max_norm: float):
        if hasattr(optimizer, "shard_sumsq"):
            sq = optimizer.shard_sumsq()
            dist.all_reduce(sq, group=self.group)
            if optimizer.local_opt is not None:
                sq = sq + optimizer.local_opt.grad_sumsq().to(sq.device) if hasattr(optimizer.local_opt, "grad_sumsq") \
                    else sq + sum(p.grad.double().pow(2).sum() for p in optimizer.local if p.grad is not None)
            total = sq.sqrt()
            optimizer.set_clip_coefficient(torch.clamp(max_norm / (total + 1e-6), max=1.0), total)
            return total
        if hasattr(optimizer, "clip_grad_norm_"):
            return optimizer.clip_grad_norm_(max_norm)
        return torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm)

    def all_reduce_mean(self, values: list) -> list:
        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        dist.all_reduce(t, group=self.group)
        return (t / self.world_size).tolist()


def init_data_parallel(device_arg: str = "auto") -> DataParallelContext:
    from .groups import ensure_process_group

    owns, device = ensure_process_group(device_arg)
    return DataParallelContext(dist.get_rank(), dist.get_world_size(), device, None, owns)
