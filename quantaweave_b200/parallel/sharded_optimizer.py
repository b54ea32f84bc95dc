"""ZeRO-style sharded AdamW over a data-parallel group (reference ``src/sharded_optimizer.py``).

The reference assigns whole replicated parameters to owner ranks (reduce to owner, owner steps, broadcast). This
implementation shards *flat*: every replicated gradient is packed into one buffer per dtype, padded to a multiple
of the group size, and

1. ``reduce_gradients``: ``reduce_scatter`` (average) -> each rank holds its contiguous gradient shard only;
2. ``step``: AdamW on the shard against an fp32 master shard (moments exist only for the shard: ZeRO-1/2 memory);
3. the updated shard is ``all_gather``-ed back into the replicated parameters.

Expert (rank-local) parameters use a local AdamW (the fused kernel on CUDA). ``state_dict`` records the shard
layout and refuses to load into a different world size or parameter set, like the reference.

On CUDA with more than one rank the collectives are fused into the optimizer kernels (``csrc/zero_fused.cu``;
``QW_ZERO_FUSED=0`` selects the NCCL path): the replicated parameters are re-homed into symmetric memory, each rank
packs its gradients into a symmetric staging buffer, the reduce-scatter kernel sums its shard straight from the
peers' buffers (fixed rank order, cast and 1/world scale fused, sums of squares for the clip norm), and the AdamW
kernel stores each updated value into every rank's parameter buffer, which is the all-gather.

Overlap with backward (fused path, ``QW_ZERO_OVERLAP=1`` by default): the staging buffer is cut into buckets of
about ``bucket_elems`` elements in reverse parameter order (the order backward produces gradients). Calling
:meth:`arm_overlap` before the step's last backward makes each parameter's post-accumulate hook copy its finished
gradient into the staging buffer and free it; when every parameter touching a bucket is staged, a side stream runs
that bucket's barrier and the reduce-scatter of this rank's part of it while backward continues on the main stream.
:meth:`reduce_gradients` then only flushes the buckets whose gradients never arrived (unused parameters) and joins
the side stream.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor

from .expert_parallel import is_expert_parameter


class ShardedAdamW:
    def __init__(self, model, ctx, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, group=None, bucket_elems: int = 1 << 24) -> None:
        self.bucket_elems = bucket_elems
        self.model, self.ctx = model, ctx
        self.group = group if group is not None else getattr(ctx, "group", None) or getattr(ctx, "dp_group", None)
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        named = list(model.named_parameters())
        # expert weights are rank-local only in an expert-parallel model (each rank holds different experts); in a
        # pipeline or plain data-parallel model every replica holds the same experts and they are sharded like the
        # rest, so their gradients are averaged over the group and counted in the clip norm
        ep = getattr(model, "expert_parallel", None)
        experts_local = ep is not None and getattr(ep, "world_size", 1) > 1
        self.shared = [p for n, p in named if not (experts_local and is_expert_parameter(n))]
        self.local = [p for n, p in named if experts_local and is_expert_parameter(n)]
        self.defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        self._groups: dict = {}
        for p in self.shared:
            self._groups.setdefault(p.dtype, []).append(p)
        self.shards: dict = {}
        for dtype, params in self._groups.items():
            total = sum(p.numel() for p in params)
            # shards are padded to a multiple of 8 elements, so the fused kernels move 16-byte vectors
            per = ((total + self.world - 1) // self.world + 7) // 8 * 8
            start = self.rank * per
            flat = torch.cat([p.detach().reshape(-1).float() for p in params])
            flat = torch.nn.functional.pad(flat, (0, per * self.world - total))
            self.shards[dtype] = {"numel": total, "per": per, "master": flat[start:start + per].clone(),
                                  "exp_avg": torch.zeros(per, device=flat.device),
                                  "exp_avg_sq": torch.zeros(per, device=flat.device), "grad": None}
        self.step_count = 0
        self.local_opt = None
        if self.local:
            if any(p.is_cuda for p in self.local):
                from ..optim.adamw import FusedAdamW

                self.local_opt = FusedAdamW(self.local, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
            else:
                self.local_opt = torch.optim.AdamW(self.local, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        self.param_groups = [dict(self.defaults, params=self.shared)] + (self.local_opt.param_groups if self.local_opt else [])
        self._clip = None
        self.fused = (self.world > 1 and bool(self.shared) and all(p.is_cuda for p in self.shared)
                      and os.environ.get("QW_ZERO_FUSED", "1") != "0")
        if self.fused:
            self._setup_fused()

    # ---- fused path (CUDA) --------------------------------------------------------------------------
    def _setup_fused(self) -> None:
        """Re-home the replicated parameters into symmetric memory and create the gradient staging buffers."""
        from .p2p import P2PTransport, _Channel

        device = self.shared[0].device
        transport = P2PTransport.for_group(self.group, device)
        symm = transport.symm
        name = transport._group_name()
        self._ready, self._done = _Channel(transport), _Channel(transport)
        self._transport = transport
        for dtype, params in self._groups.items():
            sh = self.shards[dtype]
            n = sh["per"] * self.world
            pbuf = symm.empty(n, dtype=dtype, device=device)
            gbuf = symm.empty(n, dtype=dtype, device=device)
            hp, hg = symm.rendezvous(pbuf, name), symm.rendezvous(gbuf, name)
            pbuf.zero_()
            gbuf.zero_()
            offset = 0
            with torch.no_grad():
                for p in params:
                    view = pbuf[offset:offset + p.numel()].view_as(p)
                    view.copy_(p.detach())
                    p.data = view
                    offset += p.numel()
            sh.update(pbuf=pbuf, gbuf=gbuf, handles=(hp, hg),
                      ppeers=torch.tensor([int(x) for x in hp.buffer_ptrs], dtype=torch.int64, device=device),
                      gpeers=torch.tensor([int(x) for x in hg.buffer_ptrs], dtype=torch.int64, device=device),
                      code=0 if dtype == torch.float32 else 1)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group, device_ids=[device.index if device.index is not None else torch.cuda.current_device()])
        self._armed = False
        self._overlap = os.environ.get("QW_ZERO_OVERLAP", "1") != "0"
        if self._overlap:
            self._setup_buckets(device)

    # ---- overlap of the reduce-scatter with backward ------------------------------------------------
    def _setup_buckets(self, device) -> None:
        """Cut every dtype's staging buffer into 8-aligned buckets, from the end (backward's order), and hook the
        parameters. ``self._buckets``: (dtype, lo, hi, number of parameters touching it), in launch order."""
        self._comm = torch.cuda.Stream(device)
        self._buckets: list = []
        self._param_buckets: dict = {}  # id(param) -> (dtype, offset, bucket indices)
        for dtype, params in self._groups.items():
            sh = self.shards[dtype]
            end = sh["per"] * self.world
            offsets, offset = [], 0
            for p in params:
                offsets.append(offset)
                offset += p.numel()
            cuts = [end]
            for off in reversed(offsets):
                if cuts[-1] - off >= self.bucket_elems:
                    cut = off // 8 * 8
                    if 0 < cut < cuts[-1]:
                        cuts.append(cut)
            cuts.append(0)
            cuts = sorted(set(cuts), reverse=True)  # descending: the first bucket covers the buffer's end
            first = len(self._buckets)
            for hi, lo in zip(cuts, cuts[1:]):
                self._buckets.append([dtype, lo, hi, 0])
            for p, off in zip(params, offsets):
                touched = [first + b for b, (hi, lo) in enumerate(zip(cuts, cuts[1:])) if off < hi and off + p.numel() > lo]
                for b in touched:
                    self._buckets[b][3] += 1
                self._param_buckets[id(p)] = (dtype, off, touched)
                p.register_post_accumulate_grad_hook(self._on_grad)

    def arm_overlap(self) -> None:
        """Stage gradients and reduce-scatter them bucket by bucket during the next backward (the step's last)."""
        if not (self.fused and self._overlap):
            return
        device = self.shared[0].device
        self._armed = True
        self._pending = [b[3] for b in self._buckets]
        self._staged: set = set()
        self._launched = [False] * len(self._buckets)
        self._next_launch = 0
        for dtype in self._groups:
            sh = self.shards[dtype]
            sh["grad"] = torch.empty(sh["per"], device=device, dtype=torch.float32)
        from ..ops import ext

        C = ext()
        self._bucket_span = []
        total = 0
        for dtype, lo, hi, _ in self._buckets:
            per = self.shards[dtype]["per"]
            a, e = max(lo, self.rank * per), min(hi, (self.rank + 1) * per)
            blocks = C.zero_rs_blocks(e - a) if e > a else 0
            self._bucket_span.append((a, e, total, blocks))
            total += blocks
        self._partial = torch.zeros(max(total, 1), device=device, dtype=torch.float64)
        self._launch_ready()

    def _on_grad(self, p) -> None:
        if not self._armed or id(p) in self._staged:
            return
        dtype, off, touched = self._param_buckets[id(p)]
        self.shards[dtype]["gbuf"][off:off + p.numel()].copy_(p.grad.reshape(-1))
        p.grad = None
        self._staged.add(id(p))
        for b in touched:
            self._pending[b] -= 1
        self._launch_ready()

    def _launch_ready(self) -> None:
        """Launch, in bucket order, every bucket whose parameters are all staged (same order on every rank)."""
        while self._next_launch < len(self._buckets) and self._pending[self._next_launch] == 0:
            self._launch(self._next_launch)
            self._next_launch += 1

    def _launch(self, b: int) -> None:
        from ..ops import ext

        dtype = self._buckets[b][0]
        sh = self.shards[dtype]
        a, e, first_block, blocks = self._bucket_span[b]
        staged = torch.cuda.Event()
        staged.record()
        with torch.cuda.stream(self._comm):
            self._comm.wait_event(staged)
            self._barrier(self._ready)  # every rank has staged this bucket
            if e > a:
                base = self.rank * sh["per"]
                ext().zero_reduce_scatter(sh["gpeers"], sh["code"], a, sh["grad"][a - base:e - base],
                                          self._partial[first_block:first_block + blocks])
        self._launched[b] = True

    def _finish_overlap(self) -> None:
        """Stage the gradients that never arrived (unused parameters: zeros), launch what is left, join."""
        for dtype, params in self._groups.items():
            gbuf = self.shards[dtype]["gbuf"]
            for p in params:
                if id(p) in self._staged:
                    continue
                _, off, touched = self._param_buckets[id(p)]
                if p.grad is None:
                    gbuf[off:off + p.numel()].zero_()
                else:
                    gbuf[off:off + p.numel()].copy_(p.grad.reshape(-1))
                    p.grad = None
                self._staged.add(id(p))
                for b in touched:
                    self._pending[b] -= 1
        self._launch_ready()
        torch.cuda.current_stream().wait_stream(self._comm)
        total = self._partial.sum()
        for i, dtype in enumerate(self._groups):
            self.shards[dtype]["sumsq"] = total if i == 0 else torch.zeros_like(total)
        self._armed = False

    def _barrier(self, channel) -> None:
        from ..ops import ext

        parity = channel.next()
        ext().ep_signal(channel.peer_flags[parity], self.rank, channel.epoch)
        channel.wait(parity)

    def _reduce_fused(self) -> None:
        from ..ops import ext

        C = ext()
        for dtype, params in self._groups.items():
            gbuf = self.shards[dtype]["gbuf"]
            offset = 0
            for p in params:
                n = p.numel()
                if p.grad is None:
                    gbuf[offset:offset + n].zero_()
                else:
                    gbuf[offset:offset + n].copy_(p.grad.reshape(-1))
                    p.grad = None
                offset += n
        self._barrier(self._ready)  # every rank's gradients are staged
        for dtype in self._groups:
            sh = self.shards[dtype]
            grad = torch.empty(sh["per"], device=sh["gbuf"].device, dtype=torch.float32)
            partial = torch.empty(C.zero_rs_blocks(sh["per"]), device=grad.device, dtype=torch.float64)
            C.zero_reduce_scatter(sh["gpeers"], sh["code"], self.rank * sh["per"], grad, partial)
            sh["grad"], sh["sumsq"] = grad, partial.sum()

    # ---- gradients ------------------------------------------------------------------------------
    def reduce_gradients(self) -> None:
        if self.fused and self._armed:
            self._finish_overlap()
            return
        if self.fused:
            self._reduce_fused()
            return
        for dtype, params in self._groups.items():
            for p in params:
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
            sh = self.shards[dtype]
            flat = torch.cat([p.grad.reshape(-1).float() for p in params])
            flat = torch.nn.functional.pad(flat, (0, sh["per"] * self.world - sh["numel"]))
            out = torch.empty(sh["per"], device=flat.device, dtype=flat.dtype)
            if self.world > 1:
                dist.reduce_scatter_tensor(out, flat, group=self.group)
                out /= self.world
            else:
                out.copy_(flat)
            sh["grad"] = out
            for p in params:
                p.grad = None

    def shard_sumsq(self) -> Tensor:
        total = None
        for sh in self.shards.values():
            if sh["grad"] is not None:
                s = sh["sumsq"] if (self.fused and "sumsq" in sh) else sh["grad"].double().pow(2).sum()
                total = s if total is None else total + s
        if total is None:
            device = next(iter(self.shards.values()))["master"].device if self.shards else "cpu"
            total = torch.zeros((), dtype=torch.float64, device=device)
        return total

    def set_clip_coefficient(self, coef: Tensor, norm=None) -> None:
        self._clip = coef
        if self.local_opt is not None and hasattr(self.local_opt, "set_clip_coefficient"):
            self.local_opt.set_clip_coefficient(coef, norm)

    # ---- update ---------------------------------------------------------------------------------
    @torch.no_grad()
    def step(self) -> None:
        group = self.param_groups[0]
        lr = group["lr"]
        beta1, beta2 = group["betas"]
        eps, wd = group["eps"], group["weight_decay"]
        self.step_count += 1
        t = self.step_count
        if self.fused:
            self._step_fused(lr, beta1, beta2, eps, wd, t)
            return
        for dtype, params in self._groups.items():
            sh = self.shards[dtype]
            g = sh["grad"]
            if g is None:
                continue
            if self._clip is not None:
                g = g * self._clip.to(g.device, g.dtype)
            p = sh["master"]
            p.mul_(1 - lr * wd)
            sh["exp_avg"].lerp_(g, 1 - beta1)
            sh["exp_avg_sq"].mul_(beta2).addcmul_(g, g, value=1 - beta2)
            denom = (sh["exp_avg_sq"].sqrt() / (1 - beta2 ** t) ** 0.5).add_(eps)
            p.addcdiv_(sh["exp_avg"], denom, value=-lr / (1 - beta1 ** t))
            full = torch.empty(sh["per"] * self.world, device=p.device, dtype=p.dtype)
            if self.world > 1:
                dist.all_gather_into_tensor(full, p, group=self.group)
            else:
                full.copy_(p)
            offset = 0
            for q in params:
                q.data.copy_(full[offset:offset + q.numel()].view_as(q).to(q.dtype))
                offset += q.numel()
            sh["grad"] = None
        if self.local_opt is not None:
            if len(self.param_groups) > 1:
                for g_ in self.local_opt.param_groups:
                    g_["lr"] = lr
            self.local_opt.step()
        self._clip = None

    def _step_fused(self, lr, beta1, beta2, eps, wd, t) -> None:
        from ..ops import ext

        C = ext()
        clip = None if self._clip is None else self._clip.reshape(-1)[:1].float().contiguous()
        for dtype in self._groups:
            sh = self.shards[dtype]
            if sh["grad"] is None:
                continue
            C.zero_adamw_gather(sh["master"], sh["exp_avg"], sh["exp_avg_sq"], sh["grad"], clip, lr, beta1, beta2,
                                eps, wd, t, sh["ppeers"], sh["code"], self.rank * sh["per"], sh["numel"])
            sh["grad"] = None
            sh.pop("sumsq", None)
        self._barrier(self._done)  # every shard's update has landed in every rank's parameters
        if self.local_opt is not None:
            if len(self.param_groups) > 1:
                for g_ in self.local_opt.param_groups:
                    g_["lr"] = lr
            self.local_opt.step()
        self._clip = None

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.model.parameters():
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def state_numel(self) -> int:
        return sum(2 * sh["per"] for sh in self.shards.values())

    def state_dict(self) -> dict:
        keep = ("numel", "per", "master", "exp_avg", "exp_avg_sq")
        return {"shards": {str(k): {n: v for n, v in sh.items() if n in keep} for k, sh in self.shards.items()},
                "step": self.step_count, "world": self.world, "rank": self.rank,
                "local": self.local_opt.state_dict() if self.local_opt is not None else None}

    def load_state_dict(self, state: dict) -> None:
        if state["world"] != self.world or state["rank"] != self.rank:
            raise ValueError("sharded optimizer state was saved with a different world size or rank")
        for key, saved in state["shards"].items():
            match = [d for d in self.shards if str(d) == key]
            if not match or saved["numel"] != self.shards[match[0]]["numel"]:
                raise ValueError("sharded optimizer state was saved for a different parameter set")
            sh = self.shards[match[0]]
            for name in ("master", "exp_avg", "exp_avg_sq"):
                sh[name].copy_(saved[name])
        self.step_count = int(state["step"])
        if self.local_opt is not None and state.get("local") is not None:
            self.local_opt.load_state_dict(state["local"])
