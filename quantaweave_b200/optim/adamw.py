"""Fused multi-tensor AdamW for CUDA parameters.

* bf16 parameters get an fp32 master copy; fp32 parameters are updated in place.
* One kernel computes the global gradient norm (fixed-order fp64 reduction, deterministic); the clip coefficient
  stays on the device and is folded into the single fused update kernel that walks every parameter.
* The update matches ``torch.optim.AdamW`` (decoupled weight decay, bias-corrected moments).
* ``overlap_with_forward(model)``: later ``step()`` calls run the update on a side stream, part by part in the order
  the forward uses the parameters (``model.parameter_parts()``), and a forward pre-hook makes the compute stream
  wait for a part just before its first use. The update is bound by HBM bandwidth and the next forward mostly by
  the tensor cores, so most of it hides. The gradients and clip coefficient of an in-flight update stay referenced
  until the next ``step()``; ``finish()`` joins the side stream (timers, checkpoints and ``state_dict`` need it).
  Measured on one B200 with benchmark configuration 2 it is neutral (the persistent GEMM and attention kernels of
  the forward leave the update few SM resources), so it is opt-in.

State is kept as the usual ``self.state[p]`` dict (``step``, ``exp_avg``, ``exp_avg_sq`` and ``master`` for bf16
parameters), always in fp32; ``state_dict``/``load_state_dict`` preserve those dtypes.
"""

from __future__ import annotations

from typing import Iterable, Optional

import torch
from torch import Tensor

from ..ops import ext


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params: Iterable, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, moment_bits: int = 32) -> None:
        if moment_bits not in (8, 32):
            raise ValueError("moment_bits must be 8 or 32")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.moment_bits = moment_bits
        self._chunk = None
        self._clip: Optional[Tensor] = None
        # per-parameter factor applied to the stored gradient inside the fused kernels (norm and update), e.g.
        # 1/ep for expert gradients that the expert-parallel backward sums over every rank's tokens
        self.grad_scale: dict = {}
        self._norm_buf: Optional[Tensor] = None
        self._side = None          # overlap: side stream, part of each parameter, pending per-part events
        self._part_of: dict = {}
        self._part_events: list = []
        self._inflight = None

    # ---- state -----------------------------------------------------------------------------------
    def _init_state(self, p: Tensor) -> dict:
        state = self.state[p]
        if "exp_avg" not in state:
            state["step"] = 0
            if self.moment_bits == 8:
                self._alloc8(p, state, None)
            else:
                state["exp_avg"] = torch.zeros(p.shape, device=p.device, dtype=torch.float32)
                state["exp_avg_sq"] = torch.zeros(p.shape, device=p.device, dtype=torch.float32)
            if p.dtype != torch.float32:
                state["master"] = p.detach().float().contiguous()
        return state

    @staticmethod
    def _alloc8(p: Tensor, state: dict, saved: Optional[Tensor]) -> None:
        """One byte buffer per tensor: [m int8 x P][sqrt(v) uint8 x P][fp32 scales x 2 per 2048 block], P = numel
        rounded up to 16; ``exp_avg`` / ``exp_avg_sq`` are views of its two parts (the kernel derives the rest)."""
        n = p.numel()
        padded = (n + 15) // 16 * 16
        blocks = (n + 2047) // 2048
        buf = torch.zeros(2 * padded + 8 * blocks, device=p.device, dtype=torch.uint8) if saved is None else \
            saved.to(p.device, torch.uint8).contiguous()
        state["state8"] = buf
        state["exp_avg"] = buf[:padded]
        state["exp_avg_sq"] = buf[padded:2 * padded]

    def _params(self):
        for group in self.param_groups:
            for p in group["params"]:
                yield group, p

    def _build_tables(self, params: list[Tensor], device) -> tuple[Tensor, Tensor, Tensor]:
        """AdamTensor records (8 x int64 each) and the chunk -> (tensor, start) map.

        The chunk map depends only on the tensor sizes and is cached; the records are rebuilt only when a pointer or
        a per-tensor factor changed (gradients are usually reallocated every step), so the host cost per step is one
        small table, not one Python entry per chunk."""
        import struct

        C = ext()
        rows = []
        for p in params:
            st = self.state[p]
            g = p.grad
            tail = struct.unpack("<q", struct.pack("<if", 0 if g.dtype == torch.float32 else 1,
                                                   float(st["decay_scale"])))[0]
            scale = struct.unpack("<q", struct.pack("<fi", float(self.grad_scale.get(p, 1.0)), 0))[0]
            rows.append((p.data_ptr(), g.data_ptr(), st["master"].data_ptr() if "master" in st else 0,
                         st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(), p.numel(), tail, scale))
        key = (str(device), tuple(rows))
        tables = self.__dict__.setdefault("_table_cache", {})  # one entry per parameter list (parts of a step)
        if key in tables:
            return tables[key]
        sizes = tuple(r[5] for r in rows)
        chunk_cache = self.__dict__.setdefault("_chunk_cache", {})
        if (str(device), sizes) not in chunk_cache:
            chunk = C.adam_chunk_size()
            numels = torch.tensor(sizes, dtype=torch.int64)
            counts = (numels + chunk - 1) // chunk
            owner = torch.repeat_interleave(torch.arange(len(sizes), dtype=torch.int32), counts)
            first = torch.repeat_interleave(torch.cumsum(counts, 0) - counts, counts)
            starts = (torch.arange(owner.numel(), dtype=torch.int64) - first) * chunk
            chunk_cache[(str(device), sizes)] = (owner.to(device), starts.to(device))
        ct, cs = chunk_cache[(str(device), sizes)]
        table = torch.tensor(rows, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
        if len(tables) > 64:  # gradients were reallocated: drop the stale tables of earlier steps
            tables.clear()
        tables[key] = (table, ct, cs)
        return table, ct, cs

    def _live(self):
        out = []
        for group, p in self._params():
            if p.grad is None:
                continue
            if not p.grad.is_contiguous():
                p.grad = p.grad.contiguous()
            st = self._init_state(p)
            st["decay_scale"] = 1.0
            out.append((group, p))
        return out

    # ---- clipping --------------------------------------------------------------------------------
    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, extra_sumsq: Optional[Tensor] = None) -> Tensor:
        """Global L2 norm of all gradients (plus ``extra_sumsq`` from other ranks' shards); the clip coefficient is
        applied inside the next ``step()``. Returns the norm as a 0-d device tensor.

        With ``overlap_with_forward`` (and no ``extra_sumsq``) the norm pass is deferred into ``step()`` on the side
        stream as well; the returned tensor then holds the norm once ``finish()`` has run."""
        if self._side is not None and extra_sumsq is None:
            live = self._live()
            if not live:
                return torch.zeros(())
            device = live[0][1].device
            if self._norm_buf is None or self._norm_buf.device != device:
                self._norm_buf = torch.zeros(2, device=device, dtype=torch.float32)
            self._deferred_clip = float(max_norm)
            return self._norm_buf[0]
        C = ext()
        live = self._live()
        if not live:
            return torch.zeros(())
        params = [p for _, p in live]
        device = params[0].device
        table, ct, cs = self._build_tables(params, device)
        partial = torch.empty(max(1, ct.numel()), device=device, dtype=torch.float64)
        norm = torch.empty(2, device=device, dtype=torch.float32)
        C.adam_grad_norm(table, ct, cs, partial, extra_sumsq, float(max_norm), norm)
        self._clip = norm
        return norm[0]

    @torch.no_grad()
    def grad_sumsq(self, subset: Optional[Iterable[Tensor]] = None) -> Tensor:
        """Sum of squared (scaled) gradients as an fp64 device scalar, over all parameters or ``subset``; used for
        norms that combine several ranks."""
        C = ext()
        live = self._live()
        params = [p for _, p in live]
        if subset is not None:
            wanted = {id(p) for p in subset}
            params = [p for p in params if id(p) in wanted]
        if not params:
            return torch.zeros((), dtype=torch.float64)
        table, ct, cs = self._build_tables(params, params[0].device)
        partial = torch.empty(max(1, ct.numel()), device=params[0].device, dtype=torch.float64)
        C.adam_sumsq(table, ct, cs, partial)
        return partial.sum()

    def set_clip_coefficient(self, coef: Tensor, norm: Optional[Tensor] = None) -> None:
        """Use an externally computed clip coefficient (device scalar) in the next step."""
        n = norm.float().reshape(()) if norm is not None else torch.zeros((), device=coef.device)
        self._clip = torch.stack([n, coef.float().reshape(())])

    # ---- overlap with the next forward -----------------------------------------------------------------
    def overlap_with_forward(self, model) -> None:
        """Run later updates on a side stream in the forward's order of use (see the module docstring)."""
        parts = model.parameter_parts()
        self._side = torch.cuda.Stream()
        # small strided blocks fit beside the forward's persistent kernels but stream too slowly: measured slower
        # (291k vs 312k tokens/s on one B200) than full-size blocks on the side stream, so they stay off
        self._small_blocks = 0
        self._part_of = {id(p): i for i, (_, params) in enumerate(parts) for p in params}
        self._part_events = [None] * len(parts)
        for i, (module, _) in enumerate(parts):
            module.register_forward_pre_hook(self._waiter(i))

    def _waiter(self, i: int):
        def hook(module, args):
            event = self._part_events[i]
            if event is not None:
                torch.cuda.current_stream().wait_event(event)
                self._part_events[i] = None
        return hook

    def finish(self) -> None:
        """The current stream waits for every update in flight on the side stream."""
        if self._side is not None:
            torch.cuda.current_stream().wait_stream(self._side)
            self._part_events = [None] * len(self._part_events)

    # ---- step ------------------------------------------------------------------------------------
    def _step_live(self, live: list) -> None:
        by_group: dict[int, list[Tensor]] = {}
        for group, p in live:
            by_group.setdefault(id(group), []).append(p)
        for group in self.param_groups:
            params = by_group.get(id(group), [])
            if not params:
                continue
            steps = {self.state[p]["step"] for p in params}
            for p in params:
                self.state[p]["step"] += 1
            if len(steps) != 1:  # parameters that joined late: step them one group at a time per step count
                for p in params:
                    self._step_tensors([p], group, self.state[p]["step"])
            else:
                self._step_tensors(params, group, steps.pop() + 1)

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        live = self._live()
        if self._side is None or not live:
            self._step_live(live)
        else:
            # the side stream starts after everything queued so far (gradients, clip coefficient); the gradients
            # and the coefficient of this update stay referenced until the next step
            self._side.wait_stream(torch.cuda.current_stream())
            self._inflight = ([p.grad for _, p in live], self._clip)
            parts: dict[int, list] = {}
            for group, p in live:
                parts.setdefault(self._part_of.get(id(p), 0), []).append((group, p))
            with torch.cuda.stream(self._side):
                clip_max = self.__dict__.pop("_deferred_clip", None)
                if clip_max is not None:  # the norm pass deferred by clip_grad_norm_, ahead of the updates
                    C = ext()
                    params = [p for _, p in live]
                    table, ct, cs = self._build_tables(params, params[0].device)
                    partial = torch.empty(max(1, ct.numel()), device=params[0].device, dtype=torch.float64)
                    C.adam_grad_norm(table, ct, cs, partial, None, clip_max, self._norm_buf)
                    self._clip = self._norm_buf
                    self._inflight = (self._inflight, partial, self._norm_buf)
                for i in range(len(self._part_events)):
                    if i in parts:
                        self._step_live(parts[i])
                    event = torch.cuda.Event()
                    event.record(self._side)
                    self._part_events[i] = event
        self._clip = None
        return loss

    def _step_tensors(self, params: list[Tensor], group: dict, step: int) -> None:
        C = ext()
        table, ct, cs = self._build_tables(params, params[0].device)
        beta1, beta2 = group["betas"]
        # beside the next forward the update uses small strided blocks that fit next to its persistent kernels
        small = self.__dict__.get("_small_blocks", 0) if torch.cuda.current_stream() == self._side else 0
        C.adam_step(table, ct, cs, float(group["lr"]), float(beta1), float(beta2), float(group["eps"]),
                    float(group["weight_decay"]), int(step), self._clip, self.moment_bits == 8, small)

    # ---- checkpoints -----------------------------------------------------------------------------
    def state_dict(self) -> dict:
        self.finish()
        index = {}
        groups = []
        for group in self.param_groups:
            ids = []
            for p in group["params"]:
                index.setdefault(id(p), len(index))
                ids.append(index[id(p)])
            groups.append({k: v for k, v in group.items() if k != "params"} | {"params": ids})
        state = {}
        for group in self.param_groups:
            for p in group["params"]:
                if p in self.state and "exp_avg" in self.state[p]:
                    st = self.state[p]
                    skip = {"decay_scale"} | ({"exp_avg", "exp_avg_sq"} if "state8" in st else set())
                    state[index[id(p)]] = {k: v for k, v in st.items() if k not in skip}
        return {"state": state, "param_groups": groups}

    def load_state_dict(self, state_dict: dict) -> None:
        self.finish()
        params = [p for group in self.param_groups for p in group["params"]]
        for group, saved in zip(self.param_groups, state_dict["param_groups"]):
            for key, value in saved.items():
                if key != "params":
                    group[key] = value
        for idx, st in state_dict["state"].items():
            p = params[int(idx)]
            new = {"step": int(st["step"])}
            if "state8" in st:
                if self.moment_bits != 8:
                    raise ValueError("checkpoint holds 8-bit optimizer moments; build the optimizer with moment_bits=8")
                self._alloc8(p, new, st["state8"])
            elif self.moment_bits == 8 and "exp_avg" in st:
                raise ValueError("checkpoint holds fp32 optimizer moments; build the optimizer with moment_bits=32")
            for key in ("exp_avg", "exp_avg_sq", "master"):
                if key in st and key not in new:
                    new[key] = st[key].to(device=p.device, dtype=torch.float32).contiguous()
            if p.dtype != torch.float32 and "master" not in new:
                new["master"] = p.detach().float().contiguous()
            self.state[p] = new
