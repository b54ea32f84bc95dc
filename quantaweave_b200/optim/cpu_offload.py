"""AdamW with its moments in pinned host memory (reference ``src/cpu_offload_optimizer.py``).

Each step copies every gradient to a reused pinned staging buffer, applies the ``torch.optim.AdamW`` update on the
CPU against an fp32 host master copy, and copies the new weights back. Frees 8 bytes/parameter of device memory
(12 for bf16 parameters, whose fp32 master also lives on the host) at the cost of host<->device traffic per step.
"""

from __future__ import annotations

from typing import Iterable

import torch


class CPUOffloadAdamW(torch.optim.Optimizer):
    def __init__(self, parameters: Iterable, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01) -> None:
        items = list(parameters)
        if items and not isinstance(items[0], dict):
            items = [p for p in items if p.requires_grad]  # frozen parameters hold no optimizer state
        super().__init__(items, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))

    def state_numel(self) -> int:
        """Elements of optimizer state (the two AdamW moments) kept in host memory instead of device memory."""
        return sum(st["exp_avg"].numel() + st["exp_avg_sq"].numel() for st in self.state.values() if "exp_avg" in st)

    def _host_state(self, p: torch.Tensor) -> dict:
        st = self.state[p]
        if "exp_avg" not in st:
            pin = p.is_cuda
            st["step"] = 0
            st["exp_avg"] = torch.zeros(p.shape, dtype=torch.float32, pin_memory=pin)
            st["exp_avg_sq"] = torch.zeros(p.shape, dtype=torch.float32, pin_memory=pin)
            st["master"] = p.detach().to("cpu", torch.float32).clone()
            if pin:
                st["master"] = st["master"].pin_memory()
        if "staging" not in st:  # a reused transfer buffer; never saved
            st["staging"] = torch.empty(p.shape, dtype=torch.float32, pin_memory=p.is_cuda)
        return st

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            lr, eps, wd = group["lr"], group["eps"], group["weight_decay"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self._host_state(p)
                st["staging"].copy_(p.grad.float(), non_blocking=False)
                g = st["staging"]
                st["step"] += 1
                t = st["step"]
                master = st["master"]
                master.mul_(1 - lr * wd)
                st["exp_avg"].lerp_(g, 1 - beta1)
                st["exp_avg_sq"].mul_(beta2).addcmul_(g, g, value=1 - beta2)
                step_size = lr / (1 - beta1 ** t)
                denom = (st["exp_avg_sq"].sqrt() / (1 - beta2 ** t) ** 0.5).add_(eps)
                master.addcdiv_(st["exp_avg"], denom, value=-step_size)
                p.copy_(master.to(p.device, p.dtype, non_blocking=p.is_cuda))
        return loss

    def state_dict(self) -> dict:
        base = super().state_dict()
        # the base class hands out the live per-parameter dicts: filter copies, never the optimizer's own state
        base["state"] = {idx: {k: v for k, v in st.items() if k != "staging"} for idx, st in base["state"].items()}
        return base

    def load_state_dict(self, state_dict: dict) -> None:
        params = [p for g in self.param_groups for p in g["params"]]
        for group, saved in zip(self.param_groups, state_dict["param_groups"]):
            for key, value in saved.items():
                if key != "params":
                    group[key] = value
        for idx, st in state_dict["state"].items():
            p = params[int(idx)]
            host = self._host_state(p)
            host["step"] = int(st["step"])
            for key in ("exp_avg", "exp_avg_sq", "master"):
                if key in st:
                    host[key].copy_(st[key].to(torch.float32))
