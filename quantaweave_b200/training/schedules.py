"""Open-loop schedules and closed-loop controllers for MoE training.

Behaviour and state-dict contents match the reference ``src/moe_schedules.py`` (``ScheduleConfig`` :15-64,
``TrainingController`` :67-214) so that a resumed run continues the same trajectory:

* LR: linear warmup, then constant / cosine / linear decay to ``min_lr_ratio``; plateau halving by ``lr_scale``;
* router aux weight: optional linear anneal to ``aux_coef_end``, times an adaptive factor from load imbalance;
* router temperature: optional anneal from ``temperature_start``, times an exploration boost when experts go idle;
* capacity factor: grows when the dropped fraction exceeds ``drop_threshold``, shrinks otherwise; optional release
  step after which capacity is not enforced.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, fields
from typing import Optional


@dataclass
class ScheduleConfig:
    lr: float = 3e-4
    total_steps: int = 0
    warmup_steps: int = 0
    lr_decay: str = "constant"
    min_lr_ratio: float = 0.1
    plateau_patience: int = 0
    plateau_factor: float = 0.5
    plateau_min_delta: float = 1e-3
    min_lr_scale: float = 0.05
    aux_coef: float = 0.01
    aux_coef_end: Optional[float] = None
    aux_adapt: bool = False
    aux_factor_min: float = 0.25
    aux_factor_max: float = 4.0
    aux_up: float = 1.05
    aux_down: float = 0.98
    balance_low: float = 0.25
    balance_high: float = 1.0
    capacity_factor: float = 1.25
    capacity_adapt: bool = False
    capacity_min: float = 1.0
    capacity_max: float = 4.0
    capacity_up: float = 1.1
    capacity_down: float = 0.99
    drop_threshold: float = 0.01
    capacity_release_step: int = 0
    temperature_start: Optional[float] = None
    temperature_end: float = 1.0
    temperature_steps: int = 0
    temperature_adapt: bool = False
    temperature_boost_max: float = 4.0
    dead_expert_fraction: float = 0.5
    interval: int = 50

    def __post_init__(self) -> None:
        if self.lr_decay not in {"constant", "cosine", "linear"}:
            raise ValueError("lr_decay must be constant, cosine or linear")
        if self.interval < 1:
            raise ValueError("interval must be positive")
        if not 0 <= self.min_lr_ratio <= 1:
            raise ValueError("min_lr_ratio must be in [0, 1]")
        if self.capacity_min > self.capacity_max:
            raise ValueError("capacity_min cannot exceed capacity_max")


class TrainingController:
    _STATE = ("lr_scale", "aux_factor", "temperature_boost", "capacity_factor", "released", "best_loss",
              "stale_intervals")

    def __init__(self, config: ScheduleConfig, base_temperature: float = 1.0) -> None:
        self.config = config
        self.base_temperature = base_temperature
        self.lr_scale = 1.0
        self.aux_factor = 1.0
        self.temperature_boost = 1.0
        self.capacity_factor = config.capacity_factor
        self.released = False
        self.best_loss = math.inf
        self.stale_intervals = 0
        self._losses: list[float] = []
        self._drops: list[float] = []
        self.history: list[dict] = []

    # ---- open loop -------------------------------------------------------------
    def lr_at(self, step: int) -> float:
        c = self.config
        if c.warmup_steps and step < c.warmup_steps:
            return c.lr * (step + 1) / c.warmup_steps * self.lr_scale
        span = c.total_steps - c.warmup_steps
        if c.lr_decay == "constant" or span <= 0:
            return c.lr * self.lr_scale
        t = min(1.0, max(0.0, (step - c.warmup_steps) / span))
        if c.lr_decay == "cosine":
            factor = c.min_lr_ratio + (1 - c.min_lr_ratio) * 0.5 * (1 + math.cos(math.pi * t))
        else:
            factor = 1 - (1 - c.min_lr_ratio) * t
        return c.lr * factor * self.lr_scale

    def aux_coef_at(self, step: int) -> float:
        c = self.config
        if c.aux_coef_end is None or c.total_steps <= 0:
            base = c.aux_coef
        else:
            base = c.aux_coef + (c.aux_coef_end - c.aux_coef) * min(1.0, step / c.total_steps)
        return base * self.aux_factor

    def temperature_at(self, step: int) -> float:
        c = self.config
        if c.temperature_start is None:
            base = self.base_temperature
        elif c.temperature_steps <= 0:
            base = c.temperature_start
        else:
            base = c.temperature_start + (c.temperature_end - c.temperature_start) * min(1.0, step / c.temperature_steps)
        return base * self.temperature_boost

    # ---- closed loop -------------------------------------------------------------
    def observe(self, loss: float, dropped_fraction: float) -> None:
        self._losses.append(loss)
        self._drops.append(dropped_fraction)

    def should_update(self, step: int) -> bool:
        return step % self.config.interval == 0

    def update(self, step: int, imbalance: Optional[float] = None, active_fraction: Optional[float] = None) -> dict:
        c = self.config
        changes: dict[str, float] = {}
        if self._losses:
            mean_loss = sum(self._losses) / len(self._losses)
            if mean_loss < self.best_loss - c.plateau_min_delta:
                self.best_loss, self.stale_intervals = mean_loss, 0
            else:
                self.stale_intervals += 1
            if c.plateau_patience and self.stale_intervals >= c.plateau_patience:
                scale = max(self.lr_scale * c.plateau_factor, c.min_lr_scale)
                if scale != self.lr_scale:
                    self.lr_scale = scale
                    changes["lr_scale"] = scale
                self.stale_intervals = 0
        if c.capacity_adapt and not self.released and self._drops:
            drops = sum(self._drops) / len(self._drops)
            if drops > c.drop_threshold:
                target = min(self.capacity_factor * c.capacity_up, c.capacity_max)
            else:
                target = max(self.capacity_factor * c.capacity_down, c.capacity_min)
            if target != self.capacity_factor:
                self.capacity_factor = target
                changes["capacity_factor"] = target
        if c.aux_adapt and imbalance is not None:
            if imbalance > c.balance_high:
                factor = min(self.aux_factor * c.aux_up, c.aux_factor_max)
            elif imbalance < c.balance_low:
                factor = max(self.aux_factor * c.aux_down, c.aux_factor_min)
            else:
                factor = self.aux_factor
            if factor != self.aux_factor:
                self.aux_factor = factor
                changes["aux_factor"] = factor
        if c.temperature_adapt and active_fraction is not None:
            if active_fraction < c.dead_expert_fraction:
                boost = min(self.temperature_boost * 1.05, c.temperature_boost_max)
            else:
                boost = max(self.temperature_boost * 0.98, 1.0)
            if boost != self.temperature_boost:
                self.temperature_boost = boost
                changes["temperature_boost"] = boost
        if c.capacity_release_step and step >= c.capacity_release_step and not self.released:
            self.released = True
            changes["capacity_released"] = 1.0
        self._losses.clear()
        self._drops.clear()
        if changes:
            self.history.append({"step": step, **changes})
        return changes

    def apply(self, model, optimizer, step: int) -> dict[str, float]:
        lr = self.lr_at(step)
        for group in optimizer.param_groups:
            group["lr"] = lr
        controls = dict(capacity_factor=self.capacity_factor, drop_overflow_tokens=not self.released,
                        router_temperature=self.temperature_at(step), router_aux_loss_coef=self.aux_coef_at(step))
        model.set_routing_controls(**controls)
        return {"lr": lr, "capacity_factor": self.capacity_factor, "capacity_enforced": float(not self.released),
                "router_temperature": controls["router_temperature"],
                "router_aux_loss_coef": controls["router_aux_loss_coef"]}

    # ---- checkpoint state --------------------------------------------------------
    def state_dict(self) -> dict:
        state = {"config": asdict(self.config)}
        state.update({name: getattr(self, name) for name in self._STATE})
        state["history"] = list(self.history)
        return state

    def load_state_dict(self, state: dict) -> None:
        for name in self._STATE:
            setattr(self, name, state[name])
        self.history = list(state.get("history", []))


def schedule_field_names() -> list[str]:
    return [f.name for f in fields(ScheduleConfig)]
