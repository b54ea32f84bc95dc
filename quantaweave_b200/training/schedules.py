"""Open-loop schedules and closed-loop controllers for MoE training.

The option names, their defaults, the controllers' decisions and the state-dict keys are those of the reference
``src/moe_schedules.py`` (``ScheduleConfig`` :15-64, ``TrainingController`` :67-214), so a run resumed from either
framework's checkpoint continues the same trajectory. What each knob does:

* LR: linear warmup, then constant / cosine / linear decay to ``min_lr_ratio``; plateau halving by ``lr_scale``;
* router aux weight: optional linear anneal to ``aux_coef_end``, times an adaptive factor from load imbalance;
* router temperature: optional anneal from ``temperature_start``, times an exploration boost when experts go idle;
* capacity factor: grows when the dropped fraction exceeds ``drop_threshold``, shrinks otherwise; optional release
  step after which capacity is not enforced.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, fields
from typing import Callable, Optional


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


def _ramp(start: float, end: float, progress: float) -> float:
    """Linear interpolation from ``start`` to ``end``; ``progress`` is clipped to [0, 1]."""
    return start + (end - start) * min(1.0, max(0.0, progress))


def _nudge(value: float, direction: int, up: float, down: float, low: float, high: float) -> float:
    """One multiplicative controller move: ``direction`` +1 scales by ``up`` (capped at ``high``), -1 by ``down``
    (floored at ``low``), 0 leaves the value alone."""
    if direction > 0:
        return min(value * up, high)
    if direction < 0:
        return max(value * down, low)
    return value


# decay shapes after warmup: multiplier of the peak LR at progress t in [0, 1], given the floor ratio
_DECAY: dict[str, Callable[[float, float], float]] = {
    "constant": lambda t, floor: 1.0,
    "linear": lambda t, floor: _ramp(1.0, floor, t),
    "cosine": lambda t, floor: floor + (1.0 - floor) * 0.5 * (1.0 + math.cos(math.pi * t)),
}


class TrainingController:
    """Step-indexed schedules (``lr_at``, ``aux_coef_at``, ``temperature_at``) times the multipliers that the
    closed-loop rules maintain. The trainer calls ``observe`` every step, ``update`` every ``interval`` steps with
    the load imbalance and the active-expert share, and ``apply`` before each step."""

    # persistent controller state, in state-dict order
    _STATE = ("lr_scale", "aux_factor", "temperature_boost", "capacity_factor", "released", "best_loss",
              "stale_intervals")

    def __init__(self, config: ScheduleConfig, base_temperature: float = 1.0) -> None:
        self.config = config
        self.base_temperature = base_temperature
        self.lr_scale = self.aux_factor = self.temperature_boost = 1.0
        self.capacity_factor = config.capacity_factor
        self.released = False
        self.best_loss = math.inf
        self.stale_intervals = 0
        self._window: list[tuple[float, float]] = []  # (loss, dropped fraction) since the last update
        self.history: list[dict] = []

    # ---- open loop -------------------------------------------------------------------------------------------
    def lr_at(self, step: int) -> float:
        c = self.config
        if c.warmup_steps and step < c.warmup_steps:  # the (step+1)-th of warmup_steps equal increments
            return c.lr * (step + 1) / c.warmup_steps * self.lr_scale
        span = c.total_steps - c.warmup_steps
        if span <= 0:
            return c.lr * self.lr_scale
        progress = min(1.0, max(0.0, (step - c.warmup_steps) / span))
        return c.lr * _DECAY[c.lr_decay](progress, c.min_lr_ratio) * self.lr_scale

    def aux_coef_at(self, step: int) -> float:
        c = self.config
        annealed = c.aux_coef_end is not None and c.total_steps > 0
        base = _ramp(c.aux_coef, c.aux_coef_end, step / c.total_steps) if annealed else c.aux_coef
        return base * self.aux_factor

    def temperature_at(self, step: int) -> float:
        c = self.config
        if c.temperature_start is None:
            base = self.base_temperature
        elif c.temperature_steps > 0:
            base = _ramp(c.temperature_start, c.temperature_end, step / c.temperature_steps)
        else:
            base = c.temperature_start
        return base * self.temperature_boost

    # ---- closed loop -----------------------------------------------------------------------------------------
    def observe(self, loss: float, dropped_fraction: float) -> None:
        self._window.append((loss, dropped_fraction))

    def should_update(self, step: int) -> bool:
        return step % self.config.interval == 0

    def _plateau(self, losses: list) -> Optional[float]:
        """Track the best interval-mean loss; after ``plateau_patience`` intervals without a gain of at least
        ``plateau_min_delta``, scale the LR by ``plateau_factor`` (not below ``min_lr_scale``) and start over."""
        c = self.config
        if not losses:
            return None
        mean = sum(losses) / len(losses)
        improved = mean < self.best_loss - c.plateau_min_delta
        self.best_loss = mean if improved else self.best_loss
        self.stale_intervals = 0 if improved else self.stale_intervals + 1
        if not (c.plateau_patience and self.stale_intervals >= c.plateau_patience):
            return None
        self.stale_intervals = 0
        return max(self.lr_scale * c.plateau_factor, c.min_lr_scale)

    def update(self, step: int, imbalance: Optional[float] = None, active_fraction: Optional[float] = None) -> dict:
        """Run the closed-loop rules on the interval just ended; returns the values that changed."""
        c = self.config
        losses = [loss for loss, _ in self._window]
        drops = [drop for _, drop in self._window]
        self._window = []
        proposals: list[tuple[str, str, Optional[float]]] = [("lr_scale", "lr_scale", self._plateau(losses))]
        if c.capacity_adapt and not self.released and drops:
            heavy = sum(drops) / len(drops) > c.drop_threshold
            proposals.append(("capacity_factor", "capacity_factor",
                              _nudge(self.capacity_factor, 1 if heavy else -1, c.capacity_up, c.capacity_down,
                                     c.capacity_min, c.capacity_max)))
        if c.aux_adapt and imbalance is not None:
            direction = 1 if imbalance > c.balance_high else (-1 if imbalance < c.balance_low else 0)
            proposals.append(("aux_factor", "aux_factor",
                              _nudge(self.aux_factor, direction, c.aux_up, c.aux_down, c.aux_factor_min,
                                     c.aux_factor_max)))
        if c.temperature_adapt and active_fraction is not None:
            idle = active_fraction < c.dead_expert_fraction
            proposals.append(("temperature_boost", "temperature_boost",
                              _nudge(self.temperature_boost, 1 if idle else -1, 1.05, 0.98, 1.0,
                                     c.temperature_boost_max)))
        changes: dict[str, float] = {}
        for attribute, key, value in proposals:
            if value is not None and value != getattr(self, attribute):
                setattr(self, attribute, value)
                changes[key] = value
        if c.capacity_release_step and step >= c.capacity_release_step and not self.released:
            self.released = True
            changes["capacity_released"] = 1.0
        if changes:
            self.history.append({"step": step, **changes})
        return changes

    def apply(self, model, optimizer, step: int) -> dict[str, float]:
        """Set this step's LR on every parameter group and the routing controls on the model; returns the values
        for the metrics log."""
        lr = self.lr_at(step)
        for group in optimizer.param_groups:
            group["lr"] = lr
        temperature, aux = self.temperature_at(step), self.aux_coef_at(step)
        model.set_routing_controls(capacity_factor=self.capacity_factor, drop_overflow_tokens=not self.released,
                                   router_temperature=temperature, router_aux_loss_coef=aux)
        return {"lr": lr, "capacity_factor": self.capacity_factor, "capacity_enforced": 0.0 if self.released else 1.0,
                "router_temperature": temperature, "router_aux_loss_coef": aux}

    # ---- checkpoint state --------------------------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"config": asdict(self.config), **{name: getattr(self, name) for name in self._STATE},
                "history": [dict(entry) for entry in self.history]}

    def load_state_dict(self, state: dict) -> None:
        for name in self._STATE:
            setattr(self, name, state[name])
        self.history = [dict(entry) for entry in state.get("history", [])]


def schedule_field_names() -> list[str]:
    """Every ``ScheduleConfig`` option name, in declaration order."""
    return [f.name for f in fields(ScheduleConfig)]
