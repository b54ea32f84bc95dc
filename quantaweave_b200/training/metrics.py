"""JSONL training metrics with throughput, plateau and stability detection (reference ``src/training_metrics.py``).

``MetricsLogger.log`` keeps the reference's wall-clock ``tokens_per_second`` field for log compatibility; the
benchmark numbers of this framework come from CUDA events reduced as a max over ranks (``utils.timing``).
"""

from __future__ import annotations

import json
import math
import time
from pathlib import Path
from typing import Optional, Sequence


def detect_plateau(losses: Sequence[float], window: int = 20, tolerance: float = 0.005) -> bool:
    """True when the last window's mean improved on the previous window's by less than ``tolerance`` (relative)."""
    if len(losses) < 2 * window:
        return False
    recent = sum(losses[-window:]) / window
    previous = sum(losses[-2 * window:-window]) / window
    return previous - recent < tolerance * abs(previous)


def first_stable_step(steps: Sequence[int], losses: Sequence[float], window: int = 20, tolerance: float = 0.02) -> Optional[int]:
    """First step after which consecutive window means never move by more than ``tolerance`` (relative)."""
    if len(losses) < 2 * window:
        return None
    means = [sum(losses[i:i + window]) / window for i in range(0, len(losses) - window + 1, window)]
    for start in range(len(means) - 1):
        tail = means[start:]
        if all(abs(a - b) <= tolerance * max(abs(a), 1e-9) for a, b in zip(tail, tail[1:])):
            return int(steps[start * window])
    return None


class MetricsLogger:
    def __init__(self, path: Optional[Path], total_parameters: int = 0, active_parameters: int = 0) -> None:
        self.path = Path(path) if path is not None else None
        self.total_parameters = total_parameters
        self.active_parameters = active_parameters
        self.steps: list[int] = []
        self.losses: list[float] = []
        self.started = time.perf_counter()
        self.tokens = 0
        self.last: dict = {}
        if self.path is not None:
            self.path.parent.mkdir(parents=True, exist_ok=True)

    def log(self, step: int, tokens: int, **values) -> dict:
        self.tokens += tokens
        elapsed = max(time.perf_counter() - self.started, 1e-9)
        record = {"step": step, "tokens_per_second": self.tokens / elapsed, **values}
        self.last = record
        loss = values.get("loss")
        if loss is not None and math.isfinite(loss):
            self.steps.append(step)
            self.losses.append(loss)
        if self.path is not None:
            with self.path.open("a") as handle:
                handle.write(json.dumps(record) + "\n")
        return record

    def summary(self) -> dict:
        losses = self.losses
        tail = [l for s, l in zip(self.steps, losses) if s > self.steps[-1] - 20] if losses else []
        ratio = self.active_parameters / self.total_parameters if self.total_parameters else None
        return {
            "steps_logged": len(losses),
            "final_loss": sum(tail) / len(tail) if tail else None,
            "best_loss": min(losses) if losses else None,
            "tokens_per_second": self.tokens / max(time.perf_counter() - self.started, 1e-9),
            "plateaued": detect_plateau(losses),
            "first_stable_step": first_stable_step(self.steps, losses),
            "total_parameters": self.total_parameters,
            "active_parameters": self.active_parameters,
            "active_parameter_ratio": ratio,
        }
