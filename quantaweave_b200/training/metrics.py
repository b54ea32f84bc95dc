"""JSONL training metrics: one record per logged step, plus a run summary with plateau and stability verdicts.

Public names and record keys follow the reference ``src/training_metrics.py`` (``MetricsLogger`` :33-76,
``detect_plateau`` :10, ``first_stable_step`` :20), because the trainer's log, the experiment manager and the
benchmark report read them. ``tokens_per_second`` in these records is host wall-clock throughput since the logger
was made (as in the reference); the framework's benchmark figures come from CUDA events reduced as a max over
ranks (``utils.timing``).

Stability is judged on block means: the loss sequence is cut into consecutive blocks of ``window`` values and
each block is replaced by its mean. A run has *plateaued* when the last ``window`` losses improve on the
``window`` before them by less than ``tolerance`` of the earlier mean. It is *stable from* the first block after
which no two neighbouring block means differ by more than ``tolerance`` of the earlier one; that block's first
step is reported.
"""

from __future__ import annotations

import json
import math
import time
from pathlib import Path
from typing import Optional, Sequence


def _mean(values: Sequence[float]) -> float:
    return math.fsum(values) / len(values)


def _block_means(values: Sequence[float], width: int) -> list[float]:
    """Means of the complete, non-overlapping blocks of ``width`` values (a trailing partial block is dropped)."""
    return [_mean(values[i:i + width]) for i in range(0, len(values) // width * width, width)]


def _within(earlier: float, later: float, tolerance: float) -> bool:
    return abs(later - earlier) <= tolerance * max(abs(earlier), 1e-9)


def detect_plateau(losses: Sequence[float], window: int = 20, tolerance: float = 0.005) -> bool:
    """Whether the mean of the last ``window`` losses beat the mean of the ``window`` before it by less than
    ``tolerance`` (relative to the earlier mean). Fewer than ``2 * window`` losses: not enough evidence, False."""
    if window <= 0 or len(losses) < 2 * window:
        return False
    tail = list(losses[-2 * window:])
    earlier, later = _mean(tail[:window]), _mean(tail[window:])
    return earlier - later < tolerance * abs(earlier)


def first_stable_step(steps: Sequence[int], losses: Sequence[float], window: int = 20,
                      tolerance: float = 0.02) -> Optional[int]:
    """First step of the earliest block from which every later block mean stays within ``tolerance`` of the one
    before it; None while the newest pair of blocks still moves, or with fewer than two blocks."""
    if window <= 0 or len(losses) < 2 * window:
        return None
    means = _block_means(list(losses), window)
    # walk back from the newest block while each neighbour pair is close: the longest stable suffix
    first = len(means) - 1
    while first > 0 and _within(means[first - 1], means[first], tolerance):
        first -= 1
    if first == len(means) - 1:
        return None
    return int(steps[first * window])


class MetricsLogger:
    """Appends one JSON object per logged step to ``path`` (when given) and keeps what the summary needs.

    ``log(step, tokens, **values)`` adds ``tokens`` to the running count, writes ``{"step", "tokens_per_second",
    **values}`` and returns that record; finite ``loss`` values feed the summary."""

    TAIL_STEPS = 20  # ``final_loss`` averages the losses logged within the last 20 steps

    def __init__(self, path: Optional[Path], total_parameters: int = 0, active_parameters: int = 0) -> None:
        self.path = None if path is None else Path(path)
        self.total_parameters = total_parameters
        self.active_parameters = active_parameters
        self.steps: list[int] = []
        self.losses: list[float] = []
        self.tokens = 0
        self.last: dict = {}
        self.started = time.perf_counter()
        if self.path is not None:
            self.path.parent.mkdir(parents=True, exist_ok=True)

    def _throughput(self) -> float:
        return self.tokens / max(time.perf_counter() - self.started, 1e-9)

    def _append(self, record: dict) -> None:
        if self.path is None:
            return
        line = json.dumps(record)
        with open(self.path, "a") as sink:
            sink.write(line + "\n")

    def log(self, step: int, tokens: int, **values) -> dict:
        self.tokens += tokens
        record = dict(step=step, tokens_per_second=self._throughput())
        record.update(values)
        loss = values.get("loss")
        if isinstance(loss, (int, float)) and math.isfinite(loss):
            self.steps.append(step)
            self.losses.append(float(loss))
        self._append(record)
        self.last = record
        return record

    def _final_loss(self) -> Optional[float]:
        if not self.losses:
            return None
        horizon = self.steps[-1] - self.TAIL_STEPS
        recent = [loss for step, loss in zip(self.steps, self.losses) if step > horizon]
        return _mean(recent)

    def summary(self) -> dict:
        total, active = self.total_parameters, self.active_parameters
        return {
            "steps_logged": len(self.losses),
            "final_loss": self._final_loss(),
            "best_loss": min(self.losses, default=None),
            "tokens_per_second": self._throughput(),
            "plateaued": detect_plateau(self.losses),
            "first_stable_step": first_stable_step(self.steps, self.losses),
            "total_parameters": total,
            "active_parameters": active,
            "active_parameter_ratio": (active / total) if total else None,
        }
