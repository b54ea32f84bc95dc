"""Bayesian optimisation over a mixed search space: Gaussian process + expected improvement.

Feature parity with the reference ``src/bayes_opt.py`` (``SearchSpace`` :27-128, ``GaussianProcess`` :131-165,
``expected_improvement`` :167-173, ``BayesianOptimizer`` :175-237): the same space entries as the sweeps (a list is a
choice; ``{"loguniform"|"uniform"|"int": [lo, hi]}``), minimisation, failed points never re-proposed.

Method (textbook GP regression, Rasmussen & Williams ch. 2 and 4): inputs encoded into [0, 1] (log scale for
loguniform; numeric choices by rank, other choices one-hot); targets standardised; Matérn-5/2 kernel
``k(r) = (1 + √5 r/ℓ + 5r²/3ℓ²) exp(-√5 r/ℓ)``; the length scale ℓ and noise are picked on a grid by the log
marginal likelihood ``-½ yᵀα - Σ log diag(L)``; the next point maximises expected improvement
``(f* - μ)Φ(z) + σφ(z)`` over random candidates plus jittered copies of the best points.
"""

from __future__ import annotations

import json
import math
import random
from typing import Callable, Optional

import torch


def _bounded(entry) -> Optional[tuple[str, float, float]]:
    if isinstance(entry, dict) and len(entry) == 1:
        kind, bounds = next(iter(entry.items()))
        return kind, bounds[0], bounds[1]
    return None


class SearchSpace:
    def __init__(self, spec: dict) -> None:
        if not spec:
            raise ValueError("the search space is empty")
        self.spec = dict(spec)
        self.names = list(spec)
        self.widths: dict[str, int] = {}
        for name, entry in self.spec.items():
            if isinstance(entry, list):
                if not entry:
                    raise ValueError(f"'{name}' has no choices")
                self.widths[name] = 1 if self._numeric(entry) else len(entry)
                continue
            b = _bounded(entry)
            ok = b is not None and b[0] in {"loguniform", "uniform", "int"} and b[1] < b[2]
            if ok and b[0] == "loguniform" and b[1] <= 0:
                raise ValueError(f"'{name}': loguniform bounds must be positive")
            if not ok:
                raise ValueError(f"unsupported search-space entry for '{name}': {entry!r}")
            self.widths[name] = 1
        self.dimension = sum(self.widths.values())

    @staticmethod
    def _numeric(choices: list) -> bool:
        return all(isinstance(v, (int, float)) and not isinstance(v, bool) for v in choices)

    @staticmethod
    def _to_unit(kind: str, lo: float, hi: float, value: float) -> float:
        if kind == "loguniform":
            return (math.log(value) - math.log(lo)) / (math.log(hi) - math.log(lo))
        return (value - lo) / (hi - lo)

    @staticmethod
    def _from_unit(kind: str, lo: float, hi: float, unit: float):
        unit = min(1.0, max(0.0, unit))
        if kind == "loguniform":
            return min(hi, max(lo, math.exp(math.log(lo) + unit * (math.log(hi) - math.log(lo)))))
        if kind == "int":
            return int(round(lo + unit * (hi - lo)))
        return lo + unit * (hi - lo)

    def sample(self, rng: random.Random) -> dict:
        out = {}
        for name, entry in self.spec.items():
            if isinstance(entry, list):
                out[name] = rng.choice(entry)
                continue
            kind, lo, hi = _bounded(entry)
            if kind == "int":
                out[name] = rng.randint(int(lo), int(hi))
            elif kind == "loguniform":
                out[name] = min(hi, max(lo, math.exp(rng.uniform(math.log(lo), math.log(hi)))))
            else:
                out[name] = rng.uniform(lo, hi)
        return out

    def encode(self, params: dict) -> torch.Tensor:
        cols: list[float] = []
        for name, entry in self.spec.items():
            value = params[name]
            if isinstance(entry, list):
                i = entry.index(value)
                if self._numeric(entry):
                    cols.append(i / max(1, len(entry) - 1))
                else:
                    cols += [float(j == i) for j in range(len(entry))]
            else:
                cols.append(self._to_unit(*_bounded(entry), value))
        return torch.tensor(cols, dtype=torch.float64)

    def perturb(self, params: dict, rng: random.Random, scale: float = 0.1) -> dict:
        """A nearby point: bounded parameters jitter in the unit encoding, choices re-draw with probability 0.2."""
        out = {}
        for name, entry in self.spec.items():
            if isinstance(entry, list):
                out[name] = rng.choice(entry) if rng.random() < 0.2 else params[name]
            else:
                kind, lo, hi = _bounded(entry)
                out[name] = self._from_unit(kind, lo, hi, self._to_unit(kind, lo, hi, params[name]) + rng.gauss(0, scale))
        return out

    def key(self, params: dict) -> str:
        return json.dumps(params, sort_keys=True, default=str)


def matern52(a: torch.Tensor, b: torch.Tensor, length: float) -> torch.Tensor:
    r = torch.cdist(a, b) / length
    s = math.sqrt(5.0) * r
    return (1.0 + s + (5.0 / 3.0) * r * r) * torch.exp(-s)


class GaussianProcess:
    """Zero-mean GP on standardised targets; (length, noise) chosen on a grid by marginal likelihood."""

    LENGTHS = (0.1, 0.2, 0.35, 0.6, 1.0)
    NOISES = (1e-6, 1e-4, 1e-2, 1e-1)

    def fit(self, x: torch.Tensor, y: torch.Tensor) -> "GaussianProcess":
        self.x = x
        self.mean = y.mean()
        self.scale = y.std(unbiased=False).clamp(min=1e-9)
        self.y = (y - self.mean) / self.scale
        eye = torch.eye(x.size(0), dtype=x.dtype)
        best = None
        for length in self.LENGTHS:
            gram = matern52(x, x, length)
            for noise in self.NOISES:
                chol, info = torch.linalg.cholesky_ex(gram + (noise + 1e-8) * eye)
                if int(info):
                    continue
                alpha = torch.cholesky_solve(self.y[:, None], chol)
                lml = float(-0.5 * (self.y[:, None] * alpha).sum() - torch.log(torch.diagonal(chol)).sum())
                if best is None or lml > best[0]:
                    best = (lml, length, noise, chol, alpha)
        if best is None:
            raise RuntimeError("could not fit the Gaussian process")
        _, self.length, self.noise, self.chol, self.alpha = best
        return self

    def predict(self, points: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        k = matern52(points, self.x, self.length)
        mean = (k @ self.alpha).squeeze(-1)
        v = torch.cholesky_solve(k.t(), self.chol)
        var = (1.0 - (k * v.t()).sum(dim=1)).clamp(min=1e-12)
        return mean * self.scale + self.mean, var.sqrt() * self.scale


def expected_improvement(mean: torch.Tensor, std: torch.Tensor, best: float) -> torch.Tensor:
    """Expected improvement below ``best`` (minimisation)."""
    std = std.clamp(min=1e-12)
    z = (best - mean) / std
    return ((best - mean) * torch.special.ndtr(z) + std * torch.exp(-0.5 * z * z) / math.sqrt(2 * math.pi)).clamp(min=0)


class BayesianOptimizer:
    def __init__(self, space: SearchSpace, seed: int = 0, n_init: int = 5, n_candidates: int = 2000,
                 validator: Optional[Callable[[dict], Optional[str]]] = None) -> None:
        self.space, self.rng = space, random.Random(seed)
        self.n_init, self.n_candidates, self.validator = n_init, n_candidates, validator
        self.params: list[dict] = []
        self.values: list[float] = []
        self.seen: set[str] = set()

    def _ok(self, p: dict) -> bool:
        return self.space.key(p) not in self.seen and (self.validator is None or self.validator(p) is None)

    def _random(self) -> dict:
        for _ in range(1000):
            p = self.space.sample(self.rng)
            if self._ok(p):
                return p
        raise RuntimeError("could not find an unseen valid configuration; the space may be exhausted")

    def observe(self, params: dict, value: float) -> None:
        self.seen.add(self.space.key(params))
        if math.isfinite(value):
            self.params.append(params)
            self.values.append(float(value))

    def mark_failed(self, params: dict) -> None:
        """Never propose this point again, without teaching the model a made-up value."""
        self.seen.add(self.space.key(params))

    def suggest(self) -> dict:
        if len(self.values) < max(2, self.n_init):
            return self._random()
        gp = GaussianProcess().fit(torch.stack([self.space.encode(p) for p in self.params]),
                                   torch.tensor(self.values, dtype=torch.float64))
        pool = [self.space.sample(self.rng) for _ in range(self.n_candidates)]
        for i in sorted(range(len(self.values)), key=self.values.__getitem__)[:3]:
            for scale in (0.03, 0.1, 0.2):
                pool += [self.space.perturb(self.params[i], self.rng, scale) for _ in range(60)]
        pool = [p for p in pool if self._ok(p)]
        if not pool:
            return self._random()
        mean, std = gp.predict(torch.stack([self.space.encode(p) for p in pool]))
        ei = expected_improvement(mean, std, min(self.values))
        if float(ei.max()) <= 1e-12:  # nothing promises improvement: explore where the model is least sure
            return pool[int(std.argmax())]
        return pool[int(ei.argmax())]

    def best(self) -> Optional[tuple[dict, float]]:
        if not self.values:
            return None
        i = min(range(len(self.values)), key=self.values.__getitem__)
        return self.params[i], self.values[i]
