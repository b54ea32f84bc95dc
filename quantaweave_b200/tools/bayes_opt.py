"""Bayesian optimisation over a mixed search space: Gaussian process + expected improvement.

Feature parity with the reference ``src/bayes_opt.py`` (``SearchSpace`` :27-128, ``GaussianProcess`` :131-165,
``expected_improvement`` :167-173, ``BayesianOptimizer`` :175-237): the same space entries as the sweeps (a list is a
choice; ``{"loguniform"|"uniform"|"int": [lo, hi]}``), minimisation, failed points never re-proposed.

Method (GP regression as in Rasmussen & Williams, "Gaussian Processes for Machine Learning", ch. 2 and 5): inputs
are encoded into [0, 1] (log scale for loguniform; numeric choices by rank, other choices one-hot) and targets are
standardised. The prior is a unit-variance Matérn-5/2 kernel ``k(r) = (1 + √5 r/ℓ + 5r²/3ℓ²) exp(-√5 r/ℓ)`` plus
observation noise. The length scale ℓ and the noise variance are fitted by minimising the negative log marginal
likelihood ``½ yᵀ(K+σ²I)⁻¹y + ½ log|K+σ²I| + (n/2) log 2π`` with L-BFGS from two starting points, each
parameter kept inside its bounds by a logistic map of its log. The next point maximises expected improvement
(Jones, Schonlau & Welch 1998) ``(f* - μ)Φ(z) + σφ(z)``, ``z = (f* - μ)/σ``, over a candidate pool: fresh random
draws plus local moves around the best observed points at three radii.
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


def _distances(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Euclidean distances between the rows of ``a`` and ``b`` (via the squared-norm expansion)."""
    squared = a.pow(2).sum(-1)[:, None] + b.pow(2).sum(-1)[None, :] - 2.0 * (a @ b.transpose(0, 1))
    return squared.clamp_min(0.0).sqrt()


def _matern52_of_distance(distance: torch.Tensor, length) -> torch.Tensor:
    scaled = math.sqrt(5.0) * distance / length
    return (1.0 + scaled + scaled * scaled / 3.0) * torch.exp(-scaled)


def matern52(a: torch.Tensor, b: torch.Tensor, length: float) -> torch.Tensor:
    """Unit-variance Matérn-5/2 covariance between the rows of ``a`` and the rows of ``b``."""
    return _matern52_of_distance(_distances(a, b), length)


class GaussianProcess:
    """Zero-mean GP on standardised targets; length scale and noise fitted by marginal likelihood."""

    LENGTH_BOUNDS = (0.02, 3.0)
    NOISE_BOUNDS = (1e-6, 0.5)
    STARTS = ((0.25, 1e-3), (0.8, 3e-2))  # (length, noise variance) starting points

    @staticmethod
    def _squash(raw: torch.Tensor, bounds: tuple) -> torch.Tensor:
        lo, hi = math.log(bounds[0]), math.log(bounds[1])
        return torch.exp(lo + (hi - lo) * torch.sigmoid(raw))

    @staticmethod
    def _unsquash(value: float, bounds: tuple) -> float:
        lo, hi = math.log(bounds[0]), math.log(bounds[1])
        t = min(1 - 1e-6, max(1e-6, (math.log(value) - lo) / (hi - lo)))
        return math.log(t / (1 - t))

    def _factor(self, length, noise):
        """Cholesky factor of K + (noise + jitter) I, growing the jitter until the factorisation succeeds."""
        gram = _matern52_of_distance(self._pairwise, length)
        eye = torch.eye(gram.size(0), dtype=gram.dtype)
        jitter = 1e-9
        while True:
            chol, info = torch.linalg.cholesky_ex(gram + (noise + jitter) * eye)
            if int(info) == 0 or jitter > 1e-2:
                return chol, int(info) == 0
            jitter *= 100.0

    def _objective(self, raw: torch.Tensor) -> torch.Tensor:
        length = self._squash(raw[0], self.LENGTH_BOUNDS)
        noise = self._squash(raw[1], self.NOISE_BOUNDS)
        chol, ok = self._factor(length, noise)
        if not ok:
            return torch.tensor(float("inf"), dtype=raw.dtype)
        alpha = torch.cholesky_solve(self.y[:, None], chol)
        n = self.y.numel()
        return (0.5 * (self.y[:, None] * alpha).sum() + torch.log(torch.diagonal(chol)).sum()
                + 0.5 * n * math.log(2 * math.pi))

    def fit(self, x: torch.Tensor, y: torch.Tensor) -> "GaussianProcess":
        self.x = x
        self.mean = y.mean()
        self.scale = y.std(unbiased=False).clamp(min=1e-9)
        self.y = (y - self.mean) / self.scale
        self._pairwise = _distances(x, x)
        best = None
        for length0, noise0 in self.STARTS:
            raw = torch.tensor([self._unsquash(length0, self.LENGTH_BOUNDS),
                                self._unsquash(noise0, self.NOISE_BOUNDS)], dtype=x.dtype, requires_grad=True)
            solver = torch.optim.LBFGS([raw], lr=0.5, max_iter=40, line_search_fn="strong_wolfe")

            def closure():
                solver.zero_grad()
                value = self._objective(raw)
                if torch.isfinite(value):
                    value.backward()
                return value

            try:
                solver.step(closure)
            except RuntimeError:  # a failed line search leaves raw at its last finite point
                pass
            with torch.no_grad():
                value = float(self._objective(raw))
            if math.isfinite(value) and (best is None or value < best[0]):
                best = (value, raw.detach().clone())
        if best is None:
            raise RuntimeError("could not fit the Gaussian process")
        with torch.no_grad():
            self.length = float(self._squash(best[1][0], self.LENGTH_BOUNDS))
            self.noise = float(self._squash(best[1][1], self.NOISE_BOUNDS))
            self.chol, _ = self._factor(self.length, self.noise)
            self.alpha = torch.cholesky_solve(self.y[:, None], self.chol)
        return self

    def predict(self, points: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Posterior mean and standard deviation (of the latent function) in the original target units."""
        cross = matern52(points, self.x, self.length)               # [m, n]
        mean = (cross @ self.alpha)[:, 0]
        solved = torch.linalg.solve_triangular(self.chol, cross.transpose(0, 1), upper=False)  # L⁻¹ k*
        variance = (1.0 - solved.pow(2).sum(dim=0)).clamp(min=1e-12)
        return mean * self.scale + self.mean, variance.sqrt() * self.scale


def expected_improvement(mean: torch.Tensor, std: torch.Tensor, best: float) -> torch.Tensor:
    """Expected amount by which a point with posterior ``(mean, std)`` falls below ``best`` (minimisation)."""
    normal = torch.distributions.Normal(torch.zeros((), dtype=mean.dtype), torch.ones((), dtype=mean.dtype))
    sigma = std.clamp(min=1e-12)
    gain = best - mean
    z = gain / sigma
    return (gain * normal.cdf(z) + sigma * normal.log_prob(z).exp()).clamp(min=0.0)


class BayesianOptimizer:
    """Proposes points of ``space`` to minimise an objective: random points until ``n_init`` finite values are
    known, then the expected-improvement maximiser over ``n_candidates`` random draws plus local moves around the
    three best points. ``validator(params)`` returning a message rejects a point; observed and failed points are
    never proposed again."""

    LOCAL_RADII = (0.03, 0.1, 0.2)
    LOCAL_MOVES = 60  # per radius and incumbent
    INCUMBENTS = 3

    def __init__(self, space: SearchSpace, seed: int = 0, n_init: int = 5, n_candidates: int = 2000,
                 validator: Optional[Callable[[dict], Optional[str]]] = None) -> None:
        self.space = space
        self.rng = random.Random(seed)
        self.n_init = n_init
        self.n_candidates = n_candidates
        self.validator = validator
        self.params: list[dict] = []
        self.values: list[float] = []
        self.seen: set[str] = set()

    def _admissible(self, params: dict) -> bool:
        if self.space.key(params) in self.seen:
            return False
        return self.validator is None or self.validator(params) is None

    def _fresh(self) -> dict:
        for _ in range(1000):
            candidate = self.space.sample(self.rng)
            if self._admissible(candidate):
                return candidate
        raise RuntimeError("could not find an unseen valid configuration; the space may be exhausted")

    def observe(self, params: dict, value: float) -> None:
        self.seen.add(self.space.key(params))
        if math.isfinite(value):
            self.params.append(params)
            self.values.append(float(value))

    def mark_failed(self, params: dict) -> None:
        """Never propose this point again, without teaching the model a made-up value."""
        self.seen.add(self.space.key(params))

    def _pool(self) -> list[dict]:
        ranked = sorted(range(len(self.values)), key=lambda i: self.values[i])
        pool = [self.space.sample(self.rng) for _ in range(self.n_candidates)]
        for index in ranked[: self.INCUMBENTS]:
            incumbent = self.params[index]
            for radius in self.LOCAL_RADII:
                pool.extend(self.space.perturb(incumbent, self.rng, radius) for _ in range(self.LOCAL_MOVES))
        unique: dict[str, dict] = {}
        for candidate in pool:
            key = self.space.key(candidate)
            if key not in unique and self._admissible(candidate):
                unique[key] = candidate
        return list(unique.values())

    def suggest(self) -> dict:
        if len(self.values) < max(2, self.n_init):
            return self._fresh()
        model = GaussianProcess().fit(torch.stack([self.space.encode(p) for p in self.params]),
                                      torch.tensor(self.values, dtype=torch.float64))
        pool = self._pool()
        if not pool:
            return self._fresh()
        mean, std = model.predict(torch.stack([self.space.encode(p) for p in pool]))
        score = expected_improvement(mean, std, min(self.values))
        # with no expected gain anywhere, sample where the model knows least
        pick = std.argmax() if float(score.max()) <= 1e-12 else score.argmax()
        return pool[int(pick)]

    def best(self) -> Optional[tuple[dict, float]]:
        if not self.values:
            return None
        index = min(range(len(self.values)), key=lambda i: self.values[i])
        return self.params[index], self.values[index]
