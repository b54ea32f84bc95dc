"""Bayesian optimisation (reference tests: tests/test_bayes_opt.py): the GP-guided search beats random search on a
smooth objective, every parameter kind encodes into the unit cube, bad spaces are refused, the GP interpolates and
is uncertain away from its data, expected improvement prefers a low mean and a high uncertainty, suggestions are
valid and never repeat (failed points included), non-finite observations are ignored, and the sweep runner's bayes
strategy drives training runs."""

import json
import math
import random
from pathlib import Path

import pytest
import torch

from quantaweave_b200.tools.bayes_opt import BayesianOptimizer, GaussianProcess, SearchSpace, expected_improvement


def _objective(p):
    return (math.log10(p["lr"]) + 3.0) ** 2 + (p["x"] - 0.25) ** 2 + (0.0 if p["act"] == "silu" else 0.3)


SPACE = {"lr": {"loguniform": [1e-5, 1e-1]}, "x": {"uniform": [0.0, 1.0]}, "act": ["relu", "silu", "gelu"]}


def test_bayesian_search_beats_random_search_on_a_smooth_objective():
    wins = 0
    for seed in range(3):
        opt = BayesianOptimizer(SearchSpace(SPACE), seed=seed, n_init=5, n_candidates=500)
        for _ in range(20):
            p = opt.suggest()
            opt.observe(p, _objective(p))
        rng = random.Random(100 + seed)
        space = SearchSpace(SPACE)
        random_best = min(_objective(space.sample(rng)) for _ in range(20))
        wins += opt.best()[1] < random_best
    assert wins >= 2


def test_every_parameter_kind_encodes_into_the_unit_cube():
    space = SearchSpace({"lr": {"loguniform": [1e-4, 1e-2]}, "d": {"uniform": [-1.0, 1.0]}, "n": {"int": [1, 9]},
                         "k": [1, 2, 8], "name": ["a", "b", "c"]})
    assert space.dimension == 1 + 1 + 1 + 1 + 3  # numeric choices by rank, others one-hot
    rng = random.Random(0)
    for _ in range(50):
        p = space.sample(rng)
        code = space.encode(p)
        assert code.shape == (7,) and bool(((code >= 0) & (code <= 1)).all())
        assert isinstance(p["n"], int) and 1 <= p["n"] <= 9 and p["k"] in (1, 2, 8) and p["name"] in "abc"
    low = space.encode({"lr": 1e-4, "d": -1.0, "n": 1, "k": 1, "name": "b"})
    high = space.encode({"lr": 1e-2, "d": 1.0, "n": 9, "k": 8, "name": "c"})
    assert low[:4].tolist() == [0.0, 0.0, 0.0, 0.0] and high[:4].tolist() == [1.0, 1.0, 1.0, 1.0]
    assert low[4:].tolist() == [0.0, 1.0, 0.0] and high[4:].tolist() == [0.0, 0.0, 1.0]
    mid = space.encode({"lr": 1e-3, "d": 0.0, "n": 5, "k": 2, "name": "a"})
    assert mid[:4].tolist() == pytest.approx([0.5, 0.5, 0.5, 0.5])


@pytest.mark.parametrize("bad", [{}, {"lr": {"loguniform": [0.0, 1.0]}}, {"lr": {"uniform": [1.0, 1.0]}},
                                 {"lr": {"normal": [0.0, 1.0]}}, {"k": []}, {"lr": 0.1}])
def test_bad_spaces_are_refused(bad):
    with pytest.raises(ValueError):
        SearchSpace(bad)


def test_the_gp_interpolates_its_data_and_is_uncertain_away_from_it():
    x = torch.linspace(0.0, 0.5, 9, dtype=torch.float64)[:, None]
    y = torch.sin(6 * x[:, 0])
    gp = GaussianProcess().fit(x, y)
    mean, std = gp.predict(x)
    assert torch.allclose(mean, y, atol=1e-2) and (std < 0.05).all()
    _, far = gp.predict(torch.tensor([[0.95]], dtype=torch.float64))
    assert float(far) > 5 * float(std.max())


def test_expected_improvement_prefers_low_mean_and_high_uncertainty():
    ei = expected_improvement(torch.tensor([0.0, 1.0, 1.0, 2.0]), torch.tensor([0.1, 0.1, 1.0, 1e-9]), best=1.0)
    assert ei[0] > ei[1] and ei[2] > ei[1] and float(ei[3]) == 0.0
    assert float(expected_improvement(torch.tensor([0.0]), torch.tensor([1.0]), 0.0)) == pytest.approx(
        1 / math.sqrt(2 * math.pi), rel=1e-6)


def test_suggestions_are_valid_never_repeat_and_remember_failures():
    space = SearchSpace({"k": [1, 2, 3, 4], "e": [2, 4, 8]})
    invalid = lambda p: "top-k above experts" if p["k"] > p["e"] else None  # noqa: E731
    opt = BayesianOptimizer(space, seed=0, n_init=2, n_candidates=50, validator=invalid)
    seen = []
    for i in range(10):  # 10 valid combinations: each is suggested exactly once
        p = opt.suggest()
        assert invalid(p) is None and space.key(p) not in seen
        seen.append(space.key(p))
        opt.mark_failed(p) if i % 3 == 0 else opt.observe(p, float(p["k"] + p["e"]))
    assert len(opt.values) == 6  # failed points taught the model nothing
    with pytest.raises(RuntimeError):
        opt.suggest()  # the space is exhausted


def test_non_finite_observations_are_ignored():
    opt = BayesianOptimizer(SearchSpace({"x": {"uniform": [0.0, 1.0]}}), seed=0)
    p, q = opt.suggest(), opt.suggest()
    opt.observe(p, float("nan"))
    opt.observe(q, float("inf"))
    assert opt.values == [] and opt.best() is None
    r = opt.suggest()
    opt.observe(r, 2.0)
    assert opt.best() == (r, 2.0)


def test_the_bayes_strategy_drives_training_runs(tmp_path):
    from quantaweave_b200.tools.sweep import run_sweep

    data = tmp_path / "d.jsonl"
    data.write_text("".join(json.dumps({"text": f"story {i}: the fox."}) + "\n" for i in range(40)))
    base = dict(data=[str(data)], examples=40, tokenizer="char", sequence_length=16, hidden_size=16, layers=1,
                ffn_size=16, attention_heads=2, total_experts=4, active_experts=1, batch_size=2, steps=1,
                device="cpu", no_power_tracking=True)
    out = run_sweep({"name": "bo", "strategy": "bayes", "base": base, "metric": "train.final_loss", "n_trials": 4,
                     "bayes": {"n_init": 2, "candidates": 64}, "space": {"lr": {"loguniform": [1e-4, 1e-2]}}},
                    tmp_path / "runs")
    assert len(out["trajectory"]) == 4 and all(v is not None for v in out["trajectory"])
    assert out["best"]["value"] == min(out["trajectory"])
    assert (Path(out["sweep_dir"]) / "sweep_results.md").exists()
