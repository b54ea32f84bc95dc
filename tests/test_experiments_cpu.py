"""Experiment manager, sweeps, Bayesian optimisation and the architecture calculator (reference tests:
tests/test_experiment_manager.py, tests/test_sweep.py, tests/test_bayes_opt.py, tests/test_model_scaling.py)."""

import json
import math
import random

import pytest
import torch

from quantaweave_b200.tools.bayes_opt import BayesianOptimizer, GaussianProcess, SearchSpace, expected_improvement
from quantaweave_b200.tools.experiment_manager import (compare_pareto, compare_runs, dominates, load_summaries,
                                                       pareto_front, run_experiment, update_best)
from quantaweave_b200.tools.model_scaling import b200_plan, make_spec
from quantaweave_b200.tools.sweep import expand_grid, invalid_reason, run_sweep, sample_random


def _base(tmp_path):
    from test_tools_cpu import _corpus

    data = _corpus(tmp_path / "data.jsonl", 60)
    return dict(data=[str(data)], examples=40, tokenizer="char", sequence_length=16, hidden_size=16, layers=1,
                ffn_size=32, attention_heads=2, total_experts=4, active_experts=1, batch_size=2, steps=2,
                device="cpu", no_power_tracking=True)


def test_experiment_run_best_and_compare(tmp_path):
    base = _base(tmp_path)
    runs = tmp_path / "runs"
    a = run_experiment({"name": "a", "train": {**base, "lr": 1e-3}, "promotion_threshold": 0.1}, runs)
    b = run_experiment({"name": "b", "train": {**base, "lr": 3e-3}}, runs)
    assert a["status"] == b["status"] == "completed"
    for f in ("config.json", "summary.json", "report.md", "metrics.jsonl", "train.log", "model/model.pt"):
        assert (runs / a["run_id"] / f).exists(), f
    best = json.loads((runs / "best.json").read_text())
    assert best["objective"] == "train.final_loss"
    summaries = load_summaries([runs / a["run_id"], runs / b["run_id"]])
    table = compare_runs(summaries, "train.final_loss")
    assert "| lr" in table.splitlines()[0] or " lr " in table.splitlines()[0]
    bad = run_experiment({"name": "bad", "train": {**base, "data": [str(tmp_path / "missing.jsonl")]}}, runs)
    assert bad["status"] == "failed" and (runs / bad["run_id"] / "error.txt").exists()


def test_update_best_promotion_threshold(tmp_path):
    s = {"run_id": "r1", "run_dir": "x", "train": {"final_loss": 5.0}}
    assert update_best(tmp_path, s, None, promotion_threshold=4.0)
    assert json.loads((tmp_path / "best.json").read_text())["promotable"] is False
    assert not update_best(tmp_path, {**s, "run_id": "r2", "train": {"final_loss": 6.0}}, None)
    assert update_best(tmp_path, {**s, "run_id": "r3", "train": {"final_loss": 3.0}}, None, 4.0)
    best = json.loads((tmp_path / "best.json").read_text())
    assert best["run_id"] == "r3" and best["promotable"] is True


def test_pareto_front():
    runs = [{"run_id": n, "status": "completed", "b": {"loss": l, "tps": t}}
            for n, l, t in [("a", 1.0, 10), ("b", 2.0, 30), ("c", 2.5, 20), ("d", 1.0, 5)]]
    objectives = ["b.loss:min", "b.tps:max"]
    assert {s["run_id"] for s in pareto_front(runs, objectives)} == {"a", "b"}
    assert dominates(runs[0], runs[3], [("b.loss", "min"), ("b.tps", "max")])
    assert "| a |" in compare_pareto(runs, objectives)


def test_sweep_helpers_and_grid_halving(tmp_path):
    assert len(expand_grid({"a": [1, 2], "b": [3, 4, 5]})) == 6
    trials = sample_random({"lr": {"loguniform": [1e-4, 1e-2]}, "k": [1, 2]}, 5, 0)
    assert len(trials) == 5 and all(1e-4 <= t["lr"] <= 1e-2 for t in trials)
    assert invalid_reason({"total_experts": 2, "active_experts": 3})
    assert invalid_reason({"hidden_size": 30, "attention_heads": 4})
    base = _base(tmp_path)
    cfg = {"name": "g", "strategy": "grid", "base": base, "metric": "train.final_loss", "benchmark": None,
           "space": {"lr": [1e-3, 2e-3], "active_experts": [1, 8]}}
    dry = run_sweep(cfg, tmp_path / "s", dry_run=True)
    assert dry["runnable"] == 2 and len(dry["skipped"]) == 2
    cfg.update(strategy="halving", halving={"eta": 2, "rungs": 2}, space={"lr": [1e-3, 2e-3]})
    out = run_sweep(cfg, tmp_path / "s")
    assert [r["trials"] for r in out["rungs"]] == [2, 1] and out["rungs"][1]["steps"] == 4
    assert out["best"] is not None


def test_gp_and_bayes_optimizer_find_minimum():
    x = torch.linspace(0, 1, 8, dtype=torch.float64)[:, None]
    y = (x[:, 0] - 0.3) ** 2
    gp = GaussianProcess().fit(x, y)
    mean, std = gp.predict(x)
    assert torch.allclose(mean, y, atol=1e-2) and (std < 0.05).all()
    assert float(expected_improvement(torch.tensor([0.0]), torch.tensor([1.0]), 0.0)) == pytest.approx(
        1 / math.sqrt(2 * math.pi), rel=1e-6)
    space = SearchSpace({"x": {"uniform": [0.0, 1.0]}, "c": ["p", "q"]})
    opt = BayesianOptimizer(space, seed=1, n_init=4, n_candidates=300)
    for _ in range(16):
        p = opt.suggest()
        opt.observe(p, (p["x"] - 0.7) ** 2 + (0.0 if p["c"] == "q" else 0.5))
    best, value = opt.best()
    assert best["c"] == "q" and abs(best["x"] - 0.7) < 0.15 and value < 0.03
    with pytest.raises(ValueError):
        SearchSpace({"lr": {"loguniform": [0.0, 1.0]}})


def test_model_scaling_presets_and_b200_plan():
    spec = make_spec("moe", "xl")
    assert spec.ffn_size == round(4096 * 2.75)
    assert spec.total_params == spec.embedding_params + spec.attention_params + spec.expert_params
    dense = make_spec("dense", "m")
    assert dense.manifest()["num_experts"] == 1 and dense.active_params == dense.total_params
    plan = b200_plan(make_spec("moe", "l"))
    assert plan["expert_parallel"] in (1, 2, 4) and plan["train_flops_per_token"] > 0
    assert b200_plan(make_spec("moe", "xxl"))["fits_on_one_node"] is False
    with pytest.raises(ValueError):
        make_spec("moe", "s", top_k=9)
