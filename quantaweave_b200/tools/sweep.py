"""Hyperparameter sweeps run through the experiment manager: grid, random, successive halving, Bayesian, BOHB-style.

    python -m quantaweave_b200.tools.sweep --config sweep.yaml [--dry-run]

Config and outcome parity with the reference ``src/sweep.py`` (format :1-34, ``expand_grid`` :42,
``sample_random`` :64, ``invalid_reason`` :78, ``run_sweep`` :103-177, ``run_bayes_sweep`` :180-215,
``run_bohb_sweep`` :218-291)::

    name: moe-sweep
    strategy: grid            # grid | random | halving | bayes | bohb
    base: {steps: 200, examples: 2000, sequence_length: 64}
    benchmark: {examples: 300}
    metric: benchmark.loss    # lower is better
    space: {hidden_size: [64, 128], lr: {loguniform: [1.0e-4, 1.0e-3]}}
    n_trials: 8               # random / halving / bayes / bohb budget
    halving: {eta: 2, rungs: 3}
    bayes: {n_init: 5}
    objectives: [benchmark.loss:min, train.tokens_per_second:max]   # optional Pareto report

One rung loop serves grid/random (one rung), halving (survivors, the top 1/eta by ``metric``, rerun with eta x the
steps) and bohb (halving whose base-rung trials a Gaussian process proposes, fitted on base-rung results only; the
promotion rule stays successive halving). ``bayes`` is a single sequential rung driven by the GP. Invalid
combinations (more active than total experts, heads that do not divide the hidden size) are skipped and listed.
"""

from __future__ import annotations

import argparse
import itertools
import json
import math
import random
import time
from pathlib import Path
from typing import Optional

from .bayes_opt import BayesianOptimizer, SearchSpace
from .experiment_manager import (DEFAULT_RUNS_DIR, compare_pareto, compare_runs, dig, load_config, load_summaries,
                                 pareto_front, parse_objectives, run_experiment)

STRATEGIES = ("grid", "random", "halving", "bayes", "bohb")


def expand_grid(space: dict) -> list[dict]:
    for name, options in space.items():
        if not isinstance(options, list):
            raise ValueError(f"grid search needs a list of values for '{name}'")
    names = list(space)
    return [dict(zip(names, combo)) for combo in itertools.product(*(space[n] for n in names))]


def sample_value(spec, rng: random.Random):
    if isinstance(spec, list):
        return rng.choice(spec)
    if isinstance(spec, dict) and len(spec) == 1:
        kind, (lo, hi) = next(iter(spec.items()))
        if kind == "loguniform":
            return math.exp(rng.uniform(math.log(lo), math.log(hi)))
        if kind == "uniform":
            return rng.uniform(lo, hi)
        if kind == "int":
            return rng.randint(int(lo), int(hi))
    raise ValueError(f"unsupported search-space entry {spec!r}; use a list, loguniform, uniform or int")


def sample_random(space: dict, count: int, seed: int) -> list[dict]:
    """Up to ``count`` distinct random trials (fewer when the space is smaller)."""
    rng = random.Random(seed)
    seen: dict[str, dict] = {}
    for _ in range(count * 20):
        trial = {n: sample_value(s, rng) for n, s in space.items()}
        seen.setdefault(json.dumps(trial, sort_keys=True), trial)
        if len(seen) == count:
            break
    return list(seen.values())


def invalid_reason(train: dict) -> Optional[str]:
    experts, active = train.get("total_experts", 184), train.get("active_experts", 1)
    if active > experts:
        return f"active_experts {active} exceeds total_experts {experts}"
    hidden, heads = train.get("hidden_size", 64), train.get("attention_heads", 4)
    if hidden % heads:
        return f"hidden_size {hidden} is not divisible by attention_heads {heads}"
    return None


def make_experiment(config: dict, sweep_name: str, trial: dict, steps: Optional[int] = None, label: str = "") -> dict:
    train = {**config.get("base", {}), **trial}
    if steps is not None:
        train["steps"] = steps
    return {"name": f"{sweep_name}{label}", "train": train, "benchmark": config.get("benchmark", {"examples": 300}),
            "objective": config.get("metric", "benchmark.loss"), "tags": ["sweep", config.get("name", "sweep")]}


def _scored(results: list[dict], metric: str) -> list[dict]:
    return sorted((s for s in results if s["status"] == "completed" and dig(s, metric) is not None),
                  key=lambda s: dig(s, metric))


def _optimizer(config: dict) -> BayesianOptimizer:
    base, b = config.get("base", {}), config.get("bayes", {})
    return BayesianOptimizer(SearchSpace(config["space"]), seed=config.get("seed", 0), n_init=b.get("n_init", 5),
                             n_candidates=b.get("candidates", 2000),
                             validator=lambda trial: invalid_reason({**base, **trial}))


def run_sweep(config: dict, runs_dir: Path = DEFAULT_RUNS_DIR, dry_run: bool = False) -> dict:
    name = config.get("name", "sweep")
    metric = config.get("metric", "benchmark.loss")
    strategy = config.get("strategy", "grid")
    if strategy not in STRATEGIES:
        raise ValueError("strategy must be grid, random, halving, bayes or bohb")
    base = config.get("base", {})
    budget = config.get("n_trials", 12 if strategy in {"bayes", "bohb"} else 8)
    halving = config.get("halving", {})
    eta = halving.get("eta", 2)
    rung_count = halving.get("rungs", 3) if strategy in {"halving", "bohb"} else 1
    base_steps = base.get("steps", 100) if strategy in {"halving", "bohb"} else None
    skipped: list[dict] = []
    optimizer = None
    if strategy in {"bayes", "bohb"}:
        optimizer = _optimizer(config)
        plan = {"name": name, "strategy": strategy, "candidates": budget, "runnable": budget, "skipped": []}
        if dry_run:
            return {**plan, "dry_run": True, "first_trials": [optimizer.suggest() for _ in range(min(3, budget))]}
        valid: list[dict] = []
    else:
        candidates = expand_grid(config["space"]) if strategy == "grid" else \
            sample_random(config["space"], budget, config.get("seed", 0))
        valid = []
        for trial in candidates:
            reason = invalid_reason({**base, **trial})
            (skipped.append({"trial": trial, "reason": reason}) if reason else valid.append(trial))
        plan = {"name": name, "strategy": strategy, "candidates": len(candidates), "runnable": len(valid),
                "skipped": skipped}
        if dry_run:
            return {**plan, "dry_run": True, "first_trials": valid[:5]}
    sweep_dir = Path(runs_dir) / f"{time.strftime('%Y%m%d-%H%M%S')}-{name}"
    sweep_dir.mkdir(parents=True)

    def trial_run(trial: dict, rung: int, index: int, steps: Optional[int]) -> dict:
        label = f"-r{rung}-t{index:02d}" if strategy in {"halving", "bohb", "grid", "random"} else f"-t{index:02d}"
        summary = run_experiment(make_experiment(config, name, trial, steps, label), sweep_dir, run_id=f"trial{label}")
        summary["trial"], summary["rung"] = trial, rung
        return summary

    results: list[dict] = []
    rungs: list[dict] = []
    trajectory: list[Optional[float]] = []
    survivors = valid
    for rung in range(rung_count):
        steps = base_steps * eta ** rung if base_steps is not None else None
        rung_results = []
        proposing = optimizer is not None and rung == 0
        count = budget if proposing else len(survivors)
        for index in range(count):
            trial = optimizer.suggest() if proposing else survivors[index]
            summary = trial_run(trial, rung, index, steps)
            if proposing:
                value = dig(summary, metric) if summary["status"] == "completed" else None
                optimizer.observe(trial, value) if value is not None else optimizer.mark_failed(trial)
                trajectory.append(value)
            rung_results.append(summary)
            print(f"[{name}] rung {rung} trial {index + 1}/{count} {summary['status']} "
                  f"{metric}={dig(summary, metric)}: {trial}")
        results += rung_results
        scored = _scored(rung_results, metric)
        rungs.append({"rung": rung, "steps": steps, "trials": len(rung_results), "completed": len(scored)})
        if rung < rung_count - 1:
            survivors = [s["trial"] for s in scored[: max(1, math.ceil(len(scored) / eta))]]
            if not survivors:
                break
    final_rung = max((s["rung"] for s in results), default=0)
    finals = [s for s in results if s["rung"] == final_rung]
    ranked = _scored(finals, metric)
    outcome = {**plan, "metric": metric, "rungs": rungs, "sweep_dir": str(sweep_dir),
               "best": ({"run_id": ranked[0]["run_id"], "trial": ranked[0]["trial"], "value": dig(ranked[0], metric)}
                        if ranked else None),
               "ranking": [{"run_id": s["run_id"], "trial": s["trial"], "value": dig(s, metric)} for s in ranked],
               "failed": [{"run_id": s["run_id"], "trial": s["trial"], "error": s.get("error")}
                          for s in finals if s["status"] == "failed"]}
    if optimizer is not None:
        outcome["trajectory"] = trajectory
    pareto_md = ""
    if config.get("objectives"):  # a report over the final rung; promotion still follows the scalar metric
        objectives = parse_objectives(config["objectives"])
        outcome["pareto_front"] = [{"run_id": s["run_id"], "trial": s["trial"],
                                    "values": {p: dig(s, p) for p, _ in objectives}}
                                   for s in pareto_front(finals, objectives)]
        pareto_md = "\n## Pareto front\n\n" + compare_pareto(finals, objectives) + "\n"
    (sweep_dir / "sweep_results.json").write_text(json.dumps(outcome, indent=2, default=str) + "\n")
    lines = [f"# Sweep {name} ({strategy})", "", f"metric: `{metric}` (lower is better)", "",
             compare_runs(load_summaries([sweep_dir / s["run_id"] for s in finals]), metric), pareto_md]
    if skipped:
        lines += ["", "## Skipped combinations", "", *[f"- {s['trial']}: {s['reason']}" for s in skipped]]
    (sweep_dir / "sweep_results.md").write_text("\n".join(lines) + "\n")
    return outcome


def run_bayes_sweep(config: dict, runs_dir: Path, dry_run: bool) -> dict:
    return run_sweep({**config, "strategy": "bayes"}, runs_dir, dry_run)


def run_bohb_sweep(config: dict, runs_dir: Path, dry_run: bool) -> dict:
    return run_sweep({**config, "strategy": "bohb"}, runs_dir, dry_run)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", type=Path, required=True)
    p.add_argument("--runs-dir", type=Path, default=DEFAULT_RUNS_DIR)
    p.add_argument("--dry-run", action="store_true", help="print the planned trials and stop before training")
    from .common import describe_options

    describe_options(p, {'runs_dir': "folder the sweep's runs are written to"})
    args = p.parse_args(argv)
    outcome = run_sweep(load_config(args.config), args.runs_dir, args.dry_run)
    print(json.dumps({k: v for k, v in outcome.items() if k not in {"ranking", "skipped"}}, indent=2, default=str))
    if outcome.get("best"):
        print(f"best: {outcome['best']}")


if __name__ == "__main__":
    main()
