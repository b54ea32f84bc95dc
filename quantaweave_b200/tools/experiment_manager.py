"""Experiment manager: reproducible, comparable training runs.

    python -m quantaweave_b200.tools.experiment_manager run --config configs/exp.yaml
    python -m quantaweave_b200.tools.experiment_manager list    [--runs-dir artifacts/experiments]
    python -m quantaweave_b200.tools.experiment_manager compare artifacts/experiments/* [--markdown report.md]

Parity with the reference ``src/experiment_manager.py`` (config bundle format and run layout :1-24,
``update_best`` :90-114 with the promotion threshold, ``run_experiment`` :116-167, ``compare_runs`` :216-240,
Pareto helpers :243-295, charts and CLI :298-380). A bundle (YAML or JSON)::

    name: moe-balanced
    tags: [balanced]
    train: {steps: 300, total_experts: 8, capacity_adapt: true}   # trainer options by python name
    benchmark: {examples: 500}                                    # optional final benchmark
    objective: benchmark.loss                                     # lower is better
    promotion_threshold: 3.5                                      # optional: best.json "promotable" gate

Each run gets ``<runs-dir>/<time>-<name>-<hash>/`` with config.json, metrics.jsonl, train.log, diagnostics,
checkpoints, the model, summary.json and report.md; ``best.json`` tracks the best run per objective.
"""

from __future__ import annotations

import argparse
import contextlib
import hashlib
import io
import json
import re
import subprocess
import sys
import time
import traceback
from pathlib import Path
from typing import Optional

from ..utils.routing_diagnostics import bar_chart_svg, line_chart_svg

DEFAULT_RUNS_DIR = Path("artifacts/experiments")


def load_config(path: Path) -> dict:
    path = Path(path)
    if path.suffix in {".yaml", ".yml"}:
        import yaml

        return yaml.safe_load(path.read_text())
    return json.loads(path.read_text())


def slug(text: str) -> str:
    return re.sub(r"[^a-z0-9]+", "-", text.lower()).strip("-") or "run"


def git_revision() -> Optional[str]:
    try:
        out = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True, check=True,
                             cwd=Path(__file__).parent).stdout.strip()
        return out or None
    except (OSError, subprocess.CalledProcessError):
        return None


class _Tee(io.TextIOBase):
    def __init__(self, *streams) -> None:
        self.streams = streams

    def write(self, text: str) -> int:
        for s in self.streams:
            s.write(text)
        return len(text)

    def flush(self) -> None:
        for s in self.streams:
            s.flush()


def dig(record, dotted: str):
    """``record["a"]["b"]`` for ``"a.b"``; None when any part is missing."""
    for part in dotted.split("."):
        if not isinstance(record, dict) or part not in record:
            return None
        record = record[part]
    return record


def objective_of(summary: dict, objective: Optional[str]) -> tuple[str, Optional[float]]:
    name = objective or ("benchmark.loss" if summary.get("benchmark") else "train.final_loss")
    value = dig(summary, name)
    return name, float(value) if isinstance(value, (int, float)) else None


def update_best(runs_dir: Path, summary: dict, objective: Optional[str],
                promotion_threshold: Optional[float] = None) -> bool:
    """Record ``summary`` in ``best.json`` when it beats the best on the same objective (lower is better).
    ``promotable`` is true only when the value is at or below ``promotion_threshold`` (always, without one), so the
    least bad of several failing runs is never presented as deployable."""
    name, value = objective_of(summary, objective)
    if value is None:
        return False
    best_path = Path(runs_dir) / "best.json"
    if best_path.exists():
        best = json.loads(best_path.read_text())
        if best.get("objective") == name and best["value"] <= value:
            return False
    promotable = promotion_threshold is None or value <= promotion_threshold
    best_path.write_text(json.dumps({"run_id": summary["run_id"], "objective": name, "value": value,
                                     "path": summary["run_dir"], "promotable": promotable,
                                     "promotion_threshold": promotion_threshold}, indent=2) + "\n")
    return True


def run_experiment(config: dict, runs_dir: Path = DEFAULT_RUNS_DIR, name: Optional[str] = None,
                   run_id: Optional[str] = None) -> dict:
    from ..training import trainer

    runs_dir = Path(runs_dir)
    name = name or config.get("name", "experiment")
    overrides = dict(config.get("train", {}))
    for key in ("output", "checkpoint_dir", "metrics_file", "diagnostics_dir", "resume"):
        overrides.pop(key, None)  # the manager owns the run's locations
    trainer.default_args(**overrides)  # unknown option names fail before anything is created
    digest = hashlib.sha256(json.dumps(overrides, sort_keys=True, default=str).encode()).hexdigest()[:6]
    run_id = run_id or f"{time.strftime('%Y%m%d-%H%M%S')}-{slug(name)}-{digest}"
    run_dir = runs_dir / run_id
    run_dir.mkdir(parents=True, exist_ok=False)
    steps = overrides.get("steps", trainer.default_args().steps)
    resolved = {"run_id": run_id, "name": name, "description": config.get("description"),
                "tags": config.get("tags", []), "train": overrides, "benchmark": config.get("benchmark", {}),
                "objective": config.get("objective"), "created": time.strftime("%Y-%m-%dT%H:%M:%S"),
                "git_revision": git_revision(), "argv": sys.argv}
    (run_dir / "config.json").write_text(json.dumps(resolved, indent=2, default=str) + "\n")
    args = trainer.default_args(**{"diagnostics_interval": max(1, steps // 20), **overrides},
                                output=run_dir / "model", checkpoint_dir=run_dir / "checkpoints",
                                metrics_file=run_dir / "metrics.jsonl", diagnostics_dir=run_dir / "diagnostics",
                                resume=False)
    summary: dict = {"run_id": run_id, "name": name, "run_dir": str(run_dir), "tags": resolved["tags"]}
    started = time.perf_counter()
    with (run_dir / "train.log").open("w") as log, contextlib.redirect_stdout(_Tee(sys.stdout, log)):
        try:
            result = trainer.run_training(args)
            routing = result.get("last_routing") or {}
            train = {k: result.get(k) for k in ("steps", "final_loss", "best_loss", "tokens_per_second", "plateaued",
                                                "first_stable_step", "active_parameter_ratio", "total_parameters",
                                                "active_parameters", "precision")}
            train.update(overflow_fraction=(result.get("last_log") or {}).get("overflow_fraction"),
                         routing_imbalance=routing.get("imbalance"),
                         active_expert_fraction=routing.get("active_fraction"),
                         controller_changes=len(result.get("controller_history", [])))
            summary.update(status="completed", train=train)
            if config.get("benchmark") is not None:
                summary["benchmark"] = run_final_benchmark(run_dir, args, config.get("benchmark") or {})
        except Exception as error:  # noqa: BLE001 - a failed run is recorded, not raised
            summary.update(status="failed", error=f"{type(error).__name__}: {error}")
            (run_dir / "error.txt").write_text(traceback.format_exc())
    summary["seconds"] = time.perf_counter() - started
    if summary["status"] == "completed":
        summary["is_best"] = update_best(runs_dir, summary, config.get("objective"), config.get("promotion_threshold"))
    (run_dir / "summary.json").write_text(json.dumps(summary, indent=2, default=str) + "\n")
    (run_dir / "report.md").write_text(render_run_report(resolved, summary))
    return summary


def run_final_benchmark(run_dir: Path, args, options: dict) -> dict:
    from .benchmark import build_parser, render_markdown, run_benchmark

    data = options.get("data", args.data[0] if args.data else None)
    argv = ["--checkpoint", str(run_dir / "model"), "--data", str(data), "--examples",
            str(options.get("examples", 500)), "--batch-size", str(options.get("batch_size", args.batch_size)),
            "--device", args.device, "--training-metrics", str(run_dir / "metrics.jsonl")]
    if options.get("no_routing_stats"):
        argv.append("--no-routing-stats")
    report = run_benchmark(build_parser().parse_args(argv))
    (run_dir / "benchmark.json").write_text(json.dumps(report, indent=2) + "\n")
    (run_dir / "benchmark.md").write_text(render_markdown(report))
    keep = ("loss", "perplexity", "tokens_per_second", "dropped_route_fraction", "overflow_route_fraction",
            "expert_utilization_min", "expert_utilization_max", "active_parameter_ratio", "total_parameters")
    result = {k: report[k] for k in keep}
    if "routing" in report:
        result.update(dead_experts=report["routing"]["dead_experts_total"],
                      routing_entropy=report["routing"]["entropy_mean"])
    return result


def render_run_report(config: dict, summary: dict) -> str:
    lines = [f"# {summary['name']} ({summary['run_id']})", "", f"- status: **{summary['status']}**",
             f"- wall time: {summary.get('seconds', 0):.1f}s", f"- git revision: {config.get('git_revision')}", ""]
    if config.get("description"):
        lines += [config["description"], ""]
    lines += ["## Configuration", "", "| option | value |", "|---|---|",
              *[f"| {k} | {v} |" for k, v in config["train"].items()], ""]
    if summary["status"] == "failed":
        return "\n".join(lines + ["## Failure", "", f"`{summary['error']}` (traceback in error.txt)", ""])
    for section in ("train", "benchmark"):
        if summary.get(section):
            lines += [f"## {section.capitalize()} results", "", "| metric | value |", "|---|---|",
                      *[f"| {k} | {v} |" for k, v in summary[section].items()], ""]
    return "\n".join(lines)


# ---- comparison ------------------------------------------------------------------------------------------
def load_summaries(paths: list[Path]) -> list[dict]:
    out = []
    for path in map(Path, paths):
        summary_path = path / "summary.json" if path.is_dir() else path
        if summary_path.exists():
            summary = json.loads(summary_path.read_text())
            cfg = summary_path.parent / "config.json"
            summary["config"] = json.loads(cfg.read_text()) if cfg.exists() else {}
            out.append(summary)
    return out


def _fmt(v) -> str:
    return "-" if v is None else (f"{v:.4g}" if isinstance(v, float) else str(v))


def compare_runs(summaries: list[dict], metric: str = "benchmark.loss") -> str:
    """Markdown table of the completed runs ranked by ``metric`` (lower is better) plus the options that differ."""
    done = sorted((s for s in summaries if s.get("status") == "completed"),
                  key=lambda s: (dig(s, metric) is None, dig(s, metric) or 0))
    trains = [s["config"].get("train", {}) for s in done]
    differing = [o for o in sorted({k for t in trains for k in t})
                 if len({json.dumps(t.get(o), default=str) for t in trains}) > 1]
    columns = list(dict.fromkeys(["run", metric, "train.final_loss", "benchmark.perplexity",
                                  "train.tokens_per_second", "train.active_parameter_ratio",
                                  "train.overflow_fraction", "benchmark.dead_experts"]))
    lines = ["| " + " | ".join(columns + differing) + " |", "|" + "---|" * (len(columns) + len(differing))]
    for s in done:
        train = s["config"].get("train", {})
        cells = [s["run_id"], *[_fmt(dig(s, c)) for c in columns[1:]], *[_fmt(train.get(o)) for o in differing]]
        lines.append("| " + " | ".join(cells) + " |")
    failed = [s for s in summaries if s.get("status") == "failed"]
    if failed:
        lines += ["", "Failed runs: " + ", ".join(f"{s['run_id']} ({s.get('error')})" for s in failed)]
    return "\n".join(lines)


def parse_objectives(spec) -> list[tuple[str, str]]:
    """``["benchmark.loss:min", "train.tokens_per_second:max"]`` -> [(path, direction)]; a bare path means min."""
    items = [spec] if isinstance(spec, str) else list(spec)
    out = []
    for item in items:
        path, _, direction = item.partition(":")
        direction = direction or "min"
        if direction not in {"min", "max"}:
            raise ValueError(f"objective '{item}': direction must be 'min' or 'max'")
        out.append((path.strip(), direction))
    if len(out) < 2:
        raise ValueError("multi-objective needs at least two objectives")
    return out


def dominates(a: dict, b: dict, objectives: list[tuple[str, str]]) -> bool:
    """``a`` is at least as good as ``b`` on every objective and strictly better on one."""
    strictly = False
    for path, direction in objectives:
        va, vb = dig(a, path), dig(b, path)
        if va is None or vb is None:
            return False
        sign = 1 if direction == "min" else -1
        if sign * (va - vb) > 0:
            return False
        strictly = strictly or sign * (va - vb) < 0
    return strictly


def pareto_front(summaries: list[dict], objectives) -> list[dict]:
    if objectives and isinstance(objectives[0], str):
        objectives = parse_objectives(objectives)
    pool = [s for s in summaries if s.get("status") == "completed"
            and all(dig(s, p) is not None for p, _ in objectives)]
    return [s for s in pool if not any(dominates(o, s, objectives) for o in pool if o is not s)]


def compare_pareto(summaries: list[dict], objectives) -> str:
    parsed = parse_objectives(objectives) if objectives and isinstance(objectives[0], str) else objectives
    done = [s for s in summaries if s.get("status") == "completed"]
    front = {id(s) for s in pareto_front(done, parsed)}
    columns = [f"{p} ({d})" for p, d in parsed]
    lines = ["| run | " + " | ".join(columns) + " | pareto-optimal |", "|" + "---|" * (len(columns) + 2)]
    for s in sorted(done, key=lambda s: id(s) not in front):
        lines.append(f"| {s['run_id']} | " + " | ".join(_fmt(dig(s, p)) for p, _ in parsed)
                     + f" | {'yes' if id(s) in front else ''} |")
    return "\n".join(lines)


def loss_curves_svg(summaries: list[dict]) -> str:
    series: dict[str, list[tuple[int, float]]] = {}
    for s in summaries:
        path = Path(s["run_dir"]) / "metrics.jsonl"
        if path.exists():
            rows = [json.loads(x) for x in path.read_text().splitlines() if x.strip()]
            series[s["run_id"]] = [(r["step"], r["loss"]) for r in rows if "loss" in r]
    if not any(series.values()):
        return ""
    steps = sorted({x for pts in series.values() for x, _ in pts})
    lines = {name: [dict(pts).get(x, pts[-1][1]) for x in steps] for name, pts in series.items() if pts}
    return line_chart_svg(steps, lines, "Training loss")


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="command", required=True)
    run = sub.add_parser("run", help="train one configuration file as a tracked run")
    run.add_argument("--config", type=Path, required=True)
    run.add_argument("--name")
    run.add_argument("--runs-dir", type=Path, default=DEFAULT_RUNS_DIR)
    listing = sub.add_parser("list", help="show the tracked runs and which one is best")
    listing.add_argument("--runs-dir", type=Path, default=DEFAULT_RUNS_DIR)
    cmp = sub.add_parser("compare", help="order runs by a metric and draw charts of them")
    cmp.add_argument("runs", type=Path, nargs="+")
    cmp.add_argument("--metric", default="benchmark.loss")
    cmp.add_argument("--objectives", nargs="+", help="2+ dotted.path:min|max entries (Pareto ranking)")
    cmp.add_argument("--markdown", type=Path)
    cmp.add_argument("--charts-dir", type=Path, help="folder for the loss-curve and metric-bar SVG charts")
    from .common import describe_options

    describe_options(p, {'runs_dir': 'folder of tracked runs'})
    args = p.parse_args(argv)
    if args.command == "run":
        summary = run_experiment(load_config(args.config), args.runs_dir, args.name)
        print(f"\n{summary['run_id']}: {summary['status']} in {summary['seconds']:.1f}s -> {summary['run_dir']}")
        if summary["status"] == "failed":
            sys.exit(f"run failed: {summary['error']}")
    elif args.command == "list":
        dirs = sorted(d for d in args.runs_dir.iterdir() if d.is_dir()) if args.runs_dir.exists() else []
        print(compare_runs(load_summaries(dirs)))
        best = args.runs_dir / "best.json"
        if best.exists():
            print("\nbest:", json.loads(best.read_text()))
    else:
        summaries = load_summaries(args.runs)
        table = compare_pareto(summaries, args.objectives) if args.objectives else compare_runs(summaries, args.metric)
        print(table)
        if args.markdown:
            args.markdown.write_text(table + "\n")
        if args.charts_dir:
            args.charts_dir.mkdir(parents=True, exist_ok=True)
            (args.charts_dir / "loss_curves.svg").write_text(loss_curves_svg(summaries))
            values = {s["run_id"]: dig(s, args.metric) for s in summaries
                      if isinstance(dig(s, args.metric), (int, float))}
            (args.charts_dir / "metric_bars.svg").write_text(bar_chart_svg(values, args.metric))


if __name__ == "__main__":
    main()
