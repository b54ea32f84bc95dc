"""Experiment manager: training runs that are reproducible, tracked and comparable.

    python -m quantaweave_b200.tools.experiment_manager run --config configs/exp.yaml
    python -m quantaweave_b200.tools.experiment_manager list    [--runs-dir artifacts/experiments]
    python -m quantaweave_b200.tools.experiment_manager compare artifacts/experiments/* [--markdown report.md]

The config bundle, the run folder layout, ``best.json`` with its promotion gate, and the public names follow the
reference's ``src/experiment_manager.py``. A bundle (YAML or JSON)::

    name: moe-balanced
    tags: [balanced]
    train: {steps: 300, total_experts: 8, capacity_adapt: true}   # trainer options by python name
    benchmark: {examples: 500}                                    # optional final benchmark
    objective: benchmark.loss                                     # lower is better
    promotion_threshold: 3.5                                      # optional: best.json "promotable" gate

A run is a folder ``<runs-dir>/<time>-<name>-<hash>/`` holding config.json, train.log, metrics.jsonl, diagnostics,
checkpoints, the model, summary.json and report.md. Values inside summaries are addressed by dotted paths
(``train.final_loss``); ``best.json`` in the runs folder names the best run for the objective in use.
"""

from __future__ import annotations

import argparse
import contextlib
import functools
import hashlib
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
_LOCATIONS = ("output", "checkpoint_dir", "metrics_file", "diagnostics_dir", "resume")  # chosen by the manager
_TRAIN_KEYS = ("steps", "final_loss", "best_loss", "tokens_per_second", "plateaued", "first_stable_step",
               "active_parameter_ratio", "total_parameters", "active_parameters", "precision")
_BENCH_KEYS = ("loss", "perplexity", "tokens_per_second", "dropped_route_fraction", "overflow_route_fraction",
               "expert_utilization_min", "expert_utilization_max", "active_parameter_ratio", "total_parameters")
_TABLE_COLUMNS = ("train.final_loss", "benchmark.perplexity", "train.tokens_per_second",
                  "train.active_parameter_ratio", "train.overflow_fraction", "benchmark.dead_experts")


def load_config(path: Path) -> dict:
    path = Path(path)
    text = path.read_text()
    if path.suffix.lower() in (".yaml", ".yml"):
        import yaml

        return yaml.safe_load(text)
    return json.loads(text)


def slug(text: str) -> str:
    """Lower-case words joined by dashes (``run`` when nothing is left)."""
    words = re.findall(r"[a-z0-9]+", text.lower())
    return "-".join(words) or "run"


def git_revision() -> Optional[str]:
    try:
        done = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True, check=True,
                              cwd=Path(__file__).parent)
    except (OSError, subprocess.CalledProcessError):
        return None
    return done.stdout.strip() or None


def dig(record, dotted: str):
    """The value at a dotted path (``"train.final_loss"``), or None when any step of the path is missing."""
    def step(node, key):
        return node.get(key) if isinstance(node, dict) else None

    return functools.reduce(step, dotted.split("."), record)


def objective_of(summary: dict, objective: Optional[str]) -> tuple[str, Optional[float]]:
    """(path, value) of the objective; without one, the benchmark loss when there is a benchmark, else the final
    training loss."""
    path = objective or ("benchmark.loss" if summary.get("benchmark") else "train.final_loss")
    value = dig(summary, path)
    return path, (float(value) if isinstance(value, (int, float)) else None)


def update_best(runs_dir: Path, summary: dict, objective: Optional[str],
                promotion_threshold: Optional[float] = None) -> bool:
    """Point ``best.json`` at ``summary`` if it is the lowest value seen for this objective; returns True then.

    ``promotable`` is set only when the value is at or below ``promotion_threshold`` (always when there is none), so
    the best of several poor runs is never presented as good enough to deploy."""
    path, value = objective_of(summary, objective)
    if value is None:
        return False
    record_file = Path(runs_dir) / "best.json"
    if record_file.exists():
        current = json.loads(record_file.read_text())
        if current.get("objective") == path and not value < current["value"]:
            return False
    record = {"run_id": summary["run_id"], "objective": path, "value": value, "path": summary["run_dir"],
              "promotable": promotion_threshold is None or value <= promotion_threshold,
              "promotion_threshold": promotion_threshold}
    record_file.write_text(json.dumps(record, indent=2) + "\n")
    return True


class _Fanout:
    """A text stream that writes to several streams (the console and the run's train.log)."""

    def __init__(self, *streams) -> None:
        self.streams = streams

    def write(self, text: str) -> int:
        for stream in self.streams:
            stream.write(text)
        return len(text)

    def flush(self) -> None:
        for stream in self.streams:
            stream.flush()


def _trainer_summary(result: dict) -> dict:
    train = {key: result.get(key) for key in _TRAIN_KEYS}
    routing = result.get("last_routing") or {}
    train["overflow_fraction"] = (result.get("last_log") or {}).get("overflow_fraction")
    train["routing_imbalance"] = routing.get("imbalance")
    train["active_expert_fraction"] = routing.get("active_fraction")
    train["controller_changes"] = len(result.get("controller_history", []))
    return train


def run_experiment(config: dict, runs_dir: Path = DEFAULT_RUNS_DIR, name: Optional[str] = None,
                   run_id: Optional[str] = None) -> dict:
    """Train one bundle as a tracked run and return its summary. A run that raises is recorded as failed (with
    error.txt), not re-raised; option names the trainer does not know fail before any folder is created."""
    from ..training import trainer

    runs_dir = Path(runs_dir)
    name = name or config.get("name", "experiment")
    options = {k: v for k, v in dict(config.get("train", {})).items() if k not in _LOCATIONS}
    trainer.default_args(**options)  # validates the option names
    fingerprint = hashlib.sha256(json.dumps(options, sort_keys=True, default=str).encode()).hexdigest()[:6]
    run_id = run_id or "-".join((time.strftime("%Y%m%d-%H%M%S"), slug(name), fingerprint))
    folder = runs_dir / run_id
    folder.mkdir(parents=True, exist_ok=False)
    recorded = {"run_id": run_id, "name": name, "description": config.get("description"),
                "tags": config.get("tags", []), "train": options, "benchmark": config.get("benchmark", {}),
                "objective": config.get("objective"), "created": time.strftime("%Y-%m-%dT%H:%M:%S"),
                "git_revision": git_revision(), "argv": sys.argv}
    (folder / "config.json").write_text(json.dumps(recorded, indent=2, default=str) + "\n")
    steps = options.get("steps", trainer.default_args().steps)
    args = trainer.default_args(**{"diagnostics_interval": max(1, steps // 20), **options},
                                output=folder / "model", checkpoint_dir=folder / "checkpoints",
                                metrics_file=folder / "metrics.jsonl", diagnostics_dir=folder / "diagnostics",
                                resume=False)
    summary: dict = {"run_id": run_id, "name": name, "run_dir": str(folder), "tags": recorded["tags"]}
    started = time.perf_counter()
    with (folder / "train.log").open("w") as log, contextlib.redirect_stdout(_Fanout(sys.stdout, log)):
        try:
            summary["train"] = _trainer_summary(trainer.run_training(args))
            summary["status"] = "completed"
            if config.get("benchmark") is not None:
                summary["benchmark"] = run_final_benchmark(folder, args, config.get("benchmark") or {})
        except Exception as error:  # noqa: BLE001 - recorded in the run, the caller carries on
            summary.update(status="failed", error=f"{type(error).__name__}: {error}")
            (folder / "error.txt").write_text(traceback.format_exc())
    summary["seconds"] = time.perf_counter() - started
    if summary["status"] == "completed":
        summary["is_best"] = update_best(runs_dir, summary, config.get("objective"), config.get("promotion_threshold"))
    (folder / "summary.json").write_text(json.dumps(summary, indent=2, default=str) + "\n")
    (folder / "report.md").write_text(render_run_report(recorded, summary))
    return summary


def run_final_benchmark(run_dir: Path, args, options: dict) -> dict:
    """Benchmark the run's model on ``options['data']`` (default: the first training file) and keep the headline
    figures; the full report is written beside the run as benchmark.json and benchmark.md."""
    from .benchmark import build_parser, render_markdown, run_benchmark

    data = options.get("data") or (args.data[0] if args.data else None)
    argv = ["--checkpoint", str(run_dir / "model"), "--data", str(data),
            "--examples", str(options.get("examples", 500)),
            "--batch-size", str(options.get("batch_size", args.batch_size)), "--device", args.device,
            "--training-metrics", str(run_dir / "metrics.jsonl")]
    if options.get("no_routing_stats"):
        argv.append("--no-routing-stats")
    report = run_benchmark(build_parser().parse_args(argv))
    (run_dir / "benchmark.json").write_text(json.dumps(report, indent=2) + "\n")
    (run_dir / "benchmark.md").write_text(render_markdown(report))
    kept = {key: report[key] for key in _BENCH_KEYS}
    if "routing" in report:
        kept["dead_experts"] = report["routing"]["dead_experts_total"]
        kept["routing_entropy"] = report["routing"]["entropy_mean"]
    return kept


def _markdown_table(header: list, rows: list) -> list[str]:
    return (["| " + " | ".join(map(str, header)) + " |", "|" + "---|" * len(header)]
            + ["| " + " | ".join(map(str, row)) + " |" for row in rows])


def render_run_report(config: dict, summary: dict) -> str:
    parts = [f"# {summary['name']} ({summary['run_id']})", "", f"- status: **{summary['status']}**",
             f"- wall time: {summary.get('seconds', 0):.1f}s", f"- git revision: {config.get('git_revision')}", ""]
    if config.get("description"):
        parts += [config["description"], ""]
    parts += ["## Configuration", "", *_markdown_table(["option", "value"], list(config["train"].items())), ""]
    if summary["status"] == "failed":
        parts += ["## Failure", "", f"`{summary['error']}` (traceback in error.txt)", ""]
        return "\n".join(parts)
    for section in ("train", "benchmark"):
        if summary.get(section):
            parts += [f"## {section.capitalize()} results", "",
                      *_markdown_table(["metric", "value"], list(summary[section].items())), ""]
    return "\n".join(parts)


# ---- comparison -----------------------------------------------------------------------------------------------------
def load_summaries(paths: list[Path]) -> list[dict]:
    """Summaries of the given run folders (or summary.json files), each with its ``config`` attached."""
    summaries = []
    for path in map(Path, paths):
        file = path / "summary.json" if path.is_dir() else path
        if not file.exists():
            continue
        summary = json.loads(file.read_text())
        config_file = file.with_name("config.json")
        summary["config"] = json.loads(config_file.read_text()) if config_file.exists() else {}
        summaries.append(summary)
    return summaries


def _fmt(value) -> str:
    if value is None:
        return "-"
    return f"{value:.4g}" if isinstance(value, float) else str(value)


def compare_runs(summaries: list[dict], metric: str = "benchmark.loss") -> str:
    """Markdown table of the completed runs, best (lowest ``metric``) first, with a column for every training
    option whose value differs between them; failed runs are listed underneath."""
    completed = [s for s in summaries if s.get("status") == "completed"]
    completed.sort(key=lambda s: (dig(s, metric) is None, dig(s, metric) or 0))
    options = [s["config"].get("train", {}) for s in completed]
    varying = sorted(key for key in {k for o in options for k in o}
                     if len({json.dumps(o.get(key), default=str) for o in options}) > 1)
    columns = [metric] + [c for c in _TABLE_COLUMNS if c != metric]
    rows = [[s["run_id"], *(_fmt(dig(s, c)) for c in columns), *(_fmt(o.get(k)) for k in varying)]
            for s, o in zip(completed, options)]
    lines = _markdown_table(["run", *columns, *varying], rows)
    failed = [s for s in summaries if s.get("status") == "failed"]
    if failed:
        lines += ["", "Failed runs: " + ", ".join(f"{s['run_id']} ({s.get('error')})" for s in failed)]
    return "\n".join(lines)


def parse_objectives(spec) -> list[tuple[str, str]]:
    """``["benchmark.loss:min", "train.tokens_per_second:max"]`` -> [(path, direction)]; a bare path is minimised.
    Needs at least two objectives."""
    parsed = []
    for item in ([spec] if isinstance(spec, str) else list(spec)):
        path, _, direction = item.partition(":")
        direction = direction or "min"
        if direction not in ("min", "max"):
            raise ValueError(f"objective '{item}': direction must be 'min' or 'max'")
        parsed.append((path.strip(), direction))
    if len(parsed) < 2:
        raise ValueError("a Pareto comparison needs at least two objectives")
    return parsed


def _costs(summary: dict, objectives) -> Optional[tuple]:
    """Objective values turned into costs (lower is better for all); None when one is missing."""
    values = [dig(summary, path) for path, _ in objectives]
    if any(v is None for v in values):
        return None
    return tuple(v if direction == "min" else -v for v, (_, direction) in zip(values, objectives))


def dominates(a: dict, b: dict, objectives: list[tuple[str, str]]) -> bool:
    """``a`` is no worse than ``b`` on every objective and better on at least one."""
    ca, cb = _costs(a, objectives), _costs(b, objectives)
    if ca is None or cb is None:
        return False
    return all(x <= y for x, y in zip(ca, cb)) and ca != cb


def pareto_front(summaries: list[dict], objectives) -> list[dict]:
    """Completed runs that carry every objective and that no other such run dominates."""
    if objectives and isinstance(objectives[0], str):
        objectives = parse_objectives(objectives)
    candidates = [s for s in summaries if s.get("status") == "completed" and _costs(s, objectives) is not None]
    return [s for s in candidates if not any(dominates(other, s, objectives) for other in candidates if other is not s)]


def compare_pareto(summaries: list[dict], objectives) -> str:
    parsed = parse_objectives(objectives) if objectives and isinstance(objectives[0], str) else objectives
    completed = [s for s in summaries if s.get("status") == "completed"]
    front = {id(s) for s in pareto_front(completed, parsed)}
    ordered = [s for s in completed if id(s) in front] + [s for s in completed if id(s) not in front]
    rows = [[s["run_id"], *(_fmt(dig(s, p)) for p, _ in parsed), "yes" if id(s) in front else ""] for s in ordered]
    return "\n".join(_markdown_table(["run", *(f"{p} ({d})" for p, d in parsed), "pareto-optimal"], rows))


def loss_curves_svg(summaries: list[dict]) -> str:
    """One line per run of its logged training loss (a step a run did not log repeats its last value)."""
    curves = {}
    for s in summaries:
        metrics = Path(s["run_dir"]) / "metrics.jsonl"
        if metrics.exists():
            rows = (json.loads(line) for line in metrics.read_text().splitlines() if line.strip())
            points = [(row["step"], row["loss"]) for row in rows if "loss" in row]
            if points:
                curves[s["run_id"]] = points
    if not curves:
        return ""
    steps = sorted({step for points in curves.values() for step, _ in points})
    lines = {}
    for run, points in curves.items():
        by_step, last, values = dict(points), points[-1][1], []
        for step in steps:
            values.append(by_step.get(step, last))
        lines[run] = values
    return line_chart_svg(steps, lines, "Training loss")


# ---- command line ----------------------------------------------------------------------------------------------------
def _cmd_run(args) -> None:
    summary = run_experiment(load_config(args.config), args.runs_dir, args.name)
    print(f"\n{summary['run_id']}: {summary['status']} in {summary['seconds']:.1f}s -> {summary['run_dir']}")
    if summary["status"] == "failed":
        sys.exit(f"run failed: {summary['error']}")


def _cmd_list(args) -> None:
    runs = sorted(p for p in args.runs_dir.iterdir() if p.is_dir()) if args.runs_dir.exists() else []
    print(compare_runs(load_summaries(runs)))
    best = args.runs_dir / "best.json"
    if best.exists():
        print("\nbest:", json.loads(best.read_text()))


def _cmd_compare(args) -> None:
    summaries = load_summaries(args.runs)
    table = compare_pareto(summaries, args.objectives) if args.objectives else compare_runs(summaries, args.metric)
    print(table)
    if args.markdown:
        args.markdown.write_text(table + "\n")
    if args.charts_dir:
        args.charts_dir.mkdir(parents=True, exist_ok=True)
        (args.charts_dir / "loss_curves.svg").write_text(loss_curves_svg(summaries))
        values = {s["run_id"]: dig(s, args.metric) for s in summaries}
        numeric = {run: v for run, v in values.items() if isinstance(v, (int, float))}
        (args.charts_dir / "metric_bars.svg").write_text(bar_chart_svg(numeric, args.metric))


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
    cmp.add_argument("--objectives", nargs="+", help="two or more dotted.path:min|max entries (Pareto table)")
    cmp.add_argument("--markdown", type=Path)
    cmp.add_argument("--charts-dir", type=Path, help="folder for the loss-curve and metric-bar SVG charts")
    from .common import describe_options

    describe_options(p, {"runs_dir": "folder of tracked runs"})
    args = p.parse_args(argv)
    {"run": _cmd_run, "list": _cmd_list, "compare": _cmd_compare}[args.command](args)


if __name__ == "__main__":
    main()
