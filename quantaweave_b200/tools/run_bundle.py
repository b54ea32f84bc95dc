"""Archive a finished run into its own folder named by the epoch second it finished.

Layout parity with the reference ``src/run_bundle.py`` (module docstring :1-22, ``create_run_bundle`` :304-383,
``reproduce_command`` :166-190, ``archive_data`` :102-139, ``resolve_archive_dir`` :56-61)::

    <root>/<epoch>[-n]/
        README.md  summary.json  config.json  reproduce.sh  environment.json  samples.txt
        model/                 copy of the run's output directory (weights, config, tokenizer)
        data/manifest.json     sources with sha256 (partial over 512 MB), rows used; the files when small enough
        benchmarks/            train-slice and held-out reports (JSON + Markdown) and the held-out sample
        training/              metrics.jsonl and routing diagnostics

Archiving never fails a run: every step that raises is recorded under ``warnings`` (and an ``*.error.txt``).
Held-out rows are the rows after the first ``examples`` of each file, which training never read.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import platform
import shlex
import shutil
import subprocess
import sys
import time
import traceback
from pathlib import Path
from typing import Iterable, Optional, Sequence

import torch

DEFAULT_PROMPTS = ("Once upon a time", "The ")
PARTIAL_HASH_BYTES = 16 << 20
FULL_HASH_LIMIT = 512 << 20


def add_archive_arguments(parser: argparse.ArgumentParser) -> None:
    g = parser.add_argument_group("run archive")
    g.add_argument("--archive-dir", type=Path,
                   help="keep the finished run (weights, data manifest, benchmarks, reproduce script) in "
                        "ARCHIVE_DIR/<epoch seconds>/; from the command line this defaults to artifacts/runs")
    g.add_argument("--no-archive", action="store_true", help="skip the run archive")
    g.add_argument("--archive-data-limit-mb", type=float, default=200.0,
                   help="largest data size copied into the archive, in MB (0: record hashes only)")
    g.add_argument("--archive-benchmark-examples", type=int, default=500, help="rows each archived benchmark reads")
    g.add_argument("--data-card", type=Path,
                   help="JSON file about the data (origin, licence, provenance) copied into the archive's manifest")


def resolve_archive_dir(args: argparse.Namespace, default: Path = Path("artifacts/runs")) -> None:
    """Command-line entry points archive by default, unless ``--no-archive``."""
    if getattr(args, "no_archive", False):
        args.archive_dir = None
    elif getattr(args, "archive_dir", None) is None:
        args.archive_dir = default


def epoch_folder(root: Path, now: Optional[float] = None) -> Path:
    """Create ``root/<epoch>``, or ``<epoch>-1``, ``-2``... when that second is taken (never overwrite)."""
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    epoch = int(time.time() if now is None else now)
    for n in range(10_000):
        candidate = root / (str(epoch) if n == 0 else f"{epoch}-{n}")
        try:
            candidate.mkdir()
            return candidate
        except FileExistsError:
            continue
    raise RuntimeError(f"no free archive folder under {root}")


def file_digest(path: Path) -> tuple[str, str]:
    """(sha256 hex, "full" | "partial"): files over 512 MB hash their first and last 16 MB plus their size."""
    path = Path(path)
    size = path.stat().st_size
    h = hashlib.sha256()
    with path.open("rb") as fh:
        if size <= FULL_HASH_LIMIT:
            while block := fh.read(1 << 20):
                h.update(block)
            return h.hexdigest(), "full"
        h.update(fh.read(PARTIAL_HASH_BYTES))
        fh.seek(max(0, size - PARTIAL_HASH_BYTES))
        h.update(fh.read(PARTIAL_HASH_BYTES))
    h.update(str(size).encode())
    return h.hexdigest(), "partial"


def count_rows(path: Path) -> Optional[int]:
    path = Path(path)
    if path.stat().st_size > FULL_HASH_LIMIT:
        return None
    with path.open("rb") as fh:
        return sum(1 for _ in fh)


def archive_data(data_paths: Sequence[Path], bundle: Path, limit_mb: float, rows_used: Optional[int],
                 data_card: Optional[Path] = None) -> dict:
    """Write ``data/manifest.json`` (always) and copy the files when their total size is within ``limit_mb``."""
    files = [Path(p) for p in data_paths if Path(p).is_file()]
    total = sum(p.stat().st_size for p in files)
    copy = bool(files) and limit_mb > 0 and total <= limit_mb * (1 << 20)
    target = Path(bundle) / "data"
    target.mkdir(exist_ok=True)
    unique = len({p.name for p in files}) == len(files)
    entries = []
    for i, path in enumerate(files):
        digest, coverage = file_digest(path)
        entry = {"path": str(path.resolve()), "bytes": path.stat().st_size, "sha256": digest,
                 "hash_coverage": coverage, "rows": count_rows(path), "rows_used_for_training": rows_used}
        if copy:
            name = path.name if unique else f"{i}-{path.name}"
            shutil.copy2(path, target / name)
            entry["copied_as"] = f"data/{name}"
        entries.append(entry)
    if copy:
        note = None
    elif not files:
        note = "data was not copied: no data files were found"
    else:
        note = f"data was not copied: {total / (1 << 20):.0f} MB exceeds the {limit_mb:g} MB limit"
    if note:
        note += "; the manifest records the sources and hashes so they can be matched to this run"
    manifest = {"copied": copy, "total_bytes": total, "limit_mb": limit_mb, "files": entries, "note": note}
    if data_card is not None:
        try:
            manifest["data_card"] = json.loads(Path(data_card).read_text())
        except Exception as error:  # noqa: BLE001 - recorded, never fatal
            manifest["data_card_error"] = f"could not read --data-card {data_card}: {type(error).__name__}: {error}"
    (target / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def write_held_out_sample(data_paths: Sequence[Path], skip_rows: Optional[int], count: int,
                          destination: Path) -> Optional[dict]:
    """Rows after the first ``skip_rows`` of each file (never trained on), spread evenly over the files."""
    files = [Path(p) for p in data_paths if Path(p).is_file()]
    if not files or skip_rows is None:
        return None
    per_file = max(1, count // len(files))
    rows: list[str] = []
    for path in files:
        taken = 0
        with path.open(encoding="utf-8") as fh:
            for number, line in enumerate(fh):
                if number < skip_rows or not line.strip():
                    continue
                rows.append(line.rstrip("\n"))
                taken += 1
                if taken >= per_file:
                    break
    if not rows:
        return None
    Path(destination).write_text("\n".join(rows) + "\n")
    return {"rows": len(rows), "skipped_rows_per_file": skip_rows, "file": Path(destination).name}


def reproduce_command(module: str, parser: argparse.ArgumentParser, args: argparse.Namespace,
                      skip: Sequence[str] = (), explicit: bool = False) -> str:
    """The command line that recreates ``args``: only non-default options, or every option when ``explicit`` (so
    the command keeps its meaning if a default changes later)."""
    defaults = None if explicit or any(a.required for a in parser._actions) else parser.parse_args([])
    parts = [f"python -m {module}"]
    for action in parser._actions:
        if not action.option_strings or action.dest in ("help", *skip):
            continue
        value = getattr(args, action.dest, None)
        if value is None or (defaults is not None and value == getattr(defaults, action.dest, None)):
            continue
        flag = action.option_strings[-1]
        if isinstance(action, argparse.BooleanOptionalAction):
            parts.append(action.option_strings[0] if value else action.option_strings[1])
        elif action.nargs == 0:
            if value != action.default:
                parts.append(flag)
        elif isinstance(value, (list, tuple)):
            parts.append(flag + " " + " ".join(shlex.quote(str(v)) for v in value))
        else:
            parts.append(f"{flag} {shlex.quote(str(value))}")
    return " \\\n  ".join(parts)


def environment_info(device_arg: str) -> dict:
    info = {"python": sys.version.split()[0], "torch": torch.__version__, "platform": platform.platform(),
            "argv": sys.argv}
    try:
        rev = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True, check=True,
                             cwd=Path(__file__).parent).stdout.strip()
        info["git_revision"] = rev or None
    except (OSError, subprocess.CalledProcessError):
        info["git_revision"] = None
    try:
        from dataclasses import asdict

        from ..utils.hardware import detect

        info["device"] = asdict(detect(device_arg if device_arg in {"auto", "cuda", "xpu", "cpu", "rocm"} else "auto"))
    except Exception as error:  # noqa: BLE001
        info["device"] = f"unavailable: {error}"
    return info


def write_samples(model_dir: Path, destination: Path, prompts: Iterable[str], device_arg: str, tokens: int = 200,
                  temperature: float = 0.8) -> None:
    from ..data.pipeline import load_tokenizer
    from ..training.trainer import select_device
    from .common import load_model
    from .generate import sample_text

    device = select_device(device_arg)
    model = load_model(model_dir, device)
    tokenizer = load_tokenizer(model_dir)
    torch.manual_seed(0)
    blocks = [f"temperature {temperature}, up to {tokens} tokens; sampling seed 0\n"]
    for prompt in prompts:
        blocks.append(f"=== prompt: {prompt!r}\n{sample_text(model, tokenizer, prompt, tokens, temperature, device)}\n")
    Path(destination).write_text("\n".join(blocks))


def run_benchmarks(model_dir: Path, bundle: Path, data_paths: Sequence[Path], held_out: Optional[dict],
                   metrics_file: Optional[Path], examples: int, device: str, precision: str,
                   warnings: list[str]) -> dict:
    from .benchmark import build_parser, render_markdown, run_benchmark

    out = Path(bundle) / "benchmarks"
    jobs = []
    if data_paths and Path(data_paths[0]).is_file():
        jobs.append(("train-slice", Path(data_paths[0]), "rows the model trained on"))
    if held_out is not None:
        jobs.append(("held-out", out / held_out["file"], "rows the model never saw"))
    else:
        warnings.append("no unseen rows were available for a held-out benchmark (the training run read every row)")
    results: dict = {}
    keys = ("loss", "perplexity", "tokens_per_second", "tokens", "dropped_route_fraction", "overflow_route_fraction",
            "expert_utilization_min", "expert_utilization_max")
    for name, data, what in jobs:
        try:
            argv = ["--checkpoint", str(model_dir), "--data", str(data), "--examples", str(examples),
                    "--batch-size", "16", "--device", device, "--precision", precision]
            if name == "train-slice" and metrics_file is not None and Path(metrics_file).exists():
                argv += ["--training-metrics", str(metrics_file)]
            report = run_benchmark(build_parser().parse_args(argv))
            (out / f"{name}.json").write_text(json.dumps(report, indent=2) + "\n")
            (out / f"{name}.md").write_text(f"_{what}_\n\n" + render_markdown(report))
            results[name] = {k: report[k] for k in keys}
            results[name]["what"] = what
            if "routing" in report:
                results[name]["dead_experts"] = report["routing"]["dead_experts_total"]
        except Exception as error:  # noqa: BLE001
            warnings.append(f"benchmark '{name}' failed: {type(error).__name__}: {error}")
            (out / f"{name}.error.txt").write_text(traceback.format_exc())
    if "train-slice" in results and "held-out" in results:
        results["generalisation_gap"] = results["held-out"]["loss"] - results["train-slice"]["loss"]
    return results


def render_readme(bundle: Path, kind: str, epoch: int, summary: dict, benchmarks: dict, manifest: Optional[dict],
                  reproduce: Optional[str], warnings: list[str], model_names: Sequence[str]) -> str:
    when = time.strftime("%Y-%m-%d %H:%M:%S UTC", time.gmtime(epoch))
    lines = [f"# {kind} run {Path(bundle).name}", "",
             f"Archived {when} (epoch {epoch}). The run itself took {summary.get('duration_seconds', 0):.0f} s.", ""]
    rows = []
    train = summary.get("train", {})
    for key, label in (("final_loss", "final training loss"), ("best_loss", "best training loss"), ("steps", "steps"),
                       ("tokens_per_second", "training tokens/s"),
                       ("active_parameter_ratio", "active / total parameters")):
        value = train.get(key)
        if value is not None:
            rows.append(f"| {label} | {value:.4g} |" if isinstance(value, float) else f"| {label} | {value} |")
    for name in ("train-slice", "held-out"):
        if name in benchmarks:
            b = benchmarks[name]
            rows.append(f"| {name} loss (perplexity) | {b['loss']:.4f} ({b['perplexity']:.2f}) — {b['what']} |")
    if "generalisation_gap" in benchmarks:
        rows.append(f"| generalisation gap (held-out − train) | {benchmarks['generalisation_gap']:+.4f} |")
    if rows:
        lines += ["| result | value |", "|---|---|", *rows, ""]
    if warnings:
        lines += ["## Warnings", "", *[f"- {w}" for w in warnings], ""]
    copied = manifest and manifest["copied"]
    lines += ["## Contents", "", *[f"- `{n}/` — weights, config, tokenizer" for n in model_names],
              "- `data/` — the training data" + (" (copied)" if copied else
                                                 " (not copied; `manifest.json` records the sources and hashes)"),
              "- `benchmarks/` — `train-slice` (rows it trained on) and `held-out` (rows it never saw), JSON and Markdown",
              "- `training/` — `metrics.jsonl` and routing diagnostics (`diagnostics/index.html`)",
              "- `config.json`, `reproduce.sh`, `environment.json`, `summary.json`, `samples.txt`", ""]
    if kind == "train":
        lines += ["## Use this model", "", "```bash",
                  f"python -m quantaweave_b200.tools.generate --checkpoint {bundle}/model --prompt \"Once upon a time\"",
                  f"python -m quantaweave_b200.tools.benchmark --checkpoint {bundle}/model --data <jsonl> "
                  "--output /tmp/bench.json",
                  f"python -m quantaweave_b200.tools.export --checkpoint {bundle}/model --output {bundle}/export "
                  "--quantize 8",
                  f"python -m quantaweave_b200.tools.finetune --checkpoint {bundle}/model --data <jsonl> "
                  f"--output {bundle}/qlora",
                  "```", ""]
    if reproduce:
        lines += ["## Reproduce", "", "```bash", reproduce, "```", ""]
    return "\n".join(lines)


def create_run_bundle(root: Path, *, kind: str, model_dirs: dict[str, Path], benchmark_model: Optional[Path],
                      data_paths: Sequence[Path], options: dict, summary: dict, started: float,
                      reproduce: Optional[str] = None, reproduce_full: Optional[str] = None,
                      finished: Optional[float] = None, metrics_file: Optional[Path] = None,
                      diagnostics_dir: Optional[Path] = None, skip_rows: Optional[int] = None,
                      benchmark_examples: int = 500, device: str = "auto", precision: str = "auto",
                      data_limit_mb: float = 200.0, sample_prompts: Optional[Sequence[str]] = None,
                      now: Optional[float] = None, data_card: Optional[Path] = None) -> Path:
    """Write the archive folder and return its path. ``model_dirs`` maps folder name -> directory to copy."""
    warnings: list[str] = []
    bundle = epoch_folder(Path(root), now)
    epoch = int(bundle.name.split("-")[0])
    for sub in ("benchmarks", "training"):
        (bundle / sub).mkdir(exist_ok=True)

    def attempt(label: str, action):
        try:
            return action()
        except Exception as error:  # noqa: BLE001 - archiving never fails a run
            warnings.append(f"{label} failed: {type(error).__name__}: {error}")
            (bundle / f"{label.replace(' ', '_')}.error.txt").write_text(traceback.format_exc())
            return None

    for name, source in model_dirs.items():
        attempt(f"copy {name}", lambda n=name, s=source: shutil.copytree(
            s, bundle / n, ignore=shutil.ignore_patterns("shards", ".*.tmp", ".*.previous")))
    manifest = attempt("archive data", lambda: archive_data(data_paths, bundle, data_limit_mb, skip_rows, data_card))
    if manifest and not manifest["copied"] and manifest["note"]:
        warnings.append(manifest["note"])
    held_out = attempt("held-out sample", lambda: write_held_out_sample(
        data_paths, skip_rows, benchmark_examples, bundle / "benchmarks" / "heldout_sample.jsonl"))
    benchmarks: dict = {}
    if benchmark_model is not None:
        benchmarks = attempt("benchmarks", lambda: run_benchmarks(
            Path(benchmark_model), bundle, data_paths, held_out, metrics_file, benchmark_examples, device, precision,
            warnings)) or {}
    else:
        warnings.append("no benchmark was run for this output (it is not a standalone checkpoint)")
    if metrics_file is not None and Path(metrics_file).exists():
        shutil.copy2(metrics_file, bundle / "training" / "metrics.jsonl")
    if diagnostics_dir is not None and Path(diagnostics_dir).exists():
        shutil.copytree(diagnostics_dir, bundle / "training" / "diagnostics", dirs_exist_ok=True)
    if benchmark_model is not None and (Path(benchmark_model) / "model.pt").exists():
        prompts = list(sample_prompts or DEFAULT_PROMPTS)
        attempt("samples", lambda: write_samples(Path(benchmark_model), bundle / "samples.txt", prompts, device))

    finished = time.time() if finished is None else finished
    summary = {**summary, "duration_seconds": finished - started}
    (bundle / "config.json").write_text(json.dumps(options, indent=2, default=str) + "\n")
    if reproduce or reproduce_full:
        (bundle / "reproduce.sh").write_text(
            "#!/usr/bin/env bash\n# every option is listed, so this stays correct if defaults change\n"
            "set -euo pipefail\n" + (reproduce_full or reproduce) + "\n")
    (bundle / "environment.json").write_text(json.dumps(environment_info(device), indent=2, default=str) + "\n")
    record = {"kind": kind, "epoch": epoch, "folder": bundle.name, "started_epoch": int(started),
              "training_finished_epoch": int(finished), "archived_epoch": epoch,
              "duration_seconds": summary["duration_seconds"], "results": summary, "benchmarks": benchmarks,
              "data": {"copied": bool(manifest and manifest["copied"]),
                       "total_bytes": manifest["total_bytes"] if manifest else None},
              "held_out": held_out, "warnings": warnings}
    (bundle / "summary.json").write_text(json.dumps(record, indent=2, default=str) + "\n")
    readme = render_readme(bundle, kind, epoch, {"duration_seconds": summary["duration_seconds"], "train": summary},
                           benchmarks, manifest, reproduce, warnings, list(model_dirs))
    (bundle / "README.md").write_text(readme)
    return bundle
