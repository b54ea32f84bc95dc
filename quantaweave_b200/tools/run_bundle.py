"""Archive a finished run in a folder of its own, named by the epoch second it was archived.

The folder layout, the file names and the function names follow the reference's ``src/run_bundle.py``::

    <root>/<epoch>[-n]/
        README.md  summary.json  config.json  reproduce.sh  environment.json  samples.txt
        model/                 copy of the run's output directory (weights, config, tokenizer)
        data/manifest.json     every data file with its sha256 (partial for very large files) and rows used;
                               the files themselves when they are small enough
        benchmarks/            reports on rows the model trained on and on rows it never saw, and that sample
        training/              metrics.jsonl and routing diagnostics

Archiving never fails the run it archives: ``_Archive.step`` turns an exception into a warning (listed in
summary.json and the README) plus a ``<step>.error.txt`` with the traceback. The unseen rows are the rows after the
first ``examples`` of each data file, which training never read.
"""

from __future__ import annotations

import argparse
import contextlib
import hashlib
import itertools
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
PARTIAL_HASH_BYTES = 16 << 20  # head and tail hashed for files over FULL_HASH_LIMIT
FULL_HASH_LIMIT = 512 << 20
_MB = 1 << 20


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
    """Command-line runs are archived unless ``--no-archive``; library calls only when asked."""
    if getattr(args, "no_archive", False):
        args.archive_dir = None
    elif getattr(args, "archive_dir", None) is None:
        args.archive_dir = default


def epoch_folder(root: Path, now: Optional[float] = None) -> Path:
    """Create and return ``root/<epoch>``; when that name is taken, ``<epoch>-1``, ``<epoch>-2``, ... (never reuse)."""
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    stamp = str(int(time.time() if now is None else now))
    for name in itertools.chain([stamp], (f"{stamp}-{n}" for n in range(1, 10_000))):
        try:
            (root / name).mkdir()
        except FileExistsError:
            continue
        return root / name
    raise RuntimeError(f"no free archive folder under {root}")


def file_digest(path: Path) -> tuple[str, str]:
    """(sha256, coverage): the whole file up to FULL_HASH_LIMIT bytes ("full"); above it, the first and last
    PARTIAL_HASH_BYTES and the size ("partial"), so multi-GB corpora are recorded without reading them through."""
    path = Path(path)
    size = path.stat().st_size
    digest = hashlib.sha256()
    with path.open("rb") as handle:
        if size <= FULL_HASH_LIMIT:
            for block in iter(lambda: handle.read(_MB), b""):
                digest.update(block)
            return digest.hexdigest(), "full"
        digest.update(handle.read(PARTIAL_HASH_BYTES))
        handle.seek(max(0, size - PARTIAL_HASH_BYTES))
        digest.update(handle.read(PARTIAL_HASH_BYTES))
    digest.update(str(size).encode())
    return digest.hexdigest(), "partial"


def count_rows(path: Path) -> Optional[int]:
    """Lines in the file (a last line without a newline counts), or None when it is over FULL_HASH_LIMIT."""
    path = Path(path)
    size = path.stat().st_size
    if size > FULL_HASH_LIMIT:
        return None
    newlines, last = 0, b"\n"
    with path.open("rb") as handle:
        for block in iter(lambda: handle.read(_MB), b""):
            newlines += block.count(b"\n")
            last = block[-1:]
    return newlines + (1 if size and last != b"\n" else 0)


def archive_data(data_paths: Sequence[Path], bundle: Path, limit_mb: float, rows_used: Optional[int],
                 data_card: Optional[Path] = None) -> dict:
    """Write ``data/manifest.json`` and, when all the files together fit ``limit_mb``, copies of them."""
    sources = [Path(p) for p in data_paths if Path(p).is_file()]
    total = sum(p.stat().st_size for p in sources)
    copying = bool(sources) and limit_mb > 0 and total <= limit_mb * _MB
    folder = Path(bundle) / "data"
    folder.mkdir(exist_ok=True)
    clash = len({p.name for p in sources}) < len(sources)  # same file name from different folders
    entries = []
    for index, source in enumerate(sources):
        digest, coverage = file_digest(source)
        entry = {"path": str(source.resolve()), "bytes": source.stat().st_size, "sha256": digest,
                 "hash_coverage": coverage, "rows": count_rows(source), "rows_used_for_training": rows_used}
        if copying:
            name = f"{index}-{source.name}" if clash else source.name
            shutil.copy2(source, folder / name)
            entry["copied_as"] = f"data/{name}"
        entries.append(entry)
    if copying:
        note = None
    else:
        reason = ("no data files were found" if not sources
                  else f"{total / _MB:.0f} MB exceeds the {limit_mb:g} MB limit")
        note = (f"data was not copied: {reason}; the manifest records the sources and hashes so they can be "
                "matched to this run")
    manifest = {"copied": copying, "total_bytes": total, "limit_mb": limit_mb, "files": entries, "note": note}
    if data_card is not None:
        try:
            manifest["data_card"] = json.loads(Path(data_card).read_text())
        except Exception as error:  # noqa: BLE001 - an unreadable card is recorded, never fatal
            manifest["data_card_error"] = f"could not read --data-card {data_card}: {type(error).__name__}: {error}"
    (folder / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def write_held_out_sample(data_paths: Sequence[Path], skip_rows: Optional[int], count: int,
                          destination: Path) -> Optional[dict]:
    """Up to ``count`` non-empty rows from past the first ``skip_rows`` of each file, split evenly over the files;
    None when there are no such rows."""
    sources = [Path(p) for p in data_paths if Path(p).is_file()]
    if not sources or skip_rows is None:
        return None
    quota = max(1, count // len(sources))
    picked: list[str] = []
    for source in sources:
        with source.open(encoding="utf-8") as handle:
            unseen = (line.rstrip("\n") for line in itertools.islice(handle, skip_rows, None) if line.strip())
            picked.extend(itertools.islice(unseen, quota))
    if not picked:
        return None
    Path(destination).write_text("\n".join(picked) + "\n")
    return {"rows": len(picked), "skipped_rows_per_file": skip_rows, "file": Path(destination).name}


def _option_tokens(action: argparse.Action, value) -> list[str]:
    """The command-line words that set ``action`` to ``value``."""
    if isinstance(action, argparse.BooleanOptionalAction):
        return [action.option_strings[0] if value else action.option_strings[1]]
    flag = action.option_strings[-1]
    if action.nargs == 0:  # store_true / store_false
        return [flag] if value != action.default else []
    if isinstance(value, (list, tuple)):
        return [flag + " " + " ".join(shlex.quote(str(v)) for v in value)]
    return [f"{flag} {shlex.quote(str(value))}"]


def reproduce_command(module: str, parser: argparse.ArgumentParser, args: argparse.Namespace,
                      skip: Sequence[str] = (), explicit: bool = False) -> str:
    """The command that recreates ``args``: the options that differ from their defaults, or every option when
    ``explicit`` (so the command keeps its meaning even if a default changes later)."""
    reference = None if explicit or any(a.required for a in parser._actions) else parser.parse_args([])
    words = [f"python -m {module}"]
    for action in parser._actions:
        if not action.option_strings or action.dest == "help" or action.dest in skip:
            continue
        value = getattr(args, action.dest, None)
        if value is None or (reference is not None and value == getattr(reference, action.dest, None)):
            continue
        words.extend(_option_tokens(action, value))
    return " \\\n  ".join(words)


def environment_info(device_arg: str) -> dict:
    info = {"python": sys.version.split()[0], "torch": torch.__version__, "platform": platform.platform(),
            "argv": sys.argv, "git_revision": None}
    with contextlib.suppress(OSError, subprocess.CalledProcessError):
        revision = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True,
                                  check=True, cwd=Path(__file__).parent).stdout.strip()
        info["git_revision"] = revision or None
    try:
        from dataclasses import asdict

        from ..utils.hardware import detect

        known = device_arg if device_arg in ("auto", "cuda", "xpu", "cpu", "rocm") else "auto"
        info["device"] = asdict(detect(known))
    except Exception as error:  # noqa: BLE001 - a device that cannot be described does not stop the archive
        info["device"] = f"unavailable: {error}"
    return info


def write_samples(model_dir: Path, destination: Path, prompts: Iterable[str], device_arg: str, tokens: int = 200,
                  temperature: float = 0.8) -> None:
    """A few sampled continuations of the archived model, with the sampling settings on the first line."""
    from ..data.pipeline import load_tokenizer
    from ..training.trainer import select_device
    from .common import load_model
    from .generate import sample_text

    device = select_device(device_arg)
    model, tokenizer = load_model(model_dir, device), load_tokenizer(model_dir)
    torch.manual_seed(0)
    parts = [f"temperature {temperature}, up to {tokens} tokens; sampling seed 0\n"]
    parts += [f"=== prompt: {prompt!r}\n{sample_text(model, tokenizer, prompt, tokens, temperature, device)}\n"
              for prompt in prompts]
    Path(destination).write_text("\n".join(parts))


_BENCHMARK_KEYS = ("loss", "perplexity", "tokens_per_second", "tokens", "dropped_route_fraction",
                   "overflow_route_fraction", "expert_utilization_min", "expert_utilization_max")


def run_benchmarks(model_dir: Path, bundle: Path, data_paths: Sequence[Path], held_out: Optional[dict],
                   metrics_file: Optional[Path], examples: int, device: str, precision: str,
                   warnings: list[str]) -> dict:
    """Benchmark the model on the first data file (rows it trained on) and on the held-out sample (rows it never
    saw); the difference of the two losses is reported as the generalisation gap."""
    from .benchmark import build_parser, render_markdown, run_benchmark

    folder = Path(bundle) / "benchmarks"
    jobs = []
    if data_paths and Path(data_paths[0]).is_file():
        jobs.append(("train-slice", Path(data_paths[0]), "rows the model trained on", True))
    if held_out is None:
        warnings.append("no unseen rows were available for a held-out benchmark (the training run read every row)")
    else:
        jobs.append(("held-out", folder / held_out["file"], "rows the model never saw", False))
    results: dict = {}
    for name, data, meaning, with_training_metrics in jobs:
        argv = ["--checkpoint", str(model_dir), "--data", str(data), "--examples", str(examples), "--batch-size",
                "16", "--device", device, "--precision", precision]
        if with_training_metrics and metrics_file is not None and Path(metrics_file).exists():
            argv += ["--training-metrics", str(metrics_file)]
        try:
            report = run_benchmark(build_parser().parse_args(argv))
        except Exception as error:  # noqa: BLE001 - one failed benchmark is a warning
            warnings.append(f"benchmark '{name}' failed: {type(error).__name__}: {error}")
            (folder / f"{name}.error.txt").write_text(traceback.format_exc())
            continue
        (folder / f"{name}.json").write_text(json.dumps(report, indent=2) + "\n")
        (folder / f"{name}.md").write_text(f"_{meaning}_\n\n" + render_markdown(report))
        results[name] = {key: report[key] for key in _BENCHMARK_KEYS}
        results[name]["what"] = meaning
        if "routing" in report:
            results[name]["dead_experts"] = report["routing"]["dead_experts_total"]
    if {"train-slice", "held-out"} <= results.keys():
        results["generalisation_gap"] = results["held-out"]["loss"] - results["train-slice"]["loss"]
    return results


_README_RESULTS = (("final_loss", "final training loss"), ("best_loss", "best training loss"), ("steps", "steps"),
                   ("tokens_per_second", "training tokens/s"), ("active_parameter_ratio", "active / total parameters"))


def render_readme(bundle: Path, kind: str, epoch: int, summary: dict, benchmarks: dict, manifest: Optional[dict],
                  reproduce: Optional[str], warnings: list[str], model_names: Sequence[str]) -> str:
    archived = time.strftime("%Y-%m-%d %H:%M:%S UTC", time.gmtime(epoch))
    train = summary.get("train", {})
    rows = []
    for key, label in _README_RESULTS:
        if train.get(key) is not None:
            value = train[key]
            rows.append(f"| {label} | {value:.4g} |" if isinstance(value, float) else f"| {label} | {value} |")
    for name in ("train-slice", "held-out"):
        if name in benchmarks:
            b = benchmarks[name]
            rows.append(f"| {name} loss (perplexity) | {b['loss']:.4f} ({b['perplexity']:.2f}) — {b['what']} |")
    if "generalisation_gap" in benchmarks:
        rows.append(f"| generalisation gap (held-out − train) | {benchmarks['generalisation_gap']:+.4f} |")
    copied = bool(manifest and manifest["copied"])
    sections = [[f"# {kind} run {Path(bundle).name}", "",
                 f"Archived {archived} (epoch {epoch}). The run itself took {summary.get('duration_seconds', 0):.0f} s.",
                 ""]]
    if rows:
        sections.append(["| result | value |", "|---|---|", *rows, ""])
    if warnings:
        sections.append(["## Warnings", "", *(f"- {w}" for w in warnings), ""])
    sections.append(["## Contents", "", *(f"- `{n}/` — weights, config, tokenizer" for n in model_names),
                     "- `data/` — the training data" + (" (copied)" if copied else
                                                       " (not copied; `manifest.json` records the sources and hashes)"),
                     "- `benchmarks/` — `train-slice` (rows it trained on) and `held-out` (rows it never saw), JSON "
                     "and Markdown",
                     "- `training/` — `metrics.jsonl` and routing diagnostics (`diagnostics/index.html`)",
                     "- `config.json`, `reproduce.sh`, `environment.json`, `summary.json`, `samples.txt`", ""])
    if kind == "train":
        model = f"{bundle}/model"
        sections.append(["## Use this model", "", "```bash",
                         f"python -m quantaweave_b200.tools.generate --checkpoint {model} --prompt \"Once upon a time\"",
                         f"python -m quantaweave_b200.tools.benchmark --checkpoint {model} --data <jsonl> "
                         "--output /tmp/bench.json",
                         f"python -m quantaweave_b200.tools.export --checkpoint {model} --output {bundle}/export "
                         "--quantize 8",
                         f"python -m quantaweave_b200.tools.finetune --checkpoint {model} --data <jsonl> "
                         f"--output {bundle}/qlora", "```", ""])
    if reproduce:
        sections.append(["## Reproduce", "", "```bash", reproduce, "```", ""])
    return "\n".join(line for section in sections for line in section)


class _Archive:
    """The archive folder being filled; ``step`` runs one part and records its failure instead of raising."""

    def __init__(self, root: Path, now: Optional[float]) -> None:
        self.folder = epoch_folder(Path(root), now)
        self.epoch = int(self.folder.name.split("-")[0])
        self.warnings: list[str] = []
        for sub in ("benchmarks", "training"):
            (self.folder / sub).mkdir(exist_ok=True)

    def step(self, label: str, action):
        try:
            return action()
        except Exception as error:  # noqa: BLE001 - archiving never fails the run
            self.warnings.append(f"{label} failed: {type(error).__name__}: {error}")
            (self.folder / f"{label.replace(' ', '_')}.error.txt").write_text(traceback.format_exc())
            return None

    def write_json(self, name: str, payload) -> None:
        (self.folder / name).write_text(json.dumps(payload, indent=2, default=str) + "\n")


def create_run_bundle(root: Path, *, kind: str, model_dirs: dict[str, Path], benchmark_model: Optional[Path],
                      data_paths: Sequence[Path], options: dict, summary: dict, started: float,
                      reproduce: Optional[str] = None, reproduce_full: Optional[str] = None,
                      finished: Optional[float] = None, metrics_file: Optional[Path] = None,
                      diagnostics_dir: Optional[Path] = None, skip_rows: Optional[int] = None,
                      benchmark_examples: int = 500, device: str = "auto", precision: str = "auto",
                      data_limit_mb: float = 200.0, sample_prompts: Optional[Sequence[str]] = None,
                      now: Optional[float] = None, data_card: Optional[Path] = None) -> Path:
    """Fill a new archive folder and return it; ``model_dirs`` maps a folder name in the archive to the directory
    copied there."""
    archive = _Archive(root, now)
    folder = archive.folder
    for name, source in model_dirs.items():
        archive.step(f"copy {name}", lambda n=name, s=source: shutil.copytree(
            s, folder / n, ignore=shutil.ignore_patterns("shards", ".*.tmp", ".*.previous")))
    manifest = archive.step("archive data",
                            lambda: archive_data(data_paths, folder, data_limit_mb, skip_rows, data_card))
    if manifest and manifest["note"]:
        archive.warnings.append(manifest["note"])
    held_out = archive.step("held-out sample", lambda: write_held_out_sample(
        data_paths, skip_rows, benchmark_examples, folder / "benchmarks" / "heldout_sample.jsonl"))
    benchmarks: dict = {}
    if benchmark_model is None:
        archive.warnings.append("no benchmark was run for this output (it is not a standalone checkpoint)")
    else:
        benchmarks = archive.step("benchmarks", lambda: run_benchmarks(
            Path(benchmark_model), folder, data_paths, held_out, metrics_file, benchmark_examples, device,
            precision, archive.warnings)) or {}
    if metrics_file is not None and Path(metrics_file).exists():
        shutil.copy2(metrics_file, folder / "training" / "metrics.jsonl")
    if diagnostics_dir is not None and Path(diagnostics_dir).exists():
        shutil.copytree(diagnostics_dir, folder / "training" / "diagnostics", dirs_exist_ok=True)
    if benchmark_model is not None and (Path(benchmark_model) / "model.pt").exists():
        prompts = list(sample_prompts or DEFAULT_PROMPTS)
        # looked up through the module at call time, so a replacement installed by the caller is used
        archive.step("samples", lambda: sys.modules[__name__].write_samples(
            Path(benchmark_model), folder / "samples.txt", prompts, device))
    finished = time.time() if finished is None else finished
    results = {**summary, "duration_seconds": finished - started}
    archive.write_json("config.json", options)
    if reproduce or reproduce_full:
        (folder / "reproduce.sh").write_text("#!/usr/bin/env bash\n# every option is spelled out, so a later change "
                                             "of a default does not change this run\nset -euo pipefail\n"
                                             + (reproduce_full or reproduce) + "\n")
    archive.write_json("environment.json", environment_info(device))
    archive.write_json("summary.json", {
        "kind": kind, "epoch": archive.epoch, "folder": folder.name, "started_epoch": int(started),
        "training_finished_epoch": int(finished), "archived_epoch": archive.epoch,
        "duration_seconds": results["duration_seconds"], "results": results, "benchmarks": benchmarks,
        "data": {"copied": bool(manifest and manifest["copied"]),
                 "total_bytes": manifest["total_bytes"] if manifest else None},
        "held_out": held_out, "warnings": archive.warnings})
    (folder / "README.md").write_text(render_readme(
        folder, kind, archive.epoch, {"duration_seconds": results["duration_seconds"], "train": results},
        benchmarks, manifest, reproduce, archive.warnings, list(model_dirs)))
    return folder
