"""Run archives (reference tests: tests/test_run_bundle.py): epoch-second folders that never overwrite, archiving
off in the library unless asked, the caller's options and the temp directory left as they were (also when the run
fails), a reproduce script that recreates the exact weights, archive failures recorded as warnings, large data
recorded by hash instead of copied, the held-out benchmark skipped when every row was trained on, packed-token runs
archived without a benchmark, and one archive per multi-process run."""

import json
import os
import shlex
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import pytest
import torch

from quantaweave_b200.tools import run_bundle as rb
from quantaweave_b200.training.trainer import default_args, run_training

REPO = Path(__file__).resolve().parents[1]


def _corpus(path: Path, rows: int = 60) -> Path:
    path.write_text("".join(json.dumps({"text": f"story {i}: the quick brown fox jumps over the lazy dog."}) + "\n"
                            for i in range(rows)))
    return path


def _args(tmp: Path, data: Path, **extra):
    options = dict(data=[data] if data is not None else [], steps=6, batch_size=2, sequence_length=16, examples=30,
                   hidden_size=16, layers=2, ffn_size=24, attention_heads=2, total_experts=4, active_experts=2, vocab_size=64, device="cpu",
                   checkpoint_interval=0, no_power_tracking=True, output=tmp / "out", checkpoint_dir=tmp / "ck",
                   archive_benchmark_examples=10)
    options.update(extra)
    return default_args(**options)


def _only_bundle(root: Path) -> Path:
    bundles = [p for p in root.iterdir() if p.is_dir()]
    assert len(bundles) == 1, bundles
    return bundles[0]


@pytest.fixture(autouse=True)
def _private_tempdir(tmp_path, monkeypatch):
    """Each test gets its own temporary directory, so files that concurrently running tests leave in the shared
    one are never counted as this test's leftovers."""
    private = tmp_path / "tempdir"
    private.mkdir()
    monkeypatch.setattr(tempfile, "tempdir", str(private))


def _temp_leftovers() -> set:
    root = Path(tempfile.gettempdir())
    return {p.name for p in root.glob("diagnostics-*")} | {p.name for p in root.glob("tmp*.jsonl")}


def test_folders_are_named_by_the_epoch_second_and_never_overwrite(tmp_path):
    runs = tmp_path / "runs"
    assert rb.epoch_folder(runs, now=1789939200.9).name == "1789939200"
    assert rb.epoch_folder(runs, now=1789939200).name == "1789939200-1"
    assert rb.epoch_folder(runs, now=1789939200).name == "1789939200-2"
    assert rb.epoch_folder(runs, now=1789939201).name == "1789939201"
    before = int(time.time())
    assert before <= int(rb.epoch_folder(runs).name) <= before + 2


def test_the_library_does_not_archive_unless_asked_and_restores_the_callers_options(tmp_path):
    data = _corpus(tmp_path / "d.jsonl")
    leftovers = _temp_leftovers()
    run_training(_args(tmp_path / "a", data))
    run_training(_args(tmp_path / "b", data, archive_dir=tmp_path / "never", no_archive=True))
    assert not (tmp_path / "never").exists()
    args = _args(tmp_path / "c", data, archive_dir=tmp_path / "archive")
    summary = run_training(args)
    assert Path(summary["archive"]).parent == tmp_path / "archive"
    # archiving used a temporary metrics file and diagnostics folder: both are gone and the options are as given
    assert args.metrics_file is None and args.diagnostics_dir is None and args.diagnostics_interval == 0
    assert _temp_leftovers() == leftovers


def test_a_failing_run_leaves_no_temporary_files_and_no_half_made_archive(tmp_path):
    data = _corpus(tmp_path / "d.jsonl")
    leftovers = _temp_leftovers()
    args = _args(tmp_path, data, archive_dir=tmp_path / "archive", curriculum="rarity", curriculum_steps=0)
    with pytest.raises(ValueError):
        run_training(args)
    assert _temp_leftovers() == leftovers
    assert args.metrics_file is None and args.diagnostics_dir is None and args.diagnostics_interval == 0
    assert not (tmp_path / "archive").exists() or not any((tmp_path / "archive").iterdir())


def test_the_reproduce_script_recreates_the_exact_weights(tmp_path):
    data = _corpus(tmp_path / "d.jsonl")
    args = _args(tmp_path, data, archive_dir=tmp_path / "archive", lr=2e-3, curriculum="entropy",
                 curriculum_steps=6, capacity_factor=0.7)
    run_training(args)
    bundle = _only_bundle(tmp_path / "archive")
    script = (bundle / "reproduce.sh").read_text()
    assert "--lr 0.002" in script and "--seed 0" in script and "--curriculum entropy" in script  # every option
    assert "--archive-dir" not in script and "--no-archive" not in script
    command = (script.replace(str(args.output), str(tmp_path / "rerun-out"))
               .replace(str(args.checkpoint_dir), str(tmp_path / "rerun-ck"))
               .replace("python -m ", f"{shlex.quote(sys.executable)} -m ").rstrip("\n") + " --no-archive\n")
    (tmp_path / "rerun.sh").write_text(command)
    env = {**os.environ, "PYTHONPATH": str(REPO), "PYTHONHASHSEED": "0"}
    subprocess.run(["bash", str(tmp_path / "rerun.sh")], cwd=REPO, check=True, capture_output=True, env=env,
                   timeout=600)
    a = torch.load(bundle / "model" / "model.pt", weights_only=False)["model"]
    b = torch.load(tmp_path / "rerun-out" / "model.pt", weights_only=False)["model"]
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_archive_failures_become_warnings(tmp_path, monkeypatch):
    def broken(*args, **kwargs):
        raise OSError("disk full")

    monkeypatch.setattr(rb, "write_samples", broken)
    data = _corpus(tmp_path / "d.jsonl")
    summary = run_training(_args(tmp_path, data, archive_dir=tmp_path / "archive"))
    bundle = Path(summary["archive"])
    record = json.loads((bundle / "summary.json").read_text())
    assert any("samples failed" in w and "disk full" in w for w in record["warnings"])
    assert (bundle / "samples.error.txt").exists() and (bundle / "model" / "model.pt").exists()
    assert "## Warnings" in (bundle / "README.md").read_text()


def test_large_data_is_recorded_by_hash_not_copied(tmp_path, monkeypatch):
    data = _corpus(tmp_path / "d.jsonl", rows=200)
    size = data.stat().st_size
    digest, coverage = rb.file_digest(data)
    assert coverage == "full" and len(digest) == 64
    monkeypatch.setattr(rb, "FULL_HASH_LIMIT", size // 2)
    monkeypatch.setattr(rb, "PARTIAL_HASH_BYTES", 256)
    partial, coverage = rb.file_digest(data)
    assert coverage == "partial" and partial != digest and rb.count_rows(data) is None
    bundle = tmp_path / "bundle"
    bundle.mkdir()
    manifest = rb.archive_data([data], bundle, limit_mb=size / 2 / (1 << 20), rows_used=30)
    assert not manifest["copied"] and "exceeds" in manifest["note"] and not (bundle / "data" / data.name).exists()
    entry = manifest["files"][0]
    assert entry["sha256"] == partial and entry["hash_coverage"] == "partial" and entry["rows_used_for_training"] == 30
    card = tmp_path / "card.json"
    card.write_text(json.dumps({"license": "CC0"}))
    assert rb.archive_data([data], bundle, 100, 30, data_card=card)["data_card"] == {"license": "CC0"}


def test_without_unseen_rows_only_the_training_benchmark_runs(tmp_path):
    data = _corpus(tmp_path / "d.jsonl", rows=30)
    summary = run_training(_args(tmp_path, data, examples=30, archive_dir=tmp_path / "archive"))
    record = json.loads((Path(summary["archive"]) / "summary.json").read_text())
    assert "train-slice" in record["benchmarks"] and "held-out" not in record["benchmarks"]
    assert any("no unseen rows" in w for w in record["warnings"])


def test_packed_token_runs_are_archived_without_a_benchmark(tmp_path):
    from quantaweave_b200.tools.prepare_tokens import main as prepare

    data = _corpus(tmp_path / "d.jsonl")
    prepare(["pack", "--data", str(data), "--tokenizer", "char", "--vocab-size", "64", "--output",
             str(tmp_path / "packed")])
    summary = run_training(_args(tmp_path, None, token_data=tmp_path / "packed",
                                 archive_dir=tmp_path / "archive"))
    bundle = Path(summary["archive"])
    record = json.loads((bundle / "summary.json").read_text())
    assert record["benchmarks"] == {} and (bundle / "model" / "model.pt").exists()
    assert any("no benchmark" in w for w in record["warnings"])


def _archived_ep_run(rank, world, tmp):
    from test_parallel_cpu import _trainer_case

    return _trainer_case(rank, world, tmp, 2, {"archive_dir": Path(tmp) / "archive", "checkpoint_interval": 0})


def test_a_multi_process_run_creates_exactly_one_archive_with_the_consolidated_model(tmp_path):
    from test_parallel_cpu import run_ranks

    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM

    run_ranks(_archived_ep_run, 2, (str(tmp_path),))
    bundle = _only_bundle(tmp_path / "archive")
    cfg = QuantaWeaveConfig.load(bundle / "model" / "config.json")
    QuantaWeaveMoEForCausalLM(cfg).load_state_dict(
        torch.load(bundle / "model" / "model.pt", weights_only=False)["model"])  # every expert, in one file
    assert not (bundle / "model" / "shards").exists()
