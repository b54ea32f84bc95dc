"""Trainer features end to end on CPU (reference tests: tests/test_training_features.py, tests/test_future_features.py):
a validation split scored only on its own interval, multi-domain training with the specialisation loss and domain
weights, PII redaction of the training text, the CPU-offload optimizer with exact resume, routing diagnostics
output, curriculum ordering, and option validation."""

import json
from pathlib import Path

import pytest
import torch

from quantaweave_b200.training.trainer import default_args, run_training
from quantaweave_b200.utils.checkpoint_io import load_checkpoint as load_file


def _corpus(tmp: Path) -> list[Path]:
    prose = tmp / "prose.jsonl"
    code = tmp / "code.jsonl"
    prose.write_text("".join(json.dumps({"text": f"story {i}: the fox met the dog near the river bank. "
                                                 "contact me at jane.doe@example.com"}) + "\n" for i in range(40)))
    code.write_text("".join(json.dumps({"text": f"def f{i}(x):\n    return x * {i} + 1\n"}) + "\n" for i in range(40)))
    return [prose, code]


def _args(tmp: Path, name: str, steps: int, **extra):
    options = dict(data=_corpus(tmp), vocab_size=96, sequence_length=32, batch_size=4, hidden_size=32, layers=2,
                   ffn_size=64, attention_heads=2, total_experts=4, active_experts=2, steps=steps, device="cpu",
                   seed=0, no_power_tracking=True, no_archive=True, output=tmp / name / "out",
                   checkpoint_dir=tmp / name / "ckpt", checkpoint_interval=4, metrics_file=tmp / name / "m.jsonl",
                   log_interval=1)
    options.update(extra)
    return default_args(**options)


def _rows(path: Path) -> list[dict]:
    return [json.loads(line) for line in path.read_text().splitlines()]


def test_validation_is_scored_only_on_its_interval(tmp_path):
    run_training(_args(tmp_path, "val", 6, val_fraction=0.2, val_interval=3, val_batches=2))
    rows = _rows(tmp_path / "val" / "m.jsonl")
    with_val = [r["step"] for r in rows if "val_loss" in r]
    assert with_val == [3, 6] and all(r["val_loss"] > 0 for r in rows if "val_loss" in r)


def test_multi_domain_training_with_specialisation_loss_weights_and_diagnostics(tmp_path):
    summary = run_training(_args(tmp_path, "dom", 4, domain_specialization_coef=0.1,
                                 domain_weights="prose=3,code=1", diagnostics_interval=2,
                                 diagnostics_dir=tmp_path / "dom" / "diag"))
    assert summary["steps"] == 4
    rows = _rows(tmp_path / "dom" / "m.jsonl")
    assert all("domain_loss" in r for r in rows)
    log = tmp_path / "dom" / "diag" / "routing_log.jsonl"
    assert log.exists() and _rows(log)[0]["layers"]
    assert (tmp_path / "dom" / "diag" / "index.html").exists()


def test_redact_pii_changes_the_training_text(tmp_path):
    plain = run_training(_args(tmp_path, "plain", 1))
    redacted = run_training(_args(tmp_path, "red", 1, redact_pii=True))
    del plain, redacted
    vocab_plain = (tmp_path / "plain" / "out" / "vocab.json").read_text()
    vocab_red = (tmp_path / "red" / "out" / "vocab.json").read_text()
    assert "@" in vocab_plain and "@" not in vocab_red  # the e-mail address never reached the tokenizer


def test_cpu_offload_optimizer_trains_and_resumes_exactly(tmp_path):
    run_training(_args(tmp_path, "straight", 8, optimizer="adamw_cpu_offload"))
    run_training(_args(tmp_path, "split", 4, optimizer="adamw_cpu_offload"))
    run_training(_args(tmp_path, "split", 8, optimizer="adamw_cpu_offload"))
    a = load_file(tmp_path / "straight" / "out" / "model.pt")["model"]
    b = load_file(tmp_path / "split" / "out" / "model.pt")["model"]
    for key in a:
        assert torch.equal(a[key], b[key]), key


def test_curriculum_run_and_option_validation(tmp_path):
    summary = run_training(_args(tmp_path, "cur", 3, curriculum="rarity", curriculum_steps=10))
    assert summary["steps"] == 3
    for bad in (dict(curriculum="rarity", curriculum_steps=0), dict(shard_optimizer=True),
                dict(gradient_accumulation_steps=0)):
        with pytest.raises(ValueError):
            run_training(_args(tmp_path, "bad", 1, **bad))
