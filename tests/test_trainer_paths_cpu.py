"""Trainer paths on CPU (reference tests: tests/test_training_features.py): checkpoint metadata, the closed-loop
controllers' effect on the saved model, capacity release, aux/temperature adaptation, the BPE and packed-token data
paths, activation checkpointing and bf16 autocast through training, device detection and precision choice, exact
parameter counts and the expert-count suggestion."""

import json
from pathlib import Path

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.training.trainer import default_args, run_training
from quantaweave_b200.utils import hardware as hw
from quantaweave_b200.utils.checkpoint_io import load_checkpoint


def _corpus(path: Path, rows: int = 60) -> Path:
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text("".join(json.dumps({"text": f"story {i}: the quick brown fox jumps over the lazy dog."}) + "\n"
                            for i in range(rows)))
    return path


def _args(tmp: Path, **extra):
    base = dict(data=[_corpus(tmp / "d.jsonl")], steps=4, batch_size=2, sequence_length=16, examples=60,
                hidden_size=16, layers=2, ffn_size=16, attention_heads=2, total_experts=4, active_experts=2,
                vocab_size=64, device="cpu", checkpoint_interval=0, no_power_tracking=True, seed=0,
                output=tmp / "out", checkpoint_dir=tmp / "ck")
    base.update(extra)
    return default_args(**base)


def test_checkpoints_carry_resume_metadata(tmp_path):
    run_training(_args(tmp_path, checkpoint_interval=2, lr_decay="cosine"))
    meta = json.loads((tmp_path / "ck" / "metadata.json").read_text())
    assert meta["step"] == 4 and meta["torch"] == torch.__version__ and len(meta["config_hash"]) > 8
    assert meta["resume_fields"]["hidden_size"] == 16 and meta["schedule"] and meta["data"]["samples_consumed"] == 8
    payload = load_checkpoint(tmp_path / "ck" / "model.pt")
    assert payload["step"] == 4 and payload["extra"]["config_hash"] == meta["config_hash"]
    assert {"python", "torch"} <= set(payload["rng_state"]) and payload["optimizer"]["state"]
    for name in ("config.json", "vocab.json", "tokenizer_meta.json"):
        assert (tmp_path / "ck" / name).exists(), name


def test_the_capacity_controller_grows_capacity_in_the_saved_model_and_release_switches_it_off(tmp_path):
    run_training(_args(tmp_path / "grow", capacity_factor=0.3, capacity_adapt=True, drop_threshold=0.0,
                       controller_interval=1, steps=4))
    grown = json.loads((tmp_path / "grow" / "out" / "config.json").read_text())["capacity_factor"]
    assert grown > 0.3
    run_training(_args(tmp_path / "rel", capacity_factor=0.3, capacity_adapt=True, controller_interval=1,
                       capacity_release_step=2, steps=4))
    released = QuantaWeaveConfig.load(tmp_path / "rel" / "out" / "config.json")
    assert released.drop_overflow_tokens is False  # release switches capacity enforcement off in the saved model


def test_aux_and_temperature_adaptation_run_and_stay_finite(tmp_path):
    summary = run_training(_args(tmp_path, aux_adapt=True, temperature_adapt=True, temperature_start=2.0,
                                 temperature_steps=4, aux_coef_end=0.05, controller_interval=1, log_interval=1,
                                 metrics_file=tmp_path / "m.jsonl"))
    rows = [json.loads(x) for x in (tmp_path / "m.jsonl").read_text().splitlines()]
    assert summary["steps"] == 4 and all(torch.isfinite(torch.tensor(r["loss"])) for r in rows)
    assert summary["controller_history"]


def test_bpe_tokenizer_and_packed_token_corpus_paths(tmp_path):
    from quantaweave_b200.data.pipeline import load_tokenizer
    from quantaweave_b200.tools.prepare_tokens import main as prepare

    run_training(_args(tmp_path / "bpe", tokenizer="bpe", tokenizer_path=tmp_path / "tok", vocab_size=300))
    tok = load_tokenizer(tmp_path / "bpe" / "out")
    assert tok.kind == "bpe" and json.loads((tmp_path / "bpe" / "out" / "config.json").read_text())[
        "vocab_size"] == tok.vocab_size
    data = _corpus(tmp_path / "p.jsonl")
    prepare(["pack", "--data", str(data), "--tokenizer", "char", "--vocab-size", "64", "--output",
             str(tmp_path / "packed")])
    summary = run_training(_args(tmp_path / "tok", data=[], token_data=tmp_path / "packed"))
    assert summary["steps"] == 4 and load_tokenizer(tmp_path / "tok" / "out").kind == "char"


def test_activation_checkpointing_does_not_change_training(tmp_path):
    run_training(_args(tmp_path / "a"))
    run_training(_args(tmp_path / "b", activation_checkpointing=True))
    a = load_checkpoint(tmp_path / "a" / "out" / "model.pt")["model"]
    b = load_checkpoint(tmp_path / "b" / "out" / "model.pt")["model"]
    for key in a:
        assert torch.allclose(a[key], b[key], atol=1e-6), key


def test_bf16_autocast_training_on_cpu_stays_finite(tmp_path):
    summary = run_training(_args(tmp_path, precision="bf16", log_interval=1, metrics_file=tmp_path / "m.jsonl"))
    assert summary["precision"] == "bf16"
    losses = [json.loads(x)["loss"] for x in (tmp_path / "m.jsonl").read_text().splitlines()]
    assert len(losses) == 4 and all(torch.isfinite(torch.tensor(losses)))


def test_detect_and_precision_choice():
    info = hw.detect("cpu")
    assert info.backend == "cpu" and info.torch_device == torch.device("cpu")
    assert hw.choose_precision(info) == "fp32" and hw.choose_precision(info, "bf16") == "bf16"
    with pytest.raises(ValueError):
        hw.choose_precision(info, "fp16")  # no fp16 autocast on the host
    with pytest.raises(ValueError):
        hw.choose_precision(info, "int8")
    gpu = hw.DeviceInfo("cuda", "fake", 1, 8 << 30, 8 << 30, bf16=False, fp16=True, runtime="test")
    assert hw.choose_precision(gpu) == "fp16"
    with pytest.raises(ValueError):
        hw.choose_precision(gpu, "bf16")
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            hw.detect("cuda")


def test_parameter_counts_match_a_real_model():
    config = QuantaWeaveConfig(vocab_size=64, hidden_size=16, layers=2, ffn_size=24, num_experts=4, top_k=2,
                               attention_heads=2, max_sequence_length=17)
    counts = hw.parameter_counts(config)
    model = QuantaWeaveMoEForCausalLM(config)
    assert counts["total"] == sum(p.numel() for p in model.parameters())
    assert counts["experts"] == 2 * 4 * 3 * 16 * 24 and counts["per_expert"] == 3 * 16 * 24
    assert counts["active"] == counts["total"] - 2 * (4 - 2) * counts["per_expert"]
    assert hw.training_state_bytes(config) == 16 * counts["total"]


def test_the_expert_suggestion_grows_with_memory_and_respects_its_cap():
    def suggest(gb, cap=256):
        info = hw.DeviceInfo("cpu", "fake", 1, int(gb * 1e9), int(gb * 1e9), True, False, "t")
        return hw.suggest_num_experts(info, 256, 512, 4, 2, 7168, 128, cap=cap)

    assert 2 <= suggest(1) <= suggest(4) <= suggest(16) and suggest(1) < suggest(16)
    assert suggest(1000, cap=32) == 32


def test_step_values_are_read_back_only_at_flush_points_with_the_same_results(tmp_path, monkeypatch):
    from quantaweave_b200.training import trainer

    every = run_training(_args(tmp_path / "every", steps=10, log_interval=1, metrics_file=tmp_path / "a.jsonl"))
    flushes = []
    original = trainer.StepScalars.flush

    def counting(self, reduce):
        flushes.append([step for step, _, _ in self.rows])
        return original(self, reduce)

    monkeypatch.setattr(trainer.StepScalars, "flush", counting)
    sparse = run_training(_args(tmp_path / "sparse", steps=10, log_interval=5, controller_interval=50,
                                metrics_file=tmp_path / "b.jsonl"))
    assert flushes == [[1, 2, 3, 4, 5], [6, 7, 8, 9, 10]]  # two transfers instead of ten
    dense_rows = {r["step"]: r for r in map(json.loads, (tmp_path / "a.jsonl").read_text().splitlines())}
    for row in map(json.loads, (tmp_path / "b.jsonl").read_text().splitlines()):
        assert row["loss"] == dense_rows[row["step"]]["loss"]
        assert row["overflow_routes"] == dense_rows[row["step"]]["overflow_routes"]
    assert sparse["last_log"]["loss"] == every["last_log"]["loss"]  # (final_loss averages the logged tail)
