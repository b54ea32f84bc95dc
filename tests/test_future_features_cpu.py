"""Features added on top of the core trainer (reference tests: tests/test_future_features.py): the auto-architecture
shape search, SentencePiece through training and chat, validation-option checks, the optimizer factory, the ONNX
export's clean skip / failure report, BOHB and Pareto sweeps, and the straggler-capacity option check."""

import json
import sys
import types
from pathlib import Path

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig
from quantaweave_b200.utils import hardware as hw


def _device(gb: float) -> hw.DeviceInfo:
    return hw.DeviceInfo("cpu", "fake", 1, int(gb * 1e9), int(gb * 1e9), True, False, "test")


def _corpus(path: Path, rows: int = 60) -> Path:
    path.write_text("".join(json.dumps({"text": f"story {i}: the quick brown fox jumps over the lazy dog."}) + "\n"
                            for i in range(rows)))
    return path


# ---- auto architecture ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("quality", ["capacity", "balanced", "dense"])
def test_auto_architecture_fills_its_budget_with_a_buildable_config(quality):
    info = _device(8.0)
    shape = hw.auto_architecture(info, 7168, 0.45, quality)
    config = QuantaWeaveConfig(vocab_size=7168, hidden_size=shape["hidden_size"], layers=shape["layers"],
                               ffn_size=shape["ffn_size"], num_experts=shape["total_experts"],
                               top_k=shape["active_experts"], attention_heads=shape["attention_heads"],
                               max_sequence_length=shape["sequence_length"] + 1)
    assert hw.parameter_counts(config)["total"] == shape["total_parameters"]
    assert 0.9 < shape["training_state_fraction_of_budget"] <= 1.0
    assert shape["training_state_bytes"] <= 0.45 * info.total_memory_bytes


def test_capacity_and_dense_spend_the_budget_differently_and_more_memory_buys_a_bigger_model():
    capacity = hw.auto_architecture(_device(8.0), quality="capacity")
    dense = hw.auto_architecture(_device(8.0), quality="dense")
    assert dense["total_experts"] == dense["active_experts"] == 1
    assert dense["active_parameters"] == dense["total_parameters"]
    assert capacity["active_experts"] == 1 and capacity["total_experts"] >= 64
    assert capacity["active_parameters"] < capacity["total_parameters"] / 10
    assert dense["hidden_size"] > capacity["hidden_size"]  # without an expert pool, width carries the budget
    small, large = hw.auto_architecture(_device(8.0)), hw.auto_architecture(_device(40.0))
    assert large["total_parameters"] > 3 * small["total_parameters"]
    assert large["hidden_size"] >= small["hidden_size"] and large["layers"] >= small["layers"]


def test_auto_architecture_rejects_bad_input_and_shapes_that_fit_no_device():
    with pytest.raises(ValueError, match="quality"):
        hw.auto_architecture(_device(8.0), quality="bogus")
    with pytest.raises(ValueError, match="memory_fraction"):
        hw.auto_architecture(_device(8.0), memory_fraction=0)
    with pytest.raises(ValueError, match="memory"):
        hw.auto_architecture(hw.DeviceInfo("cpu", "fake", 1, 0, 0, True, False, "test"))
    with pytest.raises(ValueError, match="no architecture fits"):
        hw.auto_architecture(_device(0.001), memory_fraction=0.5, quality="dense")
    tiny_budget = hw.auto_architecture(_device(1.0), memory_fraction=0.005, quality="dense")
    assert tiny_budget["hidden_size"] == 64 and tiny_budget["training_state_fraction_of_budget"] > 1  # over the
    # requested share, still far inside the device: the smallest shape is returned, not an error


def test_the_hardware_cli_reports_the_chosen_architecture(capsys):
    hw.main(["--device", "cpu", "--auto-architecture", "--quality", "capacity"])
    report = json.loads(capsys.readouterr().out)
    assert report["auto_architecture"]["quality"] == "capacity"
    assert report["parameters"]["total"] == report["auto_architecture"]["total_parameters"]


def test_trainer_auto_architecture_replaces_the_shape_and_pins_it_in_the_reproduce_script(tmp_path):
    from quantaweave_b200.training.trainer import default_args, run_training

    args = default_args(data=[_corpus(tmp_path / "d.jsonl")], steps=2, batch_size=2, examples=60, device="cpu",
                        checkpoint_interval=0, vocab_size=64, no_power_tracking=True, auto_architecture=True,
                        auto_architecture_quality="dense", auto_architecture_memory_fraction=1e-6,
                        output=tmp_path / "out", checkpoint_dir=tmp_path / "ck", archive_dir=tmp_path / "archive",
                        archive_benchmark_examples=4)
    args.sequence_length = 16  # keep the CPU step small; the shape search sets it, so override after resolving
    summary = run_training(args)
    config = json.loads((tmp_path / "out" / "config.json").read_text())
    assert config["num_experts"] == 1 and config["top_k"] == 1 and config["hidden_size"] == args.hidden_size
    script = (Path(summary["archive"]) / "reproduce.sh").read_text()
    assert "--auto-architecture" not in script.replace("\\\n", " ").split()
    assert f"--hidden-size {args.hidden_size}" in script and f"--total-experts {args.total_experts}" in script


# ---- SentencePiece end to end ---------------------------------------------------------------------------------------
def test_training_and_chatting_with_a_sentencepiece_tokenizer(tmp_path):
    from quantaweave_b200.data.pipeline import load_tokenizer
    from quantaweave_b200.tools import chat
    from quantaweave_b200.training.trainer import default_args, run_training

    data = tmp_path / "d.jsonl"
    data.write_text("".join(json.dumps({"text": f"the quick brown fox {i} jumps over the lazy dog"}) + "\n"
                            for i in range(60)))
    options = dict(data=[data], steps=3, batch_size=2, sequence_length=16, examples=60, hidden_size=16, layers=1,
                   ffn_size=16, attention_heads=2, total_experts=2, active_experts=1, vocab_size=60,
                   tokenizer="sentencepiece", tokenizer_path=tmp_path / "tok", device="cpu", checkpoint_interval=0,
                   no_power_tracking=True, output=tmp_path / "out", checkpoint_dir=tmp_path / "ck")
    run_training(default_args(**options))
    assert (tmp_path / "tok" / "tokenizer.model").exists()  # trained once, at --tokenizer-path
    tok = load_tokenizer(tmp_path / "out")
    config = json.loads((tmp_path / "out" / "config.json").read_text())
    assert tok.kind == "sentencepiece" and config["vocab_size"] == tok.vocab_size
    assert tok.decode(tok.encode("the lazy dog")) == "the lazy dog"
    stamp = (tmp_path / "tok" / "tokenizer.model").stat().st_mtime_ns
    run_training(default_args(**{**options, "output": tmp_path / "out2", "checkpoint_dir": tmp_path / "ck2"}))
    assert (tmp_path / "tok" / "tokenizer.model").stat().st_mtime_ns == stamp  # the second run reuses it
    assert load_tokenizer(tmp_path / "out2").vocab_size == tok.vocab_size
    model, loaded = chat.load_for_chat(tmp_path / "out", None, 0, torch.device("cpu"))
    session = chat.ChatSession(model, loaded, torch.device("cpu"), "fp32", chat.Settings(temperature=0, tokens=5))
    reply = session.send("the quick")
    assert reply.tokens <= 5 and reply.unknown_characters == []  # a subword model has no unknown characters


# ---- option validation ------------------------------------------------------------------------------------------------
def _tiny(tmp_path, **extra):
    from quantaweave_b200.training.trainer import default_args

    base = dict(data=[_corpus(tmp_path / "d.jsonl")], steps=1, batch_size=2, sequence_length=16, examples=60,
                hidden_size=16, layers=1, ffn_size=16, attention_heads=2, total_experts=2, active_experts=1,
                vocab_size=64, device="cpu", checkpoint_interval=0, no_power_tracking=True,
                output=tmp_path / "out", checkpoint_dir=tmp_path / "ck")
    base.update(extra)
    return default_args(**base)


@pytest.mark.parametrize("bad,match", [
    (dict(val_fraction=0.2, val_interval=0), "val-interval"),
    (dict(val_fraction=0.2, pipeline_parallel=True), "pipeline"),
    (dict(optimizer="adamw8bit", shard_optimizer=True, data_parallel=True), "shard-optimizer"),
    (dict(optimizer="adamw_cpu_offload", shard_optimizer=True, data_parallel=True), "shard-optimizer"),
    (dict(straggler_capacity=True), "expert-parallel"),
])
def test_incompatible_options_are_refused_before_training(tmp_path, bad, match):
    from quantaweave_b200.training.trainer import run_training

    with pytest.raises(ValueError, match=match):
        run_training(_tiny(tmp_path, **bad))


def test_a_domain_too_small_to_split_is_refused_and_no_fraction_means_no_validation(tmp_path):
    from quantaweave_b200.training.trainer import run_training

    small = tmp_path / "small.jsonl"
    small.write_text(json.dumps({"text": "one short rare row", "domain": "rare"}) + "\n")  # exactly one window
    with pytest.raises(ValueError, match="too few"):
        run_training(_tiny(tmp_path, data=[_corpus(tmp_path / "d.jsonl"), small], val_fraction=0.1, val_interval=1))
    rows_file = tmp_path / "m.jsonl"
    summary = run_training(_tiny(tmp_path, steps=2, metrics_file=rows_file, log_interval=1))
    assert summary["val_loss"] is None and not any("val_loss" in json.loads(x) for x in rows_file.read_text().splitlines())


# ---- the optimizer factory ----------------------------------------------------------------------------------------------
def test_build_optimizer_classes_and_checks():
    from quantaweave_b200.optim.cpu_offload import CPUOffloadAdamW
    from quantaweave_b200.training.trainer import build_optimizer

    params = [torch.nn.Parameter(torch.zeros(3))]
    assert isinstance(build_optimizer("adamw", params, 1e-3), torch.optim.AdamW)
    assert isinstance(build_optimizer("adamw_cpu_offload", params, 1e-3), CPUOffloadAdamW)
    with pytest.raises(RuntimeError, match="CUDA"):
        build_optimizer("adamw8bit", params, 1e-3)
    with pytest.raises(ValueError):
        build_optimizer("lion", params, 1e-3)


def test_the_finetuner_builds_its_optimizer_through_the_same_factory():
    import inspect

    from quantaweave_b200.tools import finetune

    assert "build_optimizer" in inspect.getsource(finetune)


# ---- ONNX ---------------------------------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def small_checkpoint(tmp_path_factory):
    from test_tools_cpu import _train

    tmp = tmp_path_factory.mktemp("onnx")
    _train(tmp, steps=1)
    return tmp / "out"


def test_onnx_is_skipped_cleanly_without_the_package(small_checkpoint, tmp_path, monkeypatch):
    from quantaweave_b200.tools.export import export_bundle

    monkeypatch.setitem(sys.modules, "onnx", None)  # import onnx -> ImportError
    meta = export_bundle(small_checkpoint, tmp_path / "bundle", onnx=True)
    assert meta["onnx"]["status"] == "skipped" and "onnx" in meta["onnx"]["reason"]
    assert not (tmp_path / "bundle" / "model.onnx").exists() and (tmp_path / "bundle" / "model.torchscript.pt").exists()


def test_an_onnx_exporter_failure_is_reported_not_raised(small_checkpoint, tmp_path, monkeypatch):
    from quantaweave_b200.tools.export import export_bundle

    monkeypatch.setitem(sys.modules, "onnx", types.ModuleType("onnx"))

    def broken(*args, **kwargs):
        raise RuntimeError("unsupported operator")

    monkeypatch.setattr(torch.onnx, "export", broken)
    meta = export_bundle(small_checkpoint, tmp_path / "bundle", onnx=True)
    assert meta["onnx"]["status"] == "failed" and "unsupported operator" in meta["onnx"]["reason"]
    assert not (tmp_path / "bundle" / "model.onnx").exists()


# ---- sweeps: BOHB and Pareto -----------------------------------------------------------------------------------------------
def _sweep_base(tmp_path):
    return dict(data=[str(_corpus(tmp_path / "d.jsonl"))], examples=40, tokenizer="char", sequence_length=16,
                hidden_size=16, layers=1, ffn_size=16, attention_heads=2, total_experts=4, active_experts=1,
                batch_size=2, steps=1, device="cpu", no_power_tracking=True)


def test_bohb_proposes_the_base_rung_then_promotes_survivors_and_never_an_invalid_trial(tmp_path):
    from quantaweave_b200.tools.sweep import run_sweep

    cfg = {"name": "b", "strategy": "bohb", "base": _sweep_base(tmp_path), "metric": "train.final_loss",
           "n_trials": 4, "halving": {"eta": 2, "rungs": 2}, "bayes": {"n_init": 2, "candidates": 64},
           "space": {"lr": {"loguniform": [1e-4, 1e-2]}, "active_experts": [1, 2, 8]},
           "objectives": ["train.final_loss:min", "train.tokens_per_second:max"]}
    out = run_sweep(cfg, tmp_path / "runs")
    assert [r["trials"] for r in out["rungs"]] == [4, 2] and out["rungs"][1]["steps"] == 2
    trials = [json.loads(p.read_text())["train"] for p in Path(out["sweep_dir"]).glob("*/config.json")]
    assert trials and all(t["active_experts"] <= t["total_experts"] for t in trials)  # 8 of 4 is never proposed
    assert len(out["trajectory"]) == 4 and out["pareto_front"] and out["best"] is not None
    preview = run_sweep(cfg, tmp_path / "dry", dry_run=True)
    assert preview["dry_run"] and len(preview["first_trials"]) == 3 and not (tmp_path / "dry").exists()
    with pytest.raises(ValueError, match="strategy"):
        run_sweep({**cfg, "strategy": "bohbb"}, tmp_path / "typo")


def test_a_grid_sweep_reports_a_pareto_front_only_with_objectives(tmp_path):
    from quantaweave_b200.tools.sweep import run_sweep

    cfg = {"name": "g", "strategy": "grid", "base": _sweep_base(tmp_path), "metric": "train.final_loss",
           "space": {"lr": [1e-3, 3e-3]}}
    plain = run_sweep(cfg, tmp_path / "a")
    assert "pareto_front" not in plain
    with_objectives = run_sweep({**cfg, "objectives": ["train.final_loss:min", "train.tokens_per_second:max"]},
                                tmp_path / "b")
    assert 1 <= len(with_objectives["pareto_front"]) <= 2
    assert "## Pareto front" in (Path(with_objectives["sweep_dir"]) / "sweep_results.md").read_text()
