"""CPU tests of the run tooling: training with routing diagnostics and a run archive, the benchmark report, the
plain sampler and the reproduce command (reference tests: tests/test_run_bundle.py, tests/test_benchmark.py,
tests/test_routing_diagnostics.py)."""

import json
from pathlib import Path

import torch

from quantaweave_b200.training.trainer import build_parser, default_args, run_training


def _corpus(path: Path, rows: int = 120) -> Path:
    words = ["the cat sat on the mat", "a dog ran far away", "numbers 12 34 56", "sun and moon, stars!"]
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w") as fh:
        for i in range(rows):
            fh.write(json.dumps({"text": f"{words[i % 4]} {i}", "domain": "story" if i % 2 else "code"}) + "\n")
    return path


def _train(tmp: Path, **extra):
    data = _corpus(tmp / "data.jsonl")
    options = dict(data=[data], examples=60, tokenizer="char", sequence_length=32, hidden_size=32, layers=2,
                   ffn_size=64, attention_heads=2, total_experts=4, active_experts=2, batch_size=4, steps=6,
                   device="cpu", seed=0, no_power_tracking=True, output=tmp / "out", checkpoint_dir=tmp / "ckpt",
                   metrics_file=tmp / "metrics.jsonl", diagnostics_dir=tmp / "diag", diagnostics_interval=2)
    options.update(extra)
    return data, run_training(default_args(**options))


def test_training_archive_bundle(tmp_path):
    data, summary = _train(tmp_path, archive_dir=tmp_path / "runs", archive_benchmark_examples=20)
    bundle = Path(summary["archive"])
    assert bundle.parent == tmp_path / "runs" and bundle.name.split("-")[0].isdigit()
    for name in ("README.md", "summary.json", "config.json", "reproduce.sh", "environment.json", "samples.txt",
                 "model/model.pt", "model/config.json", "data/manifest.json", "training/metrics.jsonl",
                 "training/diagnostics/index.html", "benchmarks/train-slice.json", "benchmarks/held-out.md"):
        assert (bundle / name).exists(), name
    record = json.loads((bundle / "summary.json").read_text())
    assert record["kind"] == "train" and "generalisation_gap" in record["benchmarks"]
    manifest = json.loads((bundle / "data/manifest.json").read_text())
    assert manifest["copied"] and manifest["files"][0]["rows_used_for_training"] == 60
    assert "python -m quantaweave_b200.train" in (bundle / "reproduce.sh").read_text()
    diag = [json.loads(line) for line in (tmp_path / "diag" / "routing_log.jsonl").read_text().splitlines()]
    assert len(diag) == 3 and len(diag[0]["layers"]) == 2
    layer = diag[0]["layers"][0]
    assert abs(sum(layer["requested_share"]) - 1) < 1e-6 and 0 <= layer["drop_rate"] <= 1


def test_benchmark_report_and_markdown(tmp_path):
    from quantaweave_b200.tools.benchmark import build_parser as bench_parser, render_markdown, run_benchmark

    data, _ = _train(tmp_path)
    args = bench_parser().parse_args(["--checkpoint", str(tmp_path / "out"), "--data", str(data), "--examples", "30",
                                      "--batch-size", "4", "--device", "cpu", "--training-metrics",
                                      str(tmp_path / "metrics.jsonl")])
    report = run_benchmark(args)
    assert report["tokens"] > 0 and report["perplexity"] > 1
    assert len(report["routing"]["per_layer"]) == 2
    assert report["training_stability"]["logged_steps"] == 6
    assert abs(report["expert_utilization_mean"] - 0.25) < 1e-6  # shares of all routes over 4 experts
    assert "## Routing" in render_markdown(report)


def test_sample_text_stops_and_decodes(tmp_path):
    from quantaweave_b200.data.pipeline import load_tokenizer
    from quantaweave_b200.tools.common import load_model
    from quantaweave_b200.tools.generate import sample_text

    _train(tmp_path)
    model = load_model(tmp_path / "out", torch.device("cpu"))
    tok = load_tokenizer(tmp_path / "out")
    torch.manual_seed(0)
    text = sample_text(model, tok, "the", 12, 0.8, torch.device("cpu"))
    assert text.startswith("the") and len(text) <= 3 + 12 * 4


def test_reproduce_command_lists_non_defaults():
    from quantaweave_b200.tools.run_bundle import reproduce_command

    parser = build_parser()
    args = parser.parse_args(["--steps", "7", "--no-resume", "--data", "a.jsonl", "b.jsonl"])
    cmd = reproduce_command("quantaweave_b200.train", parser, args)
    assert "--steps 7" in cmd and "--no-resume" in cmd and "--data a.jsonl b.jsonl" in cmd
    assert "--lr" not in cmd
    full = reproduce_command("quantaweave_b200.train", parser, args, explicit=True)
    assert "--lr 0.0003" in full


def test_hardware_cli_auto_architecture(capsys):
    import json

    from quantaweave_b200.utils.hardware import main

    main(["--device", "cpu", "--auto-architecture", "--quality", "capacity", "--precision", "fp32"])
    report = json.loads(capsys.readouterr().out)
    assert report["precision"] == "fp32" and report["shape"]["total_experts"] >= 1
    assert report["parameters"]["total"] > 0 and report["suggested_num_experts"] >= 1


def test_reference_helper_names(tmp_path):
    """``build_vocab`` (trainer) and ``layer_weight`` (decoder) from the reference's public module surface."""
    import json

    import torch

    from quantaweave_b200.inference.fast_decode import Unsupported, layer_weight
    from quantaweave_b200.inference.quantization import QuantizedLinear
    from quantaweave_b200.training.trainer import build_vocab

    corpus = tmp_path / "c.jsonl"
    corpus.write_text(json.dumps({"text": "abcab"}) + "\n" + json.dumps({"text": "cd"}) + "\n")
    vocab = build_vocab(corpus, 64)
    assert {"a", "b", "c", "d"} <= set(vocab)
    linear = torch.nn.Linear(64, 8, bias=False)
    assert torch.equal(layer_weight(linear), linear.weight.detach())
    q = QuantizedLinear.from_linear(linear, 8) if hasattr(QuantizedLinear, "from_linear") else None
    if q is not None:
        assert (layer_weight(q) - linear.weight).abs().max() < 0.05
    try:
        layer_weight(torch.nn.ReLU())
        raise AssertionError("expected Unsupported")
    except Unsupported:
        pass


def test_every_command_line_option_is_documented():
    import importlib

    from quantaweave_b200.training.trainer import build_parser as train_parser

    parsers = {"train": train_parser()}
    for name in ("chat", "serve", "finetune", "distill", "benchmark", "generate"):
        parsers[name] = importlib.import_module(f"quantaweave_b200.tools.{name}").build_parser()
    for name, parser in parsers.items():
        bare = [a.option_strings[-1] for a in parser._actions if a.option_strings and a.dest != "help" and not a.help]
        assert not bare, (name, bare)
