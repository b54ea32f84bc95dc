"""Distillation, benchmark and sampler paths on CPU (reference tests: tests/test_deploy_and_distill.py): logit
distillation from a teacher checkpoint lowers the teacher-student KL, a teacher with another tokenizer is refused,
the sequence length is checked against the student's context, the benchmark's diagnostic pass can be skipped, and
the sampler runs from character and BPE checkpoints."""

import torch
import torch.nn.functional as F

from quantaweave_b200.data.pipeline import load_tokenizer
from quantaweave_b200.tools.common import load_model
from quantaweave_b200.tools.distill import build_parser, run_distillation

CPU = torch.device("cpu")


def _kl(teacher_dir, student_dir, text):
    teacher, student = load_model(teacher_dir, CPU).eval(), load_model(student_dir, CPU).eval()
    ids = torch.tensor([load_tokenizer(teacher_dir).encode(text)[:32]])
    with torch.no_grad():
        t = F.log_softmax(teacher(ids)["logits"].float(), -1)
        s = F.log_softmax(student(ids)["logits"].float(), -1)
    return float(F.kl_div(s, t, log_target=True, reduction="batchmean"))


def _distill_args(tmp_path, student, data, *extra):
    return build_parser().parse_args(["--student", str(student), "--teacher-data", str(data), "--batch-size", "2",
                                      "--sequence-length", "32", "--examples", "60", "--device", "cpu",
                                      "--checkpoint-interval", "0", "--no-archive", "--output",
                                      str(tmp_path / "distilled"), "--checkpoint-dir", str(tmp_path / "dck"), *extra])


def test_logit_distillation_moves_the_student_towards_the_teacher(tmp_path):
    from test_tools_cpu import _train

    data, _ = _train(tmp_path / "teacher", steps=30, lr=3e-3)
    _train(tmp_path / "student", steps=1, seed=1)
    text = "the cat sat on the mat 12 a dog ran far away numbers"
    before = _kl(tmp_path / "teacher" / "out", tmp_path / "student" / "out", text)
    result = run_distillation(_distill_args(tmp_path, tmp_path / "student" / "out", data, "--teacher-checkpoint",
                                            str(tmp_path / "teacher" / "out"), "--steps", "12", "--lr", "3e-3",
                                            "--alpha", "1.0"))
    assert result["mode"] == "logit"
    after = _kl(tmp_path / "teacher" / "out", tmp_path / "distilled", text)
    assert after < before, (before, after)


def test_a_teacher_with_another_tokenizer_is_refused_for_logit_distillation(tmp_path):
    import pytest
    from test_tools_cpu import _train

    data, _ = _train(tmp_path / "student", steps=1)
    _train(tmp_path / "teacher", steps=1, tokenizer="bpe", tokenizer_path=tmp_path / "bpe", vocab_size=300)
    with pytest.raises(ValueError, match="tokenizer"):
        run_distillation(_distill_args(tmp_path, tmp_path / "student" / "out", data, "--teacher-checkpoint",
                                       str(tmp_path / "teacher" / "out"), "--steps", "1"))


def test_sequence_distillation_checks_the_length_against_the_students_context(tmp_path):
    import pytest
    from test_tools_cpu import _train

    data, _ = _train(tmp_path / "student", steps=1)  # trained with 32-token windows
    args = _distill_args(tmp_path, tmp_path / "student" / "out", data, "--steps", "1")
    args.sequence_length = 64
    with pytest.raises(ValueError, match="sequence-length"):
        run_distillation(args)
    args.sequence_length = 32
    assert run_distillation(args)["mode"] == "sequence"


def test_the_benchmark_can_skip_its_routing_pass(tmp_path):
    from test_tools_cpu import _train

    from quantaweave_b200.tools.benchmark import build_parser as bench_parser, render_markdown, run_benchmark

    data, _ = _train(tmp_path, steps=1)
    argv = ["--checkpoint", str(tmp_path / "out"), "--data", str(data), "--examples", "8", "--batch-size", "4",
            "--device", "cpu"]
    full = run_benchmark(bench_parser().parse_args(argv))
    quick = run_benchmark(bench_parser().parse_args(argv + ["--no-routing-stats"]))
    assert "routing" in full and "routing" not in quick
    assert quick["loss"] == full["loss"]
    assert "### Per layer" in render_markdown(full) and "### Per layer" not in render_markdown(quick)


def test_the_sampler_runs_from_character_and_bpe_checkpoints(tmp_path, capsys):
    from test_tools_cpu import _train

    from quantaweave_b200.tools.generate import main as generate

    _train(tmp_path / "char", steps=1)
    _train(tmp_path / "bpe", steps=1, tokenizer="bpe", tokenizer_path=tmp_path / "tok", vocab_size=300)
    capsys.readouterr()  # drop the training logs
    for name in ("char", "bpe"):
        torch.manual_seed(0)
        generate(["--checkpoint", str(tmp_path / name / "out"), "--prompt", "the cat", "--tokens", "6",
                  "--device", "cpu", "--temperature", "0.8"])
        text = capsys.readouterr().out
        assert text.startswith("the cat") and len(text.strip()) > len("the cat"), (name, text)
