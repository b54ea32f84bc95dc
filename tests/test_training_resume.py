"""benchmark configuration 1: CPU fp32 tiny MoE (RoPE + RMSNorm), 20 AdamW steps (lr 3e-4, betas 0.9/0.95, wd 0.1),
checkpoint at step 10, resume, and compare weights/loss/routing bit-exactly against an uninterrupted run."""

import json
from pathlib import Path

import torch

from quantaweave_b200.training.trainer import default_args, load_checkpoint, run_training
from quantaweave_b200.utils.checkpoint_io import load_checkpoint as load_file


def _args(tmp: Path, name: str, steps: int, **extra):
    options = dict(preset="tiny-cpu", synthetic_data="uniform", vocab_size=512, sequence_length=128, batch_size=8,
                   steps=steps, lr=3e-4, adam_beta1=0.9, adam_beta2=0.95, weight_decay=0.1, device="cpu",
                   seed=0, no_power_tracking=True, output=tmp / name / "out",
                   checkpoint_dir=tmp / name / "ckpt", checkpoint_interval=10,
                   metrics_file=tmp / name / "metrics.jsonl")
    options.update(extra)
    return default_args(**options)


def _metrics(path: Path) -> list[dict]:
    return [json.loads(line) for line in path.read_text().splitlines()]


def test_exact_resume_config1(tmp_path):
    straight = run_training(_args(tmp_path, "straight", 20))
    # interrupted run: stop at 10 (checkpoint written at step 10), then resume to 20 in a new call
    run_training(_args(tmp_path, "split", 10))
    resumed = run_training(_args(tmp_path, "split", 20))
    assert straight["steps"] == resumed["steps"] == 20
    a = load_file(tmp_path / "straight" / "out" / "model.pt")
    b = load_file(tmp_path / "split" / "out" / "model.pt")
    assert a.keys() == b.keys()
    for key in a["model"]:
        assert torch.equal(a["model"][key], b["model"][key]), key
    m1 = _metrics(tmp_path / "straight" / "metrics.jsonl")
    m2 = _metrics(tmp_path / "split" / "metrics.jsonl")
    tail1 = {r["step"]: r for r in m1 if r["step"] > 10}
    tail2 = {r["step"]: r for r in m2 if r["step"] > 10}
    assert tail1.keys() == tail2.keys()
    for step in tail1:
        for key in ("loss", "router_aux", "dropped_routes", "overflow_routes", "grad_norm"):
            assert tail1[step][key] == tail2[step][key], (step, key)


def test_resume_refuses_changed_config(tmp_path):
    run_training(_args(tmp_path, "run", 2, checkpoint_interval=2))
    import pytest

    with pytest.raises(ValueError, match="different run configuration"):
        run_training(_args(tmp_path, "run", 4, checkpoint_interval=2, lr=1e-3, batch_size=4))


def test_interrupted_save_falls_back_to_previous(tmp_path):
    run_training(_args(tmp_path, "crash", 2, checkpoint_interval=2))
    ckpt = tmp_path / "crash" / "ckpt"
    # simulate a crash between the two renames of the atomic save: only ".ckpt.previous" exists
    ckpt.rename(ckpt.with_name(".ckpt.previous"))
    from quantaweave_b200 import QuantaWeaveMoEForCausalLM, preset

    model = QuantaWeaveMoEForCausalLM(preset("tiny-cpu", max_sequence_length=129))
    opt = torch.optim.AdamW(model.parameters())
    assert load_checkpoint(ckpt, model, opt, torch.device("cpu")) == 2
