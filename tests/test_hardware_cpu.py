"""Batch-size probe and recommendation on CPU with faked memory and clocks (reference tests: tests/test_autotune.py):
the probe stops at the headroom limit, recommends the knee of the throughput curve, holds the optimizer's state while
it measures and leaves the weights alone, ends at an out-of-memory error but propagates any other, and the
recommendation picks activation checkpointing only when it is measurably faster or the plain model does not fit."""

import json
from collections import Counter

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.utils import hardware as hw

CPU = torch.device("cpu")
GB = 10 ** 9


def _model():
    torch.manual_seed(0)
    return QuantaWeaveMoEForCausalLM(QuantaWeaveConfig(vocab_size=32, hidden_size=16, layers=1, ffn_size=16,
                                                       num_experts=4, top_k=1, attention_heads=2,
                                                       max_sequence_length=9, capacity_factor=0))


class _Recorder:
    """Wraps the model's forward to remember the batch size of the step being probed."""

    def __init__(self, model, fail_from=None, error=None):
        self.batch = 0
        forward = model.forward

        def wrapped(ids, *args, **kwargs):
            self.batch = ids.size(0)
            if fail_from is not None and self.batch >= fail_from:
                raise error
            return forward(ids, *args, **kwargs)

        model.forward = wrapped


class _Clock:
    """A clock read twice per timed region; the second read advances by the time ``tokens_per_second`` implies."""

    def __init__(self, recorder, tokens_per_second, sequence_length=8):
        self.recorder, self.tps, self.seq, self.t, self.reads = recorder, tokens_per_second, sequence_length, 0.0, 0

    def __call__(self):
        self.reads += 1
        if self.reads % 2 == 0:
            b = self.recorder.batch
            self.t += b * self.seq / self.tps(b)
        return self.t


def test_the_probe_stops_at_the_headroom_limit():
    model = _model()
    rec = _Recorder(model)
    result = hw.find_safe_batch_size(model, CPU, 8, limit=256, target=0, total_memory=10 * GB,
                                     peak_fn=lambda: int(0.2 * GB * rec.batch))
    # 85 % of 10 GB: batch 32 peaks at 6.4 GB and is safe, batch 64 at 12.8 GB is not
    assert result["batch_size"] == result["recommended_batch_size"] == 32
    assert [p["batch_size"] for p in result["curve"]] == [1, 2, 4, 8, 16, 32]


def test_the_probe_recommends_the_knee_not_the_largest_batch():
    speed = {1: 1e3, 2: 2e3, 4: 4e3, 8: 8e3, 16: 16e3, 32: 16.2e3, 64: 15e3}
    for target, expected in ((0.95, 16), (0.0, 64)):
        model = _model()
        rec = _Recorder(model)
        result = hw.find_safe_batch_size(model, CPU, 8, limit=64, target=target, total_memory=100 * GB,
                                         peak_fn=lambda: 0, clock=_Clock(rec, lambda b: speed[b]))
        assert result["batch_size"] == 64 and result["recommended_batch_size"] == expected
    assert result["curve"][4]["tokens_per_second"] == pytest.approx(16e3)


def test_the_probe_holds_optimizer_state_and_leaves_the_model_as_it_was(monkeypatch):
    model = _model().eval()
    before = {k: v.clone() for k, v in model.state_dict().items()}
    made = []
    zeros_like = torch.zeros_like

    def counting(tensor, *args, **kwargs):
        made.append((tuple(tensor.shape), kwargs.get("dtype")))
        return zeros_like(tensor, *args, **kwargs)

    monkeypatch.setattr(hw.torch, "zeros_like", counting)
    hw.find_safe_batch_size(model, CPU, 8, limit=2)
    monkeypatch.undo()
    held = Counter(shape for shape, dtype in made if dtype == torch.float32)
    for shape, count in Counter(tuple(p.shape) for p in model.parameters() if p.requires_grad).items():
        assert held[shape] >= 2 * count, shape  # both AdamW moments of every trainable parameter
    for key, value in model.state_dict().items():
        assert torch.equal(before[key], value), key
    assert all(p.grad is None for p in model.parameters()) and not model.training


def test_out_of_memory_ends_the_search_and_other_errors_propagate():
    model = _model()
    _Recorder(model, fail_from=8, error=torch.OutOfMemoryError("CUDA out of memory"))
    assert hw.find_safe_batch_size(model, CPU, 8, limit=64, peak_fn=lambda: 0)["batch_size"] == 4
    model = _model()
    _Recorder(model, fail_from=1, error=RuntimeError("shape mismatch"))
    with pytest.raises(RuntimeError, match="shape mismatch"):
        hw.find_safe_batch_size(model, CPU, 8)
    model = _model()
    _Recorder(model, fail_from=1, error=torch.OutOfMemoryError("CUDA out of memory"))
    with pytest.raises(RuntimeError, match="does not fit"):
        hw.find_safe_batch_size(model, CPU, 8)


def _fake_device():
    return hw.DeviceInfo("cpu", "fake", 1, 8 << 30, 8 << 30, True, False, "test")


def test_checkpointing_is_recommended_only_when_measurably_faster(monkeypatch):
    config = _model().config

    def probe(without, with_):
        def fake(model, device, sequence_length, autocast=None, **kwargs):
            on = model.activation_checkpointing
            return {"batch_size": 64 if on else 8, "recommended_batch_size": 64 if on else 8,
                    "tokens_per_second": with_ if on else without, "curve": []}

        monkeypatch.setattr(hw, "find_safe_batch_size", fake)
        return hw.recommend(_fake_device(), config, 8, probe=True)

    slower, barely, faster = probe(100.0, 90.0), probe(100.0, 103.0), probe(100.0, 140.0)
    assert not slower["activation_checkpointing_recommended"] and slower["batch_size"] == 8
    assert not barely["activation_checkpointing_recommended"]  # within 5 %: not worth the recompute
    assert faster["activation_checkpointing_recommended"] and faster["batch_size"] == 64


def test_the_recommendation_survives_a_setting_that_does_not_fit(monkeypatch):
    config = _model().config

    def only_with_checkpointing(model, device, sequence_length, autocast=None, **kwargs):
        if not model.activation_checkpointing:
            raise RuntimeError("even batch size 1 does not fit on cpu")
        return {"batch_size": 2, "recommended_batch_size": 2, "tokens_per_second": 5.0, "curve": []}

    monkeypatch.setattr(hw, "find_safe_batch_size", only_with_checkpointing)
    result = hw.recommend(_fake_device(), config, 8, probe=True)
    assert result["activation_checkpointing_recommended"] and result["batch_size"] == 2

    def never(*args, **kwargs):
        raise RuntimeError("even batch size 1 does not fit on cpu")

    monkeypatch.setattr(hw, "find_safe_batch_size", never)
    with pytest.raises(RuntimeError, match="does not fit"):
        hw.recommend(_fake_device(), config, 8, probe=True)


def test_the_report_without_a_probe_and_the_real_probe_on_cpu():
    config = _model().config
    small = hw.recommend(_fake_device(), config, 8)
    assert small["fits_training_state"] and not small["activation_checkpointing_recommended"]
    assert small["max_sequence_length"] == 8 and small["precision"] == "fp32"
    state = small["training_state_bytes"]
    half = hw.recommend(hw.DeviceInfo("cpu", "fake", 1, state * 2, 0, True, False, "t"), config, 8)
    assert half["fits_training_state"] and half["activation_checkpointing_recommended"]  # state > 40 % of memory
    over = hw.recommend(hw.DeviceInfo("cpu", "fake", 1, state * 11 // 10, 0, True, False, "t"), config, 8)
    assert not over["fits_training_state"]
    real = hw.recommend(hw.detect("cpu"), config, 8, probe=True)
    assert real["batch_size"] >= 1 and real["probe"]["curve"]
    json.dumps(real, default=str)


def test_the_trainer_applies_the_probed_batch_size(tmp_path):
    from quantaweave_b200.training.trainer import default_args, run_training

    data = tmp_path / "d.jsonl"
    data.write_text("".join(json.dumps({"text": f"story {i}: the quick brown fox jumps over the lazy dog."}) + "\n"
                            for i in range(40)))
    args = default_args(data=[data], steps=2, sequence_length=8, hidden_size=16, layers=1, ffn_size=16,
                        total_experts=2, active_experts=1, attention_heads=2, vocab_size=64, device="cpu",
                        checkpoint_interval=0, auto_batch_size=True, auto_batch_target=0, no_archive=True,
                        no_power_tracking=True, output=tmp_path / "o", checkpoint_dir=tmp_path / "c")
    run_training(args)
    assert args.batch_size >= 8  # target 0: the largest batch that fitted (on the host, up to the probe's limit)
