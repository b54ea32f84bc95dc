"""Open-loop schedules and closed-loop controllers (reference tests: tests/test_schedules_and_diagnostics.py)."""

import math

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.training.schedules import ScheduleConfig, TrainingController


def test_lr_warmup_then_cosine_and_linear_decay_to_the_floor():
    c = TrainingController(ScheduleConfig(lr=1.0, total_steps=110, warmup_steps=10, lr_decay="cosine",
                                          min_lr_ratio=0.1))
    assert c.lr_at(0) == pytest.approx(0.1) and c.lr_at(9) == pytest.approx(1.0)
    assert c.lr_at(10) == pytest.approx(1.0)
    assert c.lr_at(60) == pytest.approx(0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * 0.5)))
    assert c.lr_at(110) == pytest.approx(0.1) and c.lr_at(500) == pytest.approx(0.1)
    lin = TrainingController(ScheduleConfig(lr=2.0, total_steps=100, lr_decay="linear", min_lr_ratio=0.5))
    assert lin.lr_at(50) == pytest.approx(2.0 * 0.75) and lin.lr_at(100) == pytest.approx(1.0)
    const = TrainingController(ScheduleConfig(lr=0.3, total_steps=100))
    assert const.lr_at(0) == const.lr_at(99) == pytest.approx(0.3)
    with pytest.raises(ValueError):
        ScheduleConfig(lr_decay="step")


def test_plateau_halves_lr_down_to_its_floor():
    c = TrainingController(ScheduleConfig(lr=1.0, plateau_patience=2, plateau_factor=0.5, min_lr_scale=0.2,
                                          interval=1))
    c.observe(5.0, 0.0)
    c.update(1)  # first interval sets the best loss
    scales = []
    for step in range(2, 12):
        c.observe(5.0, 0.0)  # no improvement
        c.update(step)
        scales.append(c.lr_scale)
    assert scales[1] == 0.5 and min(scales) == pytest.approx(0.2)
    assert c.lr_at(0) == pytest.approx(0.2)


def test_capacity_grows_under_drops_relaxes_without_and_release_switches_enforcement_off():
    c = TrainingController(ScheduleConfig(capacity_factor=1.25, capacity_adapt=True, capacity_up=1.1,
                                          capacity_down=0.9, capacity_min=1.0, capacity_max=2.0, drop_threshold=0.01,
                                          capacity_release_step=5, interval=1))
    c.observe(1.0, 0.2)
    assert c.update(1)["capacity_factor"] == pytest.approx(1.375)
    for _ in range(20):
        c.observe(1.0, 0.5)
        c.update(2)
    assert c.capacity_factor == pytest.approx(2.0)
    c.observe(1.0, 0.0)
    assert c.update(3)["capacity_factor"] == pytest.approx(1.8)
    assert c.update(5).get("capacity_released") == 1.0 and c.released
    c.observe(1.0, 0.9)
    assert "capacity_factor" not in c.update(6)  # released: capacity no longer adapts


def test_aux_weight_tracks_imbalance_and_anneals_and_temperature_boosts_when_experts_idle():
    c = TrainingController(ScheduleConfig(aux_coef=0.01, aux_coef_end=0.03, total_steps=100, aux_adapt=True,
                                          aux_up=2.0, aux_down=0.5, aux_factor_max=4.0, balance_high=1.0,
                                          balance_low=0.25, temperature_adapt=True, dead_expert_fraction=0.5,
                                          temperature_start=2.0, temperature_end=1.0, temperature_steps=100,
                                          interval=1), base_temperature=1.0)
    assert c.aux_coef_at(50) == pytest.approx(0.02)
    c.update(1, imbalance=2.0, active_fraction=0.2)
    assert c.aux_factor == 2.0 and c.temperature_boost == pytest.approx(1.05)
    c.update(2, imbalance=0.1, active_fraction=0.9)
    assert c.aux_factor == 1.0 and c.temperature_boost == pytest.approx(1.05 * 0.98)
    assert c.temperature_at(50) == pytest.approx(1.5 * c.temperature_boost)


def test_controller_state_roundtrip_and_apply_to_model():
    cfg = ScheduleConfig(lr=0.5, plateau_patience=1, capacity_adapt=True, interval=1)
    c = TrainingController(cfg)
    c.observe(3.0, 0.5)
    c.update(1)
    c.observe(3.0, 0.5)
    c.update(2)
    d = TrainingController(cfg)
    d.load_state_dict(c.state_dict())
    assert d.state_dict() == c.state_dict()
    model = QuantaWeaveMoEForCausalLM(QuantaWeaveConfig(vocab_size=16, hidden_size=16, layers=1, ffn_size=16,
                                                        num_experts=2, top_k=1, attention_heads=2))
    opt = torch.optim.SGD(model.parameters(), lr=1.0)
    applied = d.apply(model, opt, 3)
    assert opt.param_groups[0]["lr"] == pytest.approx(applied["lr"]) == pytest.approx(0.5 * d.lr_scale)
    assert model.moes()[0].capacity_factor == pytest.approx(d.capacity_factor)
