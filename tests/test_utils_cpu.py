"""Utilities on CPU (reference tests: tests/test_future_features.py, tests/test_deploy_and_distill.py,
tests/test_production_readiness.py, tests/test_schedules_and_diagnostics.py): CPU-offload AdamW, energy/cost
accounting, the metrics logger and plateau detection, weight-only quantisation, the server's rate limiter and
moderation, and the quantised model's state round trip."""

import json
import time

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.inference.quantization import (QuantizedLinear, dequantize_tensor, quantize_model,
                                                     quantize_tensor)
from quantaweave_b200.optim.cpu_offload import CPUOffloadAdamW
from quantaweave_b200.training.metrics import MetricsLogger, detect_plateau, first_stable_step
from quantaweave_b200.utils.energy import PowerCostTracker


def test_cpu_offload_adamw_matches_torch_adamw_step_for_step_and_round_trips():
    torch.manual_seed(0)
    a = torch.nn.Linear(8, 4)
    b = torch.nn.Linear(8, 4)
    b.load_state_dict(a.state_dict())
    ours = CPUOffloadAdamW(a.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ref = torch.optim.AdamW(b.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for step in range(5):
        x = torch.randn(16, 8, generator=torch.Generator().manual_seed(step))
        for model, opt in ((a, ours), (b, ref)):
            opt.zero_grad()
            model(x).pow(2).mean().backward()
            opt.step()
    for p, q in zip(a.parameters(), b.parameters()):
        assert torch.allclose(p, q, atol=1e-6)
    assert ours.state_numel() == 2 * sum(p.numel() for p in a.parameters())  # both moments, on the host
    frozen = torch.nn.Linear(4, 4)
    frozen.bias.requires_grad_(False)
    assert len(CPUOffloadAdamW(parameters=frozen.parameters()).param_groups[0]["params"]) == 1  # trainable only
    again = CPUOffloadAdamW(a.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    again.load_state_dict(ours.state_dict())
    assert json.dumps(again.state_dict(), default=str) == json.dumps(ours.state_dict(), default=str)


def test_power_cost_tracker_integrates_energy_and_resumes(tmp_path):
    counter = {"uj": 0}

    def reader():
        counter["uj"] += 3_600_000_000  # 1 Wh per read, in microjoules
        return counter["uj"]

    tracker = PowerCostTracker(0.25, reader=reader)
    assert tracker.available
    time.sleep(0.01)
    first = tracker.sample()
    second = tracker.sample()
    assert first["energy_kwh_cumulative"] == pytest.approx(0.001)
    assert second["energy_kwh_cumulative"] == pytest.approx(0.002)
    assert second["cost_usd_cumulative"] == pytest.approx(0.002 * 0.25) and second["gpu_power_watts"] > 0
    log = tmp_path / "metrics.jsonl"
    log.write_text(json.dumps({"step": 1, "energy_kwh_cumulative": 1.5}) + "\n")
    resumed = PowerCostTracker(None, resume_from=log, reader=reader)
    assert resumed.energy_kwh == pytest.approx(1.5)
    assert PowerCostTracker(None, reader=lambda: None).sample() == {}


def test_metrics_logger_writes_jsonl_and_summarises_and_plateau_detection(tmp_path):
    path = tmp_path / "m.jsonl"
    logger = MetricsLogger(path, total_parameters=100, active_parameters=25)
    for step in range(1, 31):
        logger.log(step, 64, loss=5.0 / step + 1.0)
    lines = [json.loads(l) for l in path.read_text().splitlines()]
    assert len(lines) == 30 and lines[0]["step"] == 1 and "loss" in lines[0]
    summary = logger.summary()
    assert summary["steps_logged"] == 30 and summary["active_parameter_ratio"] == 0.25
    assert summary["best_loss"] == pytest.approx(5.0 / 30 + 1.0)
    assert detect_plateau([1.0] * 40) and not detect_plateau([float(40 - i) for i in range(40)])
    settling = [10.0 / (i + 1) + 1 for i in range(20)] + [1.0] * 60  # falls for 20 steps, then flat
    assert first_stable_step(list(range(80)), settling) == 20
    assert first_stable_step(list(range(10)), [1.0] * 10) is None  # too short to judge


def test_int4_packing_is_lossless_for_representable_weights_and_int8_is_close():
    scales = torch.tensor([[0.5], [0.25]])
    ints = torch.randint(-7, 8, (2, 64), generator=torch.Generator().manual_seed(1)).float()
    ints[:, 0] = 7  # symmetric codes: the group's largest magnitude (7 units) sets the scale absmax / 7
    weight = ints * scales
    q, s = quantize_tensor(weight, 4, 64)
    assert q.dtype == torch.uint8 and q.shape == (2, 32)  # two values per byte
    assert torch.equal(dequantize_tensor(q, s, 4, 64, 64), weight)
    w8 = torch.randn(16, 48)
    q8, s8 = quantize_tensor(w8, 8, 48)
    rel = (dequantize_tensor(q8, s8, 8, 48, 48) - w8).norm() / w8.norm()
    assert rel < 0.02
    layer = torch.nn.Linear(64, 16, bias=False)
    ql = QuantizedLinear.from_linear(layer, 4, 16)
    x = torch.randn(4, 64)
    assert ((ql(x) - layer(x)).norm() / layer(x).norm()) < 0.2


def test_quantize_model_shrinks_experts_keeps_router_and_runs():
    cfg = QuantaWeaveConfig(vocab_size=32, hidden_size=32, layers=1, ffn_size=64, num_experts=4, top_k=2,
                            attention_heads=2, capacity_factor=0.0)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg).eval()
    ids = torch.randint(0, 32, (1, 9))
    with torch.no_grad():
        before = model(ids)["logits"]
    router = model.moes()[0].router.weight.detach().clone()
    stats = quantize_model(model, 8)
    assert stats
    with torch.no_grad():
        after = model(ids)["logits"]
    assert torch.equal(model.moes()[0].router.weight, router)
    assert ((after - before).norm() / before.norm()) < 0.05


def test_rate_limiter_window_per_key_and_disabled():
    from quantaweave_b200.tools.serve import Moderation, RateLimiter

    limiter = RateLimiter(2, window=0.05)
    assert limiter.allow("a") and limiter.allow("a") and not limiter.allow("a")
    assert limiter.allow("b")  # per key
    time.sleep(0.06)
    assert limiter.allow("a")  # the window slid
    assert all(RateLimiter(None).allow("x") for _ in range(100))
    assert Moderation(None).blocked("anything at all") is None


def test_rate_limiter_forgets_callers_whose_window_emptied():
    from quantaweave_b200.tools.serve import RateLimiter

    limiter = RateLimiter(1, window=0.02)
    assert all(limiter.allow(f"client-{i}") for i in range(50))
    assert len(limiter.hits) == 50 and not limiter.allow("client-0")
    time.sleep(0.03)
    assert limiter.allow("client-0")  # its old call expired, so it is admitted again
    assert len(limiter.hits["client-0"]) == 1
    assert all(limiter.allow(f"client-{i}") for i in range(1, 50))
    limiter.limit = 0  # refuse everything: a caller with no admitted call in the window leaves no entry behind
    time.sleep(0.03)
    assert not limiter.allow("client-7") and "client-7" not in limiter.hits
