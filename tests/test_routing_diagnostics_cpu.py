"""Routing diagnostics (reference tests: tests/test_schedules_and_diagnostics.py): the monitor needs collected
stats, accumulates loads/drops/classes/domains over a window, snapshots the reference keys into routing_log.jsonl,
and writes SVG pages plus an index."""

import json

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.data.pipeline import CharTokenizer, token_classes
from quantaweave_b200.utils.routing_diagnostics import RoutingMonitor, bar_chart_svg, heatmap_svg, line_chart_svg


def _model(cf=0.5):
    cfg = QuantaWeaveConfig(vocab_size=40, hidden_size=16, layers=2, ffn_size=32, num_experts=4, top_k=2,
                            attention_heads=2, max_sequence_length=17, capacity_factor=cf)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(cfg).eval()
    model.set_moe_kernel("loop")
    return model


def test_monitor_requires_collected_stats():
    model = _model()
    monitor = RoutingMonitor(2, 4, 2)
    ids = torch.randint(0, 40, (2, 9))
    model(ids)
    with pytest.raises(RuntimeError):
        monitor.update(model, ids)


def test_monitor_window_snapshot_log_and_report(tmp_path):
    model = _model()
    model.set_collect_stats(True)
    tok = CharTokenizer.build(["abc def 123 !?"], 40)
    monitor = RoutingMonitor(2, 4, 2, domains=["a", "b"], token_classes=token_classes(tok), out_dir=tmp_path)
    gen = torch.Generator().manual_seed(1)
    for step in range(3):
        ids = torch.randint(0, tok.vocab_size, (2, 9), generator=gen)
        with torch.no_grad():
            model(ids)
        monitor.update(model, ids, domain_ids=torch.tensor([0, 1]))
    assert monitor.imbalance() is not None and 0 <= monitor.active_fraction() <= 1
    record = monitor.snapshot(3)
    assert record["step"] == 3 and len(record["layers"]) == 2
    layer = record["layers"][0]
    assert abs(sum(layer["requested_share"]) - 1) < 1e-6 and 0 <= layer["drop_rate"] < 1
    assert sum(layer["drops_by_expert"]) > 0  # capacity factor 0.5 drops routes
    assert set(layer) >= {"utilization", "entropy", "entropy_max", "confidence", "confidence_hist", "dead_experts"}
    assert sum(record["drops_by_token_class"].values()) > 0
    assert monitor.snapshot(4) == {}  # the window was reset
    logged = [json.loads(line) for line in (tmp_path / "routing_log.jsonl").read_text().splitlines()]
    assert len(logged) == 1 and logged[0]["step"] == 3
    monitor.record_device_utilization(torch.rand(2, 2, 4))
    index = monitor.write_report()
    pages = {p.name for p in tmp_path.glob("*.svg")}
    assert {"expert_usage_by_layer.svg", "drop_rate_over_time.svg", "router_entropy_over_time.svg",
            "specialization_layer0.svg", "domain_usage_layer0.svg", "device_utilization_layer0.svg",
            "routed_tokens_by_device.svg"} <= pages
    html = index.read_text()
    assert all(p in html for p in pages)


def test_svg_helpers_render_valid_markup():
    for svg in (heatmap_svg([[0.1, 0.9], [0.5, 0.5]], ["r0", "r1"], ["c0", "c1"], "t"),
                line_chart_svg([1, 2, 3], {"a": [0.1, 0.2, 0.3]}, "t"),
                bar_chart_svg({"x": 1.0, "y": 2.0}, "t")):
        assert svg.startswith("<svg") and svg.rstrip().endswith("</svg>")
    assert bar_chart_svg({"x": 1.0, "y": 2.0, "z": 3.0}, "t").count("<rect") >= 3


def test_window_imbalance_and_active_fraction_values():
    monitor = RoutingMonitor(2, 2, 1)
    monitor.window_updates = 1
    monitor.window_assigned = torch.tensor([[5, 5], [30, 10]])
    # layer 0 is even (0); layer 1 has shares 0.75 / 0.25: spread 0.25 over a mean share of 0.5 -> 0.5
    assert monitor.imbalance() == pytest.approx(0.25)
    monitor.window_assigned = torch.tensor([[100, 0], [95, 5]])
    # an even share is 0.5; at floor 0.1 an expert needs 5 % of the routes: 3 of the 4 (layer, expert) pairs
    assert monitor.active_fraction(0.1) == pytest.approx(0.75)
