"""Router observability: windowed per-layer expert load, entropy, confidence, drops and specialisation.

Behavioural parity with the reference ``src/routing_diagnostics.py`` (``RoutingMonitor`` :18-220, snapshot record
:131-164, ``write_report`` :178-220, SVG helpers :223-304): the same snapshot keys in ``routing_log.jsonl`` and the
same report pages (usage heatmap, per-device heatmaps, class/domain specialisation, drop rate / entropy / utilisation
over time) linked from ``index.html``.

B200 design: the window is accumulated on the device the router ran on (no host sync per update); tensors reach the
host only when a snapshot, a window metric or the report is asked for.
"""

from __future__ import annotations

import html
import json
import math
from pathlib import Path
from typing import Optional, Sequence

import torch
from torch import Tensor


class RoutingMonitor:
    def __init__(self, num_layers: int, num_experts: int, top_k: int, domains: Sequence[str] = ("default",),
                 token_classes: Optional[tuple[Tensor, list[str]]] = None, out_dir: Optional[Path] = None) -> None:
        self.num_layers, self.num_experts, self.top_k = num_layers, num_experts, top_k
        self.domains = list(domains)
        if isinstance(token_classes, dict):  # {class name: [token ids]} is accepted too
            token_classes = _class_table(token_classes) if token_classes else None
        self.token_classes = token_classes if token_classes is not None and len(token_classes[1]) else None
        self.out_dir = Path(out_dir) if out_dir is not None else None
        if self.out_dir is not None:
            self.out_dir.mkdir(parents=True, exist_ok=True)
        self.snapshots: list[dict] = []
        self.device: Optional[torch.device] = None
        self.device_load: Optional[Tensor] = None  # [world, layers, experts] from DeviceLoadTracker
        self._class_ids: Optional[Tensor] = None
        self._alloc(torch.device("cpu"))

    # ---- accumulation ---------------------------------------------------------------------------
    def _alloc(self, device: torch.device) -> None:
        L, E = self.num_layers, self.num_experts
        C = len(self.token_classes[1]) if self.token_classes else 0
        z = lambda *shape, dtype=torch.long: torch.zeros(*shape, dtype=dtype, device=device)  # noqa: E731
        self.device = device
        self.class_usage = z(L, C, E)
        self.domain_usage = z(L, len(self.domains), E)
        self.total_load = z(L, E)
        self._class_drops = z(max(C, 1))
        self._reset_window()

    def _reset_window(self) -> None:
        L, E, dev = self.num_layers, self.num_experts, self.device
        self.window_assigned = torch.zeros(L, E, dtype=torch.long, device=dev)
        self.window_load = torch.zeros(L, E, dtype=torch.long, device=dev)
        self.window_entropy = torch.zeros(L, device=dev)
        self.window_confidence = torch.zeros(L, device=dev)
        self.window_confidence_hist = torch.zeros(L, 10, device=dev)
        self.window_drops_by_expert = torch.zeros(L, E, dtype=torch.long, device=dev)
        self._class_drops = torch.zeros_like(self._class_drops)
        self.window_updates = 0

    def _move(self, device: torch.device) -> None:
        for name in ("class_usage", "domain_usage", "total_load", "_class_drops", "window_assigned", "window_load",
                     "window_entropy", "window_confidence", "window_confidence_hist", "window_drops_by_expert"):
            setattr(self, name, getattr(self, name).to(device))
        self.device = device

    @property
    def window_drops_by_class(self) -> dict[str, int]:
        if not self.token_classes:
            return {}
        counts = self._class_drops.cpu().tolist()
        return {name: c for name, c in zip(self.token_classes[1], counts) if c}

    @torch.no_grad()
    def update(self, model, input_ids: Tensor, domain_ids: Optional[Tensor] = None) -> None:
        """Fold in the routing statistics of the forward pass that just ran on ``input_ids``."""
        stats_per_layer = model.routing_stats()
        if not all(stats_per_layer):
            raise RuntimeError("model has no routing stats; call model.set_collect_stats(True) before the forward pass")
        dev = stats_per_layer[0]["expert_load"].device
        if dev != self.device:
            self._move(dev)
        E, k = self.num_experts, self.top_k
        tokens = input_ids.reshape(-1).to(dev)
        classes = None
        if self.token_classes:
            if self._class_ids is None or self._class_ids.device != dev:
                self._class_ids = self.token_classes[0].to(dev)
            classes = self._class_ids[tokens.clamp(max=self._class_ids.numel() - 1)]
        token_domains = None
        if domain_ids is not None:
            token_domains = domain_ids.to(dev).repeat_interleave(input_ids.size(-1))
        for layer, (stats, moe) in enumerate(zip(stats_per_layer, model.moes())):
            self.window_assigned[layer] += stats["expert_assigned"].to(dev)
            self.window_load[layer] += stats["expert_load"].to(dev)
            self.total_load[layer] += stats["expert_load"].to(dev)
            self.window_entropy[layer] += stats["entropy_mean"].float()
            self.window_confidence[layer] += stats["confidence_mean"].float()
            self.window_confidence_hist[layer] += stats["confidence_hist"].float()
            dropped_tokens, dropped_experts = stats["dropped_tokens"], stats["dropped_experts"]
            if dropped_experts.numel():
                self.window_drops_by_expert[layer].index_add_(0, dropped_experts.to(dev).long(),
                                                              torch.ones_like(dropped_experts, dtype=torch.long,
                                                                              device=dev))
                if classes is not None:
                    self._class_drops.index_add_(0, classes[dropped_tokens.to(dev).long()],
                                                 torch.ones(dropped_tokens.numel(), dtype=torch.long, device=dev))
            experts = moe.last_top_indices.reshape(-1).to(dev).long()
            ones = torch.ones_like(experts)
            if classes is not None:
                flat = self.class_usage[layer].view(-1)
                flat.index_add_(0, classes.repeat_interleave(k) * E + experts, ones)
            if token_domains is not None:
                flat = self.domain_usage[layer].view(-1)
                flat.index_add_(0, token_domains.long().repeat_interleave(k) * E + experts, ones)
        self.window_updates += 1

    # ---- window metrics ---------------------------------------------------------------------------
    def _window_shares(self) -> Optional[Tensor]:
        """Each expert's share of the routes its layer's router asked for in this window: ``[layers, experts]``,
        rows summing to 1 (None before any update)."""
        if not self.window_updates:
            return None
        wanted = self.window_assigned.double()
        return wanted / wanted.sum(dim=1, keepdim=True).clamp(min=1)

    def imbalance(self) -> Optional[float]:
        """How unevenly routes are spread, averaged over layers: the spread (population standard deviation) of the
        experts' shares relative to the mean share; 0 when every expert gets as many routes as the others."""
        shares = self._window_shares()
        if shares is None:
            return None
        mean = shares.mean(dim=1, keepdim=True)
        spread = (shares - mean).square().mean(dim=1).sqrt()
        return float((spread / mean.squeeze(1).clamp(min=1e-9)).mean())

    def active_fraction(self, floor: float = 0.1) -> Optional[float]:
        """Fraction of (layer, expert) pairs whose share of the routes is at least ``floor`` times the share every
        expert would get under perfectly even routing."""
        shares = self._window_shares()
        if shares is None:
            return None
        return float((shares * self.num_experts >= floor).double().mean())

    def snapshot(self, step: int, reset: bool = True) -> dict:
        """Summarise the window per layer, append it to ``snapshots`` (and to routing_log.jsonl), then start a new
        window unless ``reset`` is False."""
        if not self.window_updates:
            return {}
        windows = self.window_updates
        wanted = self.window_assigned.double().cpu()
        served = self.window_load.double().cpu()
        routes = wanted.sum(dim=1).clamp(min=1)
        per_layer = zip(served / served.sum(dim=1, keepdim=True).clamp(min=1), wanted / routes[:, None],
                        (self.window_entropy / windows).cpu().tolist(), (self.window_confidence / windows).cpu().tolist(),
                        (self.window_confidence_hist / windows).cpu().tolist(), 1 - served.sum(dim=1) / routes,
                        self.window_drops_by_expert.cpu().tolist(), (wanted == 0).sum(dim=1).tolist())
        ceiling = math.log(self.num_experts)
        layers = [{"utilization": used.tolist(), "requested_share": asked.tolist(), "entropy": entropy,
                   "entropy_max": ceiling, "confidence": confidence, "confidence_hist": histogram,
                   "drop_rate": float(dropped), "drops_by_expert": drops, "dead_experts": int(dead)}
                  for used, asked, entropy, confidence, histogram, dropped, drops, dead in per_layer]
        record = {"step": step, "layers": layers, "imbalance": self.imbalance(),
                  "active_fraction": self.active_fraction(), "drops_by_token_class": self.window_drops_by_class}
        self.snapshots.append(record)
        if self.out_dir is not None:
            with (self.out_dir / "routing_log.jsonl").open("a") as fh:
                fh.write(json.dumps(record) + "\n")
        if reset:
            self._reset_window()
        return record

    def record_device_utilization(self, per_device: Tensor) -> None:
        """Accumulate a ``[world, layers, experts]`` tensor (``DeviceLoadTracker.gather_expert_utilization``): how the
        global expert distribution of each device's own data differs across devices."""
        per_device = per_device.detach().double().cpu()
        self.device_load = per_device.clone() if self.device_load is None else self.device_load + per_device

    # ---- report ----------------------------------------------------------------------------------
    def write_report(self, out_dir: Optional[Path] = None) -> Path:
        """Render heatmaps and time series as SVG plus an ``index.html``; returns the index path."""
        out_dir = Path(out_dir) if out_dir is not None else self.out_dir
        if out_dir is None:
            raise ValueError("no output directory configured")
        out_dir.mkdir(parents=True, exist_ok=True)
        pages: list[str] = []

        def save(name: str, svg: str) -> None:
            (out_dir / name).write_text(svg)
            pages.append(name)

        experts = [str(e) for e in range(self.num_experts)]
        layer_names = [f"layer {i}" for i in range(self.num_layers)]
        total = self.total_load.double().cpu()
        if total.sum() > 0:
            share = total / total.sum(dim=1, keepdim=True).clamp(min=1)
            save("expert_usage_by_layer.svg",
                 heatmap_svg(share.tolist(), layer_names, experts, "Expert usage share by layer (whole run)"))
        if self.device_load is not None and self.device_load.sum() > 0:
            world = self.device_load.shape[0]
            devices = [f"device {r}" for r in range(world)]
            for layer in range(self.device_load.shape[1]):
                per = self.device_load[:, layer]
                share = per / per.sum(dim=1, keepdim=True).clamp(min=1)
                save(f"device_utilization_layer{layer}.svg",
                     heatmap_svg(share.tolist(), devices, [f"expert {e}" for e in range(per.shape[1])],
                                 f"Layer {layer}: global expert distribution of each device's own data"))
            save("routed_tokens_by_device.svg",
                 bar_chart_svg(dict(zip(devices, self.device_load.sum(dim=(1, 2)).tolist())),
                               "Routed tokens by device (whole run)"))
        if self.token_classes and self.class_usage.sum() > 0:
            usage_all = self.class_usage.double().cpu()
            for layer in range(self.num_layers):
                usage = usage_all[layer] / usage_all[layer].sum(dim=1, keepdim=True).clamp(min=1)
                save(f"specialization_layer{layer}.svg",
                     heatmap_svg(usage.tolist(), self.token_classes[1], experts,
                                 f"Layer {layer}: expert share per token class"))
        if len(self.domains) > 1 and self.domain_usage.sum() > 0:
            usage_all = self.domain_usage.double().cpu()
            for layer in range(self.num_layers):
                usage = usage_all[layer] / usage_all[layer].sum(dim=1, keepdim=True).clamp(min=1)
                save(f"domain_usage_layer{layer}.svg",
                     heatmap_svg(usage.tolist(), self.domains, experts, f"Layer {layer}: expert share per domain"))
        if self.snapshots:
            steps = [s["step"] for s in self.snapshots]
            per_layer = lambda key: {f"layer {i}": [s["layers"][i][key] for s in self.snapshots]  # noqa: E731
                                     for i in range(self.num_layers)}
            save("drop_rate_over_time.svg", line_chart_svg(steps, per_layer("drop_rate"), "Token drop rate over time"))
            save("router_entropy_over_time.svg",
                 line_chart_svg(steps, per_layer("entropy"),
                                f"Router entropy over time (max {math.log(self.num_experts):.2f} nats)"))
            for layer in range(self.num_layers):
                save(f"utilization_layer{layer}_over_time.svg",
                     heatmap_svg([s["layers"][layer]["utilization"] for s in self.snapshots],
                                 [f"step {s}" for s in steps], experts,
                                 f"Layer {layer}: per-expert utilization over time"))
        body = "".join(f'<h2>{html.escape(p)}</h2><img src="{html.escape(p)}" alt="{html.escape(p)}">' for p in pages)
        index = out_dir / "index.html"
        index.write_text("<!doctype html><meta charset='utf-8'><title>Routing diagnostics</title>"
                         "<style>body{font:14px sans-serif;margin:24px;max-width:1100px}img{max-width:100%}</style>"
                         f"<h1>Routing diagnostics</h1>{body or '<p>No routing data recorded.</p>'}")
        return index


def _class_table(classes: dict[str, list[int]]) -> tuple[Tensor, list[str]]:
    names = list(classes)
    size = 1 + max((max(ids) for ids in classes.values() if ids), default=0)
    table = torch.zeros(size, dtype=torch.long)
    for index, name in enumerate(names):
        table[torch.tensor(classes[name], dtype=torch.long)] = index
    return table, names


# ---- dependency-free SVG ---------------------------------------------------------------------------
def _blue(value: float) -> str:
    """Sequential white -> dark blue colour for ``value`` in [0, 1]."""
    v = min(1.0, max(0.0, value))
    lo, hi = (247, 251, 255), (8, 48, 107)
    return "rgb({},{},{})".format(*(round(a + (b - a) * v) for a, b in zip(lo, hi)))


def _svg(width: float, height: float, title: str, items: list[str]) -> str:
    head = (f'<svg xmlns="http://www.w3.org/2000/svg" width="{width:.0f}" height="{height:.0f}" '
            f'font-family="sans-serif" font-size="11">')
    caption = f'<text x="10" y="20" font-size="14" font-weight="bold">{html.escape(title)}</text>'
    return head + caption + "".join(items) + "</svg>"


def heatmap_svg(matrix: Sequence[Sequence[float]], row_labels: Sequence[str], col_labels: Sequence[str],
                title: str) -> str:
    """Rows x columns grid, each cell shaded by value / max and carrying a tooltip."""
    rows = len(matrix)
    cols = len(matrix[0]) if rows else 0
    cell = max(4, min(28, 900 // max(cols, 1)))
    x0, y0 = 96, 40
    peak = max((max(r) for r in matrix if len(r)), default=0.0) or 1.0
    items = []
    for r, row in enumerate(matrix):
        label = html.escape(str(row_labels[r]))
        items.append(f'<text x="{x0 - 6}" y="{y0 + r * cell + 0.7 * cell:.1f}" text-anchor="end">{label}</text>')
        for c, v in enumerate(row):
            items.append(f'<rect x="{x0 + c * cell}" y="{y0 + r * cell}" width="{cell}" height="{cell}" '
                         f'fill="{_blue(v / peak)}"><title>{label} / expert {html.escape(str(col_labels[c]))}: '
                         f'{v:.4f}</title></rect>')
    every = max(1, cols // 16)
    for c in range(0, cols, every):
        items.append(f'<text x="{x0 + (c + 0.5) * cell:.1f}" y="{y0 + rows * cell + 14}" text-anchor="middle">'
                     f'{html.escape(str(col_labels[c]))}</text>')
    return _svg(x0 + cols * cell + 20, y0 + rows * cell + 30, title, items)


_PALETTE = ("#1f77b4", "#d62728", "#2ca02c", "#9467bd", "#ff7f0e", "#17becf", "#8c564b", "#e377c2")


def line_chart_svg(x: Sequence[float], series: dict[str, Sequence[float]], title: str) -> str:
    """One polyline per series over shared x values, min/max axis labels and a legend."""
    W, H, x0, y0, pad = 720, 300, 60, 40, 30
    ys = [v for line in series.values() for v in line]
    lo, hi = (min(ys), max(ys)) if ys else (0.0, 1.0)
    hi = hi if hi != lo else lo + 1.0
    xl, xh = (min(x), max(x)) if len(x) else (0, 1)
    xh = xh if xh != xl else xl + 1
    px = lambda v: x0 + (v - xl) / (xh - xl) * (W - x0 - 10)  # noqa: E731
    py = lambda v: H - pad - (v - lo) / (hi - lo) * (H - pad - y0)  # noqa: E731
    items = [f'<line x1="{x0}" y1="{y0}" x2="{x0}" y2="{H - pad}" stroke="#888"/>',
             f'<line x1="{x0}" y1="{H - pad}" x2="{W - 10}" y2="{H - pad}" stroke="#888"/>',
             f'<text x="{x0 - 6}" y="{y0 + 4}" text-anchor="end">{hi:.3g}</text>',
             f'<text x="{x0 - 6}" y="{H - pad}" text-anchor="end">{lo:.3g}</text>',
             f'<text x="{x0}" y="{H - 8}">{xl}</text>',
             f'<text x="{W - 10}" y="{H - 8}" text-anchor="end">{xh}</text>']
    for i, (name, line) in enumerate(series.items()):
        colour = _PALETTE[i % len(_PALETTE)]
        pts = " ".join(f"{px(a):.1f},{py(b):.1f}" for a, b in zip(x, line))
        items.append(f'<polyline fill="none" stroke="{colour}" stroke-width="1.5" points="{pts}"/>')
        items.append(f'<text x="{W - 100}" y="{y0 + 12 * i}" fill="{colour}">{html.escape(name)}</text>')
    return _svg(W, H, title, items)


def bar_chart_svg(values: dict[str, float], title: str) -> str:
    """Horizontal bars scaled to the largest value, labelled with name and value."""
    W, x0, y0, bar, gap = 720, 140, 40, 18, 6
    peak = max(values.values(), default=0.0) or 1.0
    items = []
    for i, (name, v) in enumerate(values.items()):
        y = y0 + i * (bar + gap)
        width = v / peak * (W - x0 - 80)
        items.append(f'<text x="{x0 - 6}" y="{y + 0.75 * bar:.1f}" text-anchor="end">{html.escape(name)}</text>')
        items.append(f'<rect x="{x0}" y="{y}" width="{width:.1f}" height="{bar}" fill="#1f77b4">'
                     f'<title>{html.escape(name)}: {v:.4g}</title></rect>')
        items.append(f'<text x="{x0 + width + 6:.1f}" y="{y + 0.75 * bar:.1f}">{v:.4g}</text>')
    return _svg(W, y0 + 20 + len(values) * (bar + gap), title, items)
