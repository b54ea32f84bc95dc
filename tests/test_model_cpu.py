"""MoE and model semantics on CPU against naive restatements (the reference's model unit tests:
tests/test_quantweave.py, tests/test_model_features.py): the capacity plan keeps the highest-weight routes per
expert, skipped routes contribute exactly zero, drop vs residual accounting, static vs dynamic dispatch, router
temperature and fp32 routing under autocast, the balance loss, straggler bias, routing controls, statistics and
activation checkpointing."""

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.models.moe import TopKMoE


def _cfg(**kw):
    base = dict(vocab_size=64, hidden_size=16, layers=2, ffn_size=32, num_experts=4, top_k=2, attention_heads=2,
                max_sequence_length=17, capacity_factor=1.0, norm_type="layernorm", position_embedding="learned")
    base.update(kw)
    return QuantaWeaveConfig(**base)


def _moe(**kw):
    torch.manual_seed(0)
    moe = TopKMoE(_cfg(**kw))
    moe.kernel = "loop"
    return moe


@torch.no_grad()
def _naive(moe, x):
    """Per-route loop: top-k of the fp32 router, renormalised; per expert, routes ordered by (-weight, route index)
    and the first ``capacity`` kept. Returns (output, overflow count, tokens with every route skipped)."""
    logits = x.float() @ moe.router.weight.detach().float().T / moe.router_temperature
    w, idx = logits.softmax(-1).topk(moe.top_k, -1)
    w = w / w.sum(-1, keepdim=True)
    cap = moe.capacity(x.size(0))
    out = torch.zeros_like(x)
    overflow, kept_any = 0, torch.zeros(x.size(0), dtype=torch.bool)
    for e in range(moe.num_experts):
        routes = [(float(w[t, j]), t * moe.top_k + j) for t in range(x.size(0)) for j in range(moe.top_k)
                  if int(idx[t, j]) == e]
        routes.sort(key=lambda r: (-r[0], r[1]))
        for position, (weight, r) in enumerate(routes):
            if position >= cap:
                overflow += 1
                continue
            t = r // moe.top_k
            out[t] += weight * moe.expert_forward(e, x[t:t + 1])[0]
            kept_any[t] = True
    return out, overflow, ~kept_any


@pytest.mark.parametrize("cf,k", [(0.5, 1), (0.5, 2), (1.0, 2), (0.0, 2)])
def test_capacity_plan_matches_the_per_route_loop(cf, k):
    moe = _moe(capacity_factor=cf, top_k=k)
    x = torch.randn(1, 24, 16, generator=torch.Generator().manual_seed(1))
    out, balance, dropped, overflow, _ = moe(x)
    ref, ref_overflow, skipped = _naive(moe, x[0])
    assert torch.allclose(out[0], ref, atol=1e-6)
    assert int(overflow) == ref_overflow and int(dropped) == ref_overflow
    if cf == 0.0:
        assert ref_overflow == 0
    # a token whose every route was skipped gets exactly zero from the MoE (it keeps its residual in the block)
    assert torch.equal(out[0][skipped], torch.zeros_like(out[0][skipped]))


def test_overflow_policy_drop_reports_dropped_residual_only_overflow():
    x = torch.randn(1, 24, 16, generator=torch.Generator().manual_seed(2))
    drop = _moe(capacity_factor=0.5, overflow_policy="drop")
    residual = _moe(capacity_factor=0.5, overflow_policy="residual")
    a, _, dropped_a, overflow_a, _ = drop(x)
    b, _, dropped_b, overflow_b, _ = residual(x)
    assert torch.equal(a, b) and int(overflow_a) == int(overflow_b) > 0
    assert int(dropped_a) == int(overflow_a) and int(dropped_b) == 0


def test_static_dispatch_equals_dynamic_without_capacity():
    moe = _moe(capacity_factor=0.0)
    x = torch.randn(2, 8, 16, generator=torch.Generator().manual_seed(3))
    dynamic = moe(x)[0]
    moe.static_dispatch = True
    static = moe(x)[0]
    assert torch.allclose(dynamic, static, atol=1e-6)


def test_router_temperature_fp32_under_autocast_and_straggler_bias():
    moe = _moe(router_temperature=2.0)
    x = torch.randn(10, 16, generator=torch.Generator().manual_seed(4))
    logits, probs, idx, w = moe.route(x)
    raw = x @ moe.router.weight.T
    assert torch.allclose(logits, raw / 2.0, atol=1e-6) and torch.allclose(probs, (raw / 2.0).softmax(-1), atol=1e-6)
    assert torch.allclose(w.sum(-1), torch.ones(10))
    with torch.autocast("cpu", dtype=torch.bfloat16):
        logits_ac, probs_ac, _, _ = moe.route(x.bfloat16())
    assert logits_ac.dtype == torch.float32 and probs_ac.dtype == torch.float32
    # straggler bias moves selection only; weights stay the unbiased probabilities, renormalised
    moe.expert_bias = torch.tensor([100.0, 0.0, 0.0, 0.0])
    _, probs_b, idx_b, w_b = moe.route(x)
    assert bool((idx_b == 0).any(dim=-1).all())
    expect = probs_b.gather(1, idx_b)
    assert torch.allclose(w_b, expect / expect.sum(-1, keepdim=True))


def test_balance_loss_formula():
    moe = _moe()
    x = torch.randn(1, 20, 16, generator=torch.Generator().manual_seed(5))
    _, balance, _, _, _ = moe(x)
    _, probs, idx, _ = moe.route(x[0])
    share = torch.bincount(idx.reshape(-1), minlength=4).float() / idx.numel()
    assert torch.allclose(balance, 4 * (probs.mean(0) * share).sum())


def test_routing_controls_validate_apply_and_stats():
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(_cfg())
    model.set_moe_kernel("loop")
    for bad in (dict(capacity_factor=-1.0), dict(overflow_policy="nope"), dict(router_temperature=0.0)):
        with pytest.raises(ValueError):
            model.set_routing_controls(**bad)
    model.set_routing_controls(capacity_factor=0.5, router_temperature=1.5, router_aux_loss_coef=0.2)
    assert all(m.capacity_factor == 0.5 and m.router_temperature == 1.5 for m in model.moes())
    assert model.config.capacity_factor == 0.5 and model.router_aux_loss_coef == 0.2
    model.set_collect_stats(True)
    ids = torch.randint(0, 64, (2, 9), generator=torch.Generator().manual_seed(6))
    model(ids, labels=ids)
    stats = model.routing_stats()
    assert len(stats) == 2
    for s in stats:
        assert int(s["expert_assigned"].sum()) == 2 * 9 * 2
        assert int(s["expert_load"].sum()) + s["dropped_tokens"].numel() == 2 * 9 * 2
        assert abs(float(s["importance"].sum()) - 1.0) < 1e-5


def test_activation_checkpointing_gives_identical_gradients():
    ids = torch.randint(0, 64, (2, 17), generator=torch.Generator().manual_seed(7))
    grads = []
    for checkpointing in (False, True):
        torch.manual_seed(0)
        model = QuantaWeaveMoEForCausalLM(_cfg())
        model.set_moe_kernel("loop")
        model.activation_checkpointing = checkpointing
        model.train()
        model(ids, labels=ids)["loss"].backward()
        grads.append({n: p.grad.clone() for n, p in model.named_parameters()})
    for name, g in grads[0].items():
        assert torch.equal(g, grads[1][name]), name
