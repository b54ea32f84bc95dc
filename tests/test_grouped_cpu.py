"""The reference-API grouped expert GEMM (``moe_kernels``) on CPU: uneven counts including empty experts (the
reference's ``COUNTS``), forward and backward against per-expert matmuls, and SwiGLU over a TopKMoE's experts."""

import torch
import torch.nn.functional as F

from quantaweave_b200 import QuantaWeaveConfig, moe_kernels as mk
from quantaweave_b200.models.moe import TopKMoE

COUNTS = [0, 5, 37, 1, 0, 64, 33, 2]


def test_grouped_matmul_matches_per_expert_matmuls_forward_and_backward():
    torch.manual_seed(0)
    x = torch.randn(sum(COUNTS), 24, requires_grad=True)
    w = torch.randn(len(COUNTS), 40, 24, requires_grad=True)
    plan = mk.GroupedPlan(COUNTS, x.device)
    assert plan.rows == sum(COUNTS) and plan.padded_rows % 128 == 0
    y = mk.grouped_matmul(x, w, plan)
    g = torch.randn_like(y)
    (y * g).sum().backward()
    xr, wr = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    parts, start = [], 0
    for e, c in enumerate(COUNTS):
        parts.append(xr[start:start + c] @ wr[e].T)
        start += c
    ref = torch.cat(parts)
    (ref * g).sum().backward()
    assert torch.allclose(y, ref, atol=1e-5)
    assert torch.allclose(x.grad, xr.grad, atol=1e-5) and torch.allclose(w.grad, wr.grad, atol=1e-5)
    assert torch.equal(w.grad[0], torch.zeros_like(w.grad[0]))  # an expert with no rows gets an exact zero


def test_empty_plan_and_grouped_swiglu_over_moe_experts():
    w = torch.randn(3, 8, 16)
    empty = mk.grouped_matmul(torch.empty(0, 16), w, mk.GroupedPlan([0, 0, 0], torch.device("cpu")))
    assert empty.shape == (0, 8)
    cfg = QuantaWeaveConfig(vocab_size=8, hidden_size=16, layers=1, ffn_size=32, num_experts=4, top_k=1,
                            attention_heads=2)
    torch.manual_seed(1)
    moe = TopKMoE(cfg)
    assert mk.experts_support_grouped(moe.experts)
    counts = [3, 0, 5, 2]
    x = torch.randn(sum(counts), 16)
    y = mk.grouped_swiglu(x, moe.experts, counts)
    start, parts = 0, []
    for e, c in enumerate(counts):
        parts.append(moe.expert_forward(e, x[start:start + c]))
        start += c
    assert torch.allclose(y, torch.cat(parts), atol=1e-5)
    assert mk.compute_dtype(x) == torch.float32 and not mk.kernels_available(torch.device("cpu"))
