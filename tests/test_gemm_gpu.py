"""tcgen05 GEMM numerics against a plain PyTorch fp32 reference (dense linear layers and grouped MoE GEMMs)."""

import pytest
import torch

from conftest import cuda_ready

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ready(), reason="needs a B200")]


def _ext():
    from quantaweave_b200.ops import native_required

    return native_required()


def _close(out, ref, tol=2e-2):
    out, ref = out.float(), ref.float()
    if out.numel() == 0:
        assert ref.numel() == 0
        return
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max abs err {err} vs scale {scale}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 384, 192), (1024, 1000, 1024), (77, 3072, 512)])
def test_linear_fwd(M, N, K):
    C = _ext()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    res = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.linear_fwd(x, w, bias, res, out)
    ref = x.float() @ w.float().t() + bias + res.float()
    _close(out, ref)
    out32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    C.linear_fwd(x, w, None, None, out32)
    _close(out32, x.float() @ w.float().t(), 1e-3)
    assert C.read_status(True) == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (130, 1024, 320), (8200, 1024, 1024), (65536, 1024, 256)])
def test_linear_dgrad_wgrad(M, N, K):
    """The last two shapes have too few output tiles to fill the GPU, so the weight gradient is split over token
    chunks and reduced in a fixed order (fp32 partials)."""
    C = _ext()
    g = torch.Generator(device="cuda").manual_seed(1)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    dx = torch.empty(M, K, device="cuda", dtype=torch.float32)
    C.linear_dgrad(dy, w, dx, False)
    _close(dx, dy.float() @ w.float(), 1e-3)
    dw = torch.zeros(N, K, device="cuda", dtype=torch.float32)
    C.linear_wgrad(dy, x, dw, False)
    _close(dw, dy.float().t() @ x.float(), 1e-3)
    C.linear_wgrad(dy, x, dw, True)  # accumulate
    _close(dw, 2 * dy.float().t() @ x.float(), 1e-3)
    dwb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)  # bf16 gradient output (the split path casts)
    C.linear_wgrad(dy, x, dwb, False)
    _close(dwb, dy.float().t() @ x.float(), 1e-2)
    assert C.read_status(True) == 0


def _grouped_layout(counts, H, device):
    counts_t = torch.tensor(counts, dtype=torch.int32, device=device)
    padded = [(c + 127) // 128 * 128 for c in counts]
    offs = [0]
    for p in padded[:-1]:
        offs.append(offs[-1] + p)
    return counts_t, torch.tensor(offs, dtype=torch.int32, device=device), sum(padded), offs


@pytest.mark.parametrize("counts", [[0, 5, 37, 1, 0, 64, 33, 2], [300, 0, 129, 256]])
def test_moe_grouped_forward_backward(counts):
    C = _ext()
    torch.manual_seed(0)
    E, H, F = len(counts), 256, 256
    dev = "cuda"
    counts_t, offs_t, R, offs = _grouped_layout(counts, H, dev)
    x = torch.zeros(R, H, device=dev, dtype=torch.bfloat16)
    for e, c in enumerate(counts):
        x[offs[e]:offs[e] + c] = torch.randn(c, H, device=dev).bfloat16()
    wgu = (torch.randn(E, 2 * F, H, device=dev) * 0.05).bfloat16()
    wd = (torch.randn(E, H, F, device=dev) * 0.05).bfloat16()
    h = torch.full((R, F), 7.0, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(R, 2 * F, device=dev, dtype=torch.bfloat16)
    C.moe_gate_up_fwd(x, wgu, counts_t, offs_t, h, gu)
    y = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
    C.moe_down_fwd(h, wd, counts_t, offs_t, y)
    dy = torch.zeros(R, H, device=dev, dtype=torch.bfloat16)
    route_w = torch.zeros(R, device=dev)
    for e, c in enumerate(counts):
        dy[offs[e]:offs[e] + c] = torch.randn(c, H, device=dev).bfloat16()
        route_w[offs[e]:offs[e] + c] = torch.rand(c, device=dev)
    tiles = C.moe_dw_tiles(F)
    dgu = torch.empty_like(gu)
    hw = torch.empty_like(h)
    part = torch.empty(R, tiles, device=dev)
    C.moe_down_bwd(dy, wd, counts_t, offs_t, gu, route_w, dgu, hw, part)
    dx = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
    C.moe_gate_up_dgrad(dgu, wgu, counts_t, offs_t, dx)
    dwd = torch.empty(E, H, F, device=dev)
    C.moe_wgrad(dy, hw, counts_t, offs_t, dwd, False)
    dwgu = torch.empty(E, 2 * F, H, device=dev)
    C.moe_wgrad(dgu, x, counts_t, offs_t, dwgu, False)
    assert C.read_status(True) == 0
    for e, c in enumerate(counts):
        sl = slice(offs[e], offs[e] + c)
        pad = slice(offs[e] + c, offs[e] + (c + 127) // 128 * 128)
        xe = x[sl].float()
        g_ = xe @ wgu[e, :F].float().t()
        u_ = xe @ wgu[e, F:].float().t()
        he = torch.nn.functional.silu(g_) * u_
        _close(h[sl], he)
        _close(gu[sl, :F], g_)
        assert torch.all(h[pad] == 0)
        ye = h[sl].float() @ wd[e].float().t()
        _close(y[sl], ye)
        a = dy[sl].float() @ wd[e].float()
        w = route_w[sl][:, None]
        gf, uf = gu[sl, :F].float(), gu[sl, F:].float()
        sg = torch.sigmoid(gf)
        _close(dgu[sl, :F], w * a * uf * (sg + gf * sg * (1 - sg)), 3e-2)
        _close(dgu[sl, F:], w * a * gf * sg, 3e-2)
        _close(part[sl].sum(1), (a * (gf * sg * uf)).sum(1), 3e-2)
        _close(hw[sl], w * gf * sg * uf, 3e-2)
        _close(dx[sl], dgu[sl].float() @ wgu[e].float(), 3e-2)
        if c:
            _close(dwd[e], dy[sl].float().t() @ hw[sl].float(), 3e-2)
            _close(dwgu[e], dgu[sl].float().t() @ xe, 3e-2)
        else:
            assert torch.all(dwd[e] == 0) and torch.all(dwgu[e] == 0)


@pytest.mark.parametrize("M,N", [(2048, 3072), (1000, 1024), (64, 64)])
def test_linear_bias_grad_matches_fp32(M, N):
    """Bias gradient of the native linear layer (deterministic two-stage column sum) vs an fp32 reference."""
    from quantaweave_b200.ops.linear import linear

    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, 1024, device="cuda", generator=g).bfloat16().requires_grad_()
    w = (0.05 * torch.randn(N, 1024, device="cuda", generator=g)).bfloat16().requires_grad_()
    b = torch.zeros(N, device="cuda", requires_grad=True)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    linear(x, w, b).backward(dy)
    ref = dy.float().sum(0)
    err = (b.grad - ref).abs().max().item()
    assert err <= 1e-3 * (ref.abs().max().item() + 1), err
    first = b.grad.clone()
    b.grad = None
    linear(x, w, b).backward(dy)
    assert torch.equal(b.grad, first)  # deterministic


@pytest.mark.parametrize("T,H,E", [(4133, 1024, 64), (300, 256, 8)])
def test_router_gemms_on_tensor_cores_match_fp64(T, H, E):
    """Router logits, dX and dW run on the tcgen05 GEMM over bf16 splits of the fp32 operands; against fp64."""
    C = _ext()
    torch.manual_seed(3)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.randn(E, H, device="cuda") * 0.02
    dl = torch.randn(T, E, device="cuda") * 1e-3

    def rel(out, ref):
        return float((out.double() - ref).abs().max() / ref.abs().max())

    logits = torch.empty(T, E, device="cuda")
    C.router_logits(x, w, logits)
    assert rel(logits, x.double() @ w.double().t()) < 5e-6  # three-term split: fp32-level
    dx = torch.empty(T, H, device="cuda")
    C.router_dx(dl, w, dx)
    assert rel(dx, dl.double() @ w.double()) < 1e-4
    dw = torch.full((E, H), 0.5, device="cuda")
    ws = torch.empty(C.router_dw_split(T) * E * H, device="cuda")
    C.router_dw(dl, x, dw, True, ws)
    assert rel(dw - 0.5, dl.double().t() @ x.double()) < 1e-4
    assert C.read_status(True) == 0


@pytest.mark.parametrize("counts", [[3, 0, 200, 129], [128, 128], [0, 0, 5]])
def test_moe_kernels_api_grouped_matmul_and_swiglu(counts):
    """The reference-named ``moe_kernels`` API (``grouped_matmul``, ``grouped_swiglu``) runs the tcgen05 grouped GEMMs
    on CUDA and matches an fp32 per-expert loop, forward and backward (input and weight gradients)."""
    from torch import nn

    from quantaweave_b200 import moe_kernels
    from quantaweave_b200.ops.grouped import _native

    torch.manual_seed(4)
    dev = torch.device("cuda")
    H, F_ = 128, 192
    plan = moe_kernels.GroupedPlan(counts, dev)
    x = (torch.randn(sum(counts), H, device=dev) * 0.5).bfloat16().requires_grad_()
    w = (torch.randn(len(counts), F_, H, device=dev) * 0.05).bfloat16().requires_grad_()
    assert moe_kernels.kernels_available(dev) and _native(x, w)
    y = moe_kernels.grouped_matmul(x, w, plan)
    gy = torch.randn_like(y)
    (y.float() * gy.float()).sum().backward()
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    start, parts = 0, []
    for e, c in enumerate(counts):
        parts.append(xr[start:start + c] @ wr[e].T)
        start += c
    yr = torch.cat(parts)
    (yr * gy.float()).sum().backward()
    _close(y, yr, 2e-2)
    _close(x.grad, xr.grad, 2e-2)
    _close(w.grad, wr.grad, 2e-2)

    class Expert(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate, self.up = nn.Linear(H, F_, bias=False), nn.Linear(H, F_, bias=False)
            self.down = nn.Linear(F_, H, bias=False)

    experts = nn.ModuleList(Expert() for _ in counts).to(dev)
    assert moe_kernels.experts_support_grouped(experts)
    inp = torch.randn(sum(counts), H, device=dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = moe_kernels.grouped_swiglu(inp, experts, counts)
    start, parts = 0, []
    for e, c in zip(experts, counts):
        rows = inp[start:start + c]
        parts.append(e.down(torch.nn.functional.silu(e.gate(rows)) * e.up(rows)))
        start += c
    ref = torch.cat(parts)
    _close(out, ref, 3e-2)
