"""The allocation-free RMSNorm backward, called through its exported C symbol.

It serves callers that may not allocate device memory (hosts that own the memory budget, or code that must avoid
cudaMalloc/cudaFree because they can synchronise the device). The test checks it against the library's regular
RMSNorm backward entry point, with the same tolerances as the other norm tests, on two calls in a row (the scratch
array is shared between calls, so a stale-state bug would show on the second call). This file is named to be
collected last.
"""

import ctypes

import pytest
import torch

from conftest import cuda_ready

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ready(), reason="needs a B200")]


def _lib():
    import quantaweave_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.qw_rmsnorm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.qw_noalloc_error_message.restype = ctypes.c_char_p
    lib.qw_noalloc_error_message.argtypes = [ctypes.c_int]
    return lib, ext


def _close(out, ref, tol):
    err = (out.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"max abs err {err:.3e} vs scale {scale:.3e}"


def _case(ext, rows, hidden, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=g).bfloat16()
    dy = torch.randn(rows, hidden, device="cuda", generator=g).bfloat16()
    w = 1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device="cuda")
    ext.norm_fwd(x, None, None, w, None, y, None, rstd, 1e-5, True)
    blocks = ext.norm_bwd_blocks(rows)
    dx_ref = torch.empty_like(x)
    dw_ref = torch.empty(hidden, device="cuda")
    ext.norm_bwd(dy, x, w, None, rstd, None, dx_ref, torch.empty(blocks, hidden, device="cuda"), None, dw_ref, None,
                 True, False)
    return x, dy, w, rstd, dx_ref, dw_ref


def _fp32_rmsnorm_backward(x, dy, w, eps=1e-5):
    """Plain PyTorch fp32 RMSNorm backward (autograd through y = x * rsqrt(mean(x^2) + eps) * w)."""
    xf = x.float().requires_grad_(True)
    wf = w.float().clone().requires_grad_(True)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * wf
    y.backward(dy.float())
    return xf.grad, wf.grad


def test_noalloc_rmsnorm_backward_matches_fp32_pytorch():
    lib, ext = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, (rows, hidden) in enumerate([(777, 512), (300, 1024)]):  # two calls in a row, shared scratch
        x, dy, w, rstd, _, _ = _case(ext, rows, hidden, 100 + seed)
        dx = torch.empty_like(x)
        dw = torch.full((hidden,), float("nan"), device="cuda")
        code = lib.qw_rmsnorm_backward_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                               dx.data_ptr(), dw.data_ptr(), rows, hidden, stream)
        assert code == 0, lib.qw_noalloc_error_message(code).decode()
        torch.cuda.synchronize()
        dx_ref, dw_ref = _fp32_rmsnorm_backward(x, dy, w)
        _close(dx, dx_ref, 3e-2)
        _close(dw, dw_ref, 1e-2)


def test_noalloc_rmsnorm_backward_matches_regular_entry_point():
    lib, ext = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, (rows, hidden) in enumerate([(1000, 1024), (4097, 256)]):  # two calls in a row, shared scratch
        x, dy, w, rstd, dx_ref, dw_ref = _case(ext, rows, hidden, seed)
        dx = torch.empty_like(x)
        dw = torch.full((hidden,), float("nan"), device="cuda")
        code = lib.qw_rmsnorm_backward_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                               dx.data_ptr(), dw.data_ptr(), rows, hidden, stream)
        assert code == 0, lib.qw_noalloc_error_message(code).decode()
        torch.cuda.synchronize()
        _close(dx, dx_ref, 3e-2)
        _close(dw, dw_ref, 1e-2)


def test_noalloc_rejects_oversized_problems():
    lib, _ = _lib()
    code = lib.qw_rmsnorm_backward_noalloc(256, 256, 256, 256, 256, 256, 10_000_000, 4096, None)  # never read
    assert code == 2
    assert b"too large" in lib.qw_noalloc_error_message(code)


def test_noalloc_rejects_misaligned_rows_before_launching():
    lib, _ = _lib()
    rows, hidden = 16, 256
    buf = torch.zeros(rows * hidden + 8, device="cuda", dtype=torch.bfloat16)
    ok = buf[: rows * hidden]
    odd = buf[1: 1 + rows * hidden]  # a legal view at an odd bf16 offset: 2 bytes past a 16-byte boundary
    w = torch.ones(hidden, device="cuda")
    rstd = torch.ones(rows, device="cuda")
    dw = torch.zeros(hidden, device="cuda")
    for dy, x, dx in ((odd, ok, ok), (ok, odd, ok), (ok, ok, odd)):
        code = lib.qw_rmsnorm_backward_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                               dx.data_ptr(), dw.data_ptr(), rows, hidden, None)
        assert code == 1
        assert b"16-byte" in lib.qw_noalloc_error_message(code)
    torch.cuda.synchronize()  # nothing was launched, so the context is untouched


def test_noalloc_zero_rows_zeroes_the_weight_gradient():
    lib, _ = _lib()
    hidden = 256
    buf = torch.zeros(hidden, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(hidden, device="cuda")
    dw = torch.full((hidden,), float("nan"), device="cuda")
    code = lib.qw_rmsnorm_backward_noalloc(buf.data_ptr(), buf.data_ptr(), w.data_ptr(), w.data_ptr(), buf.data_ptr(),
                                           dw.data_ptr(), 0, hidden, torch.cuda.current_stream().cuda_stream)
    assert code == 0
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.zeros_like(dw))
