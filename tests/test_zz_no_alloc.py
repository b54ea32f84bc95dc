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
    code = lib.qw_rmsnorm_backward_noalloc(1, 1, 1, 1, 1, 1, 10_000_000, 4096, None)
    assert code == 2
    assert b"too large" in lib.qw_noalloc_error_message(code)
