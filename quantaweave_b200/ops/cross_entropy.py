"""Chunked fused linear + cross-entropy: full-vocabulary logits are never materialised.

For each chunk of rows the tcgen05 GEMM writes bf16 logits, the CE kernel turns them in place into
``softmax - onehot`` (and the per-row loss), and two GEMMs immediately produce that chunk's input gradient and
accumulate the fp32 weight gradient. The scalar ``grad_output / n_valid`` is applied at backward time on the
device, so no host synchronisation is needed. When neither input needs a gradient (evaluation, ``torch.no_grad``)
only the logits GEMM and the loss run; a frozen weight (or input) skips its own gradient GEMM.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import ext

IGNORE_INDEX = -100


class _LinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor, weight: Tensor, labels: Tensor, chunk_rows: int):
        C = ext()
        H = h.size(-1)
        h2 = h.reshape(-1, H).to(torch.bfloat16).contiguous()
        lab = labels.reshape(-1).to(torch.int64).contiguous()
        T = h2.size(0)
        V = weight.size(0)
        w = weight.to(torch.bfloat16).contiguous()
        dev = h2.device
        need_dh, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        loss_rows = torch.empty(T, device=dev, dtype=torch.float32)
        dh = torch.empty_like(h2) if need_dh else None
        dw = torch.zeros(V, H, device=dev, dtype=torch.float32) if need_dw else None
        ld = (V + 7) // 8 * 8
        logits = torch.empty(min(chunk_rows, T), ld, device=dev, dtype=torch.bfloat16)
        for start in range(0, T, chunk_rows):
            stop = min(T, start + chunk_rows)
            lg = logits[: stop - start, :V]
            C.linear_fwd(h2[start:stop], w, None, None, lg)
            C.cross_entropy_chunk(lg, lab[start:stop], 1.0, loss_rows[start:stop], IGNORE_INDEX)
            if need_dh:
                C.linear_dgrad(lg, w, dh[start:stop], False)
            if need_dw:
                C.linear_wgrad(lg, h2[start:stop], dw, True)
        n_valid = (lab != IGNORE_INDEX).sum().clamp(min=1).float()
        loss = loss_rows.sum() / n_valid
        ctx.save_for_backward(dh, dw, n_valid)
        ctx.shape, ctx.wdtype = h.shape, weight.dtype
        return loss

    @staticmethod
    def backward(ctx, grad: Tensor):
        C = ext()
        dh, dw, n_valid = ctx.saved_tensors
        scale = (grad.float() / n_valid).reshape(1).contiguous()
        if dh is not None:
            C.scale_bf16(dh, scale)
            dh = dh.reshape(ctx.shape)
        if dw is not None:
            dw = (dw * scale).to(ctx.wdtype)
        return dh, dw, None, None


def linear_cross_entropy(h: Tensor, weight: Tensor, labels: Tensor, chunk_rows: int = 16384) -> Tensor:
    """Mean CE of ``h @ weight^T`` against ``labels`` (``-100`` ignored)."""
    return _LinearCE.apply(h, weight, labels, chunk_rows)
