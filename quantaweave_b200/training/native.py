"""Prepare a model for the native B200 path.

bf16 storage for every matrix the tcgen05 GEMMs read (embeddings, attention projections, expert stacks, LM head);
fp32 for the router (the router GEMM runs in fp32, as in the reference) and for norm weights and biases. The fused
optimizer keeps fp32 master copies of the bf16 parameters. ``recompute_experts`` trades the saved gate/up
activations for a recomputation in backward (the memory-tight single-GPU setting).
"""

from __future__ import annotations

import torch

_FP32_SUFFIXES = ("router.weight",)


def prepare_model(model, precision: str = "bf16", recompute_experts: bool | None = None):
    if precision not in {"bf16", "auto"}:
        return model
    from ..ops import native_required

    native_required()
    for name, module in model.named_modules():
        for pname, param in list(module.named_parameters(recurse=False)):
            full = f"{name}.{pname}" if name else pname
            keep_fp32 = full.endswith(_FP32_SUFFIXES) or param.dim() < 2
            want = torch.float32 if keep_fp32 else torch.bfloat16
            if param.dtype != want:
                param.data = param.data.to(want)
    for moe in model.moes():
        if getattr(moe, "quant", None) is not None:
            continue  # quantised experts are inference-only: the decoder's dequant-GEMV kernels serve them
        moe.kernel = "native"
        if recompute_experts is not None:
            moe.recompute_activations = bool(recompute_experts)
    return model
