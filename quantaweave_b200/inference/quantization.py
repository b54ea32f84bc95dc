"""Weight-only int8 / int4 quantisation for inference.

Format parity with the reference ``src/quantization.py`` (``QuantizedLinear`` :21-75, ``quantize_model`` :78,
``save_quantized``/``load_quantized`` :105-117): symmetric quantisation, int8 with one scale per row by default,
int4 values clamped to [-8, 7], stored +8 as uint8 with two values per byte (low nibble = even column), scales
``[out, groups]``, the input dimension padded to a multiple of the group. Payload of ``model.int{b}.pt``:
``{"config", "bits", "group_size", "quantize_lm_head", "state_dict"}`` with per-expert keys
``experts.{e}.{gate,up,down}.{qweight,scales}``.

B200 path: expert weights are kept stacked (``q_gate_up [E, 2F, ...]``, ``q_down [E, H, ...]``) with fp16 scales,
exactly the layout the grouped dequant-GEMV kernel reads, so decoding never materialises dense weights (the reference
dequantises every expert to dense bf16 when its decoder is built).
"""

from __future__ import annotations

from pathlib import Path
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import QuantaWeaveConfig
from ..utils.checkpoint_io import load_checkpoint


def quantize_tensor(weight: Tensor, bits: int, group_size: int) -> tuple[Tensor, Tensor]:
    """Symmetric per-group quantisation of ``weight [..., out, in]`` -> (qweight, fp32 scales [..., out, groups]).

    Leading dimensions (stacked experts) are quantised in one pass, each row independently."""
    *lead, out_features, in_features = weight.shape
    padded = -(-in_features // group_size) * group_size
    w = F.pad(weight.detach().float(), (0, padded - in_features))
    grouped = w.reshape(*lead, out_features, -1, group_size)
    limit = 127 if bits == 8 else 7
    scales = (grouped.abs().amax(dim=-1) / limit).clamp(min=1e-8)
    q = torch.round(grouped / scales[..., None]).clamp(-limit - (bits == 4), limit).reshape(*lead, out_features, -1)
    if bits == 8:
        return q.to(torch.int8), scales
    unsigned = (q + 8).to(torch.uint8)
    return unsigned[..., 0::2] | (unsigned[..., 1::2] << 4), scales


def dequantize_tensor(qweight: Tensor, scales: Tensor, bits: int, group_size: int, in_features: int) -> Tensor:
    out_features = qweight.size(0)
    if bits == 8:
        values = qweight.float()
    else:
        low = (qweight & 0xF).float() - 8
        high = (qweight >> 4).float() - 8
        values = torch.stack([low, high], dim=-1).reshape(out_features, -1)
    values = values.reshape(out_features, -1, group_size) * scales.float()[..., None]
    return values.reshape(out_features, -1)[:, :in_features]


class QuantizedLinear(nn.Module):
    """Linear layer with symmetric quantised weights (int8: per-row scale by default; int4: groups of 32)."""

    def __init__(self, in_features: int, out_features: int, bits: int = 8, group_size: Optional[int] = None) -> None:
        super().__init__()
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        group_size = group_size or (in_features if bits == 8 else 32)
        if bits == 4 and group_size % 2:
            raise ValueError("group_size must be even for 4-bit weights")
        self.in_features, self.out_features, self.bits, self.group_size = in_features, out_features, bits, group_size
        self.padded = -(-in_features // group_size) * group_size
        groups = self.padded // group_size
        stored = self.padded if bits == 8 else self.padded // 2
        self.register_buffer("qweight", torch.zeros(out_features, stored, dtype=torch.int8 if bits == 8 else torch.uint8))
        self.register_buffer("scales", torch.ones(out_features, groups))

    @classmethod
    def from_linear(cls, linear: nn.Module, bits: int = 8, group_size: Optional[int] = None) -> "QuantizedLinear":
        if getattr(linear, "bias", None) is not None:
            raise ValueError("bias is not supported")
        layer = cls(linear.in_features, linear.out_features, bits, group_size).to(linear.weight.device)
        q, s = quantize_tensor(linear.weight, bits, layer.group_size)
        layer.qweight.copy_(q)
        layer.scales.copy_(s)
        return layer

    def dequantize(self) -> Tensor:
        return dequantize_tensor(self.qweight, self.scales, self.bits, self.group_size, self.in_features)

    @property
    def weight(self) -> Tensor:
        return self.dequantize()

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.dequantize().to(x.dtype))

    def stored_bytes(self) -> int:
        return self.qweight.numel() * self.qweight.element_size() + self.scales.numel() * self.scales.element_size()


class QuantizedExperts:
    """Stacked quantised expert weights of one MoE layer, in the grouped dequant-GEMV layout."""

    def __init__(self, bits: int, group_size: int, hidden: int, ffn: int) -> None:
        self.bits, self.group_size, self.hidden, self.ffn = bits, group_size, hidden, ffn

    @staticmethod
    def quantize(w_gate_up: Tensor, w_down: Tensor, bits: int, group_size: Optional[int]):
        E, F2, H = w_gate_up.shape
        F_ = F2 // 2
        g_in = group_size or (H if bits == 8 else 32)
        g_dn = group_size or (F_ if bits == 8 else 32)
        q_gu, s_gu = quantize_tensor(w_gate_up, bits, g_in)
        q_d, s_d = quantize_tensor(w_down, bits, g_dn)
        return q_gu, s_gu.half(), q_d, s_d.half(), g_in, g_dn


def quantize_moe(moe, bits: int, group_size: Optional[int]) -> tuple[int, int]:
    """Replace a ``TopKMoE``'s stacked expert parameters by quantised buffers. Returns (bytes before, after)."""
    if getattr(moe, "quant", None) is not None:
        raise ValueError("model is already quantized")
    before = moe.w_gate_up.numel() * 4 + moe.w_down.numel() * 4
    q_gu, s_gu, q_d, s_d, g_in, g_dn = QuantizedExperts.quantize(moe.w_gate_up.detach(), moe.w_down.detach(), bits,
                                                                 group_size)
    device = moe.w_gate_up.device
    del moe.w_gate_up
    del moe.w_down
    moe.register_buffer("q_gate_up", q_gu.to(device))
    moe.register_buffer("s_gate_up", s_gu.to(device))
    moe.register_buffer("q_down", q_d.to(device))
    moe.register_buffer("s_down", s_d.to(device))
    moe.quant = {"bits": bits, "group_in": g_in, "group_down": g_dn}
    # training and the per-expert path dequantise one expert at a time; without gradients on CUDA the layer expands
    # the packed stacks to bf16 in one kernel and runs the tcgen05 grouped GEMMs ("auto")
    moe.kernel = "auto"
    after = sum(t.numel() * t.element_size() for t in (q_gu, s_gu, q_d, s_d))
    return before, after


def dequantized_expert(moe, index: int) -> tuple[Tensor, Tensor]:
    q = moe.quant
    H, F2 = moe.hidden_size, 2 * moe.ffn_local
    wgu = dequantize_tensor(moe.q_gate_up[index], moe.s_gate_up[index], q["bits"], q["group_in"], H)
    wd = dequantize_tensor(moe.q_down[index], moe.s_down[index], q["bits"], q["group_down"], F2 // 2)
    return wgu, wd


def quantize_model(model, bits: int = 8, group_size: Optional[int] = None, quantize_lm_head: bool = False) -> dict:
    """Quantise every expert (and optionally the LM head) in place. Returns size statistics.

    An expert-parallel model quantises the experts it holds (each row is quantised on its own, so a rank's experts
    come out exactly as they would in the consolidated model); this serves expert-parallel decoding. Such a model
    cannot be saved as a quantised file, which must hold every expert (``save_quantized``)."""
    ep = getattr(model, "expert_parallel", None)
    if ep is not None and getattr(ep, "tp_size", 1) > 1:
        raise ValueError("tensor-parallel experts hold slices of each weight; consolidate the model before "
                         "quantizing it")
    before = after = replaced = 0
    for block in model.blocks:
        b, a = quantize_moe(block.moe, bits, group_size)
        before += b
        after += a
        replaced += 3 * block.moe.num_local_experts
    if quantize_lm_head:
        if isinstance(model.lm_head, QuantizedLinear):
            raise ValueError("model is already quantized")
        layer = QuantizedLinear.from_linear(model.lm_head, bits, group_size)
        before += model.lm_head.weight.numel() * model.lm_head.weight.element_size()
        after += layer.stored_bytes()
        replaced += 1
        model.lm_head = layer
    return {"bits": bits, "group_size": group_size, "replaced_layers": replaced, "bytes_before": before,
            "bytes_after": after, "compression": before / after if after else None}


def save_quantized(model, path: Path, stats: dict, quantize_lm_head: bool = False) -> None:
    if getattr(model, "expert_parallel", None) is not None:
        raise ValueError("a quantised file holds every expert: consolidate the expert-parallel model, then quantize "
                         "and save it")
    torch.save({"config": dict(model.config.__dict__), "bits": stats["bits"], "group_size": stats["group_size"],
                "quantize_lm_head": quantize_lm_head, "state_dict": model.state_dict()}, path)


def load_quantized(path: Path, device=torch.device("cpu")):
    from ..models.model import QuantaWeaveMoEForCausalLM

    payload = load_checkpoint(path, map_location="cpu")
    model = QuantaWeaveMoEForCausalLM(QuantaWeaveConfig.from_dict(payload["config"]))
    quantize_model(model, payload["bits"], payload["group_size"], payload["quantize_lm_head"])
    model.load_state_dict(payload["state_dict"])
    return model.to(device).eval()
