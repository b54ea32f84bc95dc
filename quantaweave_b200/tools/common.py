"""Shared helpers of the command-line tools: load a saved checkpoint directory onto a device.

A checkpoint directory (the trainer's ``--output``) holds ``config.json``, ``model.pt`` (payload key ``"model"``) and
the tokenizer files, as in the reference (``src/generate_quantweave_moe.py:41-47``). On a CUDA device the model is put
on the native sm_100a path (bf16 matrices, fp32 router and norms); elsewhere it stays on the fp32 PyTorch path.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..config import QuantaWeaveConfig
from ..utils.checkpoint_io import load_checkpoint


def read_config(directory: Path) -> QuantaWeaveConfig:
    return QuantaWeaveConfig.from_dict(json.loads((Path(directory) / "config.json").read_text()))


def load_model(directory: Path, device: torch.device, precision: str = "auto", with_payload: bool = False):
    """Build the model of ``directory`` on ``device`` and load its weights (quantised checkpoints included)."""
    from ..models.model import QuantaWeaveMoEForCausalLM

    directory = Path(directory)
    config = read_config(directory)
    payload = load_checkpoint(directory / "model.pt", map_location="cpu")
    state = payload["model"] if "model" in payload else payload["state_dict"]
    model = QuantaWeaveMoEForCausalLM(config)
    if "bits" in payload:  # a quantised export
        from ..inference.quantization import quantize_model

        quantize_model(model, payload["bits"], payload.get("group_size"), payload.get("quantize_lm_head", False))
    model.load_state_dict(state)
    model = model.to(device).eval()
    if device.type == "cuda" and precision in ("auto", "bf16"):
        from ..training.native import prepare_model

        prepare_model(model, "bf16")
    return (model, payload) if with_payload else model


def synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)
