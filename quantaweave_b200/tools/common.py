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


def load_model(checkpoint: Path, device: torch.device, precision: str = "auto", with_payload: bool = False):
    """Build the model of ``checkpoint`` on ``device`` and load its weights (quantised checkpoints included)."""
    from ..models.model import QuantaWeaveMoEForCausalLM

    checkpoint = Path(checkpoint)
    config = read_config(checkpoint)
    payload = load_checkpoint(checkpoint / "model.pt", map_location="cpu")
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


# Help text shared by the command-line tools, by option name; ``describe_options`` attaches it (with the default).
OPTION_HELP = {
    "checkpoint": "checkpoint directory (model.pt, config.json, tokenizer files)",
    "student": "checkpoint directory of the student model",
    "teacher_data": "JSONL text the student is distilled on",
    "data": "JSONL rows to read",
    "output": "directory written with the result",
    "checkpoint_dir": "directory of the resumable checkpoint",
    "runs_dir": "folder of archived runs (searched by --run and --latest)",
    "mode": "complete: continue the text; chat: User/Assistant turns with history",
    "top_k": "sample only from the k most likely tokens (0: off)",
    "top_p": "sample only from the smallest set of tokens whose probability reaches p (1: off)",
    "temperature": "sampling temperature (0: greedy)",
    "prompt": "text to continue",
    "tokens": "tokens to generate",
    "precision": "compute precision (auto: bf16 on CUDA, fp32 on CPU)",
    "device": "where to run (auto: CUDA when available)",
    "host": "interface to listen on",
    "port": "TCP port",
    "rate_limit_window": "seconds of the --rate-limit sliding window",
    "log_format": "request log lines as text or one JSON object per line",
    "group_size": "quantisation group size (default: per row for int8, 32 for int4)",
    "rank": "LoRA rank",
    "alpha": "LoRA scaling numerator (the update is scaled by alpha / rank)",
    "include_lm_head": "also adapt the LM head",
    "train_router": "also train the routers",
    "train_norms": "also train the normalisation weights",
    "optimizer": "AdamW, or AdamW with 8-bit moments (CUDA)",
    "steps": "optimizer steps",
    "checkpoint_interval": "steps between checkpoints (0: only at the end)",
    "batch_size": "sequences per step",
    "sequence_length": "tokens per training window",
    "examples": "rows read from each data file",
    "lr": "learning rate",
    "seed": "random seed",
    "resume": "continue from --checkpoint-dir when it holds a checkpoint",
    "config": "YAML or JSON configuration file",
    "name": "name of the run (default: the config's name)",
    "runs": "run directories to compare",
    "metric": "dotted path of the value to rank by (lower is better)",
    "markdown": "also write the comparison table to this file",
    "vocab_size": "vocabulary size",
    "hidden_size": "model width",
    "layers": "transformer blocks",
    "ffn_size": "hidden width of each expert",
    "total_experts": "experts per MoE layer",
    "active_experts": "experts per token (top-k)",
    "attention_heads": "attention heads",
    "capacity_factor": "per-expert capacity factor (0: unlimited)",
    "min_expert_capacity": "lower bound of the per-expert capacity",
}


def describe_options(parser, extra: dict | None = None) -> None:
    """Give every option of ``parser`` that has no help text the shared (or ``extra``) description."""
    import argparse

    table = {**OPTION_HELP, **(extra or {})}
    for action in parser._actions:
        if isinstance(action, argparse._SubParsersAction):
            for sub in action.choices.values():
                describe_options(sub, extra)
            continue
        if action.help is None and action.dest in table:
            default = action.default
            shown = "" if default in (None, False) or isinstance(default, bool) else f" (default: {default})"
            action.help = table[action.dest] + shown
