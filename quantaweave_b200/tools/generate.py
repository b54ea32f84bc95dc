"""Plain full-context sampling from a checkpoint, without a KV cache.

Same behaviour and CLI as the reference ``src/generate_quantweave_moe.py`` (``sample_text`` :16-33, ``main``
:36-51): the prompt's ids (the tokenizer's ``unk`` id when it encodes to nothing) seed the sequence; every step
re-runs the model on the newest ``max_sequence_length - 1`` ids (the trainer never trains the last position of a
window), excludes ids the tokenizer cannot produce, samples from ``softmax(logits / max(T, 0.01))`` and stops
after ``<eos>``. This is the simple reference loop; ``inference.fast_decode.FastDecoder`` is the cached decoder.
"""

from __future__ import annotations

import argparse
from pathlib import Path

import torch


def _producible(logit_count: int, tokenizer_vocab: int, device) -> torch.Tensor:
    """Additive logit mask: 0 for ids the tokenizer can emit, -inf for the model's extra (never trained) rows."""
    mask = torch.zeros(logit_count, device=device)
    mask[tokenizer_vocab:] = float("-inf")
    return mask


def sample_text(model, tokenizer, prompt: str, tokens: int, temperature: float, device: torch.device,
                precision: str = "auto") -> str:
    """Sample up to ``tokens`` ids after ``prompt`` and return the decoded prompt plus continuation."""
    from ..training.trainer import autocast_context

    sequence = torch.tensor(tokenizer.encode(prompt) or [tokenizer.unk_id], dtype=torch.long, device=device)
    window = model.config.max_sequence_length - 1
    inverse_temperature = 1.0 / max(temperature, 0.01)
    mask = None
    with torch.inference_mode():
        for _ in range(tokens):
            with autocast_context(device, precision):
                last = model(sequence[-window:].unsqueeze(0))["logits"][0, -1].float()
            if mask is None:
                mask = _producible(last.numel(), tokenizer.vocab_size, device)
            probabilities = torch.softmax((last + mask) * inverse_temperature, dim=-1)
            chosen = torch.multinomial(probabilities, 1)
            sequence = torch.cat((sequence, chosen))
            if int(chosen) == tokenizer.eos_id:
                break
    return tokenizer.decode(sequence.tolist())


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    p.add_argument("--prompt", default="Once upon a time")
    p.add_argument("--tokens", type=int, default=300)
    p.add_argument("--temperature", type=float, default=0.8)
    p.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    p.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    from .common import describe_options

    describe_options(p)
    return p


def main(argv=None) -> None:
    from ..data.pipeline import load_tokenizer
    from ..training.trainer import select_device
    from .common import load_model

    args = build_parser().parse_args(argv)
    device = select_device(args.device)
    model = load_model(args.checkpoint, device, args.precision)
    print(sample_text(model, load_tokenizer(args.checkpoint), args.prompt, args.tokens, args.temperature, device,
                      args.precision))


if __name__ == "__main__":
    main()
