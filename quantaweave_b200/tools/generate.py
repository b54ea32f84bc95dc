"""Plain full-context sampling from a checkpoint (no KV cache).

Parity with the reference ``src/generate_quantweave_moe.py`` (``sample_text`` :16-33, CLI :36-51): encode the prompt
(``unk`` if empty), keep the last ``max_sequence_length - 1`` tokens as context, mask logits of ids beyond the
tokenizer's vocabulary, sample from ``softmax(logits / max(T, 0.01))`` and stop at ``<eos>``. For cached decoding use
``quantaweave_b200.inference.fast_decode.FastDecoder``.
"""

from __future__ import annotations

import argparse
from pathlib import Path

import torch


def sample_text(model, tokenizer, prompt: str, tokens: int, temperature: float, device: torch.device,
                precision: str = "auto") -> str:
    from ..training.trainer import autocast_context

    generated = tokenizer.encode(prompt) or [tokenizer.unk_id]
    context = model.config.max_sequence_length - 1  # the last position of a training window is never trained
    with torch.inference_mode():
        for _ in range(tokens):
            window = torch.tensor([generated[-context:]], dtype=torch.long, device=device)
            with autocast_context(device, precision):
                logits = model(window)["logits"][:, -1, :].float()
            logits[:, tokenizer.vocab_size:] = float("-inf")  # ids the tokenizer never produced are untrained
            probs = (logits / max(temperature, 0.01)).softmax(dim=-1)
            next_id = int(torch.multinomial(probs, 1).item())
            generated.append(next_id)
            if next_id == tokenizer.eos_id:
                break
    return tokenizer.decode(generated)


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
    tokenizer = load_tokenizer(args.checkpoint)
    print(sample_text(model, tokenizer, args.prompt, args.tokens, args.temperature, device, args.precision))


if __name__ == "__main__":
    main()
