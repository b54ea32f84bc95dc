"""Fine-tune a (quantised) checkpoint with LoRA adapters: QLoRA for the MoE.

    python -m quantaweave_b200.tools.finetune --checkpoint artifacts/outputs/quantweave-moe-out \\
        --data new_domain.jsonl --output artifacts/outputs/qlora --bits 4 --rank 8 --steps 500 \\
        --merge-output artifacts/outputs/qlora-merged

Parity with the reference ``src/finetune_quantweave_moe.py`` (``load_base`` :34, ``evaluate`` :41-53,
``load_finetuned`` :54-65, CLI :68-91, ``run_finetune`` :92-181): experts quantised to int4/int8 and frozen, only the
adapters (and optionally routers/norms) train; the output directory holds ``adapter.pt``,
``finetune_metadata.json`` and the config/tokenizer files so ``load_finetuned`` rebuilds the model from the untouched
base checkpoint; ``--merge-output`` writes an ordinary full-precision checkpoint with the adapters folded in.
"""

from __future__ import annotations

import argparse
import json
import random
import shutil
import time
from pathlib import Path
from typing import Optional

import torch

from .lora import add_lora, load_adapter, merge_lora_state, save_adapter
from .run_bundle import add_archive_arguments, create_run_bundle, reproduce_command, resolve_archive_dir


def load_base(checkpoint: Path, device: torch.device):
    """The base model in fp32 (the fine-tune trains fp32 adapters on the per-expert path)."""
    from ..models.model import QuantaWeaveMoEForCausalLM
    from ..utils.checkpoint_io import load_checkpoint
    from .common import read_config

    model = QuantaWeaveMoEForCausalLM(read_config(checkpoint))
    model.load_state_dict(load_checkpoint(Path(checkpoint) / "model.pt", map_location="cpu")["model"])
    return model.to(device)


@torch.no_grad()
def evaluate(model, dataset, device: torch.device, precision: str, batch_size: int = 8, batches: int = 8) -> float:
    """Mean loss over the first ``batches`` batches of windows (fixed, so before/after numbers compare)."""
    from ..training.trainer import autocast_context

    model.eval()
    total, count = 0.0, 0
    for start in range(0, min(len(dataset), batch_size * batches), batch_size):
        batch = dataset.batch(range(start, min(len(dataset), start + batch_size))).to(device)
        with autocast_context(device, precision):
            total += float(model(batch, labels=batch)["loss"]) * batch.size(0)
        count += batch.size(0)
    model.train()
    return total / max(1, count)


def load_finetuned(base_checkpoint: Path, adapter_dir: Path, device: Optional[torch.device] = None):
    """Base checkpoint, quantised as it was trained, plus the saved adapter."""
    from ..inference.quantization import quantize_model

    device = device or torch.device("cpu")
    info = json.loads((Path(adapter_dir) / "finetune_metadata.json").read_text())
    model = load_base(base_checkpoint, device)
    if info["bits"]:
        quantize_model(model, info["bits"], info.get("group_size"))
    add_lora(model, info["rank"], info["alpha"], info["include_lm_head"], info["train_router"], info["train_norms"])
    load_adapter(model, Path(adapter_dir) / "adapter.pt")
    return model.eval()


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, required=True)
    p.add_argument("--data", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--merge-output", type=Path, help="also write a full-precision checkpoint with the adapters merged")
    p.add_argument("--bits", type=int, choices=(0, 4, 8), default=4, help="quantise the base experts (0 = keep fp32)")
    p.add_argument("--group-size", type=int)
    p.add_argument("--rank", type=int, default=8)
    p.add_argument("--alpha", type=float, default=16.0)
    p.add_argument("--include-lm-head", action="store_true")
    p.add_argument("--train-router", action="store_true")
    p.add_argument("--train-norms", action="store_true")
    p.add_argument("--optimizer", choices=("adamw", "adamw8bit"), default="adamw")
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--sequence-length", type=int, default=128)
    p.add_argument("--examples", type=int, default=20000)
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    p.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    add_archive_arguments(p)
    from .common import describe_options

    describe_options(p)
    return p


def run_finetune(args) -> dict:
    from ..data.pipeline import BatchStream, WindowDataset, build_corpus, load_tokenizer
    from ..inference.quantization import quantize_model
    from ..training.trainer import autocast_context, build_optimizer, select_device, write_checkpoint_metadata
    from ..utils.hardware import choose_precision, detect
    from .common import read_config

    started_at = time.time()
    device = select_device(args.device)
    random.seed(args.seed)
    torch.manual_seed(args.seed)
    tokenizer = load_tokenizer(args.checkpoint)
    model = load_base(args.checkpoint, device)
    if args.sequence_length + 1 > model.config.max_sequence_length:
        raise ValueError(f"--sequence-length {args.sequence_length} exceeds the checkpoint's context "
                         f"{model.config.max_sequence_length - 1}")
    dataset = WindowDataset(build_corpus([args.data], tokenizer, args.examples), args.sequence_length)
    if len(dataset) == 0:
        raise ValueError("the fine-tuning data holds fewer tokens than one window")
    precision = choose_precision(detect(device.type), args.precision)
    fp32_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    quant = quantize_model(model, args.bits, args.group_size) if args.bits else None
    info = add_lora(model, args.rank, args.alpha, args.include_lm_head, args.train_router, args.train_norms)
    base_loss = evaluate(model, dataset, device, precision)
    quantized_bytes = sum(p.numel() * p.element_size() for p in model.parameters()) + sum(
        b.numel() * b.element_size() for n, b in model.named_buffers()
        if n.split(".")[-1] in ("qweight", "scales", "q_gate_up", "s_gate_up", "q_down", "s_down"))
    trainable = [p for p in model.parameters() if p.requires_grad]
    optimizer = build_optimizer(args.optimizer, trainable, args.lr, device=device)
    stream = BatchStream(dataset, args.batch_size, args.seed)
    model.train()
    losses = []
    started = time.perf_counter()
    for step in range(1, args.steps + 1):
        batch, _ = stream.batch(step)
        batch = batch.to(device)
        with autocast_context(device, precision):
            loss = model(batch, labels=batch)["loss"]
        optimizer.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(trainable, 1.0)
        optimizer.step()
        losses.append(float(loss.detach()))
        if step % 10 == 0 or step == args.steps:
            print(f"finetune step={step}/{args.steps} loss={losses[-1]:.4f}")
    final_loss = evaluate(model, dataset, device, precision)

    args.output.mkdir(parents=True, exist_ok=True)
    metadata = {
        "base_checkpoint": str(args.checkpoint), "bits": args.bits, "group_size": args.group_size, "rank": args.rank,
        "alpha": args.alpha, "include_lm_head": args.include_lm_head, "train_router": args.train_router,
        "train_norms": args.train_norms, "optimizer": args.optimizer, "steps": args.steps,
        "trainable_parameters": info["trainable_parameters"], "total_parameters": info["total_parameters"],
        "trainable_fraction": info["trainable_parameters"] / info["total_parameters"],
        "fp32_parameter_bytes": fp32_bytes, "quantized_model_bytes": quantized_bytes, "quantization": quant,
        "loss_before": base_loss, "loss_after": final_loss, "seconds": time.perf_counter() - started,
        "peak_device_bytes": torch.cuda.max_memory_allocated(device) if device.type == "cuda" else None,
    }
    save_adapter(model, args.output / "adapter.pt", info, str(args.checkpoint))
    (args.output / "finetune_metadata.json").write_text(json.dumps(metadata, indent=2, default=str) + "\n")
    for name in ("config.json", "vocab.json", "tokenizer.json", "tokenizer_meta.json", "tokenizer.model"):
        if (args.checkpoint / name).exists():
            shutil.copy(args.checkpoint / name, args.output / name)
    if args.merge_output is not None:
        merged = merge_lora_state(model)
        args.merge_output.mkdir(parents=True, exist_ok=True)
        torch.save({"model": {k: v.cpu() for k, v in merged.items()}, "optimizer": None, "step": None,
                    "rng_state": {}, "extra": {"merged_from": str(args.output)}}, args.merge_output / "model.pt")
        write_checkpoint_metadata(args.merge_output, read_config(args.checkpoint),
                                  tokenizer.vocab if tokenizer.kind == "char" else tokenizer, 0, None)
    if getattr(args, "archive_dir", None) is not None and not args.no_archive:
        models = {"adapter": args.output, **({"merged": args.merge_output} if args.merge_output is not None else {})}
        bundle = create_run_bundle(
            args.archive_dir, kind="finetune", model_dirs=models, benchmark_model=args.merge_output,
            data_paths=[args.data], options=vars(args),
            summary={**metadata, "final_loss": metadata["loss_after"], "steps": args.steps}, started=started_at,
            finished=time.time(),
            reproduce=reproduce_command("quantaweave_b200.tools.finetune", build_parser(), args,
                                        skip=("archive_dir", "no_archive")),
            skip_rows=args.examples, benchmark_examples=args.archive_benchmark_examples, device=args.device,
            precision=args.precision, data_limit_mb=args.archive_data_limit_mb, data_card=args.data_card)
        metadata["archive"] = str(bundle)
        print(f"archived run to {bundle}")
    return metadata


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    resolve_archive_dir(args)
    metadata = run_finetune(args)
    print(json.dumps({k: metadata[k] for k in ("loss_before", "loss_after", "trainable_fraction",
                                               "fp32_parameter_bytes", "quantized_model_bytes")}, indent=2))


if __name__ == "__main__":
    main()
