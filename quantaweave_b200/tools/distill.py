"""Distil into a QuantaWeave student checkpoint.

Three modes, as in the reference ``src/distill_quantweave_moe.py`` (``distillation_loss`` :43-49, CLI :60-84,
``run_distillation`` :85-191):

* sequence-level (default): the student trains on teacher-generated text in ``--teacher-data``;
* logit-level (``--teacher-checkpoint``): a frozen checkpoint with the same tokenizer scores the same batches and the
  student minimises ``ce + alpha * T^2 * KL(teacher || student)``;
* cross-tokenizer (``--hf-teacher``): a Hugging Face causal LM scores the same text, aligned on token boundaries
  (``quantaweave_b200.tools.cross_tokenizer``).

The student starts from its trained weights with a fresh optimizer (the fused AdamW on CUDA) and resumes from
``--checkpoint-dir`` when one exists.
"""

from __future__ import annotations

import argparse
import random
import time
from pathlib import Path
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor

from .common import load_model  # noqa: F401  (the reference exposes it from its distillation module)
from .run_bundle import add_archive_arguments, create_run_bundle, reproduce_command, resolve_archive_dir


def distillation_loss(student_logits: Tensor, teacher_logits: Tensor, temperature: float,
                      chunk_rows: int = 8192) -> Tensor:
    """Per-token KL(teacher || student) at ``temperature`` times T^2, over every position but the last (the positions
    the LM loss scores), averaged over positions. Rows are processed in chunks so the fp32 softmax of a large
    vocabulary never exists for the whole batch at once."""
    vocab = student_logits.size(-1)
    s_all = student_logits[:, :-1].reshape(-1, vocab)
    t_all = teacher_logits[:, :-1].reshape(-1, vocab)
    total = s_all.new_zeros((), dtype=torch.float32)
    for start in range(0, s_all.size(0), chunk_rows):
        s = F.log_softmax(s_all[start:start + chunk_rows].float() / temperature, dim=-1)
        t = F.softmax(t_all[start:start + chunk_rows].float() / temperature, dim=-1)
        total = total + F.kl_div(s, t, reduction="sum")
    return total / max(1, s_all.size(0)) * temperature ** 2


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--student", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    p.add_argument("--teacher-data", type=Path, required=True)
    p.add_argument("--teacher-checkpoint", type=Path, help="distil towards the logits of this model (same tokenizer)")
    p.add_argument("--hf-teacher", help="a Hugging Face causal language model (folder or hub name) that brings its own tokenizer")
    p.add_argument("--cross-loss", choices=("auto", "marginal", "uld"), default="auto",
                   help="how --hf-teacher is matched: the next-character marginal (character students) or the ULD sorted-probability distance")
    p.add_argument("--alpha", type=float, default=1.0, help="multiplier of the distillation term added to the language-model loss")
    p.add_argument("--temperature", type=float, default=2.0, help="softmax temperature of the KL term")
    p.add_argument("--output", type=Path, default=Path("artifacts/outputs/quantweave-moe-distilled"))
    p.add_argument("--checkpoint-dir", type=Path, default=Path("artifacts/checkpoints/quantweave-distill"))
    p.add_argument("--steps", type=int, default=10000)
    p.add_argument("--checkpoint-interval", type=int, default=1000)
    p.add_argument("--examples", type=int, default=100000)
    p.add_argument("--sequence-length", type=int, default=128)
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--lr", type=float, default=1e-4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    p.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    p.add_argument("--resume", action=argparse.BooleanOptionalAction, default=True)
    add_archive_arguments(p)
    from .common import describe_options

    describe_options(p)
    return p


def run_distillation(args) -> dict:
    from ..data.pipeline import BatchStream, WindowDataset, build_corpus, load_tokenizer
    from ..models.model import QuantaWeaveMoEForCausalLM
    from ..training.trainer import (autocast_context, build_optimizer, checkpoint_exists, load_checkpoint,
                                    save_checkpoint, select_device, tokenizer_hash, tokenizer_payload)
    from ..utils.checkpoint_io import load_checkpoint as load_file
    from .common import load_model, read_config
    from .cross_tokenizer import CrossTokenizerLoss, HFTeacher

    started = time.time()
    device = select_device(args.device)
    for path in (args.student / "config.json", args.student / "model.pt"):
        if not path.exists():
            raise FileNotFoundError(f"missing student file: {path}")
    if args.hf_teacher and args.teacher_checkpoint:
        raise ValueError("choose one teacher: --teacher-checkpoint or --hf-teacher")
    random.seed(args.seed)
    torch.manual_seed(args.seed)
    config = read_config(args.student)
    tokenizer = load_tokenizer(args.student)
    if args.sequence_length + 1 > config.max_sequence_length:
        raise ValueError(f"--sequence-length {args.sequence_length} needs max_sequence_length >= "
                         f"{args.sequence_length + 1}, but the student has {config.max_sequence_length}")
    dataset = WindowDataset(build_corpus([args.teacher_data], tokenizer, args.examples), args.sequence_length)
    if len(dataset) == 0:
        raise ValueError("teacher dataset holds fewer tokens than one training window")
    stream = BatchStream(dataset, args.batch_size, args.seed)

    teacher: Optional[torch.nn.Module] = None
    if args.teacher_checkpoint is not None:
        teacher = load_model(args.teacher_checkpoint, device, args.precision)
        teacher_tok = load_tokenizer(args.teacher_checkpoint)
        if tokenizer_hash(teacher_tok) != tokenizer_hash(tokenizer) or teacher.config.vocab_size != config.vocab_size:
            raise ValueError("logit distillation needs the teacher and student to share a tokenizer and vocabulary "
                             f"size (teacher vocab {teacher.config.vocab_size}, student vocab {config.vocab_size})")
        if args.sequence_length + 1 > teacher.config.max_sequence_length:
            raise ValueError("teacher max_sequence_length is shorter than the distillation sequence length")
        for p in teacher.parameters():
            p.requires_grad_(False)
    cross = CrossTokenizerLoss(HFTeacher(args.hf_teacher, device), tokenizer, args.cross_loss) \
        if args.hf_teacher else None

    model = QuantaWeaveMoEForCausalLM(config).to(device)
    if device.type == "cuda":
        from ..training.native import prepare_model

        prepare_model(model, "bf16")
    resume = args.resume and checkpoint_exists(args.checkpoint_dir)
    if not resume:  # weights first: the fused optimizer snapshots fp32 master copies when it is built
        model.load_state_dict(load_file(args.student / "model.pt", map_location="cpu")["model"])
        print(f"initialised from student weights at {args.student / 'model.pt'}")
    optimizer = build_optimizer("adamw", list(model.parameters()), args.lr, device=device)
    start_step = 0
    if resume:
        start_step = load_checkpoint(args.checkpoint_dir, model, optimizer, device)
        print(f"resumed distillation from step {start_step}")
    mode = "cross-tokenizer" if cross is not None else "logit" if teacher is not None else "sequence"
    print(f"distillation mode: {mode}")
    model.train()
    last: dict = {}
    for step in range(start_step + 1, args.steps + 1):
        batch, _ = stream.batch(step)
        batch = batch.to(device)
        with autocast_context(device, args.precision):
            out = model(batch, labels=batch, return_logits=teacher is not None or cross is not None)
            kl, cross_stats = None, None
            if teacher is not None:
                with torch.no_grad():
                    teacher_logits = teacher(batch)["logits"]
                kl = distillation_loss(out["logits"], teacher_logits, args.temperature)
            elif cross is not None:
                kl, cross_stats = cross(out["logits"], batch)
        loss = out["loss"] + (args.alpha * kl if kl is not None else 0.0)
        optimizer.zero_grad(set_to_none=True)
        loss.backward()
        if hasattr(optimizer, "clip_grad_norm_"):
            optimizer.clip_grad_norm_(1.0)
        else:
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        optimizer.step()
        last = {"loss": float(loss.detach()), "ce_loss": float(out["loss"].detach()),
                "kl": float(kl.detach()) if kl is not None else None}
        note = f" kl={last['kl']:.4f}" if kl is not None else ""
        if cross_stats is not None:
            last["aligned_fraction"] = cross_stats["aligned_fraction"]
            note += f" aligned={cross_stats['aligned_fraction']:.0%}"
        print(f"distill_step={step}/{args.steps} loss={last['loss']:.4f}{note} "
              f"router_aux={float(out['router_aux_loss'].detach()):.4f}")
        if args.checkpoint_interval > 0 and step % args.checkpoint_interval == 0:
            save_checkpoint(args.checkpoint_dir, model, optimizer, step, tokenizer_payload(tokenizer), device)
            print(f"distillation checkpoint saved at step {step}")
    save_checkpoint(args.output, model, optimizer, args.steps, tokenizer_payload(tokenizer), device)
    print(f"distilled student saved to {args.output}")
    result = {"mode": mode, "steps": args.steps, **last}
    if getattr(args, "archive_dir", None) is not None and not args.no_archive:
        bundle = create_run_bundle(
            args.archive_dir, kind="distill", model_dirs={"model": args.output}, benchmark_model=args.output,
            data_paths=[args.teacher_data], options=vars(args), summary={**result, "final_loss": result.get("loss")},
            started=started, finished=time.time(),
            reproduce=reproduce_command("quantaweave_b200.tools.distill", build_parser(), args,
                                        skip=("archive_dir", "no_archive")),
            skip_rows=args.examples, benchmark_examples=args.archive_benchmark_examples, device=args.device,
            precision=args.precision, data_limit_mb=args.archive_data_limit_mb, data_card=args.data_card)
        result["archive"] = str(bundle)
        print(f"archived run to {bundle}")
    return result


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    resolve_archive_dir(args)
    run_distillation(args)


if __name__ == "__main__":
    main()
