"""Fine-tune a (quantised) checkpoint with LoRA adapters: QLoRA for the MoE.

    python -m quantaweave_b200.tools.finetune --checkpoint artifacts/outputs/quantweave-moe-out \\
        --data new_domain.jsonl --output artifacts/outputs/qlora --bits 4 --rank 8 --steps 500 \\
        --merge-output artifacts/outputs/qlora-merged

Same CLI, public functions and output files as the reference ``src/finetune_quantweave_moe.py`` (``load_base`` :34,
``evaluate`` :41-53, ``load_finetuned`` :54-65, CLI :68-91, ``run_finetune`` :92-181): the base experts are quantised
to int4/int8 and frozen, and only the adapters (optionally also the routers and norms) train. The output directory
holds ``adapter.pt``, ``finetune_metadata.json`` and the config/tokenizer files, so ``load_finetuned`` rebuilds the
model from the untouched base checkpoint; ``--merge-output`` writes an ordinary full-precision checkpoint with the
adapters folded in. A run is a :class:`_FineTune` object whose stages run in order: prepare, measure, train,
measure again, write the outputs, archive.
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
    """Row-weighted mean loss over a fixed prefix of the dataset (its first ``batch_size * batches`` windows),
    so numbers taken before and after training compare like for like. Leaves the model in training mode."""
    from ..training.trainer import autocast_context

    model.eval()
    rows = range(min(len(dataset), batch_size * batches))
    weighted, seen = 0.0, 0
    for first in rows[::batch_size]:
        chunk = dataset.batch(range(first, min(rows.stop, first + batch_size))).to(device)
        with autocast_context(device, precision):
            weighted += float(model(chunk, labels=chunk)["loss"]) * len(chunk)
        seen += len(chunk)
    model.train()
    return weighted / seen if seen else 0.0


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


QUANTISED_BUFFERS = ("qweight", "scales", "q_gate_up", "s_gate_up", "q_down", "s_down")
COPIED_FILES = ("config.json", "vocab.json", "tokenizer.json", "tokenizer_meta.json", "tokenizer.model")


def _bytes(tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors)


class _FineTune:
    """One fine-tuning run, stage by stage; ``record`` becomes ``finetune_metadata.json``."""

    def __init__(self, args) -> None:
        self.args = args
        self.record: dict = {}

    def prepare(self) -> None:
        from ..data.pipeline import WindowDataset, build_corpus, load_tokenizer
        from ..inference.quantization import quantize_model
        from ..training.trainer import select_device
        from ..utils.hardware import choose_precision, detect

        a = self.args
        self.device = select_device(a.device)
        random.seed(a.seed)
        torch.manual_seed(a.seed)
        self.tokenizer = load_tokenizer(a.checkpoint)
        self.model = load_base(a.checkpoint, self.device)
        context = self.model.config.max_sequence_length - 1
        if a.sequence_length > context:
            raise ValueError(f"--sequence-length {a.sequence_length} exceeds the checkpoint's context {context}")
        self.dataset = WindowDataset(build_corpus([a.data], self.tokenizer, a.examples), a.sequence_length)
        if len(self.dataset) == 0:
            raise ValueError("the fine-tuning data holds fewer tokens than one window")
        self.precision = choose_precision(detect(self.device.type), a.precision)
        full_bytes = _bytes(self.model.parameters())
        quantisation = quantize_model(self.model, a.bits, a.group_size) if a.bits else None
        self.adapters = add_lora(self.model, a.rank, a.alpha, a.include_lm_head, a.train_router, a.train_norms)
        packed = [b for name, b in self.model.named_buffers() if name.rsplit(".", 1)[-1] in QUANTISED_BUFFERS]
        total = self.adapters["total_parameters"]
        self.record.update(
            base_checkpoint=str(a.checkpoint), bits=a.bits, group_size=a.group_size, rank=a.rank, alpha=a.alpha,
            include_lm_head=a.include_lm_head, train_router=a.train_router, train_norms=a.train_norms,
            optimizer=a.optimizer, steps=a.steps, trainable_parameters=self.adapters["trainable_parameters"],
            total_parameters=total, trainable_fraction=self.adapters["trainable_parameters"] / total,
            fp32_parameter_bytes=full_bytes,
            quantized_model_bytes=_bytes(self.model.parameters()) + _bytes(packed), quantization=quantisation)

    def measure(self, key: str) -> None:
        self.record[key] = evaluate(self.model, self.dataset, self.device, self.precision)

    def train(self) -> None:
        from ..data.pipeline import BatchStream
        from ..training.trainer import autocast_context, build_optimizer

        a = self.args
        params = [p for p in self.model.parameters() if p.requires_grad]
        optimizer = build_optimizer(a.optimizer, params, a.lr, device=self.device)
        batches = BatchStream(self.dataset, a.batch_size, a.seed)
        self.model.train()
        clock = time.perf_counter()
        for step in range(1, a.steps + 1):
            tokens = batches.batch(step)[0].to(self.device)
            with autocast_context(self.device, self.precision):
                loss = self.model(tokens, labels=tokens)["loss"]
            optimizer.zero_grad(set_to_none=True)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(params, 1.0)
            optimizer.step()
            if step == a.steps or step % 10 == 0:
                print(f"finetune step={step}/{a.steps} loss={float(loss.detach()):.4f}")
        self.record["seconds"] = time.perf_counter() - clock
        on_gpu = self.device.type == "cuda"
        self.record["peak_device_bytes"] = torch.cuda.max_memory_allocated(self.device) if on_gpu else None

    def write(self) -> None:
        from ..training.trainer import write_checkpoint_metadata
        from .common import read_config

        a = self.args
        a.output.mkdir(parents=True, exist_ok=True)
        save_adapter(self.model, a.output / "adapter.pt", self.adapters, str(a.checkpoint))
        ordered = {key: self.record[key] for key in METADATA_KEYS}
        (a.output / "finetune_metadata.json").write_text(json.dumps(ordered, indent=2, default=str) + "\n")
        for name in COPIED_FILES:
            if (a.checkpoint / name).exists():
                shutil.copy(a.checkpoint / name, a.output / name)
        if a.merge_output is None:
            return
        weights = {name: tensor.cpu() for name, tensor in merge_lora_state(self.model).items()}
        a.merge_output.mkdir(parents=True, exist_ok=True)
        torch.save({"model": weights, "optimizer": None, "step": None, "rng_state": {},
                    "extra": {"merged_from": str(a.output)}}, a.merge_output / "model.pt")
        vocab = self.tokenizer.vocab if self.tokenizer.kind == "char" else self.tokenizer
        write_checkpoint_metadata(a.merge_output, read_config(a.checkpoint), vocab, 0, None)

    def archive(self, started_at: float) -> None:
        a = self.args
        if getattr(a, "archive_dir", None) is None or a.no_archive:
            return
        models = {"adapter": a.output}
        if a.merge_output is not None:
            models["merged"] = a.merge_output
        summary = {**self.record, "final_loss": self.record["loss_after"], "steps": a.steps}
        command = reproduce_command("quantaweave_b200.tools.finetune", build_parser(), a,
                                    skip=("archive_dir", "no_archive"))
        bundle = create_run_bundle(a.archive_dir, kind="finetune", model_dirs=models, benchmark_model=a.merge_output,
                                   data_paths=[a.data], options=vars(a), summary=summary, started=started_at,
                                   finished=time.time(), reproduce=command, skip_rows=a.examples,
                                   benchmark_examples=a.archive_benchmark_examples, device=a.device,
                                   precision=a.precision, data_limit_mb=a.archive_data_limit_mb,
                                   data_card=a.data_card)
        self.record["archive"] = str(bundle)
        print(f"archived run to {bundle}")


# the keys of finetune_metadata.json, in file order
METADATA_KEYS = ("base_checkpoint", "bits", "group_size", "rank", "alpha", "include_lm_head", "train_router",
                 "train_norms", "optimizer", "steps", "trainable_parameters", "total_parameters",
                 "trainable_fraction", "fp32_parameter_bytes", "quantized_model_bytes", "quantization",
                 "loss_before", "loss_after", "seconds", "peak_device_bytes")


def run_finetune(args) -> dict:
    """Quantise, attach adapters, train them, and write the adapter directory (plus optional merged checkpoint
    and run archive). Returns the metadata record."""
    started_at = time.time()
    run = _FineTune(args)
    run.prepare()
    run.measure("loss_before")
    run.train()
    run.measure("loss_after")
    run.write()
    run.archive(started_at)
    return run.record


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    resolve_archive_dir(args)
    metadata = run_finetune(args)
    print(json.dumps({k: metadata[k] for k in ("loss_before", "loss_after", "trainable_fraction",
                                               "fp32_parameter_bytes", "quantized_model_bytes")}, indent=2))


if __name__ == "__main__":
    main()
