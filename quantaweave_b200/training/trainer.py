"""``run_training``: the training entry point (library and CLI).

Behaviour follows the reference trainer ``src/train_quantweave_moe.py`` (``build_parser`` :279-405, ``default_args``
:408, ``run_training`` :462-886, ``save_checkpoint`` :58-108, ``load_checkpoint`` :123-144, ``resume_fields``
:249-264): the same option names, option validation, resume fingerprint, atomic checkpoint directory
(``.name.tmp`` → ``.name.previous`` → ``name``), RNG restore, controller/straggler/scaler state in ``extra``, metrics
log, routing diagnostics, power tracking and run archiving.

B200 differences:

* on CUDA with bf16 the model holds bf16 matrices (router and norms stay fp32) and ``FusedAdamW`` keeps fp32
  master weights and moments, with the gradient-norm clip folded into the fused update;
* the loss is a fused linear-cross-entropy (no full logits), and per-step host reads are limited to what the
  logger and controllers need;
* extra options: synthetic seeded data (uniform / Zipf), RMSNorm/RoPE/GQA architecture switches, AdamW betas and
  weight decay, ``--data-parallel`` for plain DP, and ``--preset`` for the named benchmark architectures.
"""

from __future__ import annotations

import argparse
import contextlib
import hashlib
import json
import os
import random
import shutil
import tempfile
import time
from pathlib import Path
from typing import Optional

import torch

from ..config import PRESETS, QuantaWeaveConfig
from ..data.pipeline import (BatchStream, BPETokenizer, CharTokenizer, CurriculumConfig, DomainMixture,
                             SentencePieceTokenizer, SyntheticTokenStream, WindowDataset, build_corpus,
                             difficulty_scores, load_token_bin, load_tokenizer, parse_domain_weights, read_rows,
                             token_classes)
from ..models.model import QuantaWeaveMoEForCausalLM
from ..utils.checkpoint_io import load_checkpoint as load_checkpoint_file
from ..utils.tracing import nvtx_range
from ..utils.hardware import choose_precision, detect, find_safe_batch_size, parameter_counts
from .metrics import MetricsLogger
from .schedules import ScheduleConfig, TrainingController

MUTABLE_CONFIG_FIELDS = {"capacity_factor", "drop_overflow_tokens", "overflow_policy", "router_temperature",
                         "router_aux_loss_coef"}


# ------------------------------------------------------------------------------------------ checkpoints
def save_checkpoint(path: Path, model, optimizer, step: int, vocab, device: torch.device,
                    extra: Optional[dict] = None) -> None:
    """Atomically write model, optimizer, RNG, tokenizer and metadata into directory ``path``."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.tmp")
    if tmp.exists():
        shutil.rmtree(tmp)
    tmp.mkdir(parents=True)
    rng = {"python": random.getstate(), "torch": torch.get_rng_state()}
    if device.type == "cuda":
        rng["accelerator"] = torch.cuda.get_rng_state(device)
    torch.save({"model": model.state_dict(), "optimizer": optimizer.state_dict(), "step": step, "rng_state": rng,
                "extra": extra or {}}, tmp / "model.pt")
    write_checkpoint_metadata(tmp, model.config, vocab, step, extra)
    previous = path.with_name(f".{path.name}.previous")
    if previous.exists():
        shutil.rmtree(previous)
    if path.exists():
        path.rename(previous)
    try:
        tmp.rename(path)
    except Exception:
        if path.exists():
            shutil.rmtree(path)
        if previous.exists():
            previous.rename(path)
        raise
    if previous.exists():
        shutil.rmtree(previous)


def write_checkpoint_metadata(directory: Path, config: QuantaWeaveConfig, vocab, step: int, extra: Optional[dict]) -> None:
    directory = Path(directory)
    (directory / "config.json").write_text(json.dumps(config.__dict__, indent=2) + "\n")
    if isinstance(vocab, dict):
        (directory / "vocab.json").write_text(json.dumps(vocab, ensure_ascii=False, indent=2) + "\n")
        (directory / "tokenizer_meta.json").write_text(json.dumps({"type": "char"}) + "\n")
    elif vocab is not None:
        vocab.save(directory)
    if extra:
        meta = {"step": step, "torch": torch.__version__, "saved_at": time.strftime("%Y-%m-%dT%H:%M:%S"), **extra}
        (directory / "metadata.json").write_text(json.dumps(meta, indent=2, default=str) + "\n")


def load_checkpoint(path: Path, model, optimizer, device: torch.device, extra_out: Optional[dict] = None) -> int:
    """Restore weights, optimizer and RNG (falling back to ``.name.previous``); returns the step."""
    path = Path(path)
    file = path / "model.pt"
    if not file.exists():
        fallback = path.with_name(f".{path.name}.previous") / "model.pt"
        if not fallback.exists():
            raise FileNotFoundError(f"no valid checkpoint found under {path}")
        file = fallback
    ckpt = load_checkpoint_file(file, map_location=device)
    model.load_state_dict(ckpt["model"])
    if optimizer is not None and ckpt.get("optimizer") is not None:
        optimizer.load_state_dict(ckpt["optimizer"])
    restore_rng(ckpt.get("rng_state", {}), device)
    if extra_out is not None:
        extra_out.update(ckpt.get("extra", {}))
    return int(ckpt["step"])


def restore_rng(rng_state: dict, device: torch.device) -> None:
    if "python" in rng_state:
        random.setstate(rng_state["python"])
    if "torch" in rng_state:
        torch.set_rng_state(rng_state["torch"].cpu())
    if "accelerator" in rng_state and device.type == "cuda":
        torch.cuda.set_rng_state(rng_state["accelerator"].cpu(), device)


def checkpoint_exists(path: Path) -> bool:
    path = Path(path)
    return (path / "model.pt").exists() or (path.with_name(f".{path.name}.previous") / "model.pt").exists()


# ------------------------------------------------------------------------------------------ helpers
def select_device(requested: str) -> torch.device:
    if requested == "rocm":
        requested = "cuda"
    if requested != "auto":
        return torch.device(requested)
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


class StepScalars:
    """Per-step scalars (loss, aux, dropped, overflow, domain loss, overflow fraction) held on the device until a
    flush point, so steps between logging, controller and checkpoint steps never wait for the device (survey
    collective C12: device-side accumulation, the host reads at log intervals only)."""

    COLUMNS = 6
    REDUCED = (0, 5)  # loss and overflow fraction are averaged over the ranks that saw different tokens

    def __init__(self) -> None:
        self.rows: list = []

    def push(self, step: int, values: torch.Tensor, reduce: bool) -> None:
        self.rows.append((step, values, reduce))

    def flush(self, mean_over_ranks) -> list:
        """[(step, [6 floats])] in step order, with one device->host copy and at most one collective."""
        if not self.rows:
            return []
        stacked = torch.stack([v.to(self.rows[0][1].device) for _, v, _ in self.rows]).cpu().tolist()
        pick = [(i, c) for i, (_, _, reduce) in enumerate(self.rows) if reduce for c in self.REDUCED]
        if pick:
            averaged = mean_over_ranks([stacked[i][c] for i, c in pick])
            for (i, c), value in zip(pick, averaged):
                stacked[i][c] = value
        out = [(step, row) for (step, _, _), row in zip(self.rows, stacked)]
        self.rows.clear()
        return out


def autocast_context(device: torch.device, precision: str = "auto"):
    """CPU: optional bf16 autocast of the oracle path. CUDA: the native kernels choose their own dtypes (bf16
    operands, fp32 accumulation), so no autocast region is opened."""
    if precision == "auto":
        precision = "bf16" if device.type == "cuda" else "fp32"
    if precision == "fp32" or device.type == "cuda":
        return contextlib.nullcontext()
    return torch.autocast(device.type, dtype=torch.bfloat16 if precision == "bf16" else torch.float16)


def build_optimizer(kind: str, parameters, lr: float, betas=(0.9, 0.999), weight_decay: float = 0.01, device=None):
    """``adamw`` (fused sm_100a kernel with fp32 master weights on CUDA; torch AdamW on CPU), ``adamw8bit``
    (8-bit moments, fused kernel) or ``adamw_cpu_offload`` (moments in pinned host memory)."""
    parameters = list(parameters)
    on_cuda = any(p.is_cuda for p in parameters)
    if kind == "adamw":
        if on_cuda:
            from ..optim.adamw import FusedAdamW

            return FusedAdamW(parameters, lr=lr, betas=betas, weight_decay=weight_decay)
        return torch.optim.AdamW(parameters, lr=lr, betas=betas, weight_decay=weight_decay)
    if kind == "adamw8bit":
        if not on_cuda:
            raise RuntimeError("--optimizer adamw8bit needs a CUDA device")
        from ..optim.adamw import FusedAdamW

        return FusedAdamW(parameters, lr=lr, betas=betas, weight_decay=weight_decay, moment_bits=8)
    if kind == "adamw_cpu_offload":
        from ..optim.cpu_offload import CPUOffloadAdamW

        return CPUOffloadAdamW(parameters, lr=lr, betas=betas, weight_decay=weight_decay)
    raise ValueError("optimizer must be adamw, adamw8bit or adamw_cpu_offload")


def clip_grad_norm(model, optimizer, max_norm: float):
    """Global gradient norm; CUDA folds the clip coefficient into the fused optimizer step."""
    if hasattr(optimizer, "clip_grad_norm_"):
        return optimizer.clip_grad_norm_(max_norm)
    return torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm)


def tokenizer_hash(tokenizer) -> str:
    if tokenizer is None:
        return "synthetic"
    if isinstance(tokenizer, CharTokenizer):
        text = json.dumps(tokenizer.vocab, sort_keys=True)
    elif tokenizer.kind == "sentencepiece":
        text = tokenizer.processor.serialized_model_proto().hex()
    else:
        text = tokenizer.tokenizer.to_str()
    return hashlib.sha256(text.encode()).hexdigest()[:16]


def build_vocab(path: Path, vocab_size: int) -> dict:
    """Character vocabulary of a JSONL corpus (reference ``src/train_quantweave_moe.py:54-55``)."""
    return CharTokenizer.build((text for _, text in read_rows([Path(path)])), vocab_size).vocab


def tokenizer_payload(tokenizer):
    return tokenizer.vocab if isinstance(tokenizer, CharTokenizer) else tokenizer


def resume_fields(args, config: QuantaWeaveConfig, dataset, tokenizer, world_size: int) -> dict:
    fields = {k: v for k, v in config.__dict__.items() if k not in MUTABLE_CONFIG_FIELDS}
    fields.update(
        batch_size=args.batch_size, gradient_accumulation_steps=args.gradient_accumulation_steps,
        sequence_length=args.sequence_length, seed=args.seed, world_size=world_size,
        data_fingerprint=dataset.fingerprint(), tokenizer_hash=tokenizer_hash(tokenizer),
        curriculum=[args.curriculum, args.curriculum_steps, args.curriculum_start_fraction],
        domain_weights=[args.domain_weights, args.domain_weights_end, args.domain_weights_steps],
        parallel=[bool(args.expert_parallel), args.tensor_parallel, bool(args.pipeline_parallel), args.microbatches,
                  bool(args.shard_optimizer), args.pipeline_schedule, bool(getattr(args, "sequence_parallel", False))],
        optimizer=[args.optimizer, args.adam_beta1, args.adam_beta2, args.weight_decay],
    )
    return fields


def config_hash(fields: dict) -> str:
    return hashlib.sha256(json.dumps(fields, sort_keys=True, default=str).encode()).hexdigest()[:16]


def diff_fields(saved: dict, current: dict) -> dict:
    return {k: (saved.get(k), current.get(k)) for k in sorted(set(saved) | set(current)) if saved.get(k) != current.get(k)}


# ------------------------------------------------------------------------------------------ CLI
# Help text of every trainer option, attached in ``build_parser`` (defaults are appended there).
_HELP = {
    "data": "JSONL training files (one text per row, optional \"domain\"); several files: the file stem is the domain",
    "zipf_s": "exponent of the Zipf distribution of --synthetic-data zipf",
    "tokenizer": "character tokenizer, or a byte-level BPE / SentencePiece tokenizer trained at --tokenizer-path",
    "tokenizer_path": "directory of the BPE/SentencePiece tokenizer: reused if present, otherwise trained and saved",
    "tokenizer_algorithm": "SentencePiece model type",
    "examples": "rows read from each data file; later rows stay unseen (held-out benchmark in the run archive)",
    "redact_pii": "replace e-mail addresses, phone, SSN and card numbers and IPv4 addresses before tokenising",
    "sequence_length": "tokens per training window (the model gets one more position for the shifted labels)",
    "vocab_size": "vocabulary size (character tokenizer: at least the characters seen; BPE/SentencePiece target)",
    "curriculum": "order windows from easy to hard by this difficulty score",
    "curriculum_steps": "steps over which the curriculum widens from --curriculum-start-fraction to all windows",
    "curriculum_start_fraction": "share of the easiest windows drawn from at step 0",
    "domain_weights": "sampling weights per domain, e.g. \"prose=3,code=1\" (default: proportional to size)",
    "domain_weights_end": "weights reached after --domain-weights-steps (linear blend)",
    "domain_weights_steps": "steps of the blend from --domain-weights to --domain-weights-end",
    "domain_specialization_coef": "weight of the loss that pushes different domains onto different experts",
    "val_fraction": "hold out this share of each domain's windows for validation",
    "val_interval": "steps between validation passes",
    "val_batches": "batches per validation pass",
    "val_seed": "seed of the validation split and batches",
    "auto_architecture": "pick hidden size, layers, FFN width and experts to fill part of this device's memory",
    "auto_architecture_quality": "capacity: many experts, one active; balanced: a moderate pool, two active; "
                                 "dense: one expert",
    "auto_architecture_memory_fraction": "share of device memory the training state may fill",
    "hidden_size": "model width", "layers": "transformer blocks", "ffn_size": "hidden width of each SwiGLU expert",
    "attention_heads": "query heads",
    "norm_type": "normalisation", "position_embedding": "learned absolute positions or rotary embeddings",
    "attention_bias": "biases on the QKV and output projections",
    "total_experts": "experts per MoE layer", "active_experts": "experts each token is routed to (top-k)",
    "capacity_factor": "per-expert capacity = capacity_factor x tokens x k / experts (0: unlimited)",
    "min_expert_capacity": "lower bound of the per-expert capacity",
    "drop_overflow_tokens": "enforce the capacity (off: every route reaches its expert)",
    "overflow_policy": "drop: routes over capacity contribute nothing and are reported as dropped; residual: they "
                       "are skipped the same way (the residual stream carries the token) but not counted as dropped",
    "router_temperature": "softmax temperature of the router",
    "router_aux_coef": "weight of the load-balancing auxiliary loss",
    "steps": "optimizer steps to train to (a resumed run continues up to this step)",
    "schedule_steps": "length of the learning-rate schedule (default: --steps)",
    "batch_size": "sequences per step (per data-parallel group)",
    "gradient_accumulation_steps": "micro-steps accumulated before each optimizer step",
    "lr": "peak learning rate", "adam_beta1": "AdamW beta1", "adam_beta2": "AdamW beta2",
    "weight_decay": "AdamW decoupled weight decay", "max_grad_norm": "clip the global gradient norm to this value",
    "warmup_steps": "linear warm-up steps", "lr_decay": "decay after warm-up, down to --min-lr-ratio x --lr",
    "min_lr_ratio": "floor of the decayed learning rate, as a share of --lr",
    "plateau_patience": "controller intervals without improvement before the learning rate is reduced (0: off)",
    "aux_coef_end": "anneal the aux-loss weight linearly to this value over the schedule",
    "aux_adapt": "raise the aux-loss weight while routing is imbalanced, lower it when balanced",
    "capacity_adapt": "grow the capacity factor while routes are dropped, shrink it otherwise",
    "capacity_min": "lower bound of the adapted capacity factor", "capacity_max": "upper bound of it",
    "drop_threshold": "dropped-route share above which the capacity grows",
    "capacity_release_step": "stop enforcing the capacity from this step (0: never)",
    "temperature_start": "router temperature at step 0, annealed to --router-temperature",
    "temperature_steps": "steps of the router-temperature anneal",
    "temperature_adapt": "warm the router temperature while experts sit idle",
    "controller_interval": "steps between closed-loop controller updates",
    "optimizer": "AdamW (fused sm_100a kernel on CUDA), with 8-bit moments, or with moments in host memory",
    "device": "where to train (auto: CUDA when available)",
    "precision": "compute precision (CUDA: bf16 operands with fp32 accumulation and fp32 master weights)",
    "activation_checkpointing": "recompute each block's activations in backward to save memory",
    "auto_batch_size": "probe the largest batch that fits (optimizer state included) before training",
    "auto_batch_target": "use the smallest probed batch within this share of the best throughput (0: largest)",
    "expert_parallel": "shard the experts over the ranks of torchrun (replicated layers are averaged)",
    "tensor_parallel": "split each attention layer (and expert FFN) over this many ranks",
    "pipeline_parallel": "split the layers into contiguous stages, one per rank",
    "microbatches": "micro-batches per pipeline step",
    "pipeline_schedule": "GPipe (all forwards, then all backwards) or 1F1B",
    "shard_optimizer": "ZeRO-style: each rank keeps the AdamW state of its share of the replicated parameters",
    "optimizer_overlap": "run each AdamW update on a side stream under the next forward (fused CUDA AdamW, no "
                         "pipeline or sharded optimizer)",
    "straggler_routing": "bias routing away from ranks whose experts run slower",
    "straggler_capacity": "scale each rank's expert capacity by its measured speed",
    "straggler_capacity_min": "lower bound of the per-rank capacity scale",
    "straggler_capacity_max": "upper bound of the per-rank capacity scale",
    "straggler_strength": "gain of the routing-bias controller", "straggler_max_bias": "bound of the routing bias",
    "straggler_interval": "steps between straggler measurements",
    "device_metrics": "log per-rank expert time and row imbalance",
    "seed": "seed of the initialisation and of the batch order",
    "output": "directory of the final model (model.pt, config.json, tokenizer)",
    "checkpoint_dir": "directory of the resumable checkpoint",
    "checkpoint_interval": "steps between checkpoints (0: only at the end)",
    "resume": "continue from --checkpoint-dir when it holds a checkpoint of the same run configuration",
    "allow_config_change": "resume even if the run configuration changed",
    "metrics_file": "append one JSON line of metrics per logged step",
    "electricity_rate_usd_kwh": "price used for the energy cost in the metrics",
    "no_power_tracking": "do not read GPU energy counters",
    "log_interval": "steps between metric reads and log lines (values are read back from the device only then)",
    "diagnostics_dir": "write routing diagnostics (snapshots, SVG charts, index.html) here",
    "diagnostics_interval": "steps between routing snapshots (0: off unless a controller needs them)",
    "archive_dir": "archive the finished run (weights, data manifest, benchmarks, reproduce.sh) under this folder",
    "no_archive": "do not archive the run", "archive_data_limit_mb": "copy the data into the archive up to this size",
    "archive_benchmark_examples": "rows each archived benchmark reads",
    "data_card": "JSON describing the data's source, licence and provenance, embedded in the archive manifest",
}


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    data = p.add_argument_group("data")
    data.add_argument("--data", type=Path, nargs="+", default=[Path("data/smoke/tinystories.jsonl")])
    data.add_argument("--token-data", type=Path, help="packed corpus directory (replaces --data)")
    data.add_argument("--synthetic-data", choices=("none", "uniform", "zipf"), default="none",
                      help="seeded synthetic token ids instead of a corpus (vocab = --vocab-size)")
    data.add_argument("--zipf-s", type=float, default=1.1)
    data.add_argument("--tokenizer", choices=("char", "bpe", "sentencepiece"), default="char")
    data.add_argument("--tokenizer-path", type=Path)
    data.add_argument("--tokenizer-algorithm", choices=("unigram", "bpe"), default="unigram")
    data.add_argument("--examples", type=int, default=10000)
    data.add_argument("--redact-pii", action="store_true")
    data.add_argument("--sequence-length", type=int, default=128)
    data.add_argument("--vocab-size", type=int, default=7168)
    data.add_argument("--curriculum", choices=("none", "rarity", "entropy", "uncommon"), default="none")
    data.add_argument("--curriculum-steps", type=int, default=0)
    data.add_argument("--curriculum-start-fraction", type=float, default=0.25)
    data.add_argument("--domain-weights")
    data.add_argument("--domain-weights-end")
    data.add_argument("--domain-weights-steps", type=int, default=0)
    data.add_argument("--domain-specialization-coef", type=float, default=0.0)
    data.add_argument("--val-fraction", type=float)
    data.add_argument("--val-interval", type=int, default=200)
    data.add_argument("--val-batches", type=int, default=8)
    data.add_argument("--val-seed", type=int, default=0)

    model = p.add_argument_group("model")
    model.add_argument("--preset", choices=sorted(PRESETS), help="named architecture (overrides the shape options)")
    model.add_argument("--auto-architecture", action="store_true")
    model.add_argument("--auto-architecture-quality", choices=("capacity", "balanced", "dense"), default="balanced")
    model.add_argument("--auto-architecture-memory-fraction", type=float, default=0.45)
    model.add_argument("--hidden-size", type=int, default=64)
    model.add_argument("--layers", type=int, default=2)
    model.add_argument("--ffn-size", type=int, default=128)
    model.add_argument("--attention-heads", type=int, default=4)
    model.add_argument("--kv-heads", type=int, help="grouped-query attention key/value heads (default: MHA)")
    model.add_argument("--norm-type", choices=("layernorm", "rmsnorm"), default="layernorm")
    model.add_argument("--position-embedding", choices=("learned", "rope"), default="learned")
    model.add_argument("--attention-bias", action=argparse.BooleanOptionalAction, default=True)
    model.add_argument("--init-std", type=float, help="N(0, std) initialisation instead of torch defaults")
    model.add_argument("--total-experts", type=int, default=184)
    model.add_argument("--active-experts", type=int, default=1)
    model.add_argument("--capacity-factor", type=float, default=1.25)
    model.add_argument("--min-expert-capacity", type=int, default=4)
    model.add_argument("--drop-overflow-tokens", action=argparse.BooleanOptionalAction, default=True)
    model.add_argument("--overflow-policy", choices=("drop", "residual"), default="drop")
    model.add_argument("--router-temperature", type=float, default=1.0)
    model.add_argument("--router-aux-coef", type=float, default=0.01)

    opt = p.add_argument_group("optimisation and schedules")
    opt.add_argument("--steps", type=int, default=10)
    opt.add_argument("--schedule-steps", type=int)
    opt.add_argument("--batch-size", type=int, default=2)
    opt.add_argument("--gradient-accumulation-steps", type=int, default=1)
    opt.add_argument("--lr", type=float, default=3e-4)
    opt.add_argument("--adam-beta1", type=float, default=0.9)
    opt.add_argument("--adam-beta2", type=float, default=0.999)
    opt.add_argument("--weight-decay", type=float, default=0.01)
    opt.add_argument("--max-grad-norm", type=float, default=1.0)
    opt.add_argument("--warmup-steps", type=int, default=0)
    opt.add_argument("--lr-decay", choices=("constant", "cosine", "linear"), default="constant")
    opt.add_argument("--min-lr-ratio", type=float, default=0.1)
    opt.add_argument("--plateau-patience", type=int, default=0)
    opt.add_argument("--aux-coef-end", type=float)
    opt.add_argument("--aux-adapt", action="store_true")
    opt.add_argument("--capacity-adapt", action="store_true")
    opt.add_argument("--capacity-min", type=float, default=1.0)
    opt.add_argument("--capacity-max", type=float, default=4.0)
    opt.add_argument("--drop-threshold", type=float, default=0.01)
    opt.add_argument("--capacity-release-step", type=int, default=0)
    opt.add_argument("--temperature-start", type=float)
    opt.add_argument("--temperature-steps", type=int, default=0)
    opt.add_argument("--temperature-adapt", action="store_true")
    opt.add_argument("--controller-interval", type=int, default=50)
    opt.add_argument("--optimizer", choices=("adamw", "adamw8bit", "adamw_cpu_offload"), default="adamw")

    system = p.add_argument_group("system")
    system.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    system.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    system.add_argument("--activation-checkpointing", action="store_true")
    system.add_argument("--auto-batch-size", action="store_true")
    system.add_argument("--auto-batch-target", type=float, default=0.95)
    system.add_argument("--expert-parallel", action="store_true")
    system.add_argument("--tensor-parallel", type=int, default=1)
    system.add_argument("--sequence-parallel", action="store_true",
                        help="attention tensor-parallel and experts expert-parallel over the same ranks "
                             "(--tensor-parallel = world size); token rows are sharded between the attention blocks")
    system.add_argument("--data-parallel", action="store_true", help="plain data parallelism (replicated experts)")
    system.add_argument("--pipeline-parallel", action="store_true")
    system.add_argument("--pipeline-data-parallel", type=int, default=1, help="data-parallel replicas of the pipeline")
    system.add_argument("--microbatches", type=int, default=1)
    system.add_argument("--pipeline-schedule", choices=("gpipe", "1f1b"), default="gpipe")
    system.add_argument("--shard-optimizer", action="store_true")
    system.add_argument("--optimizer-overlap", action="store_true")
    system.add_argument("--straggler-routing", action="store_true")
    system.add_argument("--straggler-capacity", action="store_true")
    system.add_argument("--straggler-capacity-min", type=float, default=0.5)
    system.add_argument("--straggler-capacity-max", type=float, default=2.0)
    system.add_argument("--straggler-strength", type=float, default=0.5)
    system.add_argument("--straggler-max-bias", type=float, default=2.0)
    system.add_argument("--straggler-interval", type=int, default=10)
    system.add_argument("--device-metrics", action="store_true")
    system.add_argument("--simulate-slow-rank", help="RANK:SECONDS_PER_ROW (testing)")
    system.add_argument("--moe-kernel", choices=("loop", "triton", "native", "auto"), default="auto",
                        help="expert compute: per-expert loop (oracle), or the grouped native kernels (triton = alias)")
    system.add_argument("--seed", type=int, default=0)

    io = p.add_argument_group("outputs")
    io.add_argument("--output", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    io.add_argument("--checkpoint-dir", type=Path, default=Path("artifacts/checkpoints/quantweave-moe-checkpoint"))
    io.add_argument("--checkpoint-interval", type=int, default=1000)
    io.add_argument("--resume", action=argparse.BooleanOptionalAction, default=True)
    io.add_argument("--allow-config-change", action="store_true")
    io.add_argument("--metrics-file", type=Path)
    io.add_argument("--electricity-rate-usd-kwh", type=float, default=0.16)
    io.add_argument("--no-power-tracking", action="store_true")
    io.add_argument("--log-interval", type=int, default=1)
    io.add_argument("--diagnostics-dir", type=Path)
    io.add_argument("--diagnostics-interval", type=int, default=0)
    io.add_argument("--archive-dir", type=Path)
    io.add_argument("--no-archive", action="store_true")
    io.add_argument("--archive-data-limit-mb", type=float, default=200.0)
    io.add_argument("--archive-benchmark-examples", type=int, default=500)
    io.add_argument("--data-card", type=Path)
    for action in p._actions:
        if action.help is None and action.dest in _HELP:
            default = action.default
            shown = "" if default in (None, False) or isinstance(default, bool) else f" (default: {default})"
            if isinstance(default, list):
                shown = " (default: " + " ".join(map(str, default)) + ")"
            action.help = _HELP[action.dest] + shown
    return p


def default_args(**overrides) -> argparse.Namespace:
    args = build_parser().parse_args([])
    for name, value in overrides.items():
        if not hasattr(args, name):
            raise TypeError(f"unknown training option '{name}'")
        setattr(args, name, value)
    return args


def schedule_config_from(args) -> ScheduleConfig:
    return ScheduleConfig(
        lr=args.lr, total_steps=args.schedule_steps or args.steps, warmup_steps=args.warmup_steps,
        lr_decay=args.lr_decay, min_lr_ratio=args.min_lr_ratio, plateau_patience=args.plateau_patience,
        aux_coef=args.router_aux_coef, aux_coef_end=args.aux_coef_end, aux_adapt=args.aux_adapt,
        capacity_factor=args.capacity_factor, capacity_adapt=args.capacity_adapt, capacity_min=args.capacity_min,
        capacity_max=args.capacity_max, drop_threshold=args.drop_threshold,
        capacity_release_step=args.capacity_release_step, temperature_start=args.temperature_start,
        temperature_end=args.router_temperature, temperature_steps=args.temperature_steps,
        temperature_adapt=args.temperature_adapt, interval=args.controller_interval)


def load_data(args, is_main: bool):
    """(tokenizer, corpus, redactor); synthetic data returns (None, None, None)."""
    if args.synthetic_data != "none":
        return None, None, None
    redactor = None
    if args.redact_pii:
        from ..utils.pii_redact import PIIRedactor

        redactor = PIIRedactor()
    if args.token_data:
        corpus, tokenizer = load_token_bin(args.token_data)
        return tokenizer, corpus, redactor
    if args.tokenizer in {"bpe", "sentencepiece"}:
        if args.tokenizer_path is None:
            raise ValueError(f"--tokenizer {args.tokenizer} needs --tokenizer-path")
        marker = "tokenizer.json" if args.tokenizer == "bpe" else "tokenizer.model"
        if (args.tokenizer_path / marker).exists():
            tokenizer = load_tokenizer(args.tokenizer_path)
        else:
            texts = (t for _, t in read_rows(args.data, args.examples, redactor))
            if args.tokenizer == "bpe":
                tokenizer = BPETokenizer.train(texts, args.vocab_size)
            else:
                tokenizer = SentencePieceTokenizer.train(texts, args.vocab_size, args.tokenizer_algorithm)
            if is_main:
                tokenizer.save(args.tokenizer_path)
    else:
        tokenizer = CharTokenizer.build((t for _, t in read_rows(args.data, redactor=redactor)), args.vocab_size)
    return tokenizer, build_corpus(args.data, tokenizer, args.examples, redactor), redactor


def apply_preset(args) -> None:
    if not args.preset:
        return
    spec = PRESETS[args.preset]
    mapping = {"vocab_size": "vocab_size", "hidden_size": "hidden_size", "layers": "layers", "ffn_size": "ffn_size",
               "attention_heads": "attention_heads", "kv_heads": "kv_heads", "num_experts": "total_experts",
               "top_k": "active_experts", "capacity_factor": "capacity_factor", "norm_type": "norm_type",
               "position_embedding": "position_embedding", "attention_bias": "attention_bias",
               "init_std": "init_std", "router_aux_loss_coef": "router_aux_coef"}
    for key, value in spec.items():
        if key in mapping:
            setattr(args, mapping[key], value)


def build_config(args, vocab_size: int) -> QuantaWeaveConfig:
    return QuantaWeaveConfig(
        vocab_size=vocab_size, hidden_size=args.hidden_size, layers=args.layers, ffn_size=args.ffn_size,
        num_experts=args.total_experts, top_k=args.active_experts, attention_heads=args.attention_heads,
        max_sequence_length=args.sequence_length + 1, router_aux_loss_coef=args.router_aux_coef,
        capacity_factor=args.capacity_factor, min_expert_capacity=args.min_expert_capacity,
        drop_overflow_tokens=args.drop_overflow_tokens, overflow_policy=args.overflow_policy,
        router_temperature=args.router_temperature, norm_type=args.norm_type,
        position_embedding=args.position_embedding, kv_heads=args.kv_heads, attention_bias=args.attention_bias,
        init_std=args.init_std)


# ------------------------------------------------------------------------------------------ training
def run_training(args) -> dict:
    """Train according to ``args`` (from ``build_parser``/``default_args``); returns a summary dict. The caller's
    output options are restored however the run ends."""
    original = (args.metrics_file, args.diagnostics_dir, args.diagnostics_interval)
    temporary: list[Path] = []
    try:
        return _run_training(args, original, temporary)
    finally:
        args.metrics_file, args.diagnostics_dir, args.diagnostics_interval = original
        for path in temporary:
            shutil.rmtree(path, ignore_errors=True) if path.is_dir() else path.unlink(missing_ok=True)


def _validate(args) -> None:
    if args.gradient_accumulation_steps < 1:
        raise ValueError("--gradient-accumulation-steps must be positive")
    if args.tensor_parallel < 1:
        raise ValueError("--tensor-parallel must be positive")
    use_ep = args.expert_parallel or args.tensor_parallel > 1
    if use_ep and args.pipeline_parallel:
        raise ValueError("--pipeline-parallel cannot be combined with --expert-parallel/--tensor-parallel")
    if use_ep and args.data_parallel:
        raise ValueError("--data-parallel is implied by --expert-parallel (replicated weights are averaged)")
    if (args.straggler_routing or args.straggler_capacity or args.device_metrics) and not use_ep:
        raise ValueError("--straggler-routing, --straggler-capacity and --device-metrics need --expert-parallel "
                         "(or --tensor-parallel)")
    if args.shard_optimizer and not (use_ep or args.data_parallel or args.pipeline_parallel):
        raise ValueError("--shard-optimizer needs a data-parallel group (--expert-parallel, --data-parallel or "
                         "--pipeline-parallel with --pipeline-data-parallel > 1)")
    if use_ep or args.pipeline_parallel or args.data_parallel:
        if args.auto_batch_size:
            raise ValueError("--auto-batch-size is not supported with multi-process parallelism")
        if args.aux_adapt or args.temperature_adapt:
            raise ValueError("--aux-adapt/--temperature-adapt need cross-rank routing statistics and are not "
                             "supported with multi-process parallelism")
        if args.precision == "fp16":
            raise ValueError("fp16 loss scaling is not supported with multi-process parallelism; use bf16 or fp32")
    if args.pipeline_parallel:
        if args.gradient_accumulation_steps != 1:
            raise ValueError("--pipeline-parallel micro-batches replace gradient accumulation; leave "
                             "--gradient-accumulation-steps at 1")
        if args.domain_specialization_coef or args.diagnostics_interval or args.diagnostics_dir:
            raise ValueError("routing diagnostics and the domain loss need every layer on one rank and are not "
                             "supported with --pipeline-parallel")
        if args.val_fraction is not None:
            raise ValueError("--val-fraction needs a full forward pass and is not supported with --pipeline-parallel")
        if args.batch_size % args.microbatches:
            raise ValueError(f"--microbatches {args.microbatches} must divide --batch-size {args.batch_size}")
    if getattr(args, "sequence_parallel", False):
        if not args.expert_parallel or args.tensor_parallel < 2:
            raise ValueError("--sequence-parallel needs --expert-parallel and --tensor-parallel equal to the world size")
        if args.shard_optimizer:
            raise ValueError("--shard-optimizer shards replicated tensors across the expert group, which holds "
                             "different attention slices under --sequence-parallel")
    if args.shard_optimizer and args.optimizer != "adamw":
        raise ValueError(f"--optimizer {args.optimizer} is not combinable with --shard-optimizer")
    if args.val_fraction is not None and args.val_interval < 1:
        raise ValueError("--val-fraction needs --val-interval >= 1 (steps between validation passes)")
    if args.curriculum != "none" and args.curriculum_steps <= 0:
        raise ValueError("--curriculum needs --curriculum-steps > 0")


@torch.no_grad()
def evaluate_validation(model, val_stream, device, precision, start_step, batches, num_domains) -> float:
    was = model.training
    model.eval()
    total, count = 0.0, 0
    try:
        for offset in range(batches):
            batch, domains = val_stream.batch(start_step * 100_000 + offset)
            batch, domains = batch.to(device), domains.to(device)
            with autocast_context(device, precision):
                out = model(batch, labels=batch, domain_ids=domains, num_domains=num_domains, return_logits=False)
            total += float(out["loss"].item())
            count += 1
    finally:
        model.train(was)
    return total / max(1, count)


def _run_training(args, original_outputs: tuple, temporary: list) -> dict:
    apply_preset(args)
    _validate(args)
    ep = pp = dp = None
    use_ep = args.expert_parallel or args.tensor_parallel > 1
    if use_ep:
        from ..parallel.expert_parallel import init_expert_parallel

        ep = init_expert_parallel(args.device, args.tensor_parallel,
                                  sequence_parallel=getattr(args, "sequence_parallel", False))
        device, rank, world_size = ep.device, ep.rank, ep.world_size
        is_main = ep.global_rank == 0
    elif args.pipeline_parallel:
        from ..parallel.pipeline_parallel import init_pipeline_parallel

        pp = init_pipeline_parallel(args.device, args.layers, data_parallel=args.pipeline_data_parallel)
        device, rank, world_size = pp.device, pp.dp_rank, pp.dp_size
        is_main = pp.global_rank == 0
    elif args.data_parallel:
        from ..parallel.data_parallel import init_data_parallel

        dp = init_data_parallel(args.device)
        device, rank, world_size = dp.device, dp.rank, dp.world_size
        is_main = dp.rank == 0
    else:
        device, rank, world_size = select_device(args.device), 0, 1
        is_main = True
        if device.type == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("CUDA was requested but is not available")
    ctx = ep if ep is not None else pp if pp is not None else dp
    say = print if is_main else (lambda *a, **k: None)

    started = time.time()
    archiving = args.archive_dir is not None and not args.no_archive and is_main
    if archiving:
        if args.metrics_file is None:
            handle, name = tempfile.mkstemp(suffix=".jsonl")
            os.close(handle)
            args.metrics_file = Path(name)
            temporary.append(args.metrics_file)
        if pp is None and args.diagnostics_dir is None:
            args.diagnostics_dir = Path(tempfile.mkdtemp(prefix="diagnostics-"))
            temporary.append(args.diagnostics_dir)
            args.diagnostics_interval = args.diagnostics_interval or max(1, args.steps // 20)
    reproduce_args = argparse.Namespace(**vars(args))
    reproduce_args.metrics_file, reproduce_args.diagnostics_dir, reproduce_args.diagnostics_interval = original_outputs

    if args.auto_architecture:
        from ..utils.hardware import auto_architecture

        shape = auto_architecture(detect(device.type), args.vocab_size, args.auto_architecture_memory_fraction,
                                  args.auto_architecture_quality)
        args.hidden_size, args.layers, args.ffn_size = shape["hidden_size"], shape["layers"], shape["ffn_size"]
        args.attention_heads = shape["attention_heads"]
        args.total_experts, args.active_experts = shape["total_experts"], shape["active_experts"]
        args.sequence_length = shape["sequence_length"]
        say(f"auto architecture ({args.auto_architecture_quality}): {shape}")
        reproduce_args.auto_architecture = False
        for name in ("hidden_size", "layers", "ffn_size", "attention_heads", "total_experts", "active_experts",
                     "sequence_length"):
            setattr(reproduce_args, name, getattr(args, name))

    # ranks that read distinct batches; under sequence parallelism every rank reads the same one
    data_rank, data_world = (0, 1) if (ep is not None and ep.sequence_parallel) else (rank, world_size)
    random.seed(args.seed)
    torch.manual_seed(args.seed)
    tokenizer, corpus, redactor = load_data(args, is_main)
    if redactor is not None and is_main and any(redactor.report().values()):
        say(f"PII redaction: {redactor.report()}")
    val_dataset = None
    if corpus is None:
        dataset = SyntheticTokenStream(args.vocab_size, args.sequence_length, args.batch_size, args.seed,
                                       args.synthetic_data, args.zipf_s, data_rank, data_world)
        vocab_size = args.vocab_size
    else:
        dataset = WindowDataset(corpus, args.sequence_length)
        if len(dataset) == 0:
            raise ValueError("The corpus holds fewer tokens than one training window")
        if args.val_fraction is not None:
            dataset, val_dataset = dataset.split_train_val(args.val_fraction, args.val_seed)
            say(f"validation split: {len(val_dataset)} windows held out, {len(dataset)} left for training")
        vocab_size = tokenizer.vocab_size if tokenizer.kind in ("bpe", "sentencepiece") else max(args.vocab_size, tokenizer.vocab_size)
    config = build_config(args, vocab_size)

    shard_id = ep.global_rank if ep is not None else (pp.stage if pp is not None else 0)
    torch.manual_seed(args.seed + shard_id)
    model = QuantaWeaveMoEForCausalLM(config, expert_parallel=ep, pipeline=pp).to(device)
    precision = choose_precision(detect(device.type), args.precision)
    if device.type == "cuda":
        from .native import prepare_model

        prepare_model(model, precision)
    if ep is not None:
        from ..parallel.expert_parallel import broadcast_shared_parameters

        broadcast_shared_parameters(model, ep)
    if dp is not None:
        dp.broadcast_parameters(model)
    if pp is not None and pp.dp_size > 1:
        pp.broadcast_parameters(model)
    model.domain_specialization_coef = args.domain_specialization_coef
    model.activation_checkpointing = args.activation_checkpointing
    scaler = torch.amp.GradScaler(device.type) if (precision == "fp16" and device.type != "cuda") else None
    autocast = lambda: autocast_context(device, precision)  # noqa: E731
    if args.moe_kernel != "auto" or device.type == "cuda":
        kernel = args.moe_kernel
        say(f"moe kernel: {model.set_moe_kernel(kernel)}")

    if args.auto_batch_size:
        found = find_safe_batch_size(model, device, args.sequence_length, autocast, target=args.auto_batch_target)
        args.batch_size = found["recommended_batch_size"]
        if corpus is None:
            dataset.batch_size = args.batch_size
        say(f"auto batch size: {args.batch_size}")

    scores = None
    if args.curriculum != "none" and corpus is not None:
        scores = difficulty_scores(dataset, args.curriculum, vocab_size)
    curriculum = CurriculumConfig(args.curriculum if scores is not None else "rarity", args.curriculum_start_fraction,
                                  args.curriculum_steps if scores is not None else 0)
    mixture = None
    if args.domain_weights and corpus is not None:
        mixture = DomainMixture(dataset.domains, parse_domain_weights(args.domain_weights),
                                parse_domain_weights(args.domain_weights_end), args.domain_weights_steps)
    if corpus is None:
        stream = dataset
    else:
        stream = BatchStream(dataset, args.batch_size, args.seed, scores, curriculum, mixture, data_rank, data_world)
    domains_active = stream.num_domains > 1
    val_stream = (BatchStream(val_dataset, args.batch_size, args.val_seed, rank=data_rank, world_size=data_world)
                  if val_dataset else None)

    betas = (args.adam_beta1, args.adam_beta2)
    if args.shard_optimizer:
        from ..parallel.sharded_optimizer import ShardedAdamW

        optimizer = ShardedAdamW(model, ctx, lr=args.lr, betas=betas, weight_decay=args.weight_decay)
    else:
        optimizer = build_optimizer(args.optimizer, model.parameters(), args.lr, betas, args.weight_decay, device)
        if getattr(args, "optimizer_overlap", False) and hasattr(optimizer, "overlap_with_forward") \
                and not args.pipeline_parallel and hasattr(model, "parameter_parts"):
            optimizer.overlap_with_forward(model)
    tracker = None
    if ep is not None and ep.world_size > 1 and (args.straggler_routing or args.straggler_capacity or args.device_metrics):
        from ..parallel.expert_parallel import DeviceLoadTracker

        tracker = DeviceLoadTracker(model, ep, strength=args.straggler_strength if args.straggler_routing else 0.0,
                                    max_bias=args.straggler_max_bias, interval=args.straggler_interval,
                                    adapt_capacity=args.straggler_capacity,
                                    capacity_scale_min=args.straggler_capacity_min,
                                    capacity_scale_max=args.straggler_capacity_max)
    if args.simulate_slow_rank:
        slow, cost = args.simulate_slow_rank.split(":")
        if ep is not None and ep.rank == int(slow):
            for moe in model.moes():
                moe.simulated_cost_per_row = float(cost)
                moe.kernel = "loop"
    engine = None
    if pp is not None:
        from ..parallel.pipeline_parallel import PipelineEngine

        engine = PipelineEngine(model, pp, args.microbatches, autocast, schedule=args.pipeline_schedule)
        if hasattr(optimizer, "arm_overlap"):  # sharded AdamW: reduce-scatter during the last backward
            engine.before_last_backward = optimizer.arm_overlap
    counts = parameter_counts(config)
    controller = TrainingController(schedule_config_from(args), base_temperature=args.router_temperature)
    adaptive = args.aux_adapt or args.temperature_adapt
    diagnostics_interval = args.diagnostics_interval or (args.controller_interval if adaptive else 0)
    monitor = None
    if diagnostics_interval and is_main:
        from ..utils.routing_diagnostics import RoutingMonitor

        classes = token_classes(tokenizer) if tokenizer is not None else None
        monitor = RoutingMonitor(config.layers, config.num_experts, config.top_k,
                                 getattr(dataset, "domains", ["synthetic"]), classes, args.diagnostics_dir)
    logger = MetricsLogger(args.metrics_file if is_main else None, counts["total"], counts["active"])
    power = None
    if is_main and not args.no_power_tracking:
        from ..utils.energy import PowerCostTracker

        power = PowerCostTracker(args.electricity_rate_usd_kwh, resume_from=args.metrics_file)

    fields = resume_fields(args, config, dataset, tokenizer, world_size)
    if ctx is not None:
        from ..parallel.checkpoint import sharded_checkpoint_exists

        resumable = sharded_checkpoint_exists(args.checkpoint_dir)
    else:
        resumable = checkpoint_exists(args.checkpoint_dir)
    start_step = 0
    if args.resume and resumable:
        extra: dict = {}
        if ctx is not None:
            from ..parallel.checkpoint import load_sharded_checkpoint

            start_step = load_sharded_checkpoint(args.checkpoint_dir, model, optimizer, ctx, extra)
        else:
            start_step = load_checkpoint(args.checkpoint_dir, model, optimizer, device, extra)
        changed = diff_fields(extra.get("resume_fields", fields), fields)
        if changed and not args.allow_config_change:
            raise ValueError(f"checkpoint {args.checkpoint_dir} was made by a different run configuration: {changed}. "
                             "Pass --allow-config-change to resume anyway, or use a fresh --checkpoint-dir.")
        if "schedule" in extra:
            controller.load_state_dict(extra["schedule"])
        if tracker is not None and extra.get("straggler"):
            tracker.load_state_dict(extra["straggler"])
        if scaler is not None and extra.get("scaler"):
            scaler.load_state_dict(extra["scaler"])
        say(f"resumed from {args.checkpoint_dir} at step {start_step}")
    say(f"device={device} precision={precision} parameters total={counts['total']:,} active/token={counts['active']:,} "
        f"experts={config.num_experts} top_k={config.top_k}"
        + (f" expert_parallel={world_size} tensor_parallel={args.tensor_parallel}" if ep is not None else "")
        + (f" pipeline_stages={pp.num_stages} microbatches={args.microbatches}" if pp is not None else "")
        + (f" data_parallel={world_size}" if dp is not None else "")
        + (" sharded_optimizer" if args.shard_optimizer else ""))
    if start_step >= args.steps:
        say(f"checkpoint already reached requested step {args.steps}")
        return {"steps": start_step, "resumed_only": True}

    def checkpoint_extra(step: int) -> dict:
        return {"resume_fields": fields, "config_hash": config_hash(fields), "schedule": controller.state_dict(),
                "data": stream.state(step), "scaler": scaler.state_dict() if scaler is not None else None,
                "straggler": tracker.state_dict() if tracker is not None else None,
                "routing_controls": {"capacity_factor": model.config.capacity_factor,
                                     "router_temperature": model.config.router_temperature,
                                     "router_aux_loss_coef": model.router_aux_loss_coef}}

    def save(path: Path, step: int) -> None:
        if hasattr(optimizer, "finish"):
            optimizer.finish()  # an update in flight on the side stream lands before the weights are read
        payload = tokenizer_payload(tokenizer) if tokenizer is not None else None
        if ctx is not None:
            from ..parallel.checkpoint import save_sharded_checkpoint

            save_sharded_checkpoint(path, model, optimizer, step, payload, ctx, checkpoint_extra(step))
        else:
            save_checkpoint(path, model, optimizer, step, payload, device, checkpoint_extra(step))

    model.train()
    optimizer.zero_grad(set_to_none=True)
    routes_per_step = args.batch_size * args.sequence_length * config.layers * config.top_k
    scalars = StepScalars()

    def mean_over_ranks(values: list) -> list:
        """Average loss and overflow fraction over the ranks that saw different tokens (one collective per flush;
        every rank flushes at the same steps)."""
        if ctx is not None and ep is not None:
            from ..parallel.expert_parallel import all_reduce_mean

            return all_reduce_mean(values, ep)
        if dp is not None:
            return dp.all_reduce_mean(values)
        return values
    window_metrics = {"imbalance": None, "active_fraction": None}
    pending_tokens = 0
    last_log: dict = {}
    val_loss = best_val = None
    for step in range(start_step + 1, args.steps + 1):
        applied = controller.apply(model, optimizer, step)
        batch, domain_ids = stream.batch(step)
        batch, domain_ids = batch.to(device, non_blocking=True), domain_ids.to(device, non_blocking=True)
        collect = bool(diagnostics_interval) and step % diagnostics_interval == 0
        model.set_collect_stats(collect)
        grad_norm = None
        if engine is not None:
            result = engine.train_step(batch)
            grad_norm = engine.clip_and_sync(optimizer, args.max_grad_norm)
            optimizer.step()
            optimizer.zero_grad(set_to_none=True)
            # the engine has already reduced these over the pipeline (host values): nothing left to all-reduce
            scalars.push(step, torch.tensor([result["loss"], result["router_aux_loss"], result["dropped_routes"],
                                             result["overflow_routes"], 0.0,
                                             result["overflow_routes"] / max(1, routes_per_step)],
                                            dtype=torch.float64), reduce=False)
        else:
            with autocast(), nvtx_range("forward"):
                out = model(batch, labels=batch, domain_ids=domain_ids,
                            num_domains=stream.num_domains if domains_active else 0, return_logits=False)
            loss = out["loss"]
            scaled = loss / args.gradient_accumulation_steps
            last_micro = step % args.gradient_accumulation_steps == 0 or step == args.steps
            if last_micro and args.shard_optimizer and scaler is None and hasattr(optimizer, "arm_overlap"):
                optimizer.arm_overlap()  # reduce-scatter the gradient buckets while this backward runs
            with nvtx_range("backward"):
                (scaler.scale(scaled) if scaler is not None else scaled).backward()
            if step % args.gradient_accumulation_steps == 0 or step == args.steps:
                with nvtx_range("grad_sync"):
                    if ep is not None:
                        from ..parallel.expert_parallel import clip_grad_norm_parallel, sync_gradients

                        sync_gradients(model, ep, optimizer if args.shard_optimizer else None)
                        grad_norm = clip_grad_norm_parallel(model, ep, args.max_grad_norm, bool(args.shard_optimizer), optimizer)
                    elif dp is not None:
                        dp.sync_gradients(model, optimizer if args.shard_optimizer else None)
                        grad_norm = dp.clip_grad_norm(model, optimizer, args.max_grad_norm)
                    else:
                        if scaler is not None:
                            scaler.unscale_(optimizer)
                        grad_norm = clip_grad_norm(model, optimizer, args.max_grad_norm)
                with nvtx_range("optimizer"):
                    if scaler is not None:
                        scaler.step(optimizer)
                        scaler.update()
                    else:
                        optimizer.step()
                    optimizer.zero_grad(set_to_none=True)
            # kept on the device: read back (and averaged over ranks) in one transfer at the next flush point
            overflow = out["overflow_routes"].detach().double()
            scalars.push(step, torch.stack([loss.detach().double(), out["router_aux_loss"].detach().double(),
                                            out["dropped_routes"].detach().double(), overflow,
                                            out["domain_loss"].detach().double(),
                                            overflow / max(1, routes_per_step)]), reduce=True)
        device_metrics = tracker.update(step) if tracker is not None else None
        pending_tokens += args.batch_size * args.sequence_length * data_world
        flush_now = (step % args.log_interval == 0 or step == args.steps or controller.should_update(step)
                     or (args.checkpoint_interval > 0 and step % args.checkpoint_interval == 0))
        if flush_now:
            if hasattr(optimizer, "finish"):
                optimizer.finish()  # a norm or update still on the optimizer's side stream lands before it is read
            for _, (loss_value, aux_value, dropped, overflow_count, domain_value, overflow_fraction) in \
                    scalars.flush(mean_over_ranks):
                controller.observe(loss_value, overflow_fraction)
            dropped_value, overflow_value = int(dropped), int(overflow_count)
        if tracker is not None and collect:
            util = tracker.gather_expert_utilization()
            if monitor is not None:
                monitor.record_device_utilization(util)
        if collect and monitor is not None:
            monitor.update(model, batch, domain_ids)
            window_metrics = {"imbalance": monitor.imbalance(), "active_fraction": monitor.active_fraction()}
            monitor.snapshot(step)
        if controller.should_update(step):
            changes = controller.update(step, **window_metrics)
            if changes:
                say(f"controller step={step}: {changes}")
            window_metrics = {"imbalance": None, "active_fraction": None}
        fresh_val = None
        if val_stream is not None and (step % args.val_interval == 0 or step == args.steps):
            val_loss = fresh_val = evaluate_validation(model, val_stream, device, precision, step, args.val_batches,
                                                       val_stream.num_domains if domains_active else 0)
            best_val = val_loss if best_val is None else min(best_val, val_loss)
            say(f"step={step}/{args.steps} val_loss={val_loss:.4f}")
        if step % args.log_interval == 0 or step == args.steps:
            if device.type == "cuda":
                from ..ops.status import check_device_status

                check_device_status()  # raises CommTimeoutError / DeviceStatusError if a kernel gave up on a wait
            extra_fields = {}
            if device_metrics:
                extra_fields.update(time_imbalance=device_metrics["time_imbalance"],
                                    rows_imbalance=device_metrics["rows_imbalance"])
            if fresh_val is not None:
                extra_fields["val_loss"] = fresh_val
            if power is not None:
                extra_fields.update(power.sample())
            last_log = logger.log(step, pending_tokens, loss=loss_value, router_aux=aux_value,
                                  dropped_routes=dropped_value, overflow_routes=overflow_value,
                                  overflow_fraction=overflow_fraction, domain_loss=domain_value,
                                  grad_norm=float(grad_norm) if grad_norm is not None else None, **applied,
                                  **extra_fields)
            pending_tokens = 0
            say(f"step={step}/{args.steps} loss={loss_value:.4f} router_aux={aux_value:.4f} "
                f"dropped_routes={dropped_value} overflow_routes={overflow_value}")
        if args.checkpoint_interval > 0 and step % args.checkpoint_interval == 0:
            save(args.checkpoint_dir, step)
            say(f"checkpoint saved at step {step} to {args.checkpoint_dir}")

    model.set_collect_stats(False)
    save(args.output if ctx is None else args.output / "shards", args.steps)
    if ctx is not None:
        from ..parallel.checkpoint import consolidate_checkpoint
        from ..parallel.groups import finish

        finish(ctx)
        if is_main:
            consolidate_checkpoint(args.output / "shards", args.output)
    say(f"saved checkpoint to {args.output}")
    if monitor is not None and args.diagnostics_dir is not None:
        say(f"routing diagnostics: {monitor.write_report()}")
    summary = logger.summary()
    summary.update(steps=args.steps, output=str(args.output), precision=precision,
                   controller_history=controller.history,
                   last_routing=monitor.snapshots[-1] if monitor is not None and monitor.snapshots else None,
                   stream=stream.state(args.steps), last_log=last_log, val_loss=val_loss, best_val_loss=best_val,
                   val_windows=len(val_dataset) if val_dataset is not None else None,
                   energy_kwh_total=power.energy_kwh if power is not None else None,
                   cost_usd_total=(power.energy_kwh * args.electricity_rate_usd_kwh) if power is not None else None)
    if archiving:
        from ..tools.run_bundle import create_run_bundle, reproduce_command

        if args.auto_batch_size:
            reproduce_args.auto_batch_size, reproduce_args.batch_size = False, args.batch_size
        bundle = create_run_bundle(
            args.archive_dir, kind="train", model_dirs={"model": args.output},
            benchmark_model=None if (args.token_data or corpus is None) else args.output,
            data_paths=[] if (args.token_data or corpus is None) else list(args.data), options=vars(args),
            summary=summary, started=started,
            reproduce=reproduce_command("quantaweave_b200.train", build_parser(), reproduce_args,
                                        skip=("archive_dir", "no_archive")),
            reproduce_full=reproduce_command("quantaweave_b200.train", build_parser(), reproduce_args,
                                             skip=("archive_dir", "no_archive"), explicit=True),
            finished=time.time(), metrics_file=args.metrics_file,
            diagnostics_dir=args.diagnostics_dir if monitor is not None else None,
            skip_rows=None if args.token_data else args.examples, benchmark_examples=args.archive_benchmark_examples,
            device=args.device if ctx is None else "auto", precision=args.precision,
            data_limit_mb=args.archive_data_limit_mb, data_card=args.data_card)
        summary["archive"] = str(bundle)
        say(f"archived run to {bundle}")
    return summary


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    from ..tools.run_bundle import resolve_archive_dir

    resolve_archive_dir(args)
    run_training(args)


if __name__ == "__main__":
    main()
