"""Sharded checkpoints: per-rank save/load, consolidation into one ``model.pt``, and resharding.

File format follows the reference (``src/expert_parallel.py:388-547``): each rank writes ``model.rank{r}.pt`` =
``{model, optimizer, step, rng_state, world_size, rank, layout, extra}`` (replaced atomically with ``os.replace``);
rank 0 adds ``config.json``, tokenizer files and ``metadata.json``; ``layout`` is
``{"kind": "ep", ep_rank, ep_size, tp_rank, tp_size}`` or ``{"kind": "pp", stage, stages, layer_start, layer_end}``
(pipeline shards may also carry ``dp_rank``/``dp_size``). ``consolidate_checkpoint`` merges TP slices, renumbers
experts globally and concatenates pipeline stages into an ordinary checkpoint with ``"optimizer": None``;
``reshard_checkpoint`` splits one checkpoint into ``ep x tp`` weights-only shards.

Sequence-parallel shards (attention tensor-parallel and experts expert-parallel over the same ranks) carry
``"sequence_parallel": true`` in their ``ep`` layout, with ``tp_rank == ep_rank == rank``: rank r holds attention
slice r and experts ``[r * E/world, (r+1) * E/world)``, whole.
"""

from __future__ import annotations

import json
import os
import random
import re
import shutil
from pathlib import Path
from typing import Optional

import torch

from ..config import QuantaWeaveConfig
from ..utils.checkpoint_io import load_checkpoint
from .tensor_parallel import is_tp_sharded_shared, merge_state_dicts, merge_tensors, shard_state_dict

EXPERT_KEY = re.compile(r"(experts\.)(\d+)(\.)")
BLOCK_KEY = re.compile(r"^blocks\.(\d+)\.")
_COPIED = ("config.json", "vocab.json", "tokenizer.json", "tokenizer.model", "tokenizer_meta.json", "metadata.json")


def shard_path(directory, rank: int) -> Path:
    return Path(directory) / f"model.rank{rank}.pt"


def sharded_checkpoint_exists(directory) -> bool:
    return shard_path(directory, 0).exists()


def _barrier() -> None:
    from .groups import barrier

    barrier()


def save_sharded_checkpoint(directory, model, optimizer, step: int, tokenizer, ctx, extra: dict) -> None:
    from ..training.trainer import write_checkpoint_metadata

    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    tmp = directory / f".model.rank{ctx.global_rank}.pt.tmp"
    torch.save({"model": model.state_dict(), "optimizer": optimizer.state_dict() if optimizer is not None else None,
                "step": step, "rng_state": {"python": random.getstate(), "torch": torch.get_rng_state()},
                "world_size": ctx.global_size, "rank": ctx.global_rank, "layout": ctx.layout(), "extra": extra}, tmp)
    os.replace(tmp, shard_path(directory, ctx.global_rank))
    _barrier()
    if ctx.global_rank == 0:
        write_checkpoint_metadata(directory, model.config, tokenizer, step, extra)
    _barrier()


def load_sharded_checkpoint(directory, model, optimizer, ctx, extra_out: Optional[dict] = None) -> int:
    """Every rank reads its own shard; the ranks agree on success first (one small all-reduce), so a missing or
    unreadable shard makes EVERY rank raise the same error instead of leaving the others waiting in a collective."""
    import torch.distributed as dist

    from ..training.trainer import restore_rng

    path = shard_path(directory, ctx.global_rank)
    ckpt, problem = None, None
    try:
        ckpt = load_checkpoint(path, map_location=ctx.device)
    except Exception as exc:  # noqa: BLE001 - reported collectively below
        problem = f"{path}: {type(exc).__name__}: {exc}"
    if dist.is_initialized() and ctx.global_size > 1:
        ok = torch.tensor([0 if problem else 1], dtype=torch.int32,
                          device=ctx.device if ctx.device.type == "cuda" else "cpu")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if not int(ok.item()) and problem is None:
            problem = "another rank could not read its shard"
    if problem is not None:
        raise RuntimeError(f"cannot resume from the sharded checkpoint in {directory} (rank {ctx.global_rank}): "
                           f"{problem}")
    if ckpt["world_size"] != ctx.global_size or ckpt.get("layout", ctx.layout()) != ctx.layout():
        raise ValueError(f"checkpoint was written with layout {ckpt.get('layout')} on {ckpt['world_size']} ranks but "
                         f"this run is {ctx.layout()} on {ctx.global_size}")
    model.load_state_dict(ckpt["model"])
    if ckpt.get("optimizer") is not None and optimizer is not None:
        optimizer.load_state_dict(ckpt["optimizer"])
    restore_rng(ckpt.get("rng_state", {}), ctx.device)
    if extra_out is not None:
        extra_out.update(ckpt.get("extra", {}))
    return int(ckpt["step"])


def _merge_expert_parallel(states: list) -> dict:
    """[(ep_rank, tp-merged state)] -> one state with experts renumbered globally."""
    indices = [int(m.group(2)) for key in states[0][1] for m in [EXPERT_KEY.search(key)] if m]
    per_rank = max(indices) + 1 if indices else 0
    merged: dict = {}
    for ep_rank, state in states:
        for key, tensor in state.items():
            match = EXPERT_KEY.search(key)
            if match is None:
                merged.setdefault(key, tensor)
            else:
                index = ep_rank * per_rank + int(match.group(2))
                merged[EXPERT_KEY.sub(lambda m: f"{m.group(1)}{index}{m.group(3)}", key, count=1)] = tensor
    return merged


def _merge_sequence_parallel(shards: list, config: Optional[QuantaWeaveConfig]) -> dict:
    """Attention slices merged over all ranks, experts renumbered by rank, replicated tensors from rank 0."""
    shards = sorted(shards, key=lambda s: s["layout"]["ep_rank"])
    qf = None
    if config is not None and config.num_kv_heads != config.attention_heads:
        qf = config.attention_heads / (config.attention_heads + 2 * config.num_kv_heads)
    states = []
    for shard in shards:
        state = dict(shard["model"])
        for key in list(state):
            if is_tp_sharded_shared(key):
                state[key] = merge_tensors(key, [s["model"][key] for s in shards], qf)
        states.append((shard["layout"]["ep_rank"], state))
    return _merge_expert_parallel(states)


def _sequence_parallel_shard(state: dict, rank: int, world: int, config: QuantaWeaveConfig) -> dict:
    """One rank's sequence-parallel shard of a full state: attention slice ``rank``, its experts whole."""
    per = config.num_experts // world
    attention = {k: v for k, v in state.items() if is_tp_sharded_shared(k)}
    out = shard_state_dict(attention, rank, world, config)
    for key, tensor in state.items():
        if key in attention:
            continue
        match = EXPERT_KEY.search(key)
        if match is None:
            out[key] = tensor
            continue
        index = int(match.group(2))
        if rank * per <= index < (rank + 1) * per:
            out[EXPERT_KEY.sub(lambda m: f"{m.group(1)}{index - rank * per}{m.group(3)}", key, count=1)] = tensor
    return out


def _merge_pipeline(shards: list) -> dict:
    merged: dict = {}
    for shard in sorted(shards, key=lambda s: s["layout"]["stage"]):
        if shard["layout"].get("dp_rank", 0) != 0:
            continue
        start = shard["layout"]["layer_start"]
        for key, tensor in shard["model"].items():
            match = BLOCK_KEY.match(key)
            if match:
                key = f"blocks.{start + int(match.group(1))}." + key[match.end():]
            merged[key] = tensor
    return merged


def _config(directory: Path) -> Optional[QuantaWeaveConfig]:
    path = directory / "config.json"
    return QuantaWeaveConfig.load(path) if path.exists() else None


def consolidate_checkpoint(shards_dir, output_dir) -> None:
    shards_dir, output_dir = Path(shards_dir), Path(output_dir)
    shards, rank = [], 0
    while shard_path(shards_dir, rank).exists():
        shards.append(load_checkpoint(shard_path(shards_dir, rank), map_location="cpu"))
        rank += 1
    if not shards:
        raise FileNotFoundError(f"no shards under {shards_dir}")
    world = shards[0]["world_size"]
    if len(shards) != world:
        raise ValueError(f"expected {world} shards under {shards_dir}, found {len(shards)}")
    for shard in shards:
        shard.setdefault("layout", {"kind": "ep", "ep_rank": shard["rank"], "ep_size": world, "tp_rank": 0, "tp_size": 1})
    kind = shards[0]["layout"]["kind"]
    if kind == "pp":
        merged = _merge_pipeline(shards)
    elif kind == "dp":
        merged = shards[0]["model"]
    elif shards[0]["layout"].get("sequence_parallel"):
        merged = _merge_sequence_parallel(shards, _config(shards_dir))
    else:
        config = _config(shards_dir)
        by_ep: dict = {}
        for shard in shards:
            by_ep.setdefault(shard["layout"]["ep_rank"], []).append(shard)
        states = []
        for ep_rank in sorted(by_ep):
            group = sorted(by_ep[ep_rank], key=lambda s: s["layout"]["tp_rank"])
            tp_states = [s["model"] for s in group]
            states.append((ep_rank, merge_state_dicts(tp_states, config) if len(tp_states) > 1 else tp_states[0]))
        merged = _merge_expert_parallel(states)
    output_dir.mkdir(parents=True, exist_ok=True)
    torch.save({"model": merged, "optimizer": None, "step": shards[0]["step"], "rng_state": {},
                "extra": shards[0]["extra"]}, output_dir / "model.pt")
    for name in _COPIED:
        if (shards_dir / name).exists():
            shutil.copy(shards_dir / name, output_dir / name)


def reshard_checkpoint(checkpoint_dir, output_dir, ep_size: int, tp_size: int = 1,
                       sequence_parallel: bool = False) -> dict:
    """Split a single-file checkpoint into ``ep_size x tp_size`` weights-only shards (optimizer ``None``); with
    ``sequence_parallel`` into ``ep_size`` shards for the orthogonal mapping (``tp_size`` must equal ``ep_size``)."""
    checkpoint_dir, output_dir = Path(checkpoint_dir), Path(output_dir)
    cfg_dict = json.loads((checkpoint_dir / "config.json").read_text())
    config = QuantaWeaveConfig.from_dict(cfg_dict)
    if sequence_parallel:
        if tp_size not in (1, ep_size):
            raise ValueError("sequence-parallel shards put attention TP and expert EP on the same ranks: "
                             "tp_size must equal ep_size")
        if config.num_experts % ep_size or config.attention_heads % ep_size or config.num_kv_heads % ep_size:
            raise ValueError(f"experts and attention heads must be divisible by {ep_size}")
        ckpt = load_checkpoint(checkpoint_dir / "model.pt", map_location="cpu")
        output_dir.mkdir(parents=True, exist_ok=True)
        for rank in range(ep_size):
            torch.save({"model": _sequence_parallel_shard(ckpt["model"], rank, ep_size, config), "optimizer": None,
                        "step": ckpt.get("step", 0), "rng_state": {}, "world_size": ep_size, "rank": rank,
                        "layout": {"kind": "ep", "ep_rank": rank, "ep_size": ep_size, "tp_rank": rank,
                                   "tp_size": ep_size, "sequence_parallel": True},
                        "extra": ckpt.get("extra", {})}, shard_path(output_dir, rank))
        for name in _COPIED:
            if (checkpoint_dir / name).exists():
                shutil.copy(checkpoint_dir / name, output_dir / name)
        return {"ep_size": ep_size, "tp_size": ep_size, "world_size": ep_size, "sequence_parallel": True,
                "per_rank_experts": config.num_experts // ep_size,
                "shards": [str(shard_path(output_dir, r)) for r in range(ep_size)]}
    if config.num_experts % ep_size:
        raise ValueError(f"num_experts {config.num_experts} must be divisible by ep_size {ep_size}")
    if tp_size > 1:
        if config.attention_heads % tp_size or config.num_kv_heads % tp_size:
            raise ValueError(f"attention heads must be divisible by tp_size {tp_size}")
        if config.ffn_size % tp_size:
            raise ValueError(f"ffn_size {config.ffn_size} must be divisible by tp_size {tp_size}")
    ckpt = load_checkpoint(checkpoint_dir / "model.pt", map_location="cpu")
    state = ckpt["model"]
    per_rank = config.num_experts // ep_size
    output_dir.mkdir(parents=True, exist_ok=True)
    for ep_rank in range(ep_size):
        keep = range(ep_rank * per_rank, (ep_rank + 1) * per_rank)
        ep_state: dict = {}
        for key, tensor in state.items():
            match = EXPERT_KEY.search(key)
            if match is None:
                ep_state[key] = tensor
                continue
            index = int(match.group(2))
            if index in keep:
                local = index - ep_rank * per_rank
                ep_state[EXPERT_KEY.sub(lambda m: f"{m.group(1)}{local}{m.group(3)}", key, count=1)] = tensor
        for tp_rank in range(tp_size):
            shard_state = shard_state_dict(ep_state, tp_rank, tp_size, config) if tp_size > 1 else ep_state
            global_rank = ep_rank * tp_size + tp_rank
            torch.save({"model": shard_state, "optimizer": None, "step": ckpt.get("step", 0), "rng_state": {},
                        "world_size": ep_size * tp_size, "rank": global_rank,
                        "layout": {"kind": "ep", "ep_rank": ep_rank, "ep_size": ep_size, "tp_rank": tp_rank,
                                   "tp_size": tp_size},
                        "extra": ckpt.get("extra", {})}, shard_path(output_dir, global_rank))
    for name in _COPIED:
        if (checkpoint_dir / name).exists():
            shutil.copy(checkpoint_dir / name, output_dir / name)
    return {"ep_size": ep_size, "tp_size": tp_size, "world_size": ep_size * tp_size, "per_rank_experts": per_rank,
            "shards": [str(shard_path(output_dir, r)) for r in range(ep_size * tp_size)]}
