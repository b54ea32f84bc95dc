"""Process-group plumbing: one process per GPU, ``torch.distributed`` with NCCL on CUDA and gloo on CPU.

Rendezvous comes from torchrun's environment (``RANK``, ``WORLD_SIZE``, ``LOCAL_RANK``, ``MASTER_ADDR``/``PORT``).
A finite timeout (``QW_PG_TIMEOUT_S``, default 600 s) makes ranks that wait on a dead peer fail with an error
instead of hanging.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def ensure_process_group(device_arg: str = "auto") -> tuple[bool, torch.device]:
    """(owns_group, device) after joining or creating the default process group."""
    if dist.is_initialized():
        if dist.get_backend() == "nccl":
            return False, torch.device("cuda", torch.cuda.current_device())
        return False, torch.device("cpu")
    missing = [name for name in ("RANK", "WORLD_SIZE") if name not in os.environ]
    if missing:
        raise RuntimeError("multi-process parallelism needs a process group; launch with torchrun (missing "
                           + ", ".join(missing) + ")")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    local = int(os.environ.get("LOCAL_RANK", 0))
    timeout = timedelta(seconds=float(os.environ.get("QW_PG_TIMEOUT_S", "600")))
    if device_arg in {"auto", "cuda", "rocm"} and torch.cuda.is_available():
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", rank=int(os.environ["RANK"]), world_size=int(os.environ["WORLD_SIZE"]),
                                timeout=timeout, device_id=device)
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", rank=int(os.environ["RANK"]), world_size=int(os.environ["WORLD_SIZE"]),
                                timeout=timeout)
    return True, device


def barrier() -> None:
    if not dist.is_initialized():
        return
    if dist.get_backend() == "nccl":
        dist.barrier(device_ids=[torch.cuda.current_device()])
    else:
        dist.barrier()


def finish(ctx) -> None:
    barrier()
    if getattr(ctx, "owns_process_group", False) and dist.is_initialized():
        dist.destroy_process_group()
