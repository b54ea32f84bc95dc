"""In-kernel NVLink exchange for expert-parallel dispatch/combine (the transport that replaces NCCL all-to-all).

Buffers come from PyTorch's symmetric memory (CUDA VMM allocations mapped into every peer); this module passes the
peers' raw addresses to the ``p2p_push`` kernel, which stores each destination's block straight into that peer's
receive buffer with SM stores over NVLink and publishes a per-source flag with a system-scope release store.
``p2p_wait`` spins on the local flags with acquire loads and a time budget (a lost peer becomes a status code, not a
hang). Receive buffers alternate between two parities: a rank can run at most one exchange ahead of a peer, so the
buffer it writes is never one the peer is still reading. NVLS multicast is disabled: only plain peer stores are used.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor

_TRANSPORTS: dict = {}


class P2PTransport:
    def __init__(self, group, device: torch.device, capacity_bytes: int = 64 << 20) -> None:
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm

        self.symm = symm
        self.group = group if group is not None else dist.group.WORLD
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(self.group.group_name)
            except Exception:  # noqa: BLE001 - newer releases enable every group implicitly
                pass
        self.world = dist.get_world_size(self.group)
        self.me = dist.get_rank(self.group)
        self.device = device
        self.epoch = 0
        self.timeout_s = float(os.environ.get("QW_P2P_TIMEOUT_S", "5"))
        self.capacity = 0
        self._buffers = None
        flags = symm.empty(2 * self.world, dtype=torch.int32, device=device)
        flags.zero_()
        self._flags = flags
        self._flags_handle = symm.rendezvous(flags, self._group_name())
        ptrs = [int(p) for p in self._flags_handle.buffer_ptrs]
        self._peer_flags = [torch.tensor([p + parity * self.world * 4 for p in ptrs], dtype=torch.int64, device=device)
                            for parity in range(2)]
        self._done = torch.zeros(self.world, dtype=torch.int32, device=device)
        dist.barrier(group=self.group, device_ids=[device.index] if device.type == "cuda" else None)
        self._grow(capacity_bytes)

    def _group_name(self):
        return self.group.group_name

    @classmethod
    def for_group(cls, group, device) -> "P2PTransport":
        key = (id(group), str(device))
        if key not in _TRANSPORTS:
            _TRANSPORTS[key] = cls(group, device)
        return _TRANSPORTS[key]

    def _grow(self, nbytes: int) -> None:
        """Collective: every rank must request the same size (exchange sizes are identical across ranks)."""
        nbytes = (nbytes + (1 << 20) - 1) // (1 << 20) * (1 << 20)
        if nbytes <= self.capacity:
            return
        torch.cuda.synchronize(self.device)
        bufs = []
        for _ in range(2):
            t = self.symm.empty(nbytes, dtype=torch.uint8, device=self.device)
            h = self.symm.rendezvous(t, self._group_name())
            peers = torch.tensor([int(p) for p in h.buffer_ptrs], dtype=torch.int64, device=self.device)
            bufs.append((t, h, peers))
        self._buffers = bufs
        self.capacity = nbytes

    def exchange(self, t: Tensor) -> Tensor:
        """Even all-to-all: block ``d`` of ``t`` (split along dim 0 into ``world`` blocks) goes to rank ``d``; the
        result holds block ``s`` from every source ``s`` at position ``s``."""
        from ..ops import ext

        C = ext()
        t = t.contiguous()
        nbytes = t.numel() * t.element_size()
        if nbytes % (16 * self.world):
            raise ValueError("p2p exchange: each block must be a multiple of 16 bytes")
        self._grow(nbytes)
        self.epoch += 1
        parity = self.epoch % 2
        buf, _, peers = self._buffers[parity]
        C.p2p_push(t, nbytes // self.world, peers, self._peer_flags[parity], self.me, self.epoch, self._done)
        C.p2p_wait(self._flags[parity * self.world:(parity + 1) * self.world], self.world, self.epoch, self.timeout_s)
        return buf[:nbytes].view(t.dtype).view(t.shape).clone()

    def exchange_counts(self, kept: Tensor) -> Tensor:
        padded = torch.zeros(self.world, 4 * ((kept.numel() // self.world + 3) // 4), dtype=kept.dtype,
                             device=kept.device)
        padded[:, : kept.numel() // self.world] = kept.view(self.world, -1)
        out = self.exchange(padded)
        return out[:, : kept.numel() // self.world].reshape(-1).contiguous()


class _Channel:
    """Two-parity symmetric buffers with per-source flags and an epoch (one direction of the fused EP exchange)."""

    def __init__(self, transport: "P2PTransport") -> None:
        self.t = transport
        symm, dev, world = transport.symm, transport.device, transport.world
        self.flags = symm.empty(2 * world, dtype=torch.int32, device=dev)
        self.flags.zero_()
        handle = symm.rendezvous(self.flags, transport._group_name())
        ptrs = [int(p) for p in handle.buffer_ptrs]
        self.peer_flags = [torch.tensor([p + parity * world * 4 for p in ptrs], dtype=torch.int64, device=dev)
                           for parity in range(2)]
        self._flag_handle = handle
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        self.capacity = 0
        self.bufs: list = []

    def grow(self, nbytes: int) -> None:
        """Collective: every rank asks for the same size."""
        nbytes = (nbytes + (1 << 20) - 1) // (1 << 20) * (1 << 20)
        if nbytes <= self.capacity:
            return
        t = self.t
        torch.cuda.synchronize(t.device)
        bufs = []
        for _ in range(2):
            buf = t.symm.empty(nbytes, dtype=torch.uint8, device=t.device)
            handle = t.symm.rendezvous(buf, t._group_name())
            peers = torch.tensor([int(p) for p in handle.buffer_ptrs], dtype=torch.int64, device=t.device)
            bufs.append((buf, handle, peers))
        self.bufs = bufs
        self.capacity = nbytes

    def next(self) -> int:
        self.epoch += 1
        return self.epoch % 2

    def wait(self, parity: int) -> None:
        from ..ops import ext

        w = self.t.world
        ext().p2p_wait(self.flags[parity * w:(parity + 1) * w], w, self.epoch, self.t.timeout_s)


class FusedTransport(P2PTransport):
    """Expert-parallel exchange fused into the routing kernels (``csrc/ep_fused.cu``).

    ``dispatch`` stores each routed row (and its weight and the per-expert counts) straight into the owning rank's
    receive buffer; ``return_buffer`` / ``publish`` / ``gather`` let the expert rank's GEMM write its output into its
    own symmetric buffer and each source rank pull and reduce its rows with NVLink loads. Plain ``exchange`` (used for
    small tensors) is the P2P push of ``P2PTransport``."""

    def __init__(self, group, device: torch.device, capacity_bytes: int = 1 << 20) -> None:
        super().__init__(group, device, capacity_bytes)
        self.send = _Channel(self)
        self.back = _Channel(self)
        dist.barrier(group=self.group, device_ids=[device.index] if device.type == "cuda" else None)

    @classmethod
    def for_group(cls, group, device) -> "FusedTransport":
        key = ("fused", id(group), str(device))
        if key not in _TRANSPORTS:
            _TRANSPORTS[key] = cls(group, device)
        return _TRANSPORTS[key]

    @staticmethod
    def _layout(rows: int, H: int, groups: int) -> tuple[int, int, int]:
        w_off = (rows * H * 2 + 255) // 256 * 256
        c_off = (w_off + rows * 4 + 255) // 256 * 256
        return w_off, c_off, c_off + groups * 4

    def dispatch(self, x: Tensor, route_row: Tensor, top_w, kept, k: int, E: int, local: int, slot: int,
                 pad_counts: Tensor | None = None):
        """Rows (and, when given, weights and counts) of this rank's routes into the owners' receive buffers.
        Returns views of this rank's receive buffer: rows [world*local*slot, H] bf16, weights [rows] fp32, counts
        [world*local] int32 (valid until the next dispatch of the other parity)."""
        from ..ops import ext

        C = ext()
        H = x.size(1)
        groups = self.world * local
        rows = groups * slot
        w_off, c_off, total = self._layout(rows, H, groups)
        ch = self.send
        ch.grow(total)
        parity = ch.next()
        buf, _, peers = ch.bufs[parity]
        C.ep_dispatch(x.contiguous(), route_row, top_w, kept, k, E, local, slot, self.me, peers, w_off, c_off,
                      ch.peer_flags[parity], ch.epoch, ch.done)
        ch.wait(parity)
        rows_t = buf[: rows * H * 2].view(torch.bfloat16).view(rows, H)
        w_t = buf[w_off:w_off + rows * 4].view(torch.float32)
        counts = buf[c_off:c_off + groups * 4].view(torch.int32)
        counts_for_pad = counts if kept is not None else pad_counts
        C.ep_pad(counts_for_pad, slot, rows_t, w_t if top_w is not None else None)
        return rows_t, w_t, counts

    def return_buffer(self, rows: int, H: int) -> Tensor:
        ch = self.back
        ch.grow(rows * H * 2)
        self._back_parity = ch.next()
        buf = ch.bufs[self._back_parity][0]
        return buf[: rows * H * 2].view(torch.bfloat16).view(rows, H)

    def publish(self) -> None:
        from ..ops import ext

        ch = self.back
        ext().ep_signal(ch.peer_flags[self._back_parity], self.me, ch.epoch)

    def gather(self, route_row: Tensor, top_w, extra, k: int, local: int, slot: int, out: Tensor) -> Tensor:
        from ..ops import ext

        ch = self.back
        ch.wait(self._back_parity)
        ext().ep_gather(ch.bufs[self._back_parity][2], route_row, top_w, extra, None, k, local, slot, self.me, out)
        return out
