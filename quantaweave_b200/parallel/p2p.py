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


def _index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


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
        dist.barrier(group=self.group, device_ids=[_index(device)] if device.type == "cuda" else None)
        self._grow(capacity_bytes)

    def _group_name(self):
        return self.group.group_name

    @classmethod
    def for_group(cls, group, device) -> "P2PTransport":
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:  # collectives and symmetric memory name the GPU
            device = torch.device("cuda", torch.cuda.current_device())
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


class _RowStore:
    """A persistent symmetric receive buffer that one layer's forward dispatch writes into and its backward reads
    (the rows, routing weights and counts of every source). It stays mapped in every peer; ``held`` is set while a
    pending backward still needs its contents."""

    def __init__(self, transport: "P2PTransport", nbytes: int) -> None:
        t = transport
        self.nbytes = nbytes
        self.buf = t.symm.empty(nbytes, dtype=torch.uint8, device=t.device)
        self.handle = t.symm.rendezvous(self.buf, t._group_name())
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=t.device)
        self.held = False


class FusedTransport(P2PTransport):
    """Expert-parallel exchange fused into the routing kernels and the expert GEMMs (``csrc/ep_fused.cu``,
    ``csrc/gemm_tcgen05.cuh`` peer-store epilogue).

    * ``dispatch`` (the permute): each routed row, its routing weight and this rank's per-expert counts are stored
      straight into the owning rank's receive buffer. In the forward pass that buffer is the layer's own persistent
      :class:`_RowStore`, so the rows the backward needs are never copied; the backward's gradient rows use the
      two-parity send channel.
    * combine: the expert rank's down-projection GEMM (forward) or input-gradient GEMM (backward) stores each output
      row over NVLink into the SOURCE rank's return buffer, at the row the source's own routing plan names
      (``route_row``); ``publish`` releases a flag to every peer, ``wait_returned`` waits for all expert ranks, and
      the source reduces its top-k rows locally in a fixed order. Only routed rows cross NVLink.

    Store reuse is safe without extra synchronisation: a rank finishes a layer's forward only after every expert
    rank pushed that layer's outputs, which each does after its GEMMs finished reading the layer's store; a backward
    reads the store before it pushes the layer's input gradients, which every source waits for.
    """

    def __init__(self, group, device: torch.device, capacity_bytes: int = 1 << 20) -> None:
        super().__init__(group, device, capacity_bytes)
        self.send = _Channel(self)
        self.back = _Channel(self)
        self._stores: dict = {}
        dist.barrier(group=self.group, device_ids=[_index(device)] if device.type == "cuda" else None)

    @classmethod
    def for_group(cls, group, device) -> "FusedTransport":
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        key = ("fused", id(group), str(device))
        if key not in _TRANSPORTS:
            _TRANSPORTS[key] = cls(group, device)
        return _TRANSPORTS[key]

    @staticmethod
    def _layout(rows: int, H: int, groups: int) -> tuple[int, int, int]:
        w_off = (rows * H * 2 + 255) // 256 * 256
        c_off = (w_off + rows * 4 + 255) // 256 * 256
        return w_off, c_off, c_off + groups * 4

    def store_for(self, key, rows: int, H: int, groups: int, hold: bool) -> _RowStore:
        """The first free persistent store of layer ``key`` that fits (a new one, collectively, if none does);
        ``hold`` marks it busy until :meth:`release`. Every rank takes the same path, so allocations match."""
        need = self._layout(rows, H, groups)[2]
        pool = self._stores.setdefault(key, [])
        store = next((s for s in pool if not s.held and s.nbytes >= need), None)
        if store is None:
            torch.cuda.synchronize(self.device)
            store = _RowStore(self, (need + (1 << 20) - 1) // (1 << 20) * (1 << 20))
            pool.append(store)
        store.held = hold
        return store

    @staticmethod
    def release(store: _RowStore) -> None:
        store.held = False

    def dispatch(self, x: Tensor, route_row: Tensor, top_w, kept, k: int, E: int, local: int, slot: int,
                 pad_counts: Tensor | None = None, store: _RowStore | None = None):
        """Rows (and, when given, weights and counts) of this rank's routes into the owners' receive buffers: the
        layer ``store`` when given, else the send channel's current parity. Returns views of this rank's receive
        buffer: rows [world*local*slot, H] bf16, weights [rows] fp32, counts [world*local] int32."""
        from ..ops import ext

        C = ext()
        H = x.size(1)
        groups = self.world * local
        rows = groups * slot
        w_off, c_off, total = self._layout(rows, H, groups)
        ch = self.send
        parity = ch.next()
        if store is None:
            ch.grow(total)
            buf, _, peers = ch.bufs[parity]
        else:
            buf, peers = store.buf, store.peers
        C.ep_dispatch(x.contiguous(), route_row, top_w, kept, k, E, local, slot, self.me, peers, w_off, c_off,
                      ch.peer_flags[parity], ch.epoch, ch.done)
        ch.wait(parity)
        rows_t = buf[: rows * H * 2].view(torch.bfloat16).view(rows, H)
        w_t = buf[w_off:w_off + rows * 4].view(torch.float32)
        counts = buf[c_off:c_off + groups * 4].view(torch.int32)
        counts_for_pad = counts if kept is not None else pad_counts
        C.ep_pad(counts_for_pad, slot, rows_t, w_t if top_w is not None else None)
        return rows_t, w_t, counts

    def return_buffer(self, rows: int, H: int) -> tuple[Tensor, Tensor]:
        """(this rank's return buffer [rows, H] bf16 for the next combine, every rank's buffer address): the expert
        GEMM's peer-store epilogue writes into the addresses, this rank reduces from its own buffer."""
        ch = self.back
        ch.grow(rows * H * 2)
        self._back_parity = ch.next()
        buf, _, peers = ch.bufs[self._back_parity]
        return buf[: rows * H * 2].view(torch.bfloat16).view(rows, H), peers

    def publish(self) -> None:
        """Release this rank's pushed rows to every peer (after the pushing GEMM, in stream order)."""
        from ..ops import ext

        ch = self.back
        ext().ep_signal(ch.peer_flags[self._back_parity], self.me, ch.epoch)

    def wait_returned(self) -> None:
        """Wait (bounded) until every expert rank has published its rows into this rank's return buffer."""
        self.back.wait(self._back_parity)
