"""Continuous batching: concurrent generation requests share the decode steps of one ``FastDecoder``.

The reference server runs one request at a time behind an ``asyncio.Lock`` (``src/serve_quantweave.py:211-354``)
and its decoder is batch-1 (``src/fast_decode.py:86-379``). Here the decoder's ``max_batch`` cache rows are slots:

* ``submit`` queues a request (prompt ids, token budget, sampling settings, seed, stop ids, optional per-token
  callback);
* ``step`` admits queued requests into free slots — each prompt is prefilled into its own cache row — then runs ONE
  decode step over all slots (the full batch, so the captured CUDA graph replays), samples every active row with its
  own settings and generator, delivers the token and retires rows that hit a stop id or their budget. Idle slots
  decode a dummy token at position 0 of their own row, which the next request's prefill overwrites.

Requests therefore join and leave between steps without waiting for each other, and a step costs the same whether
one or ``max_batch`` requests are active.
"""

from __future__ import annotations

import threading
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch

from .fast_decode import FastDecoder, filter_logits


@dataclass
class GenerationRequest:
    prompt: list
    max_new: int
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 0
    stop_ids: tuple = ()
    on_token: Optional[Callable[[int], None]] = None
    logit_bias: Optional[torch.Tensor] = None  # added to the logits before sampling (e.g. -inf on invalid ids)
    cancelled: bool = False  # set (e.g. by ``on_token`` on a text stop string) to retire the request after this token
    # results
    tokens: list = field(default_factory=list)
    finish_reason: Optional[str] = None
    done: threading.Event = field(default_factory=threading.Event)

    def wait(self, timeout: Optional[float] = None) -> list:
        if not self.done.wait(timeout):
            raise TimeoutError("generation did not finish in time")
        return self.tokens


class ContinuousBatcher:
    def __init__(self, decoder: FastDecoder) -> None:
        if decoder.native and not hasattr(decoder, "_C"):
            from ..ops import ext

            decoder._C = ext()  # the native prefill's RoPE / attention entry points
        self.decoder = decoder
        self.slots = decoder.max_batch
        self.active: dict[int, GenerationRequest] = {}
        self.waiting: deque = deque()
        self.lock = threading.Lock()
        self._position = [0] * self.slots
        self._next_token = [0] * self.slots
        self._generators: dict[int, torch.Generator] = {}
        self.steps = 0

    # ---- queue --------------------------------------------------------------------------------------------
    def submit(self, request: GenerationRequest) -> GenerationRequest:
        if not request.prompt:
            raise ValueError("a request needs at least one prompt token")
        if request.max_new < 1:
            raise ValueError("max_new must be positive")
        if len(request.prompt) + request.max_new > self.decoder.capacity:
            raise ValueError(f"prompt ({len(request.prompt)}) + max_new ({request.max_new}) exceed the decoder "
                             f"context {self.decoder.capacity}")
        with self.lock:
            self.waiting.append(request)
        return request

    def withdraw(self, request: GenerationRequest) -> bool:
        """Take a request that has not reached a slot yet back out of the queue; False once it is decoding."""
        with self.lock:
            try:
                self.waiting.remove(request)
            except ValueError:
                return False
        request.finish_reason = "withdrawn"
        request.done.set()
        return True

    def pending(self) -> int:
        with self.lock:
            return len(self.waiting) + len(self.active)

    # ---- scheduling ---------------------------------------------------------------------------------------
    def _admit(self) -> None:
        while True:
            with self.lock:
                free = [s for s in range(self.slots) if s not in self.active]
                if not free or not self.waiting:
                    return
                request = self.waiting.popleft()
            slot = free[0]
            prompt = list(request.prompt)
            try:
                self.decoder._prefill(torch.tensor([prompt[:-1]], dtype=torch.long), first_row=slot)
            except BaseException as exc:
                # the request left the queue but never reached a slot: finish it here so its waiter returns
                request.finish_reason = f"error: {exc}"
                request.done.set()
                raise
            self._position[slot] = len(prompt) - 1
            self._next_token[slot] = prompt[-1]
            self._generators[slot] = torch.Generator().manual_seed(request.seed)
            with self.lock:
                self.active[slot] = request

    def _sample(self, logits: torch.Tensor, request: GenerationRequest, generator: torch.Generator) -> int:
        if request.logit_bias is not None:
            logits = logits + request.logit_bias
        if request.temperature <= 0:
            return int(logits.argmax())
        filtered = filter_logits(logits[None] / request.temperature, request.top_k, request.top_p)[0]
        return int(torch.multinomial(filtered.softmax(-1), 1, generator=generator))

    @torch.no_grad()
    def step(self) -> int:
        """Admit queued requests, advance every active one by one token; returns the number still active."""
        self._admit()
        with self.lock:
            rows = sorted(self.active)
        if not rows:
            return 0
        dev = self.decoder.device
        tokens = torch.tensor([self._next_token[s] if s in rows else 0 for s in range(self.slots)], device=dev)
        positions = torch.tensor([self._position[s] if s in rows else 0 for s in range(self.slots)],
                                 dtype=torch.int32, device=dev)
        logits = self.decoder.run_step(tokens, positions)[rows].float().cpu()
        self.steps += 1
        for i, slot in enumerate(rows):
            request = self.active[slot]
            token = self._sample(logits[i], request, self._generators[slot])
            request.tokens.append(token)
            if request.on_token is not None:
                request.on_token(token)
            self._position[slot] += 1
            self._next_token[slot] = token
            reason = None
            if request.cancelled or token in request.stop_ids:
                reason = "stop"
            elif len(request.tokens) >= request.max_new or self._position[slot] + 1 >= self.decoder.capacity:
                reason = "length"
            if reason is not None:
                request.finish_reason = reason
                with self.lock:
                    del self.active[slot]
                request.done.set()
        with self.lock:
            return len(self.active)

    def run_until_idle(self) -> None:
        while self.pending():
            self.step()


class BatchingWorker:
    """A background thread that keeps stepping a ``ContinuousBatcher`` while requests are queued or active."""

    def __init__(self, batcher: ContinuousBatcher) -> None:
        self.batcher = batcher
        self._wake = threading.Event()
        self._stop = threading.Event()
        self.error: Optional[BaseException] = None
        self._thread = threading.Thread(target=self._loop, name="qw-batcher", daemon=True)
        self._thread.start()

    def submit(self, request: GenerationRequest) -> GenerationRequest:
        if self._stop.is_set():
            raise RuntimeError("the batching worker is closed")
        self.batcher.submit(request)
        self._wake.set()
        return request

    def _loop(self) -> None:
        while not self._stop.is_set():
            if not self.batcher.pending():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                self.batcher.step()
            except BaseException as exc:  # noqa: BLE001 - fail every waiting request instead of hanging them
                self.error = exc
                self._fail_all(f"error: {exc}")

    def _fail_all(self, reason: str) -> None:
        with self.batcher.lock:
            stuck = list(self.batcher.active.values()) + list(self.batcher.waiting)
            self.batcher.active.clear()
            self.batcher.waiting.clear()
        for request in stuck:
            request.finish_reason = reason
            request.done.set()

    def close(self) -> None:
        """Stop stepping; requests still queued or in flight finish with reason ``closed``."""
        self._stop.set()
        self._wake.set()
        self._thread.join(timeout=5)
        self._fail_all("closed")
