"""Serve a checkpoint over HTTP (FastAPI).

    python -m quantaweave_b200.tools.serve --latest --host 127.0.0.1 --port 8000
    curl -s localhost:8000/generate -d '{"prompt": "Once upon a time", "temperature": 0}'
    curl -s localhost:8000/chat -d '{"messages": [{"role": "user", "content": "hi"}]}'
    curl -N localhost:8000/generate/stream -d '{"prompt": "Once upon a time", "tokens": 200}'   # SSE

Parity with the reference ``src/serve_quantweave.py`` (routes ``/health``, ``/metrics``, ``/generate``, ``/chat``,
``/generate/stream`` :377-413; ``RateLimiter`` :114, ``Moderation`` :138, Prometheus ``Metrics`` :158, ``Server``
:217-345 with the queue / timeout / API-key semantics; JSON logs :84-106). Requests reuse the chat tool's
``ChatSession`` so a request behaves like the equivalent ``tools.chat -m`` call. The decoder's KV cache is per-request
state, so requests are serialised behind an asyncio lock and generation runs in a worker thread.

``--batching N`` serves ``/generate`` and ``/generate/stream`` through continuous batching
(``inference.batching``): up to N requests decode together, joining and leaving between decode steps, with no lock
around generation. Greedy output matches the serialised path. Seeded sampling is reproducible but draws differently
(per-request multinomial sampling instead of the session's Gumbel noise). ``/chat`` keeps the serialised session.

Hardening, all opt-in: ``--api-key`` (Bearer or X-API-Key on every route but /health), ``--rate-limit`` per caller per
``--rate-limit-window``, ``--max-queue`` (429 once that many wait), ``--request-timeout`` (503 when a request waits
that long to START; a generation in progress is never cancelled), ``--moderation-blocklist`` (422 on a regex match;
a keyword guardrail, not a safety system).
"""

import argparse
import asyncio
import bisect
import contextlib
import hmac
import json
import logging
import re
import threading
import time
import uuid
from collections import Counter, defaultdict
from pathlib import Path
from typing import Optional

import torch
from pydantic import BaseModel, Field

from .chat import DEFAULT_CHECKPOINT, ChatSession, Settings, load_for_chat, resolve_model

logger = logging.getLogger("quantaweave_b200.serve")


class ClientDisconnected(Exception):
    """Raised inside a streaming producer's worker thread once its client has gone away, to end the generation."""


class GenerateRequest(BaseModel):
    prompt: str
    tokens: int = Field(200, ge=1, le=8192)
    temperature: float = Field(0.8, ge=0)
    top_k: int = Field(0, ge=0)
    top_p: float = Field(1.0, gt=0, le=1)
    seed: Optional[int] = None
    stop: list[str] = Field(default_factory=list)


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatRequest(BaseModel):
    messages: list[ChatMessage]
    system: str = ""
    tokens: int = Field(200, ge=1, le=8192)
    temperature: float = Field(0.8, ge=0)
    top_k: int = Field(0, ge=0)
    top_p: float = Field(1.0, gt=0, le=1)
    seed: Optional[int] = None


class JSONLogFormatter(logging.Formatter):
    """One JSON object per line: time, level, message and every ``extra=`` field."""

    _STANDARD = set(vars(logging.LogRecord("", 0, "", 0, "", (), None))) | {"message", "asctime"}

    def format(self, record: logging.LogRecord) -> str:
        payload = {"time": self.formatTime(record, "%Y-%m-%dT%H:%M:%S"), "level": record.levelname,
                   "message": record.getMessage()}
        payload.update({k: v for k, v in vars(record).items() if k not in self._STANDARD})
        return json.dumps(payload, default=str)


def configure_logging(log_format: str) -> None:
    handler = logging.StreamHandler()
    handler.setFormatter(JSONLogFormatter() if log_format == "json"
                         else logging.Formatter("%(asctime)s %(levelname)s %(message)s"))
    logger.handlers = [handler]
    logger.setLevel(logging.INFO)
    logger.propagate = False


class RateLimiter:
    """At most ``limit`` calls per ``window`` seconds per key (sliding window, in memory); ``None`` disables it.

    Each key keeps the sorted monotonic times of its admitted calls; expired times are cut with one bisection, and a
    key whose window has emptied is forgotten, so memory stays bounded by the callers active in the last window.
    """

    def __init__(self, limit: Optional[int], window: float = 60.0) -> None:
        self.limit, self.window = limit, window
        self.hits: dict[str, list[float]] = {}

    def allow(self, key: str) -> bool:
        if self.limit is None:
            return True
        now = time.monotonic()
        times = self.hits.pop(key, [])
        del times[:bisect.bisect_left(times, now - self.window)]
        admitted = len(times) < self.limit
        if admitted:
            times.append(now)
        if times:
            self.hits[key] = times
        return admitted


class Moderation:
    """Case-insensitive regex blocklist (one pattern per line; blank and ``#`` lines ignored)."""

    def __init__(self, patterns_file: Optional[Path]) -> None:
        self.patterns: list[re.Pattern] = []
        if patterns_file is not None:
            for line in Path(patterns_file).read_text().splitlines():
                line = line.strip()
                if line and not line.startswith("#"):
                    self.patterns.append(re.compile(line, re.IGNORECASE))

    def blocked(self, text: str) -> Optional[str]:
        return next((p.pattern for p in self.patterns if p.search(text)), None)


def _sample(name: str, value, **labels) -> str:
    """One exposition line: ``quantweave_<name>{k="v",...} value`` (floats with 6 decimals)."""
    label_text = "{" + ",".join(f'{k}="{v}"' for k, v in labels.items()) + "}" if labels else ""
    return f"quantweave_{name}{label_text} {value:.6f}" if isinstance(value, float) else \
        f"quantweave_{name}{label_text} {value}"


class Metrics:
    """Prometheus text exposition: requests by route/status, errors, request seconds, tokens, in-flight gauge.

    ``_FAMILIES`` lists each metric family once (name, type, help, and how its samples are read off this object);
    :meth:`render` writes the ``# HELP`` / ``# TYPE`` header and the samples of every family in that order.
    """

    _FAMILIES = (
        ("requests_total", "counter", "Total requests by route and status.",
         lambda m: [_sample("requests_total", n, route=r, status=c) for (r, c), n in sorted(m.requests_total.items())]),
        ("errors_total", "counter", "Total error responses (status >= 400) by route.",
         lambda m: [_sample("errors_total", n, route=r) for r, n in sorted(m.errors_total.items())]),
        ("request_seconds_sum", "counter", "Total request handling seconds by route.",
         lambda m: [line for r in sorted(m.seconds_sum)
                    for line in (_sample("request_seconds_sum", m.seconds_sum[r], route=r),
                                 _sample("request_seconds_count", m.seconds_count[r], route=r))]),
        ("tokens_generated_total", "counter", "Total tokens generated across all requests.",
         lambda m: [_sample("tokens_generated_total", m.tokens_generated_total)]),
        ("requests_in_flight", "gauge", "Requests currently being handled.",
         lambda m: [_sample("requests_in_flight", m.requests_in_flight)]),
    )

    def __init__(self) -> None:
        self.requests_total: Counter = Counter()
        self.errors_total: Counter = Counter()
        self.seconds_sum: dict[str, float] = defaultdict(float)
        self.seconds_count: Counter = Counter()
        self.tokens_generated_total = 0
        self.requests_in_flight = 0

    def observe(self, route: str, status: int, seconds: float, tokens: int = 0) -> None:
        self.requests_total[route, status] += 1
        if status >= 400:
            self.errors_total[route] += 1
        self.seconds_sum[route] += seconds
        self.seconds_count[route] += 1
        self.tokens_generated_total += tokens

    def render(self) -> str:
        lines = []
        for name, kind, text, samples in self._FAMILIES:
            lines += [f"# HELP quantweave_{name} {text}", f"# TYPE quantweave_{name} {kind}", *samples(self)]
        return "\n".join(lines) + "\n"


def reply_payload(reply) -> dict:
    return {"text": reply.response, "tokens": reply.tokens, "seconds": reply.seconds,
            "tokens_per_second": reply.tokens_per_second, "stop_reason": reply.stop_reason,
            "unknown_characters": reply.unknown_characters, "truncated_context": reply.truncated_context}


class Server:
    """The loaded model, with access to its stateful decoder serialised across requests."""

    def __init__(self, checkpoint, adapter, device: torch.device, precision: str, use_cache: bool = True, *,
                 api_key: Optional[str] = None, rate_limit: Optional[int] = None, rate_limit_window: float = 60.0,
                 request_timeout: Optional[float] = None, max_queue: Optional[int] = None,
                 moderation_patterns: Optional[Path] = None, sessions: Optional[tuple] = None,
                 batching: int = 0) -> None:
        from ..utils.hardware import choose_precision, detect

        self.checkpoint, self.adapter, self.device = checkpoint, adapter, device
        self.precision = choose_precision(detect(device.type), precision)
        if sessions is None:
            model, tokenizer = load_for_chat(checkpoint, adapter, 0, device)
            complete = ChatSession(model, tokenizer, device, self.precision, Settings(mode="complete"), use_cache)
            chat = ChatSession(model, tokenizer, device, self.precision, Settings(mode="chat"), use_cache=False)
            chat.decoder, chat.cache_note = complete.decoder, complete.cache_note  # one decoder (and graph) per model
            sessions = (complete, chat)
        self.complete_session, self.chat_session = sessions
        self.lock = asyncio.Lock()
        self.started_at = time.time()
        self.requests_served = 0
        self.api_key = api_key
        self.rate_limiter = RateLimiter(rate_limit, rate_limit_window)
        self.request_timeout, self.max_queue = request_timeout, max_queue
        self.waiting = 0
        self.moderation = Moderation(moderation_patterns)
        self.metrics = Metrics()
        self.worker = None
        if batching > 0:
            from ..inference.batching import BatchingWorker, ContinuousBatcher
            from ..inference.fast_decode import FastDecoder

            model = self.complete_session.model
            self.batch_decoder = FastDecoder(model, device, self.precision, max_batch=batching)
            self.worker = BatchingWorker(ContinuousBatcher(self.batch_decoder))

    def close(self) -> None:
        if self.worker is not None:
            self.worker.close()

    def _admit_batched(self) -> None:
        from fastapi import HTTPException

        batcher = self.worker.batcher
        if self.max_queue is not None and batcher.pending() >= batcher.slots + self.max_queue:
            raise HTTPException(429, f"too many requests already queued (max {self.max_queue})")

    def _batched(self, request: GenerateRequest, on_text=None, handle: Optional[list] = None) -> dict:
        """One completion through the continuous batcher: the same prompt handling, stop strings (with hold-back
        when streaming), EOS and reply fields as ``ChatSession.send`` in complete mode. ``handle`` (a list) receives
        the queued job, so a caller whose client went away can cancel it."""
        import random

        from fastapi import HTTPException

        from ..inference.batching import GenerationRequest

        session, dec = self.complete_session, self.batch_decoder
        tok = session.tokenizer
        prompt = request.prompt
        ids = tok.encode(prompt) or [tok.eos_id]
        budget = max(1, min(request.tokens, dec.capacity - 1))
        truncated = len(ids) + budget > dec.capacity
        if truncated:
            ids = ids[-(dec.capacity - budget):]
        stops = [x for x in request.stop if x]
        holdback = max((len(x) for x in stops), default=1) - 1
        bias = torch.zeros(dec.vocab)
        if session.valid_ids < dec.vocab:
            bias[session.valid_ids:] = float("-inf")
        if tok.unk_id is not None and 0 <= tok.unk_id < dec.vocab:
            bias[tok.unk_id] = float("-inf")
        state = {"generated": [], "text": "", "emitted": 0, "reason": "length"}
        seed = request.seed if request.seed is not None else random.randrange(1 << 31)
        job = GenerationRequest(ids, budget, request.temperature, request.top_k, request.top_p, seed,
                                stop_ids=(tok.eos_id,), logit_bias=bias)

        def on_token(token: int) -> None:
            if token == tok.eos_id:
                state["reason"] = "eos"
                return
            state["generated"].append(token)
            text = tok.decode(state["generated"])
            hits = [text.find(x) for x in stops if x in text]
            if hits:
                state["text"], state["reason"] = text[: min(hits)], "stop"
                job.cancelled = True
                return
            state["text"] = text
            if on_text is not None:
                safe = max(state["emitted"], len(text) - holdback)
                if safe > state["emitted"]:
                    on_text(text[state["emitted"]:safe])
                    state["emitted"] = safe

        job.on_token = on_token
        if handle is not None:
            handle.append(job)
        started = time.perf_counter()
        self.worker.submit(job)
        if self.request_timeout is not None and not job.done.wait(self.request_timeout):
            if self.worker.batcher.withdraw(job):  # still queued behind busy slots after the start timeout
                raise HTTPException(503, f"timed out after {self.request_timeout}s waiting to start "
                                         "(every decode slot is busy)")
        job.wait()
        if job.finish_reason == "closed":
            raise HTTPException(503, "the server is shutting down")
        if job.finish_reason and job.finish_reason.startswith("error"):
            raise HTTPException(500, job.finish_reason)
        text = state["text"]
        if on_text is not None and len(text) > state["emitted"]:
            on_text(text[state["emitted"]:])
        seconds = time.perf_counter() - started
        count = len(state["generated"])
        return {"text": text, "tokens": count, "seconds": seconds,
                "tokens_per_second": count / seconds if seconds > 0 else 0.0, "stop_reason": state["reason"],
                "unknown_characters": session.unknown_characters(prompt), "truncated_context": truncated}

    def info(self) -> dict:
        s = self.complete_session
        return {"checkpoint": str(self.checkpoint), "adapter": str(self.adapter) if self.adapter else None,
                "device": str(self.device), "precision": self.precision, "decoding": s.cache_note,
                "tokenizer": s.tokenizer.kind, "vocab_size": s.tokenizer.vocab_size,
                "context_length": s.model.config.max_sequence_length - 1,
                "uptime_seconds": time.time() - self.started_at, "requests_served": self.requests_served,
                "auth_required": self.api_key is not None, "rate_limit": self.rate_limiter.limit,
                "request_timeout": self.request_timeout, "max_queue": self.max_queue,
                "batching_slots": self.worker.batcher.slots if self.worker is not None else 0}

    async def _acquire(self) -> None:
        """Take the generation lock. A request that finds it free always proceeds (even ``max_queue=0``); one that
        must wait is refused past ``max_queue`` waiters and gives up after ``request_timeout`` seconds."""
        from fastapi import HTTPException

        if not self.lock.locked():
            await self.lock.acquire()
            return
        if self.max_queue is not None and self.waiting >= self.max_queue:
            raise HTTPException(429, f"too many requests already queued (max {self.max_queue})")
        self.waiting += 1
        try:
            if self.request_timeout is None:
                await self.lock.acquire()
            else:
                try:
                    await asyncio.wait_for(self.lock.acquire(), timeout=self.request_timeout)
                except asyncio.TimeoutError:
                    raise HTTPException(503, f"timed out after {self.request_timeout}s waiting to start "
                                             "(the server may still be busy with an earlier request)") from None
        finally:
            self.waiting -= 1

    def _check(self, text: str, what: str) -> None:
        from fastapi import HTTPException

        pattern = self.moderation.blocked(text)
        if pattern is not None:
            raise HTTPException(422, f"{what} blocked by moderation pattern: {pattern}")

    def _complete_settings(self, r: GenerateRequest) -> Settings:
        return Settings(mode="complete", tokens=r.tokens, temperature=r.temperature, top_k=r.top_k, top_p=r.top_p,
                        seed=r.seed, stop=r.stop)

    async def generate(self, request: GenerateRequest) -> dict:
        self._check(request.prompt, "prompt")
        if self.worker is not None:
            self._admit_batched()
            payload = await asyncio.to_thread(self._batched, request)
            self.requests_served += 1
            self.metrics.tokens_generated_total += payload["tokens"]
            return payload
        await self._acquire()
        try:
            self.complete_session.settings = self._complete_settings(request)
            reply = await asyncio.to_thread(self.complete_session.send, request.prompt)
            self.requests_served += 1
        finally:
            self.lock.release()
        self.metrics.tokens_generated_total += reply.tokens
        return reply_payload(reply)

    async def chat(self, request: ChatRequest) -> dict:
        from fastapi import HTTPException

        if not request.messages or request.messages[-1].role != "user":
            raise HTTPException(422, "messages must end with a 'user' turn")
        self._check(request.messages[-1].content, "message")
        await self._acquire()
        try:
            session = self.chat_session
            session.reset()
            session.settings = Settings(mode="chat", tokens=request.tokens, temperature=request.temperature,
                                        top_k=request.top_k, top_p=request.top_p, seed=request.seed,
                                        system=request.system)
            for turn in request.messages[:-1]:
                if turn.role == "user":
                    session.history.append((turn.content, ""))
                elif turn.role == "assistant" and session.history:
                    session.history[-1] = (session.history[-1][0], turn.content)
            reply = await asyncio.to_thread(session.send, request.messages[-1].content)
            self.requests_served += 1
        finally:
            self.lock.release()
        self.metrics.tokens_generated_total += reply.tokens
        return reply_payload(reply)

    async def _relay(self, produce, cancel=None, interrupt: bool = False):
        """Server-sent events from a blocking producer: ``produce(on_text)`` runs in a worker thread and returns the
        reply payload; every piece it hands to ``on_text`` is sent as ``data: {"text": ...}`` as soon as it exists,
        and the payload follows as ``event: done``. A sentinel queued when the producer returns (or raises) ends the
        stream.

        If the client goes away first, ``cancel`` is called and, with ``interrupt``, the next ``on_text`` call raises
        :class:`ClientDisconnected` inside the worker thread, which ends the producer early. A thread cannot be
        stopped from outside, so the generator then waits until the worker has actually returned: whatever the
        producer uses (the session and its KV cache, guarded by the caller's lock) is free by the time the caller
        releases that lock."""
        loop = asyncio.get_running_loop()
        pieces: asyncio.Queue = asyncio.Queue()
        finished = object()
        gone = threading.Event()

        def on_text(piece: str) -> None:
            if interrupt and gone.is_set():
                raise ClientDisconnected("the streaming client went away")
            loop.call_soon_threadsafe(pieces.put_nowait, piece)

        def work():
            try:
                return produce(on_text)
            finally:
                loop.call_soon_threadsafe(pieces.put_nowait, finished)

        task = asyncio.ensure_future(asyncio.to_thread(work))
        try:
            while (piece := await pieces.get()) is not finished:
                yield f"data: {json.dumps({'text': piece})}\n\n"
            payload = await task
        finally:
            if not task.done():
                gone.set()
                if cancel is not None:
                    cancel()
                while not task.done():  # asyncio.wait never cancels the task it waits on
                    try:
                        await asyncio.wait({task})
                    except asyncio.CancelledError:
                        continue
                if not task.cancelled():
                    task.exception()  # retrieved: the producer's ClientDisconnected is expected here
        self.requests_served += 1
        self.metrics.tokens_generated_total += payload["tokens"]
        yield f"event: done\ndata: {json.dumps(payload)}\n\n"

    async def stream_generate(self, request: GenerateRequest):
        """Server-sent events: ``data: {"text": ...}`` per piece, then ``event: done`` with the full reply. With the
        batching worker the request joins the shared decode; otherwise it holds the session lock while it streams."""
        self._check(request.prompt, "prompt")
        if self.worker is not None:
            self._admit_batched()
            handle: list = []

            def retire() -> None:  # the client went away mid-stream: retire its job at the next decode step
                for job in handle:
                    job.cancelled = True

            events = self._relay(lambda on_text: self._batched(request, on_text, handle), retire)
            async with contextlib.aclosing(events):
                async for event in events:
                    yield event
            return
        await self._acquire()
        try:
            self.complete_session.settings = self._complete_settings(request)
            events = self._relay(lambda on_text: reply_payload(self.complete_session.send(request.prompt, on_text)),
                                 interrupt=True)
            async with contextlib.aclosing(events):
                async for event in events:
                    yield event
        finally:
            self.lock.release()


def build_app(server: Server):
    from fastapi import Depends, FastAPI, HTTPException, Request
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI(title="QuantaWeave-B200 inference server")

    def require_auth(request: Request) -> None:
        """Bearer token or ``X-API-Key``; compared in constant time so the key cannot be probed by timing."""
        if server.api_key is None:
            return
        scheme, _, token = request.headers.get("authorization", "").partition(" ")
        presented = token.strip() if scheme.lower() == "bearer" else request.headers.get("x-api-key", "")
        if not hmac.compare_digest(presented.encode(), server.api_key.encode()):
            raise HTTPException(401, "invalid or missing API key (Authorization: Bearer <key> or X-API-Key: <key>)")

    def require_rate_limit(request: Request) -> None:
        caller = request.headers.get("x-api-key") or (request.client.host if request.client else "unknown")
        if not server.rate_limiter.allow(caller):
            raise HTTPException(429, "rate limit exceeded")

    async def timed(route: str, handler):
        request_id = uuid.uuid4().hex[:12]
        server.metrics.requests_in_flight += 1
        started = time.perf_counter()
        status = 200
        try:
            return await handler()
        except HTTPException as error:
            status = error.status_code
            raise
        except ValueError as error:
            status = 422
            raise HTTPException(422, str(error)) from error
        except Exception:
            status = 500
            raise
        finally:
            seconds = time.perf_counter() - started
            server.metrics.requests_in_flight -= 1
            server.metrics.observe(route, status, seconds)
            logger.log(logging.INFO if status < 400 else logging.WARNING, f"{route} {status} {seconds:.3f}s",
                       extra={"request_id": request_id, "route": route, "status": status,
                              "seconds": round(seconds, 4)})

    @app.get("/health")
    async def health():
        return {"status": "ok", **server.info()}

    @app.get("/metrics")
    async def metrics(_auth: None = Depends(require_auth)):
        return PlainTextResponse(server.metrics.render(), media_type="text/plain; version=0.0.4")

    @app.post("/generate")
    async def generate(request: GenerateRequest, _auth: None = Depends(require_auth),
                       _rate: None = Depends(require_rate_limit)):
        return await timed("/generate", lambda: server.generate(request))

    @app.post("/chat")
    async def chat(request: ChatRequest, _auth: None = Depends(require_auth),
                   _rate: None = Depends(require_rate_limit)):
        return await timed("/chat", lambda: server.chat(request))

    @app.post("/generate/stream")
    async def generate_stream(request: GenerateRequest, _auth: None = Depends(require_auth),
                              _rate: None = Depends(require_rate_limit)):
        return StreamingResponse(server.stream_generate(request), media_type="text/event-stream")

    app.state.server = server
    return app


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, help=f"a checkpoint directory (default {DEFAULT_CHECKPOINT})")
    p.add_argument("--run", help="archived run to load, by its epoch-second name under --runs-dir or by path")
    p.add_argument("--latest", action="store_true", help="load the most recent archived run that holds a model")
    p.add_argument("--adapter", type=Path, help="QLoRA adapter folder, applied on top of --checkpoint")
    p.add_argument("--runs-dir", type=Path, default=Path("artifacts/runs"))
    p.add_argument("--no-cache", action="store_true", help="plain forward pass per token instead of the KV cache")
    p.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    p.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--batching", type=int, default=0, metavar="N",
                   help="continuous batching of /generate and /generate/stream over N decoder slots (0 = one "
                        "request at a time)")
    h = p.add_argument_group("hardening")
    h.add_argument("--api-key", help="require this key (Authorization: Bearer or X-API-Key) on every route but /health")
    h.add_argument("--rate-limit", type=int, help="429 past this many requests per --rate-limit-window per caller")
    h.add_argument("--rate-limit-window", type=float, default=60.0)
    h.add_argument("--request-timeout", type=float, help="503 when a request waits this long merely to start")
    h.add_argument("--max-queue", type=int, help="429 once this many requests are already waiting to start")
    h.add_argument("--moderation-blocklist", type=Path, help="regex patterns (one per line); a match is a 422")
    h.add_argument("--log-format", choices=("text", "json"), default="text")
    from .common import describe_options

    describe_options(p)
    return p


def main(argv=None) -> None:
    from ..training.trainer import select_device

    args = build_parser().parse_args(argv)
    configure_logging(args.log_format)
    checkpoint, adapter = resolve_model(args.checkpoint, args.adapter, args.run, args.latest, args.runs_dir)
    device = select_device(args.device)
    server = Server(checkpoint, adapter, device, args.precision, use_cache=not args.no_cache, api_key=args.api_key,
                    rate_limit=args.rate_limit, rate_limit_window=args.rate_limit_window,
                    request_timeout=args.request_timeout, max_queue=args.max_queue,
                    moderation_patterns=args.moderation_blocklist, batching=args.batching)
    print(f"model: {checkpoint}" + (f" + adapter {adapter}" if adapter else "")
          + f"  device: {device}  decoding: {server.complete_session.cache_note}")
    if server.api_key is None:
        print("WARNING: no --api-key set; this server accepts unauthenticated requests from anyone who can reach it.")
    import uvicorn

    uvicorn.run(build_app(server), host=args.host, port=args.port, log_level="info")


if __name__ == "__main__":
    main()
