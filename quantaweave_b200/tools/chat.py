"""Send messages to a model: an interactive session, one-off messages, or a batch of test messages.

    python -m quantaweave_b200.tools.chat --latest                      # interactive, newest archived run
    python -m quantaweave_b200.tools.chat --checkpoint DIR -m "Once upon a time"
    python -m quantaweave_b200.tools.chat --latest --messages-file tests.jsonl --json
    printf 'Once upon a time\\n' | python -m quantaweave_b200.tools.chat --latest

Parity with the reference ``src/chat_quantweave_moe.py`` (``choose_token`` :54, ``Settings`` :62, ``Reply`` :80,
``ChatSession`` :96-188, ``resolve_model`` :216-232, ``read_messages`` :251-273, ``run_batch`` :276-296, ``repl``
:329-395, CLI :407-494; exit code 1 when an expectation fails). ``complete`` mode continues the message as text (what
a base model does); ``chat`` mode wraps the conversation in ``User:`` / ``Assistant:`` turns and stops at the next
``User:`` line. Sampling is restricted to ids the tokenizer has, never emits ``<unk>``; temperature 0 is greedy.

Decoding runs on ``FastDecoder`` (KV cache; on CUDA the sm_100a decode kernels captured in a CUDA graph); ``--no-cache``
falls back to a full forward pass per token. The usable context is ``max_sequence_length - 1`` tokens.
"""

from __future__ import annotations

import argparse
import json
import re
import sys
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Callable, Iterator, Optional, Sequence

import torch

RUNS_DIR = Path("artifacts/runs")
DEFAULT_CHECKPOINT = Path("artifacts/outputs/quantweave-moe-out")
CHAT_STOPS = ("\nUser:", "\nSystem:")


def choose_token(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                 generator: Optional[torch.Generator]) -> int:
    from ..inference.fast_decode import filter_logits

    if temperature <= 0:
        return int(logits.argmax())
    probs = filter_logits(logits / temperature, top_k, top_p).softmax(dim=-1)
    return int(torch.multinomial(probs, 1, generator=generator))


@dataclass
class Settings:
    mode: str = "complete"
    tokens: int = 200
    temperature: float = 0.8
    top_k: int = 0
    top_p: float = 1.0
    seed: Optional[int] = None
    stop: list[str] = field(default_factory=list)
    system: str = ""

    def validate(self) -> None:
        if self.mode not in {"complete", "chat"}:
            raise ValueError("mode must be complete or chat")
        if self.tokens < 1 or self.temperature < 0 or self.top_k < 0 or not 0 < self.top_p <= 1:
            raise ValueError("tokens must be >= 1, temperature >= 0, top_k >= 0, and top_p in (0, 1]")


@dataclass
class Reply:
    message: str
    prompt: str
    response: str
    tokens: int
    seconds: float
    stop_reason: str  # eos | stop | length
    unknown_characters: list[str] = field(default_factory=list)
    truncated_context: bool = False

    @property
    def tokens_per_second(self) -> float:
        return self.tokens / self.seconds if self.seconds > 0 else 0.0


class ChatSession:
    def __init__(self, model, tokenizer, device: torch.device, precision: str, settings: Settings,
                 use_cache: bool = True) -> None:
        from ..inference.fast_decode import FastDecoder, Unsupported

        settings.validate()
        self.model, self.tokenizer, self.device = model, tokenizer, device
        self.precision, self.settings = precision, settings
        self.history: list[tuple[str, str]] = []
        self.valid_ids = tokenizer.vocab_size
        model.eval()
        self.decoder = None
        self.cache_note = "no cache (full forward pass per token)"
        if use_cache:
            try:
                self.decoder = FastDecoder(model, device, precision)
                self.decoder.warm(settings.temperature, settings.top_k, settings.top_p)
                self.cache_note = self.decoder.description
            except Unsupported as error:
                self.cache_note = f"no cache ({error})"

    def reset(self) -> None:
        self.history.clear()

    def format_prompt(self, message: str) -> str:
        if self.settings.mode == "complete":
            return message
        parts = [f"System: {self.settings.system}\n"] if self.settings.system else []
        parts += [f"User: {u}\nAssistant: {a}\n" for u, a in self.history]
        parts.append(f"User: {message}\nAssistant:")
        return "".join(parts)

    def unknown_characters(self, text: str) -> list[str]:
        vocab = getattr(self.tokenizer, "vocab", None)
        if self.tokenizer.kind != "char" or vocab is None:
            return []
        return sorted({ch for ch in text if ch not in vocab})

    def _plain_tokens(self, ids: list[int], generated: list[int], generator, usable: int) -> Iterator[int]:
        """No cache: one full forward pass over the last ``usable`` tokens per new token."""
        from ..training.trainer import autocast_context

        s, tok = self.settings, self.tokenizer
        while True:
            window = torch.tensor([(ids + generated)[-usable:]], dtype=torch.long, device=self.device)
            with autocast_context(self.device, self.precision):
                logits = self.model(window)["logits"][0, -1].float()
            logits[self.valid_ids:] = float("-inf")
            if tok.unk_id is not None and tok.unk_id < self.valid_ids:
                logits[tok.unk_id] = float("-inf")
            yield choose_token(logits, s.temperature, s.top_k, s.top_p, generator)

    @torch.inference_mode()
    def send(self, message: str, on_text: Optional[Callable[[str], None]] = None) -> Reply:
        """Generate a reply; ``on_text`` receives it as produced, never a partial stop string."""
        s, tok, dec = self.settings, self.tokenizer, self.decoder
        prompt = self.format_prompt(message)
        stops = [x for x in ([*CHAT_STOPS] if s.mode == "chat" else []) + list(s.stop) if x]
        ids = tok.encode(prompt) or [tok.eos_id]
        usable = dec.capacity if dec is not None else self.model.config.max_sequence_length - 1
        generator = torch.Generator(device=self.device).manual_seed(s.seed) if s.seed is not None else None
        holdback = max((len(x) for x in stops), default=1) - 1
        generated: list[int] = []
        text, emitted, reason = "", 0, "length"
        per_char = tok.kind == "char"  # a character's text never depends on its neighbours
        started = time.perf_counter()
        if dec is not None:
            source = dec.stream(ids, s.tokens, temperature=s.temperature, top_k=s.top_k, top_p=s.top_p,
                                valid_ids=self.valid_ids, unk_id=tok.unk_id, generator=generator)
        else:
            source = self._plain_tokens(ids, generated, generator, usable)
        for step, token in enumerate(source):
            if step >= s.tokens:
                break
            if token == tok.eos_id:
                reason = "eos"
                break
            generated.append(token)
            text = text + tok.inverse.get(token, "?") if per_char else tok.decode(generated)
            hits = [text.find(x) for x in stops if x in text]
            if hits:
                text, reason = text[: min(hits)], "stop"
                break
            if on_text is not None:
                safe = max(emitted, len(text) - holdback)
                if safe > emitted:
                    on_text(text[emitted:safe])
                    emitted = safe
        source.close()
        if on_text is not None and len(text) > emitted:
            on_text(text[emitted:])
        seconds = time.perf_counter() - started
        response = text.strip() if s.mode == "chat" else text
        if s.mode == "chat":
            self.history.append((message, response))
        return Reply(message, prompt, response, len(generated), seconds, reason, self.unknown_characters(prompt),
                     len(ids) > usable)


# ---- which model --------------------------------------------------------------------------------------------
def run_folders(root: Path = RUNS_DIR) -> list[Path]:
    """Archived runs (``<epoch>`` or ``<epoch>-<n>``), oldest first."""
    root = Path(root)
    if not root.is_dir():
        return []
    keyed = []
    for path in root.iterdir():
        m = re.fullmatch(r"(\d+)(?:-(\d+))?", path.name)
        if path.is_dir() and m:
            keyed.append(((int(m.group(1)), int(m.group(2) or 0)), path))
    return [p for _, p in sorted(keyed)]


def usable_model(run: Path) -> Optional[tuple[Path, Optional[Path]]]:
    """(checkpoint dir, adapter dir) of an archived run, or None when it holds no model."""
    run = Path(run)
    for sub in ("model", "merged"):
        if (run / sub / "model.pt").exists():
            return run / sub, None
    if (run / "adapter" / "adapter.pt").exists():
        meta = json.loads((run / "adapter" / "finetune_metadata.json").read_text())
        return Path(meta["base_checkpoint"]), run / "adapter"
    return None


def resolve_model(checkpoint: Optional[Path], adapter: Optional[Path], run: Optional[str], latest: bool,
                  root: Path = RUNS_DIR) -> tuple[Path, Optional[Path]]:
    if checkpoint is not None:
        return Path(checkpoint), adapter
    if run is not None:
        folder = Path(run) if Path(run).is_dir() else Path(root) / run
        found = usable_model(folder) if folder.is_dir() else None
        if found is None:
            raise FileNotFoundError(f"no model found in run '{run}' (looked in {folder})")
        return found
    if latest:
        for folder in reversed(run_folders(root)):
            found = usable_model(folder)
            if found is not None:
                return found
        raise FileNotFoundError(f"no archived run with a model under {root}")
    return DEFAULT_CHECKPOINT, adapter


def load_for_chat(checkpoint: Path, adapter: Optional[Path], quantize: int, device: torch.device):
    """(model, tokenizer): an adapter over its (quantised) base, or the checkpoint, optionally quantised in memory."""
    from ..data.pipeline import load_tokenizer

    if adapter is not None:
        from .finetune import load_finetuned

        model = load_finetuned(checkpoint, adapter, device)
    else:
        from .common import load_model

        model = load_model(checkpoint, torch.device("cpu"))
        if quantize:
            from ..inference.quantization import quantize_model

            quantize_model(model, quantize)
        model = model.to(device)
    return model.eval(), load_tokenizer(checkpoint)


# ---- batches of test messages --------------------------------------------------------------------------------
def read_messages(path: Path) -> list[dict]:
    """``.jsonl``: ``{"message"|"prompt", "expect"?: str|list, "tokens", "temperature", "mode", ...}`` per line;
    anything else: one message per line. Blank lines and ``#`` comments are skipped."""
    path = Path(path)
    items = []
    for number, line in enumerate(path.read_text(encoding="utf-8").splitlines(), start=1):
        if not line.strip() or line.lstrip().startswith("#"):
            continue
        if path.suffix == ".jsonl":
            try:
                item = json.loads(line)
            except json.JSONDecodeError as error:
                raise ValueError(f"{path}:{number}: not valid JSON ({error})") from error
            message = item.get("message", item.get("prompt"))
            if message is None:
                raise ValueError(f"{path}:{number}: needs a 'message' field")
            item["message"] = message
        else:
            item = {"message": line}
        expect = item.get("expect")
        item["expect"] = [expect] if isinstance(expect, str) else list(expect or [])
        items.append(item)
    return items


def run_batch(session: ChatSession, items: Sequence[dict], conversation: bool,
              emit: Callable[[dict], None]) -> list[dict]:
    """Send each message (per-message settings override the session's for that message only)."""
    results = []
    base = asdict(session.settings)
    for item in items:
        if not conversation:
            session.reset()
        overrides = {k: item[k] for k in ("mode", "tokens", "temperature", "top_k", "top_p", "seed") if k in item}
        session.settings = Settings(**{**base, **overrides})
        try:
            reply = session.send(item["message"])
        finally:
            session.settings = Settings(**base)
        missing = [needle for needle in item["expect"] if needle not in reply.response]
        result = {**asdict(reply), "tokens_per_second": reply.tokens_per_second, "expect": item["expect"],
                  "passed": None if not item["expect"] else not missing, "missing": missing}
        results.append(result)
        emit(result)
    return results


# ---- interactive session -------------------------------------------------------------------------------------
HELP = """commands:
  /help                  this text
  /reset                 forget the conversation (chat mode)
  /mode complete|chat    switch modes
  /set NAME VALUE        temperature, top_k, top_p, tokens, seed (a number or "none"), system (text)
  /show                  current settings
  /history               the conversation so far
  /save FILE             write the conversation as JSON lines
  /quit                  leave (also Ctrl-D)
anything else is sent to the model."""


def apply_setting(settings: Settings, name: str, value: str) -> None:
    """Change one setting; a value that fails validation leaves the settings untouched."""
    casts = {"temperature": float, "top_p": float, "top_k": int, "tokens": int}
    trial = Settings(**asdict(settings))
    if name == "seed":
        trial.seed = None if value.lower() == "none" else int(value)
    elif name == "system":
        trial.system = value
    elif name in casts:
        setattr(trial, name, casts[name](value))
    else:
        raise ValueError(f"unknown setting '{name}' (try: temperature, top_k, top_p, tokens, seed, system)")
    trial.validate()
    setattr(settings, name, getattr(trial, name))


def _command(session: ChatSession, command: str, rest: str, out) -> bool:
    """Run one ``/command``; returns False to leave the session."""
    if command in {"quit", "exit"}:
        return False
    if command == "help":
        print(HELP, file=out)
    elif command == "reset":
        session.reset()
        print("conversation cleared", file=out)
    elif command == "mode":
        mode = rest.strip()
        Settings(**{**asdict(session.settings), "mode": mode}).validate()
        session.settings.mode = mode
        session.reset()
        print(f"mode: {mode}", file=out)
    elif command == "set":
        name, _, value = rest.strip().partition(" ")
        apply_setting(session.settings, name, value.strip())
        print(f"{name} = {getattr(session.settings, name)!r}", file=out)
    elif command == "show":
        print(json.dumps(asdict(session.settings)), file=out)
    elif command == "history":
        for user, reply in session.history:
            print(f"you: {user}\nmodel: {reply}", file=out)
    elif command == "save":
        target = Path(rest.strip())
        target.write_text("".join(json.dumps({"user": u, "assistant": a}) + "\n" for u, a in session.history))
        print(f"saved {len(session.history)} turns to {target}", file=out)
    else:
        print(f"unknown command /{command}; /help lists them", file=out)
    return True


def repl(session: ChatSession, out=None, ask: Optional[Callable[[str], str]] = None,
         transcript: Optional[Callable[[dict], None]] = None, show_stats: bool = True) -> None:
    out = sys.stdout if out is None else out
    ask = input if ask is None else ask
    try:
        import readline  # noqa: F401  (line editing where available)
    except ImportError:
        pass
    print(f"QuantaWeave chat ({session.settings.mode} mode). /help for commands, /quit to leave.", file=out)
    while True:
        try:
            line = ask("you> ").rstrip("\n")
        except EOFError:
            print(file=out)
            return
        if not line.strip():
            continue
        if line.startswith("/"):
            command, _, rest = line[1:].partition(" ")
            try:
                if not _command(session, command, rest, out):
                    return
            except (ValueError, OSError) as error:
                print(f"error: {error}", file=out)
            continue
        out.write(line if session.settings.mode == "complete" else "model> ")
        out.flush()
        reply = session.send(line, on_text=lambda piece: (out.write(piece), out.flush()))
        print(file=out)
        if reply.unknown_characters:
            print("  note: not in this model's vocabulary and replaced by <unk>: "
                  + " ".join(map(repr, reply.unknown_characters)), file=out)
        if show_stats:
            print(f"  [{reply.tokens} tokens, {reply.tokens_per_second:.0f} tok/s, stopped: {reply.stop_reason}]",
                  file=out)
        if transcript is not None:
            transcript({**asdict(reply), "tokens_per_second": reply.tokens_per_second,
                        "settings": asdict(session.settings)})


class _NullStream:
    def write(self, text: str) -> int:
        return len(text)

    def flush(self) -> None:
        pass


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    m = p.add_argument_group("which model")
    m.add_argument("--checkpoint", type=Path, help=f"a checkpoint directory (default {DEFAULT_CHECKPOINT})")
    m.add_argument("--run", help="archived run to load, by its epoch-second name under --runs-dir or by path")
    m.add_argument("--latest", action="store_true", help="load the most recent archived run that holds a model")
    m.add_argument("--adapter", type=Path, help="QLoRA adapter folder, applied on top of --checkpoint")
    m.add_argument("--quantize", type=int, choices=(0, 4, 8), default=0, help="quantise the experts in memory")
    m.add_argument("--runs-dir", type=Path, default=RUNS_DIR)
    s = p.add_argument_group("sending messages")
    s.add_argument("-m", "--message", action="append", default=[], help="a message to send; give it several times for several messages")
    s.add_argument("--messages-file", type=Path, help=".txt (one per line) or .jsonl ({message, expect, ...})")
    s.add_argument("--conversation", action="store_true", help="batch mode keeps the history between messages")
    s.add_argument("--json", action="store_true", help="write each reply as a JSON line rather than plain text")
    s.add_argument("--transcript", type=Path, help="log each message and reply as a line in this JSONL file")
    s.add_argument("--interactive", action="store_true", help="always run the interactive session (even on a pipe)")
    s.add_argument("--quiet", action="store_true", help="print replies only, without timing lines or notes")
    g = p.add_argument_group("generation")
    g.add_argument("--mode", choices=("complete", "chat"), default="complete")
    g.add_argument("--system", default="", help="system text that opens the conversation (chat mode)")
    g.add_argument("--tokens", type=int, default=200, help="upper limit of generated tokens for each reply")
    g.add_argument("--temperature", type=float, default=0.8, help="sampling temperature; 0 always takes the most likely token")
    g.add_argument("--top-k", type=int, default=0)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--seed", type=int, help="seed for the sampler, for repeatable replies")
    g.add_argument("--stop", action="append", default=[], help="end the reply at this text; may be given several times")
    g.add_argument("--no-cache", action="store_true", help="plain forward pass per token instead of the KV cache")
    g.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    g.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    from .common import describe_options

    describe_options(p)
    return p


def main(argv: Optional[Sequence[str]] = None) -> int:
    from ..training.trainer import select_device
    from ..utils.hardware import choose_precision, detect

    parser = build_parser()
    args = parser.parse_args(argv)
    settings = Settings(mode=args.mode, tokens=args.tokens, temperature=args.temperature, top_k=args.top_k,
                        top_p=args.top_p, seed=args.seed, stop=list(args.stop), system=args.system)
    try:
        settings.validate()
        checkpoint, adapter = resolve_model(args.checkpoint, args.adapter, args.run, args.latest, args.runs_dir)
        items = [{"message": msg, "expect": []} for msg in args.message]
        if args.messages_file is not None:
            items += read_messages(args.messages_file)
        if args.interactive and items:
            parser.error("--interactive cannot be combined with --message/--messages-file")
        if not items and not args.interactive and not sys.stdin.isatty():
            items = [{"message": line.rstrip("\n"), "expect": []} for line in sys.stdin if line.strip()]
    except (ValueError, FileNotFoundError) as error:
        parser.error(str(error))
    device = select_device(args.device)
    model, tokenizer = load_for_chat(checkpoint, adapter, args.quantize, device)
    precision = choose_precision(detect(device.type), args.precision)
    session = ChatSession(model, tokenizer, device, precision, settings, use_cache=not args.no_cache)
    status = sys.stderr if not args.quiet else _NullStream()
    print(f"model: {checkpoint}" + (f" + adapter {adapter}" if adapter else "")
          + f"  device: {device}  precision: {precision}"
          + (f"  experts quantized to int{args.quantize}" if args.quantize and adapter is None else "")
          + f"  decoding: {session.cache_note}", file=status)
    log = None
    if args.transcript is not None:
        args.transcript.parent.mkdir(parents=True, exist_ok=True)
        log = args.transcript.open("a", encoding="utf-8")
    write = (lambda entry: (log.write(json.dumps(entry) + "\n"), log.flush())) if log else None
    try:
        if not items:
            repl(session, transcript=write, show_stats=not args.quiet)
            return 0

        def emit(result: dict) -> None:
            if write:
                write({**result, "settings": asdict(session.settings)})
            if args.json:
                print(json.dumps(result), flush=True)
                return
            print(f"> {result['message']}")
            print(result["response"])
            if args.quiet:
                return
            if result["unknown_characters"]:
                print(f"  note: replaced by <unk>: {' '.join(map(repr, result['unknown_characters']))}", file=status)
            verdict = "" if result["passed"] is None else (
                "  PASS" if result["passed"] else f"  FAIL (missing {result['missing']})")
            print(f"  [{result['tokens']} tokens, {result['tokens_per_second']:.0f} tok/s, "
                  f"stopped: {result['stop_reason']}]{verdict}", file=status)

        results = run_batch(session, items, args.conversation, emit)
    finally:
        if log:
            log.close()
    failed = [r for r in results if r["passed"] is False]
    checked = [r for r in results if r["passed"] is not None]
    if checked and not args.quiet:
        print(f"{len(checked) - len(failed)}/{len(checked)} checks passed", file=status)
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
