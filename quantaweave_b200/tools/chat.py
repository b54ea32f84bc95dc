"""Talk to a trained model: an interactive session, one-off messages, or a file of test messages.

    python -m quantaweave_b200.tools.chat --latest                      # interactive, newest archived run
    python -m quantaweave_b200.tools.chat --checkpoint DIR -m "Once upon a time"
    python -m quantaweave_b200.tools.chat --latest --messages-file tests.jsonl --json
    printf 'Once upon a time\\n' | python -m quantaweave_b200.tools.chat --latest

Same names, options and behaviour as the reference's ``src/chat_quantweave_moe.py`` (``choose_token``, ``Settings``,
``Reply``, ``ChatSession``, ``resolve_model``, ``read_messages``, ``run_batch``, ``repl`` and the command line, whose
exit code is 1 when an expectation fails).

How it works here:

* A reply is produced by a token source (the KV-cache ``FastDecoder`` stream, or one full forward pass per token
  with ``--no-cache``) feeding a ``_StopScanner``. The scanner owns the reply text: it cuts at the earliest stop
  string and releases streamed text only once no stop string can still begin inside it, so a caller never sees part
  of a stop string.
* ``complete`` mode continues the message; ``chat`` mode renders the conversation as ``User:`` / ``Assistant:``
  turns after an optional system line and stops at the next turn marker.
* Only ids the tokenizer can decode are ever sampled, and never ``<unk>``; temperature 0 is greedy. At most
  ``max_sequence_length - 1`` tokens of context are read (the last position of a training window is never trained).
"""

from __future__ import annotations

import argparse
import json
import re
import sys
import time
from dataclasses import asdict, dataclass, field, fields, replace
from pathlib import Path
from typing import Callable, Iterator, Optional, Sequence

import torch

RUNS_DIR = Path("artifacts/runs")
DEFAULT_CHECKPOINT = Path("artifacts/outputs/quantweave-moe-out")
CHAT_STOPS = ("\nUser:", "\nSystem:")  # the next turn marker ends an assistant reply


# ---- sampling ----------------------------------------------------------------------------------------------------
def choose_token(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                 generator: Optional[torch.Generator]) -> int:
    """Greedy at temperature 0, otherwise a draw from the top-k / nucleus-filtered softmax."""
    from ..inference.fast_decode import filter_logits

    if temperature <= 0:
        return int(torch.argmax(logits))
    weights = torch.softmax(filter_logits(logits / temperature, top_k, top_p), dim=-1)
    return int(torch.multinomial(weights, 1, generator=generator).item())


# ---- settings and replies ------------------------------------------------------------------------------------------
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
        problems = []
        if self.mode not in ("complete", "chat"):
            problems.append("mode must be complete or chat")
        if self.tokens < 1:
            problems.append("tokens must be at least 1")
        if self.temperature < 0:
            problems.append("temperature cannot be negative")
        if self.top_k < 0:
            problems.append("top_k cannot be negative")
        if not 0.0 < self.top_p <= 1.0:
            problems.append("top_p must lie in (0, 1]")
        if problems:
            raise ValueError("; ".join(problems))


@dataclass
class Reply:
    message: str
    prompt: str
    response: str
    tokens: int
    seconds: float
    stop_reason: str  # "eos", "stop" or "length"
    unknown_characters: list[str] = field(default_factory=list)
    truncated_context: bool = False

    @property
    def tokens_per_second(self) -> float:
        return self.tokens / self.seconds if self.seconds > 0 else 0.0


class _StopScanner:
    """Accumulates reply text, finds the first stop string, and decides how much text is safe to stream."""

    def __init__(self, stops: Sequence[str]) -> None:
        self.stops = [s for s in stops if s]
        self.reserve = max((len(s) for s in self.stops), default=1) - 1
        self.text = ""
        self.shown = 0
        self.stopped = False

    def extend(self, text: str) -> None:
        self.text = text
        cut = min((i for i in (text.find(s) for s in self.stops) if i >= 0), default=-1)
        if cut >= 0:
            self.text, self.stopped = text[:cut], True

    def release(self, final: bool = False) -> str:
        """Text not yet shown that can no longer turn into the start of a stop string (all of it when ``final``)."""
        limit = len(self.text) if (final or self.stopped) else max(self.shown, len(self.text) - self.reserve)
        piece, self.shown = self.text[self.shown:limit], max(self.shown, limit)
        return piece


# ---- the session -----------------------------------------------------------------------------------------------------
class ChatSession:
    def __init__(self, model, tokenizer, device: torch.device, precision: str, settings: Settings,
                 use_cache: bool = True) -> None:
        from ..inference.fast_decode import FastDecoder, Unsupported

        settings.validate()
        self.model, self.tokenizer, self.device, self.precision = model.eval(), tokenizer, device, precision
        self.settings = settings
        self.history: list[tuple[str, str]] = []
        self.valid_ids = tokenizer.vocab_size  # the model may score ids the tokenizer never produces
        self.decoder = None
        self.cache_note = "no cache (full forward pass per token)"
        if not use_cache:
            return
        try:
            self.decoder = FastDecoder(model, device, precision)
        except Unsupported as why:
            self.cache_note = f"no cache ({why})"
            return
        self.decoder.warm(settings.temperature, settings.top_k, settings.top_p)
        self.cache_note = self.decoder.description

    def reset(self) -> None:
        self.history = []

    def format_prompt(self, message: str) -> str:
        if self.settings.mode != "chat":
            return message
        turns = [f"User: {user}\nAssistant: {answer}\n" for user, answer in self.history]
        opening = [f"System: {self.settings.system}\n"] if self.settings.system else []
        return "".join(opening + turns) + f"User: {message}\nAssistant:"

    def unknown_characters(self, text: str) -> list[str]:
        vocab = getattr(self.tokenizer, "vocab", None) if self.tokenizer.kind == "char" else None
        return sorted(set(text) - set(vocab)) if vocab is not None else []

    def _context_limit(self) -> int:
        return self.decoder.capacity if self.decoder is not None else self.model.config.max_sequence_length - 1

    def _uncached(self, ids: list[int], generator) -> Iterator[int]:
        """One full forward pass over the newest ``_context_limit()`` tokens per generated token."""
        from ..training.trainer import autocast_context

        s, limit = self.settings, self._context_limit()
        banned = torch.zeros(0, dtype=torch.long)
        if self.tokenizer.unk_id is not None and self.tokenizer.unk_id < self.valid_ids:
            banned = torch.tensor([self.tokenizer.unk_id])
        context = list(ids)
        while True:
            window = torch.tensor([context[-limit:]], dtype=torch.long, device=self.device)
            with autocast_context(self.device, self.precision):
                scores = self.model(window)["logits"][0, -1].float()
            scores[self.valid_ids:] = float("-inf")
            scores[banned.to(scores.device)] = float("-inf")
            token = choose_token(scores, s.temperature, s.top_k, s.top_p, generator)
            context.append(token)
            yield token

    def _cached(self, ids: list[int], generator) -> Iterator[int]:
        s = self.settings
        return self.decoder.stream(ids, s.tokens, temperature=s.temperature, top_k=s.top_k, top_p=s.top_p,
                                   valid_ids=self.valid_ids, unk_id=self.tokenizer.unk_id, generator=generator)

    @torch.inference_mode()
    def send(self, message: str, on_text: Optional[Callable[[str], None]] = None) -> Reply:
        """Generate a reply to ``message``; ``on_text`` receives the reply piece by piece, never part of a stop."""
        s, tok = self.settings, self.tokenizer
        prompt = self.format_prompt(message)
        ids = tok.encode(prompt) or [tok.eos_id]
        stops = list(s.stop) + (list(CHAT_STOPS) if s.mode == "chat" else [])
        scanner = _StopScanner(stops)
        generator = None if s.seed is None else torch.Generator(device=self.device).manual_seed(s.seed)
        source = (self._cached if self.decoder is not None else self._uncached)(ids, generator)
        produced: list[int] = []
        reason = "length"
        character_level = tok.kind == "char"  # a character's text does not depend on its neighbours
        started = time.perf_counter()
        try:
            for token in source:
                if len(produced) >= s.tokens:
                    break
                if token == tok.eos_id:
                    reason = "eos"
                    break
                produced.append(token)
                text = scanner.text + tok.inverse.get(token, "?") if character_level else tok.decode(produced)
                scanner.extend(text)
                if scanner.stopped:
                    reason = "stop"
                    break
                if on_text is not None:
                    piece = scanner.release()
                    if piece:
                        on_text(piece)
        finally:
            source.close()
        if on_text is not None:
            rest = scanner.release(final=True)
            if rest:
                on_text(rest)
        elapsed = time.perf_counter() - started
        response = scanner.text.strip() if s.mode == "chat" else scanner.text
        if s.mode == "chat":
            self.history.append((message, response))
        return Reply(message=message, prompt=prompt, response=response, tokens=len(produced), seconds=elapsed,
                     stop_reason=reason, unknown_characters=self.unknown_characters(prompt),
                     truncated_context=len(ids) > self._context_limit())


# ---- choosing a model -----------------------------------------------------------------------------------------------
_RUN_NAME = re.compile(r"(\d+)(?:-(\d+))?")


def run_folders(root: Path = RUNS_DIR) -> list[Path]:
    """Archived runs, oldest first: folders named ``<epoch seconds>`` or ``<epoch seconds>-<n>``."""
    root = Path(root)
    if not root.is_dir():
        return []
    runs = []
    for entry in root.iterdir():
        match = _RUN_NAME.fullmatch(entry.name)
        if match and entry.is_dir():
            runs.append((int(match[1]), int(match[2] or 0), entry))
    return [path for *_, path in sorted(runs)]


def usable_model(run: Path) -> Optional[tuple[Path, Optional[Path]]]:
    """(checkpoint, adapter) held by an archived run: its trained or merged model, else its adapter over the base the
    adapter names; None when the run holds none of them."""
    run = Path(run)
    for folder in (run / "model", run / "merged"):
        if (folder / "model.pt").exists():
            return folder, None
    adapter = run / "adapter"
    if (adapter / "adapter.pt").exists():
        base = json.loads((adapter / "finetune_metadata.json").read_text())["base_checkpoint"]
        return Path(base), adapter
    return None


def resolve_model(checkpoint: Optional[Path], adapter: Optional[Path], run: Optional[str], latest: bool,
                  root: Path = RUNS_DIR) -> tuple[Path, Optional[Path]]:
    """An explicit checkpoint wins; then a named run (epoch name under ``root`` or a path); then the newest run that
    holds a model; otherwise the default output folder."""
    if checkpoint is not None:
        return Path(checkpoint), adapter
    if run is not None:
        folder = Path(run) if Path(run).is_dir() else Path(root) / run
        found = usable_model(folder) if folder.is_dir() else None
        if found is None:
            raise FileNotFoundError(f"no model found in run '{run}' (looked in {folder})")
        return found
    if latest:
        found = next(filter(None, map(usable_model, reversed(run_folders(root)))), None)
        if found is None:
            raise FileNotFoundError(f"no archived run with a model under {root}")
        return found
    return DEFAULT_CHECKPOINT, adapter


def load_for_chat(checkpoint: Path, adapter: Optional[Path], quantize: int, device: torch.device):
    """(model, tokenizer): the adapter applied over its base, or the checkpoint, with experts quantised in memory when
    ``quantize`` is 4 or 8."""
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


# ---- batches of test messages ----------------------------------------------------------------------------------------
_OVERRIDABLE = ("mode", "tokens", "temperature", "top_k", "top_p", "seed")


def read_messages(path: Path) -> list[dict]:
    """Messages to send. A ``.jsonl`` file holds one object per line with ``message`` (or ``prompt``), optional
    ``expect`` (a string or a list of strings that must appear in the reply) and per-message settings; any other
    file holds one message per line. Blank lines and lines starting with ``#`` are skipped."""
    path = Path(path)
    structured = path.suffix == ".jsonl"
    items = []
    for number, raw in enumerate(path.read_text(encoding="utf-8").splitlines(), start=1):
        if not raw.strip() or raw.lstrip().startswith("#"):
            continue
        if not structured:
            items.append({"message": raw, "expect": []})
            continue
        try:
            item = json.loads(raw)
        except json.JSONDecodeError as error:
            raise ValueError(f"{path}:{number}: not valid JSON ({error})") from error
        text = item["message"] if "message" in item else item.get("prompt")
        if text is None:
            raise ValueError(f"{path}:{number}: needs a 'message' field")
        wanted = item.get("expect") or []
        items.append({**item, "message": text, "expect": [wanted] if isinstance(wanted, str) else list(wanted)})
    return items


def run_batch(session: ChatSession, items: Sequence[dict], conversation: bool,
              emit: Callable[[dict], None]) -> list[dict]:
    """Send every message; a message's own settings apply to it alone. Each result records whether every expected
    string appeared (``passed`` is None when nothing was expected)."""
    base = session.settings
    results = []
    for item in items:
        if not conversation:
            session.reset()
        session.settings = replace(base, **{k: item[k] for k in _OVERRIDABLE if k in item})
        try:
            reply = session.send(item["message"])
        finally:
            session.settings = base
        missing = [needle for needle in item["expect"] if needle not in reply.response]
        result = dict(asdict(reply), tokens_per_second=reply.tokens_per_second, expect=item["expect"],
                      passed=(not missing) if item["expect"] else None, missing=missing)
        emit(result)
        results.append(result)
    return results


# ---- interactive session ---------------------------------------------------------------------------------------------
HELP = """commands:
  /help                  show this list
  /reset                 start the conversation over (chat mode)
  /mode complete|chat    change mode (and start over)
  /set NAME VALUE        temperature, top_k, top_p, tokens, seed (a number or "none") or system (text)
  /show                  print the current settings
  /history               print the conversation so far
  /save FILE             write the conversation to FILE as JSON lines
  /quit                  leave (Ctrl-D works too)
any other line is sent to the model."""

_SETTING_TYPES = {"temperature": float, "top_p": float, "top_k": int, "tokens": int,
                  "seed": lambda v: None if v.lower() == "none" else int(v), "system": str}


def apply_setting(settings: Settings, name: str, value: str) -> None:
    """Change one setting in place; a value that does not parse or validate leaves every setting as it was."""
    if name not in _SETTING_TYPES:
        raise ValueError(f"unknown setting '{name}' (try: {', '.join(_SETTING_TYPES)})")
    candidate = replace(settings, **{name: _SETTING_TYPES[name](value)})
    candidate.validate()
    setattr(settings, name, getattr(candidate, name))


def _cmd_help(session, rest, out):
    print(HELP, file=out)


def _cmd_reset(session, rest, out):
    session.reset()
    print("conversation cleared", file=out)


def _cmd_mode(session, rest, out):
    mode = rest.strip()
    replace(session.settings, mode=mode).validate()
    session.settings.mode = mode
    session.reset()
    print(f"mode: {mode}", file=out)


def _cmd_set(session, rest, out):
    name, _, value = rest.strip().partition(" ")
    apply_setting(session.settings, name, value.strip())
    print(f"{name} = {getattr(session.settings, name)!r}", file=out)


def _cmd_show(session, rest, out):
    print(json.dumps(asdict(session.settings)), file=out)


def _cmd_history(session, rest, out):
    for user, answer in session.history:
        print(f"you: {user}\nmodel: {answer}", file=out)


def _cmd_save(session, rest, out):
    target = Path(rest.strip())
    target.write_text("".join(json.dumps({"user": u, "assistant": a}) + "\n" for u, a in session.history))
    print(f"saved {len(session.history)} turns to {target}", file=out)


_COMMANDS = {"help": _cmd_help, "reset": _cmd_reset, "mode": _cmd_mode, "set": _cmd_set, "show": _cmd_show,
             "history": _cmd_history, "save": _cmd_save}


def repl(session: ChatSession, out=None, ask: Optional[Callable[[str], str]] = None,
         transcript: Optional[Callable[[dict], None]] = None, show_stats: bool = True) -> None:
    """Read lines until ``/quit`` or end of input; ``/commands`` change the session, other lines are sent."""
    out = sys.stdout if out is None else out
    ask = input if ask is None else ask
    try:
        import readline  # noqa: F401  (line editing where the platform has it)
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
            name, _, rest = line[1:].partition(" ")
            if name in ("quit", "exit"):
                return
            handler = _COMMANDS.get(name)
            if handler is None:
                print(f"unknown command /{name}; /help lists them", file=out)
                continue
            try:
                handler(session, rest, out)
            except (ValueError, OSError) as error:
                print(f"error: {error}", file=out)
            continue
        out.write(line if session.settings.mode == "complete" else "model> ")
        out.flush()
        reply = session.send(line, on_text=lambda piece: (out.write(piece), out.flush()))
        print(file=out)
        if reply.unknown_characters:
            print("  note: not in this model's vocabulary and replaced by <unk>: "
                  + " ".join(repr(c) for c in reply.unknown_characters), file=out)
        if show_stats:
            print(f"  [{reply.tokens} tokens, {reply.tokens_per_second:.0f} tok/s, stopped: {reply.stop_reason}]",
                  file=out)
        if transcript is not None:
            transcript(dict(asdict(reply), tokens_per_second=reply.tokens_per_second,
                            settings=asdict(session.settings)))


# ---- command line ----------------------------------------------------------------------------------------------------
def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    which = p.add_argument_group("which model")
    which.add_argument("--checkpoint", type=Path, help=f"checkpoint directory to load (default {DEFAULT_CHECKPOINT})")
    which.add_argument("--run", help="archived run to load, by its epoch-second name under --runs-dir or by path")
    which.add_argument("--latest", action="store_true", help="load the most recent archived run that holds a model")
    which.add_argument("--adapter", type=Path, help="QLoRA adapter folder, applied on top of --checkpoint")
    which.add_argument("--quantize", type=int, choices=(0, 4, 8), default=0,
                       help="quantise the experts to int4 or int8 after loading (0: keep them as saved)")
    which.add_argument("--runs-dir", type=Path, default=RUNS_DIR)
    send = p.add_argument_group("what to send")
    send.add_argument("-m", "--message", action="append", default=[],
                      help="a message to send; give it several times for several messages")
    send.add_argument("--messages-file", type=Path,
                      help="messages to send: one per line, or JSON lines with message, expect and settings")
    send.add_argument("--conversation", action="store_true", help="keep the history between the messages of a batch")
    send.add_argument("--json", action="store_true", help="write each reply as a JSON line rather than plain text")
    send.add_argument("--transcript", type=Path, help="log each message and reply as a line in this JSONL file")
    send.add_argument("--interactive", action="store_true",
                      help="start the interactive session even when standard input is not a terminal")
    send.add_argument("--quiet", action="store_true", help="print replies only, without timing lines or notes")
    gen = p.add_argument_group("generation")
    gen.add_argument("--mode", choices=("complete", "chat"), default="complete")
    gen.add_argument("--system", default="", help="system text that opens the conversation (chat mode)")
    gen.add_argument("--tokens", type=int, default=200, help="upper limit of generated tokens for each reply")
    gen.add_argument("--temperature", type=float, default=0.8,
                     help="sampling temperature; 0 always takes the most likely token")
    gen.add_argument("--top-k", type=int, default=0)
    gen.add_argument("--top-p", type=float, default=1.0)
    gen.add_argument("--seed", type=int, help="seed for the sampler, for repeatable replies")
    gen.add_argument("--stop", action="append", default=[], help="end the reply at this text; may be given several times")
    gen.add_argument("--no-cache", action="store_true",
                     help="run a full forward pass per token instead of decoding with the KV cache")
    gen.add_argument("--precision", choices=("auto", "bf16", "fp16", "fp32"), default="auto")
    gen.add_argument("--device", choices=("auto", "cuda", "rocm", "xpu", "cpu"), default="auto")
    from .common import describe_options

    describe_options(p)
    return p


class _NullStream:
    def write(self, text: str) -> int:
        return len(text)

    def flush(self) -> None:
        pass


def _batch_printer(args, status, session, write):
    def emit(result: dict) -> None:
        if write is not None:
            write(dict(result, settings=asdict(session.settings)))
        if args.json:
            print(json.dumps(result), flush=True)
            return
        print(f"> {result['message']}\n{result['response']}")
        if args.quiet:
            return
        if result["unknown_characters"]:
            print("  note: replaced by <unk>: " + " ".join(map(repr, result["unknown_characters"])), file=status)
        if result["passed"] is None:
            verdict = ""
        else:
            verdict = "  PASS" if result["passed"] else f"  FAIL (missing {result['missing']})"
        print(f"  [{result['tokens']} tokens, {result['tokens_per_second']:.0f} tok/s, "
              f"stopped: {result['stop_reason']}]{verdict}", file=status)

    return emit


def main(argv: Optional[Sequence[str]] = None) -> int:
    from ..training.trainer import select_device
    from ..utils.hardware import choose_precision, detect

    parser = build_parser()
    args = parser.parse_args(argv)
    chosen = {f.name: getattr(args, f.name) for f in fields(Settings) if f.name != "stop"}
    settings = Settings(**chosen, stop=list(args.stop))
    try:
        settings.validate()
        checkpoint, adapter = resolve_model(args.checkpoint, args.adapter, args.run, args.latest, args.runs_dir)
        items = [{"message": text, "expect": []} for text in args.message]
        if args.messages_file is not None:
            items.extend(read_messages(args.messages_file))
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
    status = _NullStream() if args.quiet else sys.stderr
    described = f"model: {checkpoint}" + (f" + adapter {adapter}" if adapter else "")
    described += f"  device: {device}  precision: {precision}"
    if args.quantize and adapter is None:
        described += f"  experts quantized to int{args.quantize}"
    print(described + f"  decoding: {session.cache_note}", file=status)
    log = None
    if args.transcript is not None:
        args.transcript.parent.mkdir(parents=True, exist_ok=True)
        log = args.transcript.open("a", encoding="utf-8")

    def write(entry: dict) -> None:
        log.write(json.dumps(entry) + "\n")
        log.flush()

    try:
        if not items:
            repl(session, transcript=write if log else None, show_stats=not args.quiet)
            return 0
        results = run_batch(session, items, args.conversation,
                            _batch_printer(args, status, session, write if log else None))
    finally:
        if log is not None:
            log.close()
    checked = [r for r in results if r["passed"] is not None]
    failures = sum(1 for r in checked if not r["passed"])
    if checked and not args.quiet:
        print(f"{len(checked) - failures}/{len(checked)} checks passed", file=status)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
