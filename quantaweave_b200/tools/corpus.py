"""Corpus builders: a TinyStories smoke sample, a language-weighted code + docs pre-training corpus, and fixed-length
packing of token streams.

Parity with the reference dataset builders (``src/prepare_smoke_dataset.py``, ``src/build_code_corpus.py`` with its
language weights and 50..100k character row filter, ``src/data.py`` budget-driven streaming, ``src/pack_dataset.py``
``group_texts``). They stream from the Hugging Face hub through the ``datasets`` package, so they need network
access; every output is plain ``{"text", "domain"}`` JSONL that ``prepare_tokens pack`` and the trainer read.
Packing writes the framework's ``tokens.bin`` corpus (``prepare_tokens``) rather than an Arrow dataset for an
external trainer.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Iterable, Iterator, Optional

CHARS_PER_TOKEN_ESTIMATE = 4.0
CODE_LANGUAGE_WEIGHTS = {"python": 0.40, "javascript": 0.15, "java": 0.15, "cpp": 0.10, "go": 0.10, "rust": 0.05,
                         "shell": 0.05}
MIN_CHARS, MAX_CHARS = 50, 100_000


def _hub(*args, **kwargs):
    try:
        from datasets import load_dataset
    except ImportError as error:  # pragma: no cover
        raise RuntimeError("corpus builders need the `datasets` package and network access") from error
    return load_dataset(*args, **kwargs)


def write_rows(rows: Iterable[dict], output: Path, text_key: str, domain: Optional[str], token_budget: int,
               min_chars: int = 1, max_chars: Optional[int] = None, token_count_key: Optional[str] = None,
               append: bool = False) -> tuple[int, int]:
    """Write ``{"text", "domain"}`` rows until ``token_budget`` (estimated at 4 chars/token unless the row carries an
    exact count). Returns (tokens, rows)."""
    tokens = written = 0
    with Path(output).open("a" if append else "w", encoding="utf-8") as out:
        for row in rows:
            if tokens >= token_budget:
                break
            text = (row.get(text_key) or "").strip() if text_key == "text" else row.get(text_key) or ""
            if len(text) < min_chars or (max_chars is not None and len(text) > max_chars):
                continue
            out.write(json.dumps({"text": text, **({"domain": domain} if domain else {})}, ensure_ascii=False) + "\n")
            exact = row.get(token_count_key) if token_count_key else None
            tokens += int(exact or len(text) / CHARS_PER_TOKEN_ESTIMATE)
            written += 1
    return tokens, written


def smoke_sample(examples: int, output: Path) -> int:
    output.parent.mkdir(parents=True, exist_ok=True)
    _, written = _limited(_hub("roneneldan/TinyStories", split="train", streaming=True), examples, output)
    return written


def _limited(rows, examples: int, output: Path) -> tuple[int, int]:
    def take() -> Iterator[dict]:
        n = 0
        for row in rows:
            if (row.get("text") or "").strip():
                yield row
                n += 1
                if n >= examples:
                    return
    return write_rows(take(), output, "text", None, token_budget=1 << 62)


def language_budgets(total_tokens: int, code_fraction: float) -> dict[str, int]:
    """Token budget per code language (by ``CODE_LANGUAGE_WEIGHTS``) plus ``docs_nl`` for the rest."""
    code = int(total_tokens * code_fraction)
    budgets = {lang: int(code * w) for lang, w in CODE_LANGUAGE_WEIGHTS.items()}
    budgets["docs_nl"] = total_tokens - code
    return budgets


def code_corpus(total_tokens: int, code_fraction: float, output: Path) -> dict:
    output.parent.mkdir(parents=True, exist_ok=True)
    output.write_text("")
    report = {}
    for lang, budget in language_budgets(total_tokens, code_fraction).items():
        if lang == "docs_nl":
            rows = _hub("HuggingFaceFW/fineweb-edu", "sample-100BT", split="train", streaming=True)
            report[lang] = write_rows(rows, output, "text", "docs_nl", budget, MIN_CHARS, None, "token_count", True)
        else:
            rows = _hub("bigcode/starcoderdata", data_dir=lang, split="train", streaming=True)
            report[lang] = write_rows(rows, output, "content", f"code_{lang}", budget, MIN_CHARS, MAX_CHARS,
                                      None, True)
    return {k: {"tokens": t, "rows": r} for k, (t, r) in report.items()}


def group_texts(token_lists: Iterable[list[int]], sequence_length: int, eos_id: int) -> Iterator[list[int]]:
    """Concatenate documents (each followed by ``eos_id``) and cut whole ``sequence_length`` chunks; the tail that
    does not fill a chunk is dropped."""
    buffer: list[int] = []
    for ids in token_lists:
        buffer.extend(ids)
        buffer.append(eos_id)
        while len(buffer) >= sequence_length:
            yield buffer[:sequence_length]
            buffer = buffer[sequence_length:]


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="command", required=True)
    s = sub.add_parser("smoke", help="a bounded TinyStories sample")
    s.add_argument("--examples", type=int, default=100_000)
    s.add_argument("--output", type=Path, default=Path("data/smoke/tinystories.jsonl"))
    c = sub.add_parser("code", help="language-weighted code + docs corpus")
    c.add_argument("--total-tokens", type=int, default=2_500_000_000)
    c.add_argument("--code-fraction", type=float, default=0.85)
    c.add_argument("--output", type=Path, default=Path("data/raw/quantweave-code-corpus.jsonl"))
    from .common import describe_options

    describe_options(p, {'total_tokens': 'approximate token budget of the corpus', 'code_fraction': 'share of code among the tokens', 'output': 'JSONL file to write'})
    args = p.parse_args(argv)
    if args.command == "smoke":
        if args.examples < 1:
            p.error("--examples must be greater than zero")
        print(f"wrote {smoke_sample(args.examples, args.output)} examples to {args.output}")
    else:
        print(json.dumps(code_corpus(args.total_tokens, args.code_fraction, args.output), indent=2))


if __name__ == "__main__":
    main()
