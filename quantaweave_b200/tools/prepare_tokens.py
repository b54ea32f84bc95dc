"""Train a tokenizer and/or pack JSONL text into a memory-mapped token corpus (``tokens.bin`` + ``meta.json``).

    python -m quantaweave_b200.tools.prepare_tokens bpe --data a.jsonl --vocab-size 4096 --output tok/bpe4k
    python -m quantaweave_b200.tools.prepare_tokens sentencepiece --data a.jsonl --vocab-size 4096 --output tok/sp4k
    python -m quantaweave_b200.tools.prepare_tokens pack --data a.jsonl b.jsonl --tokenizer tok/bpe4k --output data/t
    python -m quantaweave_b200.tools.prepare_tokens pack --data a.jsonl --tokenizer char --vocab-size 7168 --output d

Parity with the reference ``src/prepare_tokens.py`` (subcommands bpe / sentencepiece / pack, ``--redact-pii``). Rows
may carry a ``domain`` field; otherwise the domain is ``default`` (one file) or the file stem. The packed corpus is
what ``--token-data`` of the trainer reads (memory-mapped, so a corpus far larger than host RAM streams from disk).
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="command", required=True)
    for name, text in (("bpe", "train a byte-level BPE tokenizer"),
                       ("sentencepiece", "train a sentencepiece (unigram or BPE) tokenizer"),
                       ("pack", "tokenize JSONL into tokens.bin + meta.json")):
        c = sub.add_parser(name, help=text)
        c.add_argument("--data", type=Path, nargs="+", required=True)
        c.add_argument("--examples", type=int, help="read at most this many rows from each JSONL file")
        c.add_argument("--output", type=Path, required=True)
        c.add_argument("--redact-pii", action="store_true", help="best-effort PII redaction first")
        if name == "pack":
            c.add_argument("--tokenizer", default="char", help="'char' or a directory saved by bpe/sentencepiece")
            c.add_argument("--vocab-size", type=int, default=7168, help="vocabulary size of the character tokenizer")
        else:
            c.add_argument("--vocab-size", type=int, default=4096)
        if name == "sentencepiece":
            c.add_argument("--algorithm", choices=("unigram", "bpe"), default="unigram")
    from .common import describe_options

    describe_options(p, {"data": "JSONL files to read", "output": "directory to write", "algorithm": "SentencePiece model type"})
    return p


def main(argv=None) -> dict:
    from ..data.pipeline import (BPETokenizer, CharTokenizer, SentencePieceTokenizer, load_tokenizer, read_rows,
                                 write_token_bin)

    args = build_parser().parse_args(argv)
    redactor = None
    if args.redact_pii:
        from ..utils.pii_redact import PIIRedactor

        redactor = PIIRedactor()

    def texts():
        return (text for _, text in read_rows(args.data, args.examples, redactor))

    def report_redaction() -> None:
        if redactor is not None and redactor.total():
            print(f"PII redaction: {redactor.report()}")

    if args.command in {"bpe", "sentencepiece"}:
        if args.command == "bpe":
            tok = BPETokenizer.train(texts(), args.vocab_size)
        else:
            tok = SentencePieceTokenizer.train(texts(), args.vocab_size, args.algorithm)
        tok.save(args.output)
        print(f"trained {args.command} tokenizer with {tok.vocab_size} tokens -> {args.output}")
        report_redaction()
        return {"tokenizer": args.command, "vocab_size": tok.vocab_size}
    tok = CharTokenizer.build(texts(), args.vocab_size) if args.tokenizer == "char" else load_tokenizer(
        Path(args.tokenizer))
    meta = write_token_bin(args.data, tok, args.output, args.examples, redactor)
    print(json.dumps({k: meta[k] for k in ("tokenizer", "vocab_size", "dtype", "total_tokens")}))
    for seg in meta["segments"]:
        print(f"  domain {seg['domain']}: {seg['length']:,} tokens")
    report_redaction()
    return meta


if __name__ == "__main__":
    main()
