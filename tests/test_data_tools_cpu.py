"""Token preparation CLI and corpus helpers (reference test: tests/test_prepare_tokens.py)."""

import json

from quantaweave_b200.data.pipeline import load_token_bin
from quantaweave_b200.tools.corpus import group_texts, language_budgets, write_rows
from quantaweave_b200.tools.prepare_tokens import main as prepare


def test_pack_char_and_bpe(tmp_path):
    from test_tools_cpu import _corpus

    data = _corpus(tmp_path / "d.jsonl", 50)
    meta = prepare(["pack", "--data", str(data), "--tokenizer", "char", "--vocab-size", "64",
                    "--output", str(tmp_path / "chars")])
    assert meta["total_tokens"] > 500 and {s["domain"] for s in meta["segments"]} == {"story", "code"}
    corpus, tok = load_token_bin(tmp_path / "chars")
    assert tok.kind == "char"
    prepare(["bpe", "--data", str(data), "--vocab-size", "300", "--output", str(tmp_path / "bpe")])
    meta = prepare(["pack", "--data", str(data), "--tokenizer", str(tmp_path / "bpe"),
                    "--output", str(tmp_path / "bpetok")])
    assert meta["tokenizer"] == "bpe" and meta["total_tokens"] > 0


def test_group_texts_and_budgets(tmp_path):
    chunks = list(group_texts([[1, 2, 3], [4, 5], [6]], 3, 0))
    assert chunks == [[1, 2, 3], [0, 4, 5], [0, 6, 0]]
    budgets = language_budgets(1000, 0.8)
    assert budgets["docs_nl"] == 200 and budgets["python"] == 320 and sum(budgets.values()) <= 1000
    rows = [{"content": "x" * 40}, {"content": "y" * 80}, {"content": "z" * 200}, {"content": "w" * 80}]
    tokens, written = write_rows(rows, tmp_path / "o.jsonl", "content", "code_py", 40, min_chars=50, max_chars=150)
    lines = [json.loads(x) for x in (tmp_path / "o.jsonl").read_text().splitlines()]
    assert written == 2 and tokens == 40 and lines[0] == {"text": "y" * 80, "domain": "code_py"}
