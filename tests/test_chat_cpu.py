"""The chat tool's generation loop and command line on CPU (reference tests: tests/test_chat.py). A scripted model
emits a chosen token per forward pass, so sampling filters, stop strings, streaming hold-back, context windowing,
vocabulary masking, chat turns, run selection and the CLI's input modes are checked exactly."""

import io
import json
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from quantaweave_b200.data.pipeline import CharTokenizer
from quantaweave_b200.tools import chat
from quantaweave_b200.inference.fast_decode import filter_logits

CPU = torch.device("cpu")
TOK = CharTokenizer.build(["abcdefghijklmnopqrstuvwxyz \nUser:EN!."], 64)
MODEL_VOCAB = 96  # the model scores more ids than the tokenizer has


def ids(text):
    return TOK.encode(text)


class Scripted(torch.nn.Module):
    """Puts a large logit on the next scripted id at the last position and records every window length."""

    def __init__(self, script, context=32, invalid_first=False):
        super().__init__()
        self.script, self.calls, self.windows, self.invalid_first = list(script), 0, [], invalid_first
        self.config = SimpleNamespace(max_sequence_length=context)
        self.anchor = torch.nn.Parameter(torch.zeros(1))

    def forward(self, window):
        self.windows.append(window.size(1))
        logits = torch.zeros(1, window.size(1), MODEL_VOCAB)
        logits[0, -1, self.script[min(self.calls, len(self.script) - 1)]] = 50.0
        if self.invalid_first:
            logits[0, -1, MODEL_VOCAB - 1] = 60.0  # an id the tokenizer does not have, ranked first
        self.calls += 1
        return {"logits": logits}


def session(script, context=32, invalid=False, **settings):
    values = {"temperature": 0.0, "tokens": 20, **settings}
    return chat.ChatSession(Scripted(script, context, invalid), TOK, CPU, "fp32", chat.Settings(**values))


def test_top_k_and_top_p_keep_the_right_tokens_in_any_order():
    logits = torch.log(torch.tensor([0.5, 0.3, 0.15, 0.05]))
    kept = lambda **kw: torch.isfinite(filter_logits(logits, **kw)).tolist()  # noqa: E731
    assert kept(top_k=2) == [True, True, False, False]
    assert kept(top_p=0.7) == [True, True, False, False]  # the token that crosses 0.7 stays
    assert kept(top_p=0.4) == [True, False, False, False]
    assert kept(top_k=3, top_p=0.7) == [True, True, False, False] and all(kept(top_p=1.0))
    assert torch.equal(filter_logits(logits, top_k=10), logits)
    shuffled = torch.log(torch.tensor([0.05, 0.5, 0.15, 0.3]))
    assert torch.isfinite(filter_logits(shuffled, top_p=0.7)).tolist() == [False, True, False, True]


def test_greedy_is_argmax_and_sampling_is_seeded_and_follows_the_distribution():
    logits = torch.log(torch.tensor([0.1, 0.6, 0.3]))
    assert chat.choose_token(logits, 0.0, 0, 1.0, None) == 1 and chat.choose_token(logits, 1.0, 1, 1.0, None) == 1

    def draws(seed):
        return [chat.choose_token(logits, 1.0, 0, 1.0, torch.Generator().manual_seed(seed + i)) for i in range(400)]

    assert draws(0) == draws(0) and draws(0) != draws(1000)
    assert 0.5 < sum(d == 1 for d in draws(0)) / 400 < 0.7
    assert {chat.choose_token(logits, 0.05, 0, 1.0, torch.Generator().manual_seed(i)) for i in range(50)} == {1}


def test_eos_length_and_token_accounting():
    reply = session([*ids("ab"), TOK.eos_id]).send("hello")
    assert (reply.response, reply.stop_reason, reply.tokens) == ("ab", "eos", 2)
    reply = session(ids("a") * 5, tokens=3).send("hello")
    assert (reply.response, reply.stop_reason, reply.tokens) == ("aaa", "length", 3) and reply.tokens_per_second > 0


def test_ids_outside_the_tokenizer_and_unk_are_never_sampled():
    assert session(ids("b") * 6, tokens=6, invalid=True).send("hi").response == "bbbbbb"
    assert "<unk>" not in session([TOK.unk_id] * 3 + ids("c") * 3, tokens=3).send("hi").response


def test_stop_strings_cut_the_reply_and_streaming_never_shows_part_of_one():
    s = session(ids("hi\nUser: x"), mode="chat", tokens=12)
    pieces = []
    reply = s.send("q", on_text=pieces.append)
    assert (reply.response, reply.stop_reason) == ("hi", "stop") and "".join(pieces).strip() == "hi"
    shown = ""
    for piece in pieces:
        shown += piece
        assert "\n" not in shown  # the start of "\nUser:" is held back until it is known not to be a stop
    pieces = []
    reply = session(ids("xEN!abc"), stop=["EN!!"], tokens=7).send("q", on_text=pieces.append)
    assert reply.response == "".join(pieces) == "xEN!abc" and reply.stop_reason == "length"
    stopped = session(ids("xxEN!!z"), stop=["EN!!"], tokens=7).send("q")
    assert (stopped.response, stopped.stop_reason) == ("xx", "stop")


def test_long_prompts_are_windowed_one_short_of_the_context_and_empty_prompts_work():
    s = session(ids("ab"), context=8, tokens=2)
    reply = s.send("a" * 40)
    assert reply.truncated_context and max(s.model.windows) <= 7 and reply.response == "ab"
    assert session(ids("ab"), tokens=2).send("").response == "ab"


def test_unknown_characters_are_reported_for_character_models():
    s = session(ids("a"))
    assert s.send("héllo ☕").unknown_characters == ["é", "☕"] and s.unknown_characters("plain text") == []


def test_chat_turns_history_reset_and_stateless_completion():
    s = session(ids("ok"), mode="chat", system="Be brief.", tokens=2)
    assert s.format_prompt("hi") == "System: Be brief.\nUser: hi\nAssistant:"
    s.send("first")
    assert s.history == [("first", "ok")]
    assert s.format_prompt("second") == "System: Be brief.\nUser: first\nAssistant: ok\nUser: second\nAssistant:"
    s.reset()
    assert s.history == []
    plain = session(ids("ok"), tokens=2)
    assert plain.format_prompt("raw") == "raw"
    plain.send("x")
    assert plain.history == []


def test_settings_validation():
    for bad in (dict(mode="shout"), dict(tokens=0), dict(temperature=-1), dict(top_p=0.0), dict(top_p=1.5),
                dict(top_k=-1)):
        with pytest.raises(ValueError):
            chat.Settings(**bad).validate()
    chat.Settings(temperature=0.0, top_p=1.0).validate()


def _run(root: Path, name: str, kind: str = "model") -> Path:
    folder = root / name / kind
    folder.mkdir(parents=True)
    if kind == "adapter":
        (folder / "adapter.pt").write_bytes(b"x")
        (folder / "finetune_metadata.json").write_text(json.dumps({"base_checkpoint": "/base"}))
    else:
        (folder / "model.pt").write_bytes(b"x")
    return root / name


def test_runs_sort_by_epoch_numerically_and_latest_skips_runs_without_a_model(tmp_path):
    _run(tmp_path, "900")
    _run(tmp_path, "1000")
    _run(tmp_path, "1000-2", "merged")
    _run(tmp_path, "1000-10", "adapter")
    (tmp_path / "1001").mkdir()  # no model in it
    (tmp_path / "notes").mkdir()
    assert [p.name for p in chat.run_folders(tmp_path)] == ["900", "1000", "1000-2", "1000-10", "1001"]
    assert chat.resolve_model(None, None, None, True, tmp_path) == (Path("/base"), tmp_path / "1000-10" / "adapter")
    assert chat.resolve_model(None, None, "1000-2", False, tmp_path) == (tmp_path / "1000-2" / "merged", None)
    with pytest.raises(FileNotFoundError):
        chat.resolve_model(None, None, "1001", False, tmp_path)
    with pytest.raises(FileNotFoundError):
        chat.resolve_model(None, None, None, True, tmp_path / "empty")


def test_message_files_text_and_jsonl(tmp_path):
    txt = tmp_path / "m.txt"
    txt.write_text("first\n\n# a comment\nsecond\n")
    assert [i["message"] for i in chat.read_messages(txt)] == ["first", "second"]
    jl = tmp_path / "m.jsonl"
    jl.write_text('{"prompt": "a", "expect": "x"}\n{"message": "b", "expect": ["y", "z"], "tokens": 3}\n')
    items = chat.read_messages(jl)
    assert [i["expect"] for i in items] == [["x"], ["y", "z"]] and items[1]["tokens"] == 3
    for bad in ('{"text": "no message"}\n', "not json\n"):
        jl.write_text(bad)
        with pytest.raises(ValueError):
            chat.read_messages(jl)


def test_batch_overrides_apply_to_one_message_and_expectations_are_checked():
    s = session(ids("abcdef"), tokens=4)
    emitted = []
    results = chat.run_batch(s, [{"message": "x", "expect": ["ab"], "tokens": 2},
                                 {"message": "y", "expect": ["zz"]}, {"message": "z", "expect": []}],
                             False, emitted.append)
    assert results[0]["tokens"] == 2 and results[0]["passed"] is True
    assert results[1]["passed"] is False and results[1]["missing"] == ["zz"] and results[2]["passed"] is None
    assert s.settings.tokens == 4 and len(emitted) == 3  # the override did not outlive its message


def test_interactive_commands_and_unknown_character_notes(tmp_path):
    s = session(ids("ok"), tokens=2)
    lines = iter(["/set temperature 0.5", "/set top_p 7", "/mode chat", "/show", "hi", "/history",
                  f"/save {tmp_path / 't.jsonl'}", "/reset", "/help", "/nope", "héllo", "/quit"])
    out = io.StringIO()
    chat.repl(s, out=out, ask=lambda prompt: next(lines))
    text = out.getvalue()
    assert "temperature = 0.5" in text and "error:" in text and "mode: chat" in text and "you: hi" in text
    assert "conversation cleared" in text and "/reset" in text and "unknown command /nope" in text
    assert "not in this model's vocabulary" in text and "'é'" in text
    assert json.loads((tmp_path / "t.jsonl").read_text().splitlines()[0]) == {"user": "hi", "assistant": "ok"}


# ---- the command line, against a small trained checkpoint ------------------------------------------------------
@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from test_tools_cpu import _train

    tmp = tmp_path_factory.mktemp("chatcli")
    _train(tmp, steps=3)
    return tmp / "out"


def _cli(checkpoint, *extra):
    return ["--checkpoint", str(checkpoint), "--device", "cpu", "--tokens", "6", *extra]


def test_one_off_messages_are_deterministic_greedy_and_reproducible_seeded(checkpoint, capsys):
    outputs = []
    for flags in (["--temperature", "0"], ["--temperature", "0"], ["--seed", "4"], ["--seed", "4"]):
        assert chat.main(_cli(checkpoint, "-m", "the", "--quiet", *flags)) == 0
        outputs.append(capsys.readouterr().out)
    assert outputs[0] == outputs[1] and outputs[2] == outputs[3]


def test_json_output_transcript_and_quiet(checkpoint, capsys, tmp_path):
    log = tmp_path / "t" / "log.jsonl"
    assert chat.main(_cli(checkpoint, "-m", "the", "-m", "a", "--json", "--quiet", "--temperature", "0",
                          "--transcript", str(log))) == 0
    captured = capsys.readouterr()
    rows = [json.loads(line) for line in captured.out.splitlines()]
    assert [r["message"] for r in rows] == ["the", "a"] and captured.err == ""
    assert len(log.read_text().splitlines()) == 2


def test_piped_stdin_and_the_interactive_flag(checkpoint, capsys, monkeypatch):
    monkeypatch.setattr("sys.stdin", io.StringIO("the\n\na dog\n"))
    assert chat.main(_cli(checkpoint, "--json", "--quiet", "--temperature", "0")) == 0
    assert [json.loads(x)["message"] for x in capsys.readouterr().out.splitlines()] == ["the", "a dog"]
    typed = iter(["the", "/quit"])
    monkeypatch.setattr("builtins.input", lambda prompt="": next(typed))
    assert chat.main(_cli(checkpoint, "--interactive", "--quiet", "--temperature", "0")) == 0
    assert "QuantaWeave chat" in capsys.readouterr().out
    with pytest.raises(SystemExit):
        chat.main(_cli(checkpoint, "--interactive", "-m", "x"))


def test_bad_options_and_missing_models_are_clean_errors(checkpoint, tmp_path, capsys):
    for argv in (_cli(checkpoint, "-m", "x", "--temperature", "-1"), _cli(checkpoint, "-m", "x", "--top-p", "0"),
                 ["--run", "12345", "--runs-dir", str(tmp_path), "-m", "x"],
                 ["--latest", "--runs-dir", str(tmp_path), "-m", "x"]):
        with pytest.raises(SystemExit) as error:
            chat.main(argv)
        assert error.value.code == 2
    assert "error" in capsys.readouterr().err


def test_runs_latest_and_a_quantised_model(checkpoint, tmp_path, capsys):
    import shutil

    shutil.copytree(checkpoint, tmp_path / "runs" / "1700000000" / "model")
    assert chat.main(["--latest", "--runs-dir", str(tmp_path / "runs"), "--device", "cpu", "-m", "the",
                      "--tokens", "4", "--temperature", "0", "--quantize", "8"]) == 0
    err = capsys.readouterr().err
    assert "1700000000" in err and "int8" in err
    assert chat.main(["--run", "1700000000", "--runs-dir", str(tmp_path / "runs"), "--device", "cpu", "-m", "the",
                      "--tokens", "4", "--no-cache"]) == 0
    assert "decoding: no cache" in capsys.readouterr().err
