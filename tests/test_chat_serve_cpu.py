"""Chat session, batch messages, REPL and the HTTP server on CPU (reference tests: tests/test_chat.py,
tests/test_serve.py)."""

import io
import json

import pytest
import torch

from quantaweave_b200.tools.chat import (ChatSession, Settings, apply_setting, load_for_chat, main as chat_main,
                                         read_messages, repl, resolve_model, run_batch)


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    from test_tools_cpu import _train

    tmp = tmp_path_factory.mktemp("chat")
    _train(tmp, steps=4)
    return tmp / "out"


def _session(ckpt, use_cache=True, **kw):
    model, tok = load_for_chat(ckpt, None, 0, torch.device("cpu"))
    return ChatSession(model, tok, torch.device("cpu"), "fp32", Settings(**kw), use_cache=use_cache)


def test_cached_and_plain_decoding_agree_greedy(trained):
    cached = _session(trained, temperature=0.0, tokens=12).send("the cat")
    plain = _session(trained, use_cache=False, temperature=0.0, tokens=12).send("the cat")
    assert cached.response == plain.response and cached.tokens == plain.tokens
    assert cached.stop_reason in {"eos", "length", "stop"}


def test_seeded_sampling_is_reproducible_and_stop_strings_cut(trained):
    a = _session(trained, temperature=1.0, tokens=20, seed=3).send("a dog")
    b = _session(trained, temperature=1.0, tokens=20, seed=3).send("a dog")
    assert a.response == b.response
    if a.response:
        cut = a.response[len(a.response) // 2]
        c = _session(trained, temperature=1.0, tokens=20, seed=3, stop=[cut]).send("a dog")
        assert c.stop_reason == "stop" and cut not in c.response


def test_chat_mode_history_and_prompt(trained):
    s = _session(trained, mode="chat", temperature=0.0, tokens=5, system="be brief")
    s.send("hi")
    assert s.format_prompt("next").startswith("System: be brief\nUser: hi\nAssistant:")
    assert len(s.history) == 1
    apply_setting(s.settings, "top_p", "0.5")
    with pytest.raises(ValueError):
        apply_setting(s.settings, "top_p", "2")
    assert s.settings.top_p == 0.5


def test_messages_file_batch_and_exit_code(trained, tmp_path, capsys):
    path = tmp_path / "m.jsonl"
    path.write_text('{"message": "the", "expect": "zzzz-not-there", "tokens": 3}\n# comment\n{"prompt": "a"}\n')
    items = read_messages(path)
    assert [i["message"] for i in items] == ["the", "a"] and items[0]["expect"] == ["zzzz-not-there"]
    s = _session(trained, temperature=0.0, tokens=4)
    results = run_batch(s, items, False, lambda r: None)
    assert results[0]["passed"] is False and results[1]["passed"] is None and results[0]["tokens"] <= 3
    code = chat_main(["--checkpoint", str(trained), "--messages-file", str(path), "--json", "--quiet",
                      "--device", "cpu", "--temperature", "0"])
    assert code == 1
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert len(lines) == 2


def test_repl_commands(trained):
    s = _session(trained, temperature=0.0, tokens=3)
    inputs = iter(["/set temperature 0.5", "/mode chat", "hello", "/history", "/bogus", "/quit"])
    out = io.StringIO()
    repl(s, out=out, ask=lambda _: next(inputs))
    text = out.getvalue()
    assert "temperature = 0.5" in text and "mode: chat" in text and "you: hello" in text and "unknown command" in text


def test_resolve_model_latest_run(tmp_path, trained):
    import shutil

    root = tmp_path / "runs"
    shutil.copytree(trained, root / "100" / "model")
    (root / "200").mkdir()  # no model: skipped
    assert resolve_model(None, None, None, True, root) == (root / "100" / "model", None)
    with pytest.raises(FileNotFoundError):
        resolve_model(None, None, "999", False, root)


def test_http_server_routes(trained, tmp_path):
    from fastapi.testclient import TestClient

    from quantaweave_b200.tools.serve import Server, build_app

    blocklist = tmp_path / "block.txt"
    blocklist.write_text("# comment\nforbidden\n")
    server = Server(trained, None, torch.device("cpu"), "fp32", api_key="k", rate_limit=6,
                    moderation_patterns=blocklist)
    client = TestClient(build_app(server))
    auth = {"Authorization": "Bearer k"}
    assert client.get("/health").json()["status"] == "ok"
    assert client.post("/generate", json={"prompt": "the"}).status_code == 401
    r = client.post("/generate", json={"prompt": "the", "temperature": 0, "tokens": 5}, headers=auth)
    assert r.status_code == 200 and r.json()["tokens"] <= 5
    assert client.post("/generate", json={"prompt": "a forbidden word"}, headers=auth).status_code == 422
    r = client.post("/chat", json={"messages": [{"role": "user", "content": "hi"}], "tokens": 4, "temperature": 0},
                    headers=auth)
    assert r.status_code == 200
    assert client.post("/chat", json={"messages": [{"role": "assistant", "content": "x"}]},
                       headers=auth).status_code == 422
    with client.stream("POST", "/generate/stream", json={"prompt": "the", "tokens": 4, "temperature": 0},
                       headers=auth) as resp:
        body = "".join(resp.iter_text())
    assert "event: done" in body
    metrics = client.get("/metrics", headers={"X-API-Key": "k"}).text
    assert 'quantweave_requests_total{route="/generate",status="200"} 1' in metrics
    codes = [client.post("/generate", json={"prompt": "t", "tokens": 1}, headers=auth).status_code for _ in range(4)]
    assert 429 in codes


def test_http_server_continuous_batching(trained):
    """``batching=4``: concurrent /generate requests share decode steps; greedy replies equal the serialised
    server's, stop strings cut the text, and streaming delivers the same text."""
    import asyncio

    from fastapi.testclient import TestClient

    from quantaweave_b200.tools.serve import GenerateRequest, Server, build_app

    serial = Server(trained, None, torch.device("cpu"), "fp32")
    batched = Server(trained, None, torch.device("cpu"), "fp32", batching=4)
    try:
        prompts = ["the cat", "a", "the dog sat", "once", "the"]
        requests = [GenerateRequest(prompt=p, tokens=6 + i, temperature=0) for i, p in enumerate(prompts)]

        async def together():
            return await asyncio.gather(*(batched.generate(r) for r in requests))

        replies = asyncio.run(together())
        for r, got in zip(requests, replies):
            want = asyncio.run(serial.generate(r))
            assert got["text"] == want["text"] and got["tokens"] == want["tokens"], (r.prompt, got, want)
            assert got["stop_reason"] == want["stop_reason"]
        full = replies[0]["text"]
        if len(full) > 2:
            cut = asyncio.run(batched.generate(GenerateRequest(prompt="the cat", tokens=6, temperature=0,
                                                               stop=[full[1:3]])))
            assert cut["stop_reason"] == "stop" and cut["text"] == full[:1]
        client = TestClient(build_app(batched))
        with client.stream("POST", "/generate/stream", json={"prompt": "the cat", "tokens": 6, "temperature": 0}) as resp:
            body = "".join(resp.iter_text())
        events = [block.splitlines() for block in body.split("\n\n") if block.strip()]
        pieces = [json.loads(lines[0][len("data: "):])["text"] for lines in events if lines[0].startswith("data: ")]
        done = [json.loads(lines[1][len("data: "):]) for lines in events if lines[0] == "event: done"]
        assert len(done) == 1 and done[0]["text"] == full
        assert "".join(pieces) == full
    finally:
        batched.close()


def test_stream_disconnect_waits_for_the_worker_thread(trained):
    """A streaming client that goes away mid-reply ends the producer inside its worker thread, and the relay returns
    only after that thread has returned, so the session lock is never released while the session is still in use."""
    import asyncio
    import threading

    from quantaweave_b200.tools.serve import ClientDisconnected, GenerateRequest, Server

    server = Server(trained, None, torch.device("cpu"), "fp32")
    release, worker_done, outcome = threading.Event(), threading.Event(), []

    def produce(on_text):
        try:
            on_text("a")
            release.wait(10)
            on_text("b")  # the client is gone by now: this raises inside the worker
            outcome.append("kept going")
        except ClientDisconnected:
            outcome.append("stopped")
            raise
        finally:
            worker_done.set()

    async def disconnecting_client():
        events = server._relay(produce, interrupt=True)
        assert '"a"' in await events.__anext__()
        threading.Timer(0.3, release.set).start()
        await events.aclose()
        assert worker_done.is_set()  # aclose came back only after the worker returned

    asyncio.run(disconnecting_client())
    assert outcome == ["stopped"]

    async def stream_then_generate():
        events = server.stream_generate(GenerateRequest(prompt="the", tokens=64, temperature=0))
        await events.__anext__()  # first piece arrives; the client then disconnects
        await events.aclose()
        assert not server.lock.locked()
        reply = await server.generate(GenerateRequest(prompt="the", tokens=4, temperature=0))
        assert reply["tokens"] <= 4

    asyncio.run(stream_then_generate())
