"""Production hardening on CPU (reference tests: tests/test_production_readiness.py): the single checkpoint loader,
PII redaction (shapes, per-category counts, in the trainer and the token packer), data cards in the archive manifest,
the experiment manager's promotion gate, and the HTTP server's API key, rate limit, moderation, queue bound, start
timeout, Prometheus metrics, structured logs and health report."""

import asyncio
import io
import json
import logging
import re
from pathlib import Path

import pytest
import torch

from quantaweave_b200.utils.checkpoint_io import load_checkpoint
from quantaweave_b200.utils.pii_redact import PIIRedactor

PACKAGE = Path(__file__).resolve().parents[1] / "quantaweave_b200"


# ---- checkpoint loading ---------------------------------------------------------------------------------------
def test_load_checkpoint_round_trips_a_mixed_payload_and_honours_map_location(tmp_path):
    payload = {"model": {"w": torch.arange(6.0).view(2, 3)}, "step": 7, "rng_state": torch.get_rng_state(),
               "extra": {"note": "x", "history": [1.5, 2.5]}}
    torch.save(payload, tmp_path / "c.pt")
    back = load_checkpoint(tmp_path / "c.pt")
    assert back["step"] == 7 and back["extra"] == payload["extra"] and torch.equal(back["model"]["w"],
                                                                                    payload["model"]["w"])
    assert load_checkpoint(str(tmp_path / "c.pt"), map_location="cpu")["model"]["w"].device.type == "cpu"


def test_every_package_module_unpickles_checkpoints_through_the_one_loader():
    offenders = [str(p.relative_to(PACKAGE)) for p in PACKAGE.rglob("*.py")
                 if p.name != "checkpoint_io.py" and "torch.load(" in p.read_text()]
    assert not offenders, offenders


# ---- PII redaction ---------------------------------------------------------------------------------------------
def test_redactor_catches_common_shapes_counts_them_and_leaves_ordinary_text_alone():
    redactor = PIIRedactor()
    text = ("mail jane.doe@example.com or call (555) 123-4567; ssn 123-45-6789; card 4111 1111 1111 1111; "
            "host 192.168.0.12")
    out = redactor.redact(text)
    for secret in ("jane.doe@example.com", "123-4567", "123-45-6789", "4111 1111", "192.168.0.12"):
        assert secret not in out, secret
    for tag in ("<EMAIL>", "<PHONE>", "<SSN>", "<CREDIT_CARD>", "<IPV4>"):
        assert tag in out, tag
    assert redactor.report() == {"EMAIL": 1, "PHONE": 1, "SSN": 1, "CREDIT_CARD": 1, "IPV4": 1}
    plain = "version 1.2 shipped in 2024 with 3 new features, see page 12."
    assert PIIRedactor().redact(plain) == plain


def test_the_token_packer_redacts_when_asked(tmp_path):
    from quantaweave_b200.data.pipeline import load_token_bin
    from quantaweave_b200.tools.prepare_tokens import main as prepare

    data = tmp_path / "d.jsonl"
    data.write_text("".join(json.dumps({"text": f"row {i} write to someone{i}@example.com today"}) + "\n"
                            for i in range(20)))
    texts = {}
    for name, extra in (("plain", []), ("redacted", ["--redact-pii"])):
        prepare(["pack", "--data", str(data), "--tokenizer", "char", "--vocab-size", "96",
                 "--output", str(tmp_path / name), *extra])
        corpus, tok = load_token_bin(tmp_path / name)
        texts[name] = tok.decode(corpus.read(0, 400).tolist())
    assert "@example.com" in texts["plain"] and "@example.com" not in texts["redacted"]
    assert "<EMAIL>" in texts["redacted"]


# ---- data cards and the promotion gate ------------------------------------------------------------------------
def test_data_cards_are_embedded_verbatim_or_recorded_as_an_error(tmp_path):
    from quantaweave_b200.tools.run_bundle import archive_data

    data = tmp_path / "d.jsonl"
    data.write_text('{"text": "a"}\n')
    card = tmp_path / "card.json"
    card.write_text(json.dumps({"source": "synthetic", "license": "CC0", "pii": "none"}))
    for name, card_path, check in (("ok", card, lambda m: m["data_card"]["license"] == "CC0"),
                                   ("bad", tmp_path / "missing.json", lambda m: "data_card_error" in m),
                                   ("none", None, lambda m: "data_card" not in m and "data_card_error" not in m)):
        bundle = tmp_path / name
        bundle.mkdir()
        assert check(archive_data([data], bundle, 10, 1, card_path)), name


def test_trainer_data_card_flag_reaches_the_archive_manifest(tmp_path):
    from quantaweave_b200.training.trainer import default_args, run_training

    data = tmp_path / "d.jsonl"
    data.write_text("".join(json.dumps({"text": f"story {i}: a fox and a dog."}) + "\n" for i in range(30)))
    card = tmp_path / "card.json"
    card.write_text(json.dumps({"license": "CC-BY"}))
    summary = run_training(default_args(data=[data], steps=2, batch_size=2, sequence_length=16, examples=20,
                                        hidden_size=16, layers=1, ffn_size=16, attention_heads=2, total_experts=2,
                                        active_experts=1, vocab_size=64, device="cpu", checkpoint_interval=0,
                                        no_power_tracking=True, output=tmp_path / "o", checkpoint_dir=tmp_path / "c",
                                        archive_dir=tmp_path / "runs", data_card=card, archive_benchmark_examples=5))
    manifest = json.loads((Path(summary["archive"]) / "data" / "manifest.json").read_text())
    assert manifest["data_card"] == {"license": "CC-BY"}


@pytest.mark.parametrize("threshold,value,promotable", [(None, 9.0, True), (3.5, 4.0, False), (3.5, 3.0, True)])
def test_best_run_is_promotable_only_under_the_threshold(tmp_path, threshold, value, promotable):
    from quantaweave_b200.tools.experiment_manager import update_best

    summary = {"run_id": "r1", "run_dir": str(tmp_path / "r1"), "train": {"final_loss": value}}
    assert update_best(tmp_path, summary, None, threshold)
    best = json.loads((tmp_path / "best.json").read_text())
    assert best["promotable"] is promotable and best["value"] == value and best["objective"] == "train.final_loss"
    worse = {"run_id": "r2", "run_dir": str(tmp_path / "r2"), "train": {"final_loss": value + 1}}
    assert not update_best(tmp_path, worse, None, threshold)  # only a better run replaces the record


# ---- the HTTP server ---------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from test_tools_cpu import _train

    tmp = tmp_path_factory.mktemp("prod")
    _train(tmp, steps=2)
    return tmp / "out"


def _server(checkpoint, **kw):
    from quantaweave_b200.tools.serve import Server

    return Server(checkpoint, None, torch.device("cpu"), "fp32", **kw)


def _client(server):
    from fastapi.testclient import TestClient

    from quantaweave_b200.tools.serve import build_app

    return TestClient(build_app(server))


def test_the_server_is_open_by_default(checkpoint):
    client = _client(_server(checkpoint))
    assert client.post("/generate", json={"prompt": "the", "tokens": 2, "temperature": 0}).status_code == 200
    assert client.get("/metrics").status_code == 200


def test_api_key_gates_every_route_but_health_and_accepts_both_headers(checkpoint):
    client = _client(_server(checkpoint, api_key="s3cret"))
    body = {"prompt": "the", "tokens": 2, "temperature": 0}
    assert client.get("/health").status_code == 200
    for headers in ({}, {"Authorization": "Bearer wrong"}, {"X-API-Key": "nope"}):
        assert client.post("/generate", json=body, headers=headers).status_code == 401
    assert client.get("/metrics").status_code == 401
    assert client.post("/generate", json=body, headers={"Authorization": "Bearer s3cret"}).status_code == 200
    assert client.post("/generate", json=body, headers={"X-API-Key": "s3cret"}).status_code == 200
    assert client.get("/metrics", headers={"X-API-Key": "s3cret"}).status_code == 200


def test_rate_limit_and_moderation(checkpoint, tmp_path):
    blocklist = tmp_path / "block.txt"
    blocklist.write_text("# patterns\nsecret\\s+plan\n")
    client = _client(_server(checkpoint, rate_limit=2, moderation_patterns=blocklist))
    body = {"prompt": "the", "tokens": 1, "temperature": 0}
    codes = [client.post("/generate", json=body).status_code for _ in range(3)]
    assert codes == [200, 200, 429]
    client = _client(_server(checkpoint, moderation_patterns=blocklist))
    assert client.post("/generate", json={"prompt": "the SECRET   plan"}).status_code == 422
    chat = {"messages": [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "ok"},
                         {"role": "user", "content": "tell me the secret plan"}]}
    assert client.post("/chat", json=chat).status_code == 422
    chat["messages"][-1]["content"] = "hello"
    assert client.post("/chat", json={**chat, "tokens": 2, "temperature": 0}).status_code == 200


def test_the_queue_bound_and_the_start_timeout(checkpoint):
    from fastapi import HTTPException

    from quantaweave_b200.tools.serve import GenerateRequest

    request = GenerateRequest(prompt="the", tokens=1, temperature=0)

    async def scenario():
        free = _server(checkpoint, max_queue=0)
        assert (await free.generate(request))["tokens"] <= 1  # a free lock is never refused, even with no queue
        bounded = _server(checkpoint, max_queue=1)
        await bounded.lock.acquire()  # an earlier request is still generating
        waiter = asyncio.ensure_future(bounded.generate(request))
        await asyncio.sleep(0.05)
        assert bounded.waiting == 1
        with pytest.raises(HTTPException) as full:
            await bounded.generate(request)
        assert full.value.status_code == 429
        bounded.lock.release()
        assert (await waiter)["tokens"] <= 1 and bounded.waiting == 0
        slow = _server(checkpoint, request_timeout=0.05)
        await slow.lock.acquire()
        with pytest.raises(HTTPException) as timed_out:
            await slow.generate(request)
        assert timed_out.value.status_code == 503 and slow.waiting == 0
        slow.lock.release()

    asyncio.run(scenario())


def test_metrics_are_valid_prometheus_text(checkpoint):
    client = _client(_server(checkpoint))
    client.post("/generate", json={"prompt": "the", "tokens": 2, "temperature": 0})
    client.post("/chat", json={"messages": [{"role": "assistant", "content": "x"}]})
    text = client.get("/metrics").text
    sample = re.compile(r'^[a-zA-Z_:][a-zA-Z0-9_:]*(\{[a-zA-Z_][a-zA-Z0-9_]*="[^"]*"(,[a-zA-Z_][a-zA-Z0-9_]*="[^"]*")*\})?'
                        r' -?[0-9.e+-]+$')
    helped, typed = set(), set()
    for line in text.splitlines():
        if line.startswith("# HELP "):
            helped.add(line.split()[2])
        elif line.startswith("# TYPE "):
            typed.add(line.split()[2])
            assert line.split()[3] in {"counter", "gauge"}
        else:
            assert sample.match(line), line
    assert helped == typed and "quantweave_requests_total" in typed
    assert 'quantweave_requests_total{route="/chat",status="422"} 1' in text
    assert 'quantweave_errors_total{route="/chat"} 1' in text


def test_json_logs_one_object_per_line_and_a_structured_line_per_request(checkpoint):
    from quantaweave_b200.tools import serve

    stream = io.StringIO()
    handler = logging.StreamHandler(stream)
    handler.setFormatter(serve.JSONLogFormatter())
    record = logging.LogRecord("x", logging.WARNING, __file__, 1, "hello %s", ("world",), None)
    record.request_id = "abc"
    parsed = json.loads(serve.JSONLogFormatter().format(record))
    assert parsed["message"] == "hello world" and parsed["level"] == "WARNING" and parsed["request_id"] == "abc"
    serve.configure_logging("json")
    assert isinstance(serve.logger.handlers[0].formatter, serve.JSONLogFormatter)
    serve.configure_logging("text")
    assert not isinstance(serve.logger.handlers[0].formatter, serve.JSONLogFormatter)
    serve.logger.addHandler(handler)
    try:
        _client(_server(checkpoint)).post("/generate", json={"prompt": "the", "tokens": 1, "temperature": 0})
    finally:
        serve.logger.removeHandler(handler)
    lines = [json.loads(line) for line in stream.getvalue().splitlines()]
    assert lines and lines[-1]["route"] == "/generate" and lines[-1]["status"] == 200
    assert len(lines[-1]["request_id"]) == 12 and lines[-1]["seconds"] >= 0


def test_health_reports_the_hardening_configuration(checkpoint):
    info = _client(_server(checkpoint, api_key="k", rate_limit=5, request_timeout=2.5, max_queue=3)).get(
        "/health").json()
    assert info["status"] == "ok" and info["auth_required"] is True
    assert (info["rate_limit"], info["request_timeout"], info["max_queue"]) == (5, 2.5, 3)
    assert info["context_length"] > 0 and "KV cache" in info["decoding"] and info["batching_slots"] == 0


def test_generate_matches_the_chat_session_and_concurrent_requests_never_mix(checkpoint):
    from quantaweave_b200.tools.chat import ChatSession, Settings, load_for_chat
    from quantaweave_b200.tools.serve import GenerateRequest

    server = _server(checkpoint)
    model, tokenizer = load_for_chat(checkpoint, None, 0, torch.device("cpu"))
    session = ChatSession(model, tokenizer, torch.device("cpu"), "fp32", Settings(temperature=0.0, tokens=8))
    prompts = ["the cat", "a dog", "numbers 1", "sun and"]
    expected = [session.send(p).response for p in prompts]
    single = asyncio.run(server.generate(GenerateRequest(prompt=prompts[0], tokens=8, temperature=0.0)))
    assert single["text"] == expected[0]

    async def together():
        return await asyncio.gather(*(server.generate(GenerateRequest(prompt=p, tokens=8, temperature=0.0))
                                      for p in prompts))

    replies = asyncio.run(together())  # serialised behind the lock, each on a fresh decoder state
    assert [r["text"] for r in replies] == expected
    with pytest.raises(Exception):
        GenerateRequest(prompt="x", tokens=0)  # validated before it reaches the model
    with pytest.raises(Exception):
        GenerateRequest(prompt="x", temperature=-1)
