"""Continuous batching over the decoder's cache rows (CPU, fp32 decode path)."""

import threading

import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.inference.batching import BatchingWorker, ContinuousBatcher, GenerationRequest
from quantaweave_b200.inference.fast_decode import FastDecoder


def _model():
    cfg = QuantaWeaveConfig(vocab_size=64, hidden_size=32, layers=2, ffn_size=64, num_experts=4, top_k=2,
                            attention_heads=4, kv_heads=2, max_sequence_length=65, capacity_factor=0.0,
                            norm_type="rmsnorm", position_embedding="rope", init_std=0.2)
    torch.manual_seed(0)
    return QuantaWeaveMoEForCausalLM(cfg).eval()


PROMPTS = [[1, 2, 3], [5], [7, 8, 9, 10, 11], [2, 2], [3, 1, 4, 1, 5, 9]]
BUDGETS = [5, 7, 3, 6, 4]


def _run(model, requests):
    batcher = ContinuousBatcher(FastDecoder(model, torch.device("cpu"), max_batch=4))
    for r in requests:
        batcher.submit(r)
    batcher.run_until_idle()
    return batcher


def test_requests_decoded_together_match_each_alone_and_the_full_forward():
    model = _model()
    together = [GenerationRequest(p, n) for p, n in zip(PROMPTS, BUDGETS)]
    batcher = _run(model, together)
    alone = []
    for p, n in zip(PROMPTS, BUDGETS):
        r = GenerationRequest(p, n)
        _run(model, [r])
        alone.append(r.tokens)
    assert [r.tokens for r in together] == alone
    assert all(r.finish_reason == "length" and len(r.tokens) == n for r, n in zip(together, BUDGETS))
    # five requests over four slots: the fifth joined when the first finished, no step ran for a lone request
    assert batcher.steps < sum(BUDGETS)
    with torch.no_grad():  # greedy decoding equals argmax of the full-context forward
        ids = list(PROMPTS[2])
        for _ in range(BUDGETS[2]):
            ids.append(int(model(torch.tensor([ids]))["logits"][0, -1].argmax()))
    assert ids[len(PROMPTS[2]):] == together[2].tokens


def test_sampling_is_seeded_per_request_and_stop_ids_end_a_request():
    model = _model()
    a = GenerationRequest([4, 5, 6], 8, temperature=1.0, top_k=10, seed=7)
    b = GenerationRequest([4, 5, 6], 8, temperature=1.0, top_k=10, seed=7)
    c = GenerationRequest([4, 5, 6], 8, temperature=1.0, top_k=10, seed=8)
    _run(model, [a, b, c])
    assert a.tokens == b.tokens
    stop = a.tokens[2]
    d = GenerationRequest([4, 5, 6], 8, temperature=1.0, top_k=10, seed=7, stop_ids=(stop,))
    _run(model, [d])
    assert d.finish_reason == "stop" and d.tokens[-1] == stop and len(d.tokens) <= 3


def test_worker_thread_serves_concurrent_submitters():
    model = _model()
    worker = BatchingWorker(ContinuousBatcher(FastDecoder(model, torch.device("cpu"), max_batch=4)))
    results = {}
    streamed = {i: [] for i in range(len(PROMPTS))}

    def client(i):
        r = GenerationRequest(PROMPTS[i], BUDGETS[i], on_token=streamed[i].append)
        worker.submit(r)
        results[i] = r.wait(timeout=60)

    threads = [threading.Thread(target=client, args=(i,)) for i in range(len(PROMPTS))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    worker.close()
    assert worker.error is None
    for i in range(len(PROMPTS)):
        assert results[i] == streamed[i] and len(results[i]) == BUDGETS[i]
    expected = []
    for p, n in zip(PROMPTS, BUDGETS):
        r = GenerationRequest(p, n)
        _run(model, [r])
        expected.append(r.tokens)
    assert [results[i] for i in range(len(PROMPTS))] == expected


def test_a_failing_prefill_and_closing_the_worker_never_leave_a_request_waiting(monkeypatch):
    import pytest

    model = _model()
    worker = BatchingWorker(ContinuousBatcher(FastDecoder(model, torch.device("cpu"), max_batch=2)))
    original = worker.batcher.decoder._prefill

    def prefill(prompts, first_row=0):
        if 63 in prompts.tolist()[0]:
            raise RuntimeError("bad prompt")
        return original(prompts, first_row)

    monkeypatch.setattr(worker.batcher.decoder, "_prefill", prefill)
    bad = worker.submit(GenerationRequest([63, 1, 2], 4))
    bad.wait(timeout=30)
    assert bad.finish_reason.startswith("error") and "bad prompt" in bad.finish_reason
    assert isinstance(worker.error, RuntimeError)
    good = worker.submit(GenerationRequest([1, 2], 3))
    assert len(good.wait(timeout=30)) == 3 and good.finish_reason == "length"  # the worker keeps serving
    worker._stop.set()  # stop stepping first, so the next request stays queued until close
    worker._thread.join(timeout=5)
    queued = worker.batcher.submit(GenerationRequest([1, 2], 3))
    worker.close()
    assert queued.wait(timeout=1) == [] and queued.finish_reason == "closed"
    with pytest.raises(RuntimeError, match="closed"):
        worker.submit(GenerationRequest([1], 1))


def test_a_stream_closed_early_cancels_its_batched_job(tmp_path):
    import asyncio
    import time

    from test_tools_cpu import _train

    from quantaweave_b200.tools.serve import GenerateRequest, Server

    _train(tmp_path, steps=1)
    server = Server(tmp_path / "out", None, torch.device("cpu"), "fp32", batching=2)
    jobs = []
    submit = server.worker.submit
    server.worker.submit = lambda job: jobs.append(job) or submit(job)
    try:
        async def first_piece_then_leave():
            stream = server.stream_generate(GenerateRequest(prompt="the", tokens=60, temperature=0.0, stop=[]))
            async for _ in stream:
                break  # the client disconnects after the first event
            await stream.aclose()

        asyncio.run(first_piece_then_leave())
        deadline = time.time() + 10
        while server.worker.batcher.pending() and time.time() < deadline:
            time.sleep(0.02)
        assert server.worker.batcher.pending() == 0
        assert jobs[0].done.is_set() and jobs[0].cancelled
        assert len(jobs[0].tokens) < jobs[0].max_new  # retired early, not decoded to its budget
    finally:
        server.close()


def test_queued_requests_can_be_withdrawn_and_the_server_times_out_waiting_ones(tmp_path):
    import asyncio
    import time

    import pytest
    from fastapi import HTTPException
    from test_tools_cpu import _train

    from quantaweave_b200.tools.serve import GenerateRequest, Server

    batcher = ContinuousBatcher(FastDecoder(_model(), torch.device("cpu"), max_batch=1))
    first, second = GenerationRequest([1, 2], 3), GenerationRequest([3], 3)
    batcher.submit(first)
    batcher.submit(second)
    batcher.step()  # `first` holds the only slot
    assert batcher.withdraw(second) and second.finish_reason == "withdrawn" and second.done.is_set()
    assert not batcher.withdraw(first)  # already decoding: it runs to the end
    batcher.run_until_idle()
    assert first.finish_reason == "length"

    _train(tmp_path, steps=1)
    server = Server(tmp_path / "out", None, torch.device("cpu"), "fp32", batching=1, request_timeout=0.2)
    try:
        # a worker whose slots never free up: every step makes no progress, so requests stay queued
        server.worker.batcher.step = lambda: time.sleep(0.01)
        with pytest.raises(HTTPException) as waited:
            asyncio.run(server.generate(GenerateRequest(prompt="the", tokens=2, temperature=0.0)))
        assert waited.value.status_code == 503 and server.worker.batcher.pending() == 0
    finally:
        server.close()
