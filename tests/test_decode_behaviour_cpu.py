"""KV-cache decoder behaviour on CPU against the model's own forward pass (reference tests:
tests/test_fast_decode.py): every cached step equals the full forward at that position (routing top-k, router
temperature and a straggler selection bias included), prefill leaves the same cache as stepping, the prompt is read
inside a context one shorter than the learned-position window, the oldest half slides out when the cache fills,
streaming equals a host-driven loop across slides, sampling is per-seed reproducible and honours top-k / top-p / the
vocabulary mask, first-token frequencies follow the softmax, quantised and LoRA models decode like their own forward,
and layouts the decoder cannot serve are refused cleanly (the chat tool then decodes without a cache)."""

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.inference.fast_decode import FastDecoder, Unsupported

CPU = torch.device("cpu")


def _model(layers=3, experts=8, top_k=2, context=24, temperature=1.0, seed=0, **extra):
    torch.manual_seed(seed)
    cfg = QuantaWeaveConfig(vocab_size=64, hidden_size=32, layers=layers, ffn_size=48, num_experts=experts,
                            top_k=top_k, attention_heads=4, max_sequence_length=context, capacity_factor=0.0,
                            router_temperature=temperature, **extra)
    model = QuantaWeaveMoEForCausalLM(cfg).eval()
    model.set_routing_controls(drop_overflow_tokens=False)  # no capacity at inference, in the oracle too
    return model


def _forward(model, tokens):
    with torch.no_grad():
        return model(torch.tensor([tokens]))["logits"][0]


def _tokens(n, seed, low=0):
    return torch.randint(low, 64, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def _greedy_by_hand(model, prompt, count):
    dec = FastDecoder(model, CPU, "fp32")
    logits, out = dec.feed(prompt), []
    for _ in range(count):
        out.append(int(logits.argmax()))
        logits = dec.append(out[-1])
    return out


@pytest.mark.parametrize("top_k,temperature,biased", [(1, 1.0, False), (2, 0.7, True), (3, 2.0, False)])
def test_each_cached_step_equals_the_full_forward(top_k, temperature, biased):
    model = _model(top_k=top_k, temperature=temperature)
    if biased:
        for i, moe in enumerate(model.moes()):
            moe.expert_bias = torch.randn(moe.num_experts, generator=torch.Generator().manual_seed(i))
    tokens = _tokens(23, 1)
    full = _forward(model, tokens)
    dec = FastDecoder(model, CPU, "fp32")
    assert torch.allclose(dec.feed(tokens[:1]), full[0], atol=1e-5)
    for pos in range(1, 23):
        assert torch.allclose(dec.append(tokens[pos]), full[pos], atol=1e-5), pos


def test_rope_gqa_rmsnorm_layout_steps_like_the_full_forward():
    model = _model(norm_type="rmsnorm", position_embedding="rope", kv_heads=2, attention_bias=False)
    tokens = _tokens(20, 2)
    full = _forward(model, tokens)
    dec = FastDecoder(model, CPU, "fp32")
    assert torch.allclose(dec.feed(tokens[:6]), full[5], atol=1e-5)
    for pos in range(6, 20):
        assert torch.allclose(dec.append(tokens[pos]), full[pos], atol=1e-5), pos


def test_prefill_leaves_the_cache_that_stepping_builds():
    model = _model()
    tokens = _tokens(17, 3)
    stepped = FastDecoder(model, CPU, "fp32")
    for token in tokens:
        stepped._run(token)
    read = FastDecoder(model, CPU, "fp32")
    assert torch.allclose(read.feed(tokens), _forward(model, tokens)[-1], atol=1e-5)
    for a, b in zip(stepped.layers, read.layers):
        assert torch.allclose(a.keys[:, :, :17], b.keys[:, :, :17], atol=1e-5)
        assert torch.allclose(a.values[:, :, :17], b.values[:, :, :17], atol=1e-5)
    assert read.length == 17 and read.tokens == tokens


def test_prefill_puts_the_models_routing_settings_back():
    model = _model()
    model.set_routing_controls(capacity_factor=1.25, drop_overflow_tokens=True)
    before = [(m.capacity_factor, m.drop_overflow_tokens, m.kernel) for m in model.moes()]
    FastDecoder(model, CPU, "fp32")._prefill(torch.tensor([[1, 2, 3]]))
    assert [(m.capacity_factor, m.drop_overflow_tokens, m.kernel) for m in model.moes()] == before


def test_the_context_is_one_shorter_than_the_learned_position_window():
    dec = FastDecoder(_model(context=24), CPU, "fp32")
    assert dec.capacity == 23
    tokens = list(range(1, 40))
    dec.feed(tokens)
    assert dec.tokens == tokens[-23:] and dec.length == 23  # only the newest 23 tokens are read


def test_a_full_cache_drops_its_oldest_half_and_rereads_the_rest():
    model = _model(context=13)  # capacity 12
    dec = FastDecoder(model, CPU, "fp32")
    tokens = _tokens(30, 4)
    dec.feed(tokens[:1])
    kept = tokens[:1]
    for token in tokens[1:]:
        logits = dec.append(token)
        if len(kept) >= 12:
            kept = kept[-6:]
        kept = kept + [token]
        assert dec.tokens == kept and dec.length == len(kept) <= 12
        assert torch.allclose(logits, _forward(model, kept)[-1], atol=1e-5)  # what a fresh read of `kept` gives


@pytest.mark.parametrize("count", [1, 8, 20, 61])
def test_greedy_streaming_equals_the_host_loop_across_slides(count):
    model = _model(context=13)
    prompt = _tokens(5, 5, low=2)
    streamed = list(FastDecoder(model, CPU, "fp32").stream(prompt, count, temperature=0.0))
    assert len(streamed) == count and streamed == _greedy_by_hand(model, prompt, count)


def test_long_single_token_and_empty_prompts():
    model = _model(context=13)
    assert len(list(FastDecoder(model, CPU, "fp32").stream(list(range(2, 50)), 5, temperature=0.0))) == 5
    assert len(list(FastDecoder(model, CPU, "fp32").stream([7], 5, temperature=0.0))) == 5
    with pytest.raises(ValueError):
        list(FastDecoder(model, CPU, "fp32").stream([], 5, temperature=0.0))


def test_sampling_is_seeded_and_honours_top_k_top_p_and_the_vocabulary_mask():
    dec = FastDecoder(_model(context=30), CPU, "fp32")

    def run(seed, **kw):
        return list(dec.stream([3, 4, 5], 30, temperature=1.0, generator=torch.Generator().manual_seed(seed), **kw))

    assert run(1) == run(1) and run(1) != run(2)
    greedy = list(dec.stream([3, 4, 5], 30, temperature=0.0))
    assert run(5, top_k=1) == greedy and run(5, top_p=1e-6) == greedy
    assert all(0 < t < 20 for t in run(3, valid_ids=20, unk_id=0))  # ids >= 20 and the unknown id never appear


def test_first_token_frequencies_follow_the_softmax():
    model = _model(context=16)
    dec = FastDecoder(model, CPU, "fp32")
    prompt = [3, 4, 5, 6]
    probs = torch.softmax(_forward(model, prompt)[-1], dim=-1)
    gen = torch.Generator().manual_seed(0)
    trials = 1500
    counts = torch.zeros(64)
    for _ in range(trials):
        counts[next(iter(dec.stream(prompt, 1, temperature=1.0, generator=gen)))] += 1
    assert (counts / trials - probs).abs().max() < 0.05


def test_a_cold_temperature_is_greedy_and_an_abandoned_stream_leaves_the_decoder_usable():
    model = _model(context=30)
    dec = FastDecoder(model, CPU, "fp32")
    cold = [list(dec.stream([3, 4], 12, temperature=1e-3, generator=torch.Generator().manual_seed(s)))
            for s in range(4)]
    assert all(c == cold[0] for c in cold)
    gen = dec.stream([3, 4], 50, temperature=0.0)
    first = [next(gen) for _ in range(3)]
    gen.close()
    assert first == _greedy_by_hand(model, [3, 4], 3)
    assert list(dec.stream([3, 4], 5, temperature=0.0)) == _greedy_by_hand(model, [3, 4], 5)


def test_quantised_and_lora_models_decode_like_their_own_forward():
    from quantaweave_b200.inference.quantization import quantize_model
    from quantaweave_b200.tools.lora import add_lora

    model = _model(top_k=2)
    quantize_model(model, 8)
    tokens = _tokens(14, 6)
    assert torch.allclose(FastDecoder(model, CPU, "fp32").feed(tokens), _forward(model, tokens)[-1], atol=1e-4)
    model = _model(top_k=2)
    add_lora(model, rank=4, alpha=8)
    for module in model.modules():
        if hasattr(module, "lora_b"):
            with torch.no_grad():
                module.lora_b.normal_(0, 0.1, generator=torch.Generator().manual_seed(7))
    assert torch.allclose(FastDecoder(model, CPU, "fp32").feed(tokens), _forward(model, tokens)[-1], atol=1e-4)


def test_layouts_the_decoder_cannot_serve_are_refused_and_chat_falls_back():
    from quantaweave_b200.data.pipeline import CharTokenizer
    from quantaweave_b200.parallel.expert_parallel import ExpertParallelContext
    from quantaweave_b200.tools.chat import ChatSession, Settings

    with pytest.raises(Unsupported):
        FastDecoder(torch.nn.Linear(2, 2), CPU)
    ctx = ExpertParallelContext(0, 1, CPU, tp_size=2)
    tp_model = QuantaWeaveMoEForCausalLM(QuantaWeaveConfig(vocab_size=8, hidden_size=16, layers=1, ffn_size=8,
                                                           num_experts=2, top_k=1, attention_heads=2,
                                                           max_sequence_length=8), expert_parallel=ctx)
    with pytest.raises(Unsupported):
        FastDecoder(tp_model, CPU)
    session = ChatSession(tp_model.eval(), CharTokenizer.build(["ab"], 8), CPU, "fp32", Settings())
    assert session.decoder is None and "no cache" in session.cache_note
