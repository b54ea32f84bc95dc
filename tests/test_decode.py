"""FastDecoder: the cached step reproduces the full forward (CPU oracle), quantised formats round-trip, and the
native B200 decoder (bf16 / int8 per-channel / int4 g128 experts) matches the CPU oracle."""

import pytest
import torch

from conftest import cuda_ready
from quantaweave_b200 import QuantaWeaveMoEForCausalLM, preset


def _model(**kw):
    cfg = preset("tiny-cpu", max_sequence_length=65, **kw)
    torch.manual_seed(0)
    m = QuantaWeaveMoEForCausalLM(cfg).eval()
    for moe in m.moes():
        moe.drop_overflow_tokens = False
    return m


@pytest.mark.parametrize("layout", [dict(), dict(norm_type="layernorm", position_embedding="learned",
                                                 attention_bias=True, kv_heads=2)])
def test_cpu_decoder_matches_full_forward(layout):
    from quantaweave_b200.inference.fast_decode import FastDecoder

    model = _model(**layout)
    ids = torch.randint(0, 512, (1, 20), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        full = model(ids)["logits"][0]
    dec = FastDecoder(model, torch.device("cpu"))
    logits = dec.feed(ids[0, :5].tolist())
    assert torch.allclose(logits, full[4], atol=1e-4), (logits - full[4]).abs().max()
    for pos in range(5, 20):
        logits = dec.append(int(ids[0, pos]))
        assert torch.allclose(logits, full[pos], atol=1e-4), pos


def test_cpu_batched_generate_matches_single():
    from quantaweave_b200.inference.fast_decode import FastDecoder

    model = _model()
    prompts = torch.randint(0, 512, (3, 7), generator=torch.Generator().manual_seed(2))
    batched = FastDecoder(model, torch.device("cpu"), max_batch=3).generate(prompts, 6)
    for b in range(3):
        single = FastDecoder(model, torch.device("cpu")).generate(prompts[b:b + 1], 6)
        assert torch.equal(single[0], batched[b])


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ready(), reason="needs a B200")
@pytest.mark.parametrize("bits,group", [(None, None), (8, None), (4, 128)])
def test_native_decoder_matches_cpu_oracle(bits, group):
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.inference.quantization import quantize_model

    model = _model(hidden_size=256, attention_heads=4, ffn_size=256)
    if bits is not None:
        quantize_model(model, bits, group)
    prompts = torch.randint(0, 512, (4, 16), generator=torch.Generator().manual_seed(3))
    cpu = FastDecoder(model, torch.device("cpu"), max_batch=4)
    cpu._prefill(prompts[:, :-1])
    ref = cpu.run_step(prompts[:, -1], torch.full((4,), 15)).clone()
    gpu_model = model.cuda()
    dec = FastDecoder(gpu_model, torch.device("cuda"), max_batch=4)
    assert dec.uses_graph
    from quantaweave_b200.ops import ext

    dec._C = ext()
    dec._prefill(prompts[:, :-1].cuda())
    got = dec.run_step(prompts[:, -1].cuda(), torch.full((4,), 15, device="cuda")).cpu()
    err = (got - ref).abs().max().item()
    assert err < 0.05 * ref.abs().max().item() + 0.05, err
    tokens = dec.generate(prompts.cuda(), 8)
    assert tokens.shape == (4, 8)
    assert ext().read_status(True) == 0
