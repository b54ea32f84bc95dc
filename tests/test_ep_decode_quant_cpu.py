"""Quantised expert-parallel decoding on 2 gloo ranks: each rank quantises only the experts it holds (int4 g8 and
int8 per-channel) and decodes SPMD with one all-reduce per MoE layer; the greedy tokens equal the single-process
decoder's over the fully quantised model. A quantised file still needs the consolidated model."""

import pytest
import torch

from quantaweave_b200 import QuantaWeaveMoEForCausalLM

from test_parallel_cpu import run_ranks, tiny_config


def _case(rank, world, bits, group):
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.inference.quantization import quantize_model, save_quantized
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel

    cfg = tiny_config(capacity_factor=0.0, max_sequence_length=33, attention_heads=4, kv_heads=2)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg).eval()
    ep = init_expert_parallel("cpu", 1)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).eval()
    per = cfg.num_experts // world
    state = {}
    for key, value in full.state_dict().items():
        if ".experts." in key:
            e = int(key.split(".experts.")[1].split(".")[0])
            if rank * per <= e < (rank + 1) * per:
                state[key.replace(f".experts.{e}.", f".experts.{e - rank * per}.")] = value
        else:
            state[key] = value
    model.load_state_dict(state)
    quantize_model(full, bits, group)
    quantize_model(model, bits, group)  # only this rank's experts
    for layer, (a, b) in enumerate(zip(full.moes(), model.moes())):
        assert torch.equal(a.q_gate_up[rank * per:(rank + 1) * per], b.q_gate_up), layer
    with pytest.raises(ValueError, match="consolidate"):
        save_quantized(model, "/dev/null", {"bits": bits, "group_size": group})
    prompts = torch.randint(0, 64, (2, 5), generator=torch.Generator().manual_seed(9))
    got = FastDecoder(model, torch.device("cpu"), max_batch=2).generate(prompts, 8)
    want = FastDecoder(full, torch.device("cpu"), max_batch=2).generate(prompts, 8)
    assert torch.equal(got, want), (got, want)
    return got.tolist()


@pytest.mark.parametrize("bits,group", [(4, 8), (8, None)])
def test_quantised_expert_parallel_decode_matches_the_single_process_decoder(bits, group):
    results = run_ranks(_case, 2, (bits, group))
    assert results[0] == results[1]
