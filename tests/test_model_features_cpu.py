"""More model semantics on CPU (reference tests: tests/test_quantweave.py, tests/test_model_features.py): the
domain-specialisation loss and its gradient, per-expert profiling, routing statistics only on request, config
validation, the character dataset's document packing, unlimited capacity, the benchmark's exact parameter counts and
the 30B-A1B architecture preset."""

import json

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.models.moe import TopKMoE


def _cfg(**kw):
    base = dict(vocab_size=64, hidden_size=16, layers=2, ffn_size=32, num_experts=4, top_k=2, attention_heads=2,
                max_sequence_length=17, capacity_factor=1.25)
    base.update(kw)
    return QuantaWeaveConfig(**base)


def test_the_domain_loss_is_the_mean_cosine_overlap_of_domain_routing_profiles():
    moe = TopKMoE(_cfg())
    same = torch.tensor([[0.7, 0.1, 0.1, 0.1]] * 4)
    domains = torch.tensor([0, 0, 1, 1])
    assert float(moe._domain_loss(same, domains, 2)) == pytest.approx(1.0)  # identical profiles overlap fully
    apart = torch.tensor([[1.0, 0, 0, 0], [1.0, 0, 0, 0], [0, 0, 1.0, 0], [0, 0, 1.0, 0]])
    assert float(moe._domain_loss(apart, domains, 2)) == pytest.approx(0.0)  # disjoint experts: no overlap
    assert float(moe._domain_loss(apart, torch.zeros(4, dtype=torch.long), 2)) == 0.0  # one domain present
    three = torch.tensor([[1.0, 0, 0, 0], [0, 1.0, 0, 0], [1 / 2 ** 0.5, 1 / 2 ** 0.5, 0, 0]])
    # pairs: (0,1) 0, (0,2) and (1,2) 1/sqrt(2); the mean over ordered pairs
    assert float(moe._domain_loss(three, torch.tensor([0, 1, 2]), 3)) == pytest.approx(2 / 2 ** 0.5 / 3)


def test_the_domain_loss_enters_the_training_loss_and_the_router_gradient():
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(_cfg())
    ids = torch.randint(0, 64, (4, 17), generator=torch.Generator().manual_seed(1))
    domains = torch.tensor([0, 0, 1, 1])
    grads, losses = [], []
    for coef in (0.0, 5.0):
        model.zero_grad()
        model.domain_specialization_coef = coef
        out = model(ids, labels=ids, domain_ids=domains, num_domains=2)
        out["loss"].backward()
        losses.append((float(out["loss"].detach()), float(out["domain_loss"].detach())))
        grads.append(model.moes()[0].router.weight.grad.clone())
    (plain, no_domain), (with_domain, domain) = losses
    assert no_domain == 0.0 and 0 < domain <= 1
    assert with_domain == pytest.approx(plain + 5.0 * domain, rel=1e-5)
    assert not torch.allclose(grads[0], grads[1])


def test_expert_profiling_accumulates_time_for_the_experts_that_ran():
    torch.manual_seed(0)
    moe = TopKMoE(_cfg(capacity_factor=0.0))
    moe.profile_experts = True
    moe.simulated_cost_per_row = 1e-3
    x = torch.randn(1, 12, 16)
    moe(x)
    used = torch.bincount(moe.last_top_indices.reshape(-1), minlength=4)
    seconds = torch.as_tensor(moe.expert_seconds)
    assert (seconds[used > 0] >= 1e-3 * used[used > 0]).all() and (seconds[used == 0] == 0).all()


def test_routing_statistics_are_collected_only_on_request_and_describe_the_batch():
    torch.manual_seed(0)
    moe = TopKMoE(_cfg(capacity_factor=0.0))
    x = torch.randn(1, 10, 16)
    moe(x)
    assert moe.last_stats == {}
    moe.collect_stats = True
    moe(x)
    stats = moe.last_stats
    assert int(stats["expert_assigned"].sum()) == 10 * 2 and int(stats["expert_load"].sum()) == 20
    assert float(stats["importance"].sum()) == pytest.approx(1.0, abs=1e-5)
    assert int(stats["confidence_hist"].sum()) == 10 and 0 < float(stats["entropy_mean"]) <= float(torch.log(
        torch.tensor(4.0)))


@pytest.mark.parametrize("bad", [dict(hidden_size=30, attention_heads=4), dict(top_k=5), dict(num_experts=0),
                                 dict(capacity_factor=-1.0), dict(overflow_policy="keep"), dict(kv_heads=3),
                                 dict(router_temperature=0.0), dict(max_sequence_length=1)])
def test_invalid_configurations_are_rejected(bad):
    with pytest.raises(ValueError):
        _cfg(**bad)


def test_unlimited_capacity_keeps_every_route():
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(_cfg(capacity_factor=0.0))
    out = model(torch.randint(0, 64, (3, 17)))
    assert int(out["dropped_routes"]) == 0 and int(out["overflow_routes"]) == 0


def test_the_character_dataset_packs_documents_instead_of_truncating(tmp_path):
    from quantaweave_b200.data.pipeline import CharacterDataset, CharTokenizer

    data = tmp_path / "d.jsonl"
    rows = ["abcdefghij" * 3, "klmnop" * 2, "qrstuvwxyz"]
    data.write_text("".join(json.dumps({"text": r}) + "\n" for r in rows))
    tok = CharTokenizer.build(rows, 64)
    ds = CharacterDataset(data, tok.vocab, sequence_length=9, limit=None)
    stream = [t for r in rows for t in tok.encode(r) + [tok.eos_id]]  # documents joined with an end token
    assert len(ds) == len(stream) // 10 and len(ds) > 0
    assert torch.equal(ds[0], torch.tensor(stream[:10]))  # the first window crosses into the second document
    short = tmp_path / "s.jsonl"
    short.write_text(json.dumps({"text": "abc"}) + "\n")
    assert len(CharacterDataset(short, tok.vocab, sequence_length=9, limit=None)) == 0


def test_the_benchmark_reports_exact_parameter_counts(tmp_path):
    from test_tools_cpu import _train

    from quantaweave_b200.tools.benchmark import build_parser, run_benchmark
    from quantaweave_b200.utils.hardware import parameter_counts

    data, _ = _train(tmp_path, steps=1)
    report = run_benchmark(build_parser().parse_args(["--checkpoint", str(tmp_path / "out"), "--data", str(data),
                                                      "--examples", "8", "--batch-size", "4", "--device", "cpu"]))
    config = QuantaWeaveConfig.load(tmp_path / "out" / "config.json")
    counts = parameter_counts(config)
    assert report["total_parameters"] == counts["total"]
    assert report["active_parameters_per_token_estimate"] == counts["active"]
    assert report["active_parameter_ratio"] == pytest.approx(counts["active"] / counts["total"])


def test_the_l_preset_is_the_30b_total_1b_active_target():
    from quantaweave_b200.tools.model_scaling import make_spec

    spec = make_spec("moe", "l")
    assert 29e9 < spec.total_params < 32e9 and 0.9e9 < spec.active_params < 1.2e9


def test_every_public_name_resolves():
    import quantaweave_b200 as package

    for name in package.__all__:
        assert getattr(package, name) is not None, name
    assert {"QuantaWeaveBlock", "SparseSwiGLU", "TopKMoE", "load_tokenizer", "add_lora"} <= set(package.__all__)


def test_a_block_takes_the_reference_argument_order():
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(_cfg(capacity_factor=0.0))
    block = model.blocks[0]
    x = torch.randn(2, 5, 16)
    mask = torch.triu(torch.ones(5, 5, dtype=torch.bool), diagonal=1)  # what the reference passes
    with torch.no_grad():
        with_mask = block(x, mask)[0]
        without = block(x)[0]
    assert torch.equal(with_mask, without)
