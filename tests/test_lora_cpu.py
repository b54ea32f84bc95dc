"""LoRA / QLoRA on the stacked experts (reference tests: tests/test_lora.py, tests/test_finetune.py)."""

import json
from pathlib import Path

import pytest
import torch

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.inference.quantization import quantize_model
from quantaweave_b200.tools.lora import add_lora, adapter_state, load_adapter, merge_lora_state, save_adapter


def _model(seed=0):
    torch.manual_seed(seed)
    cfg = QuantaWeaveConfig(vocab_size=64, hidden_size=32, layers=2, ffn_size=48, num_experts=4, top_k=2,
                            attention_heads=2, max_sequence_length=17, capacity_factor=8.0)
    return QuantaWeaveMoEForCausalLM(cfg).eval()


def _perturb(model):
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "lora" in name:
                p.add_(0.05 * torch.randn_like(p))


@pytest.mark.parametrize("bits", [0, 8])
def test_adapter_starts_as_noop_and_merges_exactly(bits):
    model = _model()
    if bits:
        quantize_model(model, bits)
    x = torch.randint(0, 64, (2, 16))
    before = model(x)["logits"]
    info = add_lora(model, rank=4, alpha=8.0, include_lm_head=True, train_router=True)
    assert info["wrapped_layers"] == 2 * 4 * 3 + 1
    assert torch.allclose(model(x)["logits"], before, atol=1e-6)
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert all("lora" in n or n.endswith("router.weight") for n in trainable)
    _perturb(model)
    adapted = model(x)["logits"]
    assert not torch.allclose(adapted, before, atol=1e-4)
    merged = merge_lora_state(model)
    assert "blocks.0.moe.experts.3.down.weight" in merged and "lm_head.weight" in merged
    assert not any("lora" in k or k.endswith("qweight") for k in merged)
    plain = _model(seed=1)
    plain.load_state_dict(merged)
    assert torch.allclose(plain(x)["logits"], adapted, atol=1e-4)


def test_adapter_file_round_trip(tmp_path):
    model = _model()
    quantize_model(model, 4, 16)
    info = add_lora(model, rank=2, alpha=4.0)
    _perturb(model)
    state = adapter_state(model)
    assert "blocks.1.moe.experts.2.gate.lora_a" in state and state["blocks.1.moe.experts.2.gate.lora_a"].shape == (2, 32)
    assert state["blocks.1.moe.experts.2.down.lora_b"].shape == (32, 2)
    save_adapter(model, tmp_path / "adapter.pt", info)
    other = _model()
    quantize_model(other, 4, 16)
    add_lora(other, rank=2, alpha=4.0)
    load_adapter(other, tmp_path / "adapter.pt")
    x = torch.randint(0, 64, (1, 16))
    assert torch.equal(other(x)["logits"], model(x)["logits"])
    bad = _model()
    add_lora(bad, rank=2, alpha=4.0, include_lm_head=False)
    torch.save({"state": {"nope.lora_a": torch.zeros(1)}, "info": {}}, tmp_path / "bad.pt")
    with pytest.raises(ValueError, match="unknown tensors"):
        load_adapter(bad, tmp_path / "bad.pt")


def test_finetune_cli_improves_and_reloads(tmp_path):
    from test_tools_cpu import _train

    from quantaweave_b200.tools.finetune import build_parser, evaluate, load_finetuned, run_finetune

    data, _ = _train(tmp_path)
    args = build_parser().parse_args([
        "--checkpoint", str(tmp_path / "out"), "--data", str(data), "--output", str(tmp_path / "qlora"),
        "--merge-output", str(tmp_path / "merged"), "--bits", "4", "--group-size", "16", "--rank", "4",
        "--steps", "15", "--batch-size", "4", "--sequence-length", "32", "--examples", "60", "--lr", "1e-2",
        "--device", "cpu", "--no-archive"])
    meta = run_finetune(args)
    assert meta["loss_after"] < meta["loss_before"]
    assert 0 < meta["trainable_fraction"] < 0.5
    assert json.loads((tmp_path / "qlora" / "finetune_metadata.json").read_text())["rank"] == 4
    model = load_finetuned(tmp_path / "out", tmp_path / "qlora")
    from quantaweave_b200.data.pipeline import WindowDataset, build_corpus, load_tokenizer

    ds = WindowDataset(build_corpus([data], load_tokenizer(tmp_path / "out"), 60), 32)
    assert abs(evaluate(model, ds, torch.device("cpu"), "fp32") - meta["loss_after"]) < 1e-4
    assert (Path(tmp_path / "merged") / "model.pt").exists()
