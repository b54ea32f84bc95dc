"""A checkpoint in the reference's layout loads unchanged (reference: ``src/quantweave_moe_model.py:51-60, 275-340``
module names; ``src/train_quantweave_moe.py`` checkpoint payload). The checkpoint is written by hand here: a
``config.json`` with only the reference's fourteen fields, a ``model.pt`` payload with per-expert
``experts.{e}.{gate,up,down}.weight`` tensors in ``nn.Linear`` layout, ``nn.MultiheadAttention`` packed projections
and LayerNorms, and a character ``vocab.json`` without tokenizer metadata. The reference's ``model.int{b}.pt``
payload (``src/quantization.py:105-117``: per-expert ``qweight``/``scales`` with fp32 scales) and its LoRA adapter
file (``src/lora.py:86-104``: ``{state, info, base_checkpoint}`` with ``...{proj}.lora_a``/``lora_b``) load too, and
its ``model.rank{r}.pt`` expert- and pipeline-parallel shards (``src/expert_parallel.py:396-544``) consolidate."""

import json

import torch
import torch.nn.functional as F

from quantaweave_b200 import QuantaWeaveConfig
from quantaweave_b200.tools.common import load_model

REFERENCE_CONFIG = dict(vocab_size=40, hidden_size=16, layers=2, ffn_size=24, num_experts=3, top_k=2,
                        attention_heads=2, max_sequence_length=12, router_aux_loss_coef=0.01, capacity_factor=0.0,
                        min_expert_capacity=4, drop_overflow_tokens=True, overflow_policy="drop",
                        router_temperature=1.0)


def _reference_state(cfg: dict) -> dict:
    g = torch.Generator().manual_seed(0)
    H, F_, V, E = cfg["hidden_size"], cfg["ffn_size"], cfg["vocab_size"], cfg["num_experts"]
    r = lambda *shape: 0.1 * torch.randn(*shape, generator=g)  # noqa: E731
    state = {"token_embedding.weight": r(V, H), "position_embedding.weight": r(cfg["max_sequence_length"], H)}
    for layer in range(cfg["layers"]):
        p = f"blocks.{layer}."
        state.update({p + "attention_norm.weight": 1 + r(H), p + "attention_norm.bias": r(H),
                      p + "attention.in_proj_weight": r(3 * H, H), p + "attention.in_proj_bias": r(3 * H),
                      p + "attention.out_proj.weight": r(H, H), p + "attention.out_proj.bias": r(H),
                      p + "moe_norm.weight": 1 + r(H), p + "moe_norm.bias": r(H), p + "moe.router.weight": r(E, H)})
        for e in range(E):
            q = f"{p}moe.experts.{e}."
            state.update({q + "gate.weight": r(F_, H), q + "up.weight": r(F_, H), q + "down.weight": r(H, F_)})
    state.update({"final_norm.weight": 1 + r(H), "final_norm.bias": r(H), "lm_head.weight": r(V, H)})
    return state


def _write(tmp_path):
    state = _reference_state(REFERENCE_CONFIG)
    (tmp_path / "config.json").write_text(json.dumps(REFERENCE_CONFIG))
    vocab = {"<unk>": 0, "<eos>": 1, **{ch: i + 2 for i, ch in enumerate("abcdefghijklmnopqrstuvwxyz .,!?")}}
    (tmp_path / "vocab.json").write_text(json.dumps(vocab))
    torch.save({"model": state, "optimizer": None, "step": 5, "rng_state": {}, "extra": {}}, tmp_path / "model.pt")
    return state


def _layer_norm(x, w, b):
    return F.layer_norm(x, (x.size(-1),), w, b, 1e-5)


@torch.no_grad()
def _reference_forward(state: dict, cfg: dict, ids: torch.Tensor) -> torch.Tensor:
    """The reference architecture restated in plain fp32 PyTorch, without expert capacity (capacity_factor 0)."""
    H, heads, E, k = cfg["hidden_size"], cfg["attention_heads"], cfg["num_experts"], cfg["top_k"]
    T = ids.size(1)
    h = state["token_embedding.weight"][ids] + state["position_embedding.weight"][:T]
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    for layer in range(cfg["layers"]):
        p = f"blocks.{layer}."
        a = _layer_norm(h, state[p + "attention_norm.weight"], state[p + "attention_norm.bias"])
        qkv = a @ state[p + "attention.in_proj_weight"].T + state[p + "attention.in_proj_bias"]
        q, kk, v = (t.view(1, T, heads, H // heads).transpose(1, 2) for t in qkv.split(H, -1))
        scores = (q @ kk.transpose(-1, -2)) / (H // heads) ** 0.5
        o = scores.masked_fill(mask, float("-inf")).softmax(-1) @ v
        o = o.transpose(1, 2).reshape(1, T, H)
        h = h + o @ state[p + "attention.out_proj.weight"].T + state[p + "attention.out_proj.bias"]
        m = _layer_norm(h, state[p + "moe_norm.weight"], state[p + "moe_norm.bias"])[0]
        probs = (m @ state[p + "moe.router.weight"].T).softmax(-1)
        w, idx = probs.topk(k, -1)
        w = w / w.sum(-1, keepdim=True)
        out = torch.zeros_like(m)
        for t in range(T):
            for j in range(k):
                q_ = f"{p}moe.experts.{int(idx[t, j])}."
                x = m[t]
                y = (F.silu(state[q_ + "gate.weight"] @ x) * (state[q_ + "up.weight"] @ x)) @ state[q_ + "down.weight"].T
                out[t] += w[t, j] * y
        h = h + out[None]
    h = _layer_norm(h, state["final_norm.weight"], state["final_norm.bias"])
    return h @ state["lm_head.weight"].T


def test_a_reference_layout_checkpoint_loads_and_computes_the_reference_function(tmp_path):
    state = _write(tmp_path)
    config = QuantaWeaveConfig.load(tmp_path / "config.json")
    assert (config.norm_type, config.position_embedding, config.attention_bias, config.kv_heads) == (
        "layernorm", "learned", True, None)  # the additions default to the reference architecture
    model = load_model(tmp_path, torch.device("cpu")).eval()
    saved = model.state_dict()
    assert saved.keys() == state.keys() and all(torch.equal(saved[k], state[k]) for k in state)  # same key layout
    ids = torch.tensor([[3, 7, 1, 12, 5, 9, 2, 20, 4, 6, 8]])
    with torch.no_grad():
        got = model(ids)["logits"]
    assert torch.allclose(got, _reference_forward(state, REFERENCE_CONFIG, ids), atol=1e-5)


def test_the_chat_loader_reads_a_reference_character_vocabulary(tmp_path):
    from quantaweave_b200.tools.chat import ChatSession, Settings, load_for_chat

    _write(tmp_path)
    model, tokenizer = load_for_chat(tmp_path, None, 0, torch.device("cpu"))
    assert tokenizer.kind == "char" and tokenizer.vocab_size == 33
    reply = ChatSession(model, tokenizer, torch.device("cpu"), "fp32", Settings(temperature=0, tokens=4)).send("ab")
    assert reply.tokens <= 4


def _reference_quantize(weight: torch.Tensor, bits: int, group: int):
    """The reference payload's per-layer encoding, restated: symmetric per-group codes (int8 in [-127, 127]; int4 in
    [-8, 7] stored +8, two per byte, low nibble = even column) with fp32 scales, input padded to the group."""
    out, cols = weight.shape
    padded = -(-cols // group) * group
    grouped = F.pad(weight, (0, padded - cols)).reshape(out, -1, group)
    limit = 127 if bits == 8 else 7
    scales = (grouped.abs().amax(-1) / limit).clamp(min=1e-8)
    codes = torch.round(grouped / scales[..., None]).clamp(-limit - (bits == 4), limit).reshape(out, -1)
    if bits == 8:
        return codes.to(torch.int8), scales
    unsigned = (codes + 8).to(torch.uint8)
    return unsigned[:, 0::2] | (unsigned[:, 1::2] << 4), scales


def _reference_dequantize(q: torch.Tensor, scales: torch.Tensor, bits: int, group: int, cols: int):
    if bits == 8:
        values = q.float()
    else:
        values = torch.stack([(q & 0xF).float() - 8, (q >> 4).float() - 8], -1).reshape(q.size(0), -1)
    return (values.reshape(q.size(0), -1, group) * scales[..., None]).reshape(q.size(0), -1)[:, :cols]


def test_a_reference_quantized_payload_loads_and_dequantizes_to_the_same_weights(tmp_path):
    import pytest

    from quantaweave_b200.inference.quantization import dequantized_expert, load_quantized

    for bits, group in ((8, None), (4, 8)):
        state = _reference_state(REFERENCE_CONFIG)
        expected = {}
        for key in [k for k in state if ".experts." in k]:
            weight = state.pop(key)
            g = group or weight.size(1)  # int8 without a group size: one scale per output row
            q, s = _reference_quantize(weight, bits, g)
            state[key.replace(".weight", ".qweight")], state[key.replace(".weight", ".scales")] = q, s
            expected[key] = _reference_dequantize(q, s, bits, g, weight.size(1))
        payload = {"config": REFERENCE_CONFIG, "bits": bits, "group_size": group, "quantize_lm_head": False,
                   "state_dict": state}
        torch.save(payload, tmp_path / f"model.int{bits}.pt")
        model = load_quantized(tmp_path / f"model.int{bits}.pt")
        for layer, moe in enumerate(model.moes()):
            for e in range(moe.num_local_experts):
                wgu, wd = dequantized_expert(moe, e)
                p = f"blocks.{layer}.moe.experts.{e}."
                want = torch.cat([expected[p + "gate.weight"], expected[p + "up.weight"]])
                # scales are held as fp16 for the decode kernels: a relative difference of at most 2^-11
                assert torch.allclose(wgu, want, rtol=1e-3, atol=1e-6), (bits, p)
                assert torch.allclose(wd, expected[p + "down.weight"], rtol=1e-3, atol=1e-6), (bits, p)
        dense = {k: v for k, v in model.state_dict().items() if ".experts." not in k}
        assert all(torch.equal(dense[k], state[k]) for k in dense if k in state)
        with pytest.raises(Exception):
            load_quantized(tmp_path / "missing.pt")


def test_a_reference_lora_adapter_file_loads_and_merges_to_the_same_weights(tmp_path):
    from quantaweave_b200.tools.lora import add_lora, load_adapter, merge_lora_state

    base = _write(tmp_path)
    rank, alpha = 4, 8.0
    g = torch.Generator().manual_seed(3)
    adapter, merged_want = {}, dict(base)
    for key in [k for k in base if ".experts." in k] + ["lm_head.weight"]:
        out_f, in_f = base[key].shape
        a, b = torch.randn(rank, in_f, generator=g), 0.1 * torch.randn(out_f, rank, generator=g)
        stem = key[: -len(".weight")]
        adapter[stem + ".lora_a"], adapter[stem + ".lora_b"] = a, b  # the reference's per-projection names
        merged_want[key] = base[key] + (alpha / rank) * (b @ a)
    adapter["blocks.0.moe.router.weight"] = base["blocks.0.moe.router.weight"] + 0.5  # an unfrozen router
    merged_want["blocks.0.moe.router.weight"] = adapter["blocks.0.moe.router.weight"]
    info = {"rank": rank, "alpha": alpha, "include_lm_head": True}
    torch.save({"state": adapter, "info": info, "base_checkpoint": str(tmp_path)}, tmp_path / "adapter.pt")
    model = load_model(tmp_path, torch.device("cpu"))
    add_lora(model, rank=rank, alpha=alpha, include_lm_head=True, train_router=True)
    assert load_adapter(model, tmp_path / "adapter.pt") == info
    merged = merge_lora_state(model)
    assert merged.keys() == merged_want.keys()
    for key, want in merged_want.items():
        assert torch.allclose(merged[key], want, atol=1e-5), key


def test_reference_expert_and_pipeline_shards_consolidate_into_the_full_model(tmp_path):
    import re

    from quantaweave_b200.parallel.checkpoint import consolidate_checkpoint
    from quantaweave_b200.utils.checkpoint_io import load_checkpoint

    config = {**REFERENCE_CONFIG, "num_experts": 4}
    full = _reference_state(config)
    expert = re.compile(r"(\.experts\.)(\d+)(\.)")

    def shard(ep_rank, experts, layout):
        state = {}
        for key, value in full.items():
            m = expert.search(key)
            if m is None:
                state[key] = value  # replicated tensors: every rank holds a copy
            elif int(m.group(2)) in experts:  # local expert numbering on each rank
                state[expert.sub(lambda mm: f"{mm.group(1)}{int(mm.group(2)) - experts[0]}{mm.group(3)}", key)] = value
        payload = {"model": state, "optimizer": None, "step": 9, "rng_state": {}, "world_size": 2, "rank": ep_rank,
                   "extra": {"note": "reference"}}
        if layout:
            payload["layout"] = {"kind": "ep", "ep_rank": ep_rank, "ep_size": 2, "tp_rank": 0, "tp_size": 1}
        return payload

    for with_layout in (True, False):  # older reference shards carry no "layout": expert parallelism is assumed
        root = tmp_path / f"ep{int(with_layout)}"
        root.mkdir()
        (root / "config.json").write_text(json.dumps(config))
        for rank, experts in ((0, [0, 1]), (1, [2, 3])):
            torch.save(shard(rank, experts, with_layout), root / f"model.rank{rank}.pt")
        consolidate_checkpoint(root, root / "merged")
        merged = load_checkpoint(root / "merged" / "model.pt")
        assert merged["step"] == 9 and merged["extra"] == {"note": "reference"}
        assert merged["model"].keys() == full.keys()
        assert all(torch.equal(merged["model"][k], full[k]) for k in full)
    pipe = tmp_path / "pp"
    pipe.mkdir()
    block = re.compile(r"^blocks\.(\d+)\.")
    for stage, (start, end) in enumerate(((0, 1), (1, 2))):
        state = {}
        for key, value in full.items():
            m = block.match(key)
            if m and start <= int(m.group(1)) < end:
                state[f"blocks.{int(m.group(1)) - start}." + key[m.end():]] = value
            elif not m and (key.startswith(("token_", "position_")) if stage == 0 else
                             key.startswith(("final_norm", "lm_head"))):
                state[key] = value
        torch.save({"model": state, "optimizer": None, "step": 2, "rng_state": {}, "world_size": 2, "rank": stage,
                    "layout": {"kind": "pp", "stage": stage, "stages": 2, "layer_start": start, "layer_end": end},
                    "extra": {}}, pipe / f"model.rank{stage}.pt")
    consolidate_checkpoint(pipe, pipe / "merged")
    merged = load_checkpoint(pipe / "merged" / "model.pt")["model"]
    assert merged.keys() == full.keys() and all(torch.equal(merged[k], full[k]) for k in full)
