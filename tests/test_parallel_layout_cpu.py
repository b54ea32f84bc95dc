"""Sharding layouts and multi-process training on CPU (reference tests: tests/test_parallelism.py,
tests/test_expert_parallel.py): tensor-parallel slicing round trips, divisibility checks, pipeline layer
partitioning, the launcher-environment requirement, consolidation renumbering experts and validating the shard set,
and 2-rank gloo training that resumes exactly, keeps replicated weights identical and, with the sharded optimizer,
trains like the unsharded one while holding less state per rank."""

import pytest
import torch
import torch.distributed as dist

from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
from quantaweave_b200.parallel.checkpoint import consolidate_checkpoint, reshard_checkpoint, shard_path
from quantaweave_b200.parallel.tensor_parallel import merge_state_dicts, shard_state_dict
from quantaweave_b200.utils.checkpoint_io import load_checkpoint

from test_parallel_cpu import _trainer_case, run_ranks


def _config(**kw):
    base = dict(vocab_size=64, hidden_size=32, layers=2, ffn_size=32, num_experts=4, top_k=2, attention_heads=4,
                max_sequence_length=17, norm_type="rmsnorm", position_embedding="rope", attention_bias=False)
    base.update(kw)
    return QuantaWeaveConfig(**base)


@pytest.mark.parametrize("tp,extra", [(2, {}), (4, {}), (2, dict(kv_heads=2)),
                                      (2, dict(attention_bias=True, norm_type="layernorm"))])
def test_tensor_parallel_slices_merge_back_to_the_full_state(tp, extra):
    config = _config(**extra)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(config).state_dict()
    shards = [shard_state_dict(full, r, tp, config) for r in range(tp)]
    q = shards[0]["blocks.0.attention.in_proj_weight"]
    assert q.size(0) * tp == full["blocks.0.attention.in_proj_weight"].size(0)
    merged = merge_state_dicts(shards, config)
    assert merged.keys() == full.keys()
    for key in full:
        assert torch.equal(merged[key], full[key]), key


def _saved(tmp_path, **kw):
    from quantaweave_b200.training.trainer import save_checkpoint

    config = _config(**kw)
    torch.manual_seed(0)
    model = QuantaWeaveMoEForCausalLM(config)
    save_checkpoint(tmp_path / "full", model, torch.optim.AdamW(model.parameters()), 3, {"a": 0}, torch.device("cpu"))
    return model


def test_resharding_needs_divisible_experts_and_heads(tmp_path):
    _saved(tmp_path)
    with pytest.raises(ValueError, match="divisible"):
        reshard_checkpoint(tmp_path / "full", tmp_path / "x", ep_size=3)
    with pytest.raises(ValueError, match="divisible"):
        reshard_checkpoint(tmp_path / "full", tmp_path / "y", ep_size=1, tp_size=3)


def test_consolidation_renumbers_experts_and_validates_the_shard_set(tmp_path):
    model = _saved(tmp_path)
    info = reshard_checkpoint(tmp_path / "full", tmp_path / "shards", ep_size=2)
    assert info["per_rank_experts"] == 2
    rank1 = load_checkpoint(shard_path(tmp_path / "shards", 1))["model"]
    assert torch.equal(rank1["blocks.0.moe.experts.0.down.weight"],
                       model.state_dict()["blocks.0.moe.experts.2.down.weight"])  # local expert 0 is global 2
    consolidate_checkpoint(tmp_path / "shards", tmp_path / "merged")
    merged = load_checkpoint(tmp_path / "merged" / "model.pt")
    assert merged["step"] == 3
    for key, value in model.state_dict().items():
        assert torch.equal(merged["model"][key], value), key
    shard_path(tmp_path / "shards", 1).unlink()
    with pytest.raises(ValueError, match="expected 2 shards"):
        consolidate_checkpoint(tmp_path / "shards", tmp_path / "again")
    with pytest.raises(FileNotFoundError):
        consolidate_checkpoint(tmp_path / "nothing", tmp_path / "again")


def test_layers_are_partitioned_into_contiguous_balanced_stages():
    from quantaweave_b200.parallel.pipeline_parallel import partition_layers

    assert partition_layers(5, 2) == [(0, 3), (3, 5)]
    assert partition_layers(4, 4) == [(0, 1), (1, 2), (2, 3), (3, 4)]
    assert partition_layers(7, 3) == [(0, 3), (3, 5), (5, 7)]
    for bad in ((2, 3), (4, 0)):
        with pytest.raises(ValueError):
            partition_layers(*bad)


def test_multi_process_parallelism_needs_the_launcher_environment(monkeypatch):
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel

    assert not dist.is_initialized()
    for name in ("RANK", "WORLD_SIZE"):
        monkeypatch.delenv(name, raising=False)
    with pytest.raises(RuntimeError, match="torchrun"):
        init_expert_parallel("cpu")


def _weights(path):
    return load_checkpoint(path)["model"]


def test_expert_parallel_training_resumes_exactly_and_keeps_replicated_weights_identical(tmp_path):
    run_ranks(_trainer_case, 2, (str(tmp_path / "straight"), 4))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 2))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 4))  # resumes from the step-2 shards
    a = _weights(tmp_path / "straight" / "out" / "model.pt")
    b = _weights(tmp_path / "split" / "out" / "model.pt")
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)
    r0 = _weights(shard_path(tmp_path / "straight" / "out" / "shards", 0))
    r1 = _weights(shard_path(tmp_path / "straight" / "out" / "shards", 1))
    shared = [k for k in r0 if ".experts." not in k]
    assert shared and all(torch.equal(r0[k], r1[k]) for k in shared)
    assert not torch.equal(r0["blocks.0.moe.experts.0.down.weight"], r1["blocks.0.moe.experts.0.down.weight"])


def test_the_sharded_optimizer_trains_like_adamw_and_holds_less_state_per_rank(tmp_path):
    run_ranks(_trainer_case, 2, (str(tmp_path / "plain"), 3))
    run_ranks(_trainer_case, 2, (str(tmp_path / "zero"), 3, {"shard_optimizer": True}))
    a = _weights(tmp_path / "plain" / "out" / "model.pt")
    b = _weights(tmp_path / "zero" / "out" / "model.pt")
    for key in a:
        assert torch.allclose(a[key], b[key], atol=1e-5), key

    def state_numel(path):
        state = load_checkpoint(path)["optimizer"]
        tensors = []

        def walk(obj):
            if isinstance(obj, torch.Tensor):
                tensors.append(obj.numel())
            elif isinstance(obj, dict):
                for v in obj.values():
                    walk(v)
            elif isinstance(obj, (list, tuple)):
                for v in obj:
                    walk(v)

        walk(state)
        return sum(tensors)

    plain = state_numel(shard_path(tmp_path / "plain" / "ckpt", 0))
    zero = state_numel(shard_path(tmp_path / "zero" / "ckpt", 0))
    assert 0 < zero < plain


def test_pipeline_training_resumes_exactly_and_consolidates(tmp_path):
    extra = {"pipeline_parallel": True, "expert_parallel": False, "microbatches": 2}
    run_ranks(_trainer_case, 2, (str(tmp_path / "straight"), 4, extra))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 2, extra))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 4, extra))
    a = _weights(tmp_path / "straight" / "out" / "model.pt")
    b = _weights(tmp_path / "split" / "out" / "model.pt")
    assert all(torch.equal(a[k], b[k]) for k in a)
    config = QuantaWeaveConfig.load(tmp_path / "straight" / "out" / "config.json")
    QuantaWeaveMoEForCausalLM(config).load_state_dict(a)  # every layer, one plain model


def test_the_pipeline_engine_checks_its_schedule_and_micro_batches():
    from quantaweave_b200.parallel.pipeline_parallel import PipelineContext, PipelineEngine

    ctx = PipelineContext(0, 1, torch.device("cpu"), 0, 2, False, 0, 1, None, None)
    model = QuantaWeaveMoEForCausalLM(_config())
    with pytest.raises(ValueError, match="schedule"):
        PipelineEngine(model, ctx, 2, schedule="zigzag")
    with pytest.raises(ValueError, match="microbatches"):
        PipelineEngine(model, ctx, 0)


def test_1f1b_training_runs_repeated_steps_and_resumes_exactly(tmp_path):
    extra = {"pipeline_parallel": True, "expert_parallel": False, "microbatches": 2, "pipeline_schedule": "1f1b"}
    run_ranks(_trainer_case, 2, (str(tmp_path / "straight"), 5, extra))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 2, extra))
    run_ranks(_trainer_case, 2, (str(tmp_path / "split"), 5, extra))
    a = _weights(tmp_path / "straight" / "out" / "model.pt")
    b = _weights(tmp_path / "split" / "out" / "model.pt")
    assert all(torch.equal(a[k], b[k]) for k in a)
