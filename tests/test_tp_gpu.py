"""Tensor parallelism on 2 B200s.

* Fused tensor-parallel attention: the GEMM + all-reduce kernels over NVLink peer memory (forward row-parallel output
  projection, backward column-parallel input projection) against the NCCL all-reduce path, same shards, same inputs.
* Sequence parallelism (attention TP and experts EP over the same GPUs) on the native kernels against the single-GPU
  model."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import cuda_ready

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ready() or torch.cuda.device_count() < 2, reason="needs 2 B200s")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(rank, world):
    from quantaweave_b200 import QuantaWeaveConfig
    from quantaweave_b200.models.layers import Attention
    from quantaweave_b200.ops import ext
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel
    from quantaweave_b200.parallel.tensor_parallel import FusedTPReducer, TensorParallelAttention, shard_state_dict

    torch.cuda.set_device(rank)
    ep = init_expert_parallel("cuda", world)
    cfg = QuantaWeaveConfig(vocab_size=64, hidden_size=256, layers=1, ffn_size=256, num_experts=4, top_k=1,
                            attention_heads=4, kv_heads=2, max_sequence_length=129, norm_type="rmsnorm",
                            position_embedding="rope", attention_bias=True, init_std=0.02)
    torch.manual_seed(1)
    ref = Attention(cfg)
    tp = TensorParallelAttention(cfg, ep)
    full_state = {f"blocks.0.attention.{k}": v for k, v in ref.state_dict().items()}
    with torch.no_grad():  # a non-zero output bias, so its fused addition is exercised
        full_state["blocks.0.attention.out_proj.bias"] = torch.randn(256) * 0.1
    shard = shard_state_dict(full_state, ep.tp_rank, ep.tp_size, cfg)
    tp.load_state_dict({k.replace("blocks.0.attention.", ""): v for k, v in shard.items()}, strict=False)
    tp = tp.cuda()
    x = torch.randn(2, 128, 256, generator=torch.Generator().manual_seed(3)).cuda()
    g = torch.randn(2, 128, 256, generator=torch.Generator().manual_seed(4)).cuda()
    results = {}
    for fused in ("1", "0"):
        os.environ["QW_TP_FUSED"] = fused
        tp.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_()
        y = tp(xi)
        (y.float() * g).sum().backward()
        results[fused] = (y.float(), xi.grad.float(), {n: p.grad.float() for n, p in tp.named_parameters()})
    assert FusedTPReducer._instances, "the fused path did not run"
    torch.cuda.synchronize()

    def rel(a, b):
        return float((a - b).norm() / (b.norm() + 1e-12))

    y1, dx1, gr1 = results["1"]
    y0, dx0, gr0 = results["0"]
    assert rel(y1, y0) < 1e-2, rel(y1, y0)
    assert rel(dx1, dx0) < 1e-2, rel(dx1, dx0)
    for name, value in gr0.items():
        assert rel(gr1[name], value) < 2e-2, (name, rel(gr1[name], value))
    # every rank holds the same reduced output
    gathered = [torch.empty_like(y1) for _ in range(world)]
    dist.all_gather(gathered, y1.contiguous(), group=ep.tp_group)
    assert torch.equal(gathered[0], gathered[1])
    assert ext().read_status(True) == 0
    return rel(y1, y0)


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    try:
        queue.put((rank, "ok", _case(rank, world)))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_fused_tensor_parallel_attention_matches_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for _ in range(world):
        rank, status, payload = queue.get(timeout=600)
        if status != "ok":
            for p in procs:
                p.join(timeout=30)
            raise AssertionError(f"rank {rank} failed:\n{payload}")
    for p in procs:
        p.join(timeout=60)


def _sp_case(rank, world):
    """Sequence parallelism on the native kernels: attention TP and experts EP over the same 2 GPUs."""
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.ops import ext
    from quantaweave_b200.parallel.expert_parallel import clip_grad_norm_parallel, init_expert_parallel, sync_gradients
    from quantaweave_b200.parallel.tensor_parallel import is_tp_sharded_shared, shard_state_dict, shard_tensor
    from quantaweave_b200.training.native import prepare_model

    torch.cuda.set_device(rank)
    cfg = QuantaWeaveConfig(vocab_size=512, hidden_size=256, layers=2, ffn_size=256, num_experts=8, top_k=2,
                            attention_heads=4, kv_heads=2, max_sequence_length=129, capacity_factor=0.0,
                            router_aux_loss_coef=0.0, norm_type="rmsnorm", position_embedding="rope",
                            attention_bias=False, init_std=0.02)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg).cuda()
    prepare_model(full, "bf16")
    ctx = init_expert_parallel("cuda", world, sequence_parallel=True)
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ctx).cuda()
    prepare_model(model, "bf16")
    per = cfg.num_experts // world
    full_state = full.state_dict()
    attention = {k: v for k, v in full_state.items() if is_tp_sharded_shared(k)}
    state = shard_state_dict(attention, rank, world, cfg)
    for key, value in full_state.items():
        if key in attention:
            continue
        if ".experts." in key:
            e = int(key.split(".experts.")[1].split(".")[0])
            if rank * per <= e < (rank + 1) * per:
                state[key.replace(f".experts.{e}.", f".experts.{e - rank * per}.")] = value
        else:
            state[key] = value
    model.load_state_dict(state)
    batch = torch.randint(0, cfg.vocab_size, (2, 129), generator=torch.Generator().manual_seed(1)).cuda()
    out = model(batch, labels=batch, return_logits=False)
    out["loss"].backward()
    sync_gradients(model, ctx)
    norm = float(clip_grad_norm_parallel(model, ctx, 1e9))
    loss = out["loss"].detach().float().clone()
    dist.all_reduce(loss)
    ref = full(batch, labels=batch, return_logits=False)
    ref["loss"].backward()
    ref_norm = float(torch.sqrt(sum(p.grad.double().pow(2).sum() for p in full.parameters())))
    assert abs(float(loss) / world - float(ref["loss"])) < 2e-2, (float(loss) / world, float(ref["loss"]))
    assert abs(norm - ref_norm) < 5e-2 * ref_norm, (norm, ref_norm)
    qf = cfg.attention_heads / (cfg.attention_heads + 2 * cfg.num_kv_heads)
    ref_grads = {n: p.grad.float() for n, p in full.named_parameters()}
    # expert and router gradients also move with the few near-tie top-2 decisions that flip between the sharded and
    # the single-GPU model (bf16 activations reduced in a different order): up to 0.25 observed (identical for the
    # fused and the NCCL exchange), 0.35 allowed; a sharding or reduction bug moves a gradient by ~0.5-1.4. Every
    # other matrix within 0.1, and the median of all within 0.05.
    rels = []
    for name, p in model.named_parameters():
        expect = ref_grads[name]
        expert = name.endswith(("w_gate_up", "w_down"))
        if expert:
            expect = expect[rank * per:(rank + 1) * per]
        elif is_tp_sharded_shared(name):
            expect = shard_tensor(name, expect, rank, world, qf)
        rel = float((p.grad.float() - expect).norm() / (expect.norm() + 1e-12))
        rels.append(rel)
        routing = expert or name.endswith("router.weight")
        assert rel < (0.35 if routing else 0.1 if p.dim() >= 2 else 0.3), (name, rel)
    assert sorted(rels)[len(rels) // 2] < 0.05, rels
    assert ext().read_status(True) == 0
    return float(loss)


def _sp_worker(rank, world, port, queue, fused):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1", QW_TP_FUSED=fused)
    try:
        queue.put((rank, "ok", _sp_case(rank, world)))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("fused", ["1", "0"])
def test_sequence_parallel_native_matches_single_gpu(fused):
    """fused "1": row all-gather by NVLink peer stores and reduce-scatter inside the projection GEMMs; "0": NCCL."""
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, queue, fused)) for r in range(world)]
    for p in procs:
        p.start()
    for _ in range(world):
        rank, status, payload = queue.get(timeout=600)
        if status != "ok":
            for p in procs:
                p.join(timeout=30)
            raise AssertionError(f"rank {rank} failed:\n{payload}")
    for p in procs:
        p.join(timeout=60)


def _grid_case(rank, world):
    """The EP x TP grid at tensor-parallel 2 on the native kernels: attention heads and every expert's F dimension
    split over the two GPUs (one expert-parallel rank), against the single-GPU model with the full weights."""
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.ops import ext
    from quantaweave_b200.parallel.expert_parallel import clip_grad_norm_parallel, init_expert_parallel, sync_gradients
    from quantaweave_b200.parallel.tensor_parallel import is_tp_sharded, shard_state_dict, shard_tensor
    from quantaweave_b200.training.native import prepare_model

    torch.cuda.set_device(rank)
    cfg = QuantaWeaveConfig(vocab_size=512, hidden_size=256, layers=2, ffn_size=512, num_experts=4, top_k=2,
                            attention_heads=4, kv_heads=2, max_sequence_length=129, capacity_factor=1.25,
                            norm_type="rmsnorm", position_embedding="rope", attention_bias=False, init_std=0.02)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg).cuda()
    prepare_model(full, "bf16")
    ctx = init_expert_parallel("cuda", world)  # tensor-parallel over both ranks, expert-parallel size 1
    model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ctx).cuda()
    prepare_model(model, "bf16")
    model.load_state_dict(shard_state_dict(full.state_dict(), ctx.tp_rank, ctx.tp_size, cfg))
    batch = torch.randint(0, cfg.vocab_size, (2, 129), generator=torch.Generator().manual_seed(1)).cuda()
    out = model(batch, labels=batch, return_logits=False)
    out["loss"].backward()
    sync_gradients(model, ctx)
    norm = float(clip_grad_norm_parallel(model, ctx, 1e9))
    ref = full(batch, labels=batch, return_logits=False)
    ref["loss"].backward()
    ref_norm = float(torch.sqrt(sum(p.grad.double().pow(2).sum() for p in full.parameters())))
    assert abs(float(out["loss"]) - float(ref["loss"])) < 2e-2, (float(out["loss"]), float(ref["loss"]))
    assert abs(norm - ref_norm) < 5e-2 * ref_norm, (norm, ref_norm)
    qf = cfg.attention_heads / (cfg.attention_heads + 2 * cfg.num_kv_heads)
    full_grads = {}
    for name, p in full.named_parameters():  # expert stacks -> per-expert keys so they slice like the checkpoint
        if name.endswith("w_gate_up"):
            f = cfg.ffn_size
            for e in range(cfg.num_experts):
                full_grads[name.replace("w_gate_up", f"experts.{e}.gate.weight")] = p.grad[e, :f].float()
                full_grads[name.replace("w_gate_up", f"experts.{e}.up.weight")] = p.grad[e, f:].float()
        elif name.endswith("w_down"):
            for e in range(cfg.num_experts):
                full_grads[name.replace("w_down", f"experts.{e}.down.weight")] = p.grad[e].float()
        else:
            full_grads[name] = p.grad.float()
    for name, p in model.named_parameters():
        if name.endswith(("w_gate_up", "w_down")):
            f = cfg.ffn_size // world
            for e in range(cfg.num_experts):
                if name.endswith("w_gate_up"):
                    pieces = {"gate": p.grad[e, :f], "up": p.grad[e, f:]}
                else:
                    pieces = {"down": p.grad[e]}
                for proj, got in pieces.items():
                    key = name.replace("w_gate_up" if proj != "down" else "w_down", f"experts.{e}.{proj}.weight")
                    expect = shard_tensor(key, full_grads[key], rank, world, qf)
                    rel = float((got.float() - expect).norm() / (expect.norm() + 1e-12))
                    assert rel < 0.2, (key, rel)  # routing flips between the two models: see _sp_case
            continue
        expect = full_grads[name]
        if is_tp_sharded(name):
            expect = shard_tensor(name, expect, rank, world, qf)
        rel = float((p.grad.float() - expect).norm() / (expect.norm() + 1e-12))
        assert rel < (0.1 if p.dim() >= 2 else 0.3), (name, rel)
    assert ext().read_status(True) == 0
    return float(out["loss"])


def _grid_worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    try:
        queue.put((rank, "ok", _grid_case(rank, world)))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tensor_parallel_experts_on_the_grid_match_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_grid_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for _ in range(world):
        rank, status, payload = queue.get(timeout=600)
        if status != "ok":
            for p in procs:
                p.join(timeout=30)
            raise AssertionError(f"rank {rank} failed:\n{payload}")
    for p in procs:
        p.join(timeout=60)
