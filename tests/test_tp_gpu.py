"""Fused tensor-parallel attention on 2 B200s: the GEMM + all-reduce kernels over NVLink peer memory (forward
row-parallel output projection, backward column-parallel input projection) against the NCCL all-reduce path, same
shards, same inputs."""

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
