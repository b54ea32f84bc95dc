"""Expert-parallel decoding on 2 B200s: the native graph-captured step with the NVLink partial-output exchange
(``csrc/ep_decode.cu``) against the single-GPU native decoder over the full model, bf16 and int4 experts.

Both decoders are fed the same tokens (the single-GPU decoder's greedy choices), and every step's logits are compared,
so one rounding difference cannot make the two token streams diverge and hide or fake agreement."""

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


def _case(rank, world, bits):
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.inference.fast_decode import FastDecoder
    from quantaweave_b200.inference.quantization import quantize_model
    from quantaweave_b200.ops import ext
    from quantaweave_b200.parallel.expert_parallel import init_expert_parallel

    torch.cuda.set_device(rank)
    cfg = QuantaWeaveConfig(vocab_size=512, hidden_size=256, layers=3, ffn_size=256, num_experts=8, top_k=2,
                            attention_heads=4, kv_heads=2, max_sequence_length=65, capacity_factor=0.0,
                            norm_type="rmsnorm", position_embedding="rope", attention_bias=False, init_std=0.05)
    torch.manual_seed(0)
    full = QuantaWeaveMoEForCausalLM(cfg).eval()
    ep = init_expert_parallel("cuda", 1, transport="nccl")
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
    if bits:
        quantize_model(full, bits, 128)
        quantize_model(model, bits, 128)  # each rank quantises only the experts it holds
    full, model = full.cuda(), model.cuda()
    batch = 2
    ref = FastDecoder(full, torch.device("cuda"), max_batch=batch)
    dec = FastDecoder(model, torch.device("cuda"), max_batch=batch)
    assert dec.native and dec.uses_graph and dec.ep is not None
    prompts = torch.randint(0, cfg.vocab_size, (batch, 9), generator=torch.Generator().manual_seed(5)).cuda()
    ref._prefill(prompts[:, :-1])
    dec._prefill(prompts[:, :-1])
    token = prompts[:, -1]
    worst = 0.0
    for i in range(12):
        positions = torch.full((batch,), 8 + i, dtype=torch.int32, device="cuda")
        want = ref.run_step(token, positions).clone()
        got = dec.run_step(token, positions).clone()
        scale = float(want.abs().max())
        worst = max(worst, float((got - want).abs().max()) / scale)
        token = want.argmax(-1)  # both decoders are fed the reference's choice
    torch.cuda.synchronize()
    assert ext().read_status(True) == 0
    assert worst < 2e-2, worst
    # every rank computes the same logits (the exchange sums the partials in rank order)
    gathered = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(gathered, got)
    assert all(torch.equal(gathered[0], g) for g in gathered)
    return worst


def _worker(rank, world, port, bits, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QW_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    try:
        queue.put((rank, "ok", _case(rank, world, bits)))
    except Exception:  # noqa: BLE001
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("bits", [0, 4])
def test_expert_parallel_native_decode_matches_single_gpu(bits):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, bits, queue)) for r in range(world)]
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
