"""Headline benchmark: MoE training tokens/sec (benchmark configuration 2) on N GPUs of one node.

    python bench.py --gpus 1 --steps 10 --warmup 3
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W
    python bench.py --impl reference ...      # the unmodified reference build, same metric and config

Config 2: vocab 32000, d_model 1024, 16 layers, 16 heads, 64 SwiGLU experts (hidden 2816), top_k 2, capacity 1.25,
aux 0.01, 32 sequences of 2048 (+1 label token) per GPU, Zipf(1.1) token ids from a seeded generator, random init
N(0, 0.02), bf16 compute, AdamW with fp32 master weights. Experts are sharded expert-parallel over the N GPUs.

``value`` is device-timed (CUDA events, barrier + synchronize on both sides, max over ranks) over exactly K full
training steps (forward, backward, gradient clip, optimizer step) with inputs already on the device; ``e2e``
repeats K steps through the public training API with the per-step pinned host->device input copy and the
device->host loss read inside the timed region. Every step touches far more than the 126 MB L2, so no flush is
needed between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
import traceback

os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "MoE train tokens/sec"
BASELINE_VALUE = None  # the reference publishes no tokens/s figure for this config, so vs_baseline is null

CONFIG2 = dict(vocab_size=32000, hidden_size=1024, layers=16, attention_heads=16, num_experts=64, ffn_size=2816,
               top_k=2, capacity_factor=1.25, router_aux_loss_coef=0.01)


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--trace", help="write a chrome trace of one extra (untimed) step to this path (diagnostics)")
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--seqs-per-gpu", type=int, default=32)
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--layers", type=int, default=CONFIG2["layers"], help="debug override (the metric needs 16)")
    p.add_argument("--recompute", choices=("auto", "on", "off"), default="on",
                   help="recompute the expert gate/up activations in backward (on at every N by default, so the "
                        "scaling curve compares steps doing the same work; auto: only with more than 16 local "
                        "experts)")
    p.add_argument("--transport", choices=("auto", "fused", "p2p", "nccl"), default=os.environ.get("QW_EP_TRANSPORT", "auto"),
                   help="expert-parallel exchange: fused (dispatch kernel and expert-GEMM epilogue store rows "
                        "into peers over NVLink), p2p (peer-store exchange of padded buffers), nccl (all_to_all), "
                        "auto (fused on CUDA)")
    p.add_argument("--optimizer-overlap", choices=("on", "off"), default="off",
                   help="run each step's AdamW update on a side stream under the next forward (the timed regions "
                        "wait for the last update before they end). Off by default: measured on one B200 it did not "
                        "help (311.7k vs 314.8k tokens/s), because the persistent GEMM and attention kernels leave "
                        "the update too few SM resources to run beside them")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-launch-count", action="store_true",
                   help="skip the profiler-based launch count (for runs under an external profiler)")
    p.add_argument("--kernel-breakdown", action="store_true",
                   help="after timing, profile one extra step and print per-kernel CUDA time shares to stderr")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def dist_setup(gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # short enough that a rank left waiting on a collective fails within minutes instead of holding the GPUs
        timeout_s = float(os.environ.get("QW_PG_TIMEOUT_S", "180"))
        os.environ["QW_PG_TIMEOUT_S"] = str(timeout_s)
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=torch.device("cuda", local))
    return rank, world, local


def emit(rank: int, record: dict) -> None:
    if rank == 0:
        print(json.dumps(record), flush=True)


def count_launches(step_fn) -> int:
    """Kernels of this framework's extension launched by one step (profiled once, outside the timed region)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours = [n for n in names if "qw::" in n or n.startswith("void qw::")]
    return len(ours)


E2E_D2H = ("every step's loss is copied into pinned host memory without blocking and read on the host once the "
           "next step is queued (the last one before the timer stops)")


def e2e_loop(step_fn, steps: int) -> float:
    """Run ``step_fn(i)`` for ``steps`` steps (each copies its inputs from pinned host memory); every step's loss
    goes device -> pinned host buffer with a non-blocking copy and is read on the host after the next step has been
    queued, as a training loop with asynchronous loss logging does. Returns the last loss."""
    import torch

    slots = [torch.empty(1, dtype=torch.float32).pin_memory() for _ in range(2)]
    pending = None
    value = float("nan")
    for i in range(steps):
        loss = step_fn(i)
        slot = slots[i % 2]
        slot.copy_(loss.detach().float().reshape(1), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record()
        if pending is not None:  # the previous step's loss, read while this step runs
            pending[1].synchronize()
            value = float(pending[0][0])
        pending = (slot, ready)
    if pending is not None:
        pending[1].synchronize()
        value = float(pending[0][0])
    return value


def kernel_breakdown(step_fn, report: bool = True) -> None:
    """Per-kernel CUDA time of one step (shares only; numbers taken under a profiler are never reported)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    if not report:
        return
    totals: dict = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            name = e.name[:110]
            t, n = totals.get(name, (0.0, 0))
            totals[name] = (t + e.device_time_total, n + 1)
    grand = sum(t for t, _ in totals.values()) or 1.0
    print(f"kernel breakdown: {grand / 1e3:.1f} ms of device time in one step", file=sys.stderr)
    for name, (t, n) in sorted(totals.items(), key=lambda kv: -kv[1][0])[:40]:
        print(f"  {100 * t / grand:5.1f}%  {t / 1e3:8.2f} ms  x{n:<5d} {name}", file=sys.stderr)


def save_trace(step_fn, path) -> None:
    """Chrome trace (host + device timeline) of one step, for finding idle gaps; diagnostics only. ``path`` None:
    run the step under the profiler without writing (ranks other than 0)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    if path:
        prof.export_chrome_trace(path)


# ================================================================================================ native arm
def run_native(args, rank, world, local):
    import torch

    sys.path.insert(0, ROOT)
    from quantaweave_b200 import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM
    from quantaweave_b200.data.pipeline import SyntheticTokenStream
    from quantaweave_b200.optim.adamw import FusedAdamW
    from quantaweave_b200.training.native import prepare_model
    from quantaweave_b200.utils.timing import ClockSampler, DeviceTimer

    # the reference's layout (LayerNorm, learned positions, biased MHA projections) so both arms run the same
    # architecture with the same N(0, 0.02) initialisation and therefore the same routing statistics
    cfg = QuantaWeaveConfig(**{**CONFIG2, "layers": args.layers}, max_sequence_length=args.seq_len + 1,
                            norm_type="layernorm", position_embedding="learned", attention_bias=True, init_std=0.02)
    ep = None
    if world > 1:
        from quantaweave_b200.parallel.expert_parallel import init_expert_parallel

        ep = init_expert_parallel("cuda", 1, transport=args.transport)
    torch.manual_seed(args.seed + rank)
    with torch.device("cuda"):
        model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep)
    local_experts = cfg.num_experts // world
    recompute = args.recompute == "on" or (args.recompute == "auto" and local_experts > 16)
    prepare_model(model, "bf16", recompute_experts=recompute)
    if ep is not None:
        from quantaweave_b200.parallel.expert_parallel import broadcast_shared_parameters

        broadcast_shared_parameters(model, ep)
    model.train()
    opt = FusedAdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    if args.optimizer_overlap == "on":  # each step's update runs on a side stream under the next forward
        opt.overlap_with_forward(model)
    stream = SyntheticTokenStream(cfg.vocab_size, args.seq_len, args.seqs_per_gpu, seed=args.seed,
                                  distribution="zipf", zipf_s=1.1, rank=rank, world_size=world)

    from quantaweave_b200.utils.tracing import nvtx_range  # no-ops unless QW_NVTX=1

    def train_step(batch):
        with nvtx_range("forward"):
            out = model(batch, labels=batch, return_logits=False)
        with nvtx_range("backward"):
            out["loss"].backward()
        with nvtx_range("grad_sync"):
            if ep is not None:
                from quantaweave_b200.parallel.expert_parallel import clip_grad_norm_parallel, sync_gradients

                sync_gradients(model, ep, None)
                clip_grad_norm_parallel(model, ep, 1.0, False, opt)
            else:
                opt.clip_grad_norm_(1.0)
        with nvtx_range("optimizer"):
            opt.step()
            opt.zero_grad(set_to_none=True)
        return out["loss"]

    host_batches = [stream.batch(i)[0].pin_memory() for i in range(args.warmup + 2 * args.steps + 1)]
    dev_batches = [b.to("cuda", non_blocking=True) for b in host_batches[: args.warmup + args.steps]]
    for i in range(args.warmup):
        train_step(dev_batches[i])
    torch.cuda.synchronize()
    # ---- device-timed K steps (inputs resident) ----
    with ClockSampler(local) as clocks:
        with DeviceTimer() as t:
            for i in range(args.steps):
                loss = train_step(dev_batches[args.warmup + i])
            opt.finish()  # the last step's update is inside the timed region
    ms_per_step = t.ms / args.steps
    tokens_per_step = args.seqs_per_gpu * args.seq_len * world
    value = tokens_per_step / (ms_per_step / 1000.0)
    final_loss = float(loss.item())
    from quantaweave_b200.ops.status import check_device_status

    check_device_status()  # a kernel that gave up on a bounded wait invalidates the measurement
    with torch.no_grad():
        probe = model(dev_batches[-1], labels=dev_batches[-1], return_logits=False)
        routes = args.seqs_per_gpu * (args.seq_len + 1) * cfg.top_k * args.layers
        overflow_fraction = float(probe["overflow_routes"]) / routes
    del dev_batches
    # ---- end-to-end: pinned H2D of each step's inputs and D2H of its loss inside the timed region ----
    e2e = None
    if not args.no_e2e:
        h2d = host_batches[0].numel() * host_batches[0].element_size()
        with DeviceTimer() as te:
            loss_value = e2e_loop(lambda i: train_step(host_batches[args.warmup + args.steps + i].to(
                "cuda", non_blocking=True)), args.steps)
            opt.finish()
        e2e = {"value": tokens_per_step / (te.ms / args.steps / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": 4 * world, "ms_per_step": te.ms / args.steps,
               "final_loss": loss_value, "d2h": E2E_D2H}
    def step_and_finish(batch):
        loss = train_step(batch)
        opt.finish()
        return loss

    launches = None if args.no_launch_count else count_launches(
        lambda: step_and_finish(host_batches[-1].to("cuda"))) * args.steps
    # every rank runs the profiled steps (they contain collectives); only rank 0 reports
    if args.kernel_breakdown:
        kernel_breakdown(lambda: step_and_finish(host_batches[-1].to("cuda")), report=rank == 0)
    if args.trace:
        save_trace(lambda: step_and_finish(host_batches[-1].to("cuda")), args.trace if rank == 0 else None)
    peak_gb = torch.cuda.max_memory_allocated() / 1e9
    emit(rank, {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
        "data": "synthetic: seeded Zipf(1.1) token ids, random-init N(0,0.02) weights",
        "config": {"model": "moe-1b-e64 (benchmark configuration 2: vocab 32000, d1024, 16 layers, 16 heads, 64 experts "
                            "h2816, top2, cf1.25; reference layout: LayerNorm, learned positions, biased MHA)"
                            if args.layers == 16 else
                            f"DEBUG {args.layers}-layer variant of config 2",
                   "global_batch": args.seqs_per_gpu * world, "seq_len": args.seq_len,
                   "parallelism": f"ep{world}" if world > 1 else "single-gpu (all 64 experts local)",
                   "ep_transport": ep.transport if ep is not None else None,
                   "l2": "no flush: every step streams >100 GB through HBM, far above the 126 MB L2",
                   "recompute_expert_activations": recompute, "optimizer": "fused AdamW, fp32 master, clip 1.0" + (
                       "; each update on a side stream under the next step's forward, joined before the timer stops"
                       if args.optimizer_overlap == "on" else "")},
        "clocks": clocks.summary(), "e2e": e2e, "gpu_launches": launches, "impl": "native",
        "final_loss": final_loss, "peak_mem_gb": round(peak_gb, 1), "overflow_fraction": round(overflow_fraction, 4),
    })


# ================================================================================================ reference arm
REFERENCE_MODULE = "quantweave_moe_model.py"  # the reference's model module; its directory holds all its modules


def _module_dir(path: str):
    return path if path and os.path.isfile(os.path.join(path, REFERENCE_MODULE)) else None


def locate_reference_src(root: str = ROOT, environ=None):
    """Find the directory that holds the unmodified reference's top-level modules.

    The reference is a flat collection of modules (``quantweave_moe_model.py``, ``moe_kernels.py``,
    ``expert_parallel.py``, ...) that import each other by bare name, and its ``pyproject.toml`` declares
    ``py-modules = []``, so a ``pip install --target baseline/_ref`` lays down only a ``*.dist-info`` folder. The
    modules are therefore looked up, in order, at:

    1. ``$QW_REFERENCE_SRC`` (an explicit override);
    2. any directory under ``baseline/_ref`` (four levels deep at most) that contains the model module;
    3. the source tree recorded by the install: ``direct_url.json`` of each ``baseline/_ref/*.dist-info`` holds a
       ``file://`` URL of the installed project, whose ``src/`` (or root) holds the modules;
    4. the current import path (a ``PYTHONPATH`` that already exposes the modules).

    Returns ``(directory or None, searched)``; ``searched`` lists every place looked at, for the error line.
    """
    import glob
    import importlib.util
    from urllib.parse import unquote, urlparse

    environ = os.environ if environ is None else environ
    searched = []
    explicit = environ.get("QW_REFERENCE_SRC")
    if explicit:
        searched.append(f"$QW_REFERENCE_SRC={explicit}")
        if _module_dir(explicit):
            return explicit, searched
    base = os.path.join(root, "baseline", "_ref")
    searched.append(f"{base}/**/{REFERENCE_MODULE}")
    if os.path.isdir(base):
        for dirpath, dirnames, filenames in os.walk(base):
            depth = dirpath[len(base):].count(os.sep)
            dirnames[:] = sorted(d for d in dirnames if not d.startswith(".") and d != "__pycache__") if depth < 4 else []
            if REFERENCE_MODULE in filenames:
                return dirpath, searched
        for info in sorted(glob.glob(os.path.join(base, "*.dist-info", "direct_url.json"))):
            try:
                with open(info) as f:
                    url = json.load(f).get("url", "")
            except (OSError, ValueError):
                searched.append(f"{info} (unreadable)")
                continue
            parsed = urlparse(url)
            if parsed.scheme != "file":
                searched.append(f"{info}: {url} (not a local path)")
                continue
            project = unquote(parsed.path)
            for candidate in (os.path.join(project, "src"), project):
                searched.append(f"{candidate} (from {os.path.relpath(info, root)})")
                if _module_dir(candidate):
                    return candidate, searched
    spec = importlib.util.find_spec(REFERENCE_MODULE[:-3])
    searched.append("sys.path")
    if spec is not None and spec.origin:
        return os.path.dirname(spec.origin), searched
    return None, searched


def _listing(path: str, limit: int = 12) -> str:
    if not os.path.isdir(path):
        return f"{os.path.relpath(path, ROOT)} does not exist"
    names = sorted(os.listdir(path))
    more = f" (+{len(names) - limit} more)" if len(names) > limit else ""
    return f"{os.path.relpath(path, ROOT)}: [{', '.join(names[:limit])}]{more}"


def run_reference(args, rank, world, local):
    import torch

    ref_src, searched = locate_reference_src()
    if ref_src is None:
        emit(rank, {"impl": "reference",
                    "unavailable": f"reference modules not found; searched {'; '.join(searched)}; "
                                   f"{_listing(os.path.join(ROOT, 'baseline', '_ref'))}"})
        return
    sys.path.insert(0, ref_src)
    from quantweave_moe_model import QuantaWeaveConfig, QuantaWeaveMoEForCausalLM  # the reference's own modules

    sys.path.insert(0, ROOT)
    from quantaweave_b200.data.pipeline import SyntheticTokenStream
    from quantaweave_b200.utils.timing import ClockSampler, DeviceTimer

    cfg = QuantaWeaveConfig(vocab_size=CONFIG2["vocab_size"], hidden_size=CONFIG2["hidden_size"], layers=args.layers,
                            ffn_size=CONFIG2["ffn_size"], num_experts=CONFIG2["num_experts"], top_k=CONFIG2["top_k"],
                            attention_heads=CONFIG2["attention_heads"], max_sequence_length=args.seq_len + 1,
                            router_aux_loss_coef=CONFIG2["router_aux_loss_coef"],
                            capacity_factor=CONFIG2["capacity_factor"])
    device = torch.device("cuda", local)
    ep = None
    if world > 1:
        from expert_parallel import init_expert_parallel, broadcast_shared_parameters

        ep = init_expert_parallel("cuda", 1)
    torch.manual_seed(args.seed + rank)
    try:
        model = QuantaWeaveMoEForCausalLM(cfg, expert_parallel=ep).to(device)
        with torch.no_grad():  # the config's N(0, 0.02) initialisation, applied through the public module tree
            for name, param in model.named_parameters():
                if param.dim() >= 2:
                    param.normal_(0.0, 0.02)
        if ep is not None:
            broadcast_shared_parameters(model, ep)
        kernel = "loop"
        if ep is None:
            from moe_kernels import kernels_available

            if kernels_available(device):
                kernel = model.set_moe_kernel("triton")
        optimizer = torch.optim.AdamW(model.parameters(), lr=3e-4)
        stream = SyntheticTokenStream(cfg.vocab_size, args.seq_len, args.seqs_per_gpu, seed=args.seed,
                                      distribution="zipf", zipf_s=1.1, rank=rank, world_size=world)
        model.train()

        def train_step(batch):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(batch, labels=batch)
            loss = out["loss"]
            loss.backward()
            if ep is not None:
                from expert_parallel import clip_grad_norm_parallel, sync_gradients

                sync_gradients(model, ep, None)
                clip_grad_norm_parallel(model, ep, 1.0, False)
            else:
                torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            optimizer.step()
            optimizer.zero_grad(set_to_none=True)
            return loss

        host = [stream.batch(i)[0].pin_memory() for i in range(args.warmup + 2 * args.steps)]
        dev = [b.to(device) for b in host[: args.warmup + args.steps]]
        for i in range(args.warmup):
            train_step(dev[i])
        with ClockSampler(local) as clocks:
            with DeviceTimer() as t:
                for i in range(args.steps):
                    loss = train_step(dev[args.warmup + i])
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            probe = model(dev[-1], labels=dev[-1])
        overflow_fraction = float(probe["overflow_routes"]) / (args.seqs_per_gpu * (args.seq_len + 1) * cfg.top_k
                                                               * args.layers)
        del dev, probe
        tokens = args.seqs_per_gpu * args.seq_len * world
        ms = t.ms / args.steps
        e2e = None
        if not args.no_e2e:  # the same loop as the native arm's
            with DeviceTimer() as te:
                e2e_loop(lambda i: train_step(host[args.warmup + args.steps + i].to(device, non_blocking=True)),
                         args.steps)
            e2e = {"value": tokens / (te.ms / args.steps / 1000.0), "unit": "tokens/s",
                   "h2d_bytes_per_step": host[0].numel() * host[0].element_size() * world,
                   "d2h_bytes_per_step": 4 * world, "d2h": E2E_D2H}
        emit(rank, {"metric": METRIC, "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "impl": "reference",
                    "data": "synthetic: seeded Zipf(1.1) token ids, random-init N(0,0.02) weights",
                    "reference_src": os.path.relpath(ref_src, ROOT),
                    "config": {"model": "reference architecture at config-2 shape (LayerNorm, learned positions, MHA)",
                               "global_batch": args.seqs_per_gpu * world, "seq_len": args.seq_len,
                               "parallelism": f"ep{world}" if world > 1 else "single-gpu",
                               "moe_kernel": kernel},
                    "clocks": clocks.summary(), "e2e": e2e, "final_loss": float(loss.item()),
                    "overflow_fraction": round(overflow_fraction, 4),
                    "peak_mem_gb": round(torch.cuda.max_memory_allocated() / 1e9, 1)})
    except torch.OutOfMemoryError as exc:
        emit(rank, {"impl": "reference", "unavailable": f"out of memory on B200 at config 2: {str(exc)[:160]}"})


def main():
    args = parse()
    try:
        rank, world, local = dist_setup(args.gpus)
    except SystemExit:
        raise
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, local)
        else:
            run_native(args, rank, world, local)
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    try:
        main()
    except Exception:  # noqa: BLE001
        traceback.print_exc()
        sys.exit(1)
