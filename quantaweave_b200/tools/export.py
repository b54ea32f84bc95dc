"""Export a checkpoint as a self-contained inference bundle.

    python -m quantaweave_b200.tools.export --checkpoint artifacts/outputs/quantweave-moe-out \\
        --output artifacts/exports/moe --quantize 8 --benchmark-data data/smoke/tinystories.jsonl

Bundle parity with the reference ``src/export_quantweave.py`` (``LogitsOnly`` :30, ``try_onnx`` :60-103,
``export_bundle`` :106-182, ``load_exported`` :185): a traced TorchScript graph with dynamic batch and sequence
(``model.torchscript.pt`` + ``model.graph.txt``), an optional ONNX file (``--onnx``), an optional int8/int4 weight-only
copy with its logit cosine, the tokenizer and config, and ``export_metadata.json`` (sizes, sha256, numerical parity,
optional benchmark). The exported graph evaluates every expert densely with router weights (no capacity, no
data-dependent control flow): it is for portability and correctness, not sparse speed. The trace runs the fp32
PyTorch path on the CPU; the sm_100a kernels are not part of the exported artefact.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import shutil
from pathlib import Path
from typing import Optional

import torch
from torch import nn


class LogitsOnly(nn.Module):
    def __init__(self, model) -> None:
        super().__init__()
        self.model = model

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids)["logits"]


def sha256(path: Path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as fh:
        while block := fh.read(1 << 20):
            h.update(block)
    return h.hexdigest()


def load_checkpoint_model(checkpoint: Path):
    from ..models.model import QuantaWeaveMoEForCausalLM
    from ..utils.checkpoint_io import load_checkpoint
    from .common import read_config

    state = load_checkpoint(Path(checkpoint) / "model.pt", map_location="cpu")
    model = QuantaWeaveMoEForCausalLM(read_config(checkpoint))
    model.load_state_dict(state["model"])
    return model.eval(), state


def parity_shapes(config) -> list[tuple[int, int]]:
    longest = config.max_sequence_length
    return [(1, longest), (3, max(2, longest // 2)), (2, 2)]


def try_onnx(wrapper: LogitsOnly, example: torch.Tensor, path: Path, max_sequence_length: int) -> dict:
    """ONNX through the ``torch.export`` exporter with dynamic batch/sequence dims, round-tripped through
    onnxruntime at a second shape when available. The trace uses batch 2: a traced dimension of size 1 is treated
    as static by ``torch.export``."""
    try:
        import onnx  # noqa: F401
    except ImportError:
        return {"status": "skipped", "reason": "the `onnx` package is not installed"}
    try:
        sample = example if example.size(0) != 1 else example.expand(2, -1).contiguous()
        dims = {0: torch.export.Dim("batch"), 1: torch.export.Dim("sequence", max=max_sequence_length)}
        torch.onnx.export(wrapper, (sample,), str(path), input_names=["input_ids"], output_names=["logits"],
                          dynamic_shapes={"input_ids": dims}, dynamo=True)
    except Exception as error:  # noqa: BLE001 - exporter failures are reported, not fatal
        path.unlink(missing_ok=True)
        return {"status": "failed", "reason": f"{type(error).__name__}: {error}"[:300]}
    result = {"status": "ok", "file": path.name}
    try:
        import onnxruntime as ort

        session = ort.InferenceSession(str(path), providers=["CPUExecutionProvider"])
        probe = torch.randint(0, wrapper.model.config.vocab_size,
                              (example.size(0) + 1, min(max_sequence_length, example.size(1) + 3)))
        with torch.inference_mode():
            expected = wrapper(probe)
        actual = torch.from_numpy(session.run(None, {"input_ids": probe.numpy()})[0])
        result.update(dynamic_shape_verified=True, verified_max_abs_diff=float((actual - expected).abs().max()))
    except ImportError:
        result.update(dynamic_shape_verified=False,
                      note="onnxruntime is not installed; the export was not round-tripped at another shape")
    return result


def export_bundle(checkpoint: Path, output: Path, quantize_bits: Optional[int] = None, onnx: bool = False,
                  benchmark_data: Optional[Path] = None, group_size: Optional[int] = None) -> dict:
    from ..data.pipeline import load_tokenizer
    from ..inference.quantization import load_quantized, quantize_model, save_quantized

    checkpoint, output = Path(checkpoint), Path(output)
    output.mkdir(parents=True, exist_ok=True)
    model, state = load_checkpoint_model(checkpoint)
    config = model.config
    tokenizer = load_tokenizer(checkpoint)
    model.set_static_dispatch(True)
    wrapper = LogitsOnly(model).eval()
    meta: dict = {"format": 1, "source_checkpoint": str(checkpoint), "training_step": state.get("step"),
                  "config": dict(config.__dict__), "tokenizer": tokenizer.kind,
                  "parameters": {"total": sum(p.numel() for p in model.parameters())}, "files": {}}
    example = torch.randint(0, config.vocab_size, (1, min(8, config.max_sequence_length)))
    with torch.inference_mode():
        traced = torch.jit.trace(wrapper, example, check_trace=False)
    traced.save(str(output / "model.torchscript.pt"))
    (output / "model.graph.txt").write_text(str(traced.graph))

    # parity: the reloaded trace vs eager at shapes the trace never saw; static dense vs the sparse (no-drop) path
    reloaded = torch.jit.load(str(output / "model.torchscript.pt"))
    worst = 0.0
    with torch.inference_mode():
        for batch, length in parity_shapes(config):
            ids = torch.randint(0, config.vocab_size, (batch, length))
            worst = max(worst, float((reloaded(ids) - wrapper(ids)).abs().max()))
        ids = torch.randint(0, config.vocab_size, (2, min(8, config.max_sequence_length)))
        static = wrapper(ids)
        model.set_static_dispatch(False)
        drop = model.moes()[0].drop_overflow_tokens
        model.set_routing_controls(drop_overflow_tokens=False)
        sparse = model(ids)["logits"]
        model.set_routing_controls(drop_overflow_tokens=drop)
        model.set_static_dispatch(True)
    meta["parity"] = {"traced_vs_eager_max_abs_diff": worst,
                      "static_vs_sparse_max_abs_diff": float((static - sparse).abs().max()),
                      "shapes_checked": [list(s) for s in parity_shapes(config)]}
    if onnx:
        meta["onnx"] = try_onnx(wrapper, example, output / "model.onnx", config.max_sequence_length - 1)
    if quantize_bits:
        qmodel, _ = load_checkpoint_model(checkpoint)
        stats = quantize_model(qmodel, quantize_bits, group_size)
        filename = f"model.int{quantize_bits}.pt"
        save_quantized(qmodel, output / filename, stats)
        with torch.inference_mode():
            model.set_static_dispatch(False)
            model.set_routing_controls(drop_overflow_tokens=False)
            ref = model(ids)["logits"]
            approx = load_quantized(output / filename)(ids)["logits"]
            model.set_static_dispatch(True)
        cosine = torch.nn.functional.cosine_similarity(ref.flatten(), approx.flatten(), dim=0)
        meta["quantized"] = {**stats, "file": filename, "logit_cosine_similarity": float(cosine)}
    for name in ("config.json", "tokenizer_meta.json", "vocab.json", "tokenizer.json", "tokenizer.model"):
        if (checkpoint / name).exists():
            shutil.copy(checkpoint / name, output / name)
    if benchmark_data is not None:
        from .benchmark import build_parser, run_benchmark

        report = run_benchmark(build_parser().parse_args(["--checkpoint", str(checkpoint), "--data",
                                                          str(benchmark_data), "--device", "cpu",
                                                          "--no-routing-stats"]))
        meta["benchmark"] = {k: report[k] for k in ("loss", "perplexity", "tokens_per_second", "tokens",
                                                    "active_parameters_per_token_estimate")}
    for file in sorted(output.iterdir()):
        if file.is_file() and file.name != "export_metadata.json":
            meta["files"][file.name] = {"bytes": file.stat().st_size, "sha256": sha256(file)}
    (output / "export_metadata.json").write_text(json.dumps(meta, indent=2) + "\n")
    return meta


def load_exported(directory: Path):
    """(traced module, tokenizer, metadata) of a bundle; needs no model code."""
    from ..data.pipeline import load_tokenizer

    directory = Path(directory)
    meta = json.loads((directory / "export_metadata.json").read_text())
    return torch.jit.load(str(directory / "model.torchscript.pt")).eval(), load_tokenizer(directory), meta


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--quantize", type=int, choices=(4, 8), help="add a copy with int4 or int8 expert weights")
    p.add_argument("--group-size", type=int, help="quantisation group (default: per row for int8, 32 for int4)")
    p.add_argument("--onnx", action="store_true", help="attempt an ONNX file as well (requires the onnx package)")
    p.add_argument("--benchmark-data", type=Path, help="measure the source model's loss, perplexity and speed on these rows")
    from .common import describe_options

    describe_options(p, {'output': 'directory of the export bundle'})
    args = p.parse_args(argv)
    meta = export_bundle(args.checkpoint, args.output, args.quantize, args.onnx, args.benchmark_data,
                         args.group_size)
    print(json.dumps({k: meta[k] for k in ("parity", "parameters") if k in meta} | {"files": list(meta["files"])},
                     indent=2))


if __name__ == "__main__":
    main()
