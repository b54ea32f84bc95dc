"""Export a checkpoint as a self-contained inference bundle.

    python -m quantaweave_b200.tools.export --checkpoint artifacts/outputs/quantweave-moe-out \\
        --output artifacts/exports/moe --quantize 8 --benchmark-data data/smoke/tinystories.jsonl

The bundle holds the same files as the reference exporter's (``src/export_quantweave.py``: ``export_bundle``
:106-182, ``load_exported`` :185): ``model.torchscript.pt`` (a trace with dynamic batch and sequence) and
``model.graph.txt``, an optional ``model.onnx``, an optional ``model.int{4,8}.pt`` weight-only copy, the tokenizer
and config files, and ``export_metadata.json`` with sizes, sha256 digests, numerical checks and an optional
benchmark. The traced graph evaluates every expert densely, weighted by the router (no capacity and no
data-dependent control flow), so it is portable and exact but not sparse-fast. It is traced from the fp32 PyTorch
path on the CPU; the sm_100a kernels are not part of the exported artefact.

The export runs as a sequence of stages (:class:`_Export`), each adding one section to the metadata.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import shutil
from contextlib import contextmanager
from pathlib import Path
from typing import Optional

import torch
from torch import nn

TOKENIZER_FILES = ("config.json", "tokenizer_meta.json", "vocab.json", "tokenizer.json", "tokenizer.model")
TRACE_FILE, GRAPH_FILE, ONNX_FILE, META_FILE = ("model.torchscript.pt", "model.graph.txt", "model.onnx",
                                                "export_metadata.json")


class LogitsOnly(nn.Module):
    """The model with a tensor-in, tensor-out signature (token ids -> logits), as tracers need."""

    def __init__(self, model) -> None:
        super().__init__()
        self.model = model

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids)["logits"]


def sha256(path: Path) -> str:
    digest = hashlib.sha256()
    with open(path, "rb") as source:
        for block in iter(lambda: source.read(1 << 20), b""):
            digest.update(block)
    return digest.hexdigest()


def load_checkpoint_model(checkpoint: Path):
    """(model in eval mode on the CPU, raw checkpoint payload)."""
    from ..models.model import QuantaWeaveMoEForCausalLM
    from ..utils.checkpoint_io import load_checkpoint
    from .common import read_config

    payload = load_checkpoint(Path(checkpoint) / "model.pt", map_location="cpu")
    model = QuantaWeaveMoEForCausalLM(read_config(checkpoint))
    model.load_state_dict(payload["model"])
    model.eval()
    return model, payload


def parity_shapes(config) -> list[tuple[int, int]]:
    """(batch, length) pairs the traced graph is checked at; none equals the tracing example's shape."""
    full = config.max_sequence_length
    return [(1, full), (2, max(3, full // 3)), (4, 3)]


def _random_ids(config, batch: int, length: int) -> torch.Tensor:
    return torch.randint(0, config.vocab_size, (batch, length))


def try_onnx(wrapper: LogitsOnly, example: torch.Tensor, path: Path, max_sequence_length: int) -> dict:
    """An ONNX file from the ``torch.export`` exporter with symbolic batch and sequence dimensions; when
    onnxruntime is present it is run at a shape different from the example's and compared with PyTorch.
    Failures are reported in the returned section, never raised."""
    try:
        import onnx  # noqa: F401
    except ImportError:
        return {"status": "skipped", "reason": "the `onnx` package is not installed"}
    # torch.export specialises a dimension whose example size is 1, so the batch dimension is exported from a
    # batch of at least two rows
    sample = example.repeat(2, 1) if example.size(0) < 2 else example
    symbolic = {"input_ids": {0: torch.export.Dim("batch"),
                              1: torch.export.Dim("sequence", max=max_sequence_length)}}
    try:
        torch.onnx.export(wrapper, (sample,), str(path), input_names=["input_ids"], output_names=["logits"],
                          dynamic_shapes=symbolic, dynamo=True)
    except Exception as error:  # noqa: BLE001 - an exporter failure is data for the metadata
        path.unlink(missing_ok=True)
        return {"status": "failed", "reason": f"{type(error).__name__}: {error}"[:300]}
    section = {"status": "ok", "file": path.name}
    try:
        import onnxruntime
    except ImportError:
        section.update(dynamic_shape_verified=False,
                       note="onnxruntime is not installed; the export was not round-tripped at another shape")
        return section
    probe = _random_ids(wrapper.model.config, sample.size(0) + 1, min(max_sequence_length, sample.size(1) + 3))
    runtime = onnxruntime.InferenceSession(str(path), providers=["CPUExecutionProvider"])
    got = torch.from_numpy(runtime.run(None, {"input_ids": probe.numpy()})[0])
    with torch.inference_mode():
        want = wrapper(probe)
    section.update(dynamic_shape_verified=True, verified_max_abs_diff=float((got - want).abs().max()))
    return section


@contextmanager
def _sparse_no_drop(model):
    """Temporarily run the model's sparse routing path without capacity drops (restored afterwards)."""
    keep_drop = model.moes()[0].drop_overflow_tokens
    model.set_static_dispatch(False)
    model.set_routing_controls(drop_overflow_tokens=False)
    try:
        yield model
    finally:
        model.set_routing_controls(drop_overflow_tokens=keep_drop)
        model.set_static_dispatch(True)


class _Export:
    """One export: the stages fill ``self.meta``; :meth:`run` orders them."""

    def __init__(self, checkpoint: Path, output: Path) -> None:
        from ..data.pipeline import load_tokenizer

        self.checkpoint, self.output = Path(checkpoint), Path(output)
        self.output.mkdir(parents=True, exist_ok=True)
        self.model, payload = load_checkpoint_model(self.checkpoint)
        self.config = self.model.config
        self.model.set_static_dispatch(True)
        self.wrapper = LogitsOnly(self.model).eval()
        self.example = _random_ids(self.config, 1, min(8, self.config.max_sequence_length))
        self.check_ids = _random_ids(self.config, 2, min(8, self.config.max_sequence_length))
        self.meta: dict = {"format": 1, "source_checkpoint": str(self.checkpoint),
                           "training_step": payload.get("step"), "config": dict(vars(self.config)),
                           "tokenizer": load_tokenizer(self.checkpoint).kind,
                           "parameters": {"total": sum(p.numel() for p in self.model.parameters())}, "files": {}}

    def trace(self) -> None:
        with torch.inference_mode():
            traced = torch.jit.trace(self.wrapper, self.example, check_trace=False)
        traced.save(str(self.output / TRACE_FILE))
        (self.output / GRAPH_FILE).write_text(str(traced.graph))

    def check(self) -> None:
        """The saved trace against eager execution at unseen shapes, and the dense (static) dispatch against the
        sparse router path with capacity off (the two must agree when nothing is dropped)."""
        reloaded = torch.jit.load(str(self.output / TRACE_FILE))
        shapes = parity_shapes(self.config)
        with torch.inference_mode():
            traced_gap = max(float((reloaded(ids) - self.wrapper(ids)).abs().max())
                             for ids in (_random_ids(self.config, b, n) for b, n in shapes))
            dense = self.wrapper(self.check_ids)
            with _sparse_no_drop(self.model):
                sparse = self.model(self.check_ids)["logits"]
        self.meta["parity"] = {"traced_vs_eager_max_abs_diff": traced_gap,
                               "static_vs_sparse_max_abs_diff": float((dense - sparse).abs().max()),
                               "shapes_checked": [list(shape) for shape in shapes]}

    def onnx(self) -> None:
        self.meta["onnx"] = try_onnx(self.wrapper, self.example, self.output / ONNX_FILE,
                                     self.config.max_sequence_length - 1)

    def quantized_copy(self, bits: int, group_size: Optional[int]) -> None:
        from ..inference.quantization import load_quantized, quantize_model, save_quantized

        copy, _ = load_checkpoint_model(self.checkpoint)
        stats = quantize_model(copy, bits, group_size)
        name = f"model.int{bits}.pt"
        save_quantized(copy, self.output / name, stats)
        with torch.inference_mode(), _sparse_no_drop(self.model):
            exact = self.model(self.check_ids)["logits"].flatten()
            approx = load_quantized(self.output / name)(self.check_ids)["logits"].flatten()
        cosine = float(torch.nn.functional.cosine_similarity(exact, approx, dim=0))
        self.meta["quantized"] = {**stats, "file": name, "logit_cosine_similarity": cosine}

    def tokenizer_files(self) -> None:
        for name in TOKENIZER_FILES:
            if (self.checkpoint / name).exists():
                shutil.copy(self.checkpoint / name, self.output / name)

    def benchmark(self, data: Path) -> None:
        from .benchmark import build_parser, run_benchmark

        argv = ["--checkpoint", str(self.checkpoint), "--data", str(data), "--device", "cpu", "--no-routing-stats"]
        report = run_benchmark(build_parser().parse_args(argv))
        keys = ("loss", "perplexity", "tokens_per_second", "tokens", "active_parameters_per_token_estimate")
        self.meta["benchmark"] = {key: report[key] for key in keys}

    def manifest(self) -> None:
        files = sorted(f for f in self.output.iterdir() if f.is_file() and f.name != META_FILE)
        self.meta["files"] = {f.name: {"bytes": f.stat().st_size, "sha256": sha256(f)} for f in files}
        (self.output / META_FILE).write_text(json.dumps(self.meta, indent=2) + "\n")

    def run(self, quantize_bits: Optional[int], onnx: bool, benchmark_data: Optional[Path],
            group_size: Optional[int]) -> dict:
        self.trace()
        self.check()
        if onnx:
            self.onnx()
        if quantize_bits:
            self.quantized_copy(quantize_bits, group_size)
        self.tokenizer_files()
        if benchmark_data is not None:
            self.benchmark(benchmark_data)
        self.manifest()
        return self.meta


def export_bundle(checkpoint: Path, output: Path, quantize_bits: Optional[int] = None, onnx: bool = False,
                  benchmark_data: Optional[Path] = None, group_size: Optional[int] = None) -> dict:
    """Write the bundle for ``checkpoint`` into ``output`` and return its metadata."""
    return _Export(checkpoint, output).run(quantize_bits, onnx, benchmark_data, group_size)


def load_exported(directory: Path):
    """(traced module, tokenizer, metadata) of a bundle; needs no model code."""
    from ..data.pipeline import load_tokenizer

    directory = Path(directory)
    module = torch.jit.load(str(directory / TRACE_FILE)).eval()
    return module, load_tokenizer(directory), json.loads((directory / META_FILE).read_text())


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", type=Path, default=Path("artifacts/outputs/quantweave-moe-out"))
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--quantize", type=int, choices=(4, 8), help="add a copy with int4 or int8 expert weights")
    p.add_argument("--group-size", type=int, help="quantisation group (default: per row for int8, 32 for int4)")
    p.add_argument("--onnx", action="store_true", help="attempt an ONNX file as well (requires the onnx package)")
    p.add_argument("--benchmark-data", type=Path,
                   help="measure the source model's loss, perplexity and speed on these rows")
    from .common import describe_options

    describe_options(p, {"output": "directory of the export bundle"})
    args = p.parse_args(argv)
    meta = export_bundle(args.checkpoint, args.output, args.quantize, args.onnx, args.benchmark_data,
                         args.group_size)
    summary = {key: meta[key] for key in ("parity", "parameters") if key in meta}
    summary["files"] = list(meta["files"])
    print(json.dumps(summary, indent=2))


if __name__ == "__main__":
    main()
