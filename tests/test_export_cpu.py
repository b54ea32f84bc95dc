"""Export bundle: TorchScript trace with dynamic shapes, parity, quantised copy, manifest (reference test:
tests/test_export.py)."""

import json

import torch

from quantaweave_b200.tools.export import export_bundle, load_exported


def test_export_bundle_parity_and_quantized_copy(tmp_path):
    from test_tools_cpu import _train

    data, _ = _train(tmp_path, steps=3)
    meta = export_bundle(tmp_path / "out", tmp_path / "export", quantize_bits=8, benchmark_data=data)
    assert meta["parity"]["traced_vs_eager_max_abs_diff"] < 1e-4
    assert meta["parity"]["static_vs_sparse_max_abs_diff"] < 1e-4
    assert meta["quantized"]["logit_cosine_similarity"] > 0.99
    for name in ("model.torchscript.pt", "model.graph.txt", "model.int8.pt", "config.json", "vocab.json"):
        assert name in meta["files"] and len(meta["files"][name]["sha256"]) == 64
    assert meta["benchmark"]["tokens"] > 0
    module, tok, saved = load_exported(tmp_path / "export")
    ids = torch.tensor([tok.encode("the cat sat")])
    assert module(ids).shape == (1, ids.size(1), saved["config"]["vocab_size"])
    assert json.loads((tmp_path / "export" / "export_metadata.json").read_text())["format"] == 1
