"""The bench's reference arm finds the reference's modules in every install layout it can meet."""

import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _modules(directory):
    os.makedirs(directory, exist_ok=True)
    for name in ("quantweave_moe_model.py", "moe_kernels.py", "expert_parallel.py"):
        with open(os.path.join(directory, name), "w") as f:
            f.write("# stand-in\n")
    return directory


def _dist_info(root, url):
    info = os.path.join(root, "baseline", "_ref", "quantweave-0.1.0.dist-info")
    os.makedirs(info, exist_ok=True)
    with open(os.path.join(info, "direct_url.json"), "w") as f:
        json.dump({"dir_info": {}, "url": url}, f)
    return info


def test_modules_copied_under_baseline_ref(tmp_path):
    src = _modules(str(tmp_path / "baseline" / "_ref" / "src"))
    found, searched = bench.locate_reference_src(str(tmp_path), environ={})
    assert found == src and searched


def test_metadata_only_install_follows_direct_url(tmp_path):
    project = tmp_path / "somewhere" / "reference"
    src = _modules(str(project / "src"))
    _dist_info(str(tmp_path), "file://" + str(project))
    found, _ = bench.locate_reference_src(str(tmp_path), environ={})
    assert found == src


def test_flat_project_and_percent_encoded_url(tmp_path):
    project = tmp_path / "with space"
    src = _modules(str(project))
    _dist_info(str(tmp_path), "file://" + str(project).replace(" ", "%20"))
    found, _ = bench.locate_reference_src(str(tmp_path), environ={})
    assert found == src


def test_explicit_override_wins(tmp_path):
    _modules(str(tmp_path / "baseline" / "_ref" / "src"))
    other = _modules(str(tmp_path / "elsewhere"))
    found, _ = bench.locate_reference_src(str(tmp_path), environ={"QW_REFERENCE_SRC": other})
    assert found == other


def test_missing_reports_every_place_searched(tmp_path, monkeypatch):
    _dist_info(str(tmp_path), "file:///nonexistent/reference")
    monkeypatch.setattr(sys, "path", [p for p in sys.path if p])  # the repo's own test tree has no such module
    found, searched = bench.locate_reference_src(str(tmp_path), environ={"QW_REFERENCE_SRC": "/nonexistent/x"})
    assert found is None
    text = " ".join(searched)
    assert "QW_REFERENCE_SRC" in text and "/nonexistent/reference/src" in text and "sys.path" in text


@pytest.mark.parametrize("depth_ok", [True, False])
def test_walk_depth_is_bounded(tmp_path, depth_ok):
    parts = ["a", "b", "c"] if depth_ok else ["a", "b", "c", "d", "e", "f"]
    src = _modules(str(tmp_path.joinpath("baseline", "_ref", *parts)))
    found, _ = bench.locate_reference_src(str(tmp_path), environ={})
    assert (found == src) if depth_ok else (found is None or found != src)
