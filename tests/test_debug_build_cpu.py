"""The bounds-checking debug build (``QW_DEBUG_BOUNDS=1``) compiles for sm_100a. No GPU is needed: nvcc
cross-compiles the sources whose kernels carry index checks, with the same flags the extension build passes."""

import shutil
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "csrc"


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
@pytest.mark.parametrize("source", ["moe_routing.cu", "ep_fused.cu"])
def test_the_bounds_checked_kernels_compile_for_sm100a(source, tmp_path):
    assert "in_bounds(" in (CSRC / source).read_text()  # the file really carries debug index checks
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-DQW_DEBUG_BOUNDS=1",
           f"-I{CSRC}", "-c", str(CSRC / source), "-o", str(tmp_path / "out.o")]
    result = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stderr[-2000:]
