"""Deployment files stay well-formed (reference: ``scripts/*.sh``, ``deploy/``): every launch script and the Slurm
batch file pass ``bash -n``, the Kubernetes manifests parse as YAML with the expected kinds, and every Python module a
script launches exists."""

import re
import subprocess
from pathlib import Path

import pytest
import yaml

ROOT = Path(__file__).resolve().parents[1]
SCRIPTS = sorted((ROOT / "deploy" / "launch").glob("*.sh")) + sorted((ROOT / "deploy" / "slurm").glob("*.sbatch"))


@pytest.mark.parametrize("script", SCRIPTS, ids=lambda p: p.name)
def test_shell_scripts_parse_and_launch_modules_that_exist(script):
    result = subprocess.run(["bash", "-n", str(script)], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    for module in re.findall(r"-m\s+(quantaweave_b200(?:\.\w+)+)", script.read_text()):
        path = ROOT / Path(*module.split("."))
        assert path.with_suffix(".py").exists() or (path / "__init__.py").exists(), module


def test_kubernetes_manifests_parse():
    kinds = set()
    for manifest in (ROOT / "deploy" / "k8s").glob("*.yaml"):
        for document in yaml.safe_load_all(manifest.read_text()):
            if document:
                assert "apiVersion" in document and "kind" in document, manifest.name
                kinds.add(document["kind"])
    assert {"Deployment", "Service", "Job"} <= kinds
