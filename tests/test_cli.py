"""The gfxinfer-b200 command line (the reference's `gfxinfer` CLI, src/cli/main.cpp:38-67):
CPU-side commands here, GPU commands in test_cli_gpu.py."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "gfxinfer_b200", "gfxinfer-b200")


@pytest.fixture(scope="module")
def cli():
    from gfxinfer_b200 import build

    build.build()
    assert os.access(CLI, os.X_OK)
    return CLI


def test_usage(cli):
    result = subprocess.run([cli], capture_output=True, text=True)
    assert result.returncode == 2 and "usage" in result.stderr


def test_inspect_lists_an_artifact(cli, tmp_path):
    from gfxinfer_b200 import artifact as gx

    path = tmp_path / "a.gfxi"
    gx.write(path, {"target_arch": "sm_100a", "model_id": "qwen-hybrid", "weights_id": "w", "recipe_id": "b200-v1"},
             [gx.TensorWrite("model.language_model.norm.weight", gx.DTYPE_BF16, gx.QUANT_NONE, (8,), b"\0" * 16)])
    result = subprocess.run([cli, "inspect", str(path)], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    assert "recipe b200-v1" in result.stdout and "model.language_model.norm.weight" in result.stdout
    assert "bf16" in result.stdout and "[8]" in result.stdout


def test_inspect_rejects_a_corrupt_artifact(cli, tmp_path):
    path = tmp_path / "bad.gfxi"
    path.write_bytes(b"not an artifact" * 40)
    result = subprocess.run([cli, "inspect", str(path)], capture_output=True, text=True)
    assert result.returncode == 1 and "status 3" in result.stderr
