"""GPU commands of the gfxinfer-b200 CLI: bench-gemv validates sampled rows against a float64
reconstruction (src/cli/main.cpp:1661-1682), block-bench and spec-bench require exact token
parity with serial greedy decode (:866-887, :961-979)."""
import subprocess

import pytest

from test_cli import cli  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


def _run(cli, *args):
    result = subprocess.run([cli, *args], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout + result.stderr
    return result.stdout


@pytest.mark.parametrize("fmt", ["w2", "w3", "w4"])
@pytest.mark.parametrize("activation", ["a4", "a8", "f16"])
def test_bench_gemv(cli, fmt, activation):  # noqa: F811
    out = _run(cli, "bench-gemv", "--format", fmt, "--rows", "1024", "--columns", "2048", "--batch", "5",
               "--activation", activation, "--iterations", "20")
    assert "validation:         pass" in out


def test_probe(cli):  # noqa: F811
    assert "sm_10" in _run(cli, "probe")


def test_decode_block_and_spec_bench(cli, tmp_path):  # noqa: F811
    assert "decode speed" in _run(cli, "decode-bench", "--small", "--steps", "16")
    assert "exact token IDs" in _run(cli, "block-bench", "--small", "--width", "12")
    assert "exact token IDs" in _run(cli, "spec-bench", "--small", "--depth", "4", "--tokens", "40")
    assert "exact token IDs" in _run(cli, "spec-bench", "--small", "--depth", "3", "--tokens", "30", "--eager")
    path = str(tmp_path / "small.gfxi")
    _run(cli, "export", path, "--small")
    assert "recipe b200-v1" in _run(cli, "inspect", path)
    assert "exact token IDs" in _run(cli, "spec-bench", "--artifact", path, "--context", "320", "--depth", "2",
                                     "--tokens", "24")
