"""Build libgfxb200.so (all CUDA kernels + the C++ host runtime) and the gfxinfer-b200 CLI for sm_100a.

    python -m gfxinfer_b200.build [--force] [--verbose]

Objects go to gfxinfer_b200/_build; the shared library is written in-tree at
gfxinfer_b200/libgfxb200.so so it travels with the repository snapshot.
The numerics flags are part of the contract with the CPU oracle: -fmad=false
(no implicit a*b+c fusion), IEEE division and square root, denormals kept.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import subprocess
import sys

PACKAGE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PACKAGE)
CSRC = os.path.join(PACKAGE, "csrc")
BUILD = os.path.join(PACKAGE, "_build")
LIBRARY = os.path.join(PACKAGE, "libgfxb200.so")
CLI = os.path.join(PACKAGE, "gfxinfer-b200")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
HOST_CXX = "/usr/bin/g++"
NCCL_INCLUDE = "/usr/include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++20", "-lineinfo", f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}",
          "-Xcompiler", "-fPIC,-Wall", "-ccbin", HOST_CXX]
NUMERICS = ["-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"]


def _sources() -> list[str]:
    files = []
    for pattern in ("kernels/*.cu", "host/*.cpp", "host/*.cu"):
        files.extend(sorted(glob.glob(os.path.join(CSRC, pattern))))
    return files


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
            + glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
            + glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True))


def _object(source: str) -> str:
    rel = os.path.relpath(source, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(source: str, verbose: bool) -> str:
    obj = _object(source)
    cmd = [NVCC, *ARCH, *COMMON, *NUMERICS, "-c", source, "-o", obj]
    if source.endswith(".cu"):
        cmd[1:1] = ["-x", "cu"]
        cmd += ["-Xptxas", "-v"] if verbose else []
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"compilation failed: {source}\n{result.stdout}\n{result.stderr}")
    return result.stderr if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = _sources()
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    stale = [s for s in sources if force or not os.path.exists(_object(s))
             or os.path.getmtime(_object(s)) < max(os.path.getmtime(s), newest_header)]
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        for log in pool.map(lambda s: _compile(s, verbose), stale):
            if log:
                print(log, file=sys.stderr)
    objects = [_object(s) for s in sources]
    if stale or not os.path.exists(LIBRARY):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIBRARY, *objects, "-lcudart", "-ldl",
               "-Xlinker", "-rpath,$ORIGIN"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed\n{result.stdout}\n{result.stderr}")
    _build_cli(force or bool(stale), newest_header)
    return LIBRARY


def _build_cli(force: bool, newest_header: float) -> None:
    """The gfxinfer-b200 command line (csrc/cli/main.cpp), linked against the library."""
    source = os.path.join(CSRC, "cli", "main.cpp")
    if not force and os.path.exists(CLI) and os.path.getmtime(CLI) >= max(os.path.getmtime(source), newest_header):
        return
    cmd = [NVCC, *ARCH, *COMMON, "-o", CLI, source, f"-L{PACKAGE}", "-lgfxb200", "-lcudart",
           "-Xlinker", "-rpath,$ORIGIN"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"CLI build failed\n{result.stdout}\n{result.stderr}")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
