"""Run every decode-path kernel once inside a profiler window.

    python -m gfxinfer_b200.profile_kernels [--layers 4] [--position 200]
    ncu --profile-from-start off --clock-control none --metrics ... python -m gfxinfer_b200.profile_kernels

Builds a config-2-width engine (hidden 5120, MLP 17408 W3, 48/16 GDN heads, 24/4 attention heads,
W4 LM head over 151936 rows) with `--layers` layers, decodes `--position` tokens on the per-operation
path, then brackets with cudaProfilerStart/Stop: one per-operation greedy step, one 8-token verifier
block, one persistent token-kernel step and one fp16-activation GEMV [17408 x 5120] W3.
"""
from __future__ import annotations

import argparse

import torch

from . import abi, ops
from . import session as gs


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--layers", type=int, default=4)
    parser.add_argument("--position", type=int, default=200)
    args = parser.parse_args()
    cfg = dict(gs.CONFIG2, layers=args.layers, max_context=512)
    engine = gs.Engine.create(gs.model_config(**cfg), include_mtp=False)
    launches = gs.QwenDecodeSession.create(engine, step_kernel=abi.STEP_LAUNCHES, use_graphs=False)
    persistent = gs.QwenDecodeSession.create(engine, step_kernel=abi.STEP_PERSISTENT, use_graphs=False)
    token = 1
    for _ in range(args.position):
        token = launches.greedy_step(token)
    other = 1
    for _ in range(3):
        other = persistent.greedy_step(other)
    rows, cols = 17408, 5120
    codes = torch.randint(0, 256, (rows * cols * 3 // 8,), dtype=torch.uint8, device="cuda")
    scales = (torch.rand(rows * cols // 128, device="cuda") * 0.01 + 0.001).half()
    x = torch.randn(1, cols, device="cuda").half()
    out = torch.empty(1, rows, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    launches.greedy_step(token)
    launches.block_step([1, 2, 3, 4, 5, 6, 7, 8])
    persistent.greedy_step(other)
    ops.lowbit_gemv_f16(2, [(codes, scales, out, rows, False)], x)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    launches.close()
    persistent.close()
    engine.close()
    print("ok")


if __name__ == "__main__":
    main()
