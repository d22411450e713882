"""bench-gemv: time one low-bit GEMV launch on B200 (the reference's `gfxinfer bench-gemv`).

    python -m gfxinfer_b200.bench_gemv --format w3 --rows 17408 --columns 5120 --batch 1 \
        [--activation a4|a8] [--iterations 60] [--copies 6] [--matrices 1..4] [--no-graph]

Mirrors src/cli/main.cpp:1529-1700: seeded random code bytes, fp16 scales drawn
U(0.002, 0.08), activations U(-2, 2) rounded to fp16; timed launches; a sampled
check of rows {0, N/2, N-1} against a float64 reconstruction (tolerance 0.3 %
of max(1, |y|), as the reference). Reports the mean launch time, the
reference's packed-code GB/s and the full algorithmic GB/s (codes + fp16
scales + activation + fp32 outputs). Launches rotate over `copies` weight
buffers so every launch reads HBM, and are replayed from a CUDA graph unless
--no-graph (host launch overhead would otherwise dominate small shapes).
--matrices M runs M matrices of the shape sharing one input in one launch
(the MLP gate+up launch is --matrices 2 of [17408 x 5120]).
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import BITS_TO_FORMAT
from . import ops

FORMATS = {"w2": 2, "w3": 3, "w4": 4}


def _decode_rowmajor(codes_row: np.ndarray, bits: int, columns: int) -> np.ndarray:
    """Reference row-major codes (quantization.cpp:126-150) -> signed levels."""
    if bits == 2:
        c = np.unpackbits(codes_row[:, None], axis=1, bitorder="little").reshape(-1, 4, 2)
        code = c[:, :, 0] + 2 * c[:, :, 1]
        return (code.reshape(-1)[:columns] * 2 - 3).astype(np.int64)
    if bits == 4:
        low, high = codes_row & 15, codes_row >> 4
        code = np.stack([low, high], axis=1).reshape(-1)[:columns].astype(np.int64)
        return np.where(code >= 8, code - 16, code)
    groups = columns // 128
    planes = codes_row.reshape(groups, 3, 16)
    bits_ = np.unpackbits(planes, axis=2, bitorder="little")  # [g][plane][128]
    code = bits_[:, 0] + 2 * bits_[:, 1] + 4 * bits_[:, 2]
    return code.reshape(-1).astype(np.int64) - 4


def run(fmt: str, rows: int, columns: int, batch: int, activation: str, iterations: int, copies: int,
        graph: bool, seed: int = 0x1200, matrices: int = 1) -> dict:
    bits = FORMATS[fmt]
    fmt_id = BITS_TO_FORMAT[bits]
    ops.require_sm100(0)
    rng = np.random.default_rng(seed)
    row_bytes = columns * bits // 8
    groups = columns // 128
    weights, scales, host = [], [], None
    for i in range(copies * matrices):
        codes = rng.integers(0, 256, size=rows * row_bytes, dtype=np.uint8)
        scale16 = rng.uniform(0.002, 0.08, size=rows * groups).astype(np.float16)
        if i == 0:
            host = (codes.reshape(rows, row_bytes), scale16.reshape(rows, groups).astype(np.float64))
        weights.append(ops.repack_rowmajor(fmt_id, torch.from_numpy(codes).cuda(), rows, columns))
        scales.append(ops.tile_scales(torch.from_numpy(scale16).cuda(), rows, columns))
    x16 = rng.uniform(-2.0, 2.0, size=(batch, columns)).astype(np.float16)
    x = torch.from_numpy(x16).cuda()
    act_bits = 4 if activation == "a4" else 8
    codes_a, scales_a, sums_a, _ = ops.pack_activation(x, act_bits)
    outs = [torch.empty((batch, rows), dtype=torch.float32, device="cuda") for _ in range(matrices)]
    out = outs[0]

    def launch(i: int) -> None:
        c = (i % copies) * matrices
        ops.lowbit_gemv(fmt_id, [(weights[c + j], scales[c + j], outs[j], rows, False) for j in range(matrices)],
                        codes_a, scales_a, sums_a, columns, batch)

    for i in range(10):
        launch(i)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            for i in range(iterations):
                launch(i)
        g.replay()
        torch.cuda.synchronize()
        start.record()
        g.replay()
        stop.record()
    else:
        start.record()
        for i in range(iterations):
            launch(i)
        stop.record()
    stop.synchronize()
    mean_us = start.elapsed_time(stop) * 1000.0 / iterations
    # the last launch used copy (iterations - 1) % copies; recompute copy 0 for the check
    launch(0)
    torch.cuda.synchronize()
    y = out.cpu().numpy()
    codes0, scales0 = host
    a = codes_a.cpu().numpy().astype(np.int64)
    k = np.arange(128)
    offset = ((k & 15) >> 2) * 32 + (k >> 5) * 8 + ((k & 31) >> 4) * 4 + (k & 3)
    a_logical = a.reshape(batch, groups, 128)[:, :, offset].reshape(batch, columns)
    a_scale = scales_a.cpu().numpy().astype(np.float64)
    max_error = 0.0
    for r in (0, rows // 2, rows - 1):
        w = _decode_rowmajor(codes0[r], bits, columns).reshape(groups, 128)
        for b in range(batch):
            dots = (w * a_logical[b].reshape(groups, 128)).sum(axis=1)
            expected = float((dots * scales0[r] * a_scale[b]).sum())
            error = abs(expected - float(y[b, r]))
            max_error = max(max_error, error)
            if not np.isfinite(y[b, r]) or error > 0.003 * max(1.0, abs(expected)):
                raise SystemExit(f"validation failed at batch {b} row {r}: expected={expected} actual={y[b, r]}")
    code_bytes = rows * row_bytes * matrices
    algorithmic = (code_bytes + matrices * rows * groups * 2 + batch * (columns * act_bits // 8 + groups * 2)
                   + matrices * batch * rows * 4)
    return {"format": fmt, "shape": [rows, columns], "matrices": matrices, "batch": batch, "activation": activation,
            "mean_launch_us": round(mean_us, 3), "packed_GBps": round(code_bytes / mean_us / 1e3, 1),
            "algorithmic_GBps": round(algorithmic / mean_us / 1e3, 1), "algorithmic_bytes": algorithmic,
            "launches_per_second": round(1e6 / mean_us, 1), "max_sampled_error": max_error,
            "validation": "pass", "graph": graph, "copies": copies}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--format", choices=sorted(FORMATS), default="w3")
    parser.add_argument("--rows", type=int, default=17408)
    parser.add_argument("--columns", type=int, default=5120)
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--activation", choices=["a4", "a8"], default="a4")
    parser.add_argument("--iterations", type=int, default=60)
    parser.add_argument("--copies", type=int, default=6)
    parser.add_argument("--matrices", type=int, default=1, choices=[1, 2, 3, 4])
    parser.add_argument("--no-graph", action="store_true")
    args = parser.parse_args()
    print(json.dumps(run(args.format, args.rows, args.columns, args.batch, args.activation, args.iterations,
                         args.copies, not args.no_graph, matrices=args.matrices)))


if __name__ == "__main__":
    main()
