"""Child process of test_cluster_splits_bit_exact (tests/test_gemv_gpu.py).

Runs the GEMV over shapes whose group counts do not divide evenly by the
cluster size (or by the pipelined kernel's K-chunks, or the persistent
single-token kernel's parts) that the parent chose through the environment,
and compares every output bit with the oracle.
Exit status 0 when all match.
"""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle_lib import W2, W3, W4, Oracle  # noqa: E402


def main() -> int:
    from gfxinfer_b200 import ops

    ops.require_sm100(0)
    oracle = Oracle()
    cases = [(W3, 48, 17 * 128, 1), (W4, 32, 3 * 128, 8), (W2, 160, 40 * 128, 5), (W3, 16, 128, 2),
             (W4, 48, 40 * 128, 2), (W3, 32, 136 * 128, 3), (W2, 16, 131 * 128, 8), (W3, 48, 17 * 128, 12),
             (W4, 32, 40 * 128, 16)]
    if os.environ.get("GFXB_GEMV_LEAN_PARTS"):
        # one token through the persistent kernel: several rounds of tiles per cluster (the ring and the
        # dot slots wrap), uneven parts, multi-round small matrices
        cases += [(W3, 4800, 40 * 128, 1), (W4, 2048, 48 * 128, 1), (W3, 640, 136 * 128, 1),
                  (W2, 1024, 131 * 128, 1), (W4, 48, 40 * 128, 1), (W3, 3216, 20 * 128, 1)]
    for fmt, rows, cols, batch in cases:
        rng = np.random.default_rng(rows * 7 + cols + batch)
        w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
        status, codes, scales = oracle.quantize(w, fmt)
        assert status == 0
        scales16 = scales.astype(np.float16).reshape(rows, cols // 128)
        logical = oracle.logical(codes, rows, cols, fmt)
        b200 = ops.repack_rowmajor(fmt, torch.from_numpy(codes).cuda(), rows, cols)
        tiled = ops.tile_scales(torch.from_numpy(scales16.reshape(-1).copy()).cuda(), rows, cols)
        x16 = rng.normal(0.0, 1.0, size=(batch, cols)).astype(np.float16)
        a_codes, a_scales, a_sums, _ = ops.pack_activation(torch.from_numpy(x16).cuda(), 4)
        out = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
        ops.lowbit_gemv(fmt, [(b200, tiled, out, rows, False)], a_codes, a_scales, a_sums, cols, batch)
        torch.cuda.synchronize()
        _, s4, a4 = oracle.quantize_a4(x16)
        want = oracle.gemv(logical, scales16, a4, s4)
        if not np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32)):
            print(f"mismatch: fmt {fmt} rows {rows} cols {cols} batch {batch}")
            return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
