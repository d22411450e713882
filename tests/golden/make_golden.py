"""Regenerate tests/golden/quantization_golden.npz from the reference's own packer.

Runs only where the reference checkout is present (it builds oracle/_ref from
the reference's src/quantization.cpp in place). The GPU box and the CPU test
suite read the committed .npz; nothing at test time needs the reference.

    python tests/golden/make_golden.py
"""
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle_lib import W2, W3, W4, Reference  # noqa: E402


def main() -> None:
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    ref = Reference()
    out = {}
    for fmt, name in ((W2, "w2"), (W3, "w3"), (W4, "w4")):
        # tests/quantization_test.cpp:12-22: 3x256, mt19937(1200), N(0, 0.25), injected 0/+2/-2.
        values = ref.test_matrix(1200, 0.25, 3, 256)
        values[0, 0] = 0.0
        values[1, 17] = 2.0
        values[2, 93] = -2.0
        status, codes, scales = ref.quantize(values, fmt)
        assert status == 0
        out[f"rmse_{name}_input"] = values
        out[f"rmse_{name}_codes"] = codes
        out[f"rmse_{name}_scales"] = scales
        # tests/quantization_test.cpp:49-56: 32x256, mt19937(1201), N(0, 0.5), then gfx12 tiling.
        tile_values = ref.test_matrix(1201, 0.5, 32, 256)
        status, codes, scales = ref.quantize(tile_values, fmt)
        assert status == 0
        status, tiled, tiled_scales = ref.tile(codes, scales, 32, 256, fmt)
        assert status == 0
        out[f"tile_{name}_input"] = tile_values
        out[f"tile_{name}_codes"] = codes
        out[f"tile_{name}_scales"] = scales
        out[f"tile_{name}_tiled"] = tiled
        out[f"tile_{name}_tiled_scales"] = tiled_scales
        # A config-0-shaped slice: N(0, 0.02) weights, 64 rows x 512 columns.
        rng = np.random.default_rng(2024 + fmt)
        slice_values = rng.normal(0.0, 0.02, size=(64, 512)).astype(np.float32)
        status, codes, scales = ref.quantize(slice_values, fmt)
        assert status == 0
        status, tiled, tiled_scales = ref.tile(codes, scales, 64, 512, fmt)
        assert status == 0
        out[f"slice_{name}_input"] = slice_values
        out[f"slice_{name}_codes"] = codes
        out[f"slice_{name}_scales"] = scales
        out[f"slice_{name}_tiled"] = tiled
        out[f"slice_{name}_tiled_scales"] = tiled_scales
    # tests/quantization_test.cpp:126-132: K = 127 is rejected.
    status, _, _ = ref.quantize(np.zeros((1, 127), np.float32), W4)
    out["k127_status"] = np.array([status], np.int32)
    np.savez_compressed(os.path.join(HERE, "quantization_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "quantization_golden.npz"))


if __name__ == "__main__":
    main()
