"""The CPU oracle is pinned to the reference before anything is checked against it.

Golden vectors come from the reference's own src/quantization.cpp
(tests/golden/make_golden.py); the cases mirror tests/quantization_test.cpp.
"""
import os

import numpy as np
import pytest

from oracle_lib import W2, W3, W4, Reference

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "quantization_golden.npz"))
FORMATS = [(W2, "w2"), (W3, "w3"), (W4, "w4")]


@pytest.mark.parametrize("fmt,name", FORMATS)
def test_quantizer_matches_reference_golden(oracle, fmt, name):
    for case in ("rmse", "tile", "slice"):
        status, codes, scales = oracle.quantize(GOLDEN[f"{case}_{name}_input"], fmt)
        assert status == 0
        np.testing.assert_array_equal(codes, GOLDEN[f"{case}_{name}_codes"])
        np.testing.assert_array_equal(scales.view(np.uint32), GOLDEN[f"{case}_{name}_scales"].view(np.uint32))


@pytest.mark.parametrize("fmt,name", FORMATS)
def test_gfx12_tiling_matches_reference_golden(oracle, fmt, name):
    for case, rows, cols in (("tile", 32, 256), ("slice", 64, 512)):
        status, tiled, tiled_scales = oracle.tile(GOLDEN[f"{case}_{name}_codes"], GOLDEN[f"{case}_{name}_scales"], rows, cols, fmt)
        assert status == 0
        np.testing.assert_array_equal(tiled, GOLDEN[f"{case}_{name}_tiled"])
        np.testing.assert_array_equal(tiled_scales, GOLDEN[f"{case}_{name}_tiled_scales"])


@pytest.mark.parametrize("fmt,name,bound", [(W2, "w2", 0.8), (W3, "w3", 0.4), (W4, "w4", 0.2)])
def test_round_trip_rmse_bounds(oracle, fmt, name, bound):
    # tests/quantization_test.cpp:12-47, 119-121
    values = GOLDEN[f"rmse_{name}_input"]
    status, codes, scales = oracle.quantize(values, fmt)
    q = oracle.logical(codes, 3, 256, fmt).astype(np.float64)
    restored = q * np.repeat(scales.reshape(3, 2).astype(np.float64), 128, axis=1)
    rmse = np.sqrt(((values - restored) ** 2).sum() / (values.astype(np.float64) ** 2).sum())
    assert rmse <= bound


def test_rejects_k_not_multiple_of_128(oracle):
    status, _, _ = oracle.quantize(np.zeros((1, 127), np.float32), W4)
    assert status == 1 and GOLDEN["k127_status"][0] == 1


def test_rejects_non_finite(oracle):
    values = np.zeros((2, 128), np.float32)
    values[1, 5] = np.nan
    status, _, _ = oracle.quantize(values, W3)
    assert status == 1


@pytest.mark.parametrize("fmt,name", FORMATS)
def test_tiled_layout_decodes_to_dequantized_weight(oracle, fmt, name):
    # tests/quantization_test.cpp:49-113: every (row, column) of the tiled layout decodes exactly.
    rows, cols = 32, 256
    tiled = GOLDEN[f"tile_{name}_tiled"]
    tiled_scales = GOLDEN[f"tile_{name}_tiled_scales"]
    q = oracle.logical(GOLDEN[f"tile_{name}_codes"], rows, cols, fmt)
    scales = GOLDEN[f"tile_{name}_scales"].reshape(rows, cols // 128)
    frag = {W2: 8, W3: 12, W4: 16}[fmt]
    groups = cols // 128
    for row in range(rows):
        for col in range(cols):
            tile, local_row = divmod(row, 16)
            group, k_tile, local_col = col // 128, (col % 128) // 32, col % 32
            base = (((tile * groups + group) * 4 + k_tile) * 16 + local_row) * frag
            if fmt == W3:
                bit = local_col * 3
                word = int(tiled[base + bit // 8]) | (int(tiled[base + bit // 8 + 1]) << 8 if bit // 8 + 1 < frag else 0)
                value = ((word >> (bit % 8)) & 7) - 4
            elif fmt == W4:
                code = (int(tiled[base + local_col // 2]) >> ((local_col % 2) * 4)) & 15
                value = code - 16 if code >= 8 else code
            else:
                code = (int(tiled[base + local_col // 4]) >> ((local_col % 4) * 2)) & 3
                value = code * 2 - 3
            assert value == q[row, col]
            assert tiled_scales[(tile * groups + group) * 16 + local_row] == scales[row, group]


@pytest.mark.skipif(not Reference.available(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("fmt", [W2, W3, W4])
def test_quantizer_matches_reference_build_random(oracle, fmt):
    ref = Reference()
    rng = np.random.default_rng(fmt)
    values = rng.normal(0.0, 0.02, size=(48, 1024)).astype(np.float32)
    values[3, :128] = 0.0
    _, codes_ref, scales_ref = ref.quantize(values, fmt)
    _, codes, scales = oracle.quantize(values, fmt)
    np.testing.assert_array_equal(codes, codes_ref)
    np.testing.assert_array_equal(scales, scales_ref)


def test_fp16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(7)
    samples = np.concatenate([
        rng.normal(0, 1, 20000), rng.normal(0, 3e4, 2000), rng.normal(0, 1e-5, 2000),
        rng.normal(0, 1e-7, 2000), [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 2**-24, 2**-25, 3 * 2**-26, np.inf, -np.inf],
    ]).astype(np.float32)
    expect = samples.astype(np.float16).view(np.uint16)
    got = np.array([oracle.lib.or_f32_to_f16(float(v)) for v in samples], np.uint16)
    np.testing.assert_array_equal(got, expect)
    halves = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    finite = halves[(halves & 0x7C00) != 0x7C00]
    back = np.array([oracle.lib.or_f16_to_f32(int(h)) for h in finite[::7]], np.float32)
    np.testing.assert_array_equal(back, finite[::7].view(np.float16).astype(np.float32))


def test_bf16_conversion_matches_torch(oracle):
    import torch

    rng = np.random.default_rng(8)
    samples = rng.normal(0, 1, 5000).astype(np.float32)
    expect = torch.from_numpy(samples).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([oracle.lib.or_f32_to_bf16(float(v)) for v in samples], np.uint16)
    np.testing.assert_array_equal(got, expect)


def _ulp_error(got, want):
    spacing = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    return np.abs(got.astype(np.float64) - want) / spacing


def test_exp_accuracy(oracle):
    xs = np.concatenate([np.linspace(-87, 88.5, 20001), np.random.default_rng(1).normal(0, 5, 5000)]).astype(np.float32)
    got = np.array([oracle.lib.or_expf(float(x)) for x in xs], np.float32)
    want = np.exp(xs.astype(np.float64))
    assert _ulp_error(got, want).max() <= 2.0
    assert oracle.lib.or_expf(-np.inf) == 0.0 and oracle.lib.or_expf(-200.0) == 0.0
    assert np.isinf(oracle.lib.or_expf(100.0))


def test_log1p_accuracy(oracle):
    xs = np.concatenate([np.exp(np.linspace(-30, 20, 20001)), [0.0, 1e-30, 1.0]]).astype(np.float32)
    got = np.array([oracle.lib.or_log1pf(float(x)) for x in xs], np.float32)
    want = np.log1p(xs.astype(np.float64))
    nonzero = want > 0
    assert _ulp_error(got[nonzero], want[nonzero]).max() <= 4.0


def _numpy_a4(x16):
    """Independent numpy restatement of lowbit_gemv.hip:373-407."""
    x = x16.astype(np.float32).reshape(x16.shape[0], -1, 128)
    amax = np.abs(x).max(axis=2)
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(7.0)).astype(np.float16)
    q = np.clip(np.rint(x / scale.astype(np.float32)[..., None]), -7, 7).astype(np.int8)
    return q.reshape(x16.shape), scale


def test_a4_quantizer_matches_numpy_restatement(oracle):
    rng = np.random.default_rng(11)
    x = rng.normal(0, 1.3, size=(5, 5120)).astype(np.float16)
    x[0, :128] = 0
    x[1, 128:256] = 0.5  # exact ties at x/s = 7 and rounding of half steps
    packed, scales, values = oracle.quantize_a4(x)
    q_np, s_np = _numpy_a4(x)
    np.testing.assert_array_equal(values, q_np)
    np.testing.assert_array_equal(scales.view(np.uint16), s_np.view(np.uint16))
    assert packed.shape == (5, 2560)
    assert np.all(scales[0, 0] == np.float16(1.0))


def test_a8_quantizer_matches_numpy_restatement(oracle):
    rng = np.random.default_rng(12)
    x = rng.normal(0, 2.0, size=(3, 1024)).astype(np.float16)
    q, scales = oracle.quantize_a8(x)
    xf = x.astype(np.float32).reshape(3, -1, 128)
    amax = np.abs(xf).max(axis=2)
    s = (amax / np.float32(127.0)).astype(np.float16)
    q_np = np.clip(np.rint(xf / s.astype(np.float32)[..., None]), -127, 127).astype(np.int8).reshape(3, 1024)
    np.testing.assert_array_equal(q, q_np)
    np.testing.assert_array_equal(scales, s)


def test_gemv_int_close_to_float64(oracle):
    rng = np.random.default_rng(5)
    w = rng.integers(-4, 4, size=(64, 1024), dtype=np.int8)
    ws = rng.uniform(0.002, 0.08, size=(64, 8)).astype(np.float16)
    x = rng.normal(0, 1, size=(3, 1024)).astype(np.float16)
    _, a_scales, a = oracle.quantize_a4(x)
    out = oracle.gemv(w, ws, a, a_scales)
    dots = (w.astype(np.int64).reshape(64, 8, 128)[None] * a.astype(np.int64).reshape(3, 1, 8, 128)).sum(-1)
    exact = (dots * ws.astype(np.float64)[None] * a_scales.astype(np.float64)[:, None, :]).sum(-1)
    np.testing.assert_allclose(out, exact, rtol=1e-5, atol=1e-5)


def test_argmax_lowest_index_on_ties(oracle):
    logits = np.array([1.0, 3.0, -2.0, 3.0, 3.0], np.float32)
    assert oracle.lib.or_argmax(logits.ctypes.data, 5) == 1
