"""GEMV parity on the GPU: the CUDA path through the C ABI vs the CPU oracle.

Bit-exact on activation codes/scales and on GEMV outputs (the kernel follows
the reference's per-group int32 dot + ordered fp32 fma chain), at BASELINE
config-0 size ([17408 x 5120] W3, weights N(0, 0.02) packed by the oracle's
restatement of the reference quantizer, fp16 scales, batch 1 and 5).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import W2, W3, W4  # noqa: E402


@pytest.fixture(scope="module")
def ops():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import ops as gops

    gops.require_sm100(0)
    return gops


def _quantized(oracle, rows, cols, fmt, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, std, size=(rows, cols)).astype(np.float32)
    status, codes, scales = oracle.quantize(w, fmt)
    assert status == 0
    scales16 = scales.astype(np.float16).reshape(rows, cols // 128)  # converter.cpp:385-386 (RNE)
    logical = oracle.logical(codes, rows, cols, fmt)
    return codes, scales16, logical


def _device_b200(ops, codes, scales16, rows, cols, fmt):
    d_codes = torch.from_numpy(codes).cuda()
    b200 = ops.repack_rowmajor(fmt, d_codes, rows, cols)
    tiled = ops.tile_scales(torch.from_numpy(scales16.reshape(-1).copy()).cuda(), rows, cols)
    return b200, tiled


def _activations(batch, cols, seed):
    rng = np.random.default_rng(seed)
    return rng.normal(0.0, 1.0, size=(batch, cols)).astype(np.float16)


def _run_gemv(ops, fmt, b200, tiled, rows, cols, x16, bits, f16_out=False):
    x = torch.from_numpy(x16).cuda()
    codes, scales, sums, _ = ops.pack_activation(x, bits)
    out = torch.empty((x16.shape[0], rows), dtype=torch.float16 if f16_out else torch.float32, device="cuda")
    ops.lowbit_gemv(fmt, [(b200, tiled, out, rows, f16_out)], codes, scales, sums, cols, x16.shape[0])
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("batch", [1, 5, 9])
@pytest.mark.parametrize("bits", [4, 8])
def test_config0_w3_gemv_bit_exact(oracle, ops, batch, bits):
    rows, cols = 17408, 5120
    codes, scales16, logical = _quantized(oracle, rows, cols, W3, seed=0)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, W3)
    x16 = _activations(batch, cols, seed=100 + batch)
    got = _run_gemv(ops, W3, b200, tiled, rows, cols, x16, bits)
    if bits == 4:
        _, a_scales, a = oracle.quantize_a4(x16)
    else:
        a, a_scales = oracle.quantize_a8(x16)
    want = oracle.gemv(logical, scales16, a, a_scales)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bits", [4, 8])
def test_activation_pack_bit_exact(oracle, ops, bits):
    x16 = _activations(7, 17408, seed=3)
    x16[0, :128] = 0
    x = torch.from_numpy(x16).cuda()
    codes, scales, sums, packed = ops.pack_activation(x, bits, want_packed_a4=(bits == 4))
    torch.cuda.synchronize()
    if bits == 4:
        want_packed, want_scales, want_values = oracle.quantize_a4(x16)
        np.testing.assert_array_equal(packed.cpu().numpy(), want_packed)
        ref_packed, ref_scales = ops.quantize_a4(x)
        np.testing.assert_array_equal(ref_packed.cpu().numpy(), want_packed)
        np.testing.assert_array_equal(ref_scales.cpu().numpy().view(np.uint16), want_scales.view(np.uint16))
    else:
        want_values, want_scales = oracle.quantize_a8(x16)
        ref_q, ref_scales = ops.quantize_a8(x)
        np.testing.assert_array_equal(ref_q.cpu().numpy(), want_values)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint16), want_scales.view(np.uint16))
    # fragment order: within each 128-group, k -> t*32 + s*8 + half*4 + j
    k = np.arange(128)
    offset = ((k & 15) >> 2) * 32 + (k >> 5) * 8 + ((k & 31) >> 4) * 4 + (k & 3)
    frag = codes.cpu().numpy().reshape(7, -1, 128)
    logical = np.empty_like(frag)
    logical[..., k] = frag[..., offset]
    np.testing.assert_array_equal(logical.reshape(7, -1), want_values)
    np.testing.assert_array_equal(sums.cpu().numpy(), want_values.reshape(7, -1, 128).astype(np.int32).sum(-1))


@pytest.mark.parametrize("fmt", [W2, W3, W4])
@pytest.mark.parametrize("batch", [1, 2, 8, 9, 17, 32])
def test_formats_and_batches_bit_exact(oracle, ops, fmt, batch):
    rows, cols = 96, 1152
    codes, scales16, logical = _quantized(oracle, rows, cols, fmt, seed=fmt * 31 + batch)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, fmt)
    x16 = _activations(batch, cols, seed=batch)
    for bits in (4, 8):
        got = _run_gemv(ops, fmt, b200, tiled, rows, cols, x16, bits)
        if bits == 4:
            _, a_scales, a = oracle.quantize_a4(x16)
        else:
            a, a_scales = oracle.quantize_a8(x16)
        want = oracle.gemv(logical, scales16, a, a_scales)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("cols", [128, 256, 1024 + 128])
def test_small_k_edges(oracle, ops, cols):
    rows = 16
    codes, scales16, logical = _quantized(oracle, rows, cols, W3, seed=cols)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, W3)
    x16 = _activations(3, cols, seed=cols)
    got = _run_gemv(ops, W3, b200, tiled, rows, cols, x16, 4)
    _, a_scales, a = oracle.quantize_a4(x16)
    np.testing.assert_array_equal(got, oracle.gemv(logical, scales16, a, a_scales))


def test_fused_multi_matrix_and_f16_output(oracle, ops):
    cols = 640
    shapes = [160, 48, 16, 96]
    mats = [_quantized(oracle, r, cols, W4, seed=50 + i) for i, r in enumerate(shapes)]
    dev = [_device_b200(ops, c, s, r, cols, W4) for (c, s, _), r in zip(mats, shapes)]
    x16 = _activations(4, cols, seed=9)
    x = torch.from_numpy(x16).cuda()
    codes, scales, sums, _ = ops.pack_activation(x, 4)
    outs = [torch.empty((4, r), dtype=torch.float16 if i == 1 else torch.float32, device="cuda")
            for i, r in enumerate(shapes)]
    ops.lowbit_gemv(W4, [(b, t, o, r, i == 1) for i, ((b, t), o, r) in enumerate(zip(dev, outs, shapes))],
                    codes, scales, sums, cols, 4)
    torch.cuda.synchronize()
    _, a_scales, a = oracle.quantize_a4(x16)
    for i, ((_, s16, logical), out) in enumerate(zip(mats, outs)):
        want = oracle.gemv(logical, s16, a, a_scales)
        got = out.cpu().numpy()
        if i == 1:
            np.testing.assert_array_equal(got.view(np.uint16), want.astype(np.float16).view(np.uint16))
        else:
            np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("fmt", [W2, W3, W4])
def test_reference_layout_dropins_bit_exact(oracle, ops, fmt):
    rows, cols, batch = 64, 512, 5
    codes, scales16, logical = _quantized(oracle, rows, cols, fmt, seed=77 + fmt)
    status, gfx12, gfx12_scales = oracle.tile(codes, scales16.astype(np.float32).reshape(-1), rows, cols, fmt)
    assert status == 0
    d_gfx12 = torch.from_numpy(gfx12).cuda()
    d_tiled_scales = torch.from_numpy(gfx12_scales.astype(np.float16)).cuda()
    # gfx12 -> b200 repack equals row-major -> b200 repack
    b200_a = ops.repack_gfx12(fmt, d_gfx12, rows, cols)
    b200_b, tiled_b = _device_b200(ops, codes, scales16, rows, cols, fmt)
    assert torch.equal(b200_a, b200_b)
    assert torch.equal(d_tiled_scales, tiled_b)
    x16 = _activations(batch, cols, seed=fmt)
    x = torch.from_numpy(x16).cuda()
    packed, a4_scales = ops.quantize_a4(x)
    got4 = ops.gfx12_i4_gemm(fmt, d_gfx12, d_tiled_scales, packed, a4_scales, rows, cols, batch)
    q8, a8_scales = ops.quantize_a8(x)
    got8 = ops.gfx12_i8_gemm(fmt, d_gfx12, d_tiled_scales, q8, a8_scales, rows, cols, batch)
    torch.cuda.synchronize()
    _, s4, a4 = oracle.quantize_a4(x16)
    a8, s8 = oracle.quantize_a8(x16)
    np.testing.assert_array_equal(got4.cpu().numpy(), oracle.gemv(logical, scales16, a4, s4))
    np.testing.assert_array_equal(got8.cpu().numpy(), oracle.gemv(logical, scales16, a8, s8))


# ---- fp16 activations (lowbit_gemv.hip:757-834) ------------------------------
# The reference accumulates fp16(q * scale) * x in fp32 on its matrix cores; the
# CUDA path does the same on the f16 tensor cores, so the summation order is
# the hardware's. Tolerance: |got - exact| <= 1e-3 * max(1, |exact|), the
# north-star bound for fp32-accumulated GEMV outputs (an fp32 accumulation of
# K = 17408 terms stays near 1e-6 relative).
F16_TOLERANCE = 1e-3


def _assert_f16_close(got, exact):
    err = np.abs(got.astype(np.float64) - exact) / np.maximum(1.0, np.abs(exact))
    assert err.max() <= F16_TOLERANCE, err.max()


@pytest.mark.parametrize("batch", [1, 5])
def test_config0_w3_f16_activation_gemv(oracle, ops, batch):
    rows, cols = 17408, 5120
    codes, scales16, logical = _quantized(oracle, rows, cols, W3, seed=0)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, W3)
    x16 = _activations(batch, cols, seed=300 + batch)
    out = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
    ops.lowbit_gemv_f16(W3, [(b200, tiled, out, rows, False)], torch.from_numpy(x16).cuda())
    torch.cuda.synchronize()
    _assert_f16_close(out.cpu().numpy(), oracle.gemv_f16(logical, scales16, x16))


@pytest.mark.parametrize("fmt", [W2, W3, W4])
@pytest.mark.parametrize("batch", [1, 3, 8, 9, 32])
def test_f16_activation_formats_batches_and_layouts(oracle, ops, fmt, batch):
    rows, cols = 80, 1280
    codes, scales16, logical = _quantized(oracle, rows, cols, fmt, seed=fmt * 7 + batch)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, fmt)
    x16 = _activations(batch, cols, seed=batch + 40)
    x = torch.from_numpy(x16).cuda()
    exact = oracle.gemv_f16(logical, scales16, x16)
    out32 = torch.empty((batch, 48), dtype=torch.float32, device="cuda")  # rows 0-47, fp32
    out16 = torch.empty((batch, 32), dtype=torch.float16, device="cuda")  # rows 48-79, fp16
    ops.lowbit_gemv_f16(fmt, [(b200, tiled, out32, 48, False), (b200[48 * cols * {1: 2, 2: 3, 3: 4}[fmt] // 8:],
                              tiled[48 * cols // 128:], out16, 32, True)], x)
    status, gfx12, gfx12_scales = oracle.tile(codes, scales16.astype(np.float32).reshape(-1), rows, cols, fmt)
    assert status == 0
    dropin = ops.gfx12_f16_gemm(fmt, torch.from_numpy(gfx12).cuda(),
                                torch.from_numpy(gfx12_scales.astype(np.float16)).cuda(), x, rows, cols, batch)
    torch.cuda.synchronize()
    _assert_f16_close(out32.cpu().numpy(), exact[:, :48])
    # fp16 outputs: the same bound plus the final rounding to fp16 (half an ulp, 2^-11 relative)
    half = out16.cpu().numpy().astype(np.float64)
    bound = F16_TOLERANCE * np.maximum(1.0, np.abs(exact[:, 48:])) + 2.0 ** -11 * np.abs(exact[:, 48:])
    assert (np.abs(half - exact[:, 48:]) <= bound).all()
    _assert_f16_close(dropin.cpu().numpy(), exact)


def test_f16_activation_rejects_bad_arguments(ops):
    from gfxinfer_b200 import GfxbError

    x = torch.zeros((1, 256), dtype=torch.float16, device="cuda")
    w = torch.zeros(16 * 256 // 2, dtype=torch.uint8, device="cuda")
    s = torch.zeros(16 * 2, dtype=torch.float16, device="cuda")
    with pytest.raises(GfxbError):
        ops.gfx12_f16_gemm(W4, w, s, x, 16, 255, 1)  # K not a multiple of 128
    with pytest.raises(GfxbError):
        ops.gfx12_f16_gemm(W4, w, s, x, 16, 256, 33)  # batch beyond 32
    with pytest.raises(GfxbError):
        ops.gfx12_f16_gemm(W4, w[1:], s, x, 16, 256, 1)  # misaligned weights


# ---- wide matrices: K split over a cluster ----------------------------------
# Long-K shapes with few 16-row tiles (the MLP down projection [5120 x 17408],
# the attention/GDN output projections [5120 x 6144]) split each tile's groups
# over a cluster of CTAs; the non-leader CTAs send their int32 dots to the
# leader with asynchronous shared-memory stores, and the leader runs the same
# ordered fp32 chain, so the outputs stay bit-identical to the oracle. From 3
# tokens on, the ranks instead pass the chain's accumulators along (two
# 8-token mma blocks beyond 8 tokens). The cases cover ragged splits (G = 131,
# G = 17), a single-tile matrix and 9 and 16 tokens.
@pytest.mark.parametrize("fmt,rows,cols,batch,bits", [
    (W3, 5120, 17408, 1, 4),
    (W3, 5120, 17408, 8, 4),
    (W4, 5120, 6144, 1, 4),
    (W4, 5120, 6144, 5, 8),
    (W2, 1024, 16768, 3, 8),
    (W4, 16, 2176, 2, 4),
    (W3, 1024, 17408, 9, 4),
    (W4, 5120, 6144, 16, 8),
])
def test_wide_k_bit_exact(oracle, ops, fmt, rows, cols, batch, bits):
    codes, scales16, logical = _quantized(oracle, rows, cols, fmt, seed=rows + cols + batch)
    b200, tiled = _device_b200(ops, codes, scales16, rows, cols, fmt)
    x16 = _activations(batch, cols, seed=cols + batch)
    got = _run_gemv(ops, fmt, b200, tiled, rows, cols, x16, bits)
    if bits == 4:
        _, a_scales, a = oracle.quantize_a4(x16)
    else:
        a, a_scales = oracle.quantize_a8(x16)
    np.testing.assert_array_equal(got.view(np.uint32), oracle.gemv(logical, scales16, a, a_scales).view(np.uint32))


@pytest.mark.parametrize("parts", ["1", "2", "4", "8", "pipe", "lean1", "lean2", "lean4", "lean8"])
def test_cluster_splits_bit_exact(parts):
    """Every cluster size of the streaming GEMV, the pipelined GEMV on every
    shape, and every split of the persistent single-token GEMV, in a fresh
    process (the choice is read once per process): G = 17 over 8 CTAs leaves
    two CTAs without groups; G = 136 and 131 stream each tile in several
    K-chunks; the persistent kernel runs several rounds of tiles per cluster."""
    import os
    import subprocess
    import sys

    if parts == "pipe":
        env = dict(os.environ, GFXB_GEMV_PIPE="2", GFXB_GEMV_LEAN="0")
    elif parts.startswith("lean"):
        env = dict(os.environ, GFXB_GEMV_LEAN_PARTS=parts[4:])
    else:
        env = dict(os.environ, GFXB_GEMV_PARTS=parts, GFXB_GEMV_LEAN="0")
    child = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gemv_split_child.py")
    result = subprocess.run([sys.executable, child], env=env, capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout + result.stderr
