"""The device weight packer and converter vs the reference's own packer.

* gfxb_quantize_group128 / gfxb_tile_group128_for_gfx12 on the golden vectors the
  reference's src/quantization.cpp produced (tests/golden/quantization_golden.npz: the
  matrices of tests/quantization_test.cpp and config-0-shaped slices): codes, fp32 scales
  and tiled bytes bit-exact.
* The full config-0 matrix ([17408 x 5120] W3, weights N(0, 0.02)): bit-exact against the
  oracle's restatement (pinned to the reference by the golden vectors) and, where the
  reference build travels with the repository, against the reference itself.
* dequantize_group128 / dequantized_weight, the reference's argument rejections (K % 128,
  non-finite weights, formats).
* The converter (write_quantized, converter.cpp:345-393): a model given as fp32 weights is
  converted into a b200-v1 artifact and into the reference's tiled recipe on the GPU. The
  tiled artifact is byte-identical, tensor for tensor, to one assembled on the CPU with the
  reference packing rules, and engines loaded from both artifacts decode identically.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import SMALL_MODEL, W2, W3, W4, Reference, model_config, prompt_tokens  # noqa: E402

GOLDEN = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quantization_golden.npz"))
FORMATS = {"w2": W2, "w3": W3, "w4": W4}


@pytest.fixture(scope="module")
def ops():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import ops as module

    module.require_sm100(0)
    return module


def _bf16_bits(values: np.ndarray) -> np.ndarray:
    bits = values.astype(np.float32).view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("name", sorted(FORMATS))
@pytest.mark.parametrize("kind", ["rmse", "tile", "slice"])
def test_quantizer_and_tiler_match_reference_golden(ops, name, kind):
    fmt = FORMATS[name]
    values = GOLDEN[f"{kind}_{name}_input"]
    rows, cols = values.shape
    codes, scales = ops.quantize_group128(fmt, torch.from_numpy(values).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), GOLDEN[f"{kind}_{name}_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy().reshape(-1).view(np.uint32),
                                  GOLDEN[f"{kind}_{name}_scales"].view(np.uint32))
    if kind != "rmse":
        tiled, tiled_scales = ops.tile_group128_for_gfx12(fmt, codes, scales, rows, cols)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tiled.cpu().numpy(), GOLDEN[f"{kind}_{name}_tiled"])
        np.testing.assert_array_equal(tiled_scales.cpu().numpy().reshape(-1).view(np.uint32),
                                      GOLDEN[f"{kind}_{name}_tiled_scales"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_bf16_input_equals_fp32_of_the_same_values(ops, oracle, name):
    fmt = FORMATS[name]
    rng = np.random.default_rng(7)
    bits = _bf16_bits(rng.normal(0, 0.02, (48, 384)))
    values = (bits.astype(np.uint32) << 16).view(np.float32)
    got_codes, got_scales = ops.quantize_group128(fmt, torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16))
    status, want_codes, want_scales = oracle.quantize(values, fmt)
    assert status == 0
    np.testing.assert_array_equal(got_codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(got_scales.cpu().numpy().reshape(-1).view(np.uint32), want_scales.view(np.uint32))


def test_config0_matrix_bit_exact(ops, oracle):
    """W fp32 N(0, 0.02) [17408 x 5120] packed to W3."""
    rows, cols = 17408, 5120
    values = (np.random.default_rng(0).standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    codes, scales = ops.quantize_group128(W3, torch.from_numpy(values).cuda())
    got_codes, got_scales = codes.cpu().numpy(), scales.cpu().numpy().reshape(-1)
    oracle.lib.or_set_threads(os.cpu_count() or 1)
    status, want_codes, want_scales = oracle.quantize(values, W3)
    assert status == 0
    np.testing.assert_array_equal(got_codes, want_codes)
    np.testing.assert_array_equal(got_scales.view(np.uint32), want_scales.view(np.uint32))
    if Reference.available():
        status, ref_codes, ref_scales = Reference().quantize(values, W3)
        assert status == 0
        np.testing.assert_array_equal(got_codes, ref_codes)
        np.testing.assert_array_equal(got_scales.view(np.uint32), ref_scales.view(np.uint32))


def _levels(codes_row: np.ndarray, fmt: int, cols: int) -> np.ndarray:
    if fmt == W2:
        c = np.stack([(codes_row >> (2 * k)) & 3 for k in range(4)], axis=1).reshape(-1)[:cols]
        return c.astype(np.int64) * 2 - 3
    if fmt == W4:
        c = np.stack([codes_row & 15, codes_row >> 4], axis=1).reshape(-1)[:cols].astype(np.int64)
        return np.where(c >= 8, c - 16, c)
    planes = codes_row.reshape(cols // 128, 3, 16)
    b = np.unpackbits(planes, axis=2, bitorder="little")
    return (b[:, 0] + 2 * b[:, 1] + 4 * b[:, 2]).reshape(-1).astype(np.int64) - 4


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_dequantize(ops, name):
    import ctypes

    from gfxinfer_b200 import lib

    fmt = FORMATS[name]
    codes, scales = GOLDEN[f"slice_{name}_codes"], GOLDEN[f"slice_{name}_scales"]
    rows, cols = GOLDEN[f"slice_{name}_input"].shape
    got = ops.dequantize_group128(fmt, torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda(), rows, cols)
    row_bytes = codes.size // rows
    want = np.stack([_levels(codes[r * row_bytes:(r + 1) * row_bytes], fmt, cols).astype(np.float32)
                     * np.repeat(scales.reshape(rows, -1)[r], 128) for r in range(rows)])
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    ptr = lambda a: a.ctypes.data  # noqa: E731
    for r, c in ((0, 0), (5, 129), (rows - 1, cols - 1)):
        assert lib().gfxb_dequantized_weight(fmt, ptr(codes), ptr(scales), rows, cols, r, c) == want[r, c]
        if Reference.available():
            assert Reference().lib.ref_dequantized_weight(ptr(codes), ptr(scales), rows, cols, fmt, r, c) == want[r, c]
    assert np.isnan(lib().gfxb_dequantized_weight(fmt, ptr(codes), ptr(scales), rows, cols, rows, 0))
    assert np.isnan(lib().gfxb_dequantized_weight(fmt, ptr(codes), ptr(scales), rows, cols, 0, cols))
    del ctypes


def test_rejections(ops):
    from gfxinfer_b200 import GfxbError

    with pytest.raises(GfxbError) as error:  # tests/quantization_test.cpp:126-132
        ops.quantize_group128(W4, torch.zeros((1, 127), device="cuda"))
    assert error.value.status == int(GOLDEN["k127_status"][0]) == 1
    bad = torch.zeros((16, 256), device="cuda")
    bad[3, 200] = float("nan")
    with pytest.raises(GfxbError) as error:
        ops.quantize_group128(W3, bad)
    assert error.value.status == 1 and "non-finite" in str(error.value)
    bad[3, 200] = float("inf")
    with pytest.raises(GfxbError):
        ops.convert_group128(W4, bad)
    with pytest.raises(GfxbError) as error:
        ops.quantize_group128(7, torch.zeros((16, 128), device="cuda"))
    assert error.value.status == 4
    # the quantizer still runs after a rejected call
    codes, _ = ops.quantize_group128(W4, torch.ones((16, 128), device="cuda"))
    assert codes.numel() == 16 * 64


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_convert_layouts(ops, name):
    """convert_group128 = quantize, then the engine's layout, then fp16 scales rounded to nearest even."""
    fmt = FORMATS[name]
    rows, cols = 64, 512
    values = torch.from_numpy(GOLDEN[f"slice_{name}_input"]).cuda()
    codes, scales = ops.quantize_group128(fmt, values)
    half = scales.reshape(-1).to(torch.float16)
    b200_codes, b200_scales = ops.convert_group128(fmt, values, ops.LAYOUT_B200)
    assert torch.equal(b200_codes, ops.repack_rowmajor(fmt, codes, rows, cols))
    assert torch.equal(b200_scales.view(torch.int16), ops.tile_scales(half, rows, cols).view(torch.int16))
    gfx12_codes, gfx12_scales = ops.convert_group128(fmt, values, ops.LAYOUT_GFX12)
    np.testing.assert_array_equal(gfx12_codes.cpu().numpy(), GOLDEN[f"slice_{name}_tiled"])
    np.testing.assert_array_equal(gfx12_scales.cpu().numpy(),
                                  GOLDEN[f"slice_{name}_tiled_scales"].astype(np.float16))
    row_codes, row_scales = ops.convert_group128(fmt, values, ops.LAYOUT_ROWMAJOR)
    assert torch.equal(row_codes, codes)
    assert torch.equal(row_scales.view(torch.int16), half.view(torch.int16))


def _fp32_model(cfg, include_mtp: bool) -> dict:
    """Every tensor of the model as fp32 (matrices N(0, 0.02); norm weights near 0, the GDN norm
    near 1, conv taps and gates in the synthetic ranges), with the reference names."""
    rng = np.random.default_rng(cfg.seed)
    H, I = cfg.hidden, cfg.intermediate
    nk, nv = cfg.gdn_key_heads * 128, cfg.gdn_value_heads * 128
    t = {}

    def mat(name, rows, cols):
        t[name] = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))

    def vec(name, shape, lo, hi):
        t[name] = rng.uniform(lo, hi, shape).astype(np.float32)

    def mlp(prefix):
        vec(prefix + "input_layernorm.weight", (H,), -0.1, 0.1)
        vec(prefix + "post_attention_layernorm.weight", (H,), -0.1, 0.1)
        mat(prefix + "mlp.gate_proj.weight", I, H)
        mat(prefix + "mlp.up_proj.weight", I, H)
        mat(prefix + "mlp.down_proj.weight", H, I)

    def attention(prefix):
        mat(prefix + "self_attn.q_proj.weight", cfg.q_heads * 512, H)
        mat(prefix + "self_attn.k_proj.weight", cfg.kv_heads * 256, H)
        mat(prefix + "self_attn.v_proj.weight", cfg.kv_heads * 256, H)
        mat(prefix + "self_attn.o_proj.weight", H, cfg.q_heads * 256)
        vec(prefix + "self_attn.q_norm.weight", (256,), -0.1, 0.1)
        vec(prefix + "self_attn.k_norm.weight", (256,), -0.1, 0.1)

    for i in range(cfg.layers):
        prefix = f"model.language_model.layers.{i}."
        mlp(prefix)
        if (i + 1) % cfg.attention_interval == 0:
            attention(prefix)
        else:
            p = prefix + "linear_attn."
            mat(p + "in_proj_qkv.weight", 2 * nk + nv, H)
            mat(p + "in_proj_z.weight", nv, H)
            mat(p + "in_proj_a.weight", cfg.gdn_value_heads, H)
            mat(p + "in_proj_b.weight", cfg.gdn_value_heads, H)
            mat(p + "out_proj.weight", H, nv)
            vec(p + "conv1d.weight", (2 * nk + nv, 1, 4), -0.5, 0.5)
            vec(p + "A_log", (cfg.gdn_value_heads,), -1.0, 1.0)
            vec(p + "dt_bias", (cfg.gdn_value_heads,), -1.0, 1.0)
            vec(p + "norm.weight", (128,), 0.8, 1.2)
    t["model.language_model.embed_tokens.weight"] = rng.standard_normal((cfg.vocab, H), dtype=np.float32)
    mat("lm_head.weight", cfg.vocab, H)
    vec("model.language_model.norm.weight", (H,), -0.1, 0.1)
    if include_mtp:
        mlp("mtp.layers.0.")
        attention("mtp.layers.0.")
        mat("mtp.fc.weight", H, 2 * H)
        for name in ("mtp.pre_fc_norm_embedding.weight", "mtp.pre_fc_norm_hidden.weight", "mtp.norm.weight"):
            vec(name, (H,), -0.1, 0.1)
    return t


def _cpu_tiled_artifact(oracle, tensors, path, mlp_bits, layers):
    """The reference's conversion on the CPU: choose_quantization (converter.cpp:98-119),
    quantize_group128 + tile_group128_for_gfx12 (the reference build when present, else the
    oracle's restatement), fp16 scales, bf16 for the rest, written with the reference recipe."""
    from gfxinfer_b200 import artifact as gx

    packer = Reference() if Reference.available() else oracle
    out = []
    for name, values in sorted(tensors.items()):
        if values.ndim == 2 and values.shape[0] % 16 == 0 and values.shape[1] % 128 == 0:
            fmt = W4
            if name.startswith("model.language_model.layers.") and ".mlp." in name:
                fmt = {2: W2, 3: W3, 4: W4}[mlp_bits]
            rows, cols = values.shape
            status, codes, scales = packer.quantize(values, fmt)
            assert status == 0
            status, tiled, tiled_scales = packer.tile(codes, scales, rows, cols, fmt)
            assert status == 0
            out.append(gx.TensorWrite(name, gx.DTYPE_U8, fmt, (rows, cols), tiled, tiled_scales.astype(np.float16)))
        else:
            out.append(gx.TensorWrite(name, gx.DTYPE_BF16, gx.QUANT_NONE, values.shape, _bf16_bits(values)))
    gx.write(path, {"target_arch": "gfx1200", "model_id": "qwen-hybrid", "weights_id": "fp32-seeded",
                    "recipe_id": "qwen-w3seq-w4-tiled-v9"}, out)


@pytest.mark.parametrize("mlp_bits", [3, 2])
def test_converted_artifacts_decode_identically(ops, oracle, tmp_path, mlp_bits):
    from gfxinfer_b200 import artifact as gx
    from gfxinfer_b200 import session as gs

    cfg = model_config(**dict(SMALL_MODEL, mlp_bits=mlp_bits))
    tensors = _fp32_model(cfg, include_mtp=True)
    ident = {"target_arch": "gfx1200", "model_id": "qwen-hybrid", "weights_id": "fp32-seeded",
             "recipe_id": "qwen-w3seq-w4-tiled-v9"}
    gpu_tiled, cpu_tiled, gpu_b200 = tmp_path / "gpu-tiled.gfxi", tmp_path / "cpu-tiled.gfxi", tmp_path / "b200.gfxi"
    gx.convert(gpu_tiled, ident, tensors, layout=gx.LAYOUT_GFX12, mlp_bits=mlp_bits, chunk_rows=256)
    gx.convert(gpu_b200, dict(ident, target_arch="sm_100a", recipe_id="b200-v1"), tensors, layout=gx.LAYOUT_B200,
               mlp_bits=mlp_bits, chunk_rows=512)
    _cpu_tiled_artifact(oracle, tensors, cpu_tiled, mlp_bits, cfg.layers)
    with gx.Artifact(gpu_tiled) as a, gx.Artifact(cpu_tiled) as b:
        ta, tb = a.tensors(), b.tensors()
        assert [t.name for t in ta] == [t.name for t in tb]
        for x, y in zip(ta, tb):
            assert (x.dtype, x.quantization, x.dimensions) == (y.dtype, y.quantization, y.dimensions), x.name
            assert np.array_equal(x.data, y.data), x.name
            assert (x.aux is None) == (y.aux is None) and (x.aux is None or np.array_equal(x.aux, y.aux)), x.name
    engines = [gs.Engine.from_artifact(p, max_context=cfg.max_context, draft_vocab=cfg.draft_vocab)
               for p in (gpu_b200, gpu_tiled, cpu_tiled)]
    assert engines[0].config.mlp_bits == mlp_bits
    prompt = prompt_tokens(oracle, cfg.seed + 5, cfg.vocab, 6)
    results = []
    for engine in engines:
        session = gs.QwenDecodeSession.create(engine)
        token, drafts = None, []
        for t in prompt:
            token = session.greedy_step(t)
            drafts.append(session.mtp_draft(token))  # the MTP draft follows every committed token
        stream = []
        for _ in range(24):
            stream.append(token)
            token = session.greedy_step(token)
            drafts.append(session.mtp_draft(token))  # the MTP draft follows every committed token
        results.append((stream, drafts, session.read_state(cfg.vocab)))
        session.close()
    for stream, drafts, (hidden, logits) in results[1:]:
        assert stream == results[0][0] and drafts == results[0][1]
        np.testing.assert_array_equal(hidden, results[0][2][0])
        np.testing.assert_array_equal(logits.view(np.uint32), results[0][2][1].view(np.uint32))
    assert len(set(results[0][0])) > 4
    for engine in engines:
        engine.close()
