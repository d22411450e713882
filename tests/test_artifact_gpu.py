"""Engines built from `.gfxi` artifacts (Engine::create, engine.cpp:62-216) must
decode exactly like the engine whose weights they carry.

1. Export/import: a synthetic engine is written as a "b200-v1" artifact and
   loaded again; tokens, final hidden state, logits and MTP drafts are
   compared bit for bit.
2. Reference recipe: an artifact in the reference's own layout (gfx12 tiled
   2-D tensors with sequential W3 fragments, quantization.cpp:253-318; fp16
   tiled scales; bf16 vectors; reference tensor names, qwen38_spec.cpp:32-102)
   is assembled on the CPU from the oracle's synthetic generator and tiler,
   then loaded (repacked to the B200 layout on the device): it must decode
   exactly like the synthetic engine with the same seed.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import SMALL_MODEL, model_config, prompt_tokens  # noqa: E402

# tensor kinds (shared by the engine's and the oracle's synthetic generators)
K = dict(input_norm=0, post_norm=1, gate=2, up=3, down=4, qkv=5, z=6, a=7, b=8, conv=9, a_log=10, dt_bias=11,
         gdn_norm=12, gdn_out=13, q=14, k=15, v=16, q_norm=17, k_norm=18, o=19, fc=20, pre_emb_norm=21,
         pre_hidden_norm=22, mtp_final_norm=23)
LAYER_GLOBAL, LAYER_MTP = 4096, 4097
BITS_TO_QUANT = {2: 1, 3: 2, 4: 3}


def _tid(layer, kind):
    return layer * 32 + (K[kind] if isinstance(kind, str) else kind)


def _stream(step, prompt, steps):
    token = None
    for t in prompt:
        token = step(t)
    out = []
    for _ in range(steps):
        out.append(token)
        token = step(token)
    return out


@pytest.fixture(scope="module")
def gs():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import session

    return session


def _compare(gs, oracle, a, b, cfg, steps=24):
    sa = gs.QwenDecodeSession.create(a)
    sb = gs.QwenDecodeSession.create(b)
    prompt = prompt_tokens(oracle, cfg.seed + 11, cfg.vocab, 5)
    assert _stream(sa.greedy_step, prompt, steps) == _stream(sb.greedy_step, prompt, steps)
    ha, la = sa.read_state(cfg.vocab)
    hb, lb = sb.read_state(cfg.vocab)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
    return sa, sb


def test_export_then_load_decodes_identically(gs, oracle, tmp_path):
    cfg = model_config(**SMALL_MODEL)
    synthetic = gs.Engine.create(gs.model_config(**SMALL_MODEL), include_mtp=True)
    path = tmp_path / "small.gfxi"
    synthetic.export_artifact(path, "seeded-5eed")
    from gfxinfer_b200 import artifact

    with artifact.Artifact(path) as a:
        ident = a.identity()
        assert ident == {"target_arch": "sm_100a", "model_id": "qwen-hybrid", "weights_id": "seeded-5eed",
                         "recipe_id": "b200-v1"}
        names = [t.name for t in a.tensors()]
        assert names == sorted(names)
        assert "model.language_model.layers.3.self_attn.q_proj.weight" in names
        assert "model.language_model.layers.0.linear_attn.in_proj_qkv.weight" in names
        assert "mtp.fc.weight" in names
    loaded = gs.Engine.from_artifact(path, max_context=cfg.max_context, draft_vocab=cfg.draft_vocab)
    for field in ("hidden", "intermediate", "layers", "attention_interval", "gdn_key_heads", "gdn_value_heads",
                  "q_heads", "kv_heads", "vocab", "draft_vocab", "mlp_bits", "proj_bits", "head_bits", "emb_bits"):
        assert getattr(loaded.config, field) == getattr(cfg, field), field
    assert loaded.weight_bytes() == synthetic.weight_bytes()
    _compare(gs, oracle, synthetic, loaded, cfg)
    _compare_drafts(gs, oracle, synthetic, loaded, cfg)
    synthetic.close()
    loaded.close()


def _compare_drafts(gs, oracle, a, b, cfg):
    """MTP drafts along a greedy stream (the draft follows every committed token)."""
    sa = gs.QwenDecodeSession.create(a)
    sb = gs.QwenDecodeSession.create(b)
    for t in prompt_tokens(oracle, cfg.seed + 12, cfg.vocab, 6):
        na, nb = sa.greedy_step(t), sb.greedy_step(t)
        assert na == nb
        assert sa.mtp_draft(na) == sb.mtp_draft(nb)


def _reference_artifact(oracle, cfg, path, include_mtp):
    """The synthetic model in the reference's tiled recipe, built on the CPU."""
    from gfxinfer_b200 import artifact as gx

    seed = cfg.seed
    tensors = []

    def matrix(name, tensor, rows, cols, bits):
        fmt = BITS_TO_QUANT[bits]
        codes = np.zeros(rows * oracle.lib.or_packed_row_bytes(fmt, cols), np.uint8)
        oracle.lib.or_gen_codes_rowmajor(seed, tensor, rows, cols, fmt, codes.ctypes.data)
        scales16 = np.zeros(rows * (cols // 128), np.uint16)
        oracle.lib.or_gen_scales(seed, tensor, scales16.size, fmt, scales16.ctypes.data)
        scales = scales16.view(np.float16).astype(np.float32)
        status, tiled, tiled_scales = oracle.tile(codes, scales, rows, cols, fmt)
        assert status == 0
        tensors.append(gx.TensorWrite(name, gx.DTYPE_U8, fmt, (rows, cols), tiled, tiled_scales.astype(np.float16)))

    def bf16(name, tensor, shape, lo, hi):
        count = int(np.prod(shape))
        values = np.zeros(count, np.uint16)
        oracle.lib.or_gen_bf16(seed, tensor, count, lo, hi, values.ctypes.data)
        tensors.append(gx.TensorWrite(name, gx.DTYPE_BF16, gx.QUANT_NONE, tuple(shape), values))

    H, I = cfg.hidden, cfg.intermediate
    nk, nv = cfg.gdn_key_heads * 128, cfg.gdn_value_heads * 128

    def mlp(prefix, layer):
        bf16(prefix + "input_layernorm.weight", _tid(layer, "input_norm"), (H,), -0.1, 0.1)
        bf16(prefix + "post_attention_layernorm.weight", _tid(layer, "post_norm"), (H,), -0.1, 0.1)
        matrix(prefix + "mlp.gate_proj.weight", _tid(layer, "gate"), I, H, cfg.mlp_bits)
        matrix(prefix + "mlp.up_proj.weight", _tid(layer, "up"), I, H, cfg.mlp_bits)
        matrix(prefix + "mlp.down_proj.weight", _tid(layer, "down"), H, I, cfg.mlp_bits)

    def attention(prefix, layer):
        matrix(prefix + "self_attn.q_proj.weight", _tid(layer, "q"), cfg.q_heads * 512, H, cfg.proj_bits)
        matrix(prefix + "self_attn.k_proj.weight", _tid(layer, "k"), cfg.kv_heads * 256, H, cfg.proj_bits)
        matrix(prefix + "self_attn.v_proj.weight", _tid(layer, "v"), cfg.kv_heads * 256, H, cfg.proj_bits)
        matrix(prefix + "self_attn.o_proj.weight", _tid(layer, "o"), H, cfg.q_heads * 256, cfg.proj_bits)
        bf16(prefix + "self_attn.q_norm.weight", _tid(layer, "q_norm"), (256,), -0.1, 0.1)
        bf16(prefix + "self_attn.k_norm.weight", _tid(layer, "k_norm"), (256,), -0.1, 0.1)

    for i in range(cfg.layers):
        prefix = f"model.language_model.layers.{i}."
        mlp(prefix, i)
        if (i + 1) % cfg.attention_interval == 0:
            attention(prefix, i)
        else:
            p = prefix + "linear_attn."
            matrix(p + "in_proj_qkv.weight", _tid(i, "qkv"), 2 * nk + nv, H, cfg.proj_bits)
            matrix(p + "in_proj_z.weight", _tid(i, "z"), nv, H, cfg.proj_bits)
            matrix(p + "in_proj_a.weight", _tid(i, "a"), cfg.gdn_value_heads, H, cfg.proj_bits)
            matrix(p + "in_proj_b.weight", _tid(i, "b"), cfg.gdn_value_heads, H, cfg.proj_bits)
            matrix(p + "out_proj.weight", _tid(i, "gdn_out"), H, nv, cfg.proj_bits)
            bf16(p + "conv1d.weight", _tid(i, "conv"), (2 * nk + nv, 1, 4), -0.5, 0.5)
            bf16(p + "A_log", _tid(i, "a_log"), (cfg.gdn_value_heads,), -1.0, 1.0)
            bf16(p + "dt_bias", _tid(i, "dt_bias"), (cfg.gdn_value_heads,), -1.0, 1.0)
            bf16(p + "norm.weight", _tid(i, "gdn_norm"), (128,), 0.8, 1.2)
    matrix("model.language_model.embed_tokens.weight", _tid(LAYER_GLOBAL, 0), cfg.vocab, H, cfg.emb_bits)
    matrix("lm_head.weight", _tid(LAYER_GLOBAL, 2), cfg.vocab, H, cfg.head_bits)
    bf16("model.language_model.norm.weight", _tid(LAYER_GLOBAL, 1), (H,), -0.1, 0.1)
    if include_mtp:
        mlp("mtp.layers.0.", LAYER_MTP)
        attention("mtp.layers.0.", LAYER_MTP)
        matrix("mtp.fc.weight", _tid(LAYER_MTP, "fc"), H, 2 * H, cfg.proj_bits)
        bf16("mtp.pre_fc_norm_embedding.weight", _tid(LAYER_MTP, "pre_emb_norm"), (H,), -0.1, 0.1)
        bf16("mtp.pre_fc_norm_hidden.weight", _tid(LAYER_MTP, "pre_hidden_norm"), (H,), -0.1, 0.1)
        bf16("mtp.norm.weight", _tid(LAYER_MTP, "mtp_final_norm"), (H,), -0.1, 0.1)
    tensors.sort(key=lambda t: t.name)
    gx.write(path, {"target_arch": "gfx1200", "model_id": "qwen3.8-27b", "weights_id": "synthetic-5eed",
                    "recipe_id": "tiled-v9-w3seq"}, tensors)


@pytest.mark.parametrize("mlp_bits", [3, 2])
def test_reference_tiled_recipe_decodes_like_synthetic(gs, oracle, tmp_path, mlp_bits):
    kw = dict(SMALL_MODEL, mlp_bits=mlp_bits)
    cfg = model_config(**kw)
    path = tmp_path / "reference-layout.gfxi"
    _reference_artifact(oracle, cfg, path, include_mtp=True)
    synthetic = gs.Engine.create(gs.model_config(**kw), include_mtp=True)
    loaded = gs.Engine.from_artifact(path, max_context=cfg.max_context, draft_vocab=cfg.draft_vocab)
    assert loaded.config.mlp_bits == mlp_bits
    _compare(gs, oracle, synthetic, loaded, cfg)
    _compare_drafts(gs, oracle, synthetic, loaded, cfg)
    synthetic.close()
    loaded.close()


def test_artifact_errors(gs, oracle, tmp_path):
    from gfxinfer_b200 import GfxbError
    from gfxinfer_b200 import artifact as gx

    with pytest.raises(GfxbError) as error:
        gs.Engine.from_artifact(tmp_path / "missing.gfxi")
    assert error.value.status == 2  # io_error
    path = tmp_path / "foreign.gfxi"
    gx.write(path, {"target_arch": "gfx942", "model_id": "qwen3.8-27b", "weights_id": "w", "recipe_id": "tiled-v9"},
             [gx.TensorWrite("x", gx.DTYPE_U8, gx.QUANT_NONE, (1,), b"\0")])
    with pytest.raises(GfxbError) as error:
        gs.Engine.from_artifact(path)
    assert error.value.status == 4  # unsupported target
    path = tmp_path / "empty.gfxi"
    gx.write(path, {"target_arch": "sm_100a", "model_id": "qwen-hybrid", "weights_id": "w", "recipe_id": "b200-v1"},
             [gx.TensorWrite("x", gx.DTYPE_U8, gx.QUANT_NONE, (1,), b"\0")])
    with pytest.raises(GfxbError) as error:
        gs.Engine.from_artifact(path)
    assert error.value.status == 3  # corrupt: no embedding / LM head
