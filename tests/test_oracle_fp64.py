"""An independent float64 check of the oracle's GDN, attention, Q/K-norm + RoPE and RMSNorm.

The oracle's restatements of qwen_ops.hip are bit-exact against the kernels, so a
misreading shared by both would pass every bit-exact test. These tests restate the
reference formulas a second time, directly from the reference source, in float64
numpy (no shared code, no fp32 reduction orders) and require the oracle within
1e-3 relative, the north star's tolerance for GDN and attention outputs:

* gdn_recurrent_decode, qwen_ops.hip:263-411 (q/k L2 norms with the 1/sqrt(128)
  query scale, softplus threshold 20, decay exp(-exp(A_log) softplus(a + dt_bias)),
  beta sigmoid(b), S <- decay S + k (beta (v - S^T k))^T, out = S^T q, RMS norm with
  the unoffset weight, SiLU(z) gate), several tokens in a row;
* gdn_conv_update, qwen_ops.hip:219-261 (4-tap causal conv, SiLU);
* gated_attention_decode, qwen_ops.hip:698-766 (softmax over all cached positions,
  scale 1/16, sigmoid of the second half of each 512-wide q_proj head), including
  contexts that span many 128-position chunks;
* qk_rms_norm_rope, qwen_ops.hip:599-676 (RMS norm with the +1 weight offset,
  NeoX rotation of the first 64 dims, theta 1e7);
* residual_add_rms_norm, qwen_ops.hip:176-217.
"""
import numpy as np
import pytest

from oracle_lib import _ptr

TOLERANCE = 1e-3  # relative to the largest magnitude of the compared vector


def _bf16(rng, n, lo, hi):
    v = rng.uniform(lo, hi, n).astype(np.float32)
    bits = v.view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def _bf16_value(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _f16_value(bits):
    return bits.view(np.float16).astype(np.float64)


def _relative_error(got, want):
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def _softplus(x):
    return x if x > 20.0 else np.log1p(np.exp(x))


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def gdn_fp64(qkv, z, a, b, a_log, dt_bias, norm, state, nk, nv):
    """qwen_ops.hip:263-411 in float64; qkv [T][channels] fp16 bits, state [nv][128][128]."""
    head = 128
    key_elements = nk * head
    ratio = nv // nk
    S = state.astype(np.float64).copy()
    out = np.zeros((qkv.shape[0], nv * head))
    for t in range(qkv.shape[0]):
        x = _f16_value(qkv[t])
        for vh in range(nv):
            kh = vh // ratio
            q = x[kh * head:(kh + 1) * head]
            k = x[key_elements + kh * head:key_elements + (kh + 1) * head]
            v = x[2 * key_elements + vh * head:2 * key_elements + (vh + 1) * head]
            q = q / np.sqrt(np.sum(q * q) + 1e-6) * (1.0 / np.sqrt(128.0))
            k = k / np.sqrt(np.sum(k * k) + 1e-6)
            g = -np.exp(_bf16_value(a_log[vh:vh + 1])[0]) * _softplus(a[t, vh] + _bf16_value(dt_bias[vh:vh + 1])[0])
            decay, beta = np.exp(g), _sigmoid(float(b[t, vh]))
            S[vh] *= decay
            delta = (v - S[vh].T @ k) * beta
            S[vh] += np.outer(k, delta)
            mixed = S[vh].T @ q
            inv_rms = 1.0 / np.sqrt(np.mean(mixed * mixed) + 1e-6)
            zv = z[t, vh * head:(vh + 1) * head].astype(np.float64)
            out[t, vh * head:(vh + 1) * head] = mixed * inv_rms * _bf16_value(norm) * (zv * _sigmoid(zv))
    return out, S


@pytest.mark.parametrize("nk,nv,tokens", [(16, 48, 3), (2, 6, 8)])
def test_gdn_recurrent_matches_fp64(oracle, nk, nv, tokens):
    rng = np.random.default_rng(nk * 100 + tokens)
    channels = 2 * nk * 128 + nv * 128
    qkv = rng.normal(0, 1, (tokens, channels)).astype(np.float16).view(np.uint16)
    z = rng.normal(0, 1, (tokens, nv * 128)).astype(np.float32)
    a = rng.normal(0, 1, (tokens, nv)).astype(np.float32)
    b = rng.normal(0, 1, (tokens, nv)).astype(np.float32)
    a_log, dt_bias, norm = _bf16(rng, nv, -1, 1), _bf16(rng, nv, -1, 1), _bf16(rng, 128, 0.8, 1.2)
    state = rng.normal(0, 0.01, (nv, 128, 128)).astype(np.float32)
    got_state = state.copy()
    got = np.zeros((tokens, nv * 128), np.uint16)
    oracle.lib.or_gdn_recurrent(_ptr(qkv), _ptr(z), _ptr(a), _ptr(b), _ptr(a_log), _ptr(dt_bias), _ptr(norm),
                                _ptr(got_state), _ptr(got), None, None, None, nk, nv, tokens)
    want, want_state = gdn_fp64(qkv, z, a, b, a_log, dt_bias, norm, state, nk, nv)
    for t in range(tokens):
        for vh in range(nv):
            cols = slice(vh * 128, (vh + 1) * 128)
            assert _relative_error(_f16_value(got[t, cols]), want[t, cols]) <= TOLERANCE, (t, vh)
    for vh in range(nv):
        assert _relative_error(got_state[vh].astype(np.float64), want_state[vh]) <= TOLERANCE, vh


def test_gdn_conv_matches_fp64(oracle):
    rng = np.random.default_rng(5)
    channels, tokens = 10240, 4
    projected = rng.normal(0, 1, (tokens, channels)).astype(np.float32)
    weight = _bf16(rng, channels * 4, -0.5, 0.5)
    state = rng.normal(0, 1, (channels, 4)).astype(np.float16).view(np.uint16)
    got_state = state.copy()
    got = np.zeros((tokens, channels), np.uint16)
    oracle.lib.or_gdn_conv_update(_ptr(projected), _ptr(weight), _ptr(got_state), _ptr(got), None, channels, tokens)
    taps = _f16_value(state).reshape(channels, 4)
    w = _bf16_value(weight).reshape(channels, 4)
    for t in range(tokens):
        incoming = projected[t].astype(np.float16).astype(np.float64)  # the state holds fp16 inputs
        taps = np.concatenate([taps[:, 1:], incoming[:, None]], axis=1)
        conv = np.sum(taps * w, axis=1)
        want = conv * _sigmoid(conv)
        assert _relative_error(_f16_value(got[t]), want) <= TOLERANCE
    np.testing.assert_array_equal(_f16_value(got_state).reshape(channels, 4), taps)


def attention_fp64(query, gate, keys, values, count, q_heads, kv_heads):
    """qwen_ops.hip:698-766 in float64: full softmax over positions 0 .. count - 1."""
    group = q_heads // kv_heads
    out = np.zeros((q_heads, 256))
    for h in range(q_heads):
        kvh = h // group
        q = _f16_value(query[h])
        k = _f16_value(keys[:count, kvh])
        v = _f16_value(values[:count, kvh])
        scores = (k @ q) * 0.0625
        p = np.exp(scores - scores.max())
        out[h] = (p @ v) / p.sum() * _sigmoid(gate[h, 256:].astype(np.float64))
    return out


@pytest.mark.parametrize("count", [1, 127, 129, 700, 2048, 4095])
def test_gated_attention_matches_fp64(oracle, count):
    rng = np.random.default_rng(count)
    q_heads, kv_heads = 24, 4
    query = rng.normal(0, 1, (q_heads, 256)).astype(np.float16).view(np.uint16)
    gate = rng.normal(0, 1, (q_heads, 512)).astype(np.float32)
    keys = rng.normal(0, 1, (count, kv_heads, 256)).astype(np.float16).view(np.uint16)
    values = rng.normal(0, 1, (count, kv_heads, 256)).astype(np.float16).view(np.uint16)
    got = np.zeros((q_heads, 256), np.uint16)
    oracle.lib.or_gated_attention(_ptr(query), _ptr(gate), _ptr(keys), _ptr(values), count, q_heads, kv_heads,
                                  _ptr(got))
    want = attention_fp64(query, gate, keys, values, count, q_heads, kv_heads)
    for h in range(q_heads):
        assert _relative_error(_f16_value(got[h]), want[h]) <= TOLERANCE, h


def test_qk_norm_rope_matches_fp64(oracle):
    rng = np.random.default_rng(9)
    heads, stride, positions, rotary = 24, 512, 64, 64
    x = rng.normal(0, 1, (heads, stride)).astype(np.float32)
    weight = _bf16(rng, 256, -0.1, 0.1)
    cos = np.zeros((positions, rotary // 2), np.float32)
    sin = np.zeros_like(cos)
    oracle.lib.or_rope_table(positions, rotary, 1.0e7, _ptr(cos), _ptr(sin))
    for position in (0, 1, 37, 63):
        got = np.zeros((heads, 256), np.uint16)
        oracle.lib.or_qk_norm_rope(_ptr(x), stride, _ptr(weight), heads, position, _ptr(cos), _ptr(sin), rotary,
                                   _ptr(got))
        for h in range(heads):
            v = x[h, :256].astype(np.float64)
            n = v / np.sqrt(np.mean(v * v) + 1e-6) * (1.0 + _bf16_value(weight))
            inv_freq = 1.0e7 ** (-np.arange(0, rotary, 2, dtype=np.float64) / rotary)
            angle = position * inv_freq
            first, second = n[:rotary // 2].copy(), n[rotary // 2:rotary].copy()
            n[:rotary // 2] = first * np.cos(angle) - second * np.sin(angle)
            n[rotary // 2:rotary] = second * np.cos(angle) + first * np.sin(angle)
            assert _relative_error(_f16_value(got[h]), n) <= TOLERANCE, (position, h)


def test_residual_rms_norm_matches_fp64(oracle):
    rng = np.random.default_rng(11)
    n = 5120
    residual = rng.normal(0, 1, n).astype(np.float16).view(np.uint16)
    update = rng.normal(0, 1, n).astype(np.float32)
    weight = _bf16(rng, n, -0.1, 0.1)
    got_residual = np.zeros(n, np.uint16)
    got = np.zeros(n, np.uint16)
    oracle.lib.or_residual_add_rms_norm(_ptr(residual), _ptr(update), _ptr(weight), n, 1e-6, 1, _ptr(got_residual),
                                        _ptr(got))
    summed = (_f16_value(residual) + update.astype(np.float64)).astype(np.float16).astype(np.float64)
    np.testing.assert_array_equal(_f16_value(got_residual), summed)
    want = summed / np.sqrt(np.mean(summed * summed) + 1e-6) * (1.0 + _bf16_value(weight))
    assert _relative_error(_f16_value(got), want) <= TOLERANCE
