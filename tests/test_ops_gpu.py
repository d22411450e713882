"""Operator parity on the GPU through the C ABI vs the CPU oracle (bit-exact).

Covers BASELINE config 1 (one Gated-DeltaNet decode step: 16 key / 48 value
heads x 128, conv width 4, state N(0, 0.01), a/b logits N(0, 1)), a 32-token
verifier block with rollback logs and the replay of accepted prefixes, gated
attention across chunk boundaries, Q/K RMSNorm + RoPE + KV append, the fused
residual/RMSNorm/A4 pack and SiLU/A4 pack.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import _ptr  # noqa: E402


@pytest.fixture(scope="module")
def lib():
    from gfxinfer_b200 import build

    build.build()
    import gfxinfer_b200
    from gfxinfer_b200 import ops

    ops.require_sm100(0)
    return gfxinfer_b200


_KEEP: list = []


def _dev(a: np.ndarray) -> torch.Tensor:
    """Device copy that stays alive until the test ends (a bare data_ptr() does not keep a tensor alive)."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def _host(a: np.ndarray) -> np.ndarray:
    """Contiguous host copy that stays alive until the test ends."""
    c = np.ascontiguousarray(a).copy()
    _KEEP.append(c)
    return c


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def _p(t):
    return 0 if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _bf16(rng, n, lo, hi):
    v = rng.uniform(lo, hi, n).astype(np.float32)
    return (v.view(np.uint32) + 0x7FFF + ((v.view(np.uint32) >> 16) & 1) >> 16).astype(np.uint16)


def _gdn_inputs(rng, nk, nv, batch):
    channels = 2 * nk * 128 + nv * 128
    qkv = rng.normal(0, 1, (batch, channels)).astype(np.float16)
    z = rng.normal(0, 1, (batch, nv * 128)).astype(np.float32)
    a = rng.normal(0, 1, (batch, nv)).astype(np.float32)
    b = rng.normal(0, 1, (batch, nv)).astype(np.float32)
    a_log, dt_bias, norm = _bf16(rng, nv, -1, 1), _bf16(rng, nv, -1, 1), _bf16(rng, 128, 0.8, 1.2)
    state = rng.normal(0, 0.01, (nv, 128, 128)).astype(np.float32)
    return qkv, z, a, b, a_log, dt_bias, norm, state


def _oracle_gdn(oracle, inputs, nk, nv, batch, logs=False):
    qkv, z, a, b, a_log, dt_bias, norm, state = inputs
    state = state.copy()
    out = np.zeros((batch, nv * 128), np.uint16)
    key_log = np.zeros((batch, nk * 128), np.float32) if logs else None
    delta_log = np.zeros((batch, nv * 128), np.float32) if logs else None
    decay_log = np.zeros((batch, nv), np.float32) if logs else None
    oracle.lib.or_gdn_recurrent(_ptr(qkv), _ptr(z), _ptr(a), _ptr(b), _ptr(a_log), _ptr(dt_bias), _ptr(norm),
                                _ptr(state), _ptr(out), _ptr(key_log), _ptr(delta_log), _ptr(decay_log), nk, nv, batch)
    return out, state, key_log, delta_log, decay_log


def _gpu_gdn(lib, inputs, nk, nv, batch, logs=False):
    qkv, z, a, b, a_log, dt_bias, norm, state = [_dev(x) for x in inputs]
    final = torch.empty_like(state)
    out = torch.empty((batch, nv * 128), dtype=torch.float16, device="cuda")
    key_log = torch.zeros((batch, nk * 128), device="cuda") if logs else None
    delta_log = torch.zeros((batch, nv * 128), device="cuda") if logs else None
    decay_log = torch.zeros((batch, nv), device="cuda") if logs else None
    lib.check(lib.lib().gfxb_gdn_recurrent(_p(qkv), _p(z), _p(a), _p(b), _p(a_log), _p(dt_bias), _p(norm), _p(state),
                                           _p(final), _p(out), _p(key_log), _p(delta_log), _p(decay_log), nk, nv, batch,
                                           _stream()))
    torch.cuda.synchronize()
    cpu = lambda t: None if t is None else t.cpu().numpy()  # noqa: E731
    return cpu(out).view(np.uint16), cpu(final), cpu(key_log), cpu(delta_log), cpu(decay_log)


@pytest.mark.parametrize("batch", [1, 3, 16, 17, 32])  # 2 to 16 tokens: the three-phase block form
def test_gdn_recurrent_config1_bit_exact(oracle, lib, batch):
    nk, nv = 16, 48
    rng = np.random.default_rng(batch)
    inputs = _gdn_inputs(rng, nk, nv, batch)
    want = _oracle_gdn(oracle, inputs, nk, nv, batch, logs=True)
    got = _gpu_gdn(lib, inputs, nk, nv, batch, logs=True)
    for w, g in zip(want, got):
        np.testing.assert_array_equal(np.asarray(g).view(np.uint32 if g.dtype == np.float32 else np.uint16),
                                      np.asarray(w).view(np.uint32 if w.dtype == np.float32 else np.uint16))


@pytest.mark.parametrize("accepted", [1, 6, 32])
def test_gdn_rollback_replay_equals_prefix_forward(oracle, lib, accepted):
    """Replaying `accepted` logged tokens onto the pre-block state equals running those tokens forward
    (qwen_ops.hip:467-539; the verifier's 32-token block with rollback)."""
    nk, nv, batch = 4, 12, 32
    rng = np.random.default_rng(100 + accepted)
    inputs = _gdn_inputs(rng, nk, nv, batch)
    channels = 2 * nk * 128 + nv * 128
    projected = rng.normal(0, 1, (batch, channels)).astype(np.float32)
    conv_w = _bf16(rng, channels * 4, -0.5, 0.5)
    conv_state = rng.normal(0, 1, (channels, 4)).astype(np.float16)
    # forward over the whole block on the GPU, with logs
    d_proj, d_w, d_conv = _dev(projected), _dev(conv_w), _dev(conv_state.view(np.uint16))
    conv_final = torch.empty_like(d_conv)
    conv_out = torch.empty((batch, channels), dtype=torch.int16, device="cuda")
    conv_log = torch.empty((batch, channels), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_gdn_conv_update(_p(d_proj), _p(d_w), _p(d_conv), _p(conv_final), _p(conv_out),
                                             _p(conv_log), channels, batch, _stream()))
    _, _, key_log, delta_log, decay_log = _gpu_gdn(lib, inputs, nk, nv, batch, logs=True)
    # replay the accepted prefix onto the untouched initial states
    states = _dev(inputs[7])
    conv_states = _dev(conv_state.view(np.uint16))
    lib.check(lib.lib().gfxb_gdn_restore_prefix_all(_p(conv_states), _p(states), _p(conv_log), _p(_dev(key_log)),
                                                    _p(_dev(delta_log)), _p(_dev(decay_log)), channels, nk, nv, 1,
                                                    batch, accepted, _stream()))
    torch.cuda.synchronize()
    # reference: the oracle forward over only the accepted tokens
    prefix = [_host(x[:accepted]) for x in inputs[:4]] + list(inputs[4:])
    _, want_state, _, _, _ = _oracle_gdn(oracle, prefix, nk, nv, accepted)
    np.testing.assert_array_equal(states.cpu().numpy().view(np.uint32), want_state.view(np.uint32))
    want_conv = conv_state.view(np.uint16).copy()
    out = np.zeros((accepted, channels), np.uint16)
    oracle.lib.or_gdn_conv_update(_ptr(_host(projected[:accepted])), _ptr(conv_w), _ptr(want_conv), _ptr(out), None,
                                  channels, accepted)
    np.testing.assert_array_equal(conv_states.cpu().numpy().view(np.uint16), want_conv)


def test_gdn_conv_bit_exact(oracle, lib):
    rng = np.random.default_rng(5)
    channels, batch = 10240, 5
    projected = rng.normal(0, 2, (batch, channels)).astype(np.float32)
    weight = _bf16(rng, channels * 4, -0.5, 0.5)
    state = rng.normal(0, 1, (channels, 4)).astype(np.float16).view(np.uint16)
    want_state, want_out, want_log = state.copy(), np.zeros((batch, channels), np.uint16), np.zeros((batch, channels), np.uint16)
    oracle.lib.or_gdn_conv_update(_ptr(projected), _ptr(weight), _ptr(want_state), _ptr(want_out), _ptr(want_log),
                                  channels, batch)
    d_state = _dev(state)
    out = torch.empty((batch, channels), dtype=torch.int16, device="cuda")
    log = torch.empty((batch, channels), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_gdn_conv_update(_p(_dev(projected)), _p(_dev(weight)), _p(d_state), _p(d_state), _p(out),
                                             _p(log), channels, batch, _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d_state.cpu().numpy(), want_state)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), want_out)
    np.testing.assert_array_equal(log.cpu().numpy().view(np.uint16), want_log)


def _attention_case(rng, capacity, q_heads=24, kv_heads=4, batch=3):
    query = rng.normal(0, 1, (batch, q_heads, 256)).astype(np.float16)
    gate = rng.normal(0, 1, (batch, q_heads, 512)).astype(np.float32)
    keys = rng.normal(0, 1, (capacity, kv_heads, 256)).astype(np.float16)
    values = rng.normal(0, 1, (capacity, kv_heads, 256)).astype(np.float16)
    return query, gate, keys, values


def _oracle_attention(oracle, case, base_count, q_heads=24, kv_heads=4):
    query, gate, keys, values = case
    outs = []
    for t in range(query.shape[0]):
        out = np.zeros((q_heads, 256), np.uint16)
        oracle.lib.or_gated_attention(_ptr(_host(query[t])), _ptr(_host(gate[t])), _ptr(keys), _ptr(values),
                                      base_count + t, q_heads, kv_heads, _ptr(out))
        outs.append(out)
    return np.stack(outs)


def gpu_attention(lib, case, base_count, capacity, q_heads=24, kv_heads=4):
    query, gate, keys, values = case
    batch = query.shape[0]
    scratch_bytes = lib.lib().gfxb_gated_attention_scratch_bytes(q_heads, capacity, batch)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((batch, q_heads, 256), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_gated_attention(_p(_dev(query)), _p(_dev(gate)), _p(_dev(keys)), _p(_dev(values)), _p(out),
                                             base_count, None, capacity, q_heads, kv_heads, batch, _p(scratch),
                                             scratch_bytes, _stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("base_count", [1, 100, 128, 129, 300, 509])
def test_gated_attention_bit_exact(oracle, lib, base_count):
    capacity = 512
    case = _attention_case(np.random.default_rng(base_count), capacity)
    np.testing.assert_array_equal(gpu_attention(lib, case, base_count, capacity), _oracle_attention(oracle, case, base_count))


@pytest.mark.parametrize("base_count,batch", [(2047, 3), (2048, 3), (3968, 32), (4095, 2)])
def test_gated_attention_long_context_bit_exact(oracle, lib, base_count, batch):
    """Configs 3 and 4 (contexts 2048 and 4096): up to 32 chunks merged per head, and a 32-token
    verifier block ending at the last cache slot."""
    capacity = 4096
    case = _attention_case(np.random.default_rng(base_count), capacity, batch=batch)
    np.testing.assert_array_equal(gpu_attention(lib, case, base_count, capacity),
                                  _oracle_attention(oracle, case, base_count))


def test_gated_attention_device_position_long_context(oracle, lib):
    """The graph-capture form (first position read from device memory, grid sized by the capacity)
    at capacity 4096 equals the host-count form and the oracle."""
    capacity, base_count = 4096, 3000
    case = _attention_case(np.random.default_rng(77), capacity, batch=4)
    query, gate, keys, values = case
    scratch_bytes = lib.lib().gfxb_gated_attention_scratch_bytes(24, capacity, 4)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((4, 24, 256), dtype=torch.int16, device="cuda")
    position = _dev(np.array([base_count - 1], np.uint64))
    lib.check(lib.lib().gfxb_gated_attention(_p(_dev(query)), _p(_dev(gate)), _p(_dev(keys)), _p(_dev(values)),
                                             _p(out), 0, _p(position), capacity, 24, 4, 4, _p(scratch),
                                             scratch_bytes, _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), _oracle_attention(oracle, case, base_count))


def _argmax_cases(vocab):
    """Rows of logits with planted maxima; the lowest index among equal maxima must win
    (qwen_ops.hip:782, 794-796). The kernel reads index i in block (i / 256) % 64, so ties are
    planted across blocks, across the strided passes of one block, and at the first and last index."""
    rng = np.random.default_rng(3)
    rows = []
    base = rng.normal(0, 1, vocab).astype(np.float32)
    r = base.copy(); r[[7, 300, 16391, vocab - 1]] = 9.0; rows.append(r)                # across blocks and passes
    r = base.copy(); r[[0, vocab - 1]] = 9.0; rows.append(r)                            # first and last
    r = base.copy(); r[vocab - 1] = 9.0; rows.append(r)                                 # last alone
    rows.append(np.zeros(vocab, np.float32))                                            # all equal
    rows.append(np.full(vocab, -np.inf, np.float32))                                    # all -inf
    r = base.copy(); r[::5] = np.nan; r[[1001, 99999]] = 9.0; r[0] = np.nan; rows.append(r)  # NaNs ignored
    r = base.copy(); r[[16383, 16384]] = 9.0; rows.append(r)                            # block 63 vs block 0, 2nd stride
    r = base.copy(); r[[255, 256]] = 9.0; rows.append(r)                                # adjacent blocks
    r = base.copy(); r[np.arange(64) * 256 + 17] = 9.0; rows.append(r)                  # one tie in every block
    r = np.full(vocab, np.nan, np.float32); rows.append(r)                              # all NaN
    return np.stack(rows)


def test_argmax_ties_lowest_index_bit_exact(oracle, lib):
    vocab, stride = 151936, 151936 + 64
    logits = _argmax_cases(vocab)
    batch = logits.shape[0]
    padded = np.full((batch, stride), 100.0, np.float32)  # the row padding must never be read
    padded[:, :vocab] = logits
    scratch_bytes = lib.lib().gfxb_argmax_scratch_bytes(batch)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device="cuda")
    ids = np.arange(vocab, dtype=np.uint32)[::-1].copy()
    for mapped in (False, True):
        tokens = torch.zeros(batch, dtype=torch.int32, device="cuda")
        lib.check(lib.lib().gfxb_argmax(_p(_dev(padded)), _p(_dev(ids)) if mapped else None, _p(tokens), vocab,
                                        stride, batch, _p(scratch), scratch_bytes, _stream()))
        torch.cuda.synchronize()
        got = tokens.cpu().numpy().view(np.uint32)
        want = np.array([oracle.lib.or_argmax(_ptr(_host(row)), vocab) for row in logits], np.uint32)
        assert list(want[:8]) == [7, 0, vocab - 1, 0, 0, 1001, 16383, 255]
        np.testing.assert_array_equal(got, ids[want] if mapped else want)


def test_qk_norm_rope_and_kv_append_bit_exact(oracle, lib):
    rng = np.random.default_rng(9)
    q_heads, k_heads, batch, position, capacity = 24, 4, 3, 77, 128
    q_in = rng.normal(0, 1, (batch, q_heads, 512)).astype(np.float32)
    k_in = rng.normal(0, 1, (batch, k_heads, 256)).astype(np.float32)
    v_in = rng.normal(0, 1, (batch, k_heads, 256)).astype(np.float32)
    qw, kw = _bf16(rng, 256, -0.1, 0.1), _bf16(rng, 256, -0.1, 0.1)
    cos = np.zeros((capacity, 32), np.float32)
    sin = np.zeros((capacity, 32), np.float32)
    lib.check(lib.lib().gfxb_rope_table(capacity, 64, ctypes.c_float(1e7), cos.ctypes.data, sin.ctypes.data))
    ocos, osin = np.zeros_like(cos), np.zeros_like(sin)
    oracle.lib.or_rope_table(capacity, 64, 1e7, _ptr(ocos), _ptr(osin))
    np.testing.assert_array_equal(cos, ocos)
    np.testing.assert_array_equal(sin, osin)
    q_out = torch.empty((batch, q_heads, 256), dtype=torch.int16, device="cuda")
    keys = torch.zeros((capacity, k_heads, 256), dtype=torch.int16, device="cuda")
    values = torch.zeros((capacity, k_heads, 256), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_qk_rms_norm_rope(_p(_dev(q_in)), _p(_dev(qw)), _p(q_out), q_heads, 512, _p(_dev(k_in)),
                                              _p(_dev(kw)), None, k_heads, 256, 64, _p(_dev(cos)), _p(_dev(sin)),
                                              capacity, position, None, batch, _p(_dev(v_in)), _p(keys), _p(values),
                                              capacity, _stream()))
    torch.cuda.synchronize()
    for t in range(batch):
        want_q = np.zeros((q_heads, 256), np.uint16)
        want_k = np.zeros((k_heads, 256), np.uint16)
        oracle.lib.or_qk_norm_rope(_ptr(_host(q_in[t])), 512, _ptr(qw), q_heads, position + t, _ptr(ocos), _ptr(osin), 64,
                                   _ptr(want_q))
        oracle.lib.or_qk_norm_rope(_ptr(_host(k_in[t])), 256, _ptr(kw), k_heads, position + t, _ptr(ocos), _ptr(osin), 64,
                                   _ptr(want_k))
        np.testing.assert_array_equal(q_out[t].cpu().numpy().view(np.uint16), want_q)
        np.testing.assert_array_equal(keys[position + t].cpu().numpy().view(np.uint16), want_k)
        np.testing.assert_array_equal(values[position + t].cpu().numpy().view(np.float16), v_in[t].astype(np.float16))


def _decode_attention_inputs(rng, capacity, q_heads=24, kv_heads=4, spread=1.0):
    """One decode step's projections and a filled cache; `spread` scales the query/key inputs (and with
    them the score range, so that the rescale factors underflow for large values)."""
    q_in = (rng.normal(0, 1, (q_heads, 512)) * spread).astype(np.float32)
    k_in = (rng.normal(0, 1, (kv_heads, 256)) * spread).astype(np.float32)
    v_in = rng.normal(0, 1, (kv_heads, 256)).astype(np.float32)
    qw, kw = _bf16(rng, 256, -0.5, 2.0), _bf16(rng, 256, -0.5, 2.0)
    keys = (rng.normal(0, 1, (capacity, kv_heads, 256)) * spread).astype(np.float16)
    values = rng.normal(0, 1, (capacity, kv_heads, 256)).astype(np.float16)
    return q_in, k_in, v_in, qw, kw, keys, values


def _rope(lib, capacity):
    cos = np.zeros((capacity, 32), np.float32)
    sin = np.zeros((capacity, 32), np.float32)
    lib.check(lib.lib().gfxb_rope_table(capacity, 64, ctypes.c_float(1e7), cos.ctypes.data, sin.ctypes.data))
    return cos, sin


def _three_launch_decode(lib, inputs, cos, sin, position, capacity, q_heads=24, kv_heads=4):
    q_in, k_in, v_in, qw, kw, keys, values = inputs
    d_keys, d_values = _dev(keys.view(np.int16)), _dev(values.view(np.int16))
    query = torch.empty((q_heads, 256), dtype=torch.int16, device="cuda")
    d_q = _dev(q_in)
    lib.check(lib.lib().gfxb_qk_rms_norm_rope(_p(d_q), _p(_dev(qw)), _p(query), q_heads, 512, _p(_dev(k_in)),
                                              _p(_dev(kw)), None, kv_heads, 256, 64, _p(_dev(cos)), _p(_dev(sin)),
                                              capacity, position, None, 1, _p(_dev(v_in)), _p(d_keys),
                                              _p(d_values), capacity, _stream()))
    scratch_bytes = lib.lib().gfxb_gated_attention_scratch_bytes(q_heads, capacity, 1)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((q_heads, 256), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_gated_attention(_p(query), _p(d_q), _p(d_keys), _p(d_values), _p(out), position + 1,
                                             None, capacity, q_heads, kv_heads, 1, _p(scratch), scratch_bytes,
                                             _stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16), d_keys[position].cpu().numpy(), d_values[position].cpu().numpy()


def _fused_decode(lib, inputs, cos, sin, position, capacity, scratch, q_heads=24, kv_heads=4, device_position=None):
    q_in, k_in, v_in, qw, kw, keys, values = inputs
    d_keys, d_values = _dev(keys.view(np.int16)), _dev(values.view(np.int16))
    out = torch.empty((q_heads, 256), dtype=torch.int16, device="cuda")
    lib.check(lib.lib().gfxb_decode_attention(_p(_dev(q_in)), _p(_dev(qw)), 512, _p(_dev(k_in)), _p(_dev(kw)), 256,
                                              _p(_dev(v_in)), 64, _p(_dev(cos)), _p(_dev(sin)), capacity, _p(d_keys),
                                              _p(d_values), capacity, 0 if device_position is not None else position,
                                              _p(device_position), q_heads, kv_heads, _p(out), _p(scratch),
                                              scratch.numel(), _stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16), d_keys[position].cpu().numpy(), d_values[position].cpu().numpy()


@pytest.mark.parametrize("heads", [(24, 4), (16, 2), (8, 8)], ids=["group6", "group8", "group1"])
@pytest.mark.parametrize("spread", [1.0, 4.0])
def test_decode_attention_equals_three_launch_path(lib, spread, heads):
    """The single-launch decode attention (norm + RoPE + KV append + attention + merge) against
    gfxb_qk_rms_norm_rope + gfxb_gated_attention at every chunk shape: one chunk, a chunk boundary,
    partial and full last chunks, up to 32 chunks at the last cache slot; the output and the appended
    cache row bit for bit, for three head layouts (GQA groups 6, 8 and 1). Long contexts at groups 6
    and 8 take the shared key/value stage. One zero-filled scratch serves every call (its counters
    return to zero)."""
    q_heads, kv_heads = heads
    capacity = 4096
    cos, sin = _rope(lib, capacity)
    scratch = torch.zeros(lib.lib().gfxb_decode_attention_scratch_bytes(q_heads, capacity), dtype=torch.uint8,
                          device="cuda")
    for position in (0, 1, 63, 64, 107, 108, 127, 128, 129, 255, 256, 300, 1000, 3839, 3840, 3947, 3948, 4095):
        inputs = _decode_attention_inputs(np.random.default_rng(position), capacity, q_heads, kv_heads, spread)
        want = _three_launch_decode(lib, inputs, cos, sin, position, capacity, q_heads, kv_heads)
        got = _fused_decode(lib, inputs, cos, sin, position, capacity, scratch, q_heads, kv_heads)
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w, err_msg=f"position {position}")
    tickets = scratch[-q_heads * 4:].cpu().numpy()
    assert not tickets.any()


def test_decode_attention_device_position_bit_exact(oracle, lib):
    """The graph form (position read from device memory, grid sized by the capacity) against the
    oracle's RoPE and attention."""
    capacity, position = 2048, 1500
    cos, sin = _rope(lib, capacity)
    inputs = _decode_attention_inputs(np.random.default_rng(5), capacity)
    q_in, k_in, v_in, qw, kw, keys, values = inputs
    scratch = torch.zeros(lib.lib().gfxb_decode_attention_scratch_bytes(24, capacity), dtype=torch.uint8,
                          device="cuda")
    got, got_k, got_v = _fused_decode(lib, inputs, cos, sin, position, capacity, scratch,
                                      device_position=_dev(np.array([position], np.uint64)))
    ocos, osin = np.zeros_like(cos), np.zeros_like(sin)
    oracle.lib.or_rope_table(capacity, 64, 1e7, _ptr(ocos), _ptr(osin))
    want_q = np.zeros((24, 256), np.uint16)
    want_k = np.zeros((4, 256), np.uint16)
    oracle.lib.or_qk_norm_rope(_ptr(_host(q_in)), 512, _ptr(qw), 24, position, _ptr(ocos), _ptr(osin), 64,
                               _ptr(want_q))
    oracle.lib.or_qk_norm_rope(_ptr(_host(k_in)), 256, _ptr(kw), 4, position, _ptr(ocos), _ptr(osin), 64, _ptr(want_k))
    np.testing.assert_array_equal(got_k.view(np.uint16), want_k)
    np.testing.assert_array_equal(got_v.view(np.float16), v_in.astype(np.float16))
    cache_k = keys.copy()
    cache_k[position] = want_k.view(np.float16)
    cache_v = values.copy()
    cache_v[position] = v_in.astype(np.float16)
    want = np.zeros((24, 256), np.uint16)
    oracle.lib.or_gated_attention(_ptr(_host(want_q.view(np.float16))), _ptr(_host(q_in)), _ptr(cache_k),
                                  _ptr(cache_v), position + 1, 24, 4, _ptr(want))
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bits", [4, 8])
def test_residual_norm_pack_bit_exact(oracle, lib, bits):
    rng = np.random.default_rng(bits)
    H, batch = 5120, 4
    residual = rng.normal(0, 3, (batch, H)).astype(np.float16)
    update = rng.normal(0, 2, (batch, H)).astype(np.float32)
    weight = _bf16(rng, H, -0.1, 0.1)
    res_out = torch.empty((batch, H), dtype=torch.int16, device="cuda")
    normalized = torch.empty((batch, H), dtype=torch.int16, device="cuda")
    codes = torch.empty((batch, H), dtype=torch.int8, device="cuda")
    scales = torch.empty((batch, H // 128), dtype=torch.int16, device="cuda")
    sums = torch.empty((batch, H // 128), dtype=torch.int32, device="cuda")
    lib.check(lib.lib().gfxb_residual_rms_norm_pack(_p(_dev(residual)), _p(_dev(update)), _p(res_out), _p(_dev(weight)),
                                                    _p(normalized), H, batch, ctypes.c_float(1e-6), 1, bits, _p(codes),
                                                    _p(scales), _p(sums), None, _stream()))
    torch.cuda.synchronize()
    for t in range(batch):
        want_res = np.zeros(H, np.uint16)
        want_norm = np.zeros(H, np.uint16)
        oracle.lib.or_residual_add_rms_norm(_ptr(_host(residual[t])), _ptr(_host(update[t])), _ptr(weight), H, 1e-6, 1,
                                            _ptr(want_res), _ptr(want_norm))
        np.testing.assert_array_equal(res_out[t].cpu().numpy().view(np.uint16), want_res)
        np.testing.assert_array_equal(normalized[t].cpu().numpy().view(np.uint16), want_norm)
        x16 = want_norm.view(np.float16)[None]
        if bits == 4:
            _, want_s, want_q = oracle.quantize_a4(x16)
        else:
            want_q, want_s = oracle.quantize_a8(x16)
        k = np.arange(128)
        offset = ((k & 15) >> 2) * 32 + (k >> 5) * 8 + ((k & 31) >> 4) * 4 + (k & 3)
        frag = codes[t].cpu().numpy().reshape(-1, 128)
        np.testing.assert_array_equal(frag[:, offset].reshape(-1), want_q[0])
        np.testing.assert_array_equal(scales[t].cpu().numpy().view(np.uint16), want_s[0].view(np.uint16))
        np.testing.assert_array_equal(sums[t].cpu().numpy(), want_q[0].reshape(-1, 128).astype(np.int32).sum(1))


def test_silu_pack_bit_exact(oracle, lib):
    rng = np.random.default_rng(3)
    I, batch = 17408, 2
    gate = rng.normal(0, 2, (batch, I)).astype(np.float32)
    up = rng.normal(0, 2, (batch, I)).astype(np.float32)
    product = torch.empty((batch, I), dtype=torch.int16, device="cuda")
    codes = torch.empty((batch, I), dtype=torch.int8, device="cuda")
    scales = torch.empty((batch, I // 128), dtype=torch.int16, device="cuda")
    sums = torch.empty((batch, I // 128), dtype=torch.int32, device="cuda")
    packed = torch.empty((batch, I // 2), dtype=torch.uint8, device="cuda")
    lib.check(lib.lib().gfxb_silu_multiply_pack(_p(_dev(gate)), _p(_dev(up)), I, batch, _p(product), 4, _p(codes),
                                                _p(scales), _p(sums), _p(packed), _stream()))
    torch.cuda.synchronize()
    want = np.zeros((batch, I), np.uint16)
    oracle.lib.or_silu_multiply_f16(_ptr(gate), _ptr(up), batch * I, _ptr(want))
    np.testing.assert_array_equal(product.cpu().numpy().view(np.uint16), want)
    want_packed, want_scales, _ = oracle.quantize_a4(want.view(np.float16))
    np.testing.assert_array_equal(packed.cpu().numpy(), want_packed)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint16), want_scales.view(np.uint16))


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_rounding_ties_bit_exact(oracle, lib, bits):
    """The fused packers round x / scale without a division per element; near and exact
    half-integer quotients, zero and subnormal scales must still match the reference's
    rint(x / scale) (lowbit_gemv.hip:392-405, 428-435). The SwiGLU packer is driven with
    gate = 32 (SiLU(32) = 32 in fp32) and up = x / 32, so it packs exactly x."""
    rng = np.random.default_rng(11 + bits)
    limit = 7 if bits == 4 else 127
    groups, batch = 96, 2
    x = np.zeros((batch, groups, 128), np.float32)
    for b in range(batch):
        for g in range(groups):
            kind = g % 4
            if kind == 3:  # tiny groups: subnormal fp16 scales (or zero)
                s = np.float16(rng.integers(0, 4) * 2.0 ** -24)
            else:
                s = np.float16(rng.uniform(0.001, 0.5))
            m = rng.integers(-2 * limit - 1, 2 * limit + 2, 128)
            vals = (m.astype(np.float32) * np.float32(s) / 2).astype(np.float16)
            if kind == 1:  # one fp16 ulp either side of the ties
                vals = np.nextafter(vals, np.where(rng.random(128) < 0.5, -np.inf, np.inf).astype(np.float16))
            vals[0] = np.float16(limit * float(s))  # pins amax, so scale = fp16(amax / limit) = s
            x[b, g] = vals.astype(np.float32)
    x16 = x.reshape(batch, groups * 128).astype(np.float16)
    I = groups * 128
    gate = np.full((batch, I), 32.0, np.float32)
    up = (x16.astype(np.float32) / 32.0).astype(np.float32)
    product = torch.empty((batch, I), dtype=torch.int16, device="cuda")
    codes = torch.empty((batch, I), dtype=torch.int8, device="cuda")
    scales = torch.empty((batch, I // 128), dtype=torch.int16, device="cuda")
    sums = torch.empty((batch, I // 128), dtype=torch.int32, device="cuda")
    lib.check(lib.lib().gfxb_silu_multiply_pack(_p(_dev(gate)), _p(_dev(up)), I, batch, _p(product), bits, _p(codes),
                                                _p(scales), _p(sums), None, _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(product.cpu().numpy().view(np.uint16), x16.view(np.uint16))
    if bits == 4:
        _, want_scales, want_values = oracle.quantize_a4(x16)
    else:
        want_values, want_scales = oracle.quantize_a8(x16)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint16), want_scales.view(np.uint16))
    k = np.arange(128)
    offset = ((k & 15) >> 2) * 32 + (k >> 5) * 8 + ((k & 31) >> 4) * 4 + (k & 3)
    frag = codes.cpu().numpy().reshape(batch, groups, 128)
    logical = np.empty_like(frag)
    logical[..., k] = frag[..., offset]
    np.testing.assert_array_equal(logical.reshape(batch, -1), want_values)
    np.testing.assert_array_equal(sums.cpu().numpy(), want_values.reshape(batch, groups, 128).astype(np.int32).sum(-1))
