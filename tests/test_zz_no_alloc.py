"""The allocation-free attention entry point matches the allocating one.

gfxb_gated_attention_static_scratch keeps its scratch in a fixed array inside
the library, for callers that cannot allocate device memory (frameworks that
own the memory budget, loops that cannot absorb an allocation's implicit
synchronisation). It must give the same output as gfxb_gated_attention with a
caller-provided scratch buffer, call after call, even though both calls reuse
the same array. Collected last on purpose: a failure here leaves every other
test already run.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle_lib import _ptr  # noqa: E402,F401


@pytest.fixture(scope="module")
def lib():
    from gfxinfer_b200 import build

    build.build()
    import gfxinfer_b200

    return gfxinfer_b200


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.cuda.current_device())


def _case(seed, capacity, batch, q_heads=24, kv_heads=4):
    rng = np.random.default_rng(seed)
    query = _dev(rng.normal(0, 1, (batch, q_heads, 256)).astype(np.float16))
    gate = _dev(rng.normal(0, 1, (batch, q_heads, 512)).astype(np.float32))
    keys = _dev(rng.normal(0, 1, (capacity, kv_heads, 256)).astype(np.float16))
    values = _dev(rng.normal(0, 1, (capacity, kv_heads, 256)).astype(np.float16))
    return query, gate, keys, values


def _compare(lib, capacity, base, batch, seed, device_position, q_heads=24, kv_heads=4):
    """One call of each entry point on the same inputs; returns (static, allocating) outputs."""
    api = lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    query, gate, keys, values = _case(seed, capacity, batch, q_heads, kv_heads)
    scratch_bytes = api.gfxb_gated_attention_scratch_bytes(q_heads, capacity, batch)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device="cuda")
    want = torch.empty((batch, q_heads, 256), dtype=torch.int16, device="cuda")
    got = torch.full((batch, q_heads, 256), -1, dtype=torch.int16, device="cuda")
    if device_position:
        # graph-safe form: the first token's position (base - 1) is read from device memory and the
        # grid covers the whole capacity
        position = torch.tensor([base - 1], dtype=torch.int64, device="cuda")
        host_base, pointer = 0, position.data_ptr()
    else:
        host_base, pointer = base, None
    lib.check(api.gfxb_gated_attention(query.data_ptr(), gate.data_ptr(), keys.data_ptr(), values.data_ptr(),
                                       want.data_ptr(), host_base, pointer, capacity, q_heads, kv_heads, batch,
                                       scratch.data_ptr(), scratch_bytes, stream))
    lib.check(api.gfxb_gated_attention_static_scratch(query.data_ptr(), gate.data_ptr(), keys.data_ptr(),
                                                      values.data_ptr(), got.data_ptr(), host_base, pointer,
                                                      capacity, q_heads, kv_heads, batch, stream))
    torch.cuda.synchronize()
    return got, want


@pytest.mark.gpu
def test_static_scratch_attention_matches_allocating_entry_point(lib):
    # two calls in a row with different inputs and token counts: the shared array keeps the
    # previous call's partials, which must not leak into the next result
    for seed, base, batch in ((1, 300, 3), (2, 37, 5)):
        got, want = _compare(lib, 512, base, batch, seed, device_position=False)
        # the kernels are bit-exact with each other; the tolerance our tests use for these outputs is zero
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_static_scratch_device_position_and_changing_capacity(lib):
    # the device-resident position (graph-capture form) and a partial stride that changes between
    # consecutive calls (capacity 2048, then 512, then 4096 with fewer heads)
    cases = ((2048, 1500, 2, 3, True, 24, 4), (512, 200, 4, 4, True, 24, 4), (4096, 4090, 3, 5, False, 8, 2),
             (4096, 2048, 1, 6, True, 8, 2))
    for capacity, base, batch, seed, device_position, q_heads, kv_heads in cases:
        got, want = _compare(lib, capacity, base, batch, seed, device_position, q_heads, kv_heads)
        assert torch.equal(got, want), (capacity, base, batch, device_position)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_static_scratch_on_a_second_device(lib):
    # the array's address and the attention kernel's shared-memory limit are per device
    got, want = _compare(lib, 512, 100, 2, 7, device_position=False)
    assert torch.equal(got, want)
    with torch.cuda.device(1):
        got, want = _compare(lib, 512, 100, 2, 7, device_position=False)
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_static_scratch_rejects_oversized_requests(lib):
    api = lib.lib()
    # 24 heads x 64 chunks (capacity 8192) x 258 floats x 32 tokens exceeds the 4 MiB array
    status = api.gfxb_gated_attention_static_scratch(1, 1, 1, 1, 1, 1, None, 8192, 24, 4, 32, None)
    assert status == 1
    assert b"4 MiB" in api.gfxb_last_error_message()
