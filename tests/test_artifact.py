"""`.gfxi` container parity (CPU, no GPU): this library's reader/writer
(include/gfxb/artifact.h) against the reference's own src/artifact.cpp,
compiled in place into oracle/_ref by oracle/Makefile.

The reference has artifact round-trip tests (tests/artifact_test.cpp:27-104:
write/read round trip, duplicate-name rejection, streamed writer); these are
restated here, plus cross-implementation checks: both writers produce the same
bytes for the same request, each reader opens the other's files, and both
readers reject the same corruptions with the same ErrorCode.
"""
import os

import numpy as np
import pytest

from oracle_lib import Reference

IDENTITY = {"target_arch": "sm_100a", "model_id": "qwen-hybrid", "weights_id": "unit-test", "recipe_id": "b200-v1"}
CORRUPT_ARTIFACT, INVALID_ARGUMENT, UNSUPPORTED = 3, 1, 4


@pytest.fixture(scope="module")
def gx():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import artifact

    return artifact


@pytest.fixture(scope="module")
def ref():
    if not Reference.available():
        pytest.skip("the reference checkout is not built here (oracle/_ref)")
    return Reference()


def _tensors(gx, seed=0):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, 64 * 256 * 3 // 8, dtype=np.uint8)
    scales = rng.random(64 * 2).astype(np.float16)
    norm = rng.integers(0, 2 ** 16, 300, dtype=np.uint16)
    ids = np.arange(17, dtype=np.int32)
    return [
        gx.TensorWrite("model.language_model.layers.0.mlp.gate_proj.weight", gx.DTYPE_U8, gx.QUANT_W3G128, (64, 256),
                       codes, scales),
        gx.TensorWrite("model.language_model.norm.weight", gx.DTYPE_BF16, gx.QUANT_NONE, (300,), norm),
        gx.TensorWrite("mtp.draft_head_token_ids", gx.DTYPE_I32, gx.QUANT_NONE, (17,), ids, None, 4096),
        gx.TensorWrite("linear_attn/conv1d", gx.DTYPE_BF16, gx.QUANT_NONE, (5, 1, 4), norm[:20]),
    ]


def _as_ref(tensors):
    return [(t.name, t.dtype, t.quantization, t.dimensions, t.data, t.aux, t.alignment) for t in tensors]


def test_crc64_known_answer(gx):
    # CRC-64/ECMA-182 (poly 0x42F0E1EBA9EA3693, init 0, unreflected) check value
    assert gx.crc64(b"123456789") == 0x6C40DF5F0B497347
    assert gx.crc64(b"") == 0
    assert gx.crc64(b"56789", gx.crc64(b"1234")) == gx.crc64(b"123456789")


def test_round_trip(gx, tmp_path):
    path = tmp_path / "model.gfxi"
    tensors = _tensors(gx)
    gx.write(path, IDENTITY, tensors)
    with gx.Artifact(path) as a:
        assert a.identity() == IDENTITY
        assert a.file_bytes() == os.path.getsize(path)
        got = {t.name: t for t in a.tensors()}
        assert list(got) == [t.name for t in tensors]
        for t in tensors:
            g = got[t.name]
            assert (g.dtype, g.quantization, g.dimensions) == (t.dtype, t.quantization, t.dimensions)
            assert g.data.tobytes() == np.asarray(t.data).tobytes()
            assert (g.aux is None) == (t.aux is None)
            if t.aux is not None:
                assert g.aux.tobytes() == np.asarray(t.aux).tobytes()
            assert g.data_offset % max(256, t.alignment) == 0
            assert g.data_crc64 == gx.crc64(np.asarray(t.data))
        assert a.find("model.language_model.norm.weight").dimensions == (300,)
        assert a.find("absent") is None
    assert not [p for p in os.listdir(tmp_path) if ".tmp." in p]


def test_writers_produce_identical_bytes(gx, ref, tmp_path):
    tensors = _tensors(gx, seed=1)
    mine, theirs = tmp_path / "mine.gfxi", tmp_path / "theirs.gfxi"
    gx.write(mine, IDENTITY, tensors)
    assert ref.artifact_write(theirs, IDENTITY, _as_ref(tensors)) == 0
    assert mine.read_bytes() == theirs.read_bytes()


def test_reference_reader_opens_our_files(gx, ref, tmp_path):
    path = tmp_path / "mine.gfxi"
    tensors = _tensors(gx, seed=2)
    gx.write(path, IDENTITY, tensors)
    status, count, size = ref.artifact_open(path)
    assert (status, count, size) == (0, len(tensors), os.path.getsize(path))
    with gx.Artifact(path) as a:
        for i, t in enumerate(a.tensors()):
            r = ref.artifact_tensor(path, i)
            assert r["name"] == t.name and r["dimensions"] == t.dimensions
            assert (r["data_offset"], r["data_bytes"], r["data_crc64"]) == (t.data_offset, t.data.size, t.data_crc64)
            assert r["aux_bytes"] == (0 if t.aux is None else t.aux.size)


def test_our_reader_opens_reference_files(gx, ref, tmp_path):
    path = tmp_path / "theirs.gfxi"
    tensors = _tensors(gx, seed=3)
    assert ref.artifact_write(path, {**IDENTITY, "recipe_id": "tiled-v9-w3seq", "target_arch": "gfx1200"},
                              _as_ref(tensors)) == 0
    with gx.Artifact(path) as a:
        assert a.identity()["recipe_id"] == "tiled-v9-w3seq"
        for t, g in zip(tensors, a.tensors()):
            assert g.data.tobytes() == np.asarray(t.data).tobytes()


def _corrupt(path, offset, value=None):
    data = bytearray(path.read_bytes())
    data[offset] = (data[offset] ^ 0xFF) if value is None else value
    path.write_bytes(bytes(data))


@pytest.mark.parametrize("where", ["payload", "manifest", "magic", "version", "length"])
def test_both_readers_reject_corruption_alike(gx, ref, tmp_path, where):
    from gfxinfer_b200 import GfxbError

    path = tmp_path / "bad.gfxi"
    tensors = _tensors(gx, seed=4)
    gx.write(path, IDENTITY, tensors)
    with gx.Artifact(path) as a:
        payload = a.tensors()[1].data_offset
    if where == "payload":
        _corrupt(path, payload + 3)
    elif where == "manifest":
        _corrupt(path, 256 + 12)  # first directory entry's dtype field
    elif where == "magic":
        _corrupt(path, 0)
    elif where == "version":
        _corrupt(path, 8, 2)
    else:
        path.write_bytes(path.read_bytes() + b"\0" * 256)
    expected = UNSUPPORTED if where == "version" else CORRUPT_ARTIFACT
    with pytest.raises(GfxbError) as error:
        gx.Artifact(path)
    assert error.value.status == expected
    assert ref.artifact_open(path)[0] == expected
    if where == "payload":  # without checksum verification the payload flip goes unseen by both
        gx.Artifact(path, verify_checksums=False).close()
        assert ref.artifact_open(path, verify=False)[0] == 0


@pytest.mark.parametrize("name", ["", "/abs", "a/../b", "bad name", "dup"])
def test_invalid_write_requests_are_rejected(gx, tmp_path, name):
    from gfxinfer_b200 import GfxbError

    tensors = _tensors(gx)[:1]
    if name == "dup":
        tensors = tensors + tensors
    else:
        tensors[0].name = name
    with pytest.raises(GfxbError) as error:
        gx.write(tmp_path / "x.gfxi", IDENTITY, tensors)
    assert error.value.status == INVALID_ARGUMENT
    assert not list(tmp_path.iterdir())


def test_identity_must_fit(gx, tmp_path):
    from gfxinfer_b200 import GfxbError

    with pytest.raises(GfxbError):
        gx.write(tmp_path / "x.gfxi", {**IDENTITY, "weights_id": ""}, _tensors(gx)[:1])
