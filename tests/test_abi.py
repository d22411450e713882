"""The C-ABI library loads and exports every symbol include/gfxb/*.h declares.

No compute calls: argument validation returns before any CUDA work, so these
run without a GPU.
"""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "gfxb", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(gfxb_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def library():
    from gfxinfer_b200 import build

    build.build()
    import gfxinfer_b200

    return gfxinfer_b200.lib()


def test_every_declared_symbol_is_exported(library):
    declared = _declared_symbols()
    assert len(declared) >= 10
    missing = [name for name in declared if not hasattr(library, name)]
    assert not missing, missing


def test_every_declared_symbol_has_a_python_signature():
    from gfxinfer_b200 import abi

    assert sorted(abi.SIGNATURES) == _declared_symbols()


def test_abi_version(library):
    assert library.gfxb_abi_version() == 1


def test_argument_validation_without_gpu(library):
    import gfxinfer_b200
    from gfxinfer_b200 import abi

    # batch 0 and 33, K not a multiple of 128, N not a multiple of 16: rejected before any launch
    matrix = (abi.GemvMatrix * 1)(abi.GemvMatrix(1, 1, 1, 16, 0))
    assert library.gfxb_lowbit_gemv(3, matrix, 1, 1, 1, 1, 128, 0, None) == 1
    assert library.gfxb_lowbit_gemv(3, matrix, 1, 1, 1, 1, 128, 33, None) == 1
    assert library.gfxb_lowbit_gemv(3, matrix, 1, 1, 1, 1, 127, 1, None) == 1
    bad_rows = (abi.GemvMatrix * 1)(abi.GemvMatrix(1, 1, 1, 15, 0))
    assert library.gfxb_lowbit_gemv(3, bad_rows, 1, 1, 1, 1, 128, 1, None) == 1
    assert library.gfxb_lowbit_gemv(9, matrix, 1, 1, 1, 1, 128, 1, None) == 4
    assert library.gfxb_lowbit_gemv(3, matrix, 5, 1, 1, 1, 128, 1, None) == 1
    assert b"between one and four" in library.gfxb_last_error_message()
    assert library.gfxb_quantize_activation_i4(1, 1, 1, 127, 1, None) == 1
    assert library.gfxb_quantize_activation_i8(1, 1, 1, 128, 33, None) == 1
    assert library.gfxb_pack_activation(5, 1, 1, 1, 1, None, 128, 1, None) == 1
    assert library.gfxb_gfx12_i4_gemm(2, 1, 1, 1, 1, 1, 16, 128, 1, 0, None) == 4
    assert library.gfxb_repack_rowmajor_to_b200(3, 1, 1, 17, 128, None) == 1
    with pytest.raises(gfxinfer_b200.GfxbError):
        gfxinfer_b200.check(1)
