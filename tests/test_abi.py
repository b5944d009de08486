"""CPU-side checks of the C-ABI boundary: the product library loads without a GPU,
exports every function include/triposplat_b200.h declares, and its signatures table
covers them.  No compute call is made here."""
import ctypes
import re

import pytest

from conftest import PKG, REPO

HEADER = REPO / "include" / "triposplat_b200.h"
LIB = PKG / "libtriposplat_b200.so"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(triposplat_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        import build_lib
        build_lib.build()
    return ctypes.CDLL(str(LIB))


def test_header_declares_reference_symbols():
    names = declared()
    for ref in ("triposplat_gemm_rnf8_avx512", "triposplat_gemm_rnf8_avx512_range",
                "triposplat_gemm_rnf8_avx512_tail", "triposplat_sdpa_f32_avx512_exact_q8t512",
                "triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd",
                "triposplat_layernorm_f32_avx512", "triposplat_cfg_combine_inplace_f32_avx512"):
        assert ref in names
    assert len(names) >= 35, len(names)


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if getattr(lib, n, None) is None]
    assert not missing, missing


def test_signature_table_matches_header():
    import _native

    assert set(declared()) <= set(_native.SIGNATURES), set(declared()) - set(_native.SIGNATURES)


def test_constant_queries_without_gpu(lib):
    lib.triposplat_gemm_rnf8_avx512_residual_mode.restype = ctypes.c_int
    assert lib.triposplat_gemm_rnf8_avx512_residual_mode() == 4
    lib.triposplat_sdpa_packed_output_is_blhd.restype = ctypes.c_int
    assert lib.triposplat_sdpa_packed_output_is_blhd() == 1
    assert lib.triposplat_sdpa_key_tile() == 128

