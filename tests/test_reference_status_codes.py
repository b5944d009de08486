"""The reference's own libraries (oracle/_ref, compiled from its sources) return the
status codes this library's GPU tests expect for the same invalid arguments
(tests/test_fused_entries_gpu.py), so the two agree on error behaviour; its first-version
QKV post-process equals its _v2, which this library exports under both names.  CPU only; skipped
where oracle/_ref was not built (it needs the reference checkout and an AVX-512 host)."""
import ctypes

import numpy as np
import pytest

from conftest import REPO
from test_fused_entries_gpu import MLP_BAD_SIZES, QKV_BAD_SIZES

REF = REPO / "oracle" / "_ref"
VP, I = ctypes.c_void_p, ctypes.c_int


def _lib(name):
    path = REF / name
    if not path.is_file():
        pytest.skip(f"{path.name} not built")
    flags = open("/proc/cpuinfo").read()
    if not all(f in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl")):
        pytest.skip("no AVX-512 on this host")
    return ctypes.CDLL(str(path))


def _ptr(a):
    return a.ctypes.data_as(VP)


def test_reference_mlp_status_codes():
    lib = _lib("libref_mlp_nf24.so")
    f = lib.triposplat_mlp_nf24_gelu_f32_avx512
    f.argtypes, f.restype = [VP] * 10 + [I] * 7, I
    fc = lib.triposplat_mlp_nf24_gelu_chunked_f32_avx512
    fc.argtypes, fc.restype = [VP] * 11 + [I] * 9, I
    x = np.zeros((4, 1024), np.float32)
    c1, q1 = np.zeros((1024, 4096), np.int16), np.zeros((1024, 4096), np.int8)
    c2, q2 = np.zeros((4096, 1024), np.int16), np.zeros((4096, 1024), np.int8)
    s1, s2 = np.zeros(4096, np.float32), np.zeros(1024, np.float32)
    out = np.zeros((4, 1024), np.float32)
    p = [_ptr(a) for a in (x, c1, q1, s1, s1, c2, q2, s2, s2, out)]
    assert f(*p, 4, 1024, 4096, 1024, 1024, 1024, 1) == 0
    assert f(*(p[:9] + [None]), 4, 1024, 4096, 1024, 1024, 1024, 1) == -1
    for args in MLP_BAD_SIZES:
        assert f(*p, *args, 1) == -2, args
    hid = np.zeros((2, 4096), np.float32)
    pc = p[:9] + [_ptr(hid), _ptr(out)]
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 2, 2, 1) == 0
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 1, 2, 1) == -2
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 2, 0, 1) == -2


def test_reference_qkv_direct_status_codes():
    lib = _lib("libref_gemm_nf24_qkv_direct.so")
    f = lib.triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512
    f.argtypes, f.restype = [VP] * 15 + [I] * 10, I
    B, L, K, H, D, Lp = 1, 4, 64, 1, 64, 16
    N = 3 * H * D
    z = lambda *s, dt=np.float32: np.zeros(s, dt)  # noqa: E731
    # buffers sized for the largest invalid case (L 20, L_padded 24)
    x, c, q, s = z(20, K), z(K, 4 * N, dt=np.int16), z(K, 4 * N, dt=np.int8), z(4 * N)
    fr, gm = z(3, 20, H, D), z(H, D)
    qo, pk, pv = z(B, H, 20, D), z(B, H, D, 24), z(B, H, D, 24)
    p = [_ptr(a) for a in (x, c, q, q, s, s, s, z(256), s, fr, gm, gm, qo, pk, pv)]
    assert f(*p, B, L, K, N, H, D, Lp, 1, 1, 3) == 0
    assert f(*(p[:14] + [None]), B, L, K, N, H, D, Lp, 1, 1, 3) == -1
    for args in QKV_BAD_SIZES:
        a = list(args)
        assert f(*p, *a[:8], 1, a[8]) == -2, args


def test_reference_postprocess_first_version_equals_v2(golden):
    """The reference's first post-process (scripts/native_qkv_postprocess_avx512.c:23) gives
    the bits of its _v2 on the fixture, so one implementation serves both names."""
    lib = _lib("libref_qkv_postprocess_v1.so")
    f = lib.triposplat_qkv_rope_rmsnorm_pack_f32_avx512
    f.argtypes, f.restype = [VP] * 7 + [I] * 7, I
    g = golden("elementwise")
    qkv = np.ascontiguousarray(g["post_qkv"])
    B, L, _, H, D = qkv.shape
    q = np.full((B, H, L, D), 3.0, np.float32)
    pk = np.full((B, H, D, 32), 3.0, np.float32)
    pv = np.full((B, H, D, 32), 3.0, np.float32)
    args = [np.ascontiguousarray(g[k]) for k in ("post_freqs", "post_qg", "post_kg")]
    assert f(_ptr(qkv), *(_ptr(a) for a in args), _ptr(q), _ptr(pk), _ptr(pv),
             B, L, H, D, 32, 1, 1) == 0
    np.testing.assert_array_equal(q, g["post_q"])
    np.testing.assert_array_equal(pk, g["post_pk"])
    np.testing.assert_array_equal(pv, g["post_pv"])
