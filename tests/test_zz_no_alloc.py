"""The allocation-free NF24 GEMM entry point (triposplat_gemm_nf24_noalloc).

Callers that cannot let a library allocate device memory — work recorded into a CUDA
graph, hosts whose device memory belongs to their own allocator or a fixed memory plan,
and latency-critical loops that cannot take cudaMalloc's device-wide synchronisation —
use this entry point.  It must give the same result as the regular entry point
triposplat_gemm_rnf8_avx512 (same tolerance as the GEMM parity tests: |dy| <= 2e-5 +
2e-5 |y|), on two calls in a row (the shared static scratch must not leak state from the
previous call), without growing the library workspace, and must reject problems larger
than its fixed 32 MiB scratch.

This file is collected last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _case(M, K, N, seed):
    from nf24_pack import quantize_nf24_i16_per_output_channel

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    codes, scales, _ = quantize_nf24_i16_per_output_channel(torch.randn(N, K, generator=g) * 0.02)
    b = torch.randn(N, generator=g) * 0.01
    return [t.cuda() for t in (x, codes[0], codes[1], scales[0], b)]


def _ws_allocations(lib):
    a, c = ctypes.c_uint64(), ctypes.c_uint64()
    assert lib.triposplat_b200_workspace_stats(ctypes.byref(a), ctypes.byref(c)) == 0
    return a.value, c.value


def _call_noalloc(lib, x, c01, q2, sc, b, out):
    M, K = x.shape
    N = c01.shape[1]
    cb = torch.zeros(256, device="cuda")
    return lib.triposplat_gemm_nf24_noalloc(
        x.data_ptr(), c01.data_ptr(), q2.data_ptr(), q2.data_ptr(), sc.data_ptr(), sc.data_ptr(),
        sc.data_ptr(), cb.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, K, N, 0, 3)


def test_noalloc_matches_regular_entry_on_two_calls_in_a_row():
    import _native
    from nf24_linear import nf24_linear

    lib = _native.load()
    _native.use_current_stream(lib)
    cases = [_case(4096, 1024, 3072, 11), _case(257, 1000, 512, 12)]
    refs = []
    for x, c01, q2, sc, b in cases:  # regular entry (library workspace)
        refs.append(nf24_linear(x, c01, q2, sc, b).clone())
    torch.cuda.synchronize()
    before = _ws_allocations(lib)
    outs = []
    for x, c01, q2, sc, b in cases:  # two allocation-free calls back to back
        out = torch.full((x.shape[0], c01.shape[1]), float("nan"), device="cuda")
        assert _call_noalloc(lib, x, c01, q2, sc, b, out) == 0
        outs.append(out)
    torch.cuda.synchronize()
    assert _ws_allocations(lib) == before, "the allocation-free entry grew the library workspace"
    for y, ref in zip(outs, refs):
        y, ref = y.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(y).all()
        assert (np.abs(y - ref) <= TOL + TOL * np.abs(ref)).all()
    assert lib.triposplat_b200_status() == 0


def test_noalloc_rejects_what_it_cannot_serve():
    import _native

    lib = _native.load()
    x, c01, q2, sc, b = _case(16, 64, 32, 3)
    out = torch.empty(16, 32, device="cuda")
    # 2*M*Kp*2 bytes beyond the 32 MiB scratch: M = 8192, K = 1024 needs 32 MiB + 33 KB
    big = torch.empty(8192, 1024, device="cuda")
    big_out = torch.empty(8192, 32, device="cuda")
    cb = torch.zeros(256, device="cuda")
    st = lib.triposplat_gemm_nf24_noalloc(
        big.data_ptr(), c01.data_ptr(), q2.data_ptr(), q2.data_ptr(), sc.data_ptr(), sc.data_ptr(),
        sc.data_ptr(), cb.data_ptr(), b.data_ptr(), big_out.data_ptr(), 8192, 1024, 32, 1024, 32, 0, 3)
    assert st == -6
    # N % 16 != 0 has no tensor-core path here
    st = lib.triposplat_gemm_nf24_noalloc(
        x.data_ptr(), c01.data_ptr(), q2.data_ptr(), q2.data_ptr(), sc.data_ptr(), sc.data_ptr(),
        sc.data_ptr(), cb.data_ptr(), b.data_ptr(), out.data_ptr(), 16, 64, 24, 64, 24, 0, 3)
    assert st == -4
    assert _call_noalloc(lib, x, c01, q2, sc, b, out) == 0
    torch.cuda.synchronize()
