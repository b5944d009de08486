"""The allocation-free NF24 GEMM entry point (triposplat_gemm_nf24_noalloc).

Callers that cannot let a library allocate device memory — hosts whose device memory
belongs to their own allocator or to a fixed plan made at start-up, and latency-critical
loops that cannot take cudaMalloc's device-wide synchronisation — use this entry point.
It must give the same result as the regular entry point triposplat_gemm_rnf8_avx512
(same tolerance as the GEMM parity tests: |dy| <= 2e-5 + 2e-5 |y|), on two calls in a row
(the shared static scratch must not leak state from the previous call), without growing
the library workspace, also when it is the first library call of a process (its set-up
maps the status word its kernels report bounded-wait timeouts through), and must reject
problems larger than its fixed 32 MiB scratch.

This file is collected last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import json
import subprocess
import sys
from pathlib import Path

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


_FIRST_CALL = r"""
import json, sys
import numpy as np, torch
sys.path[:0] = sys.argv[1:]
import _native
from nf24_linear import nf24_linear
from nf24_pack import quantize_nf24_i16_per_output_channel
g = torch.Generator().manual_seed(21)
x = torch.randn(300, 512, generator=g).cuda()
codes, scales, _ = quantize_nf24_i16_per_output_channel(torch.randn(256, 512, generator=g) * 0.02)
c01, q2, sc = codes[0].cuda(), codes[1].cuda(), scales[0].cuda()
b = (torch.randn(256, generator=g) * 0.01).cuda()
cb = torch.zeros(256, device="cuda")
lib = _native.load()
outs = []
for _ in range(2):  # the very first library calls of this process, then a second one
    out = torch.full((300, 256), float("nan"), device="cuda")
    st = lib.triposplat_gemm_nf24_noalloc(x.data_ptr(), c01.data_ptr(), q2.data_ptr(), q2.data_ptr(),
                                          sc.data_ptr(), sc.data_ptr(), sc.data_ptr(), cb.data_ptr(),
                                          b.data_ptr(), out.data_ptr(), 300, 512, 256, 512, 256, 0, 3)
    outs.append((st, out))
torch.cuda.synchronize()
status = int(lib.triposplat_b200_status())
ref = nf24_linear(x, c01, q2, sc, b).cpu().numpy()
ok = [bool((np.abs(o.cpu().numpy() - ref) <= 2e-5 + 2e-5 * np.abs(ref)).all()) for _, o in outs]
print(json.dumps({"status_codes": [s for s, _ in outs], "match": ok, "device_status": status}))
"""


def test_noalloc_as_first_library_call_of_a_process():
    """In a fresh process the allocation-free entry is the first library call: it sets
    itself up (scratch address, status word) and matches the regular entry."""
    repo = Path(__file__).resolve().parent.parent
    paths = [str(repo / "triposplat-cpu-avx512_b200"), str(repo)]
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL, *paths], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["status_codes"] == [0, 0] and res["match"] == [True, True]
    assert res["device_status"] == 0
