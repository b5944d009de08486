"""NF24 GEMM parity: CUDA (through the C-ABI) vs the oracle / reference golden vectors.

Tolerance (fp32 semantics, split-precision tensor cores): max |y - y_ref| <= 2e-5 + 2e-5*|y_ref|,
the reference smoke test's own rtol = atol = 2e-5 (scripts/smoke_native_rnf8_avx512.py:58).
The scalar tail path reproduces the reference's operation order and must be bit-identical.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = ATOL = 2e-5


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _pack(torch_w):
    from nf24_pack import quantize_nf24_i16_per_output_channel

    codes, scales, _ = quantize_nf24_i16_per_output_channel(torch_w)
    return codes[0].numpy(), codes[1].numpy(), scales[0].numpy()


def _run(x, c01, q2, sc, bias, start=0, count=None):
    from nf24_linear import nf24_linear

    y = nf24_linear(_cuda(x), _cuda(c01), _cuda(q2), _cuda(sc), _cuda(bias), start=start, count=count)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _assert_close(y, ref):
    err = np.abs(y - ref)
    bound = ATOL + RTOL * np.abs(ref)
    assert np.isfinite(y).all()
    assert (err <= bound).all(), f"max err {err.max():.3e} (worst ratio {(err / bound).max():.2f})"


@pytest.mark.parametrize("case", ["gemm_25x96x64", "gemm_40x96x64", "gemm_10x96x64",
                                  "gemm_3x96x5_tail", "gemm_7x100x7_tail",
                                  "gemm_33x160x96_range32_48", "gemm_130x256x144"])
def test_gemm_golden(golden, case):
    g = golden(case)
    count = int(g["count"])
    y = _run(g["x"], g["code01_t"], g["q2_t"], g["scale"], g["bias"], start=int(g["start"]),
             count=None if count < 0 else count)
    if g["code01_t"].shape[1] % 16:
        np.testing.assert_array_equal(y, g["out"])  # reference-order scalar kernel
    else:
        _assert_close(y, g["out"])


@pytest.mark.parametrize("M,K,N", [(1, 1024, 1024), (3, 64, 16), (257, 1000, 3072),
                                   (300, 4096, 1024), (513, 1024, 4096), (64, 1024, 6144),
                                   (2, 1024, 6144)])
def test_gemm_vs_oracle(oracle, M, K, N):
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g).numpy()
    w = torch.randn(N, K, generator=g) * 0.02
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    c01, q2, sc = _pack(w)
    ref = oracle.gemm_nf24(x, c01, q2, sc, b)
    _assert_close(_run(x, c01, q2, sc, b), ref)


def test_gemm_range_windows(oracle):
    g = torch.Generator().manual_seed(5)
    M, K, N = 200, 1024, 3072
    x = torch.randn(M, K, generator=g).numpy()
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    for start, count in ((0, 1024), (1024, 1024), (2048, 1024), (16, 48), (3056, 16)):
        ref = oracle.gemm_nf24(x, c01, q2, sc, b, start=start, count=count)
        _assert_close(_run(x, c01, q2, sc, b, start=start, count=count), ref)


def test_gemm_row_scale_extremes(oracle):
    """Rows of very different magnitude exercise the per-row pre-scale of the split."""
    g = torch.Generator().manual_seed(9)
    M, K, N = 64, 512, 256
    x = torch.randn(M, K, generator=g)
    mags = torch.tensor([10.0 ** e for e in range(-8, 8)]).repeat(4)
    x = (x * mags[:, None]).numpy()
    x[5, :] = 0.0
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = np.zeros(N, np.float32)
    ref = oracle.gemm_nf24(x, c01, q2, sc, b)
    y = _run(x, c01, q2, sc, b)
    scale = np.abs(x).max(axis=1, keepdims=True) * 0.02 * np.sqrt(K) + 1e-30
    assert (np.abs(y - ref) / scale).max() < 2e-6
    assert (y[5] == 0).all()


def test_gemm_full_config1_vs_oracle(oracle):
    """BASELINE config 1 at full size: M=4096, K=1024, N=3072."""
    g = torch.Generator().manual_seed(0)
    M, K, N = 4096, 1024, 3072
    x = torch.randn(M, K, generator=g).numpy()
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    ref = oracle.gemm_nf24(x, c01, q2, sc, b)
    y = _run(x, c01, q2, sc, b)
    _assert_close(y, ref)
    assert float(np.sqrt(np.mean((y - ref) ** 2))) < 1e-6


@pytest.mark.parametrize("K,start,count", [(200, 32, 96), (1024, 0, None), (72, 16, 48)])
def test_gemm_codes_copy_path_is_the_direct_path_row_for_row(oracle, K, start, count):
    """From 2048 rows on the drop-in entries first copy the codes of the requested columns
    into k-contiguous planes (K padded to 16, ragged last 64-k tile, column windows); fewer
    rows read the [K][N] planes directly.  Both decode to the same operands and issue the
    same MMAs per row, so the first 1000 rows of a 2304-row call equal a 1000-row call bit
    for bit, and the whole output stays within the oracle tolerance."""
    g = torch.Generator().manual_seed(K + start)
    M, N = 2304, 160
    x = torch.randn(M, K, generator=g).numpy()
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    big = _run(x, c01, q2, sc, b, start=start, count=count)
    small = _run(x[:1000], c01, q2, sc, b, start=start, count=count)
    np.testing.assert_array_equal(big[:1000], small)
    ref = oracle.gemm_nf24(x, c01, q2, sc, b)
    _assert_close(big, ref[:, start:start + (count or N)])


def test_gemm_error_codes():
    import _native

    lib = _native.load()
    dev = torch.zeros(4096, device="cuda")
    p = dev.data_ptr()
    f = lib.triposplat_gemm_rnf8_avx512
    fr = lib.triposplat_gemm_rnf8_avx512_range
    assert f(None, p, p, p, p, p, p, p, p, p, 2, 16, 16, 16, 16, 0, 3) == -1
    assert f(p, p, p, p, p, p, p, p, p, p, 0, 16, 16, 16, 16, 0, 3) == -2
    assert f(p, p, p, p, p, p, p, p, p, p, 2, 16, 16, 16, 16, 0, 2) == -2
    assert f(p, p, p, p, p, p, p, p, p, p, 2, 16, 16, 8, 16, 0, 3) == -3
    assert fr(p, p, p, p, p, p, p, p, p, p, 2, 16, 64, 48, 32, 16, 32, 0, 3) == -3
    assert fr(p, p, p, p, p, p, p, p, p, p, 2, 16, 64, 8, 16, 16, 16, 0, 3) == -4
    host = np.zeros(4096, np.float32)
    hp = host.ctypes.data
    assert f(hp, p, p, p, p, p, p, p, p, p, 2, 16, 16, 16, 16, 0, 3) == -9
    assert lib.triposplat_gemm_rnf8_avx512_residual_mode() == 4
    assert lib.triposplat_b200_status() == 0


def _split_buf(lib, M, K):
    n = int(lib.triposplat_b200_split_bytes(M, K))
    t = torch.empty(n + 256, dtype=torch.uint8, device="cuda")
    return t, (t.data_ptr() + 255) & ~255


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_gemm_split_epilogues(oracle, mode):
    """Split buffer + fused epilogues: store, GELU, gated residual, residual."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(40 + mode)
    B, L, K, N = 2, 150, 1024, 384
    M = B * L
    x = torch.randn(M, K, generator=g).numpy()
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    base = torch.randn(M, N, generator=g).numpy()
    gate = torch.randn(B, N, generator=g).numpy()
    y = oracle.gemm_nf24(x, c01, q2, sc, b)
    ref = {0: y, 1: oracle.gelu_tanh(y), 2: base + np.repeat(gate, L, axis=0) * y, 3: base + y}[mode]
    keep, sp = _split_buf(lib, M, K)
    xc = _cuda(x)
    assert lib.triposplat_b200_split_f32(xc.data_ptr(), M, K, K, sp) == 0
    out = _cuda(base.copy())
    gc = _cuda(gate)
    w = [_cuda(a) for a in (c01, q2, sc, b)]  # keep the device copies alive
    st = lib.triposplat_b200_gemm_nf24_split(sp, M, K, w[0].data_ptr(), w[1].data_ptr(),
                                             w[2].data_ptr(), w[3].data_ptr(), out.data_ptr(),
                                             N, N, mode, gc.data_ptr(), N, L)
    assert st == 0
    torch.cuda.synchronize()
    _assert_close(out.cpu().numpy(), ref)


def test_ln_modulate_split_then_gemm(oracle):
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(77)
    B, L, C, N = 2, 97, 1024, 256
    x = (torch.randn(B, L, C, generator=g) * 2 + 0.5).numpy()
    shift = (torch.randn(B, C, generator=g) * 0.1).numpy()
    scale = (torch.randn(B, C, generator=g) * 0.1).numpy()
    c01, q2, sc = _pack(torch.randn(N, C, generator=g) * 0.02)
    b = np.zeros(N, np.float32)
    a = oracle.modulate(oracle.layernorm(x, eps=1e-6), scale, shift).reshape(B * L, C)
    ref = oracle.gemm_nf24(a, c01, q2, sc, b)
    keep, sp = _split_buf(lib, B * L, C)
    xc, shc, scc = _cuda(x), _cuda(shift), _cuda(scale)
    assert lib.triposplat_b200_ln_modulate_split(xc.data_ptr(), B * L, C, 1e-6, shc.data_ptr(),
                                                 scc.data_ptr(), C, L, sp) == 0
    out = torch.empty(B * L, N, device="cuda")
    w = [_cuda(a) for a in (c01, q2, sc, b)]  # keep the device copies alive
    assert lib.triposplat_b200_gemm_nf24_split(sp, B * L, C, w[0].data_ptr(), w[1].data_ptr(),
                                               w[2].data_ptr(), w[3].data_ptr(), out.data_ptr(),
                                               N, N, 0, None, 0, 1) == 0
    torch.cuda.synchronize()
    _assert_close(out.cpu().numpy(), ref)


def _to_nk(lib, c01_dev, q2_dev):
    K, N = int(c01_dev.shape[0]), int(c01_dev.shape[1])
    c_nk = torch.empty(N, K, dtype=torch.int16, device="cuda")
    q_nk = torch.empty(N, K, dtype=torch.int8, device="cuda")
    assert lib.triposplat_b200_nf24_codes_to_nk(c01_dev.data_ptr(), q2_dev.data_ptr(), K, N,
                                                c_nk.data_ptr(), q_nk.data_ptr()) == 0
    return c_nk, q_nk


def test_codes_to_nk_is_a_transpose():
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(5)
    K, N = 200, 72  # ragged against the 32 x 32 tiles
    c01 = torch.randint(-636, 637, (K, N), generator=g, dtype=torch.int16)
    q2 = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8)
    c_nk, q_nk = _to_nk(lib, c01.cuda(), q2.cuda())
    torch.cuda.synchronize()
    assert torch.equal(c_nk.cpu(), c01.T.contiguous()) and torch.equal(q_nk.cpu(), q2.T.contiguous())


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_gemm_split_nk_matches_reference_layout(mode):
    """The k-contiguous code layout (the model path) decodes the same operands into the same
    MMAs but accumulates two 64-k blocks per tensor-memory partial before promoting (the
    reference layout: one), so the two differ by accumulation rounding only: within the
    GEMM tolerance everywhere and relative rmse <= 1e-6, for full weights, column windows and
    input-feature windows (ldk > K)."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(60 + mode)
    B, L, K, N = 2, 300, 1024, 640
    M = B * L
    x = torch.randn(M, K, generator=g)
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    bias = (torch.randn(N, generator=g) * 0.01).numpy()
    w = [_cuda(a) for a in (c01, q2, sc, bias)]
    c_nk, q_nk = _to_nk(lib, w[0], w[1])
    gate = torch.randn(B, N, generator=g).cuda()
    base = torch.randn(M, N, generator=g).cuda()
    for k0, kw, start, count in ((0, K, 0, N), (0, K, 128, 384), (256, 512, 0, N), (512, 256, 64, 320)):
        keep, sp = _split_buf(lib, M, kw)
        xc = x[:, k0:k0 + kw].contiguous().cuda()
        assert lib.triposplat_b200_split_f32(xc.data_ptr(), M, kw, kw, sp) == 0
        outs = []
        for nk in (False, True):
            out = base[:, start:start + count].clone()  # a copy even for the full width
            if nk:
                st = lib.triposplat_b200_gemm_nf24_split_nk(
                    sp, M, kw, c_nk.data_ptr() + 2 * k0, q_nk.data_ptr() + k0, K,
                    w[2].data_ptr(), w[3].data_ptr(), out.data_ptr(), N, start, count, count,
                    mode, gate.data_ptr(), N, L)
            else:
                st = lib.triposplat_b200_gemm_nf24_split_range(
                    sp, M, kw, w[0][k0:].data_ptr(), w[1][k0:].data_ptr(), w[2].data_ptr(),
                    w[3].data_ptr(), out.data_ptr(), N, start, count, count, mode,
                    gate.data_ptr(), N, L)
            assert st == 0, (k0, kw, start, count, st)
            outs.append(out)
        torch.cuda.synchronize()
        ref, got = outs[0].cpu().numpy(), outs[1].cpu().numpy()
        _assert_close(got, ref)
        rel = np.sqrt(np.mean((got.astype(np.float64) - ref) ** 2) / np.mean(ref.astype(np.float64) ** 2))
        assert rel <= 1e-6, (k0, kw, start, count, rel)


@pytest.mark.parametrize("K", [1024, 4096])
def test_gemm_accuracy_vs_float64(oracle, K):
    """Against the exact product (float64 over the dequantised weights), both tensor-core
    layouts (3 split-fp16 passes; truncating tensor-memory partials of one / two 64-k blocks
    promoted into round-to-nearest fp32 sums) are at least as accurate as the reference's
    own fp32 kernel (the oracle reproduces it bit for bit)."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(K)
    M, N = 512, 1024
    x = torch.randn(M, K, generator=g).numpy()
    c01, q2, sc = _pack(torch.randn(N, K, generator=g) * 0.02)
    b = (torch.randn(N, generator=g) * 0.01).numpy()
    wd = (c01.astype(np.float64) * 256 + q2.astype(np.float64)) * sc.astype(np.float64)
    exact = x.astype(np.float64) @ wd + b
    rms = np.sqrt(np.mean(exact ** 2))

    def err(y):
        return np.sqrt(np.mean((np.asarray(y, np.float64) - exact) ** 2)) / rms

    e_ref = err(oracle.gemm_nf24(x, c01, q2, sc, b))
    e_drop_in = err(_run(x, c01, q2, sc, b))
    w = [_cuda(a) for a in (c01, q2, sc, b)]
    c_nk, q_nk = _to_nk(lib, w[0], w[1])
    keep, sp = _split_buf(lib, M, K)
    xc = _cuda(x)
    assert lib.triposplat_b200_split_f32(xc.data_ptr(), M, K, K, sp) == 0
    out = torch.empty(M, N, device="cuda")
    assert lib.triposplat_b200_gemm_nf24_split_nk(sp, M, K, c_nk.data_ptr(), q_nk.data_ptr(), K,
                                                  w[2].data_ptr(), w[3].data_ptr(), out.data_ptr(),
                                                  N, 0, N, N, 0, None, 0, 1) == 0
    torch.cuda.synchronize()
    e_nk = err(out.cpu().numpy())
    assert e_drop_in <= e_ref and e_nk <= e_ref, (e_drop_in, e_nk, e_ref)


def test_gemm_split_nk_rejects_bad_arguments():
    import _native

    lib = _native.load()
    t = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    p = t.data_ptr()
    f = lib.triposplat_b200_gemm_nf24_split_nk
    assert f(None, 16, 64, p, p, 64, p, p, p, 64, 0, 64, 64, 0, None, 0, 1) == -1
    assert f(p, 16, 64, p, p, 32, p, p, p, 64, 0, 64, 64, 0, None, 0, 1) == -3   # ldk < K
    assert f(p, 16, 64, p, p, 64, p, p, p, 64, 16, 64, 64, 0, None, 0, 1) == -3  # past N
    assert f(p, 16, 64, p, p, 72, p, p, p, 64, 0, 64, 64, 0, None, 0, 1) == -4   # ldk % 16
    assert f(p, 16, 64, p + 8, p, 64, p, p, p, 64, 0, 64, 64, 0, None, 0, 1) == -4
    assert f(p, 16, 64, p, p, 64, p, p, p + 4, 64, 0, 64, 64, 0, None, 0, 1) == -4  # out
    assert f(p, 16, 64, p, p, 64, p, p, p, 64, 0, 62, 62, 0, None, 0, 1) == -4       # stride


def _split_planes(keep, sp, M, K):
    """(hi fp16 [M, K], lo fp16 [M, K], rs fp32 [Mp]) of a split buffer (K % 8 == 0)."""
    plane = (M * K * 2 + 255) // 256 * 256
    Mp = (M + 3) // 4 * 4
    raw = keep[sp - keep.data_ptr():].cpu().numpy()
    hi = raw[:M * K * 2].view(np.float16).reshape(M, K)
    lo = raw[plane:plane + M * K * 2].view(np.float16).reshape(M, K)
    rs = raw[2 * plane:2 * plane + Mp * 4].view(np.float32)
    return hi, lo, rs


@pytest.mark.parametrize("C,start,count", [(1024, 0, 512), (1024, 128, 256), (128, 0, 320)])
def test_gelu_into_split_is_the_split_of_the_gelu_output(C, start, count):
    """fc1 with its GELU written straight into the fc2 split (mode 4, scales fixed beforehand
    by triposplat_b200_ln_modulate_split_bound) against fc1 storing fp32 GELU (mode 1):
    every plane element is bit-identical to splitting that fp32 output under the bound's
    scale (hi = rn16(a), lo = rn16(a - hi), a = GELU(y) * 2^s); the scale is never below the
    exact-max scale, never looser than 2^8 here, and keeps |a| < 2^15; fc2 over both splits
    agrees to the GEMM tolerance.  C = 128 takes the LayerNorm kernel's generic path."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(90 + C + start)
    B, L, N = 2, 149, 640  # M = 298: two padding rows in the row-scale array
    M = B * L
    x = (torch.randn(B, L, C, generator=g) * 2 + 0.3).cuda()
    shift = (torch.randn(B, C, generator=g) * 0.1).cuda()
    scale = (torch.randn(B, C, generator=g) * 0.1).cuda()
    c01, q2, sc = _pack(torch.randn(N, C, generator=g) * 0.05)
    bias = (torch.randn(N, generator=g) * 0.02).numpy()
    w = [_cuda(a) for a in (c01, q2, sc, bias)]
    c_nk, q_nk = _to_nk(lib, w[0], w[1])
    wd = (c01.astype(np.float64) * 256 + q2.astype(np.float64)) * sc.astype(np.float64)
    wnorm = float(np.sqrt((wd ** 2).sum(0)).max()) * (1 + 2 ** -20)
    bmax = float(np.abs(bias).max()) * (1 + 2 ** -20)
    keep_a, spa = _split_buf(lib, M, C)
    assert lib.triposplat_b200_ln_modulate_split(x.data_ptr(), M, C, 1e-6, shift.data_ptr(),
                                                 scale.data_ptr(), C, L, spa) == 0
    hid = torch.empty(M, count, device="cuda")
    assert lib.triposplat_b200_gemm_nf24_split_nk(spa, M, C, c_nk.data_ptr(), q_nk.data_ptr(), C,
                                                  w[2].data_ptr(), w[3].data_ptr(), hid.data_ptr(),
                                                  N, start, count, count, 1, None, 0, 1) == 0
    keep_r, spr = _split_buf(lib, M, count)  # the exact-max split of the fp32 hidden layer
    assert lib.triposplat_b200_split_f32(hid.data_ptr(), M, count, count, spr) == 0
    keep_b, spb = _split_buf(lib, M, C)
    keep_h, sph = _split_buf(lib, M, count)
    assert lib.triposplat_b200_ln_modulate_split_bound(
        x.data_ptr(), M, C, 1e-6, shift.data_ptr(), scale.data_ptr(), C, L, spb, sph, count,
        wnorm, bmax) == 0
    assert lib.triposplat_b200_gemm_nf24_split_nk(spb, M, C, c_nk.data_ptr(), q_nk.data_ptr(), C,
                                                  w[2].data_ptr(), w[3].data_ptr(), sph, N, start,
                                                  count, count, 4, None, 0, 1) == 0
    torch.cuda.synchronize()
    # the LayerNorm split itself is unchanged by the extra output
    for pa, pb in zip(_split_planes(keep_a, spa, M, C), _split_planes(keep_b, spb, M, C)):
        assert np.array_equal(pa.view(np.uint8), pb.view(np.uint8))
    hi, lo, rs = _split_planes(keep_h, sph, M, count)
    _, _, rs_exact = _split_planes(keep_r, spr, M, count)
    assert (rs[M:] == 0).all()
    rs = rs[:M]
    ratio = rs / rs_exact[:M]
    assert (ratio >= 1).all() and (ratio <= 2.0 ** 8).all(), (ratio.min(), ratio.max())
    a = hid.cpu().numpy() * (np.float32(1) / rs[:, None])  # exact: a power of two
    assert np.abs(a).max() < 2.0 ** 15
    hi_ref = a.astype(np.float16)
    lo_ref = (a - hi_ref.astype(np.float32)).astype(np.float16)
    assert np.array_equal(hi.view(np.uint16), hi_ref.view(np.uint16)), int((hi != hi_ref).sum())
    assert np.array_equal(lo.view(np.uint16), lo_ref.view(np.uint16)), int((lo != lo_ref).sum())
    # fc2 over the two splits
    c2, q22, sc2 = _pack(torch.randn(C, count, generator=g) * 0.05)
    w2 = [_cuda(a) for a in (c2, q22, sc2, np.zeros(C, np.float32))]
    c2_nk, q2_nk = _to_nk(lib, w2[0], w2[1])
    outs = []
    for sp in (spr, sph):
        o = torch.empty(M, C, device="cuda")
        assert lib.triposplat_b200_gemm_nf24_split_nk(sp, M, count, c2_nk.data_ptr(), q2_nk.data_ptr(),
                                                      count, w2[2].data_ptr(), w2[3].data_ptr(),
                                                      o.data_ptr(), C, 0, C, C, 0, None, 0, 1) == 0
        outs.append(o)
    torch.cuda.synchronize()
    _assert_close(outs[1].cpu().numpy(), outs[0].cpu().numpy())


def test_gelu_into_split_rejects_bad_arguments():
    import _native

    lib = _native.load()
    t = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = (t.data_ptr() + 255) & ~255
    f = lib.triposplat_b200_gemm_nf24_split_nk
    assert f(p, 16, 64, p, p, 64, p, p, p, 64, 0, 64, 64, 5, None, 0, 1) == -2      # no mode 5
    assert f(p, 16, 64, p, p, 64, p, p, p, 64, 0, 64, 80, 4, None, 0, 1) == -4      # stride != count
    assert f(p, 16, 64, p, p, 64, p, p, p + 16, 64, 0, 64, 64, 4, None, 0, 1) == -4  # 256-byte split
    b = lib.triposplat_b200_ln_modulate_split_bound
    assert b(p, 4, 64, 1e-6, None, None, 64, 4, p, None, 64, 1.0, 0.0) == -1
    assert b(p, 4, 64, 1e-6, None, None, 64, 4, p, p, 0, 1.0, 0.0) == -2
    assert b(p, 4, 64, 1e-6, None, None, 64, 4, p, p, 64, -1.0, 0.0) == -2
    assert b(p, 4, 64, 1e-6, None, None, 64, 4, p, p, 64, float("nan"), 0.0) == -2
    assert b(p, 4, 64, 1e-6, None, None, 64, 4, p, p + 16, 64, 1.0, 0.0) == -4
    assert lib.triposplat_b200_status() == 0
