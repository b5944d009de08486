"""The reference's fused NF24 entry points on the GPU, through the C-ABI:
``triposplat_mlp_nf24_gelu_f32_avx512`` (+ the chunked variant) and
``triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512``.

Checked against the reference's own outputs (tests/golden/mlp_nf24.npz and qkv_direct.npz,
made by tests/golden/make_golden.py) with the GEMM tolerance of the reference smoke test
(rtol = atol = 2e-5, scripts/smoke_native_rnf8_avx512.py:58), against the composition of
this library's unfused entries (the same kernels: identical bits for the QKV projection,
within 1e-6 for the MLP, whose GELU is compiled into the fc1 epilogue), and for the reference's
status codes.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-5, atol=2e-5)

# (M, K, H, N, stride_x, stride_out) the reference's MLP rejects with -2
# (scripts/native_nf24_mlp_avx512.c:164-165); tests/test_reference_status_codes.py checks
# the reference library returns -2 for the same rows
MLP_BAD_SIZES = ((0, 1024, 4096, 1024, 1024, 1024), (4, 512, 4096, 1024, 1024, 1024),
                 (4, 1024, 2048, 1024, 1024, 1024), (4, 1024, 4096, 1024, 1000, 1024),
                 (4, 1024, 4096, 1024, 1024, 1000))
# (B, L, K, N, H, D, L_padded, frequency_batches, stages) rejected with -2 by the fused QKV
# projection (scripts/gemm_nf24_qkv_direct_avx512.c:117-119); base case B 1, L 4, K 64, H 1
QKV_BAD_SIZES = ((1, 4, 64, 208, 1, 64, 16, 1, 3), (1, 4, 64, 192, 1, 32, 16, 1, 3),
                 (1, 4, 64, 192, 1, 64, 8, 1, 3), (1, 20, 64, 192, 1, 64, 24, 1, 3),
                 (1, 4, 64, 192, 1, 64, 16, 3, 3), (1, 4, 64, 192, 1, 64, 16, 1, 2))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _pack_dev(w, b):
    from nf24_pack import quantize_nf24_i16_per_output_channel

    codes, scales, _ = quantize_nf24_i16_per_output_channel(torch.as_tensor(w))
    return (codes[0].cuda(), codes[1].cuda(), scales[0].cuda(), _dev(b)), \
        (codes[0].numpy(), codes[1].numpy())


def _mlp_weights(g):
    from test_oracle_golden import _make_golden

    mg = _make_golden()
    w1, w2, b1, b2 = mg.mlp_weights(int(g["seed"]))
    d1, h1 = _pack_dev(w1, b1)
    d2, h2 = _pack_dev(w2, b2)
    assert mg.code_digest(*h1) == str(g["w1_digest"])
    assert mg.code_digest(*h2) == str(g["w2_digest"])
    return d1, d2


def test_mlp_golden_plain_and_chunked(golden):
    from nf24_linear import nf24_mlp_gelu

    g = golden("mlp_nf24")
    w1, w2 = _mlp_weights(g)
    x = _dev(g["x"])[:, :1024]                       # row stride 1040
    for chunk in (None, int(g["chunk_rows"]), 1, 64):
        buf = torch.full((x.shape[0], int(g["stride_out"])), 5.0, device="cuda")
        y = nf24_mlp_gelu(x, w1, w2, out=buf[:, :1024], chunk_rows=chunk)
        torch.cuda.synchronize()
        got = buf.cpu().numpy()
        np.testing.assert_allclose(got[:, :1024], g["out"][:, :1024], **TOL)
        assert (got[:, 1024:] == 5.0).all()          # padding of each row untouched
        assert y.data_ptr() == buf.data_ptr()


def test_mlp_equals_unfused_composition():
    """Fused MLP == nf24_linear(fc1) -> GELU -> nf24_linear(fc2) through the unfused
    entries (the same split / tensor-core kernels; the GELU in the fc1 epilogue is the
    standalone GELU kernel's formula, compiled separately, hence a 1e-6 bound)."""
    from native_ops import gelu_tanh
    from nf24_linear import nf24_linear, nf24_mlp_gelu

    g = torch.Generator().manual_seed(3)
    M = 517
    x = torch.randn(M, 1024, generator=g).cuda()
    w1, _ = _pack_dev(torch.randn(4096, 1024, generator=g) * 0.02,
                      (torch.randn(4096, generator=g) * 0.01).numpy())
    w2, _ = _pack_dev(torch.randn(1024, 4096, generator=g) * 0.02,
                      (torch.randn(1024, generator=g) * 0.01).numpy())
    ref = nf24_linear(gelu_tanh(nf24_linear(x, *w1)), *w2)
    y = nf24_mlp_gelu(x, w1, w2)
    yc = nf24_mlp_gelu(x, w1, w2, chunk_rows=200)
    torch.cuda.synchronize()
    # rows are independent: chunking changes no bit
    assert torch.equal(yc, y), float((yc - y).abs().max())
    torch.testing.assert_close(y, ref, rtol=1e-6, atol=1e-6)


def test_mlp_codes_copy_path_is_the_direct_path_row_for_row():
    """From 2048 rows the fused MLP copies both weights' codes into k-contiguous planes once
    per call (the chunked variant once for all chunks); fewer rows read the [K][N] planes.
    Rows are independent and both paths issue the same MMAs per row, so the first 700 rows
    of a 2300-row call, plain or chunked, equal a 700-row call bit for bit."""
    from nf24_linear import nf24_mlp_gelu

    g = torch.Generator().manual_seed(5)
    M = 2300
    x = torch.randn(M, 1024, generator=g).cuda()
    w1, _ = _pack_dev(torch.randn(4096, 1024, generator=g) * 0.02,
                      (torch.randn(4096, generator=g) * 0.01).numpy())
    w2, _ = _pack_dev(torch.randn(1024, 4096, generator=g) * 0.02,
                      (torch.randn(1024, generator=g) * 0.01).numpy())
    y = nf24_mlp_gelu(x, w1, w2)
    yc = nf24_mlp_gelu(x, w1, w2, chunk_rows=512)
    ys = nf24_mlp_gelu(x[:700].contiguous(), w1, w2)
    torch.cuda.synchronize()
    assert torch.equal(y, yc)
    assert torch.equal(y[:700], ys)


def test_mlp_status_codes():
    import _native

    lib = _native.load()
    d = torch.zeros(4, 1024, device="cuda")
    c1 = torch.zeros(1024, 4096, dtype=torch.int16, device="cuda")
    q1 = torch.zeros(1024, 4096, dtype=torch.int8, device="cuda")
    c2 = torch.zeros(4096, 1024, dtype=torch.int16, device="cuda")
    q2 = torch.zeros(4096, 1024, dtype=torch.int8, device="cuda")
    s1 = torch.zeros(4096, device="cuda")
    s2 = torch.zeros(1024, device="cuda")
    out = torch.empty(4, 1024, device="cuda")
    p = [d.data_ptr(), c1.data_ptr(), q1.data_ptr(), s1.data_ptr(), s1.data_ptr(),
         c2.data_ptr(), q2.data_ptr(), s2.data_ptr(), s2.data_ptr(), out.data_ptr()]
    f = lib.triposplat_mlp_nf24_gelu_f32_avx512
    assert f(*p, 4, 1024, 4096, 1024, 1024, 1024, 0) == 0
    assert f(*(p[:9] + [None]), 4, 1024, 4096, 1024, 1024, 1024, 0) == -1
    for args in MLP_BAD_SIZES:
        assert f(*p, *args, 0) == -2, args
    host = np.zeros((4, 1024), np.float32)
    assert f(*([host.ctypes.data] + p[1:]), 4, 1024, 4096, 1024, 1024, 1024, 0) == -9
    fc = lib.triposplat_mlp_nf24_gelu_chunked_f32_avx512
    hid = torch.empty(2, 4096, device="cuda")
    pc = p[:9] + [hid.data_ptr(), out.data_ptr()]
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 2, 2, 0) == 0
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 1, 2, 0) == -2   # capacity < chunk
    assert fc(*pc, 4, 1024, 4096, 1024, 1024, 1024, 2, 0, 0) == -2   # chunk_rows 0
    torch.cuda.synchronize()
    assert lib.triposplat_mlp_nf24_row_tile() > 0
    assert lib.triposplat_mlp_nf24_hidden_workspace_bytes_per_thread() > 0


@pytest.mark.parametrize("fb", [1, 2])
def test_qkv_direct_golden(golden, fb):
    from nf24_linear import nf24_qkv_rope_rmsnorm_pack

    g = golden("qkv_direct")
    q, pk, pv = nf24_qkv_rope_rmsnorm_pack(
        _dev(g["x"]), _dev(g["code01_t"]), _dev(g["q2_t"]), _dev(g["scale"]), _dev(g["bias"]),
        _dev(g[f"freqs{fb}"]), _dev(g[f"qg{fb}"]), _dev(g[f"kg{fb}"]), batch=2, heads=2,
        L_padded=16)
    torch.cuda.synchronize()
    np.testing.assert_allclose(q.cpu().numpy(), g[f"q{fb}"], **TOL)
    np.testing.assert_allclose(pk.cpu().numpy(), g[f"pk{fb}"], **TOL)
    np.testing.assert_allclose(pv.cpu().numpy(), g[f"pv{fb}"], **TOL)
    assert (pk[..., 11:] == 0).all() and (pv[..., 11:] == 0).all()


def test_qkv_direct_equals_unfused_composition():
    """At the model's width (K 1024, 16 heads, L 333 padded to 336, per-batch frequencies)
    the fused entry gives the bits of nf24_linear followed by the v2 post-process."""
    from native_ops import qkv_rope_rmsnorm_pack
    from nf24_linear import nf24_linear, nf24_qkv_rope_rmsnorm_pack

    g = torch.Generator().manual_seed(9)
    B, L, H, D, K = 2, 333, 16, 64, 1024
    x = torch.randn(B * L, K, generator=g).cuda()
    w, _ = _pack_dev(torch.randn(3 * H * D, K, generator=g) * 0.02,
                     (torch.randn(3 * H * D, generator=g) * 0.01).numpy())
    ang = torch.rand(B, L, H, D // 2, generator=g) * 6.0
    freqs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).reshape(B, L, H, D).cuda()
    qg = (1.0 + 0.05 * torch.randn(H, D, generator=g)).cuda()
    kg = (1.0 + 0.05 * torch.randn(H, D, generator=g)).cuda()
    q, pk, pv = nf24_qkv_rope_rmsnorm_pack(x, *w, freqs, qg, kg, batch=B, heads=H)
    qkv = nf24_linear(x, *w).view(B, L, 3, H, D)
    rq, rpk, rpv = qkv_rope_rmsnorm_pack(qkv, freqs, qg, kg)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(pk, rpk) and torch.equal(pv, rpv)


def test_qkv_direct_codes_copy_path_is_the_direct_path():
    """From 2048 token rows (B*L) the fused QKV projection reads a k-contiguous copy of its
    codes; the result still equals nf24_linear + the v2 post-process bit for bit (the
    unfused GEMM takes the same copy path), and batch 0's first 500 tokens equal a
    500-token call (per-token arithmetic, positions 0..499 in both)."""
    from native_ops import qkv_rope_rmsnorm_pack
    from nf24_linear import nf24_linear, nf24_qkv_rope_rmsnorm_pack

    g = torch.Generator().manual_seed(11)
    B, L, H, D, K = 2, 1100, 16, 64, 1024
    x = torch.randn(B * L, K, generator=g).cuda()
    w, _ = _pack_dev(torch.randn(3 * H * D, K, generator=g) * 0.02,
                     (torch.randn(3 * H * D, generator=g) * 0.01).numpy())
    ang = torch.rand(1, L, H, D // 2, generator=g) * 6.0
    freqs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).reshape(1, L, H, D).cuda()
    qg = (1.0 + 0.05 * torch.randn(H, D, generator=g)).cuda()
    kg = (1.0 + 0.05 * torch.randn(H, D, generator=g)).cuda()
    q, pk, pv = nf24_qkv_rope_rmsnorm_pack(x, *w, freqs, qg, kg, batch=B, heads=H)
    qkv = nf24_linear(x, *w).view(B, L, 3, H, D)
    rq, rpk, rpv = qkv_rope_rmsnorm_pack(qkv, freqs, qg, kg)
    Ls = 500
    sq, spk, spv = nf24_qkv_rope_rmsnorm_pack(x[:Ls].contiguous(), *w,
                                              freqs[:, :Ls].contiguous(), qg, kg, batch=1,
                                              heads=H)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(pk, rpk) and torch.equal(pv, rpv)
    assert torch.equal(q[0, :, :Ls], sq[0])
    assert torch.equal(pk[0, :, :, :Ls], spk[0, :, :, :Ls])
    assert torch.equal(pv[0, :, :, :Ls], spv[0, :, :, :Ls])


def test_qkv_direct_status_codes():
    import _native

    lib = _native.load()
    f = lib.triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512
    B, L, K, H, D, Lp = 1, 4, 64, 1, 64, 16
    N = 3 * H * D
    t = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device="cuda")  # noqa: E731
    x, c, q, s = t(B * L, K), t(K, N, dt=torch.int16), t(K, N, dt=torch.int8), t(N)
    fr, gm = t(1, L, H, D), t(H, D)
    qo, pk, pv = t(B, H, L, D), t(B, H, D, Lp), t(B, H, D, Lp)
    p = [x, c, q, q, s, s, s, t(256), s, fr, gm, gm, qo, pk, pv]
    p = [a.data_ptr() for a in p]
    assert f(*p, B, L, K, N, H, D, Lp, 1, 0, 3) == 0
    assert f(*(p[:14] + [None]), B, L, K, N, H, D, Lp, 1, 0, 3) == -1
    for args in QKV_BAD_SIZES:
        a = list(args)
        assert f(*p, *a[:8], 0, a[8]) == -2, args
    torch.cuda.synchronize()
    assert lib.triposplat_gemm_nf24_qkv_direct_residual_mode() == 4
