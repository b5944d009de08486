"""Fused QKV post-process -> attention: bit-identical to the two-call path.

`triposplat_b200_qkv_rope_rmsnorm_sdpa_f32` (self-attention) and
`triposplat_b200_q_kv_rmsnorm_sdpa_f32` (cross-attention) write q / k / v straight into the
attention's split format; the reference route is the post-process to fp32 q and packed
k / v, then the packed SDPA.  Both must give the same bits: same RoPE / RMSNorm arithmetic,
same power-of-two pre-scales, same attention kernel.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _freqs(L, H, g):
    ang = torch.rand(L, H, 32, generator=g, dtype=torch.float64) * 6.28
    f = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).reshape(1, L, H, 64)
    return f.float().cuda()


@pytest.mark.parametrize("B,L,H", [(1, 1, 1), (2, 300, 3), (1, 1000, 2)])
def test_fused_self_attention_bitwise(B, L, H):
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(L + H)
    qkv = torch.randn(B, L, 3, H, 64, generator=g).cuda()
    fr = _freqs(L, H, g)
    qg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    kg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    Lp = (L + 15) // 16 * 16
    q = torch.empty(B, H, L, 64, device="cuda")
    pk = torch.empty(B, H, 64, Lp, device="cuda")
    pv = torch.empty(B, H, 64, Lp, device="cuda")
    ref = torch.empty(B, L, H, 64, device="cuda")
    assert lib.triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(
        qkv.data_ptr(), fr.data_ptr(), qg.data_ptr(), kg.data_ptr(), q.data_ptr(), pk.data_ptr(),
        pv.data_ptr(), B, L, H, 64, Lp, 1, 0) == 0
    assert lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
        q.data_ptr(), pk.data_ptr(), pv.data_ptr(), None, ref.data_ptr(), B, H, L, L, 64, Lp, 0, 0, 0) == 0
    out = torch.full((B, L, H, 64), float("nan"), device="cuda")
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(
        qkv.data_ptr(), fr.data_ptr(), qg.data_ptr(), kg.data_ptr(), out.data_ptr(), B, L, H, 64, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref), float((out - ref).abs().max())


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 5, 3, 1), (2, 200, 137, 2), (1, 300, 1374, 2)])
def test_fused_cross_attention_bitwise(B, Lq, Lk, H):
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(Lq * 7 + Lk)
    y = torch.randn(B, Lq, H, 64, generator=g).cuda()
    kv = torch.randn(B, Lk, 2, H, 64, generator=g).cuda()
    qg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    kg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    Lkp = (Lk + 15) // 16 * 16
    q = torch.empty(B, H, Lq, 64, device="cuda")
    pk = torch.empty(B, H, 64, Lkp, device="cuda")
    pv = torch.empty(B, H, 64, Lkp, device="cuda")
    ref = torch.empty(B, Lq, H, 64, device="cuda")
    assert lib.triposplat_b200_q_kv_rmsnorm_pack_f32(
        y.data_ptr(), kv.data_ptr(), qg.data_ptr(), kg.data_ptr(), q.data_ptr(), pk.data_ptr(),
        pv.data_ptr(), B, Lq, Lk, H, Lkp) == 0
    assert lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
        q.data_ptr(), pk.data_ptr(), pv.data_ptr(), None, ref.data_ptr(), B, H, Lq, Lk, 64, Lkp, 0, 0, 0) == 0
    out = torch.full((B, Lq, H, 64), float("nan"), device="cuda")
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_f32(
        y.data_ptr(), kv.data_ptr(), qg.data_ptr(), kg.data_ptr(), out.data_ptr(), B, Lq, Lk, H) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref), float((out - ref).abs().max())


def test_fused_entry_errors():
    import _native

    lib = _native.load()
    p = torch.zeros(1024, device="cuda").data_ptr()
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(None, p, p, p, p, 1, 4, 1, 64, 1) == -1
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(p, p, p, p, p, 1, 4, 1, 32, 1) == -2
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(p, p, p, p, p, 2, 4, 1, 64, 3) == -2
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_f32(p, p, p, p, p, 1, 0, 3, 1) == -2
    host = np.zeros(1024, np.float32)
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_f32(host.ctypes.data, p, p, p, p, 1, 2, 3, 1) == -9


def _split_buf(lib, M, K):
    n = int(lib.triposplat_b200_split_bytes(M, K))
    t = torch.empty(n + 256, dtype=torch.uint8, device="cuda")
    return t, (t.data_ptr() + 255) & ~255


def _check_output_split(keep, sp, out, B, Lq):
    """The split planes of the [B*Lq, H*64] output against the fp32 output `out`: one row
    scale per batch, never below the row's exact-max scale, |a| < 2^15, and hi / lo bit-
    identical to rn16(a), rn16(a - hi) of a = out / rs."""
    o = out.reshape(B * Lq, -1).cpu().numpy()
    M, K = o.shape
    plane = (M * K * 2 + 255) // 256 * 256
    raw = keep[sp - keep.data_ptr():].cpu().numpy()
    hi = raw[:M * K * 2].view(np.float16).reshape(M, K)
    lo = raw[plane:plane + M * K * 2].view(np.float16).reshape(M, K)
    rs = raw[2 * plane:2 * plane + M * 4].view(np.float32)
    for b in range(B):
        assert (rs[b * Lq:(b + 1) * Lq] == rs[b * Lq]).all()
    mx = np.abs(o).max(axis=1)
    exact = np.exp2(-(14 - np.floor(np.log2(mx))))
    assert (rs >= exact).all()
    a = o * (np.float32(1) / rs)[:, None]
    assert np.abs(a).max() < 2.0 ** 15
    hi_ref = a.astype(np.float16)
    lo_ref = (a - hi_ref.astype(np.float32)).astype(np.float16)
    assert np.array_equal(hi.view(np.uint16), hi_ref.view(np.uint16)), int((hi != hi_ref).sum())
    assert np.array_equal(lo.view(np.uint16), lo_ref.view(np.uint16)), int((lo != lo_ref).sum())


@pytest.mark.parametrize("B,L,H", [(2, 300, 3), (1, 1000, 2)])
def test_self_attention_into_split(B, L, H):
    """triposplat_b200_qkv_rope_rmsnorm_sdpa_split: the fp32 entry's output, split under a
    per-batch scale fixed from the V tiles' pre-scales."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(3 * L + H)
    qkv = torch.randn(B, L, 3, H, 64, generator=g).cuda()
    qkv[1 % B, :, 2] *= 40.0  # batches with different value ranges
    fr = _freqs(L, H, g)
    qg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    kg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    out = torch.empty(B, L, H, 64, device="cuda")
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(
        qkv.data_ptr(), fr.data_ptr(), qg.data_ptr(), kg.data_ptr(), out.data_ptr(), B, L, H, 64, 1) == 0
    keep, sp = _split_buf(lib, B * L, H * 64)
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_split(
        qkv.data_ptr(), fr.data_ptr(), qg.data_ptr(), kg.data_ptr(), B, L, H, 1, sp) == 0
    torch.cuda.synchronize()
    _check_output_split(keep, sp, out, B, L)


def test_cross_attention_into_split_and_cached_rows():
    """triposplat_b200_q_kv_rmsnorm_sdpa_split and the cached-planes route (q_split +
    kv_split + triposplat_b200_attend_rows_split) against the fp32 cross-attention."""
    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(17)
    B, Lq, Lk, H = 2, 200, 137, 2
    y = torch.randn(B, Lq, H, 64, generator=g).cuda()
    kv = torch.randn(B, Lk, 2, H, 64, generator=g).cuda()
    qg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    kg = (1 + 0.1 * torch.randn(H, 64, generator=g)).cuda()
    out = torch.empty(B, Lq, H, 64, device="cuda")
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_f32(
        y.data_ptr(), kv.data_ptr(), qg.data_ptr(), kg.data_ptr(), out.data_ptr(), B, Lq, Lk, H) == 0
    keep, sp = _split_buf(lib, B * Lq, H * 64)
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_split(
        y.data_ptr(), kv.data_ptr(), qg.data_ptr(), kg.data_ptr(), B, Lq, Lk, H, sp) == 0
    qb = torch.empty(int(lib.triposplat_b200_attn_q_planes_bytes(B * H, Lq)) + 256, dtype=torch.uint8, device="cuda")
    kb = torch.empty(int(lib.triposplat_b200_attn_kv_planes_bytes(B * H, Lk)) + 256, dtype=torch.uint8, device="cuda")
    qp, kp = (qb.data_ptr() + 255) & ~255, (kb.data_ptr() + 255) & ~255
    assert lib.triposplat_b200_kv_split_f32(kv.data_ptr(), kg.data_ptr(), B, Lk, H, kp) == 0
    assert lib.triposplat_b200_q_split_f32(y.data_ptr(), qg.data_ptr(), B, Lq, H, qp) == 0
    keep2, sp2 = _split_buf(lib, B * Lq, H * 64)
    assert lib.triposplat_b200_attend_rows_split(qp, kp, B, H, Lq, Lk, sp2) == 0
    torch.cuda.synchronize()
    _check_output_split(keep, sp, out, B, Lq)
    _check_output_split(keep2, sp2, out, B, Lq)
    p = sp
    assert lib.triposplat_b200_attend_rows_split(qp, kp, B, H, Lq, Lk, p + 16) == -4
    assert lib.triposplat_b200_q_kv_rmsnorm_sdpa_split(None, p, p, p, B, Lq, Lk, H, p) == -1
    assert lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_split(p, p, p, p, 2, 4, 1, 3, p) == -2
    assert lib.triposplat_b200_status() == 0
