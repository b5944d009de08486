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
