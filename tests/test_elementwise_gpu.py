"""Prologue/epilogue kernels: CUDA (C-ABI) vs golden vectors from the reference kernels.

Tolerance: rtol = atol = 2e-6 (fp32 with a different reduction order / libm), except
packed V which is a pure copy and must be bit-identical.
"""
import numpy as np
import pytest
import torch

import native_ops as ops

pytestmark = pytest.mark.gpu
TOL = dict(rtol=2e-6, atol=2e-6)


def c(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def h(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_norms_and_rope(golden):
    g = golden("elementwise")
    np.testing.assert_allclose(h(ops.layernorm(c(g["ln_x"]), c(g["ln_w"]), c(g["ln_b"]), 1e-6)), g["ln_out"], **TOL)
    np.testing.assert_allclose(h(ops.layernorm(c(g["ln_x"]), eps=1e-5)), g["ln_out_noaffine"], **TOL)
    np.testing.assert_allclose(h(ops.multihead_rmsnorm(c(g["rms_x"]), c(g["rms_gamma"]))), g["rms_out"], **TOL)
    np.testing.assert_allclose(h(ops.rope_complex(c(g["rope_x"]), c(g["rope_f"]))), g["rope_out"], **TOL)


def test_activations(golden):
    g = golden("elementwise")
    np.testing.assert_allclose(h(ops.gelu_tanh(c(g["act_x"]))), g["gelu_out"], **TOL)
    np.testing.assert_allclose(h(ops.silu(c(g["act_x"]))), g["silu_out"], **TOL)


def test_block_elementwise(golden):
    g = golden("elementwise")
    np.testing.assert_allclose(h(ops.modulate_inplace(c(g["mod_h"]), c(g["mod_scale"]), c(g["mod_shift"]))), g["mod_out"], **TOL)
    base, delta = c(g["gres_base"]), c(g["gres_delta"])
    ops.gated_residual_inplace(base, delta, c(g["gres_gate"]))
    np.testing.assert_allclose(h(base), g["gres_base_out"], **TOL)
    np.testing.assert_allclose(h(delta), g["gres_delta_out"], **TOL)
    np.testing.assert_allclose(h(ops.add_inplace(c(g["gres_base"]), c(g["gres_delta"]))), g["add_out"], **TOL)


def test_sampler_updates(golden):
    g = golden("elementwise")
    np.testing.assert_allclose(h(ops.cfg_combine_inplace(c(g["cfg_pos"]), c(g["cfg_neg"]), c(g["cfg_g"]))), g["cfg_out"], **TOL)
    np.testing.assert_allclose(h(ops.euler_update_inplace(c(g["cfg_pos"]), c(g["cfg_neg"]), c(g["euler_dt"]))), g["euler_out"], **TOL)


def test_qkv_postprocess(golden):
    g = golden("elementwise")
    q, pk, pv = ops.qkv_rope_rmsnorm_pack(c(g["post_qkv"]), c(g["post_freqs"]), c(g["post_qg"]), c(g["post_kg"]), L_padded=32)
    np.testing.assert_allclose(h(q), g["post_q"], **TOL)
    np.testing.assert_allclose(h(pk), g["post_pk"], **TOL)
    np.testing.assert_array_equal(h(pv), g["post_pv"])


def test_qkv_postprocess_first_version_symbol(golden):
    """triposplat_qkv_rope_rmsnorm_pack_f32_avx512 (the reference's first version, same
    arguments) gives the bits of _v2, zero tail included; the aux queries answer."""
    import _native

    lib = _native.load()
    g = golden("elementwise")
    qkv = c(g["post_qkv"])
    B, L, _, H, D = (int(x) for x in qkv.shape)
    fr, qg, kg = c(g["post_freqs"]), c(g["post_qg"]), c(g["post_kg"])
    outs = []
    for name in ("triposplat_qkv_rope_rmsnorm_pack_f32_avx512",
                 "triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2"):
        q = torch.full((B, H, L, D), 3.0, device="cuda")
        pk = torch.full((B, H, D, 32), 3.0, device="cuda")
        pv = torch.full((B, H, D, 32), 3.0, device="cuda")
        assert getattr(lib, name)(qkv.data_ptr(), fr.data_ptr(), qg.data_ptr(), kg.data_ptr(),
                                  q.data_ptr(), pk.data_ptr(), pv.data_ptr(), B, L, H, D, 32,
                                  int(fr.shape[0]), 0) == 0
        outs.append((h(q), h(pk), h(pv)))
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_allclose(outs[0][0], g["post_q"], **TOL)
    np.testing.assert_array_equal(outs[0][2], g["post_pv"])
    assert lib.triposplat_qkv_postprocess_token_tile() == 64  # the GPU kernel's tile (reference CPU: 16)
    assert lib.triposplat_qkv_postprocess_v2_tail_only_clear() == 1


def test_qkv_selected_postprocess(oracle, golden):
    """Selected-query variant: queries use the frequency row of their selected token."""
    g = golden("elementwise")
    qkv = g["post_qkv"]  # [B, L, 3, H, 64]
    B, L, _, H, D = qkv.shape
    sel = np.array([0, 3, 5, 18], np.int64)
    q_sel = np.ascontiguousarray(qkv[:, sel, 0])            # [B, Lq, H, 64]
    kv = np.ascontiguousarray(qkv[:, :, 1:3])               # [B, L, 2, H, 64]
    qo, pk, pv = ops.q_kv_selected_rope_rmsnorm_pack(c(q_sel), c(kv), c(g["post_freqs"]), c(sel),
                                                     c(g["post_qg"]), c(g["post_kg"]), Lk_padded=32)
    np.testing.assert_allclose(h(qo), g["post_q"][:, :, sel], **TOL)
    np.testing.assert_allclose(h(pk), g["post_pk"], **TOL)
    np.testing.assert_array_equal(h(pv), g["post_pv"])
    bad = c(np.array([0, 99, 1, 2], np.int64))
    with pytest.raises(RuntimeError):
        ops.q_kv_selected_rope_rmsnorm_pack(c(q_sel), c(kv), c(g["post_freqs"]), bad, c(g["post_qg"]), c(g["post_kg"]), Lk_padded=32)


def test_large_rows_vs_oracle(oracle):
    """Full-width rows (the block's 8193 x 1024 activations) against the oracle."""
    gen = torch.Generator().manual_seed(2)
    x = (torch.randn(2 * 8193, 1024, generator=gen) * 3 + 1).numpy()
    np.testing.assert_allclose(h(ops.layernorm(c(x), eps=1e-6)), oracle.layernorm(x, eps=1e-6), rtol=1e-5, atol=1e-5)
    xg = x[:64]
    np.testing.assert_allclose(h(ops.gelu_tanh(c(xg))), oracle.gelu_tanh(xg), **TOL)


def test_embeddings_bit_exact(golden):
    """Timestep / point-cloud position embeddings, RePo phasor and feature multiply through
    the C-ABI reproduce the reference's AVX-512 kernels bit for bit (same sin / cos method,
    operation for operation), including angles of 1e3..1e4 rad."""
    import native_ops as ops

    g = golden("embeddings")
    out = ops.timestep_embedding(c(g["ts_t"]), c(g["ts_f"]), g["ts_out"].shape[1])
    np.testing.assert_array_equal(out.cpu().numpy(), g["ts_out"])
    for dp in (0, 1):
        out = ops.pcd_position_embedding(c(g["pcd_pos"]), c(g["pcd_f"]),
                                         g[f"pcd_out{dp}"].shape[1], double_pi=bool(dp))
        np.testing.assert_array_equal(out.cpu().numpy(), g[f"pcd_out{dp}"])
    lib = __import__("_native").load()
    for name in ("a", "b"):
        dims = [int(d) for d in g[f"repo_{name}_dims"]]
        ft = [c(g[f"repo_{name}_ft{a}"]) for a in range(3)]
        fr = [c(g[f"repo_{name}_fr{a}"]) for a in range(3)]
        delta = c(g[f"repo_{name}_delta"])
        out = torch.empty(delta.shape[0], 2 * sum(dims), device="cuda")
        assert lib.triposplat_repo_phasor_f32_avx512(
            delta.data_ptr(), ft[0].data_ptr(), fr[0].data_ptr(), dims[0], ft[1].data_ptr(),
            fr[1].data_ptr(), dims[1], ft[2].data_ptr(), fr[2].data_ptr(), dims[2],
            out.data_ptr(), delta.shape[0], 0) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), g[f"repo_{name}_out"])
    lhs = c(g["mul_lhs"])
    ops.mul_inplace(lhs, c(g["mul_rhs"]))
    np.testing.assert_array_equal(lhs.cpu().numpy(), g["mul_out"])


def test_repo_phasor_mirror_and_errors():
    """native_ops.repo_phasor splits each frequency vector as tanh(f) + (f - tanh(f)) and
    returns complex64 [B, L, heads, sum(dims)]; the C-ABI returns the reference's codes."""
    import native_ops as ops

    g = torch.Generator().manual_seed(3)
    B, L, heads, dims = 2, 5, 4, (6, 5, 5)
    delta = torch.randn(B, L, 3 * heads, generator=g).cuda()
    freqs = [torch.randn(d, generator=g).cuda() for d in dims]
    z = ops.repo_phasor(delta, freqs)
    assert z.shape == (B, L, heads, sum(dims)) and z.dtype == torch.complex64
    # phasors of angle pi * f * delta (the tanh split sums back to f up to rounding)
    ang = torch.cat([delta.view(B, L, heads, 3)[..., a:a + 1] * f * np.pi for a, f in enumerate(freqs)], -1)
    ref = torch.polar(torch.ones_like(ang), ang)
    assert float((z - ref).abs().max()) < 1e-4
    lib = __import__("_native").load()
    p = delta.data_ptr()
    assert lib.triposplat_repo_phasor_f32_avx512(None, p, p, 1, p, p, 1, p, p, 1, p, 1, 0) == -1
    assert lib.triposplat_repo_phasor_f32_avx512(p, None, p, 1, p, p, 1, p, p, 1, p, 1, 0) == -2
    assert lib.triposplat_repo_phasor_f32_avx512(p, p, p, 0, p, p, 1, p, p, 1, p, 1, 0) == -3
    assert lib.triposplat_mul_inplace_f32_avx512(p, None, 4, 0) == -1
    assert lib.triposplat_pcd_position_embedding_f32_avx512(p, p, p, 2, 3, 4, 20, 0, 0) == -2


def test_sampler_kernels_bit_exact(golden):
    """CFG combine, Euler and AB2 steps round exactly like the reference (bit-identical to its
    golden outputs), and the fused CFG + Euler kernel equals the two calls in sequence."""
    lib = __import__("_native").load()
    __import__("_native").use_current_stream(lib)
    e = golden("elementwise")
    pos, neg, gg = c(e["cfg_pos"]), c(e["cfg_neg"]), c(e["cfg_g"])
    B = gg.numel()
    n = pos.numel() // B
    assert lib.triposplat_cfg_combine_inplace_f32_avx512(pos.data_ptr(), neg.data_ptr(), gg.data_ptr(), B, n, 0) == 0
    np.testing.assert_array_equal(h(pos), e["cfg_out"])
    g = golden("embeddings")
    x = c(g["ab2_x"])
    assert lib.triposplat_ab2_update_inplace_f32_avx512(
        x.data_ptr(), c(g["ab2_v"]).data_ptr(), c(g["ab2_vp"]).data_ptr(), c(g["ab2_dt"]).data_ptr(),
        c(g["ab2_pdt"]).data_ptr(), 2, 333, 0) == 0
    np.testing.assert_array_equal(h(x), g["ab2_out"])
    # fused CFG + Euler == combine then Euler
    gen = torch.Generator().manual_seed(9)
    xs = torch.randn(2, 4097, generator=gen).cuda()
    vp, vn = torch.randn(2, 4097, generator=gen).cuda(), torch.randn(2, 4097, generator=gen).cuda()
    gd, dt = torch.tensor([3.0, 2.5]).cuda(), torch.tensor([0.0427, 0.1]).cuda()
    x2, vp2 = xs.clone(), vp.clone()
    assert lib.triposplat_b200_cfg_euler_update_f32(xs.data_ptr(), vp.data_ptr(), vn.data_ptr(),
                                                    gd.data_ptr(), dt.data_ptr(), 2, 4097) == 0
    assert lib.triposplat_cfg_combine_inplace_f32_avx512(vp2.data_ptr(), vn.data_ptr(), gd.data_ptr(), 2, 4097, 0) == 0
    assert lib.triposplat_euler_update_inplace_f32_avx512(x2.data_ptr(), vp2.data_ptr(), dt.data_ptr(), 2, 4097, 0) == 0
    torch.cuda.synchronize()
    assert torch.equal(xs, x2)
