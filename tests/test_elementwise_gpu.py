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
