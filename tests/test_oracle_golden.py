"""Pin the CPU oracle (oracle/oracle.c) to golden vectors made by the reference's
own AVX-512 kernels (tests/golden/make_golden.py)."""
import numpy as np
import pytest

GEMM_CASES = ["gemm_25x96x64", "gemm_40x96x64", "gemm_10x96x64", "gemm_3x96x5_tail",
              "gemm_7x100x7_tail", "gemm_33x160x96_range32_48", "gemm_130x256x144"]
SDPA_CASES = ["sdpa_self256", "sdpa_masked256", "sdpa_cross193x256", "sdpa_cross5x17_bias",
              "sdpa_q3_k1", "sdpa_q70_k700_bias"]


@pytest.mark.parametrize("case", GEMM_CASES)
def test_gemm_oracle_bit_exact(oracle, golden, case):
    g = golden(case)
    count = int(g["count"])
    out = oracle.gemm_nf24(g["x"], g["code01_t"], g["q2_t"], g["scale"], g["bias"],
                           start=int(g["start"]), count=None if count < 0 else count)
    # same decode and the same in-order fmaf chain as the reference: bit-identical
    np.testing.assert_array_equal(out, g["out"])


@pytest.mark.parametrize("case", SDPA_CASES)
def test_sdpa_oracle_matches_reference(oracle, golden, case):
    g = golden(case)
    out = oracle.sdpa(g["q"], g["k"], g["v"], bias=g.get("bias"))
    # expf vs the reference's polynomial exp and a different reduction order
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=2e-6)
    assert np.sqrt(np.mean((out - g["out"]) ** 2)) < 2e-7
    blhd = oracle.sdpa(g["q"], g["k"], g["v"], bias=g.get("bias"), out_blhd=True)
    np.testing.assert_allclose(blhd, g["out_blhd"], rtol=0, atol=2e-6)


def test_elementwise_oracle(oracle, golden):
    g = golden("elementwise")
    tol = dict(rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(oracle.layernorm(g["ln_x"], g["ln_w"], g["ln_b"], 1e-6), g["ln_out"], **tol)
    np.testing.assert_allclose(oracle.layernorm(g["ln_x"], eps=1e-5), g["ln_out_noaffine"], **tol)
    np.testing.assert_allclose(oracle.multihead_rmsnorm(g["rms_x"], g["rms_gamma"]), g["rms_out"], **tol)
    np.testing.assert_allclose(oracle.rope_complex(g["rope_x"], g["rope_f"]), g["rope_out"], **tol)
    np.testing.assert_allclose(oracle.gelu_tanh(g["act_x"]), g["gelu_out"], **tol)
    np.testing.assert_allclose(oracle.silu(g["act_x"]), g["silu_out"], **tol)
    np.testing.assert_allclose(oracle.modulate(g["mod_h"], g["mod_scale"], g["mod_shift"]), g["mod_out"], **tol)
    b, d = oracle.gated_residual(g["gres_base"], g["gres_delta"], g["gres_gate"])
    np.testing.assert_allclose(b, g["gres_base_out"], **tol)
    np.testing.assert_allclose(d, g["gres_delta_out"], **tol)
    np.testing.assert_allclose(oracle.add(g["gres_base"], g["gres_delta"]), g["add_out"], **tol)
    np.testing.assert_allclose(oracle.cfg_combine(g["cfg_pos"], g["cfg_neg"], g["cfg_g"]), g["cfg_out"], **tol)
    np.testing.assert_allclose(oracle.euler_update(g["cfg_pos"], g["cfg_neg"], g["euler_dt"]), g["euler_out"], **tol)
    q, pk, pv = oracle.qkv_rope_rmsnorm_pack(g["post_qkv"], g["post_freqs"], g["post_qg"], g["post_kg"], Lp=32)
    np.testing.assert_allclose(q, g["post_q"], **tol)
    np.testing.assert_allclose(pk, g["post_pk"], **tol)
    np.testing.assert_array_equal(pv, g["post_pv"])


def test_oracle_error_codes(oracle):
    x = np.zeros((2, 4), np.float32)
    c = np.zeros((4, 16), np.int16)
    q = np.zeros((4, 16), np.int8)
    s = np.zeros(16, np.float32)
    with pytest.raises(RuntimeError):
        oracle.gemm_nf24(x, c, q, s, s, start=8, count=16)  # range overflow -> -3


def test_embeddings_oracle_bit_exact(oracle, golden):
    """The oracle's restatement of the reference's sin / cos method reproduces the reference
    kernels bit for bit (timestep and point-cloud position embeddings, RePo phasor, feature
    multiply), including angles of 1e3..1e4 rad where the range reduction is coarse."""
    g = golden("embeddings")
    out = oracle.timestep_embedding(g["ts_t"], g["ts_f"], output_dim=g["ts_out"].shape[1])
    np.testing.assert_array_equal(out, g["ts_out"])
    for dp in (0, 1):
        out = oracle.pcd_position_embedding(g["pcd_pos"], g["pcd_f"], g[f"pcd_out{dp}"].shape[1],
                                            double_pi=bool(dp))
        np.testing.assert_array_equal(out, g[f"pcd_out{dp}"])
    for name in ("a", "b"):
        out = oracle.repo_phasor(g[f"repo_{name}_delta"], [g[f"repo_{name}_ft{a}"] for a in range(3)],
                                 [g[f"repo_{name}_fr{a}"] for a in range(3)])
        np.testing.assert_array_equal(out, g[f"repo_{name}_out"])
    np.testing.assert_array_equal(oracle.mul(g["mul_lhs"], g["mul_rhs"]), g["mul_out"])
    np.testing.assert_array_equal(
        oracle.ab2_update(g["ab2_x"], g["ab2_v"], g["ab2_vp"], g["ab2_dt"], g["ab2_pdt"]), g["ab2_out"])


def _make_golden():
    import importlib.util
    from pathlib import Path

    path = Path(__file__).resolve().parent / "golden" / "make_golden.py"
    spec = importlib.util.spec_from_file_location("make_golden", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_fused_mlp_oracle(oracle, golden):
    """fc1 -> GELU -> fc2 composed from the oracle's GEMM and GELU equals the reference's
    fused MLP (plain and chunked) on the fixture; the codes this repository's packer makes
    from the regenerated weights are the reference packer's (digest)."""
    import torch
    from nf24_pack import quantize_nf24_i16_per_output_channel

    g = golden("mlp_nf24")
    mg = _make_golden()
    w1, w2, b1, b2 = mg.mlp_weights(int(g["seed"]))
    packed = []
    for w, digest in ((w1, g["w1_digest"]), (w2, g["w2_digest"])):
        codes, scales, _ = quantize_nf24_i16_per_output_channel(torch.from_numpy(w))
        c, q, s = codes[0].numpy(), codes[1].numpy(), scales[0].numpy()
        assert mg.code_digest(c, q) == str(digest)
        packed.append((c, q, s))
    (c1, q1, s1), (c2, q2, s2) = packed
    x = g["x"][:, :1024]
    y = oracle.gemm_nf24(oracle.gelu_tanh(oracle.gemm_nf24(x, c1, q1, s1, b1)), c2, q2, s2, b2)
    # same GEMM order; the GELU's tanh differs from the reference's polynomial by ~1e-7
    np.testing.assert_allclose(y, g["out"][:, :1024], rtol=2e-5, atol=2e-5)
    np.testing.assert_array_equal(g["out"], g["out_chunked"])
    assert (g["out"][:, 1024:] == 5.0).all()  # row padding untouched


def test_qkv_direct_oracle(oracle, golden):
    """The reference's fused QKV projection equals the oracle's GEMM followed by its
    RoPE / RMSNorm / pack restatement, with shared and per-batch frequencies."""
    g = golden("qkv_direct")
    B, H, D = 2, 2, 64
    qkv = oracle.gemm_nf24(g["x"], g["code01_t"], g["q2_t"], g["scale"], g["bias"])
    L = qkv.shape[0] // B
    qkv = qkv.reshape(B, L, 3, H, D)
    for fb in (1, B):
        q, pk, pv = oracle.qkv_rope_rmsnorm_pack(qkv, g[f"freqs{fb}"], g[f"qg{fb}"],
                                                 g[f"kg{fb}"], Lp=16)
        np.testing.assert_allclose(q, g[f"q{fb}"], rtol=2e-6, atol=2e-6)
        np.testing.assert_allclose(pk, g[f"pk{fb}"], rtol=2e-6, atol=2e-6)
        np.testing.assert_array_equal(pv, g[f"pv{fb}"])
