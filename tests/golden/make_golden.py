#!/usr/bin/env python3
"""Generate the golden vectors in this folder from the REFERENCE itself.

Run once in a container that has the reference checkout (the GPU box does not):

    make -C oracle ref REF=<reference checkout>
    python tests/golden/make_golden.py --reference <reference checkout>

Inputs are seeded; codes come from the reference's own NF24 packer
(scripts/native_linear_rnf8_avx512_patch.py:75-87, imported from the checkout)
and every output from the reference's own AVX-512 kernels compiled into
oracle/_ref.  The fixtures pin (a) the oracle restatement in oracle/oracle.c,
(b) this repository's packer and (c) the CUDA kernels, all without needing the
reference at test time.  Case shapes follow the reference's smoke tests
(scripts/smoke_native_rnf8_avx512.py:21-80 and
scripts/bench_native_sdpa_avx512_exact.py:146-161) with small head counts so the
fixtures stay a few hundred KB.
"""
from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF_LIBS = REPO / "oracle" / "_ref"

VP, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float


def ptr(a):
    return None if a is None else a.ctypes.data_as(VP)


def bind(lib, name, args):
    fn = getattr(lib, name)
    fn.argtypes = args
    fn.restype = I
    return fn


def check(status, name):
    if status != 0:
        raise RuntimeError(f"{name} -> {status}")


def gemm_cases(torch, pack, codebook, gemm_lib):
    full = bind(gemm_lib, "triposplat_gemm_rnf8_avx512", [VP] * 10 + [I] * 7)
    tail = bind(gemm_lib, "triposplat_gemm_rnf8_avx512_tail", [VP] * 10 + [I] * 7)
    rng = bind(gemm_lib, "triposplat_gemm_rnf8_avx512_range", [VP] * 10 + [I] * 9)
    cases = {
        # (M, K, N, start, count); seeds follow the reference smoke (19 + stages + n)
        "gemm_25x96x64": (25, 96, 64, 0, None),
        "gemm_40x96x64": (40, 96, 64, 0, None),
        "gemm_10x96x64": (10, 96, 64, 0, None),
        "gemm_3x96x5_tail": (3, 96, 5, 0, None),
        "gemm_7x100x7_tail": (7, 100, 7, 0, None),
        "gemm_33x160x96_range32_48": (33, 160, 96, 32, 48),
        "gemm_130x256x144": (130, 256, 144, 0, None),
    }
    for name, (m, k, n, start, count) in cases.items():
        torch.manual_seed(19 + 3 + n + m)
        x = torch.randn(m, k, dtype=torch.float32)
        w = torch.randn(n, k, dtype=torch.float32) * 0.03
        b = torch.randn(n, dtype=torch.float32) * 0.01
        codes, scales, _ = pack(w, codebook)
        c01 = codes[0].numpy()
        q2 = codes[1].numpy()
        sc = scales[0].numpy()
        xn, bn = x.numpy(), b.numpy()
        cb = codebook.numpy()
        if count is None:
            out = np.empty((m, n), np.float32)
            fn = tail if n % 16 else full
            check(fn(ptr(xn), ptr(c01), ptr(q2), ptr(q2), ptr(sc), ptr(sc), ptr(sc), ptr(cb),
                     ptr(bn), ptr(out), m, k, n, k, n, 2, 3), name)
        else:
            out = np.empty((m, count), np.float32)
            check(rng(ptr(xn), ptr(c01), ptr(q2), ptr(q2), ptr(sc), ptr(sc), ptr(sc), ptr(cb),
                      ptr(bn), ptr(out), m, k, n, start, count, k, count, 2, 3), name)
        np.savez_compressed(HERE / f"{name}.npz", x=xn, w=w.numpy(), bias=bn, code01_t=c01,
                            q2_t=q2, scale=sc, out=out, start=start,
                            count=-1 if count is None else count)


def sdpa_cases(torch, sdpa_lib, packed_lib):
    fn = bind(sdpa_lib, "triposplat_sdpa_f32_avx512_exact_q8t512", [VP] * 5 + [I] * 8)
    pk_fn = bind(packed_lib, "triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd",
                 [VP] * 5 + [I] * 9)
    cases = {
        # name: (B, H, Lq, Lk, bias spec)
        "sdpa_self256": (1, 2, 256, 256, None),
        "sdpa_masked256": (1, 2, 256, 256, ("onehot", 7, 2.0)),
        "sdpa_cross193x256": (1, 2, 193, 256, None),
        "sdpa_cross5x17_bias": (2, 2, 5, 17, ("randn",)),
        "sdpa_q3_k1": (1, 3, 3, 1, None),
        "sdpa_q70_k700_bias": (1, 2, 70, 700, ("randn",)),
    }
    gen = torch.Generator(device="cpu").manual_seed(0)
    for name, (B, H, lq, lk, bspec) in cases.items():
        q = torch.randn((B, H, lq, 64), generator=gen).numpy()
        k = torch.randn((B, H, lk, 64), generator=gen).numpy()
        v = torch.randn((B, H, lk, 64), generator=gen).numpy()
        bias = None
        if bspec is not None:
            if bspec[0] == "onehot":
                bias = np.zeros(lk, np.float32)
                bias[bspec[1]] = bspec[2]
            else:
                bias = torch.randn((lk,), generator=gen).numpy()
        out = np.empty((B, H, lq, 64), np.float32)
        check(fn(ptr(q), ptr(k), ptr(v), ptr(bias), ptr(out), B, H, lq, lk, 64,
                 int(bias is not None), 0 if bias is None else lk, 2), name)
        lkp = (lk + 15) // 16 * 16
        packk = np.zeros((B, H, 64, lkp), np.float32)
        packv = np.zeros((B, H, 64, lkp), np.float32)
        packk[..., :lk] = k.transpose(0, 1, 3, 2)
        packv[..., :lk] = v.transpose(0, 1, 3, 2)
        out_blhd = np.empty((B, lq, H, 64), np.float32)
        check(pk_fn(ptr(q), ptr(packk), ptr(packv), ptr(bias), ptr(out_blhd), B, H, lq, lk, 64,
                    lkp, int(bias is not None), 0 if bias is None else lk, 2), name + "_packed")
        extra = {} if bias is None else {"bias": bias}
        np.savez_compressed(HERE / f"{name}.npz", q=q, k=k, v=v, out=out, out_blhd=out_blhd,
                            **extra)


def elementwise_cases(torch):
    nr = __import__("ctypes").CDLL(str(REF_LIBS / "libref_norm_rope.so"))
    act = ctypes.CDLL(str(REF_LIBS / "libref_activations.so"))
    blk = ctypes.CDLL(str(REF_LIBS / "libref_block_elementwise.so"))
    smp = ctypes.CDLL(str(REF_LIBS / "libref_sampler.so"))
    qkv = ctypes.CDLL(str(REF_LIBS / "libref_qkv_postprocess_v2.so"))
    ln = bind(nr, "triposplat_layernorm_f32_avx512", [VP] * 4 + [I64, I, F, I, I])
    rms = bind(nr, "triposplat_multihead_rmsnorm_f32_avx512", [VP] * 3 + [I64, I, I, F, I])
    rope = bind(nr, "triposplat_rope_complex_f32_avx512", [VP] * 3 + [I64, I, I])
    gelu = bind(act, "triposplat_gelu_tanh_f32_avx512", [VP] * 2 + [I64, I])
    silu = bind(act, "triposplat_silu_f32_avx512", [VP] * 2 + [I64, I])
    mod = bind(blk, "triposplat_modulate_inplace_f32_avx512", [VP] * 3 + [I] * 4)
    gres = bind(blk, "triposplat_gated_residual_inplace_f32_avx512", [VP] * 3 + [I] * 4)
    add = bind(blk, "triposplat_add_inplace_f32_avx512", [VP] * 2 + [I64, I])
    cfg = bind(smp, "triposplat_cfg_combine_inplace_f32_avx512", [VP] * 3 + [I, I64, I])
    eul = bind(smp, "triposplat_euler_update_inplace_f32_avx512", [VP] * 3 + [I, I64, I])
    post = bind(qkv, "triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2", [VP] * 7 + [I] * 7)
    g = torch.Generator(device="cpu").manual_seed(1)

    def rn(*shape, s=1.0):
        return (torch.randn(shape, generator=g) * s).numpy().astype(np.float32)

    data = {}
    x = rn(5, 1000)
    w, b = 1.0 + rn(1000, s=0.02), rn(1000, s=0.1)
    out = np.empty_like(x)
    check(ln(ptr(x), ptr(w), ptr(b), ptr(out), 5, 1000, 1e-6, 1, 2), "ln")
    out2 = np.empty_like(x)
    check(ln(ptr(x), None, None, ptr(out2), 5, 1000, 1e-5, 0, 2), "ln_noaff")
    data.update(ln_x=x, ln_w=w, ln_b=b, ln_out=out, ln_out_noaffine=out2)

    x = rn(3, 7, 4, 64)
    gam = 1.0 + rn(4, 64, s=0.1)
    out = np.empty_like(x)
    check(rms(ptr(x), ptr(gam), ptr(out), 21, 4, 64, 1e-12, 2), "rms")
    data.update(rms_x=x, rms_gamma=gam, rms_out=out)

    x, f = rn(6, 64), rn(6, 64)
    out = np.empty_like(x)
    check(rope(ptr(x), ptr(f), ptr(out), 6, 64, 2), "rope")
    data.update(rope_x=x, rope_f=f, rope_out=out)

    x = np.concatenate([rn(997, s=3.0), np.array([0.0, -12.0, 12.0], np.float32)])
    out = np.empty_like(x)
    check(gelu(ptr(x), ptr(out), x.size, 2), "gelu")
    out_s = np.empty_like(x)
    check(silu(ptr(x), ptr(out_s), x.size, 2), "silu")
    data.update(act_x=x, gelu_out=out, silu_out=out_s)

    h, sc, sh = rn(2, 9, 48), rn(2, 48, s=0.2), rn(2, 48, s=0.2)
    hm = h.copy()
    check(mod(ptr(hm), ptr(sc), ptr(sh), 2, 9, 48, 2), "mod")
    base, delta, gate = rn(2, 9, 48), rn(2, 9, 48), rn(2, 48)
    bo, do = base.copy(), delta.copy()
    check(gres(ptr(bo), ptr(do), ptr(gate), 2, 9, 48, 2), "gres")
    ao = base.copy()
    check(add(ptr(ao), ptr(delta), ao.size, 2), "add")
    data.update(mod_h=h, mod_scale=sc, mod_shift=sh, mod_out=hm, gres_base=base,
                gres_delta=delta, gres_gate=gate, gres_base_out=bo, gres_delta_out=do,
                add_out=ao)

    pos, neg = rn(2, 333), rn(2, 333)
    guid = np.array([3.0, 1.5], np.float32)
    po = pos.copy()
    check(cfg(ptr(po), ptr(neg), ptr(guid), 2, 333, 2), "cfg")
    dt = np.array([0.05, 0.1], np.float32)
    so = pos.copy()
    check(eul(ptr(so), ptr(neg), ptr(dt), 2, 333, 2), "euler")
    data.update(cfg_pos=pos, cfg_neg=neg, cfg_g=guid, cfg_out=po, euler_dt=dt, euler_out=so)

    B, L, H, D, Lp = 2, 19, 2, 64, 32
    qkv_in = rn(B, L, 3, H, D)
    ang = rn(1, L, H, D // 2)
    freqs = np.stack([np.cos(ang), np.sin(ang)], -1).reshape(1, L, H, D).astype(np.float32)
    qg, kg = 1.0 + rn(H, D, s=0.1), 1.0 + rn(H, D, s=0.1)
    qo = np.empty((B, H, L, D), np.float32)
    pk = np.full((B, H, D, Lp), 7.0, np.float32)
    pv = np.full((B, H, D, Lp), 7.0, np.float32)
    check(post(ptr(qkv_in), ptr(freqs), ptr(qg), ptr(kg), ptr(qo), ptr(pk), ptr(pv),
               B, L, H, D, Lp, 1, 2), "qkv_post")
    data.update(post_qkv=qkv_in, post_freqs=freqs, post_qg=qg, post_kg=kg, post_q=qo,
                post_pk=pk, post_pv=pv)
    np.savez_compressed(HERE / "elementwise.npz", **data)


def embedding_cases(torch):
    """Timestep / point-cloud position embeddings (scripts/native_embeddings_avx512.c:58-125),
    the RePo phasor and feature multiply (scripts/native_repo_avx512.c:69-129).  Angles span
    small, large (|x| ~ 1e3..1e4 rad, where the two-constant range reduction is coarse) and
    negative values, so a restatement must follow the reference's sin/cos method exactly."""
    emb = ctypes.CDLL(str(REF_LIBS / "libref_embeddings.so"))
    rep = ctypes.CDLL(str(REF_LIBS / "libref_repo.so"))
    ts = bind(emb, "triposplat_timestep_embedding_f32_avx512", [VP] * 3 + [I] * 4)
    pcd = bind(emb, "triposplat_pcd_position_embedding_f32_avx512", [VP] * 3 + [I64] + [I] * 5)
    mul = bind(rep, "triposplat_mul_inplace_f32_avx512", [VP] * 2 + [I64, I])
    pha = bind(rep, "triposplat_repo_phasor_f32_avx512",
               [VP, VP, VP, I, VP, VP, I, VP, VP, I, VP, I64, I])
    g = torch.Generator(device="cpu").manual_seed(2)

    def rn(*shape, s=1.0):
        return (torch.randn(shape, generator=g) * s).numpy().astype(np.float32)

    data = {}
    # timestep embedding: 1000*t over the sampler's range, frequencies exp(-ln(1e4) i / half)
    half = 128
    t = np.array([999.0, 731.25, 0.5, 0.0, -3.0], np.float32)
    f = torch.exp(-float(np.log(10000)) * torch.arange(0, half, dtype=torch.float32) / half).numpy()
    out = np.full((5, 2 * half + 4), 7.0, np.float32)
    check(ts(ptr(t), ptr(f), ptr(out), 5, half, 2 * half + 4, 2), "timestep")
    data.update(ts_t=t, ts_f=f, ts_out=out)
    # point-cloud positions: 3 axes, 20 frequencies (not a multiple of 16), padded channels
    pos = rn(37, 3, s=2.0)
    pf = (2.0 ** np.linspace(0, 9, 20)).astype(np.float32)
    for dp in (0, 1):
        o = np.full((37, 128), 7.0, np.float32)
        check(pcd(ptr(pos), ptr(pf), ptr(o), 37, 3, 20, 128, dp, 2), "pcd")
        data[f"pcd_out{dp}"] = o
    data.update(pcd_pos=pos, pcd_f=pf)
    # RePo: delta [vectors, 3]; per-axis frequencies split as tanh(f) + (f - tanh(f))
    for name, dims in (("a", (10, 11, 11)), ("b", (20, 3, 17))):
        fr = [torch.randn(d, generator=g) * 3.0 for d in dims]
        fts = [x.tanh().contiguous() for x in fr]
        frs = [(x - y).contiguous() for x, y in zip(fr, fts)]
        fts = [x.numpy().astype(np.float32) for x in fts]
        frs = [x.numpy().astype(np.float32) for x in frs]
        delta = rn(53, 3, s=40.0)
        o = np.full((53, 2 * sum(dims)), 7.0, np.float32)
        check(pha(ptr(delta), ptr(fts[0]), ptr(frs[0]), dims[0], ptr(fts[1]), ptr(frs[1]), dims[1],
                  ptr(fts[2]), ptr(frs[2]), dims[2], ptr(o), 53, 2), "phasor")
        data.update({f"repo_{name}_delta": delta, f"repo_{name}_out": o,
                     f"repo_{name}_dims": np.array(dims, np.int32)})
        for a in range(3):
            data[f"repo_{name}_ft{a}"], data[f"repo_{name}_fr{a}"] = fts[a], frs[a]
    smp = ctypes.CDLL(str(REF_LIBS / "libref_sampler.so"))
    ab2 = bind(smp, "triposplat_ab2_update_inplace_f32_avx512", [VP] * 5 + [I, I64, I])
    x, v, vp = rn(2, 333), rn(2, 333), rn(2, 333)
    dt, pdt = np.array([0.05, 0.031], np.float32), np.array([0.07, 0.0], np.float32)
    xo = x.copy()
    check(ab2(ptr(xo), ptr(v), ptr(vp), ptr(dt), ptr(pdt), 2, 333, 2), "ab2")
    data.update(ab2_x=x, ab2_v=v, ab2_vp=vp, ab2_dt=dt, ab2_pdt=pdt, ab2_out=xo)
    lhs, rhs = rn(1001), rn(1001)
    prod = lhs.copy()
    check(mul(ptr(prod), ptr(rhs), 1001, 2), "mul")
    data.update(mul_lhs=lhs, mul_rhs=rhs, mul_out=prod)
    np.savez_compressed(HERE / "embeddings.npz", **data)


def shard_cases(torch):
    """A tiny NF24 shard directory written by the reference's own packer
    (scripts/native_linear_nf24_prepacked.py:202-335, format triposplat_nf24_i16_v1) from a
    seeded three-Linear safetensors checkpoint (one without bias) plus two non-Linear
    tensors; the loader here must read it, and its codes must equal this repo's packer."""
    import shutil

    from safetensors.torch import save_file
    from native_linear_nf24_prepacked import pack_nf24_i16_checkpoint

    g = torch.Generator(device="cpu").manual_seed(4)
    src = {
        "blocks.0.attn.qkv.weight": torch.randn(96, 64, generator=g) * 0.02,
        "blocks.0.attn.qkv.bias": torch.randn(96, generator=g) * 0.01,
        "blocks.0.mlp.fc1.weight": torch.randn(48, 96, generator=g) * 0.02,
        "blocks.0.mlp.fc1.bias": torch.randn(48, generator=g) * 0.01,
        "head.weight": torch.randn(16, 48, generator=g) * 0.02,
        "blocks.0.norm.gamma": 1.0 + torch.randn(64, generator=g) * 0.02,
        "pos_table": torch.randn(8, 64, generator=g),
    }
    src_path = HERE / "shards_src.safetensors"
    save_file(src, src_path.as_posix())
    out = HERE / "shards_ref"
    if out.exists():
        shutil.rmtree(out)
    pack_nf24_i16_checkpoint(src_path, out, expected_linear_count=3)


def mlp_weights(seed):
    """The fused-MLP fixture's weights, regenerated identically by the tests: numpy's PCG64
    stream (stable across numpy versions) for W1 [4096, 1024], W2 [1024, 4096] and biases."""
    g = np.random.default_rng(seed)
    w1 = (g.standard_normal((4096, 1024), dtype=np.float32) * 0.02).astype(np.float32)
    w2 = (g.standard_normal((1024, 4096), dtype=np.float32) * 0.02).astype(np.float32)
    b1 = (g.standard_normal(4096, dtype=np.float32) * 0.01).astype(np.float32)
    b2 = (g.standard_normal(1024, dtype=np.float32) * 0.01).astype(np.float32)
    return w1, w2, b1, b2


def code_digest(c01, q2):
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(c01).tobytes() +
                          np.ascontiguousarray(q2).tobytes()).hexdigest()


def fused_cases(torch, pack, codebook):
    """The reference's fused NF24 entry points: the MLP (plain and chunked,
    scripts/native_nf24_mlp_avx512.c:143, native_nf24_mlp_chunked_avx512.c:3) and the QKV
    projection with RoPE / RMSNorm / pack (scripts/gemm_nf24_qkv_direct_avx512.c:87)."""
    mlp = ctypes.CDLL(str(REF_LIBS / "libref_mlp_nf24.so"))
    qkvd = ctypes.CDLL(str(REF_LIBS / "libref_gemm_nf24_qkv_direct.so"))
    plain = bind(mlp, "triposplat_mlp_nf24_gelu_f32_avx512", [VP] * 10 + [I] * 7)
    chunked = bind(mlp, "triposplat_mlp_nf24_gelu_chunked_f32_avx512", [VP] * 11 + [I] * 9)
    direct = bind(qkvd, "triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512",
                  [VP] * 15 + [I] * 10)
    cb = codebook.numpy()

    # MLP: 11 rows (one 8-row tile + 3 tail rows), padded row strides
    M, sx, so = 11, 1040, 1056
    w1, w2, b1, b2 = mlp_weights(41)
    packed = []
    for w in (w1, w2):
        codes, scales, _ = pack(torch.from_numpy(w), codebook)
        packed.append((codes[0].numpy(), codes[1].numpy(), scales[0].numpy()))
    (c1, q1, s1), (c2, q2, s2) = packed
    x = (np.random.default_rng(42).standard_normal((M, sx), dtype=np.float32)).astype(np.float32)
    out = np.full((M, so), 5.0, np.float32)
    check(plain(ptr(x), ptr(c1), ptr(q1), ptr(s1), ptr(b1), ptr(c2), ptr(q2), ptr(s2), ptr(b2),
                ptr(out), M, 1024, 4096, 1024, sx, so, 2), "mlp")
    out_c = np.full((M, so), 5.0, np.float32)
    hidden = np.zeros((5, 4096), np.float32)
    check(chunked(ptr(x), ptr(c1), ptr(q1), ptr(s1), ptr(b1), ptr(c2), ptr(q2), ptr(s2), ptr(b2),
                  ptr(hidden), ptr(out_c), M, 1024, 4096, 1024, sx, so, 5, 4, 2), "mlp_chunked")
    np.savez_compressed(HERE / "mlp_nf24.npz", x=x, out=out, out_chunked=out_c, seed=41,
                        w1_digest=code_digest(c1, q1), w2_digest=code_digest(c2, q2),
                        stride_x=sx, stride_out=so, chunk_rows=4, hidden_rows=5)

    # QKV projection: B 2, L 11 (padded to 16), K 96, H 2 (N = 384), per-batch frequencies
    B, L, K, H, D, Lp = 2, 11, 96, 2, 64, 16
    N = 3 * H * D
    torch.manual_seed(77)
    xq = torch.randn(B * L, K, dtype=torch.float32).numpy()
    w = torch.randn(N, K, dtype=torch.float32) * 0.05
    bq = (torch.randn(N, dtype=torch.float32) * 0.01).numpy()
    codes, scales, _ = pack(w, codebook)
    cq, qq, sq = codes[0].numpy(), codes[1].numpy(), scales[0].numpy()
    data = dict(x=xq, code01_t=cq, q2_t=qq, scale=sq, bias=bq)
    rng = np.random.default_rng(78)
    for fb in (1, B):
        ang = rng.uniform(0.0, 6.0, (fb, L, H, D // 2)).astype(np.float32)
        freqs = np.stack([np.cos(ang), np.sin(ang)], -1).reshape(fb, L, H, D).astype(np.float32)
        qg = (1.0 + 0.1 * rng.standard_normal((H, D))).astype(np.float32)
        kg = (1.0 + 0.1 * rng.standard_normal((H, D))).astype(np.float32)
        qo = np.empty((B, H, L, D), np.float32)
        pk = np.full((B, H, D, Lp), 7.0, np.float32)
        pv = np.full((B, H, D, Lp), 7.0, np.float32)
        check(direct(ptr(xq), ptr(cq), ptr(qq), ptr(qq), ptr(sq), ptr(sq), ptr(sq), ptr(cb),
                     ptr(bq), ptr(freqs), ptr(qg), ptr(kg), ptr(qo), ptr(pk), ptr(pv),
                     B, L, K, N, H, D, Lp, fb, 2, 3), f"qkv_direct fb={fb}")
        data.update({f"freqs{fb}": freqs, f"qg{fb}": qg, f"kg{fb}": kg, f"q{fb}": qo,
                     f"pk{fb}": pk, f"pv{fb}": pv})
    np.savez_compressed(HERE / "qkv_direct.npz", **data)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--cases", default="gemm,sdpa,elementwise,embeddings,shards,fused",
                    help="comma-separated subset of the fixture groups to (re)write")
    args = ap.parse_args()
    cases = set(args.cases.split(","))
    sys.path.insert(0, str(args.reference / "scripts"))
    import torch
    from native_linear_nf8_avx512_patch import make_nf8_codebook  # reference packer
    from native_linear_rnf8_avx512_patch import quantize_nf24_i16_per_output_channel

    def pack(w, cb):
        codes, scales, err = quantize_nf24_i16_per_output_channel(w, cb)
        return [codes[0], codes[1]], scales, err

    codebook = make_nf8_codebook(torch)
    if "gemm" in cases:
        np.save(HERE / "nf8_codebook.npy", codebook.numpy())
        gemm_cases(torch, pack, codebook, ctypes.CDLL(str(REF_LIBS / "libref_gemm_nf24_i16.so")))
    if "sdpa" in cases:
        sdpa_cases(torch, ctypes.CDLL(str(REF_LIBS / "libref_sdpa_q8t512.so")),
                   ctypes.CDLL(str(REF_LIBS / "libref_sdpa_q8t512_packed.so")))
    if "elementwise" in cases:
        elementwise_cases(torch)
    if "embeddings" in cases:
        embedding_cases(torch)
    if "shards" in cases:
        shard_cases(torch)
    if "fused" in cases:
        fused_cases(torch, pack, codebook)
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
