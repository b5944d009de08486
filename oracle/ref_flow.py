"""The synthetic flow model and its CFG / Euler sampler composed from the REFERENCE's own
AVX-512 kernels (oracle/_ref, compiled from the reference's C sources by ``make ref``).

TEST / BASELINE INFRASTRUCTURE ONLY: used by tests/ as the full-size parity checker
(configs 3, 4 and 5), by tests/golden/make_s20_fixture.py to write the s20 fixture, and
by bench.py's CPU-baseline legs as the timed reference path.  Never part of the product.

Every op is one call of a reference kernel, in the order the reference's patched modules
chain them (scripts/native_block_elementwise_avx512_patch.py:45-54 for the block,
scripts/native_qkv_packed_attention_patch_v3.py:119-150 for the packed attention route,
scripts/triposplat_quantized_sampler.py:387-494 for the sampler):

  embed:  timestep embedding (native_embeddings_avx512.c:97) -> t_fc1 -> SiLU
          (native_silu_avx512_extra.c:28) -> t_fc2 -> SiLU -> adaLN / final_adaLN;
          cond -> cond_embedder -> SiLU -> cond_refiner; x = [x_embedder(lat) | camera_embedder(cam)]
  block:  LN (native_norm_rope_avx512.c:13) -> modulate (native_block_elementwise_avx512.c:9)
          -> NF24 qkv (gemm_nf24_i16_avx512.c:199) -> RoPE+RMSNorm+pack
          (native_qkv_postprocess_v2_avx512.c:45) -> packed exact SDPA
          (native_sdpa_avx512_exact_q8t512_packed.c:3) -> out -> gated residual (:24);
          LN -> cross_q -> multi-head RMSNorm (native_norm_rope_avx512.c:51); cross_kv(c) ->
          RMSNorm of its K half; packed exact SDPA over the condition tokens -> cross_out -> add (:37);
          LN -> modulate -> fc1 -> GELU(tanh) (native_gelu_avx512.c:44) -> fc2 -> gated residual
  final:  LN -> modulate -> final_linear / camera_head (N % 16 != 0: the tail kernel,
          gemm_nf24_i16_avx512_tail.c:8)
  step:   CFG combine + Euler update (native_sampler_avx512.c:19,56)

The layout conversions between kernels (condition K/V into the packed [B,H,64,Lkp] layout,
cross queries into [B,H,L,64]) are numpy copies, as the reference's Python glue does them.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
VP, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float


def _p(a):
    return None if a is None else a.ctypes.data_as(VP)


def _bind(lib, name, args):
    fn = getattr(lib, name)
    fn.argtypes = args
    fn.restype = I
    return fn


def _check(st, what):
    if st != 0:
        raise RuntimeError(f"reference kernel {what} returned {st}")


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class RefKernels:
    """ctypes bindings of the reference kernels the flow model needs."""

    kind = "reference"

    def __init__(self, threads: int | None = None):
        self.th = threads or host_threads()
        L = lambda n: ctypes.CDLL(str(REF / n))  # noqa: E731
        g = L("libref_gemm_nf24_i16.so")
        self.gemm = _bind(g, "triposplat_gemm_rnf8_avx512", [VP] * 10 + [I] * 7)
        self.gemm_tail = _bind(g, "triposplat_gemm_rnf8_avx512_tail", [VP] * 10 + [I] * 7)
        nr = L("libref_norm_rope.so")
        self.ln = _bind(nr, "triposplat_layernorm_f32_avx512", [VP] * 4 + [I64, I, F, I, I])
        self.rms = _bind(nr, "triposplat_multihead_rmsnorm_f32_avx512", [VP] * 3 + [I64, I, I, F, I])
        act = L("libref_activations.so")
        self.gelu = _bind(act, "triposplat_gelu_tanh_f32_avx512", [VP] * 2 + [I64, I])
        self.silu = _bind(act, "triposplat_silu_f32_avx512", [VP] * 2 + [I64, I])
        blk = L("libref_block_elementwise.so")
        self.mod = _bind(blk, "triposplat_modulate_inplace_f32_avx512", [VP] * 3 + [I] * 4)
        self.gres = _bind(blk, "triposplat_gated_residual_inplace_f32_avx512", [VP] * 3 + [I] * 4)
        self.add = _bind(blk, "triposplat_add_inplace_f32_avx512", [VP] * 2 + [I64, I])
        post = L("libref_qkv_postprocess_v2.so")
        self.post = _bind(post, "triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2", [VP] * 7 + [I] * 7)
        sd = L("libref_sdpa_q8t512_packed.so")
        self.sdpa_packed = _bind(sd, "triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd",
                                 [VP] * 5 + [I] * 9)
        smp = L("libref_sampler.so")
        self.cfg = _bind(smp, "triposplat_cfg_combine_inplace_f32_avx512", [VP] * 3 + [I, I64, I])
        self.euler = _bind(smp, "triposplat_euler_update_inplace_f32_avx512", [VP] * 3 + [I, I64, I])
        emb = L("libref_embeddings.so")
        self.temb = _bind(emb, "triposplat_timestep_embedding_f32_avx512", [VP] * 3 + [I] * 4)
        self.codebook = np.zeros(256, np.float32)  # bound, ignored by the NF24 kernels

    @staticmethod
    def available() -> bool:
        need = ("libref_gemm_nf24_i16.so", "libref_norm_rope.so", "libref_activations.so",
                "libref_block_elementwise.so", "libref_qkv_postprocess_v2.so",
                "libref_sdpa_q8t512_packed.so", "libref_sampler.so", "libref_embeddings.so")
        if not all((REF / n).is_file() for n in need):
            return False
        try:
            flags = Path("/proc/cpuinfo").read_text()
        except OSError:
            return False
        return all(f in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl"))

    def linear(self, w, x, out):
        """out[rows, N] = x[rows, K] . W^T + b with the reference NF24 kernel (tail kernel
        when N % 16 != 0, as the reference patch selects it)."""
        c01, q2, sc, b = w["code01"], w["q2"], w["scale"], w["bias"]
        K, N = c01.shape
        rows = x.size // K
        assert x.flags.c_contiguous and out.flags.c_contiguous and out.size == rows * N
        fn = self.gemm if N % 16 == 0 else self.gemm_tail
        _check(fn(_p(x), _p(c01), _p(q2), _p(q2), _p(sc), _p(sc), _p(sc), _p(self.codebook),
                  _p(b), _p(out), rows, K, N, K, N, self.th, 3), "gemm_nf24")


class RefFlowModel:
    """Forward of the synthetic flow model (batch = CFG pair) on the reference's kernels.

    ``W[name] = {code01 [K,N] int16, q2 [K,N] int8, scale [N], bias [N]}`` and
    ``P[name]`` (adaLN tables [6,h], gammas [H,64]) as numpy arrays — the packed weights
    the GPU model holds (``flow_ref.weights_to_numpy``)."""

    def __init__(self, spec, W, P, freqs, tfreqs, batch: int = 2, threads: int | None = None,
                 kernels: RefKernels | None = None):
        if kernels is None and not RefKernels.available():
            raise RuntimeError("reference kernels unavailable (oracle/_ref missing or no AVX-512)")
        self.k = kernels or RefKernels(threads)
        self.s, self.W, self.P = spec, W, P
        self.freqs = np.ascontiguousarray(freqs, np.float32)
        self.tfreqs = np.ascontiguousarray(tfreqs, np.float32)
        s = spec
        B, L, h, H, Mc = batch, s.seq, s.hidden, s.heads, s.cond_tokens
        self.B = B
        self.Lp = (L + 15) // 16 * 16
        self.Mcp = (Mc + 15) // 16 * 16
        f32 = np.float32
        e = lambda *shape: np.empty(shape, f32)  # noqa: E731
        self.x, self.a, self.y, self.o = e(B, L, h), e(B, L, h), e(B, L, h), e(B, L, h)
        self.qkv = e(B, L, 3 * h)
        self.q = e(B, H, L, 64)
        self.pk, self.pv = e(B, H, 64, self.Lp), e(B, H, 64, self.Lp)
        self.ckv = e(B, Mc, 2 * h)
        self.ck = e(B, Mc, h)
        self.cpk = np.zeros((B, H, 64, self.Mcp), f32)
        self.cpv = np.zeros((B, H, 64, self.Mcp), f32)
        self.hid = e(B, L, s.mlp)
        self.c = e(B, Mc, h)
        self.mod = e(6, B, h)
        self.fmod = e(2, B, h)

    def lin(self, name, x, out):
        self.k.linear(self.W[name], np.ascontiguousarray(x), out)
        return out

    def _silu(self, x):
        out = np.empty_like(x)
        _check(self.k.silu(_p(x), _p(out), x.size, self.k.th), "silu")
        return out

    def _ln(self, x, out):
        s = self.s
        _check(self.k.ln(_p(x), None, None, _p(out), x.size // s.hidden, s.hidden, s.eps, 0,
                         self.k.th), "layernorm")

    def _modulate(self, a, scale, shift):
        B, L, C = a.shape
        _check(self.k.mod(_p(a), _p(np.ascontiguousarray(scale)), _p(np.ascontiguousarray(shift)),
                          B, L, C, self.k.th), "modulate")

    def embed(self, x_lat, cam, t1000, cond):
        """Timestep / adaLN / condition / token embeddings; fills self.x, mod, fmod, c."""
        s, k = self.s, self.k
        B, h, Nl, Mc = self.B, s.hidden, s.latent_tokens, s.cond_tokens
        t = np.ascontiguousarray(t1000, np.float32)
        tfe = np.empty((B, s.t_freq), np.float32)
        _check(k.temb(_p(t), _p(self.tfreqs), _p(tfe), B, s.t_freq // 2, s.t_freq, k.th),
               "timestep_embedding")
        t1 = self._silu(self.lin("t_fc1", tfe, np.empty((B, h), np.float32)))
        stemb = self._silu(self.lin("t_fc2", t1, np.empty((B, h), np.float32)))
        ada = self.lin("adaLN", stemb, np.empty((B, 6 * h), np.float32))
        self.mod[...] = ada.reshape(B, 6, h).transpose(1, 0, 2)
        fada = self.lin("final_adaLN", stemb, np.empty((B, 2 * h), np.float32))
        self.fmod[...] = fada.reshape(B, 2, h).transpose(1, 0, 2)
        c0 = self._silu(self.lin("cond_embedder", np.ascontiguousarray(cond, np.float32),
                                 np.empty((B, Mc, h), np.float32)))
        self.lin("cond_refiner", c0, self.c)
        x_lat = np.ascontiguousarray(x_lat, np.float32)
        cam = np.ascontiguousarray(cam, np.float32)
        for b in range(B):
            self.lin("x_embedder", x_lat[b], self.x[b, :Nl])
            self.lin("camera_embedder", cam[b], self.x[b, Nl:])

    def block(self, i):
        s, k, P, th = self.s, self.k, self.P, self.k.th
        B, L, h, H, Mc = self.B, s.seq, s.hidden, s.heads, s.cond_tokens
        p = f"blocks.{i}."
        m = self.mod + P[p + "table"][:, None, :]  # fp32 add, as the GPU's add kernel
        x, a, y, o = self.x, self.a, self.y, self.o
        rows = B * L
        # self-attention
        self._ln(x, a)
        self._modulate(a, m[1], m[0])
        self.lin(p + "qkv", a, self.qkv)
        _check(k.post(_p(self.qkv), _p(self.freqs), _p(np.ascontiguousarray(P[p + "q_gamma"])),
                      _p(np.ascontiguousarray(P[p + "k_gamma"])), _p(self.q), _p(self.pk), _p(self.pv),
                      B, L, H, 64, self.Lp, self.freqs.shape[0], th), "qkv_postprocess_v2")
        _check(k.sdpa_packed(_p(self.q), _p(self.pk), _p(self.pv), None, _p(o), B, H, L, L, 64,
                             self.Lp, 0, 0, th), "self_sdpa")
        self.lin(p + "out", o, y)
        _check(k.gres(_p(x), _p(y), _p(np.ascontiguousarray(m[2])), B, L, h, th), "gated_residual")
        # cross-attention to the condition tokens (queries and keys RMS-normalised per head)
        self._ln(x, a)
        self.lin(p + "cross_q", a, y)
        _check(k.rms(_p(y), _p(np.ascontiguousarray(P[p + "cq_gamma"])), _p(y), rows, H, 64,
                     1e-12, th), "cross_q_rmsnorm")
        self.lin(p + "cross_kv", self.c, self.ckv)
        ckv = self.ckv.reshape(B, Mc, 2, H, 64)
        self.ck[...] = ckv[:, :, 0].reshape(B, Mc, h)
        _check(k.rms(_p(self.ck), _p(np.ascontiguousarray(P[p + "ck_gamma"])), _p(self.ck), B * Mc,
                     H, 64, 1e-12, th), "cross_k_rmsnorm")
        self.cpk[..., :Mc] = self.ck.reshape(B, Mc, H, 64).transpose(0, 2, 3, 1)
        self.cpv[..., :Mc] = ckv[:, :, 1].transpose(0, 2, 3, 1)
        self.q[...] = y.reshape(B, L, H, 64).transpose(0, 2, 1, 3)
        _check(k.sdpa_packed(_p(self.q), _p(self.cpk), _p(self.cpv), None, _p(o), B, H, L, Mc, 64,
                             self.Mcp, 0, 0, th), "cross_sdpa")
        self.lin(p + "cross_out", o, y)
        _check(k.add(_p(x), _p(y), x.size, th), "add")
        # MLP
        self._ln(x, a)
        self._modulate(a, m[4], m[3])
        self.lin(p + "fc1", a, self.hid)
        _check(k.gelu(_p(self.hid), _p(self.hid), self.hid.size, th), "gelu_tanh")
        self.lin(p + "fc2", self.hid, y)
        _check(k.gres(_p(x), _p(y), _p(np.ascontiguousarray(m[5])), B, L, h, th), "gated_residual")

    def final_layer(self):
        s = self.s
        B, Nl = self.B, s.latent_tokens
        self._ln(self.x, self.a)
        self._modulate(self.a, self.fmod[1], self.fmod[0])
        v_lat = np.empty((B, Nl, s.latent_dim), np.float32)
        v_cam = np.empty((B, 1, s.camera_dim), np.float32)
        for b in range(B):
            self.lin("final_linear", self.a[b, :Nl], v_lat[b])
            self.lin("camera_head", self.a[b, Nl:], v_cam[b])
        return v_lat, v_cam

    def forward(self, x_lat, cam, t1000, cond):
        self.embed(x_lat, cam, t1000, cond)
        for i in range(self.s.blocks):
            self.block(i)
        return self.final_layer()

    def sample(self, noise_lat, noise_cam, cond, neg_cond, t1000, dt, guidance, on_step=None):
        """``len(dt)``-step CFG / Euler sampling of one image ([1, Nl, C] latent, [1, 1, Cc]
        camera); the model runs on the [cond, uncond] pair at ``t1000[i]``.  ``on_step(i,
        v_lat, v_cam)`` sees each step's velocity pair."""
        k = self.k
        x_lat = np.ascontiguousarray(noise_lat, np.float32).copy()
        x_cam = np.ascontiguousarray(noise_cam, np.float32).copy()
        cond_pair = np.ascontiguousarray(np.concatenate([cond, neg_cond], axis=0), np.float32)
        g = np.array([guidance], np.float32)
        for i in range(len(dt)):
            vl, vc = self.forward(np.concatenate([x_lat, x_lat]), np.concatenate([x_cam, x_cam]),
                                  np.array([t1000[i], t1000[i]], np.float32), cond_pair)
            if on_step is not None:
                on_step(i, vl, vc)
            d = np.array([dt[i]], np.float32)
            for x, v in ((x_lat, vl), (x_cam, vc)):
                pos, neg = np.ascontiguousarray(v[:1]), np.ascontiguousarray(v[1:])
                _check(k.cfg(_p(pos), _p(neg), _p(g), 1, pos.size, k.th), "cfg_combine")
                _check(k.euler(_p(x), _p(pos), _p(d), 1, x.size, k.th), "euler_update")
        return x_lat, x_cam
