"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

``liboracle.so`` is the plain-C restatement in oracle.c; ``_ref/`` holds the
reference's own AVX-512 kernels compiled from its sources by ``make ref``.
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import
this module, always as the checker or the timed CPU baseline, never as part of
the product path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"

_VP = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    def __init__(self, path: Path = LIB_PATH):
        if not path.is_file():
            raise FileNotFoundError(f"{path} (run: make -C oracle)")
        lib = ctypes.CDLL(str(path))
        sig = {
            "oracle_gemm_nf24": ([_VP] * 6 + [_I] * 8),
            "oracle_sdpa": ([_VP] * 4 + [_I64, _VP] + [_I] * 6),
            "oracle_layernorm": ([_VP] * 4 + [_I64, _I, _F, _I]),
            "oracle_multihead_rmsnorm": ([_VP] * 3 + [_I64, _I, _I, _F]),
            "oracle_rope_complex": ([_VP] * 3 + [_I64, _I]),
            "oracle_gelu_tanh": ([_VP] * 2 + [_I64]),
            "oracle_silu": ([_VP] * 2 + [_I64]),
            "oracle_modulate_inplace": ([_VP] * 3 + [_I] * 3),
            "oracle_gated_residual_inplace": ([_VP] * 3 + [_I] * 3),
            "oracle_add_inplace": ([_VP] * 2 + [_I64]),
            "oracle_cfg_combine_inplace": ([_VP] * 3 + [_I, _I64]),
            "oracle_euler_update_inplace": ([_VP] * 3 + [_I, _I64]),
            "oracle_qkv_rope_rmsnorm_pack": ([_VP] * 7 + [_I] * 5),
            "oracle_timestep_embedding": ([_VP] * 3 + [_I] * 3),
            "oracle_pcd_position_embedding": ([_VP] * 3 + [_I64] + [_I] * 4),
            "oracle_mul_inplace": ([_VP] * 2 + [_I64]),
            "oracle_ab2_update_inplace": ([_VP] * 5 + [_I, _I64]),
            "oracle_repo_phasor": ([_VP, _VP, _VP, _I, _VP, _VP, _I, _VP, _VP, _I, _VP, _I64]),
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def _check(status, name):
        if status != 0:
            raise RuntimeError(f"{name} returned {status}")

    def gemm_nf24(self, x, code01_t, q2_t, scale, bias, start=0, count=None, threads=0):
        x = _f32(x)
        M, K = x.shape
        N = code01_t.shape[1]
        count = N - start if count is None else count
        out = np.empty((M, count), np.float32)
        c01 = np.ascontiguousarray(code01_t, dtype=np.int16)
        c2 = np.ascontiguousarray(q2_t, dtype=np.int8)
        self._check(self.lib.oracle_gemm_nf24(
            _p(x), _p(c01), _p(c2), _p(_f32(scale)), _p(_f32(bias)), _p(out),
            M, K, N, start, count, K, count, threads), "oracle_gemm_nf24")
        return out

    def sdpa(self, q, k, v, bias=None, out_blhd=False, threads=0):
        """q [B,H,Lq,64], k/v [B,H,Lk,64]; bias [Lk] (shared) or [B,H,Lk]."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, Lq, _ = q.shape
        Lk = k.shape[2]
        stride = 0
        if bias is not None:
            bias = _f32(bias)
            stride = 0 if bias.ndim == 1 else Lk
        out = np.empty((B, Lq, H, 64) if out_blhd else (B, H, Lq, 64), np.float32)
        self._check(self.lib.oracle_sdpa(
            _p(q), _p(k), _p(v), _p(bias), stride, _p(out),
            B, H, Lq, Lk, int(out_blhd), threads), "oracle_sdpa")
        return out

    def layernorm(self, x, w=None, b=None, eps=1e-6):
        x = _f32(x)
        out = np.empty_like(x)
        cols = x.shape[-1]
        aff = w is not None
        self._check(self.lib.oracle_layernorm(
            _p(x), _p(_f32(w)) if aff else None, _p(_f32(b)) if aff else None, _p(out),
            x.size // cols, cols, eps, int(aff)), "oracle_layernorm")
        return out

    def multihead_rmsnorm(self, x, gamma, eps=1e-12):
        x = _f32(x)
        heads, dim = gamma.shape
        out = np.empty_like(x)
        self._check(self.lib.oracle_multihead_rmsnorm(
            _p(x), _p(_f32(gamma)), _p(out), x.size // (heads * dim), heads, dim, eps),
            "oracle_multihead_rmsnorm")
        return out

    def rope_complex(self, x, freqs):
        x = _f32(x)
        out = np.empty_like(x)
        dim = x.shape[-1]
        self._check(self.lib.oracle_rope_complex(
            _p(x), _p(_f32(freqs)), _p(out), x.size // dim, dim), "oracle_rope_complex")
        return out

    def gelu_tanh(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        self._check(self.lib.oracle_gelu_tanh(_p(x), _p(out), x.size), "oracle_gelu_tanh")
        return out

    def silu(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        self._check(self.lib.oracle_silu(_p(x), _p(out), x.size), "oracle_silu")
        return out

    def modulate(self, h, scale, shift):
        h = _f32(h).copy()
        B, L, C = h.shape
        self._check(self.lib.oracle_modulate_inplace(
            _p(h), _p(_f32(scale)), _p(_f32(shift)), B, L, C), "oracle_modulate_inplace")
        return h

    def gated_residual(self, base, delta, gate):
        base = _f32(base).copy()
        delta = _f32(delta).copy()
        B, L, C = base.shape
        self._check(self.lib.oracle_gated_residual_inplace(
            _p(base), _p(delta), _p(_f32(gate)), B, L, C), "oracle_gated_residual_inplace")
        return base, delta

    def add(self, base, delta):
        base = _f32(base).copy()
        self._check(self.lib.oracle_add_inplace(_p(base), _p(_f32(delta)), base.size),
                    "oracle_add_inplace")
        return base

    def cfg_combine(self, pos, neg, guidance):
        pos = _f32(pos).copy()
        B = pos.shape[0]
        self._check(self.lib.oracle_cfg_combine_inplace(
            _p(pos), _p(_f32(neg)), _p(_f32(guidance)), B, pos.size // B),
            "oracle_cfg_combine_inplace")
        return pos

    def euler_update(self, sample, pred, dt):
        sample = _f32(sample).copy()
        B = sample.shape[0]
        self._check(self.lib.oracle_euler_update_inplace(
            _p(sample), _p(_f32(pred)), _p(_f32(dt)), B, sample.size // B),
            "oracle_euler_update_inplace")
        return sample

    def timestep_embedding(self, t, freqs, output_dim=None):
        """[batch] timesteps, [half] frequencies -> [batch, output_dim] = [cos | sin | 0]."""
        t, f = _f32(t), _f32(freqs)
        half = f.shape[0]
        output_dim = 2 * half if output_dim is None else output_dim
        out = np.empty((t.shape[0], output_dim), np.float32)
        self._check(self.lib.oracle_timestep_embedding(_p(t), _p(f), _p(out), t.shape[0], half,
                                                       output_dim), "oracle_timestep_embedding")
        return out

    def pcd_position_embedding(self, positions, freqs, channels, double_pi=False):
        """positions [rows, dims], freqs [F] -> [rows, channels] = per axis [sin | cos], 0 pad."""
        x, f = _f32(positions), _f32(freqs)
        out = np.empty((x.shape[0], channels), np.float32)
        self._check(self.lib.oracle_pcd_position_embedding(
            _p(x), _p(f), _p(out), x.shape[0], x.shape[1], f.shape[0], channels, int(double_pi)),
            "oracle_pcd_position_embedding")
        return out

    def ab2_update(self, sample, pred, prev, dt, prev_dt):
        """[batch, n] sample / predictions, dt and prev_dt [batch] -> updated sample."""
        out = _f32(sample).copy()
        b = out.shape[0]
        self._check(self.lib.oracle_ab2_update_inplace(
            _p(out), _p(_f32(pred)), _p(_f32(prev)), _p(_f32(dt)), _p(_f32(prev_dt)), b,
            out.size // b), "oracle_ab2_update_inplace")
        return out

    def mul(self, lhs, rhs):
        out = _f32(lhs).copy()
        self._check(self.lib.oracle_mul_inplace(_p(out), _p(_f32(rhs)), out.size), "oracle_mul_inplace")
        return out

    def repo_phasor(self, delta, ft, fr):
        """delta [vectors, 3]; ft / fr: three per-axis arrays -> [vectors, 2 * sum(dims)]
        interleaved (cos, sin)."""
        d = _f32(delta)
        ft, fr = [_f32(a) for a in ft], [_f32(a) for a in fr]
        dims = [a.shape[0] for a in ft]
        out = np.empty((d.shape[0], 2 * sum(dims)), np.float32)
        self._check(self.lib.oracle_repo_phasor(
            _p(d), _p(ft[0]), _p(fr[0]), dims[0], _p(ft[1]), _p(fr[1]), dims[1],
            _p(ft[2]), _p(fr[2]), dims[2], _p(out), d.shape[0]), "oracle_repo_phasor")
        return out

    def qkv_rope_rmsnorm_pack(self, qkv, freqs, q_gamma, k_gamma, Lp=None):
        qkv = _f32(qkv)
        B, L, _, H, D = qkv.shape
        Lp = ((L + 15) // 16) * 16 if Lp is None else Lp
        fb = freqs.shape[0]
        q = np.empty((B, H, L, D), np.float32)
        pk = np.empty((B, H, D, Lp), np.float32)
        pv = np.empty((B, H, D, Lp), np.float32)
        self._check(self.lib.oracle_qkv_rope_rmsnorm_pack(
            _p(qkv), _p(_f32(freqs)), _p(_f32(q_gamma)), _p(_f32(k_gamma)),
            _p(q), _p(pk), _p(pv), B, L, H, Lp, fb), "oracle_qkv_rope_rmsnorm_pack")
        return q, pk, pv


class ReferenceKernels:
    """The reference's own AVX-512 kernels built into oracle/_ref (optional)."""

    def __init__(self, ref_dir: Path = REF_DIR):
        self.dir = ref_dir
        gemm = ref_dir / "libref_gemm_nf24_i16.so"
        sdpa = ref_dir / "libref_sdpa_q8t512.so"
        if not gemm.is_file() or not sdpa.is_file():
            raise FileNotFoundError(f"reference kernels missing under {ref_dir}")
        self.gemm_lib = ctypes.CDLL(str(gemm))
        self.sdpa_lib = ctypes.CDLL(str(sdpa))
        for name, n_int in (("triposplat_gemm_rnf8_avx512", 7),
                            ("triposplat_gemm_rnf8_avx512_tail", 7),
                            ("triposplat_gemm_rnf8_avx512_range", 9)):
            fn = getattr(self.gemm_lib, name)
            fn.argtypes = [_VP] * 10 + [_I] * n_int
            fn.restype = _I
        fn = self.sdpa_lib.triposplat_sdpa_f32_avx512_exact_q8t512
        fn.argtypes = [_VP] * 5 + [_I] * 8
        fn.restype = _I

    @staticmethod
    def available(ref_dir: Path = REF_DIR) -> bool:
        if not (ref_dir / "libref_gemm_nf24_i16.so").is_file():
            return False
        try:
            flags = Path("/proc/cpuinfo").read_text()
        except OSError:
            return False
        return all(f in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl"))

    def gemm_nf24(self, x, code01_t, q2_t, scale, bias, threads=0, start=0, count=None):
        x = _f32(x)
        M, K = x.shape
        N = code01_t.shape[1]
        c01 = np.ascontiguousarray(code01_t, dtype=np.int16)
        c2 = np.ascontiguousarray(q2_t, dtype=np.int8)
        sc, bi = _f32(scale), _f32(bias)
        codebook = np.zeros(256, np.float32)
        if count is not None or start:
            count = N - start if count is None else count
            out = np.empty((M, count), np.float32)
            st = self.gemm_lib.triposplat_gemm_rnf8_avx512_range(
                _p(x), _p(c01), _p(c2), _p(c2), _p(sc), _p(sc), _p(sc), _p(codebook), _p(bi),
                _p(out), M, K, N, start, count, K, count, threads, 3)
        else:
            out = np.empty((M, N), np.float32)
            fn = (self.gemm_lib.triposplat_gemm_rnf8_avx512_tail if N % 16
                  else self.gemm_lib.triposplat_gemm_rnf8_avx512)
            st = fn(_p(x), _p(c01), _p(c2), _p(c2), _p(sc), _p(sc), _p(sc), _p(codebook), _p(bi),
                    _p(out), M, K, N, K, N, threads, 3)
        if st != 0:
            raise RuntimeError(f"reference gemm status {st}")
        return out

    def sdpa(self, q, k, v, bias=None, threads=0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, Lq, D = q.shape
        Lk = k.shape[2]
        out = np.empty_like(q)
        b = None if bias is None else _f32(bias).reshape(-1)
        st = self.sdpa_lib.triposplat_sdpa_f32_avx512_exact_q8t512(
            _p(q), _p(k), _p(v), _p(b), _p(out), B, H, Lq, Lk, D,
            int(b is not None), 0 if b is None else b.size, threads)
        if st != 0:
            raise RuntimeError(f"reference sdpa status {st}")
        return out


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
