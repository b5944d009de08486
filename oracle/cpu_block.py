"""CPU baseline: one flow-transformer block of the CFG pair, timed on the host cores.

TEST / BASELINE INFRASTRUCTURE ONLY (used by bench.py's cpu_baseline leg and its
``--impl reference`` arm).  The block is composed from the reference's own AVX-512
kernels compiled into oracle/_ref (``kind = "reference"``) — the NF24 GEMM
(scripts/gemm_nf24_i16_avx512.c), QKV post-process v2, the packed q8/tile-512 exact
SDPA, LayerNorm / RMSNorm, GELU and the block elementwise kernels — exactly as the
reference's packed-v3 route chains them (scripts/native_qkv_packed_attention_patch_v3.py).
Without AVX-512 on the host, the oracle restatement (``kind = "port"``) stands in.

The sample is one block at full size (B=2, L=8193, C=1024, 1374 condition tokens);
sec/image is extrapolated by flops: 20 steps x forward_flops / block_flops x T_block.
Codes are random int16/int8 (as scripts/bench_native_rnf8_avx512.py:120-131 does):
the kernels' cost does not depend on the values.
"""
from __future__ import annotations

import ctypes
import os
import time
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


class _RefKernels:
    kind = "reference"

    def __init__(self, threads):
        self.th = threads
        g = ctypes.CDLL(str(REF / "libref_gemm_nf24_i16.so"))
        self.gemm = _bind(g, "triposplat_gemm_rnf8_avx512", [VP] * 10 + [I] * 7)
        self.gemm_tail = _bind(g, "triposplat_gemm_rnf8_avx512_tail", [VP] * 10 + [I] * 7)
        nr = ctypes.CDLL(str(REF / "libref_norm_rope.so"))
        self.ln = _bind(nr, "triposplat_layernorm_f32_avx512", [VP] * 4 + [I64, I, F, I, I])
        self.rms = _bind(nr, "triposplat_multihead_rmsnorm_f32_avx512", [VP] * 3 + [I64, I, I, F, I])
        act = ctypes.CDLL(str(REF / "libref_activations.so"))
        self.gelu = _bind(act, "triposplat_gelu_tanh_f32_avx512", [VP] * 2 + [I64, I])
        blk = ctypes.CDLL(str(REF / "libref_block_elementwise.so"))
        self.mod = _bind(blk, "triposplat_modulate_inplace_f32_avx512", [VP] * 3 + [I] * 4)
        self.gres = _bind(blk, "triposplat_gated_residual_inplace_f32_avx512", [VP] * 3 + [I] * 4)
        self.add = _bind(blk, "triposplat_add_inplace_f32_avx512", [VP] * 2 + [I64, I])
        post = ctypes.CDLL(str(REF / "libref_qkv_postprocess_v2.so"))
        self.post = _bind(post, "triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2", [VP] * 7 + [I] * 7)
        sd = ctypes.CDLL(str(REF / "libref_sdpa_q8t512_packed.so"))
        self.sdpa_packed = _bind(sd, "triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd",
                                 [VP] * 5 + [I] * 9)

    @staticmethod
    def available() -> bool:
        if not (REF / "libref_sdpa_q8t512_packed.so").is_file():
            return False
        try:
            flags = Path("/proc/cpuinfo").read_text()
        except OSError:
            return False
        return all(f in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl"))


def _check(st, what):
    if st != 0:
        raise RuntimeError(f"{what} -> {st}")


class CpuBlock:
    """Buffers + weights for one block of the batch-2 pair, on the host."""

    def __init__(self, spec, threads=None, seed=0):
        self.s = spec
        self.th = threads or len(os.sched_getaffinity(0))
        if not _RefKernels.available():
            raise RuntimeError("reference kernels unavailable (oracle/_ref missing or no AVX-512)")
        self.k = _RefKernels(self.th)
        rng = np.random.default_rng(seed)
        s = spec
        h, B, L, Mc, H = s.hidden, 2, s.seq, s.cond_tokens, s.heads
        self.Lp = (L + 15) // 16 * 16
        self.Mcp = (Mc + 15) // 16 * 16
        self.lin = {}
        for name, k, n in (("qkv", h, 3 * h), ("out", h, h), ("cross_q", h, h), ("cross_kv", h, 2 * h),
                           ("cross_out", h, h), ("fc1", h, s.mlp), ("fc2", s.mlp, h)):
            self.lin[name] = (rng.integers(-540, 541, size=(k, n), dtype=np.int16),
                              rng.integers(-128, 128, size=(k, n), dtype=np.int8),
                              np.full(n, 0.02 / 127 / 1024, np.float32),
                              (rng.standard_normal(n) * 0.01).astype(np.float32))
        f32 = np.float32
        self.x = rng.standard_normal((B, L, h)).astype(f32)
        self.c = rng.standard_normal((B, Mc, h)).astype(f32)
        self.a = np.empty((B, L, h), f32)
        self.y = np.empty((B, L, h), f32)
        self.qkv = np.empty((B, L, 3 * h), f32)
        self.q = np.empty((B, H, L, 64), f32)
        self.pk = np.empty((B, H, 64, self.Lp), f32)
        self.pv = np.empty((B, H, 64, self.Lp), f32)
        self.o = np.empty((B, L, h), f32)
        self.ckv = np.empty((B, Mc, 2 * h), f32)
        self.cpk = np.zeros((B, H, 64, self.Mcp), f32)
        self.cpv = np.zeros((B, H, 64, self.Mcp), f32)
        self.hid = np.empty((B, L, s.mlp), f32)
        self.mod = (rng.standard_normal((6, B, h)) * 0.02).astype(f32)
        ang = rng.standard_normal((1, L, H, 32))
        self.freqs = np.stack([np.cos(ang), np.sin(ang)], -1).reshape(1, L, H, 64).astype(f32)
        self.gam = np.ones((H, 64), f32)
        self.codebook = np.zeros(256, f32)

    def _gemm(self, name, x, out, rows):
        c01, q2, sc, b = self.lin[name]
        K, N = c01.shape
        _check(self.k.gemm(_p(x), _p(c01), _p(q2), _p(q2), _p(sc), _p(sc), _p(sc), _p(self.codebook),
                           _p(b), _p(out), rows, K, N, K, N, self.th, 3), name)

    def run(self):
        s, k, th = self.s, self.k, self.th
        B, L, h, H, Mc = 2, s.seq, s.hidden, s.heads, s.cond_tokens
        x, a, y, m = self.x, self.a, self.y, self.mod
        rows, crow = B * L, B * Mc
        _check(k.ln(_p(x), None, None, _p(a), rows, h, s.eps, 0, th), "ln1")
        _check(k.mod(_p(a), _p(m[1]), _p(m[0]), B, L, h, th), "mod1")
        self._gemm("qkv", a, self.qkv, rows)
        _check(k.post(_p(self.qkv), _p(self.freqs), _p(self.gam), _p(self.gam), _p(self.q), _p(self.pk),
                      _p(self.pv), B, L, H, 64, self.Lp, 1, th), "post")
        _check(k.sdpa_packed(_p(self.q), _p(self.pk), _p(self.pv), None, _p(self.o), B, H, L, L, 64,
                             self.Lp, 0, 0, th), "self_sdpa")
        self._gemm("out", self.o, y, rows)
        _check(k.gres(_p(x), _p(y), _p(m[2]), B, L, h, th), "gres1")
        _check(k.ln(_p(x), None, None, _p(a), rows, h, s.eps, 0, th), "ln2")
        self._gemm("cross_q", a, y, rows)
        _check(k.rms(_p(y), _p(self.gam), _p(y), rows, H, 64, 1e-12, th), "rms_q")
        self._gemm("cross_kv", self.c, self.ckv, crow)
        # packed condition K/V layout and the query layout conversions the CPU route needs
        ckv = self.ckv.reshape(B, Mc, 2, H, 64)
        self.cpk[..., :Mc] = ckv[:, :, 0].transpose(0, 2, 3, 1)
        self.cpv[..., :Mc] = ckv[:, :, 1].transpose(0, 2, 3, 1)
        self.q[...] = y.reshape(B, L, H, 64).transpose(0, 2, 1, 3)
        _check(k.sdpa_packed(_p(self.q), _p(self.cpk), _p(self.cpv), None, _p(self.o), B, H, L, Mc, 64,
                             self.Mcp, 0, 0, th), "cross_sdpa")
        self._gemm("cross_out", self.o, y, rows)
        _check(k.add(_p(x), _p(y), x.size, th), "add")
        _check(k.ln(_p(x), None, None, _p(a), rows, h, s.eps, 0, th), "ln3")
        _check(k.mod(_p(a), _p(m[4]), _p(m[3]), B, L, h, th), "mod3")
        self._gemm("fc1", a, self.hid, rows)
        _check(k.gelu(_p(self.hid), _p(self.hid), self.hid.size, th), "gelu")
        self._gemm("fc2", self.hid, y, rows)
        _check(k.gres(_p(x), _p(y), _p(m[5]), B, L, h, th), "gres3")

    def block_flops(self) -> float:
        s = self.s
        B, L, h, Mc = 2, s.seq, s.hidden, s.cond_tokens
        gemm = 2.0 * B * (L * h * 3 * h + L * h * h * 3 + Mc * h * 2 * h + 2 * L * h * s.mlp)
        sdpa = 4.0 * B * s.heads * L * (L + Mc) * 64
        return gemm + sdpa


def sec_per_image_from_block(spec, block_seconds: float, block_flops: float, steps: int = 20) -> float:
    fwd = spec.flops_per_forward(batch=2)["total"]
    return steps * block_seconds * fwd / block_flops


def time_sample(spec, min_seconds=10.0, max_reps=3, threads=None):
    """Run the block until ~min_seconds of CPU work (at least once); return stats."""
    blk = CpuBlock(spec, threads=threads)
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start < min_seconds and len(times) < max_reps):
        t0 = time.perf_counter()
        blk.run()
        times.append(time.perf_counter() - t0)
    t_block = float(np.median(times))
    return {"block_seconds": t_block, "reps": len(times), "threads": blk.th, "kind": blk.k.kind,
            "block_flops": blk.block_flops(),
            "sec_per_image": sec_per_image_from_block(spec, t_block, blk.block_flops())}
