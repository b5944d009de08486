"""CPU baseline: the synthetic flow model's forward on the reference's own AVX-512 kernels,
timed on the host cores.

TEST / BASELINE INFRASTRUCTURE ONLY (used by bench.py's cpu_baseline leg and its
``--impl reference`` arm).  The model is ``ref_flow.RefFlowModel`` — the same forward the
GPU runs (embeddings, adaLN, 28 blocks with self and cross attention, final layer), every
op one call of a reference kernel compiled into oracle/_ref — followed by the sampler's
CFG combine + Euler update (scripts/native_sampler_avx512.c:19,56).  One sampler step is
cut into 30 pieces: the embeddings, each of the 28 blocks, and the final layer with the
update; a timed sample runs pieces and sec/image = 20 x (sum of the 30 pieces' times).

Codes are random int16 / int8 per Linear with a constant scale (as
scripts/bench_native_rnf8_avx512.py:120-131 does): the kernels' cost does not depend on
the values, and generating them takes seconds where packing 477 M weights would take more.
"""
from __future__ import annotations

import time

import numpy as np

from ref_flow import RefFlowModel, RefKernels, _check, _p

SAMPLER_STEPS = 20


class RefForward:
    """One batch-2 (CFG pair) sampler step of the full-size model on the reference kernels,
    as a list of pieces (callables) covering it exactly once."""

    def __init__(self, spec, threads=None, seed=0):
        from flow_model import rope_freqs, timestep_frequencies

        if not RefKernels.available():
            raise RuntimeError("reference kernels unavailable (oracle/_ref missing or no AVX-512)")
        self.s = spec
        rng = np.random.default_rng(seed)
        f32 = np.float32
        W = {}
        for name, k, n in spec.linears():
            W[name] = {"code01": rng.integers(-540, 541, size=(k, n), dtype=np.int16),
                       "q2": rng.integers(-128, 128, size=(k, n), dtype=np.int8),
                       "scale": np.full(n, 0.02 / 127 / 1024, f32),
                       "bias": rng.standard_normal(n, dtype=f32) * f32(0.01)}
        H, D = spec.heads, spec.head_dim
        P = {}
        for i in range(spec.blocks):
            p = f"blocks.{i}."
            P[p + "table"] = rng.standard_normal((6, spec.hidden), dtype=f32) * f32(0.02)
            for gname in ("q_gamma", "k_gamma", "cq_gamma", "ck_gamma"):
                P[p + gname] = f32(1.0) + rng.standard_normal((H, D), dtype=f32) * f32(0.02)
        self.m = RefFlowModel(spec, W, P, rope_freqs(spec), timestep_frequencies(spec),
                              batch=2, threads=threads)
        self.th = self.m.k.th
        self.kind = self.m.k.kind
        lat = rng.standard_normal((1, spec.latent_tokens, spec.latent_dim), dtype=f32)
        cam = rng.standard_normal((1, 1, spec.camera_dim), dtype=f32)
        cond = rng.standard_normal((1, spec.cond_tokens, spec.cond_dim), dtype=f32)
        self.x_lat, self.x_cam = lat, cam
        self.cond_pair = np.ascontiguousarray(np.concatenate([cond, np.zeros_like(cond)]))
        self.t = np.array([750.0, 750.0], f32)
        self.g = np.array([3.0], f32)
        self.dt = np.array([0.05], f32)

    def _embed(self):
        self.m.embed(np.concatenate([self.x_lat] * 2), np.concatenate([self.x_cam] * 2), self.t,
                     self.cond_pair)

    def _final_and_update(self):
        k = self.m.k
        vl, vc = self.m.final_layer()
        for x, v in ((self.x_lat, vl), (self.x_cam, vc)):
            pos, neg = np.ascontiguousarray(v[:1]), np.ascontiguousarray(v[1:])
            _check(k.cfg(_p(pos), _p(neg), _p(self.g), 1, pos.size, k.th), "cfg_combine")
            _check(k.euler(_p(x), _p(pos), _p(self.dt), 1, x.size, k.th), "euler_update")

    def pieces(self):
        """[embed, block 0, ..., block 27, final layer + CFG / Euler update]."""
        blocks = [(lambda i=i: self.m.block(i)) for i in range(self.s.blocks)]
        return [self._embed] + blocks + [self._final_and_update]


def time_pieces(fwd: RefForward, order):
    """Run pieces in ``order`` (indices into fwd.pieces()); return per-run seconds."""
    pieces = fwd.pieces()
    out = []
    for j in order:
        t0 = time.perf_counter()
        pieces[j]()
        out.append((j, time.perf_counter() - t0))
    return out


def time_sample(spec, block_reps: int = 3, threads=None):
    """Bounded sample for bench.py's cpu_baseline leg (~10-30 s of CPU work): the embedding
    piece once, ``block_reps`` blocks (median), the final piece once; one sampler step =
    embed + blocks x median block + final (every block has the same shapes)."""
    fwd = RefForward(spec, threads=threads)
    n = len(fwd.pieces())
    runs = time_pieces(fwd, [0] + list(range(1, 1 + block_reps)) + [n - 1])
    t_embed = runs[0][1]
    t_block = float(np.median([t for _, t in runs[1:-1]]))
    t_final = runs[-1][1]
    step = t_embed + spec.blocks * t_block + t_final
    return {"embed_seconds": t_embed, "block_seconds": t_block, "final_seconds": t_final,
            "step_seconds": step, "sec_per_image": SAMPLER_STEPS * step, "threads": fwd.th,
            "kind": fwd.kind, "reps": block_reps}
