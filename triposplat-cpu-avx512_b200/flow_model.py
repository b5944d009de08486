"""Synthetic TripoSplat-style flow transformer and its CFG / Euler sampler on B200.

The reference patches the upstream ``LatentSeqMMFlowModel`` (not vendored), so the
benchmark model is a seeded synthetic stand-in with the shapes BASELINE.json names:
28 blocks, hidden 1024, 16 heads x 64, MLP 4096, 8192 latent tokens on a 16x16x32
grid with 3-D RoPE (theta 10000), a 7-dim camera token, 1374 condition tokens of
dim 1024, and 206 NF24 Linears.  Every Linear, attention, norm, activation,
modulation, residual and sampler update runs through ``libtriposplat_b200.so``;
PyTorch only allocates device buffers and issues device-to-device copies.

Block (order of scripts/native_block_elementwise_avx512_patch.py:45-54 and
scripts/triposplat_attention_patch.py:4978-5034, plus BASELINE's cross-attention):
    mod_i = adaLN(SiLU(temb)) + table_i -> (shift, scale, gate) for msa and mlp
    x += gate_msa * Out(SDPA(RMSNorm(RoPE(q)), RMSNorm(RoPE(k)), v)),  qkv = QKV(mod(LN(x)))
    x += CrossOut(SDPA(RMSNorm(CrossQ(LN(x))), RMSNorm(k_c), v_c)),     kv_c = CrossKV(cond)
    x += gate_mlp * FC2(GELU_tanh(FC1(mod(LN(x)))))
RoPE is applied before the per-head RMSNorm ``x*8/max(||x||,1e-12)*gamma``
(scripts/native_qkv_postprocess_v2_avx512.c:3-24).

Sampler (scripts/triposplat_quantized_sampler.py:387-494): ``u = linspace(1, 0, K+1)``
in float64, ``t_i = s*u/(1+(s-1)*u)``, the model runs on the batch-2 pair
[cond, uncond] at ``1000*t_i``, ``v = g*v_c - (g-1)*v_u``, ``x -= (t_i - t_{i+1}) * v``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

import _native
from nf24_linear import nf24_linear
from nf24_pack import make_nf8_codebook, quantize_nf24_i16_any_device


@dataclass(frozen=True)
class FlowSpec:
    blocks: int = 28
    hidden: int = 1024
    heads: int = 16
    mlp: int = 4096
    grid: tuple = (16, 16, 32)
    latent_dim: int = 64
    camera_dim: int = 7
    cond_tokens: int = 1374
    cond_dim: int = 1024
    t_freq: int = 256
    eps: float = 1e-6
    theta: float = 10000.0
    rope_pairs: tuple = (10, 11, 11)  # complex pairs per grid axis; sums to head_dim / 2

    @property
    def latent_tokens(self) -> int:
        return int(np.prod(self.grid))

    @property
    def seq(self) -> int:  # latent tokens + 1 camera token
        return self.latent_tokens + 1

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @classmethod
    def small(cls, blocks: int = 2) -> "FlowSpec":
        """Oracle-sized model with the same structure (used by the parity tests)."""
        return cls(blocks=blocks, hidden=128, heads=2, mlp=512, grid=(4, 4, 4), latent_dim=16,
                   camera_dim=7, cond_tokens=17, cond_dim=96, t_freq=64)

    def linears(self) -> list[tuple[str, int, int]]:
        h = self.hidden
        out = [("x_embedder", self.latent_dim, h), ("camera_embedder", self.camera_dim, h),
               ("t_fc1", self.t_freq, h), ("t_fc2", h, h), ("cond_embedder", self.cond_dim, h),
               ("cond_refiner", h, h), ("adaLN", h, 6 * h), ("final_adaLN", h, 2 * h),
               ("final_linear", h, self.latent_dim), ("camera_head", h, self.camera_dim)]
        for i in range(self.blocks):
            p = f"blocks.{i}."
            out += [(p + "qkv", h, 3 * h), (p + "out", h, h), (p + "cross_q", h, h),
                    (p + "cross_kv", h, 2 * h), (p + "cross_out", h, h), (p + "fc1", h, self.mlp),
                    (p + "fc2", self.mlp, h)]
        return out

    def flops_per_forward(self, batch: int = 2, tp: int = 1) -> dict[str, float]:
        """Algorithmic flops of one forward (2*M*K*N per Linear, 4*Lq*Lk*64 per head); with
        tp > 1 one head-sharded rank's share (1/tp of the blocks, all of the rest)."""
        L, Mc = self.seq, self.cond_tokens
        gemm = 0.0
        for name, k, n in self.linears():
            rows = {"x_embedder": self.latent_tokens, "camera_embedder": 1, "t_fc1": 1, "t_fc2": 1,
                    "adaLN": 1, "final_adaLN": 1, "final_linear": self.latent_tokens,
                    "camera_head": 1, "cond_embedder": Mc, "cond_refiner": Mc}.get(name)
            share = 1.0
            if rows is None:
                rows = Mc if name.endswith("cross_kv") else L
                share = 1.0 / tp
            gemm += 2.0 * batch * rows * k * n * share
        sdpa = self.blocks * 4.0 * batch * self.heads * L * (L + Mc) * self.head_dim / tp
        return {"gemm": gemm, "sdpa": sdpa, "total": gemm + sdpa}


def rope_freqs(spec: FlowSpec) -> np.ndarray:
    """[1, L, H, 64] interleaved (cos, sin) for the 3-D grid; the camera token is unrotated."""
    gx, gy, gz = spec.grid
    n = np.arange(spec.latent_tokens)
    pos = [n // (gy * gz), (n // gz) % gy, n % gz]
    angles = []
    for axis, pairs in enumerate(spec.rope_pairs):
        inv = 1.0 / spec.theta ** (np.arange(pairs, dtype=np.float64) / pairs)
        angles.append(pos[axis][:, None].astype(np.float64) * inv[None, :])
    ang = np.concatenate(angles, axis=1)  # [Nl, 32]
    ang = np.concatenate([ang, np.zeros((1, ang.shape[1]))], axis=0)  # camera token
    f = np.stack([np.cos(ang), np.sin(ang)], axis=-1).reshape(spec.seq, 1, spec.head_dim)
    f = np.broadcast_to(f, (spec.seq, spec.heads, spec.head_dim))
    return np.ascontiguousarray(f[None].astype(np.float32))


def timestep_frequencies(spec: FlowSpec) -> np.ndarray:
    """exp(-ln(1e4) * i / half) in float32 (scripts/native_embeddings_avx512_patch.py:113-114)."""
    import torch

    half = spec.t_freq // 2
    return torch.exp(-float(np.log(10000)) * torch.arange(0, half, dtype=torch.float32) / half).numpy()


def sampler_schedule(steps: int, shift: float) -> tuple[np.ndarray, np.ndarray]:
    """Model timesteps (1000*t_i) and Euler steps (t_i - t_{i+1}), float32."""
    lin = np.linspace(1.0, 0.0, steps + 1, dtype=np.float64)
    t_seq = shift * lin / (1.0 + (shift - 1.0) * lin)
    return ((t_seq[:-1] * 1000.0).astype(np.float32),
            (t_seq[:-1] - t_seq[1:]).astype(np.float32))


@dataclass
class PackedLinear:
    code01: object  # int16 [in, out]
    q2: object      # int8  [in, out]
    scale: object   # f32 [out]
    bias: object    # f32 [out]


@dataclass
class FlowWeights:
    spec: FlowSpec
    linears: dict = field(default_factory=dict)  # name -> PackedLinear
    params: dict = field(default_factory=dict)   # name -> tensor (tables, gammas)

    def to(self, device):
        lin = {k: PackedLinear(*(t.to(device) for t in (v.code01, v.q2, v.scale, v.bias)))
               for k, v in self.linears.items()}
        return FlowWeights(self.spec, lin, {k: v.to(device) for k, v in self.params.items()})

    def nbytes(self) -> int:
        return sum(v.code01.numel() * 3 + v.scale.numel() * 8 for v in self.linears.values())


def host_float_weights(spec: FlowSpec, seed: int):
    """Yield ``(kind, name, array)`` for every weight of the model, drawn on the host from
    numpy's PCG64 stream in a fixed order: for each Linear (``spec.linears()`` order) its
    float32 ``[out, in]`` weight ~ N(0, 0.02^2) then its bias ~ N(0, 0.01^2); then per block
    the adaLN table ~ N(0, 0.02^2) and the four RMSNorm gammas ~ 1 + N(0, 0.02^2).
    The stream depends only on numpy's generator, so a parity fixture produced on one host
    can be regenerated on another."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    for name, k, n in spec.linears():
        w = rng.standard_normal((n, k), dtype=f32) * f32(0.02)
        b = rng.standard_normal(n, dtype=f32) * f32(0.01)
        yield "linear", name, (w, b)
    H, D = spec.heads, spec.head_dim
    for i in range(spec.blocks):
        p = f"blocks.{i}."
        yield "param", p + "table", rng.standard_normal((6, spec.hidden), dtype=f32) * f32(0.02)
        for gname in ("q_gamma", "k_gamma", "cq_gamma", "ck_gamma"):
            yield "param", p + gname, f32(1.0) + rng.standard_normal((H, D), dtype=f32) * f32(0.02)


def make_weights(spec: FlowSpec, seed: int = 0, device: str = "cuda",
                 source: str = "torch") -> FlowWeights:
    """Seeded random-init weights (W ~ N(0, 0.02^2), bias ~ N(0, 0.01^2), tables ~ N(0, 0.02^2),
    gammas ~ 1 + N(0, 0.02^2)) packed to NF24 where they are generated.

    ``source="torch"`` draws on ``device`` with torch's generator (the benchmark's weights);
    ``source="numpy"`` draws the same distributions on the host (``host_float_weights``) and
    packs them on ``device``, so the codes are reproducible across machines (full-size parity
    fixtures)."""
    import torch

    if source == "numpy":
        cb = make_nf8_codebook(torch).to(device)
        w = FlowWeights(spec)
        for kind, name, val in host_float_weights(spec, seed):
            if kind == "linear":
                wt = torch.from_numpy(val[0]).to(device)
                codes, scales, _ = quantize_nf24_i16_any_device(wt, cb, stats=False)
                w.linears[name] = PackedLinear(codes[0], codes[1], scales[0],
                                               torch.from_numpy(val[1]).to(device))
                del wt
            else:
                w.params[name] = torch.from_numpy(val).to(device)
        return w
    if source != "torch":
        raise ValueError(f"unknown weight source {source!r}")
    g = torch.Generator(device=device).manual_seed(seed)
    cb = make_nf8_codebook(torch).to(device)
    w = FlowWeights(spec)
    for name, k, n in spec.linears():
        wt = torch.randn(n, k, generator=g, device=device) * 0.02
        codes, scales, _ = quantize_nf24_i16_any_device(wt, cb, stats=False)
        bias = torch.randn(n, generator=g, device=device) * 0.01
        w.linears[name] = PackedLinear(codes[0], codes[1], scales[0], bias)
        del wt
    H, D = spec.heads, spec.head_dim
    for i in range(spec.blocks):
        p = f"blocks.{i}."
        w.params[p + "table"] = torch.randn(6, spec.hidden, generator=g, device=device) * 0.02
        for gname in ("q_gamma", "k_gamma", "cq_gamma", "ck_gamma"):
            w.params[p + gname] = 1.0 + torch.randn(H, D, generator=g, device=device) * 0.02
    return w


class FlowModelB200:
    """Forward of the synthetic flow model on preallocated device buffers (batch = CFG pair).

    ``forward(x_lat, cam, t1000, cond)`` runs everything.  With the fused path the condition
    side can be cached across sampler steps, as the reference's attention patch caches its
    static condition context (scripts/triposplat_attention_patch.py:906-975):
    ``precompute_condition(cond)`` runs the condition embedder / refiner and every block's
    cross K / V projection + split once, and ``forward_cached(x_lat, cam, t1000)`` runs the
    rest; together they give ``forward``'s bits."""

    supports_condition_cache = True

    def __init__(self, weights: FlowWeights, batch: int = 2, device: str = "cuda",
                 fused: bool = True):
        import torch

        self.fused = fused
        self.spec = s = weights.spec
        self.w = weights
        self.B = batch
        self.dev = device
        self.lib = _native.load()
        f32 = dict(dtype=torch.float32, device=device)
        B, L, h, H, Mc = batch, s.seq, s.hidden, s.heads, s.cond_tokens
        self.Lp = (L + 15) // 16 * 16
        self.Mcp = (Mc + 15) // 16 * 16
        self.freqs = torch.from_numpy(rope_freqs(s)).to(device)
        self.tfreqs = torch.from_numpy(timestep_frequencies(s)).to(device)
        e = torch.empty
        self.buf = {
            "tfe": e(B, s.t_freq, **f32), "t1": e(B, h, **f32), "temb": e(B, h, **f32),
            "stemb": e(B, h, **f32), "mod": e(6, B, h, **f32), "mod_i": e(6, B, h, **f32),
            "fmod": e(2, B, h, **f32),
            "c0": e(B, Mc, h, **f32), "c": e(B, Mc, h, **f32),
            "x": e(B, L, h, **f32), "a": e(B, L, h, **f32), "y": e(B, L, h, **f32),
            "qkv": e(B, L, 3 * h, **f32), "q": e(B, H, L, 64, **f32),
            "pk": e(B, H, 64, self.Lp, **f32), "pv": e(B, H, 64, self.Lp, **f32),
            "o": e(B, L, h, **f32), "ckv": e(B, Mc, 2 * h, **f32),
            "cpk": e(B, H, 64, self.Mcp, **f32), "cpv": e(B, H, 64, self.Mcp, **f32),
            "v_lat": e(B, s.latent_tokens, s.latent_dim, **f32), "v_cam": e(B, 1, s.camera_dim, **f32),
        }
        if not fused:  # the fused path writes the MLP hidden layer straight into "sp_hid"
            self.buf["hid"] = e(B, L, s.mlp, **f32)
        # split-format activation buffers for the fused path (LN/GELU/residual folded into
        # the GEMMs); 256-byte aligned as the library requires
        rows = B * L
        for name, r, k in (("sp_h", rows, h), ("sp_hid", rows, s.mlp), ("sp_c", B * Mc, h)):
            nbytes = int(self.lib.triposplat_b200_split_bytes(r, k))
            self.buf[name] = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        # k-contiguous copies of the block Linears' code planes ([N][K], one-time device
        # transpose) for the split-activation GEMMs of the fused path
        self.nk = {}
        if fused:
            _native.use_current_stream(self.lib)
            for name, lin in weights.linears.items():
                if not name.startswith("blocks."):
                    continue
                K, N = (int(d) for d in lin.code01.shape)
                c = torch.empty(N, K, dtype=torch.int16, device=device)
                q = torch.empty(N, K, dtype=torch.int8, device=device)
                self._ok(self.lib.triposplat_b200_nf24_codes_to_nk(
                    lin.code01.data_ptr(), lin.q2.data_ptr(), K, N, c.data_ptr(), q.data_ptr()),
                    f"codes_to_nk {name}")
                self.nk[name] = (c, q)
        # per block: the fc1 column-norm / bias bound that fixes the split scales of the
        # MLP hidden layer before fc1 runs (its GELU epilogue writes the fc2 split directly)
        self.gelu_bounds = {i: self._column_bound(f"blocks.{i}.fc1") for i in range(s.blocks)} if fused else {}
        # per-block adaLN tables, expanded over the batch so they add elementwise
        self.tables = {i: weights.params[f"blocks.{i}.table"][:, None, :].expand(6, B, h).contiguous()
                       for i in range(s.blocks)}
        # condition cache (fused path): per block the split K / V planes of the condition
        # tokens, filled once per image by precompute_condition, read by every step
        self.cond_planes = None
        if fused and self.supports_condition_cache:
            kvb = int(self.lib.triposplat_b200_attn_kv_planes_bytes(B * H, Mc))
            self.cond_planes = torch.empty(s.blocks, kvb + 256, dtype=torch.uint8, device=device)
            self.cond_plane_bytes = kvb + 256
            qb = int(self.lib.triposplat_b200_attn_q_planes_bytes(B * H, L))
            self.buf["cq_planes"] = torch.empty(qb + 256, dtype=torch.uint8, device=device)

    # -- helpers -------------------------------------------------------------------------
    def _column_bound(self, name):
        """(max over columns of the euclidean norm of the dequantised weight, max |bias|) of a
        block Linear, rounded up: the constants of the split-scale bound in
        triposplat_b200_ln_modulate_split_bound."""
        c, q = self.nk[name]
        lin = self.w.linears[name]
        norms = ((c.double() * 256.0 + q.double()) ** 2).sum(1).sqrt() * lin.scale.double().abs()
        up = 1.0 + 2.0 ** -20
        return float(norms.max()) * up, float(lin.bias.double().abs().max()) * up

    def _lin(self, name, x, out, start=0, count=None):
        p = self.w.linears[name]
        return nf24_linear(x, p.code01, p.q2, p.scale, p.bias, out=out, start=start, count=count,
                           lib=self.lib)

    def _ok(self, st, what):
        if int(st) != 0:
            raise RuntimeError(f"{what} returned status {st}")

    def _silu(self, x, out):
        self._ok(self.lib.triposplat_silu_f32_avx512(x.data_ptr(), out.data_ptr(), x.numel(), 0), "silu")

    def _ln(self, x, out):
        s = self.spec
        self._ok(self.lib.triposplat_layernorm_f32_avx512(
            x.data_ptr(), None, None, out.data_ptr(), x.numel() // s.hidden, s.hidden, s.eps, 0, 0),
            "layernorm")

    def _modulate(self, a, scale, shift):
        B, L, C = a.shape
        self._ok(self.lib.triposplat_modulate_inplace_f32_avx512(
            a.data_ptr(), scale.data_ptr(), shift.data_ptr(), B, L, C, 0), "modulate")

    def _gated(self, x, y, gate):
        B, L, C = x.shape
        self._ok(self.lib.triposplat_gated_residual_inplace_f32_avx512(
            x.data_ptr(), y.data_ptr(), gate.data_ptr(), B, L, C, 0), "gated_residual")

    def _add(self, x, y):
        self._ok(self.lib.triposplat_add_inplace_f32_avx512(x.data_ptr(), y.data_ptr(), x.numel(), 0), "add")

    # -- forward -------------------------------------------------------------------------
    def forward(self, x_lat, cam, t1000, cond):
        """x_lat [B,Nl,Cl], cam [B,1,Cc], t1000 [B] (already x1000), cond [B,Mc,Dc]."""
        if self.cond_planes is not None:
            self.precompute_condition(cond)
            return self.forward_cached(x_lat, cam, t1000)
        self._embed(x_lat, cam, t1000, cond)
        for i in range(self.spec.blocks):
            self._block(i)
        return self._final_layer()

    def precompute_condition(self, cond):
        """The condition path of one image: embedder -> SiLU -> refiner, then per block the
        cross K / V projection and its split planes (keys RMS-normalised per head)."""
        s, b, lib = self.spec, self.buf, self.lib
        B, H, Mc = self.B, s.heads, s.cond_tokens
        if self.cond_planes is None:
            raise RuntimeError("the condition cache needs the fused path")
        _native.use_current_stream(lib)
        self._lin("cond_embedder", cond, b["c0"])
        self._silu(b["c0"], b["c0"])
        self._lin("cond_refiner", b["c0"], b["c"])
        self._split(b["c"], self._split_ptr("sp_c"))
        for i in range(s.blocks):
            p = f"blocks.{i}."
            self._lin_split(p + "cross_kv", self._split_ptr("sp_c"), B * Mc, b["ckv"])
            self._ok(lib.triposplat_b200_kv_split_f32(
                b["ckv"].data_ptr(), self.w.params[p + "ck_gamma"].data_ptr(), B, Mc, H,
                self._cond_plane_ptr(i)), "condition kv split")

    def forward_cached(self, x_lat, cam, t1000):
        """forward() after precompute_condition() for this image's condition tokens."""
        self._embed(x_lat, cam, t1000, None)
        for i in range(self.spec.blocks):
            self._block_fused(i, cached=True)
        return self._final_layer()

    def _cond_plane_ptr(self, i):
        return (self.cond_planes[i].data_ptr() + 255) & ~255

    def _embed(self, x_lat, cam, t1000, cond):
        """Timestep / adaLN / condition / token embeddings into the block inputs."""
        s, b, lib = self.spec, self.buf, self.lib
        B, h, Nl = self.B, s.hidden, s.latent_tokens
        _native.use_current_stream(lib)
        # timestep embedding -> temb -> adaLN modulation (shared) and final modulation
        self._ok(lib.triposplat_timestep_embedding_f32_avx512(
            t1000.data_ptr(), self.tfreqs.data_ptr(), b["tfe"].data_ptr(), B, s.t_freq // 2,
            s.t_freq, 0), "timestep_embedding")
        self._lin("t_fc1", b["tfe"], b["t1"])
        self._silu(b["t1"], b["t1"])
        self._lin("t_fc2", b["t1"], b["temb"])
        self._silu(b["temb"], b["stemb"])
        for c in range(6):  # chunk-major [6, B, h] through column windows of one Linear
            self._lin("adaLN", b["stemb"], b["mod"][c], start=c * h, count=h)
        for c in range(2):
            self._lin("final_adaLN", b["stemb"], b["fmod"][c], start=c * h, count=h)
        # condition tokens (cond None: cached by precompute_condition)
        if cond is not None:
            self._lin("cond_embedder", cond, b["c0"])
            self._silu(b["c0"], b["c0"])
            self._lin("cond_refiner", b["c0"], b["c"])
            if self.fused:  # every block's cross_kv GEMM reads the same split condition tokens
                self._split(b["c"], self._split_ptr("sp_c"))
        # token embedding: [latent | camera]
        x = b["x"]
        for bb in range(B):  # per batch: the camera row sits between the batches' latents
            self._lin("x_embedder", x_lat[bb], x[bb, :Nl])
            self._lin("camera_embedder", cam[bb], x[bb, Nl:])

    def _final_layer(self):
        s, b = self.spec, self.buf
        B, Nl = self.B, s.latent_tokens
        x, a = b["x"], b["a"]
        self._ln(x, a)
        self._modulate(a, b["fmod"][1], b["fmod"][0])
        for bb in range(B):
            self._lin("final_linear", a[bb, :Nl], b["v_lat"][bb])
            self._lin("camera_head", a[bb, Nl:], b["v_cam"][bb])
        return b["v_lat"], b["v_cam"]

    def _split_ptr(self, name):
        t = self.buf[name]
        return (t.data_ptr() + 255) & ~255

    def _lin_split(self, name, split, rows, out, mode=0, gate=None, gate_ld=0, rows_per_batch=1):
        """out: a tensor, or (mode 4) the address of the split buffer the GELU output goes to."""
        p = self.w.linears[name]
        c, q = self.nk[name]
        N, K = int(c.shape[0]), int(c.shape[1])
        st = self.lib.triposplat_b200_gemm_nf24_split_nk(
            split, rows, K, c.data_ptr(), q.data_ptr(), K, p.scale.data_ptr(),
            p.bias.data_ptr(), out if isinstance(out, int) else out.data_ptr(), N, 0, N, N, mode,
            None if gate is None else gate.data_ptr(), gate_ld, rows_per_batch)
        self._ok(st, f"gemm_split {name}")

    def _ln_split(self, x, split, shift=None, scale=None, rows_per_batch=None, bound=None):
        """bound = (next_split, next_K, (wnorm, bmax)): also fix the row scales of next_split
        for a GELU-into-split GEMM."""
        s = self.spec
        rows = x.numel() // s.hidden
        rpb = s.seq if rows_per_batch is None else rows_per_batch
        args = (x.data_ptr(), rows, s.hidden, s.eps, None if shift is None else shift.data_ptr(),
                None if scale is None else scale.data_ptr(), s.hidden, rpb, split)
        if bound is None:
            self._ok(self.lib.triposplat_b200_ln_modulate_split(*args), "ln_split")
        else:
            nxt, nk, (wn, bm) = bound
            self._ok(self.lib.triposplat_b200_ln_modulate_split_bound(*args, nxt, nk, wn, bm),
                     "ln_split_bound")

    def _split(self, x, split):
        K = int(x.shape[-1])
        rows = x.numel() // K
        self._ok(self.lib.triposplat_b200_split_f32(x.data_ptr(), rows, K, K, split), "split")

    def _block(self, i):
        if self.fused:
            return self._block_fused(i)
        return self._block_reference_ops(i)

    def _block_fused(self, i, cached=False):
        """Same block, with LN/modulation fused into the activation split, GELU into the fc1
        epilogue and the (gated) residual adds into the out / cross_out / fc2 epilogues;
        cached: the condition keys / values come from precompute_condition."""
        s, b, lib = self.spec, self.buf, self.lib
        B, L, h, H, Mc = self.B, s.seq, s.hidden, s.heads, s.cond_tokens
        rows = B * L
        p = f"blocks.{i}."
        prm = self.w.params
        m = b["mod_i"]
        m.copy_(b["mod"])
        self._add(m, self.tables[i])
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (m[j] for j in range(6))
        x, y = b["x"], b["y"]
        sph, sphid = self._split_ptr("sp_h"), self._split_ptr("sp_hid")
        # self-attention
        self._ln_split(x, sph, shift_msa, scale_msa)
        self._lin_split(p + "qkv", sph, rows, b["qkv"])
        # RoPE + RMSNorm straight into the attention's split format, then the attention,
        # whose output goes straight into the out-projection's split format
        self._ok(lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_split(
            b["qkv"].data_ptr(), self.freqs.data_ptr(), prm[p + "q_gamma"].data_ptr(),
            prm[p + "k_gamma"].data_ptr(), B, L, H, 1, sph), "self_attention")
        self._lin_split(p + "out", sph, rows, x, mode=2, gate=gate_msa, gate_ld=h, rows_per_batch=L)
        # cross-attention
        self._ln_split(x, sph)
        self._lin_split(p + "cross_q", sph, rows, y)
        if cached:
            qpl = self._split_ptr("cq_planes")
            self._ok(lib.triposplat_b200_q_split_f32(y.data_ptr(), prm[p + "cq_gamma"].data_ptr(), B, L, H,
                                                     qpl), "cross q split")
            self._ok(lib.triposplat_b200_attend_rows_split(qpl, self._cond_plane_ptr(i), B, H, L, Mc, sph),
                     "cross_attention")
        else:
            self._lin_split(p + "cross_kv", self._split_ptr("sp_c"), B * Mc, b["ckv"])
            self._ok(lib.triposplat_b200_q_kv_rmsnorm_sdpa_split(
                y.data_ptr(), b["ckv"].data_ptr(), prm[p + "cq_gamma"].data_ptr(),
                prm[p + "ck_gamma"].data_ptr(), B, L, Mc, H, sph), "cross_attention")
        self._lin_split(p + "cross_out", sph, rows, x, mode=3)
        # MLP: the hidden layer's split scales fixed from a bound, GELU straight into that split
        self._ln_split(x, sph, shift_mlp, scale_mlp, bound=(sphid, s.mlp, self.gelu_bounds[i]))
        self._lin_split(p + "fc1", sph, rows, sphid, mode=4)
        self._lin_split(p + "fc2", sphid, rows, x, mode=2, gate=gate_mlp, gate_ld=h, rows_per_batch=L)

    def _block_reference_ops(self, i):
        """The block as the reference's patched modules chain their kernels (one C-ABI call per op)."""
        s, b, lib = self.spec, self.buf, self.lib
        B, L, h, H, Mc = self.B, s.seq, s.hidden, s.heads, s.cond_tokens
        p = f"blocks.{i}."
        prm = self.w.params
        m = b["mod_i"]
        m.copy_(b["mod"])
        self._add(m, self.tables[i])
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (m[j] for j in range(6))
        x, a, y = b["x"], b["a"], b["y"]
        # self-attention
        self._ln(x, a)
        self._modulate(a, scale_msa, shift_msa)
        self._lin(p + "qkv", a, b["qkv"])
        self._ok(lib.triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(
            b["qkv"].data_ptr(), self.freqs.data_ptr(), prm[p + "q_gamma"].data_ptr(),
            prm[p + "k_gamma"].data_ptr(), b["q"].data_ptr(), b["pk"].data_ptr(), b["pv"].data_ptr(),
            B, L, H, 64, self.Lp, 1, 0), "qkv_post")
        self._ok(lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
            b["q"].data_ptr(), b["pk"].data_ptr(), b["pv"].data_ptr(), None, b["o"].data_ptr(),
            B, H, L, L, 64, self.Lp, 0, 0, 0), "self_sdpa")
        self._lin(p + "out", b["o"], y)
        self._gated(x, y, gate_msa)
        # cross-attention to the condition tokens
        self._ln(x, a)
        self._lin(p + "cross_q", a, y)
        self._lin(p + "cross_kv", b["c"], b["ckv"])
        self._ok(lib.triposplat_b200_q_kv_rmsnorm_pack_f32(
            y.data_ptr(), b["ckv"].data_ptr(), prm[p + "cq_gamma"].data_ptr(),
            prm[p + "ck_gamma"].data_ptr(), b["q"].data_ptr(), b["cpk"].data_ptr(),
            b["cpv"].data_ptr(), B, L, Mc, H, self.Mcp), "cross_post")
        self._ok(lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
            b["q"].data_ptr(), b["cpk"].data_ptr(), b["cpv"].data_ptr(), None, b["o"].data_ptr(),
            B, H, L, Mc, 64, self.Mcp, 0, 0, 0), "cross_sdpa")
        self._lin(p + "cross_out", b["o"], y)
        self._add(x, y)
        # MLP
        self._ln(x, a)
        self._modulate(a, scale_mlp, shift_mlp)
        self._lin(p + "fc1", a, b["hid"])
        self._ok(lib.triposplat_gelu_tanh_f32_avx512(b["hid"].data_ptr(), b["hid"].data_ptr(),
                                                      b["hid"].numel(), 0), "gelu")
        self._lin(p + "fc2", b["hid"], y)
        self._gated(x, y, gate_mlp)


class CfgEulerSampler:
    """s-step CFG flow sampler over FlowModelB200 (batch-2 [cond, uncond] pair)."""

    def __init__(self, model: FlowModelB200, steps: int = 20, guidance: float = 3.0, shift: float = 3.0):
        import torch

        self.model = model
        self.steps = steps
        t1000, dt = sampler_schedule(steps, shift)
        dev = model.dev
        self.t_pair = torch.from_numpy(np.repeat(t1000[:, None], 2, axis=1)).to(dev)  # [K, 2]
        self.dt = torch.from_numpy(dt).to(dev)                                          # [K]
        self.g = torch.tensor([guidance], dtype=torch.float32, device=dev)
        s = model.spec
        f32 = dict(dtype=torch.float32, device=dev)
        self.x_lat = torch.empty(2, s.latent_tokens, s.latent_dim, **f32)
        self.x_cam = torch.empty(2, 1, s.camera_dim, **f32)
        self.cond_pair = torch.empty(2, s.cond_tokens, s.cond_dim, **f32)
        self.t_cur = torch.empty(2, **f32)   # the step's timestep pair, read by the body
        self.dt_cur = torch.empty(1, **f32)  # the step's Euler step
        self.graph = None
        self.graph_stream = None

    def load(self, noise_lat, noise_cam, cond, neg_cond):
        """One image's inputs; with the condition cache the condition path runs here, once
        per image, and every step reuses it."""
        self.x_lat[0].copy_(noise_lat.reshape(self.x_lat[0].shape), non_blocking=True)
        self.x_cam[0].copy_(noise_cam.reshape(self.x_cam[0].shape), non_blocking=True)
        self.cond_pair[0].copy_(cond.reshape(self.cond_pair[0].shape), non_blocking=True)
        self.cond_pair[1].copy_(neg_cond.reshape(self.cond_pair[1].shape), non_blocking=True)
        if self.cached:
            self.model.precompute_condition(self.cond_pair)

    @property
    def cached(self) -> bool:
        return getattr(self.model, "cond_planes", None) is not None

    def refresh_condition(self):
        """Re-run the once-per-image condition path on the loaded condition tokens."""
        if self.cached:
            self.model.precompute_condition(self.cond_pair)

    def _forward(self):
        if self.cached:
            return self.model.forward_cached(self.x_lat, self.x_cam, self.t_cur)
        return self.model.forward(self.x_lat, self.x_cam, self.t_cur, self.cond_pair)

    def _body(self):
        """One sampler step reading t_cur / dt_cur: everything a CUDA graph captures."""
        m, lib = self.model, self.model.lib
        self.x_lat[1].copy_(self.x_lat[0])
        self.x_cam[1].copy_(self.x_cam[0])
        v_lat, v_cam = self._forward()
        for x, v in ((self.x_lat, v_lat), (self.x_cam, v_cam)):
            # CFG combine + Euler step in one kernel (bit-identical to the reference's
            # triposplat_cfg_combine_inplace + triposplat_euler_update_inplace pair)
            st = lib.triposplat_b200_cfg_euler_update_f32(
                x[0].data_ptr(), v[0].data_ptr(), v[1].data_ptr(), self.g.data_ptr(),
                self.dt_cur.data_ptr(), 1, v[0].numel())
            if st:
                raise RuntimeError(f"sampler update returned status {st}")

    def velocity_pair(self, i: int):
        """Step i's [conditional, unconditional] velocities (latent [2, N, C], camera
        [2, 1, Cc]), without updating the state."""
        self.t_cur.copy_(self.t_pair[i])
        self.x_lat[1].copy_(self.x_lat[0])
        self.x_cam[1].copy_(self.x_cam[0])
        v_lat, v_cam = self._forward()
        return v_lat.clone(), v_cam.clone()

    def step(self, i: int):
        self.t_cur.copy_(self.t_pair[i])
        self.dt_cur.copy_(self.dt[i:i + 1])
        if self.graph is not None:
            self.graph.replay()
        else:
            self._body()

    def prepare_capture(self):
        """Run one eager step on the capture stream so the library's workspace for that
        stream is sized before capture (nothing is allocated while capturing)."""
        import torch

        self.graph_stream = torch.cuda.Stream(device=self.model.dev)
        self.graph_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.graph_stream):
            self._body()
        self.graph_stream.synchronize()

    def record_graph(self):
        """Record one sampler step into a CUDA graph, replayed by step()."""
        import torch

        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.graph_stream, capture_error_mode="relaxed"):
            self._body()
        torch.cuda.current_stream().wait_stream(self.graph_stream)
        self.graph = graph
        return graph

    def capture(self):
        self.prepare_capture()
        return self.record_graph()

    def run(self):
        for i in range(self.steps):
            self.step(i)
        return self.x_lat[0], self.x_cam[0]
