"""Query-row (sequence) sharded flow model: one rank per GPU, token rows split.

The reference runs every block over all tokens on one host
(``triposplat_attention_patch.py:4978-5034``).  Here a group of ``world`` ranks splits the
8193-token sequence by rows: rank r owns tokens ``[starts[r], starts[r+1])`` — the 8192
latent tokens in equal, 128-aligned shares, the camera token on the last rank — and runs
every per-token op of the forward on its own rows only:

* LayerNorm + modulate + split, all NF24 GEMMs (qkv, out, cross_q, cross_out, fc1, fc2) with
  their GELU / gated-residual / residual epilogues, the final layer: rows are independent,
  so nothing is exchanged;
* self-attention: each rank splits its own tokens (RoPE + RMSNorm) into its query planes
  and its key tiles of a K / V plane set; after a peer barrier it pulls the other ranks'
  key tiles over NVLink (``triposplat_b200_kv_planes_gather``) and attends its rows to all
  keys — the only exchange of the block (the K / V split planes, ~67 MB per branch in all);
* cross-attention: the condition tokens' K / V are computed on every rank (1374 rows).

Timestep embedding, adaLN and the condition path are replicated.  Every row sees exactly
the arithmetic of the unsharded model (same split planes, tiles, warps and order), so the
ranks' outputs are bit-identical to the rows of the single-GPU forward.

The plane sets alternate per block (block i writes set i % 2): a rank rewrites a set only
after every rank has passed the next block's barrier, i.e. finished pulling from it; a
forward therefore needs an even number of blocks to carry the alternation across forwards
(and CUDA-graph replays).  ``forward_steps`` yields at each exchange point so one process
can drive several ranks in lockstep on one GPU (``run_lockstep``).
"""
from __future__ import annotations

import ctypes

import _native
from flow_model import FlowModelB200, FlowSpec, FlowWeights, sampler_schedule

KEY_TILE = 128


def seq_shard_plan(spec: FlowSpec, world: int) -> list[int]:
    """Token starts of the ``world`` ranks (world + 1 entries): the latent tokens in equal
    shares of whole key tiles, the camera token (the last token) on the last rank."""
    Nl, L = spec.latent_tokens, spec.seq
    if world < 1 or world > 8:
        raise ValueError("query-row sharding runs on 1 to 8 ranks")
    if Nl % world or (Nl // world) % KEY_TILE:
        raise ValueError(f"{Nl} latent tokens do not split into {world} shares of whole "
                         f"{KEY_TILE}-token key tiles")
    return [r * (Nl // world) for r in range(world)] + [L]


class PeerPlanes:
    """Two K / V plane sets per rank and a barrier flag array, shared across the group
    through CUDA IPC (the pattern of ``head_shard.PeerReduce``)."""

    def __init__(self, lib, group, rank: int, world: int, set_bytes: int):
        import torch
        import torch.distributed as dist

        self.lib, self.rank, self.world, self.group = lib, rank, world, group
        self.local, handles = [], []
        for nbytes in (set_bytes, set_bytes, 64 * 4):
            ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
            st = lib.triposplat_b200_ipc_alloc(nbytes, ctypes.byref(ptr), h)
            if st:
                raise RuntimeError(f"ipc_alloc returned {st}")
            self.local.append(ptr.value)
            handles.append(bytes(h))
        allh = [None] * world
        dist.all_gather_object(allh, handles, group=group)
        self.opened, mapped = [], []
        for r in range(world):
            if r == rank:
                mapped.append(list(self.local))
                continue
            row = []
            for h in allh[r]:
                ptr = ctypes.c_void_p()
                st = lib.triposplat_b200_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(ptr))
                if st:
                    raise RuntimeError(f"ipc_open returned {st} for rank {r}")
                self.opened.append(ptr.value)
                row.append(ptr.value)
            mapped.append(row)
        arr = ctypes.c_uint64 * world
        self.sets = [arr(*[mapped[r][k] for r in range(world)]) for k in (0, 1)]
        self.flags = arr(*[mapped[r][2] for r in range(world)])
        self.counter = torch.zeros(1, dtype=torch.int32, device=f"cuda:{torch.cuda.current_device()}")

    def set_ptr(self, k: int) -> int:
        return self.local[k]

    def barrier(self):
        st = self.lib.triposplat_b200_peer_barrier(self.flags, self.rank, self.world,
                                                   self.counter.data_ptr())
        if st:
            raise RuntimeError(f"peer_barrier returned {st}")

    def close(self):
        import torch.distributed as dist

        for p in self.opened:
            self.lib.triposplat_b200_ipc_close(p)
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.local:
            self.lib.triposplat_b200_ipc_free(p)
        self.local = []


class SeqShardedFlowModel(FlowModelB200):
    """FlowModelB200 forward over this rank's token rows (rank ``rank`` of ``world``).

    exchange="peer": the K / V plane sets live in IPC-shared buffers; each block runs the
    peer barrier and the pull-gather kernel.  exchange="lockstep": plain device buffers;
    ``forward_steps`` yields at each exchange point and ``run_lockstep`` gathers for all
    ranks (one process, one GPU).  ``forward`` leaves this rank's velocity rows in
    ``chunk`` [B, (latent_tokens / world) * latent_dim + camera_dim, padded to 4 floats]
    (camera entries valid on the last rank) and returns it."""

    def __init__(self, weights: FlowWeights, rank: int, world: int, batch: int = 1,
                 device: str = "cuda", group=None, exchange: str = "peer"):
        import torch

        spec = weights.spec
        if exchange not in ("peer", "lockstep"):
            raise ValueError("exchange must be 'peer' or 'lockstep'")
        if spec.blocks % 2:
            raise ValueError(f"query-row sharding alternates two K / V plane sets per block; "
                             f"{spec.blocks} blocks (odd) would reuse a set with no barrier between")
        self.starts = seq_shard_plan(spec, world)
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside 0..{world - 1}")
        super().__init__(weights, batch=batch, device=device, fused=True)
        s = self.spec
        self.rank, self.world, self.group = rank, world, group
        self.t0, self.t1 = self.starts[rank], self.starts[rank + 1]
        self.Lloc = self.t1 - self.t0
        self.nlat = min(self.t1, s.latent_tokens) - self.t0
        self.has_cam = self.t1 > s.latent_tokens
        B, h, H, Lloc = self.B, s.hidden, s.heads, self.Lloc
        f32 = dict(dtype=torch.float32, device=device)
        e = torch.empty
        self.loc = {"x": e(B, Lloc, h, **f32), "a": e(B, Lloc, h, **f32), "y": e(B, Lloc, h, **f32),
                    "qkv": e(B, Lloc, 3 * h, **f32)}
        self.chunk_lat = (s.latent_tokens // world) * s.latent_dim
        # one row per batch, padded to 16 bytes so every row is a tensor-core GEMM output
        # (the drop-in GEMM sends unaligned outputs to its SIMT kernel, other rounding)
        self.chunk = torch.zeros(B, (self.chunk_lat + s.camera_dim + 3) // 4 * 4, **f32)
        for name, k in (("sp_hl", h), ("sp_hidl", s.mlp)):
            nbytes = int(self.lib.triposplat_b200_split_bytes(B * Lloc, k))
            self.buf[name] = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        qb = int(self.lib.triposplat_b200_attn_q_planes_bytes(B * H, Lloc))
        self.buf["qplanes"] = torch.empty(qb + 256, dtype=torch.uint8, device=device)
        self.kv_bytes = int(self.lib.triposplat_b200_attn_kv_planes_bytes(B * H, s.seq))
        self.exchange = exchange
        self.peer = None
        self.lock_sets = None
        if exchange == "peer":
            _native.use_current_stream(self.lib)
            self.peer = PeerPlanes(self.lib, group, rank, world, self.kv_bytes)
        else:
            self.lock_sets = [torch.empty(self.kv_bytes + 256, dtype=torch.uint8, device=device)
                              for _ in range(2)]
        self.starts_c = (ctypes.c_int * (world + 1))(*self.starts)

    # -- helpers ---------------------------------------------------------------------------
    def kv_set_ptr(self, k: int) -> int:
        if self.peer is not None:
            return self.peer.set_ptr(k)
        return (self.lock_sets[k].data_ptr() + 255) & ~255

    def _ln_split_rows(self, x, split, shift=None, scale=None, bound=None):
        self._ln_split(x, split, shift, scale, rows_per_batch=self.Lloc, bound=bound)

    def gather(self, set_ptrs):
        """Pull the other ranks' key tiles of the current block into this rank's set
        (set_ptrs: every rank's set as mapped here)."""
        s = self.spec
        st = self.lib.triposplat_b200_kv_planes_gather(set_ptrs, self.starts_c, self.world, self.rank,
                                                       self.B * s.heads, s.seq)
        self._ok(st, "kv_planes_gather")

    # -- forward ---------------------------------------------------------------------------
    def forward(self, x_lat, cam, t1000, cond):
        self.precompute_condition(cond)
        return self.forward_cached(x_lat, cam, t1000)

    def forward_cached(self, x_lat, cam, t1000):
        for _ in self.forward_steps(x_lat, cam, t1000, None):
            raise RuntimeError("forward() runs the peer exchange; drive lockstep ranks with run_lockstep")
        return self.chunk

    def forward_steps(self, x_lat, cam, t1000, cond=None):
        """The forward as a generator yielding at each exchange point (the plane set index);
        cond None: the condition cache of precompute_condition is current."""
        if cond is not None:
            self.precompute_condition(cond)
        self._embed_rows(x_lat, cam, t1000)
        for i in range(self.spec.blocks):
            yield from self._block_rows(i)
        self._final_rows()

    def _embed_rows(self, x_lat, cam, t1000):
        """Replicated timestep / adaLN path, then this rank's token rows (the condition path
        is cached by precompute_condition)."""
        s, b, lib = self.spec, self.buf, self.lib
        B, h = self.B, s.hidden
        _native.use_current_stream(lib)
        self._ok(lib.triposplat_timestep_embedding_f32_avx512(
            t1000.data_ptr(), self.tfreqs.data_ptr(), b["tfe"].data_ptr(), B, s.t_freq // 2,
            s.t_freq, 0), "timestep_embedding")
        self._lin("t_fc1", b["tfe"], b["t1"])
        self._silu(b["t1"], b["t1"])
        self._lin("t_fc2", b["t1"], b["temb"])
        self._silu(b["temb"], b["stemb"])
        for c in range(6):
            self._lin("adaLN", b["stemb"], b["mod"][c], start=c * h, count=h)
        for c in range(2):
            self._lin("final_adaLN", b["stemb"], b["fmod"][c], start=c * h, count=h)
        x = self.loc["x"]
        for bb in range(B):
            self._lin("x_embedder", x_lat[bb, self.t0:self.t0 + self.nlat], x[bb, :self.nlat])
            if self.has_cam:
                self._lin("camera_embedder", cam[bb], x[bb, self.nlat:])

    def _block_rows(self, i):
        s, b, lib, loc = self.spec, self.buf, self.lib, self.loc
        B, L, h, H, Mc = self.B, s.seq, s.hidden, s.heads, s.cond_tokens
        Lloc = self.Lloc
        rows = B * Lloc
        p = f"blocks.{i}."
        prm = self.w.params
        m = b["mod_i"]
        m.copy_(b["mod"])
        self._add(m, self.tables[i])
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (m[j] for j in range(6))
        x, y = loc["x"], loc["y"]
        sph, sphid = self._split_ptr("sp_hl"), self._split_ptr("sp_hidl")
        qpl = self._split_ptr("qplanes")
        kv = self.kv_set_ptr(i % 2)
        # self-attention: own rows split, key tiles exchanged, own rows attend to all keys
        self._ln_split_rows(x, sph, shift_msa, scale_msa)
        self._lin_split(p + "qkv", sph, rows, loc["qkv"])
        self._ok(lib.triposplat_b200_qkv_split_rows_f32(
            loc["qkv"].data_ptr(), self.freqs.data_ptr(), prm[p + "q_gamma"].data_ptr(),
            prm[p + "k_gamma"].data_ptr(), B, L, H, self.t0, self.t1, 1, qpl, kv), "qkv_split_rows")
        if self.peer is not None:
            self.peer.barrier()
            self.gather(self.peer.sets[i % 2])
        else:
            yield i % 2
        self._ok(lib.triposplat_b200_attend_rows_split(qpl, kv, B, H, Lloc, L, sph), "attend_rows")
        self._lin_split(p + "out", sph, rows, x, mode=2, gate=gate_msa, gate_ld=h, rows_per_batch=Lloc)
        # cross-attention of this rank's rows to the cached condition keys / values
        self._ln_split_rows(x, sph)
        self._lin_split(p + "cross_q", sph, rows, y)
        self._ok(lib.triposplat_b200_q_split_f32(y.data_ptr(), prm[p + "cq_gamma"].data_ptr(), B, Lloc, H,
                                                 qpl), "cross q split")
        self._ok(lib.triposplat_b200_attend_rows_split(qpl, self._cond_plane_ptr(i), B, H, Lloc, Mc, sph),
                 "cross_attention")
        self._lin_split(p + "cross_out", sph, rows, x, mode=3)
        # MLP
        self._ln_split_rows(x, sph, shift_mlp, scale_mlp, bound=(sphid, s.mlp, self.gelu_bounds[i]))
        self._lin_split(p + "fc1", sph, rows, sphid, mode=4)
        self._lin_split(p + "fc2", sphid, rows, x, mode=2, gate=gate_mlp, gate_ld=h, rows_per_batch=Lloc)

    def _final_rows(self):
        s, b, loc = self.spec, self.buf, self.loc
        x, a = loc["x"], loc["a"]
        self._ln(x, a)
        self._modulate(a, b["fmod"][1], b["fmod"][0])
        for bb in range(self.B):
            self._lin("final_linear", a[bb, :self.nlat], self.chunk[bb, :self.nlat * s.latent_dim])
            if self.has_cam:
                self._lin("camera_head", a[bb, self.nlat:],
                          self.chunk[bb, self.chunk_lat:self.chunk_lat + s.camera_dim])

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None


def run_lockstep(models, x_lat, cam, t1000, cond):
    """Drive the ranks' forwards in one process: at each exchange point every rank pulls
    the others' key tiles (same GPU, no barrier needed: the splits are already queued)."""
    gens = [m.forward_steps(x_lat, cam, t1000, cond) for m in models]
    world = len(models)
    arr = ctypes.c_uint64 * world
    while True:
        ks = [next(g, None) for g in gens]
        if all(k is None for k in ks):
            break
        if any(k is None for k in ks) or len(set(ks)) != 1:
            raise RuntimeError("ranks reached different exchange points")
        ptrs = arr(*[m.kv_set_ptr(ks[0]) for m in models])
        for m in models:
            m.gather(ptrs)
    return [m.chunk for m in models]


class SeqCfgSampler:
    """s-step CFG sampler over 2 x world ranks per image: the CFG branches on two groups of
    ``world`` query-row ranks.  The sampler state (latent | camera) is replicated on every
    rank; per step each rank's velocity rows are all-gathered over the image's ranks (one
    collective, ordered [branch 0 ranks, branch 1 ranks]) and every rank applies the same
    CFG combine + Euler update: the states stay identical and bitwise equal to the
    single-GPU batch-2 sampler."""

    def __init__(self, model: SeqShardedFlowModel, branch: int, image_group=None, steps: int = 20,
                 guidance: float = 3.0, shift: float = 3.0, exchange=None):
        import numpy as np
        import torch

        if model.B != 1:
            raise ValueError("each branch runs batch 1: build the model with batch=1")
        if branch not in (0, 1):
            raise ValueError("branch must be 0 (conditional) or 1 (unconditional)")
        self.model, self.branch, self.group, self.steps = model, branch, image_group, steps
        s, dev = model.spec, model.dev
        t1000, dt = sampler_schedule(steps, shift)
        f32 = dict(dtype=torch.float32, device=dev)
        self.t1000 = torch.from_numpy(t1000.astype(np.float32)).to(dev)
        self.dt = torch.from_numpy(dt).to(dev)
        self.g = torch.tensor([guidance], **f32)
        self.n_lat = s.latent_tokens * s.latent_dim
        self.n = self.n_lat + s.camera_dim
        self.x = torch.empty(self.n, **f32)
        self.x_lat = self.x[:self.n_lat].view(1, s.latent_tokens, s.latent_dim)
        self.x_cam = self.x[self.n_lat:].view(1, 1, s.camera_dim)
        self.cond = torch.empty(1, s.cond_tokens, s.cond_dim, **f32)
        W = model.world
        self.recv = torch.empty(2 * W, model.chunk.shape[1], **f32)
        self.t_cur = torch.empty(1, **f32)
        self.dt_cur = torch.empty(1, **f32)
        self._exchange = exchange or self._all_gather
        self.graph = None
        self.graph_stream = None

    def load(self, noise_lat, noise_cam, cond, neg_cond):
        self.x_lat.copy_(noise_lat.reshape(self.x_lat.shape), non_blocking=True)
        self.x_cam.copy_(noise_cam.reshape(self.x_cam.shape), non_blocking=True)
        c = cond if self.branch == 0 else neg_cond
        self.cond.copy_(c.reshape(self.cond.shape), non_blocking=True)
        self.model.precompute_condition(self.cond)  # once per image

    cached = True

    def refresh_condition(self):
        """Re-run the once-per-image condition path on the loaded condition tokens."""
        self.model.precompute_condition(self.cond)

    def _forward_body(self):
        self.model.forward_cached(self.x_lat, self.x_cam, self.t_cur)

    def _all_gather(self, send, recv):
        import torch.distributed as dist

        dist.all_gather_into_tensor(recv.view(-1), send, group=self.group)

    def forward_phase(self, i: int):
        self.t_cur.copy_(self.t1000[i:i + 1])
        self.dt_cur.copy_(self.dt[i:i + 1])
        if self.graph is not None:
            self.graph.replay()
        else:
            self._forward_body()

    def exchange_phase(self):
        self._exchange(self.model.chunk[0], self.recv)

    def update_phase(self):
        m, lib = self.model, self.model.lib
        W, cl = m.world, m.chunk_lat
        _native.use_current_stream(lib)
        parts = [(self.x[r * cl:(r + 1) * cl], self.recv[r, :cl], self.recv[W + r, :cl], cl) for r in range(W)]
        parts.append((self.x[self.n_lat:], self.recv[W - 1, cl:], self.recv[2 * W - 1, cl:],
                      self.n - self.n_lat))  # the camera entries (the row's padding is not read)
        for x, pos, neg, n in parts:
            st = lib.triposplat_b200_cfg_euler_update_f32(x.data_ptr(), pos.data_ptr(), neg.data_ptr(),
                                                          self.g.data_ptr(), self.dt_cur.data_ptr(), 1, n)
            if st:
                raise RuntimeError(f"sampler update returned status {st}")

    def velocity_pair(self, i: int):
        """Step i's [conditional, unconditional] velocities (latent [2, N, C], camera
        [2, 1, Cc]) assembled from the gathered rows, without updating the state."""
        import torch

        self.forward_phase(i)
        self.exchange_phase()
        m, s = self.model, self.model.spec
        W, cl = m.world, m.chunk_lat
        lat = torch.stack([torch.cat([self.recv[b * W + r, :cl] for r in range(W)]) for b in (0, 1)])
        cam = torch.stack([self.recv[b * W + W - 1, cl:cl + s.camera_dim] for b in (0, 1)])
        return lat.view(2, s.latent_tokens, s.latent_dim), cam.view(2, 1, s.camera_dim)

    def step(self, i: int):
        self.forward_phase(i)
        self.exchange_phase()
        self.update_phase()

    def run(self):
        for i in range(self.steps):
            self.step(i)
        return self.x_lat[0], self.x_cam[0]

    def prepare_capture(self):
        import torch

        self.graph_stream = torch.cuda.Stream(device=self.model.dev)
        self.graph_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.graph_stream):
            self._forward_body()
        self.graph_stream.synchronize()

    def record_graph(self):
        import torch

        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.graph_stream, capture_error_mode="relaxed"):
            self._forward_body()
        torch.cuda.current_stream().wait_stream(self.graph_stream)
        self.graph = graph
        return graph

    def capture(self):
        self.prepare_capture()
        return self.record_graph()

    @property
    def eager_launches_per_step(self) -> int:
        """Kernels launched per step outside the graph: the CFG + Euler update of each
        rank's latent rows and of the camera."""
        return self.model.world + 1
