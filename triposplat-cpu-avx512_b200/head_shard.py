"""Head-sharded (tensor-parallel) flow model: one rank per GPU, heads and MLP columns split.

The reference runs the whole block on one host (``native_block_elementwise_avx512_patch.py``
and ``triposplat_attention_patch.py:4978-5034``); on an 8-GPU box the block's work shards
by attention head and by MLP column.  With ``tp`` ranks each rank owns ``H / tp`` heads
and ``mlp / tp`` hidden columns:

* qkv, cross_q, cross_kv, fc1: column windows of the NF24 weight (the rank's heads' q / k /
  v columns, its MLP columns) through ``triposplat_b200_gemm_nf24_split_nk``; the
  attention (RoPE + RMSNorm fused, self and cross) runs on the rank's heads only.
* out, cross_out, fc2: input-feature windows of the weight -- the k-contiguous code planes
  offset by ``k0`` -- give a partial product over the rank's features; the bias is added on rank
  0 only, the partials are summed over the ranks by one all-reduce, and the (gated)
  residual add follows.
* embedders, adaLN and the final layer are replicated, so every rank holds the same
  residual stream ``x`` and ends with the same velocity.

Three reductions of the ``[B, L, hidden]`` residual update per block, either NCCL
all-reduces followed by the residual kernel, or (``reduce="peer"``) one fused kernel that
reads every rank's partial over NVLink and updates the residual.  ``forward_steps``
yields each partial buffer at its reduction point, so a single process can drive several
ranks in lockstep (the GPU parity tests); ``forward`` hands each one to ``all_reduce``
(NCCL over the tensor-parallel group by default).  The sum differs from the single-GPU
GEMM only in rounding (each rank splits its own activation window, and the partials are
added in the collective's order).
"""
from __future__ import annotations

import _native
from flow_model import FlowModelB200, FlowWeights, FlowSpec


def head_shard_plan(spec: FlowSpec, tp: int, rank: int) -> dict:
    """Windows of each block Linear that tensor-parallel rank `rank` of `tp` computes.

    Column windows (start, count) index the weight's output columns; row windows (k0, count)
    its input features.  qkv lists its q, k and v windows, cross_kv its k and v windows,
    in the slot order of the rank's [.., 3 | 2, heads, 64] attention inputs.
    """
    H, D, h, mlp = spec.heads, spec.head_dim, spec.hidden, spec.mlp
    if tp < 1 or H % tp or mlp % tp:
        raise ValueError(f"tensor-parallel size {tp} must divide heads {H} and mlp {mlp}")
    if not 0 <= rank < tp:
        raise ValueError(f"rank {rank} outside 0..{tp - 1}")
    hl = H // tp
    w, f = hl * D, mlp // tp
    if w % 16 or f % 16:
        raise ValueError("each rank's window must be a multiple of 16 columns")
    h0, f0 = rank * w, rank * f
    return {
        "heads": (rank * hl, hl),
        "width": w, "mlp_width": f,
        "qkv": [(h0, w), (h + h0, w), (2 * h + h0, w)],
        "cross_q": [(h0, w)],
        "cross_kv": [(h0, w), (h + h0, w)],
        "fc1": [(f0, f)],
        "out": (h0, w), "cross_out": (h0, w), "fc2": (f0, f),
    }


class PeerReduce:
    """Partial-product buffers shared across one tensor-parallel group through CUDA IPC.

    Every rank allocates two partial buffers (reduction points alternate between them) and
    a flag array, publishes their IPC handles with one object all-gather over `group`, and
    maps the other ranks' buffers.  ``reduce(point, x, mode, gate, ...)`` then runs the
    peer barrier and the fused reduce + residual kernel of the C-ABI on the current stream.
    """

    def __init__(self, lib, group, rank: int, world: int, numel: int):
        import ctypes

        import torch.distributed as dist

        self.lib, self.rank, self.world, self.group = lib, rank, world, group
        self.local, handles = [], []
        for nbytes in (4 * numel, 4 * numel, 64 * 4):
            ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
            st = lib.triposplat_b200_ipc_alloc(nbytes, ctypes.byref(ptr), h)
            if st:
                raise RuntimeError(f"ipc_alloc returned {st}")
            self.local.append(ptr.value)
            handles.append(bytes(h))
        allh = [None] * world
        dist.all_gather_object(allh, handles, group=group)
        self.opened = []
        mapped = []  # [rank][buffer] -> pointer in this process
        for r in range(world):
            if r == rank:
                mapped.append(list(self.local))
                continue
            row = []
            for h in allh[r]:
                ptr = ctypes.c_void_p()
                st = lib.triposplat_b200_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(h),
                                                   ctypes.byref(ptr))
                if st:
                    raise RuntimeError(f"ipc_open returned {st} for rank {r}")
                self.opened.append(ptr.value)
                row.append(ptr.value)
            mapped.append(row)
        arr = ctypes.c_uint64 * world
        self.parts = [arr(*[mapped[r][k] for r in range(world)]) for k in (0, 1)]
        self.flags = arr(*[mapped[r][2] for r in range(world)])
        import torch

        self.counter = torch.zeros(1, dtype=torch.int32, device=f"cuda:{torch.cuda.current_device()}")
        self.point = 0

    def part_ptr(self) -> int:
        """This rank's buffer for the next reduction point."""
        return self.local[self.point % 2]

    def reduce(self, x, mode: int, gate=None, gate_ld: int = 0, rows_per_batch: int = 1):
        lib = self.lib
        st = lib.triposplat_b200_peer_barrier(self.flags, self.rank, self.world,
                                              self.counter.data_ptr())
        if st:
            raise RuntimeError(f"peer_barrier returned {st}")
        rows, cols = x.numel() // x.shape[-1], int(x.shape[-1])
        st = lib.triposplat_b200_peer_reduce_residual_f32(
            self.parts[self.point % 2], self.world, x.data_ptr(), rows, cols, mode,
            None if gate is None else gate.data_ptr(), gate_ld, rows_per_batch)
        if st:
            raise RuntimeError(f"peer_reduce_residual returned {st}")
        self.point += 1

    def close(self):
        """Unmap the other ranks' buffers, wait for every rank to have done the same, then
        free this rank's (call with no work of the group in flight)."""
        import torch.distributed as dist

        for p in self.opened:
            self.lib.triposplat_b200_ipc_close(p)
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.local:
            self.lib.triposplat_b200_ipc_free(p)
        self.local = []


class HeadShardedFlowModel(FlowModelB200):
    """FlowModelB200 forward with the blocks sharded over `tp` ranks (rank `rank`).

    reduce="nccl": each row-window partial is summed by an NCCL all-reduce (or the
    caller's `all_reduce`), then the residual kernel runs; reduce="peer": the partials
    live in IPC-shared buffers and one fused kernel reads all ranks' partials over NVLink
    and updates the residual (``PeerReduce``)."""

    supports_condition_cache = False  # the cross K / V are column windows of this rank's heads

    def __init__(self, weights: FlowWeights, rank: int, tp: int, batch: int = 1,
                 device: str = "cuda", group=None, all_reduce=None, reduce: str = "nccl"):
        import torch

        if reduce == "peer" and (3 * weights.spec.blocks) % 2:
            # the two partial buffers alternate per reduction point, and a rank rewrites one
            # only after every rank has passed the next point's barrier; a forward (and so a
            # replayed CUDA graph of it) must hold an even number of points (3 per block) for
            # the alternation to carry on across forwards
            raise ValueError(f"reduce='peer' needs an even number of reduction points per forward "
                             f"(3 per block); {weights.spec.blocks} blocks give {3 * weights.spec.blocks}")
        super().__init__(weights, batch=batch, device=device, fused=True)
        s = self.spec
        self.rank, self.tp, self.group = rank, tp, group
        self.plan = pl = head_shard_plan(s, tp, rank)
        self.all_reduce = all_reduce or self._nccl_all_reduce
        if reduce not in ("nccl", "peer"):
            raise ValueError("reduce must be 'nccl' or 'peer'")
        self.peer = None
        if reduce == "peer":
            _native.use_current_stream(self.lib)
            self.peer = PeerReduce(self.lib, group, rank, tp, batch * s.seq * s.hidden)
        hs, hl = pl["heads"]
        w, f = pl["width"], pl["mlp_width"]
        B, L, h, Mc = batch, s.seq, s.hidden, s.cond_tokens
        f32 = dict(dtype=torch.float32, device=device)
        e = torch.empty
        self.buf.update({
            "qkv_l": e(B, L, 3 * w, **f32), "yq_l": e(B, L, w, **f32),
            "ckv_l": e(B, Mc, 2 * w, **f32), "part": e(B, L, h, **f32),
        })
        for name, k in (("sp_o", w), ("sp_hid_l", f)):
            nbytes = int(self.lib.triposplat_b200_split_bytes(B * L, k))
            self.buf[name] = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        # the rank's heads of the RoPE table and of the per-head gammas
        self.freqs_l = self.freqs[:, :, hs:hs + hl].contiguous()
        self.gammas_l = {k: v[hs:hs + hl].contiguous() for k, v in weights.params.items()
                         if k.endswith("_gamma")}
        # the bias of a row-window partial is added once, on rank 0
        self.zero_bias = torch.zeros(h, **f32)

    # -- GEMM windows ----------------------------------------------------------------------
    def _lin_cols(self, name, split, rows, out_ptr, start, count, stride_out, mode=0):
        p = self.w.linears[name]
        c, q = self.nk[name]
        N, K = int(c.shape[0]), int(c.shape[1])
        self._ok(self.lib.triposplat_b200_gemm_nf24_split_nk(
            split, rows, K, c.data_ptr(), q.data_ptr(), K, p.scale.data_ptr(),
            p.bias.data_ptr(), out_ptr, N, start, count, stride_out, mode, None, 0, 1),
            f"gemm columns {name}")

    def _lin_rows(self, name, split, rows, k0, count, out_ptr):
        """Partial product over input features [k0, k0 + count) into out [rows, N]."""
        p = self.w.linears[name]
        c, q = self.nk[name]
        N, K = int(c.shape[0]), int(c.shape[1])
        bias = p.bias if self.rank == 0 else self.zero_bias
        self._ok(self.lib.triposplat_b200_gemm_nf24_split_nk(
            split, rows, count, c.data_ptr() + 2 * k0, q.data_ptr() + k0, K,
            p.scale.data_ptr(), bias.data_ptr(), out_ptr, N, 0, N, N, 0, None, 0, 1),
            f"gemm rows {name}")

    def _part_ptr(self):
        return self.buf["part"].data_ptr() if self.peer is None else self.peer.part_ptr()

    def _reduce_into_x(self, mode, gate=None):
        """Sum the ranks' partials into the residual stream: x += gate * sum (mode 2) or
        x += sum (mode 3).  A generator: the NCCL path yields the partial at the reduction
        point (see forward_steps); the peer path reduces in place and yields nothing."""
        x, h, L = self.buf["x"], self.spec.hidden, self.spec.seq
        if self.peer is not None:
            self.peer.reduce(x, mode, gate, h, L)
            return
        part = self.buf["part"]
        yield part
        if mode == 2:
            self._gated(x, part, gate)
        else:
            self._add(x, part)

    def _nccl_all_reduce(self, t):
        import torch.distributed as dist

        dist.all_reduce(t, group=self.group)

    # -- forward ---------------------------------------------------------------------------
    def forward(self, x_lat, cam, t1000, cond):
        for part in self.forward_steps(x_lat, cam, t1000, cond):
            self.all_reduce(part)
        return self.buf["v_lat"], self.buf["v_cam"]

    def forward_steps(self, x_lat, cam, t1000, cond):
        """The forward as a generator: yields the partial buffer at each reduction point
        and continues once the caller has replaced it by the sum over the ranks."""
        self._embed(x_lat, cam, t1000, cond)
        for i in range(self.spec.blocks):
            yield from self._block_sharded(i)
        self._final_layer()

    def _block_sharded(self, i):
        s, b, lib, pl = self.spec, self.buf, self.lib, self.plan
        B, L, Mc = self.B, s.seq, s.cond_tokens
        hl, w = pl["heads"][1], pl["width"]
        rows = B * L
        p = f"blocks.{i}."
        g = self.gammas_l
        m = b["mod_i"]
        m.copy_(b["mod"])
        self._add(m, self.tables[i])
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (m[j] for j in range(6))
        x = b["x"]
        sph, spo, sphid = self._split_ptr("sp_h"), self._split_ptr("sp_o"), self._split_ptr("sp_hid_l")
        # self-attention over this rank's heads
        self._ln_split(x, sph, shift_msa, scale_msa)
        qkv = b["qkv_l"]
        for j, (c0, n) in enumerate(pl["qkv"]):
            self._lin_cols(p + "qkv", sph, rows, qkv.data_ptr() + 4 * j * w, c0, n, 3 * w)
        self._ok(lib.triposplat_b200_qkv_rope_rmsnorm_sdpa_split(
            qkv.data_ptr(), self.freqs_l.data_ptr(), g[p + "q_gamma"].data_ptr(),
            g[p + "k_gamma"].data_ptr(), B, L, hl, 1, spo), "self_attention")
        self._lin_rows(p + "out", spo, rows, *pl["out"], self._part_ptr())
        yield from self._reduce_into_x(2, gate_msa)
        # cross-attention over this rank's heads
        self._ln_split(x, sph)
        (c0, n), = pl["cross_q"]
        self._lin_cols(p + "cross_q", sph, rows, b["yq_l"].data_ptr(), c0, n, w)
        ckv = b["ckv_l"]
        for j, (c0, n) in enumerate(pl["cross_kv"]):
            self._lin_cols(p + "cross_kv", self._split_ptr("sp_c"), B * Mc,
                           ckv.data_ptr() + 4 * j * w, c0, n, 2 * w)
        self._ok(lib.triposplat_b200_q_kv_rmsnorm_sdpa_split(
            b["yq_l"].data_ptr(), ckv.data_ptr(), g[p + "cq_gamma"].data_ptr(),
            g[p + "ck_gamma"].data_ptr(), B, L, Mc, hl, spo), "cross_attention")
        self._lin_rows(p + "cross_out", spo, rows, *pl["cross_out"], self._part_ptr())
        yield from self._reduce_into_x(3)
        # MLP over this rank's hidden columns
        # (the bound over all fc1 columns holds for this rank's window)
        (c0, n), = pl["fc1"]
        self._ln_split(x, sph, shift_mlp, scale_mlp, bound=(sphid, n, self.gelu_bounds[i]))
        self._lin_cols(p + "fc1", sph, rows, sphid, c0, n, n, mode=4)
        self._lin_rows(p + "fc2", sphid, rows, *pl["fc2"], self._part_ptr())
        yield from self._reduce_into_x(2, gate_mlp)

    def close(self):
        """Release the IPC-shared buffers of the peer path (call before the process group
        goes away)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    # collectives per forward: three all-reduces per block
    def all_reduces_per_forward(self) -> int:
        return 3 * self.spec.blocks


def run_lockstep(models, x_lat, cam, t1000, cond):
    """Drive the ranks' forwards in one process, summing the partials in rank order at
    each reduction point (the one-GPU stand-in for the all-reduce)."""
    gens = [m.forward_steps(x_lat, cam, t1000, cond) for m in models]
    while True:
        parts = [next(g, None) for g in gens]
        if all(pt is None for pt in parts):
            break
        if any(pt is None for pt in parts):
            raise RuntimeError("ranks reached different numbers of reduction points")
        total = parts[0].clone()
        for pt in parts[1:]:
            total += pt
        for pt in parts:
            pt.copy_(total)
    return [(m.buf["v_lat"], m.buf["v_cam"]) for m in models]
