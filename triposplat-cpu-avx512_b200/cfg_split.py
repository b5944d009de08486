"""CFG-pair split over two GPUs: one sampler per process, one velocity exchange per step.

The reference evaluates the conditional and the unconditional branch of classifier-free
guidance as the two halves of one batch (``triposplat_quantized_sampler.py:435-443``);
nothing inside the forward couples them, only the combine ``v = g*v_c - (g-1)*v_u`` and
the Euler update after it (``native_sampler_avx512.c:19-89``). ``CfgSplitSampler`` runs
each branch as a batch-1 ``FlowModelB200`` forward in its own process (rank 0 of the pair:
conditional, rank 1: unconditional). Per step the two velocity fields, latent and camera
packed into one flat fp32 buffer (8192 x 64 + 7 floats at the full configuration), are
exchanged with one all-gather, and both ranks apply the same CFG combine and Euler update
to the same data, so their states stay bitwise identical, and bitwise equal to the
batch-2 ``CfgEulerSampler`` (every kernel computes a row / head / batch entry
independently of the others).

A step is three phases so a test can interleave two samplers in one process:
``forward_phase`` (model forward, velocity packed into ``send``), ``exchange_phase``
(``recv = [send_rank0, send_rank1]``) and ``update_phase`` (combine + Euler on ``recv``).
"""
from __future__ import annotations

import numpy as np

import _native
from flow_model import FlowModelB200, sampler_schedule


class CfgSplitSampler:
    """s-step CFG flow sampler whose CFG pair is split across the two ranks of `group`."""

    def __init__(self, model: FlowModelB200, branch: int, group=None, steps: int = 20,
                 guidance: float = 3.0, shift: float = 3.0, exchange=None):
        import torch

        if model.B != 1:
            raise ValueError("CfgSplitSampler runs one branch per process: build the model with batch=1")
        if branch not in (0, 1):
            raise ValueError("branch must be 0 (conditional) or 1 (unconditional)")
        self.model, self.branch, self.group, self.steps = model, branch, group, steps
        s, dev = model.spec, model.dev
        t1000, dt = sampler_schedule(steps, shift)
        f32 = dict(dtype=torch.float32, device=dev)
        self.t1000 = torch.from_numpy(t1000.astype(np.float32)).to(dev)  # [K]
        self.dt = torch.from_numpy(dt).to(dev)                           # [K]
        self.g = torch.tensor([guidance], **f32)
        self.n_lat = s.latent_tokens * s.latent_dim
        self.n = self.n_lat + s.camera_dim
        # the state x (latent | camera) is one flat buffer; the model reads views of it
        self.x = torch.empty(self.n, **f32)
        self.x_lat = self.x[:self.n_lat].view(1, s.latent_tokens, s.latent_dim)
        self.x_cam = self.x[self.n_lat:].view(1, 1, s.camera_dim)
        self.cond = torch.empty(1, s.cond_tokens, s.cond_dim, **f32)
        self.send = torch.empty(self.n, **f32)
        self.recv = torch.empty(2, self.n, **f32)  # [conditional, unconditional]
        self.t_cur = torch.empty(1, **f32)
        self.dt_cur = torch.empty(1, **f32)
        self._exchange = exchange or self._all_gather
        self.graph = None
        self.graph_stream = None

    # -- phases --------------------------------------------------------------------------
    def load(self, noise_lat, noise_cam, cond, neg_cond):
        """Same inputs on both ranks; each keeps the condition of its own branch."""
        self.x_lat.copy_(noise_lat.reshape(self.x_lat.shape), non_blocking=True)
        self.x_cam.copy_(noise_cam.reshape(self.x_cam.shape), non_blocking=True)
        c = cond if self.branch == 0 else neg_cond
        self.cond.copy_(c.reshape(self.cond.shape), non_blocking=True)
        if self.cached:  # the branch's condition path, once per image
            self.model.precompute_condition(self.cond)

    @property
    def cached(self) -> bool:
        return getattr(self.model, "cond_planes", None) is not None

    def refresh_condition(self):
        """Re-run the once-per-image condition path on the loaded condition tokens."""
        if self.cached:
            self.model.precompute_condition(self.cond)

    def _forward_body(self):
        if self.cached:
            v_lat, v_cam = self.model.forward_cached(self.x_lat, self.x_cam, self.t_cur)
        else:
            v_lat, v_cam = self.model.forward(self.x_lat, self.x_cam, self.t_cur, self.cond)
        self.send[:self.n_lat].copy_(v_lat.reshape(-1))
        self.send[self.n_lat:].copy_(v_cam.reshape(-1))

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
        self._exchange(self.send, self.recv)

    def update_phase(self):
        lib = self.model.lib
        _native.use_current_stream(lib)
        st = lib.triposplat_b200_cfg_euler_update_f32(
            self.x.data_ptr(), self.recv[0].data_ptr(), self.recv[1].data_ptr(), self.g.data_ptr(),
            self.dt_cur.data_ptr(), 1, self.n)
        if st:
            raise RuntimeError(f"sampler update returned status {st}")

    def velocity_pair(self, i: int):
        """Step i's [conditional, unconditional] velocities (latent [2, N, C], camera
        [2, 1, Cc]) after the exchange, without updating the state."""
        self.forward_phase(i)
        self.exchange_phase()
        s = self.model.spec
        return (self.recv[:, :self.n_lat].reshape(2, s.latent_tokens, s.latent_dim),
                self.recv[:, self.n_lat:].reshape(2, 1, s.camera_dim))

    def step(self, i: int):
        self.forward_phase(i)
        self.exchange_phase()
        self.update_phase()

    def run(self):
        for i in range(self.steps):
            self.step(i)
        return self.x_lat[0], self.x_cam[0]

    # -- CUDA graph of the forward (the collective stays outside the graph) -----------------
    def prepare_capture(self):
        """One eager forward on the capture stream, so the library's workspace for that
        stream is sized before capture (nothing is allocated while capturing)."""
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

    # kernels launched per step outside the graph (the fused CFG combine + Euler update)
    eager_launches_per_step = 1
