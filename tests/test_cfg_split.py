"""CFG-pair split, host side: two gloo ranks on CPU.

Each rank runs `CfgSplitSampler` for its branch with a stand-in model (a fixed,
branch-sensitive function of the state, timestep and condition) and a torch restatement of
the combine / Euler update, so only the sampler's own logic is exercised here: branch
assignment, the flat latent|camera packing, the all-gather order, and that both ranks end
in the same state as the batch-2 sampler arithmetic (numpy, float32 steps).
The CUDA path of the same class is covered by tests/test_cfg_split_gpu.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

STEPS, G, SHIFT = 4, 3.0, 3.0


class _StandInModel:
    """Deterministic stand-in with FlowModelB200's interface (batch 1, CPU tensors)."""

    def __init__(self, spec):
        self.spec, self.B, self.dev, self.lib = spec, 1, "cpu", None

    def forward(self, x_lat, x_cam, t1000, cond):
        c = cond.mean()
        v_lat = torch.sin(x_lat * 0.7 + t1000[0] * 1e-3) + c
        v_cam = torch.cos(x_cam * 1.3) - c * t1000[0] * 1e-3
        return v_lat, v_cam


def _np_forward(x_lat, x_cam, t, cond):
    c = np.float32(cond.mean(dtype=np.float32))
    v_lat = np.sin(x_lat * np.float32(0.7) + np.float32(t * 1e-3)) + c
    v_cam = np.cos(x_cam * np.float32(1.3)) - c * np.float32(t * 1e-3)
    return v_lat.astype(np.float32), v_cam.astype(np.float32)


def _inputs(spec):
    g = torch.Generator().manual_seed(3)
    lat = torch.randn(1, spec.latent_tokens, spec.latent_dim, generator=g)
    cam = torch.randn(1, 1, spec.camera_dim, generator=g)
    cond = torch.randn(1, spec.cond_tokens, spec.cond_dim, generator=g)
    neg = torch.zeros_like(cond) + 0.25
    return lat, cam, cond, neg


def _worker(rank, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from cfg_split import CfgSplitSampler
        from flow_model import FlowSpec

        spec = FlowSpec.small()

        def exchange(send, recv):  # gloo has no all_gather_into_tensor: same order, list form
            parts = [torch.empty_like(send) for _ in range(2)]
            dist.all_gather(parts, send)
            recv.copy_(torch.stack(parts))

        class CpuSampler(CfgSplitSampler):
            def update_phase(self):
                v = self.g * self.recv[0] - (self.g - 1.0) * self.recv[1]
                self.x.sub_(self.dt_cur * v)

        s = CpuSampler(_StandInModel(spec), branch=rank, steps=STEPS, guidance=G, shift=SHIFT,
                       exchange=exchange)
        s.load(*_inputs(spec))
        lat, cam = s.run()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), lat=lat.numpy(), cam=cam.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def test_cfg_split_two_gloo_ranks_match_batch2_arithmetic(tmp_path):
    from flow_model import FlowSpec, sampler_schedule

    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in (0, 1))
    # both ranks end in the same state
    assert np.array_equal(r0["lat"], r1["lat"]) and np.array_equal(r0["cam"], r1["cam"])
    # ... which is the batch-2 CFG / Euler recurrence
    spec = FlowSpec.small()
    lat, cam, cond, neg = (t.numpy() for t in _inputs(spec))
    t1000, dt = sampler_schedule(STEPS, SHIFT)
    x_lat, x_cam = lat[0].copy(), cam[0].copy()
    for i in range(STEPS):
        vc = _np_forward(x_lat, x_cam, t1000[i], cond)
        vu = _np_forward(x_lat, x_cam, t1000[i], neg)
        for x, a, b in ((x_lat, vc[0], vu[0]), (x_cam, vc[1], vu[1])):
            v = np.float32(G) * a - np.float32(G - 1.0) * b
            x -= dt[i] * v
    np.testing.assert_allclose(r0["lat"], x_lat, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r0["cam"], x_cam, rtol=1e-5, atol=1e-5)


def test_cfg_split_rejects_batch2_model():
    from cfg_split import CfgSplitSampler
    from flow_model import FlowSpec

    m = _StandInModel(FlowSpec.small())
    m.B = 2
    with pytest.raises(ValueError):
        CfgSplitSampler(m, branch=0)
    m.B = 1
    with pytest.raises(ValueError):
        CfgSplitSampler(m, branch=2)
