"""Head-sharded model on the GPU against the unsharded forward.

The sharded forward changes only rounding (each rank splits its own activation window into
the GEMM's fp16 hi/lo operands, and the partial products are summed across ranks), so its
velocities must match the single-GPU forward to a relative RMS error far below the 1e-4
end-of-sampling budget: REL_RMSE = 1e-5 here.  Checked (1) with all ranks driven in lockstep
by one process on one GPU (partials summed in rank order), at 2 / 4 / 8 ranks, and (2) as
two processes on two GPUs reducing over NCCL and over NVLink peer memory (the fused
reduce + residual kernel), and (3) the CFG split combined with head sharding (peer
reduction) as four processes on four GPUs, against the batch-2 sampler (each skipped when
fewer GPUs are visible).
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_RMSE = 1e-5


def _spec():
    from flow_model import FlowSpec

    return FlowSpec(blocks=2)


def _inputs(spec, batch, device, seed=21):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(batch, spec.latent_tokens, spec.latent_dim, generator=g)
    cam = torch.randn(batch, 1, spec.camera_dim, generator=g)
    t = torch.tensor([700.0, 300.0][:batch])
    cond = torch.randn(batch, spec.cond_tokens, spec.cond_dim, generator=g)
    return [x.to(device) for x in (lat, cam, t, cond)]


def _rel_rmse(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / max(1e-30, np.sqrt(np.mean(b ** 2))))


@pytest.mark.parametrize("tp,batch", [(2, 2), (4, 1), (8, 1)])
def test_head_shard_lockstep_one_gpu(tp, batch):
    from flow_model import FlowModelB200, make_weights
    from head_shard import HeadShardedFlowModel, run_lockstep

    spec = _spec()
    w = make_weights(spec, seed=9, device="cuda")
    inp = _inputs(spec, batch, "cuda")
    ref = [t.cpu().numpy() for t in FlowModelB200(w, batch=batch).forward(*inp)]
    models = [HeadShardedFlowModel(w, rank=r, tp=tp, batch=batch) for r in range(tp)]
    outs = run_lockstep(models, *inp)
    torch.cuda.synchronize()
    lat0, cam0 = (t.cpu().numpy() for t in outs[0])
    for lat, cam in outs[1:]:  # every rank ends with the same velocity
        assert np.array_equal(lat.cpu().numpy(), lat0) and np.array_equal(cam.cpu().numpy(), cam0)
    assert np.isfinite(lat0).all() and np.isfinite(cam0).all()
    assert _rel_rmse(lat0, ref[0]) < REL_RMSE, _rel_rmse(lat0, ref[0])
    assert _rel_rmse(cam0, ref[1]) < REL_RMSE, _rel_rmse(cam0, ref[1])


def test_range_entry_rejects_bad_windows():
    import _native
    from flow_model import make_weights

    spec = _spec()
    w = make_weights(spec, seed=9, device="cuda").linears["blocks.0.qkv"]
    lib = _native.load()
    K, N = int(w.code01.shape[0]), int(w.code01.shape[1])
    rows = 64
    split = torch.zeros(int(lib.triposplat_b200_split_bytes(rows, K)) + 256, dtype=torch.uint8,
                        device="cuda")
    sp = (split.data_ptr() + 255) & ~255
    out = torch.empty(rows, N, device="cuda")
    call = lambda start, count, stride: lib.triposplat_b200_gemm_nf24_split_range(  # noqa: E731
        sp, rows, K, w.code01.data_ptr(), w.q2.data_ptr(), w.scale.data_ptr(), w.bias.data_ptr(),
        out.data_ptr(), N, start, count, stride, 0, None, 0, 1)
    assert call(N - 16, 32, 32) != 0      # window past the last column
    assert call(8, 16, 16) != 0           # start not a multiple of 16
    assert call(0, 64, 32) != 0           # row stride shorter than the window
    assert call(16, 64, 64) == 0
    torch.cuda.synchronize()


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _nccl_init(rank, world, port):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _tp_worker(rank, port, out_dir):
    import torch.distributed as dist

    _nccl_init(rank, 2, port)
    try:
        from flow_model import FlowModelB200, make_weights
        from head_shard import HeadShardedFlowModel

        dev = f"cuda:{rank}"
        spec = _spec()
        w = make_weights(spec, seed=9, device=dev)
        inp = _inputs(spec, 2, dev)
        lat, cam = HeadShardedFlowModel(w, rank=rank, tp=2, batch=2, device=dev).forward(*inp)
        torch.cuda.synchronize(dev)
        out = {"lat": lat.cpu().numpy(), "cam": cam.cpu().numpy()}
        if rank == 0:
            ref = FlowModelB200(w, batch=2, device=dev).forward(*inp)
            out["ref_lat"], out["ref_cam"] = (t.cpu().numpy() for t in ref)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_shard_two_gpus_nccl(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_tp_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in (0, 1))
    assert np.array_equal(r0["lat"], r1["lat"]) and np.array_equal(r0["cam"], r1["cam"])
    assert _rel_rmse(r0["lat"], r0["ref_lat"]) < REL_RMSE
    assert _rel_rmse(r0["cam"], r0["ref_cam"]) < REL_RMSE


def _cfg_tp_worker(rank, port, out_dir):
    import torch.distributed as dist

    _nccl_init(rank, 4, port)
    try:
        from cfg_split import CfgSplitSampler
        from flow_model import CfgEulerSampler, FlowModelB200, make_weights
        from head_shard import HeadShardedFlowModel

        dev = f"cuda:{rank}"
        spec = _spec()
        w = make_weights(spec, seed=9, device=dev)
        # ranks {0, 1}: conditional branch, {2, 3}: unconditional; pairs {0, 2}, {1, 3}
        tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
        pair_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
        branch, tp_rank = rank // 2, rank % 2
        model = HeadShardedFlowModel(w, rank=tp_rank, tp=2, batch=1, device=dev,
                                     group=tp_groups[branch], reduce="peer")
        s = CfgSplitSampler(model, branch=branch, group=pair_groups[tp_rank], steps=3)
        g = torch.Generator().manual_seed(4)
        lat = torch.randn(1, spec.latent_tokens, spec.latent_dim, generator=g).to(dev)
        cam = torch.randn(1, 1, spec.camera_dim, generator=g).to(dev)
        cond = torch.randn(1, spec.cond_tokens, spec.cond_dim, generator=g).to(dev)
        neg = torch.zeros_like(cond)
        s.load(lat, cam, cond, neg)
        x_lat, x_cam = s.run()
        torch.cuda.synchronize(dev)
        out = {"lat": x_lat.cpu().numpy(), "cam": x_cam.cpu().numpy()}
        if rank == 0:
            ref = CfgEulerSampler(FlowModelB200(w, batch=2, device=dev), steps=3)
            ref.load(lat, cam, cond, neg)
            r_lat, r_cam = ref.run()
            out["ref_lat"], out["ref_cam"] = r_lat.cpu().numpy(), r_cam.cpu().numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        dist.barrier()
        model.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_cfg_split_with_head_shard_four_gpus(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_cfg_tp_worker, args=(_free_port(), str(tmp_path)), nprocs=4, join=True)
    rs = [np.load(tmp_path / f"rank{r}.npz") for r in range(4)]
    for r in rs[1:]:
        assert np.array_equal(r["lat"], rs[0]["lat"]) and np.array_equal(r["cam"], rs[0]["cam"])
    assert _rel_rmse(rs[0]["lat"], rs[0]["ref_lat"]) < REL_RMSE
    assert _rel_rmse(rs[0]["cam"], rs[0]["ref_cam"]) < REL_RMSE


def test_peer_reduce_kernel_one_gpu():
    """The fused reduce + residual kernel over T partial buffers (here all on one GPU, no
    barrier): x += gate[b] * (p0 + p1 + p2) summed in rank order, and x += sum."""
    import ctypes

    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    g = torch.Generator().manual_seed(6)
    B, L, C, T = 2, 37, 64, 3
    parts = [torch.randn(B * L, C, generator=g).cuda() for _ in range(T)]
    ptrs = (ctypes.c_uint64 * T)(*[p.data_ptr() for p in parts])
    gate = torch.randn(B, C, generator=g).cuda()
    x0 = torch.randn(B * L, C, generator=g).cuda()
    s = parts[0] + parts[1] + parts[2]
    x = x0.clone()
    assert lib.triposplat_b200_peer_reduce_residual_f32(ptrs, T, x.data_ptr(), B * L, C, 2,
                                                        gate.data_ptr(), C, L) == 0
    ref = torch.addcmul(x0, gate.repeat_interleave(L, 0), s)
    torch.cuda.synchronize()
    assert torch.equal(x, ref)
    x = x0.clone()
    assert lib.triposplat_b200_peer_reduce_residual_f32(ptrs, T, x.data_ptr(), B * L, C, 3,
                                                        None, 0, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(x, x0 + s)
    assert lib.triposplat_b200_peer_reduce_residual_f32(ptrs, T, x.data_ptr(), B * L, 62, 3,
                                                        None, 0, 1) == -4
    assert lib.triposplat_b200_peer_reduce_residual_f32(ptrs, 9, x.data_ptr(), B * L, C, 3,
                                                        None, 0, 1) == -2


def test_peer_barrier_times_out_and_reports():
    """A barrier whose peer never signals gives up after its 2 s budget and reports through
    the status word; the context stays usable."""
    import ctypes

    import _native

    lib = _native.load()
    _native.use_current_stream(lib)
    flags = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    ptrs = (ctypes.c_uint64 * 2)(*[f.data_ptr() for f in flags])
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.triposplat_b200_status() == 0
    assert lib.triposplat_b200_peer_barrier(ptrs, 0, 2, counter.data_ptr()) == 0
    torch.cuda.synchronize()
    assert lib.triposplat_b200_status() != 0      # rank 1's slot never reached the epoch
    assert int(flags[1][0]) == 1 and int(flags[0][0]) == 1  # our own signal went out
    lib.triposplat_b200_clear_status()
    assert lib.triposplat_b200_status() == 0
    y = torch.ones(4, device="cuda") * 2          # the context still runs work
    assert float(y.sum()) == 8.0


def _peer_worker(rank, port, out_dir):
    import torch.distributed as dist

    _nccl_init(rank, 2, port)
    try:
        from flow_model import FlowModelB200, make_weights
        from head_shard import HeadShardedFlowModel

        dev = f"cuda:{rank}"
        spec = _spec()
        w = make_weights(spec, seed=9, device=dev)
        inp = _inputs(spec, 2, dev)
        m = HeadShardedFlowModel(w, rank=rank, tp=2, batch=2, device=dev,
                                 group=dist.group.WORLD, reduce="peer")
        lat, cam = m.forward(*inp)
        lat2, cam2 = (t.clone() for t in m.forward(*inp))  # second pass: buffers reused
        torch.cuda.synchronize(dev)
        out = {"lat": lat.cpu().numpy(), "cam": cam.cpu().numpy(), "lat2": lat2.cpu().numpy()}
        if rank == 0:
            ref = FlowModelB200(w, batch=2, device=dev).forward(*inp)
            out["ref_lat"], out["ref_cam"] = (t.cpu().numpy() for t in ref)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        dist.barrier()
        m.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_shard_two_gpus_peer_reduce(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_peer_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in (0, 1))
    assert np.array_equal(r0["lat"], r1["lat"]) and np.array_equal(r0["cam"], r1["cam"])
    assert np.array_equal(r0["lat"], r0["lat2"])
    assert _rel_rmse(r0["lat"], r0["ref_lat"]) < REL_RMSE
    assert _rel_rmse(r0["cam"], r0["ref_cam"]) < REL_RMSE
