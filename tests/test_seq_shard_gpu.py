"""Query-row (sequence) sharded flow model on the GPU against the unsharded forward.

Every token row sees the arithmetic of the single-GPU model (same split planes, key tiles,
query tiles, warps and orders), so the comparison is BITWISE:
(1) all ranks driven in lockstep by one process on one GPU (2 and 4 ranks, batch 1),
    the ranks' velocity rows concatenated against FlowModelB200.forward;
(2) two processes on two GPUs exchanging key tiles over NVLink peer memory (peer barrier +
    pull-gather kernel), a forward run twice through the alternating plane sets;
(3) the CFG split with two query-row ranks per branch on four GPUs, three sampler steps
    eager and three replayed from a CUDA graph, against the single-GPU batch-2 sampler.
(2) and (3) are skipped when fewer GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _spec():
    from flow_model import FlowSpec

    return FlowSpec(blocks=2)


def _inputs(spec, batch, device, seed=31):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(batch, spec.latent_tokens, spec.latent_dim, generator=g)
    cam = torch.randn(batch, 1, spec.camera_dim, generator=g)
    t = torch.tensor([700.0, 700.0][:batch])
    cond = torch.randn(batch, spec.cond_tokens, spec.cond_dim, generator=g)
    return [x.to(device) for x in (lat, cam, t, cond)]


def _assemble(chunks, spec, world):
    """Per-rank chunks [B, n_lat/world + cam (+ padding)] -> latent [B, Nl, C] and camera
    [B, 1, Cc]."""
    cl = (spec.latent_tokens // world) * spec.latent_dim
    lat = torch.cat([c[:, :cl] for c in chunks], dim=1).view(-1, spec.latent_tokens, spec.latent_dim)
    return lat, chunks[-1][:, cl:cl + spec.camera_dim].reshape(-1, 1, spec.camera_dim)


@pytest.mark.parametrize("world,batch", [(2, 1), (4, 1)])
def test_seq_shard_lockstep_one_gpu_bitwise(world, batch):
    from flow_model import FlowModelB200, make_weights
    from seq_shard import SeqShardedFlowModel, run_lockstep

    spec = _spec()
    w = make_weights(spec, seed=13, device="cuda")
    inp = _inputs(spec, batch, "cuda")
    ref_lat, ref_cam = (t.clone() for t in FlowModelB200(w, batch=batch).forward(*inp))
    models = [SeqShardedFlowModel(w, rank=r, world=world, batch=batch, exchange="lockstep")
              for r in range(world)]
    chunks = run_lockstep(models, *inp)
    torch.cuda.synchronize()
    lat, cam = _assemble(chunks, spec, world)
    assert bool(torch.isfinite(lat).all())
    assert torch.equal(lat, ref_lat) and torch.equal(cam, ref_cam)


def test_row_entries_reject_bad_ranges():
    import ctypes

    import _native

    lib = _native.load()
    buf = torch.zeros(1 << 20, device="cuda")
    p = buf.data_ptr()
    f = lib.triposplat_b200_qkv_split_rows_f32
    assert f(p, p, p, p, 1, 300, 2, 64, 200, 1, p, p) == -3     # t0 not a tile start
    assert f(p, p, p, p, 1, 300, 2, 0, 200, 1, p, p) == -3      # t1 neither a tile end nor L
    assert f(p, p, p, p, 1, 300, 2, 0, 301, 1, p, p) == -3      # past L
    assert f(p, p, p, p, 1, 300, 2, 0, 128, 2, p, p) == -2      # frequency batches
    starts = (ctypes.c_int * 3)(0, 100, 300)
    ptrs = (ctypes.c_uint64 * 2)(p, p)
    assert lib.triposplat_b200_kv_planes_gather(ptrs, starts, 2, 0, 2, 300) == -3
    starts = (ctypes.c_int * 3)(0, 128, 299)
    assert lib.triposplat_b200_kv_planes_gather(ptrs, starts, 2, 0, 2, 300) == -3
    assert lib.triposplat_b200_kv_planes_gather(ptrs, starts, 9, 0, 2, 300) == -2
    assert lib.triposplat_b200_attend_rows_f32(p + 16, p, p, 1, 2, 64, 300) == -4
    assert lib.triposplat_b200_status() == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_init(rank, world, port):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _sp_worker(rank, port, out_dir):
    import torch.distributed as dist

    _nccl_init(rank, 2, port)
    try:
        from flow_model import FlowModelB200, make_weights
        from seq_shard import SeqShardedFlowModel

        dev = f"cuda:{rank}"
        spec = _spec()
        w = make_weights(spec, seed=13, device=dev)
        inp = _inputs(spec, 2, dev)
        m = SeqShardedFlowModel(w, rank=rank, world=2, batch=2, device=dev, group=dist.group.WORLD)
        first = m.forward(*inp).clone()
        second = m.forward(*inp).clone()  # the next forward reuses the alternating plane sets
        torch.cuda.synchronize(dev)
        out = {"chunk": first.cpu().numpy(), "chunk2": second.cpu().numpy(),
               "status": int(m.lib.triposplat_b200_status())}
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
def test_seq_shard_two_gpus_peer_exchange_bitwise(tmp_path):
    import torch.multiprocessing as mp

    spec = _spec()
    mp.spawn(_sp_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"rank{k}.npz") for k in (0, 1)]
    assert all(int(x["status"]) == 0 for x in r)
    for x in r:
        assert np.array_equal(x["chunk"], x["chunk2"])
    lat, cam = _assemble([torch.from_numpy(x["chunk"]) for x in r], spec, 2)
    assert np.array_equal(lat.numpy(), r[0]["ref_lat"]) and np.array_equal(cam.numpy(), r[0]["ref_cam"])


def _cfg_sp_worker(rank, port, out_dir):
    import torch.distributed as dist

    _nccl_init(rank, 4, port)
    try:
        from flow_model import CfgEulerSampler, FlowModelB200, make_weights
        from seq_shard import SeqCfgSampler, SeqShardedFlowModel

        dev = f"cuda:{rank}"
        spec = _spec()
        w = make_weights(spec, seed=13, device=dev)
        # ranks {0, 1}: conditional branch, {2, 3}: unconditional; query-row groups per branch
        sp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
        branch, sp_rank = rank // 2, rank % 2
        model = SeqShardedFlowModel(w, rank=sp_rank, world=2, batch=1, device=dev,
                                    group=sp_groups[branch])
        g = torch.Generator().manual_seed(4)
        lat = torch.randn(1, spec.latent_tokens, spec.latent_dim, generator=g).to(dev)
        cam = torch.randn(1, 1, spec.camera_dim, generator=g).to(dev)
        cond = torch.randn(1, spec.cond_tokens, spec.cond_dim, generator=g).to(dev)
        neg = torch.zeros_like(cond)
        s = SeqCfgSampler(model, branch=branch, image_group=dist.group.WORLD, steps=3)
        s.load(lat, cam, cond, neg)
        e_lat, e_cam = (t.clone() for t in s.run())
        s.load(lat, cam, cond, neg)
        s.capture()
        s.load(lat, cam, cond, neg)
        g_lat, g_cam = (t.clone() for t in s.run())
        torch.cuda.synchronize(dev)
        out = {"lat": e_lat.cpu().numpy(), "cam": e_cam.cpu().numpy(), "glat": g_lat.cpu().numpy(),
               "gcam": g_cam.cpu().numpy(), "status": int(model.lib.triposplat_b200_status())}
        if rank == 0:
            ref = CfgEulerSampler(FlowModelB200(w, batch=2, device=dev), steps=3)
            ref.load(lat, cam, cond, neg)
            r_lat, r_cam = ref.run()
            out["ref_lat"], out["ref_cam"] = r_lat.cpu().numpy(), r_cam.cpu().numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        s.graph = None
        torch.cuda.synchronize(dev)
        dist.barrier()
        model.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_cfg_split_with_query_rows_four_gpus_bitwise(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_cfg_sp_worker, args=(_free_port(), str(tmp_path)), nprocs=4, join=True)
    rs = [np.load(tmp_path / f"rank{r}.npz") for r in range(4)]
    for r in rs:
        assert int(r["status"]) == 0
        assert np.array_equal(r["lat"], rs[0]["ref_lat"]) and np.array_equal(r["cam"], rs[0]["ref_cam"])
        assert np.array_equal(r["glat"], r["lat"]) and np.array_equal(r["gcam"], r["cam"])
