"""Head sharding, host side: the window plan and its arithmetic on two gloo ranks (CPU).

`head_shard_plan` must tile every block Linear exactly (column windows for qkv / cross_q /
cross_kv / fc1, row windows for out / cross_out / fc2), and a block computed from those
windows -- per-rank heads, partial products with the bias on rank 0, summed by an
all-reduce -- must equal the unsharded block.  The block here is a float64 torch
restatement with dense weights (the sharding is independent of the NF24 quantisation);
the CUDA path of the same plan is covered by tests/test_head_shard_gpu.py.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _spec():
    from flow_model import FlowSpec

    return FlowSpec(blocks=1, hidden=256, heads=4, mlp=512, grid=(2, 2, 4), latent_dim=16,
                    camera_dim=7, cond_tokens=9, cond_dim=32, t_freq=32)


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_plan_tiles_every_linear(tp):
    from head_shard import head_shard_plan

    s = _spec()
    h, mlp = s.hidden, s.mlp
    plans = [head_shard_plan(s, tp, r) for r in range(tp)]
    for name, n in (("qkv", 3 * h), ("cross_q", h), ("cross_kv", 2 * h), ("fc1", mlp)):
        cols = sorted(c for pl in plans for (c0, k) in pl[name] for c in range(c0, c0 + k))
        assert cols == list(range(n)), name
    for name, k in (("out", h), ("cross_out", h), ("fc2", mlp)):
        rows = sorted(r for pl in plans for r in range(pl[name][0], pl[name][0] + pl[name][1]))
        assert rows == list(range(k)), name
    heads = sorted(hh for pl in plans for hh in range(pl["heads"][0], sum(pl["heads"])))
    assert heads == list(range(s.heads))
    # q / k / v windows of one rank are the same heads of the three planes
    for pl in plans:
        starts = [c0 for c0, _ in pl["qkv"]]
        assert starts[1] - starts[0] == h and starts[2] - starts[1] == h


def test_plan_rejects_bad_sizes():
    from head_shard import head_shard_plan

    s = _spec()
    with pytest.raises(ValueError):
        head_shard_plan(s, 3, 0)        # 4 heads do not split three ways
    with pytest.raises(ValueError):
        head_shard_plan(s, 2, 2)        # rank outside the group
    with pytest.raises(ValueError):
        head_shard_plan(s, 8, 0)        # 4 heads do not split eight ways
    with pytest.raises(ValueError):      # 24-column MLP windows are not multiples of 16
        head_shard_plan(type(s)(heads=4, hidden=256, mlp=96), 4, 0)


# -- float64 restatement of one block -------------------------------------------------------
def _weights(s, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = s.hidden
    r = lambda *shape: torch.randn(*shape, generator=g, dtype=torch.float64)  # noqa: E731
    W = {name: (r(n, k) * 0.05, r(n) * 0.01) for name, k, n in
         (("qkv", h, 3 * h), ("out", h, h), ("cross_q", h, h), ("cross_kv", h, 2 * h),
          ("cross_out", h, h), ("fc1", h, s.mlp), ("fc2", s.mlp, h))}
    G = {k: 1.0 + 0.02 * r(s.heads, s.head_dim) for k in ("q", "k", "cq", "ck")}
    mod = r(6, h) * 0.1
    return W, G, mod


def _ln(x, eps=1e-6):
    mu = x.mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(((x - mu) ** 2).mean(-1, keepdim=True) + eps)


def _rope_rms(t, cs, gamma):  # t [L, hl, 64], cs [L, hl, 32, 2]
    a, b = t[..., 0::2], t[..., 1::2]
    c, sn = cs[..., 0], cs[..., 1]
    r = torch.stack([a * c - b * sn, a * sn + b * c], -1).reshape(t.shape)
    n = torch.linalg.vector_norm(r, dim=-1, keepdim=True).clamp_min(1e-12)
    return r * 8.0 / n * gamma


def _attn(q, k, v):  # [L, hl, 64]
    s = torch.einsum("qhd,khd->hqk", q, k) / 8.0
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)


def _block(x, c, cs, W, G, mod, plan=None, reduce=lambda t: t, rank=0):
    """One block; with `plan`, only that rank's windows and an all-reduce `reduce`."""
    h = x.shape[-1]
    hs, hl = (0, G["q"].shape[0]) if plan is None else plan["heads"]
    shift1, scale1, gate1, shift2, scale2, gate2 = mod

    def cols(name, a, windows):
        w, b = W[name]
        idx = torch.cat([torch.arange(c0, c0 + n) for c0, n in windows])
        return a @ w[idx].T + b[idx]

    def rows(name, a, window):
        w, b = W[name]
        k0, n = window
        y = a @ w[:, k0:k0 + n].T + (b if rank == 0 else 0.0)
        return reduce(y)

    full = lambda name, n: [(0, n)]  # noqa: E731
    pl = plan or {"qkv": [(0, 3 * h)], "cross_q": full("cross_q", h),
                  "cross_kv": [(0, 2 * h)], "fc1": full("fc1", W["fc1"][0].shape[0]),
                  "out": (0, h), "cross_out": (0, h), "fc2": (0, W["fc2"][0].shape[1])}
    L = x.shape[0]
    a = _ln(x) * (1 + scale1) + shift1
    qkv = cols("qkv", a, pl["qkv"]).view(L, 3, hl, 64)
    g = {k: v[hs:hs + hl] for k, v in G.items()}
    q = _rope_rms(qkv[:, 0], cs[:, hs:hs + hl], g["q"])
    k = _rope_rms(qkv[:, 1], cs[:, hs:hs + hl], g["k"])
    o = _attn(q, k, qkv[:, 2]).reshape(L, hl * 64)
    x = x + gate1 * rows("out", o, pl["out"])
    yq = cols("cross_q", _ln(x), pl["cross_q"]).view(L, hl, 64)
    kv = cols("cross_kv", c, pl["cross_kv"]).view(c.shape[0], 2, hl, 64)
    rms = lambda t, gm: t * 8.0 / torch.linalg.vector_norm(t, dim=-1, keepdim=True).clamp_min(1e-12) * gm  # noqa: E731
    o = _attn(rms(yq, g["cq"]), rms(kv[:, 0], g["ck"]), kv[:, 1]).reshape(L, hl * 64)
    x = x + rows("cross_out", o, pl["cross_out"])
    a = _ln(x) * (1 + scale2) + shift2
    hid = torch.nn.functional.gelu(cols("fc1", a, pl["fc1"]), approximate="tanh")
    return x + gate2 * rows("fc2", hid, pl["fc2"])


def _inputs(s):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(s.seq, s.hidden, generator=g, dtype=torch.float64)
    c = torch.randn(s.cond_tokens, s.hidden, generator=g, dtype=torch.float64)
    ang = torch.rand(s.seq, s.heads, 32, generator=g, dtype=torch.float64) * 6.0
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1)
    return x, c, cs


def _worker(rank, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from head_shard import head_shard_plan

        s = _spec()
        W, G, mod = _weights(s)
        x, c, cs = _inputs(s)

        def reduce(t):
            dist.all_reduce(t)
            return t

        y = _block(x, c, cs, W, G, mod, plan=head_shard_plan(s, 2, rank), reduce=reduce, rank=rank)
        torch.save(y, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_sharded_block_two_gloo_ranks_matches_unsharded(tmp_path):
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    mp.spawn(_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    y0, y1 = (torch.load(tmp_path / f"rank{r}.pt") for r in (0, 1))
    assert torch.equal(y0, y1)  # both ranks hold the same residual stream
    s = _spec()
    W, G, mod = _weights(s)
    ref = _block(*_inputs(s), W, G, mod)
    assert torch.allclose(y0, ref, rtol=1e-12, atol=1e-12), float((y0 - ref).abs().max())


def test_lockstep_driver_rejects_uneven_ranks():
    from head_shard import run_lockstep

    class _Rank:
        def __init__(self, n):
            self.n = n
            self.buf = {"v_lat": None, "v_cam": None}

        def forward_steps(self, *a):
            for _ in range(self.n):
                yield torch.zeros(2)

    with pytest.raises(RuntimeError):
        run_lockstep([_Rank(2), _Rank(3)], None, None, None, None)
    assert len(run_lockstep([_Rank(2), _Rank(2)], None, None, None, None)) == 2


def test_peer_reduce_refuses_an_odd_number_of_reduction_points():
    """Three reduction points per block alternate between two partial buffers; with an odd
    block count the last point of one forward and the first of the next would share a buffer
    with no barrier between them, so the model refuses to build."""
    from flow_model import FlowWeights
    from head_shard import HeadShardedFlowModel

    with pytest.raises(ValueError, match="even number of reduction points"):
        HeadShardedFlowModel(FlowWeights(_spec()), rank=0, tp=2, device="cpu", reduce="peer")
