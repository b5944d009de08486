"""Shard directories on the GPU: Linears written by the reference's packer load into device
memory (with the k-contiguous planes) and run through the split GEMM equal to the oracle;
the synthetic flow model loaded from its own shards gives the same forward bit for bit."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_shards_on_device_gemm(oracle):
    import _native
    from nf24_shards import load_nf24_shards

    lib = _native.load()
    _native.use_current_stream(lib)
    sh = load_nf24_shards(GOLDEN / "shards_ref", device="cuda", verify_checksums=True, nk=True)
    g = torch.Generator().manual_seed(8)
    for name, lin in sh.linears.items():
        K, N = (int(d) for d in lin.code01.shape)
        M = 77
        x = torch.randn(M, K, generator=g)
        ref = oracle.gemm_nf24(x.numpy(), lin.code01.cpu().numpy(), lin.q2.cpu().numpy(),
                               lin.scale.cpu().numpy(), lin.bias.cpu().numpy())
        nbytes = int(lib.triposplat_b200_split_bytes(M, K))
        buf = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
        sp = (buf.data_ptr() + 255) & ~255
        xc = x.cuda()
        assert lib.triposplat_b200_split_f32(xc.data_ptr(), M, K, K, sp) == 0
        out = torch.empty(M, N, device="cuda")
        assert lib.triposplat_b200_gemm_nf24_split_nk(
            sp, M, K, lin.code01_nk.data_ptr(), lin.q2_nk.data_ptr(), K, lin.scale.data_ptr(),
            lin.bias.data_ptr(), out.data_ptr(), N, 0, N, N, 0, None, 0, 1) == 0
        torch.cuda.synchronize()
        y = out.cpu().numpy()
        assert (np.abs(y - ref) <= 2e-5 + 2e-5 * np.abs(ref)).all(), name


def test_flow_model_from_shards_bitwise(tmp_path):
    from flow_model import FlowModelB200, FlowSpec, make_weights
    from nf24_shards import load_flow_weights, save_flow_weights

    spec = FlowSpec.small(blocks=2)
    w = make_weights(spec, seed=12, device="cuda")
    save_flow_weights(w, tmp_path / "model")
    w2 = load_flow_weights(tmp_path / "model", spec, device="cuda", verify_checksums=True)
    g = torch.Generator().manual_seed(13)
    lat = torch.randn(2, spec.latent_tokens, spec.latent_dim, generator=g).cuda()
    cam = torch.randn(2, 1, spec.camera_dim, generator=g).cuda()
    t = torch.tensor([500.0, 500.0]).cuda()
    cond = torch.randn(2, spec.cond_tokens, spec.cond_dim, generator=g).cuda()
    a = [v.clone() for v in FlowModelB200(w, batch=2).forward(lat, cam, t, cond)]
    b = [v.clone() for v in FlowModelB200(w2, batch=2).forward(lat, cam, t, cond)]
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
