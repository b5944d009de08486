"""CPU oracle of the synthetic flow model and sampler (TEST INFRASTRUCTURE ONLY).

The same forward as triposplat-cpu-avx512_b200/flow_model.py, composed from the
oracle's restatements of the reference kernels (oracle.c), in numpy.  Used by
tests/test_model_gpu.py at reduced size as the parity checker, and timed on a
bounded sample by bench.py's cpu_baseline leg.  Never part of the product path.
"""
from __future__ import annotations

import numpy as np


class FlowOracle:
    def __init__(self, orc, spec, weights_np: dict, params_np: dict, freqs, tfreqs, threads=0):
        self.o, self.s, self.W, self.P = orc, spec, weights_np, params_np
        self.freqs, self.tfreqs, self.th = freqs, tfreqs, threads

    def lin(self, name, x, start=0, count=None):
        w = self.W[name]
        K = w["code01"].shape[0]
        lead = x.shape[:-1]
        y = self.o.gemm_nf24(x.reshape(-1, K), w["code01"], w["q2"], w["scale"], w["bias"],
                             start=start, count=count, threads=self.th)
        return y.reshape(*lead, y.shape[-1])

    @staticmethod
    def silu(x):
        return (x / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)

    def forward(self, x_lat, cam, t1000, cond):
        s, o = self.s, self.o
        B, h, H, L, Nl = x_lat.shape[0], s.hidden, s.heads, s.seq, s.latent_tokens
        ang = t1000[:, None].astype(np.float32) * self.tfreqs[None, :]
        tfe = np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)
        temb = self.lin("t_fc2", self.silu(self.lin("t_fc1", tfe)))
        st = self.silu(temb)
        mod = np.stack([self.lin("adaLN", st, c * h, h) for c in range(6)])        # [6,B,h]
        fmod = np.stack([self.lin("final_adaLN", st, c * h, h) for c in range(2)])  # [2,B,h]
        c = self.lin("cond_refiner", self.silu(self.lin("cond_embedder", cond)))
        x = np.concatenate([self.lin("x_embedder", x_lat), self.lin("camera_embedder", cam)], axis=1)
        for i in range(s.blocks):
            x = self.block(i, x, mod, c)
        a = o.modulate(o.layernorm(x, eps=s.eps), fmod[1], fmod[0])
        return self.lin("final_linear", a[:, :Nl]), self.lin("camera_head", a[:, Nl:])

    def block(self, i, x, mod, c):
        s, o, P = self.s, self.o, self.P
        B, L, h, H, Mc = x.shape[0], s.seq, s.hidden, s.heads, s.cond_tokens
        p = f"blocks.{i}."
        m = mod + P[p + "table"][:, None, :]
        a = o.modulate(o.layernorm(x, eps=s.eps), m[1], m[0])
        qkv = self.lin(p + "qkv", a).reshape(B, L, 3, H, 64)
        q, pk, pv = o.qkv_rope_rmsnorm_pack(qkv, self.freqs, P[p + "q_gamma"], P[p + "k_gamma"])
        k = pk[..., :L].transpose(0, 1, 3, 2)
        v = pv[..., :L].transpose(0, 1, 3, 2)
        att = o.sdpa(q, k, v, out_blhd=True, threads=self.th).reshape(B, L, h)
        x, _ = o.gated_residual(x, self.lin(p + "out", att), m[2])
        a = o.layernorm(x, eps=s.eps)
        cq = o.multihead_rmsnorm(self.lin(p + "cross_q", a).reshape(B, L, H, 64), P[p + "cq_gamma"])
        ckv = self.lin(p + "cross_kv", c).reshape(B, Mc, 2, H, 64)
        ck = o.multihead_rmsnorm(np.ascontiguousarray(ckv[:, :, 0]), P[p + "ck_gamma"])
        catt = o.sdpa(cq.transpose(0, 2, 1, 3), ck.transpose(0, 2, 1, 3),
                      ckv[:, :, 1].transpose(0, 2, 1, 3), out_blhd=True, threads=self.th)
        x = o.add(x, self.lin(p + "cross_out", catt.reshape(B, L, h)))
        a = o.modulate(o.layernorm(x, eps=s.eps), m[4], m[3])
        hid = o.gelu_tanh(self.lin(p + "fc1", a))
        x, _ = o.gated_residual(x, self.lin(p + "fc2", hid), m[5])
        return x

    def sample(self, noise_lat, noise_cam, cond, neg_cond, t1000, dt, guidance):
        x_lat, x_cam = noise_lat.copy(), noise_cam.copy()
        cond_pair = np.concatenate([cond, neg_cond], axis=0)
        g = np.array([guidance], np.float32)
        for i in range(len(dt)):
            vl, vc = self.forward(np.concatenate([x_lat, x_lat]), np.concatenate([x_cam, x_cam]),
                                  np.array([t1000[i], t1000[i]], np.float32), cond_pair)
            d = np.array([dt[i]], np.float32)
            x_lat = self.o.euler_update(x_lat, self.o.cfg_combine(vl[:1], vl[1:], g), d)
            x_cam = self.o.euler_update(x_cam, self.o.cfg_combine(vc[:1], vc[1:], g), d)
        return x_lat, x_cam


def weights_to_numpy(weights):
    W = {k: {"code01": v.code01.cpu().numpy(), "q2": v.q2.cpu().numpy(),
             "scale": v.scale.cpu().numpy(), "bias": v.bias.cpu().numpy()}
         for k, v in weights.linears.items()}
    P = {k: v.cpu().numpy() for k, v in weights.params.items()}
    return W, P
