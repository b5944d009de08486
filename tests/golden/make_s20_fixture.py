#!/usr/bin/env python3
"""Write the full-size s20 parity fixture from the REFERENCE's kernels.

Run once in a container that has the reference checkout (the GPU box does not):

    make -C oracle ref REF=<reference checkout>
    python tests/golden/make_s20_fixture.py --reference <reference checkout>

The model is the synthetic 28-block flow model of ``flow_model.FlowSpec()`` (206 NF24
Linears, hidden 1024, 16 heads, MLP 4096, 8192 latent tokens + 1 camera token, 1374
condition tokens).  Its float weights come from ``flow_model.host_float_weights`` (numpy
PCG64, reproducible on any host) and are packed by the reference's own NF24 packer
(scripts/native_linear_rnf8_avx512_patch.py:75-87, imported from the checkout).  Sampling
is 20 Euler flow-matching steps with CFG guidance 3.0 and timestep shift 3.0
(scripts/triposplat_quantized_sampler.py:387-494), every op one call of the reference's
AVX-512 kernels compiled into oracle/_ref (``oracle/ref_flow.RefFlowModel``).

Saved (``s20_config5.npz``, ~6 MB):
  latent [1, 8192, 64], camera [1, 1, 7]   end of sampling
  v0_latent [2, 8192, 64], v0_camera [2, 1, 7]   the first step's velocity pair
  linear_names / linear_digests   sha256 of each Linear's code01 | q2 | scale | bias bytes,
      so a test that packs the same float weights elsewhere can prove it holds the same codes
  metadata_json   seeds, shapes, sampler settings, host and wall time

The GPU test (tests/test_full_size_parity_gpu.py) regenerates the weights and inputs from
the seeds, checks the digests, runs the CUDA sampler and compares latent / camera RMSE
(scripts/compare_latent_npz.py:22-40 statistics).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import platform
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path[:0] = [str(REPO / "triposplat-cpu-avx512_b200"), str(REPO / "oracle")]

WEIGHT_SEED = 20
INPUT_SEED = 21
STEPS, GUIDANCE, SHIFT = 20, 3.0, 3.0


def linear_digest(code01, q2, scale, bias) -> str:
    h = hashlib.sha256()
    for a in (code01, q2, scale, bias):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def fixture_inputs(spec, seed: int = INPUT_SEED):
    """Seeded sampler inputs: noise latent [1, 8192, 64], noise camera [1, 1, 7], condition
    tokens [1, 1374, 1024] ~ N(0, 1); the unconditional branch's condition is zeros."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    lat = rng.standard_normal((1, spec.latent_tokens, spec.latent_dim), dtype=f32)
    cam = rng.standard_normal((1, 1, spec.camera_dim), dtype=f32)
    cond = rng.standard_normal((1, spec.cond_tokens, spec.cond_dim), dtype=f32)
    return lat, cam, cond, np.zeros_like(cond)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--out", type=Path, default=HERE / "s20_config5.npz")
    ap.add_argument("--blocks", type=int, default=28, help="28 = BASELINE config 5")
    ap.add_argument("--steps", type=int, default=STEPS)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / "scripts"))
    import torch
    from native_linear_nf8_avx512_patch import make_nf8_codebook  # reference packer
    from native_linear_rnf8_avx512_patch import quantize_nf24_i16_per_output_channel

    from flow_model import FlowSpec, host_float_weights, rope_freqs, sampler_schedule, timestep_frequencies
    from ref_flow import RefFlowModel

    spec = FlowSpec(blocks=args.blocks)
    t0 = time.time()
    cb = make_nf8_codebook(torch)
    W, P, names, digests = {}, {}, [], []
    for kind, name, val in host_float_weights(spec, WEIGHT_SEED):
        if kind == "linear":
            codes, scales, _ = quantize_nf24_i16_per_output_channel(torch.from_numpy(val[0]), cb)
            w = {"code01": codes[0].numpy(), "q2": codes[1].numpy(), "scale": scales[0].numpy(),
                 "bias": val[1]}
            W[name] = w
            names.append(name)
            digests.append(linear_digest(w["code01"], w["q2"], w["scale"], w["bias"]))
        else:
            P[name] = val
    t_pack = time.time() - t0
    print(f"packed {len(W)} linears in {t_pack:.1f} s", flush=True)

    model = RefFlowModel(spec, W, P, rope_freqs(spec), timestep_frequencies(spec),
                         threads=args.threads or None)
    lat, cam, cond, neg = fixture_inputs(spec)
    t1000, dt = sampler_schedule(args.steps, SHIFT)
    v0 = {}
    t_start = time.time()

    def on_step(i, vl, vc):
        if i == 0:
            v0["lat"], v0["cam"] = vl.copy(), vc.copy()
        print(f"step {i + 1}/{args.steps} at {time.time() - t_start:.0f} s", flush=True)

    x_lat, x_cam = model.sample(lat, cam, cond, neg, t1000, dt, GUIDANCE, on_step=on_step)
    wall = time.time() - t_start
    meta = {"spec": {"blocks": spec.blocks, "hidden": spec.hidden, "heads": spec.heads,
                     "mlp": spec.mlp, "grid": list(spec.grid), "latent_dim": spec.latent_dim,
                     "camera_dim": spec.camera_dim, "cond_tokens": spec.cond_tokens},
            "weight_seed": WEIGHT_SEED, "input_seed": INPUT_SEED, "steps": args.steps,
            "guidance": GUIDANCE, "shift": SHIFT, "kernels": "reference AVX-512 (oracle/_ref)",
            "packer": "reference quantize_nf24_i16_per_output_channel",
            "threads": model.k.th, "host": platform.processor() or platform.machine(),
            "sample_wall_s": round(wall, 1), "pack_wall_s": round(t_pack, 1)}
    np.savez(args.out, latent=x_lat, camera=x_cam, v0_latent=v0["lat"], v0_camera=v0["cam"],
             linear_names=np.array(names), linear_digests=np.array(digests),
             metadata_json=np.array(json.dumps(meta)))
    print(f"wrote {args.out} ({wall:.0f} s of sampling)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
