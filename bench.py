#!/usr/bin/env python3
"""Benchmark: s20 CFG flow sampling of the synthetic 28-block NF24 flow model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--parallel replicas|cfg] [--tp T] [--case model|gemm1|sdpa2a|sdpa2b|sdpa2c|mlp3|block4]

A step is one CFG sampler step (one forward of the batch-2 [cond, uncond] pair through
28 blocks and 206 NF24 Linears, then CFG combine + Euler update) for one image.
Multi-GPU (torchrun, one process per GPU), timing is the max over ranks:
  --parallel replicas (default): every rank samples its own image (weak scaling, no
      collective on the data path); value = (time of K steps) / K * 20 / N.
  --parallel cfg: each image's CFG pair is split over two GPUs (conditional branch on the
      even rank, unconditional on the odd one; one NCCL all-gather of the velocity per
      step); value = (time of K steps) / K * 20 / (N / 2).
  --tp T: each model runs head-sharded over T GPUs (three NCCL all-reduces per block);
      with --parallel cfg an image spans 2T GPUs, otherwise T.

Reported metric: seconds per image for 20-step sampling (lower is better), whole job.
Also reported: the end-to-end number through the public sampler API with host buffers
(H2D of each step's inputs, D2H of its result), the roofline of the dominant kernel,
per-kernel device time, and, on rank 0 at N=1, the reference CPU path timed on this host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "triposplat-cpu-avx512_b200"
sys.path[:0] = [str(PKG), str(REPO / "oracle")]

METRIC = "s20 CFG sampling sec/image; NF24 GEMM & exact-SDPA TFLOP/s vs roofline"
UNIT = "s/image"
SAMPLER_STEPS = 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", choices=("auto", "replicas", "cfg"), default="auto",
                    help="auto (default): one GPU runs the CFG pair; N > 1 GPUs run one image, "
                         "its CFG pair split over two GPU groups and, with N > 2, each branch's "
                         "token rows over N / 2 GPUs (--sp); replicas: one image per GPU; cfg: "
                         "each image's CFG pair split over two GPUs (or 2 x --tp / --sp)")
    ap.add_argument("--sp", type=int, default=0,
                    help="query-row sharding: each CFG branch's token rows over this many GPUs "
                         "(K / V tiles pulled over NVLink once per block); 0 = auto")
    ap.add_argument("--tp", type=int, default=1,
                    help="head-sharded tensor parallelism: each model (the CFG pair, or one "
                         "branch with --parallel cfg) runs on this many GPUs, heads and MLP "
                         "columns split, three NCCL all-reduces per block")
    ap.add_argument("--tp-reduce", choices=("peer", "nccl"), default="peer",
                    help="peer: the ranks' partials are summed into the residual by one kernel "
                         "reading NVLink peer memory; nccl: NCCL all-reduce + residual kernel")
    ap.add_argument("--no-graph", action="store_true",
                    help="issue every kernel from the host each step instead of replaying "
                         "the step's CUDA graph")
    ap.add_argument("--lk", type=int, default=None,
                    help="sdpa cases: override the key count (the key-tile sweep of the "
                         "attention kernel's per-item cost)")
    ap.add_argument("--case", default="model",
                    choices=("model", "gemm1", "sdpa2a", "sdpa2b", "sdpa2c", "mlp3", "block4"),
                    help="model = BASELINE config 5 (the headline); the others time one "
                         "BASELINE config on one GPU and print its own line")
    return ap.parse_args()


def run_case(args):
    """One BASELINE config on cuda:0: gemm1 = config 1, sdpa2a/b/c = config 2 (a)/(b)/(c),
    mlp3 = config 3 (LN -> fc1 -> GELU -> fc2 -> residual), block4 = config 4 (one block)."""
    import torch

    import _native
    import native_ops as ops
    from native_sdpa_ctypes import native_sdpa_f32
    from nf24_linear import nf24_linear
    from nf24_pack import quantize_nf24_i16_any_device

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    lib = _native.load()

    def packed(n, k):
        c, s_, _ = quantize_nf24_i16_any_device(torch.randn(n, k, device=dev, generator=g) * 0.02,
                                               stats=False)
        return c[0], c[1], s_[0], torch.randn(n, device=dev, generator=g) * 0.01

    if args.case == "gemm1":
        M, K, N = 4096, 1024, 3072
        x = torch.randn(M, K, device=dev, generator=g)
        c01, q2, sc, b = packed(N, K)
        out = torch.empty(M, N, device=dev)
        fn = lambda: nf24_linear(x, c01, q2, sc, b, out=out, lib=lib)  # noqa: E731
        flops, passes, what = 2.0 * M * N * K, 3, "NF24 Linear 4096x1024x3072 (config 1)"
    elif args.case.startswith("sdpa"):
        B, H, Lq = 2, 16, 8192
        Lk = 1374 if args.case == "sdpa2c" else 8192
        if args.lk:
            Lk = args.lk
        q = torch.randn(B, H, Lq, 64, device=dev, generator=g)
        k = torch.randn(B, H, Lk, 64, device=dev, generator=g)
        v = torch.randn(B, H, Lk, 64, device=dev, generator=g)
        kb = torch.randn(B, H, Lk, device=dev, generator=g) if args.case == "sdpa2b" else None
        fn = lambda: native_sdpa_f32(q, k, v, key_bias=kb)  # noqa: E731
        flops, passes = 4.0 * B * H * Lq * Lk * 64, 3
        what = {"sdpa2a": "exact SDPA self 2x16x8192^2 (config 2a)",
                "sdpa2b": "exact SDPA + key bias [2,16,8192] (config 2b)",
                "sdpa2c": "exact SDPA cross 8192x1374 (config 2c)"}[args.case]
        if args.lk:
            what += f", keys overridden to {Lk}"
    elif args.case == "mlp3":
        M, C, F = 8192, 1024, 4096
        x = torch.randn(1, M, C, device=dev, generator=g)
        gam = 1.0 + torch.randn(C, device=dev, generator=g) * 0.02
        beta = torch.zeros(C, device=dev)
        w1, w2 = packed(F, C), packed(C, F)
        a = torch.empty_like(x)
        hid = torch.empty(M, F, device=dev)
        y = torch.empty(1, M, C, device=dev)

        def fn():
            ops.layernorm(x, gam, beta, eps=1e-6, out=a)
            nf24_linear(a, *w1, out=hid, lib=lib)
            ops.gelu_tanh(hid, out=hid)
            nf24_linear(hid, *w2, out=y, lib=lib)
            ops.add_inplace(y, x)
        flops, passes, what = 2.0 * 2 * M * C * F, 3, "MLP sub-block M=8192 1024-4096-1024 (config 3)"
    else:  # block4
        from flow_model import FlowModelB200, FlowSpec, make_weights

        spec = FlowSpec(blocks=1)
        model = FlowModelB200(make_weights(spec, seed=0, device=str(dev)), device=str(dev))
        b = model.buf
        b["x"].normal_(generator=g)
        b["c"].normal_(generator=g)
        b["mod"].normal_(generator=g)
        b["mod"].mul_(0.02)
        fn = lambda: model._block(0)  # noqa: E731
        fl = spec.flops_per_forward(batch=2)
        L, Mc = spec.seq, spec.cond_tokens
        flops = 2.0 * 2 * (L * 1024 * 3072 + 3 * L * 1024 * 1024 + Mc * 1024 * 2048 + 2 * L * 1024 * 4096) \
            + 4.0 * 2 * 16 * L * (L + Mc) * 64
        passes, what = None, "one flow block, B=2 CFG pair, L=8193, 1374 cond tokens (config 4)"
        del fl
    _native.use_current_stream(lib)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(args.steps):
        fn()
    en.record()
    torch.cuda.synchronize()
    _native.check_status(lib)
    ms = st.elapsed_time(en) / args.steps
    tf = flops / (ms / 1e3) / 1e12
    peaks, src = load_peaks()
    line = {"metric": f"{what} TFLOP/s (algorithmic flops)", "value": round(tf, 1),
            "unit": "TFLOP/s", "case": args.case, "ms_per_step": round(ms, 4),
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "n_gpus": 1,
            "dtype": "f32", "data": "synthetic",
            "frac_of_bf16_burst": round(tf / float(peaks["bf16_tflops"]), 4),
            "tensor_passes": passes,
            "tensor_pipe_frac": None if passes is None else round(passes * tf / float(peaks["bf16_tflops"]), 4),
            "peak_source": src}
    print(json.dumps(line), flush=True)
    return 0


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profiled_traffic(profile: str, key: str):
    """DRAM bytes per launch (`key:` line) from a committed ncu summary, if present."""
    f = REPO / "profiles" / profile
    if not f.is_file():
        return None
    for line in f.read_text().splitlines():
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def __enter__(self):
        """Start sampling every 100 ms and return once the first sample has arrived (the
        tool takes a moment to start), so that even a short timed region is sampled."""
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        t_end = time.time() + 5.0
        while not self.lines and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.02)
        self.first = len(self.lines)  # samples from here on fall inside the timed region
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is None:
            return False
        n_exit = len(self.lines)  # samples that arrived while the region ran
        time.sleep(0.15)  # for a region shorter than the interval: the next sample
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        inside = self.lines[self.first:n_exit] or self.lines[self.first:self.first + 1]
        for line in inside:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)
        return False

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)}


def cpu_baseline(spec):
    import cpu_block

    try:
        r = cpu_block.time_sample(spec, block_reps=3)
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        return {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "unavailable",
                "sample": f"reference CPU path could not run: {exc}"}
    return {"value": round(r["sec_per_image"], 2), "unit": UNIT, "cores": r["threads"], "kind": r["kind"],
            "sample": (f"the full-size sampler step's pieces through the reference's AVX-512 kernels "
                       f"(B=2 CFG pair, L=8193, 1374 cond tokens): embeddings {r['embed_seconds']:.3f} s, "
                       f"block median of {r['reps']} = {r['block_seconds']:.3f} s (x28), final layer + "
                       f"CFG/Euler {r['final_seconds']:.3f} s; sec/image = 20 x step")}


def reference_schedule(steps: int, pieces: int) -> list[list[int]]:
    """Pieces of one sampler step run by each of ``steps`` timed steps of the reference arm:
    with steps <= pieces every piece runs exactly once (consecutive runs per step); with
    more steps, step i runs piece i mod pieces (the step is covered steps / pieces times)."""
    if steps <= pieces:
        return [[j for j in range(pieces) if j * steps // pieces == i] for i in range(steps)]
    return [[i % pieces] for i in range(steps)]


def run_reference_case(args):
    """--impl reference --case C: the reference's own AVX-512 kernels for one BASELINE
    config on the host cores (all of them), median of --steps runs after one warm-up; the
    same TFLOP/s metric as the b200 case line."""
    import ctypes

    import numpy as np

    from ref_flow import REF, RefKernels, _bind, _p, host_threads

    if not RefKernels.available():
        print(json.dumps({"impl": "reference", "case": args.case, "unavailable":
                          "reference AVX-512 kernels not built or host CPU lacks AVX-512"}))
        return 0
    rk = RefKernels()
    th = rk.th
    rng = np.random.default_rng(0)
    f32 = np.float32

    def packed(n, k):  # random codes: the kernels' cost does not depend on the values
        return {"code01": rng.integers(-540, 541, size=(k, n), dtype=np.int16),
                "q2": rng.integers(-128, 128, size=(k, n), dtype=np.int8),
                "scale": np.full(n, 0.02 / 127 / 1024, f32), "bias": rng.standard_normal(n, dtype=f32)}

    if args.case == "gemm1":
        M, K, N = 4096, 1024, 3072
        x, w, out = rng.standard_normal((M, K), dtype=f32), packed(N, K), np.empty((M, N), f32)
        fn = lambda: rk.linear(w, x, out)  # noqa: E731
        flops, what = 2.0 * M * N * K, "NF24 Linear 4096x1024x3072 (config 1)"
    elif args.case.startswith("sdpa"):
        sd = _bind(ctypes.CDLL(str(REF / "libref_sdpa_q8t512.so")), "triposplat_sdpa_f32_avx512_exact_q8t512",
                   [ctypes.c_void_p] * 5 + [ctypes.c_int] * 8)
        B, H, Lq = 2, 16, 8192
        Lk = args.lk or (1374 if args.case == "sdpa2c" else 8192)
        q = rng.standard_normal((B, H, Lq, 64), dtype=f32)
        k = rng.standard_normal((B, H, Lk, 64), dtype=f32)
        v = rng.standard_normal((B, H, Lk, 64), dtype=f32)
        bias = rng.standard_normal(Lk, dtype=f32) if args.case == "sdpa2b" else None
        o = np.empty_like(q)
        fn = lambda: sd(_p(q), _p(k), _p(v), _p(bias), _p(o), B, H, Lq, Lk, 64,  # noqa: E731
                        int(bias is not None), 0 if bias is None else Lk, th)
        flops = 4.0 * B * H * Lq * Lk * 64
        what = {"sdpa2a": "exact SDPA self 2x16x8192^2 (config 2a)",
                "sdpa2b": "exact SDPA + shared key bias [8192] (config 2b; the reference ABI's bias)",
                "sdpa2c": "exact SDPA cross 8192x1374 (config 2c)"}[args.case]
    elif args.case == "mlp3":
        M, C, F = 8192, 1024, 4096
        ln = _bind(ctypes.CDLL(str(REF / "libref_norm_rope.so")), "triposplat_layernorm_f32_avx512",
                   [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int])
        x = rng.standard_normal((M, C), dtype=f32)
        gam, beta = np.ones(C, f32), np.zeros(C, f32)
        w1, w2 = packed(F, C), packed(C, F)
        a, hid, y = np.empty_like(x), np.empty((M, F), f32), np.empty((M, C), f32)

        def fn():
            ln(_p(x), _p(gam), _p(beta), _p(a), M, C, 1e-6, 1, th)
            rk.linear(w1, a, hid)
            rk.gelu(_p(hid), _p(hid), hid.size, th)
            rk.linear(w2, hid, y)
            rk.add(_p(y), _p(x), y.size, th)
        flops, what = 2.0 * 2 * M * C * F, "MLP sub-block M=8192 1024-4096-1024 (config 3)"
    elif args.case == "block4":
        import cpu_block
        from flow_model import FlowSpec

        fwd = cpu_block.RefForward(FlowSpec())
        pieces = fwd.pieces()
        pieces[0]()
        fn = pieces[1]
        L, Mc = 8193, 1374
        flops = 2.0 * 2 * (L * 1024 * 3072 + 3 * L * 1024 * 1024 + Mc * 1024 * 2048 + 2 * L * 1024 * 4096) \
            + 4.0 * 2 * 16 * L * (L + Mc) * 64
        what = "one flow block, B=2 CFG pair, L=8193, 1374 cond tokens (config 4)"
    else:
        raise SystemExit(f"no reference case {args.case}")
    fn()
    times = []
    for _ in range(max(1, min(args.steps, 5))):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    sec = float(np.median(times))
    print(json.dumps({"metric": f"{what} TFLOP/s (algorithmic flops)", "value": round(flops / sec / 1e12, 4),
                      "unit": "TFLOP/s", "impl": "reference", "case": args.case,
                      "seconds": round(sec, 4), "runs": len(times), "higher_is_better": True,
                      "cpu_baseline": {"value": round(flops / sec / 1e12, 4), "unit": "TFLOP/s",
                                       "cores": host_threads(), "kind": "reference",
                                       "sample": f"median of {len(times)} runs after one warm-up"}}))
    return 0


def run_reference(args):
    """--impl reference: the reference's CPU kernels on the host cores, rank 0 only.

    The K timed steps together run one whole sampler step of the full-size model (the
    embeddings, 28 blocks, the final layer and the CFG / Euler update, cut into 30 pieces
    by reference_schedule) through the reference's kernels; sec/image = 20 x the time of
    that sampler step.  Warm-up steps run one block each (at most two)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.case != "model":
        return run_reference_case(args)
    from flow_model import FlowSpec
    import cpu_block
    from ref_flow import RefKernels

    spec = FlowSpec()
    if not RefKernels.available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference AVX-512 kernels not built or host CPU lacks AVX-512"}))
        return 0
    fwd = cpu_block.RefForward(spec)
    pieces = fwd.pieces()
    pieces[0]()  # embeddings first: the blocks read the token buffer they fill
    for _ in range(max(0, min(args.warmup, 2))):
        pieces[1]()
    sched = reference_schedule(args.steps, len(pieces))
    step_times, piece_time = [], {}
    for plan in sched:
        t0 = time.perf_counter()
        for j, t in cpu_block.time_pieces(fwd, plan):
            piece_time.setdefault(j, []).append(t)
        step_times.append(time.perf_counter() - t0)
    sampler_step = sum(sum(v) / len(v) for v in piece_time.values())
    value = cpu_block.SAMPLER_STEPS * sampler_step
    sample = (f"the {args.steps} timed steps run one full sampler step of the full-size model "
              f"(embeddings, 28 blocks, final layer, CFG/Euler; B=2 CFG pair, L=8193) through the "
              f"reference's AVX-512 kernels, {sampler_step:.2f} s; sec/image = 20 x that step")
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sum(step_times) / len(step_times) * 1e3, 3),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "s20 CFG flow sampling, synthetic 28-block NF24 flow model",
                       "parallelism": "host CPU (OpenMP)", "sampler_step_seconds": round(sampler_step, 3)},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": fwd.th,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def parallelism_label(split: bool, tp: int, images: int, reduce: str = "peer", sp: int = 1) -> str:
    reduce_label = ("one kernel reading the ranks' partials over NVLink and updating the residual"
                    if reduce == "peer" else "NCCL all-reduce + residual kernel")
    parts = []
    if split:
        parts.append("CFG pair split over 2 GPU groups (one NCCL all-gather of the velocity per step)")
    if tp > 1:
        parts.append(f"heads and MLP columns sharded over {tp} GPUs (3 reductions per block: "
                     f"{reduce_label})")
    if sp > 1:
        parts.append(f"token rows sharded over {sp} GPUs per branch (query-row sharding; one peer "
                     f"barrier + K/V tile pull over NVLink per block)")
    if not parts:
        return f"replicas x{images} (one image per GPU, no data-path collective)"
    return f"{images} image(s) in parallel; per image: " + "; ".join(parts)


def step0_parity(sampler, weights, dev, rank, inputs):
    """Relative rmse (and bitwise equality) of the partitioned first-step velocity pair
    against one GPU's batch-2 forward of the same inputs, computed on rank 0; every rank
    takes part in the partitioned step (its sampler state is left unchanged).  None on
    other ranks."""
    import numpy as np
    import torch

    from flow_model import FlowModelB200, sampler_schedule

    lat, cam = sampler.velocity_pair(0)
    if rank != 0:
        return None
    h_lat, h_cam, h_cond, h_neg = inputs
    t1000, _ = sampler_schedule(SAMPLER_STEPS, 3.0)
    t = torch.tensor([t1000[0], t1000[0]], dtype=torch.float32, device=dev)
    d = lambda a, b: torch.cat([a, b]).to(dev)  # noqa: E731
    ref = FlowModelB200(weights, batch=2, device=str(dev))
    r_lat, r_cam = ref.forward(d(h_lat, h_lat), d(h_cam, h_cam), t, d(h_cond, h_neg))
    torch.cuda.synchronize()
    a = torch.cat([lat.reshape(2, -1), cam.reshape(2, -1)], 1).double().cpu().numpy()
    b = torch.cat([r_lat.reshape(2, -1), r_cam.reshape(2, -1)], 1).double().cpu().numpy()
    del ref
    torch.cuda.empty_cache()
    rel = float(np.sqrt(np.mean((a - b) ** 2)) / np.sqrt(np.mean(b ** 2)))
    return {"step0_velocity_rel_rmse_vs_1gpu": rel, "bitwise_equal": bool(np.array_equal(a, b)),
            "reference": "one GPU, batch-2 forward of the same inputs and weights"}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.case != "model":
        return run_case(args)

    import torch
    import torch.distributed as dist

    import _native
    from flow_model import CfgEulerSampler, FlowModelB200, FlowSpec, make_weights

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    spec = FlowSpec()
    lib = _native.load()
    weights = make_weights(spec, seed=0, device=str(dev))
    parallel, T, SP = args.parallel, args.tp, args.sp
    if parallel == "auto":  # one image over all GPUs: CFG pair split, then query rows
        parallel = "replicas" if world == 1 else "cfg"
        if world > 2 and T == 1 and SP == 0:
            SP = world // 2
    SP = max(SP, 1)
    split = parallel == "cfg"
    if SP > 1 and (T > 1 or not split):
        raise SystemExit("--sp runs with the CFG split (--parallel cfg) and without --tp")
    W = max(T, SP)  # GPUs per CFG branch (or per CFG pair without the split)
    span = W * (2 if split else 1)  # GPUs per image
    if T < 1 or spec.heads % T or world % span or (split and world < 2):
        raise SystemExit(f"--gpus {world} does not split into images of {span} GPU(s) "
                         f"(--parallel {parallel} --tp {T} --sp {SP}; tp must divide {spec.heads} heads)")
    images, image = world // span, rank // span
    branch, w_rank = (rank // W) % 2 if split else 0, rank % W
    # every rank creates every group, in the same order
    w_groups, pair_groups, image_groups = {}, {}, {}
    if W > 1:
        for im in range(images):
            for br in range(2 if split else 1):
                base = im * span + br * W
                w_groups[(im, br)] = dist.new_group(list(range(base, base + W)))
    if split and SP == 1:
        for im in range(images):
            for j in range(W):
                pair_groups[(im, j)] = dist.new_group([im * span + j, im * span + W + j])
    if SP > 1:
        for im in range(images):
            image_groups[im] = dist.new_group(list(range(im * span, (im + 1) * span)))
    batch = 1 if split else 2
    if SP > 1:
        from seq_shard import SeqCfgSampler, SeqShardedFlowModel

        model = SeqShardedFlowModel(weights, rank=w_rank, world=SP, batch=1, device=str(dev),
                                    group=w_groups[(image, branch)])
        sampler = SeqCfgSampler(model, branch=branch, image_group=image_groups[image],
                                steps=SAMPLER_STEPS, guidance=3.0, shift=3.0)
    else:
        if T > 1:
            from head_shard import HeadShardedFlowModel

            model = HeadShardedFlowModel(weights, rank=w_rank, tp=T, batch=batch, device=str(dev),
                                         group=w_groups[(image, branch)], reduce=args.tp_reduce)
        else:
            model = FlowModelB200(weights, batch=batch, device=str(dev))
        if split:
            from cfg_split import CfgSplitSampler

            # branch 0 (conditional) on the first T ranks of the image, branch 1 on the next T
            sampler = CfgSplitSampler(model, branch=branch, group=pair_groups[(image, w_rank)],
                                      steps=SAMPLER_STEPS, guidance=3.0, shift=3.0)
        else:
            sampler = CfgEulerSampler(model, steps=SAMPLER_STEPS, guidance=3.0, shift=3.0)

    # per-image seeded inputs in pinned host memory (also the e2e source buffers)
    g = torch.Generator().manual_seed(1000 + image)
    h_lat = torch.randn(1, spec.latent_tokens, spec.latent_dim, generator=g).pin_memory()
    h_cam = torch.randn(1, 1, spec.camera_dim, generator=g).pin_memory()
    h_cond = torch.randn(1, spec.cond_tokens, spec.cond_dim, generator=g).pin_memory()
    h_neg = torch.zeros(1, spec.cond_tokens, spec.cond_dim).pin_memory()
    h_out_lat = torch.empty(spec.latent_tokens, spec.latent_dim).pin_memory()
    h_out_cam = torch.empty(1, spec.camera_dim).pin_memory()
    sampler.load(h_lat.to(dev), h_cam.to(dev), h_cond.to(dev), h_neg.to(dev))
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- multi-GPU correctness: the partitioned first step against one GPU's forward
    parity = None
    if world > 1 and parallel != "replicas":
        parity = step0_parity(sampler, weights, dev, rank, (h_lat, h_cam, h_cond, h_neg))
        barrier()

    # ---- warm-up (untimed)
    for i in range(args.warmup):
        sampler.step(i % SAMPLER_STEPS)
    torch.cuda.synchronize()
    _native.check_status(lib)

    # ---- the once-per-image condition path (cached across the sampler steps), timed once
    # and added to sec/image below
    cond_ms = 0.0
    if getattr(sampler, "cached", False):
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        c0.record()
        sampler.refresh_condition()
        c1.record()
        torch.cuda.synchronize()
        cond_ms = c0.elapsed_time(c1)
    cond_ms = max_over_ranks(cond_ms)

    # ---- capture the step into a CUDA graph (the library brackets each kernel with CUDA
    # events inside the graph, so the timed replays still yield live per-kernel times)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    if not args.no_graph:
        sampler.prepare_capture()
        lib.triposplat_b200_profile_enable(1)
        launches0 = int(lib.triposplat_b200_launch_count())
        sampler.record_graph()
        launches_per_step = int(lib.triposplat_b200_launch_count()) - launches0
        launches_per_step += getattr(sampler, "eager_launches_per_step", 0)
        lib.triposplat_b200_profile_enable(0)
    else:
        lib.triposplat_b200_profile_enable(1)
    torch.cuda.synchronize()

    # ---- timed region: K sampler steps, inputs resident in HBM
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    launches0 = int(lib.triposplat_b200_launch_count())
    with ClockSampler(uuid) as clk:
        start.record()
        for i in range(args.steps):
            sampler.step((args.warmup + i) % SAMPLER_STEPS)
        stop.record()
        torch.cuda.synchronize()
    lib.triposplat_b200_profile_enable(0)
    barrier()
    if args.no_graph:
        launches = int(lib.triposplat_b200_launch_count()) - launches0
        prof = _native.profile_collect(lib)
        prof = {k: {"launches": v["launches"], "ms": v["ms"]} for k, v in prof.items()}
    else:
        launches = launches_per_step * args.steps
        # the graph's events hold the last replay (the last timed step): one step's kernels
        prof = _native.profile_collect(lib, keep=True)
        prof = {k: {"launches": v["launches"] * args.steps, "ms": v["ms"] * args.steps}
                for k, v in prof.items()}
    ms_total = max_over_ranks(start.elapsed_time(stop))
    _native.check_status(lib)

    # ---- end-to-end through the public sampler API with host buffers
    h2d = sum(t.numel() * 4 for t in (h_lat, h_cam, h_cond, h_neg))
    d2h = (h_out_lat.numel() + h_out_cam.numel()) * 4
    barrier()
    torch.cuda.synchronize()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for i in range(args.steps):
        sampler.load(h_lat, h_cam, h_cond, h_neg)  # H2D from pinned host memory
        sampler.step((args.warmup + i) % SAMPLER_STEPS)
        h_out_lat.copy_(sampler.x_lat[0], non_blocking=True)
        h_out_cam.copy_(sampler.x_cam[0], non_blocking=True)
    e_stop.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_stop))
    finite = bool(torch.isfinite(h_out_lat).all()) and bool(torch.isfinite(h_out_cam).all())

    # ---- report
    ms_step = ms_total / args.steps
    value = (ms_step * SAMPLER_STEPS + cond_ms) / 1e3 / images
    e2e_value = e2e_ms / args.steps / 1e3 * SAMPLER_STEPS / images
    # this GPU's share: the pair, or one branch, and 1/W of the block work under --tp / --sp
    flops = spec.flops_per_forward(batch=model.B, tp=W)
    peaks, peak_src = load_peaks()
    attn = prof["sdpa_attn"]
    L, Mc, BH = spec.seq, spec.cond_tokens, model.B * spec.heads // W
    attn_flops_per_step = spec.blocks * 4.0 * BH * L * (L + Mc) * spec.head_dim
    achieved = None
    if attn["launches"]:
        launches_per_step = attn["launches"] / args.steps
        achieved = attn_flops_per_step / launches_per_step / (attn["ms"] / attn["launches"] / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"])
    # the sustained figure was measured at the power cap's lower clock; the burst one beside it
    burst = float(peaks["bf16_tflops"])
    kernels = {k: {"launches_per_step": round(v["launches"] / args.steps, 2),
                   "ms_per_step": round(v["ms"] / args.steps, 3),
                   "share": round(v["ms"] / max(1e-9, sum(x["ms"] for x in prof.values())), 4)}
               for k, v in prof.items()}
    gemm = prof["gemm_tc"]
    g_achieved = None
    if gemm["ms"]:
        g_achieved = flops["gemm"] / (gemm["ms"] / args.steps / 1e3) / 1e12
    # the dominant kernel (larger share of the step) first
    roof_attn = {"kernel": "sdpa_fwd_tc (exact SDPA, self + cross)", "bound": "tensor",
                 "achieved": None if achieved is None else round(achieved, 1),
                 "peak": peak, "unit": "TFLOP/s",
                 "frac": None if achieved is None else round(achieved / peak, 4),
                 "peak_source": f"bf16_tflops_sustained, {peak_src} (of measured)",
                 "flops": "algorithmic 4*B*H*Lq*Lk*64 per launch (3 split-fp16 tensor passes each)",
                 "tensor_pipe_frac": None if achieved is None else round(3 * achieved / peak, 4),
                 "tensor_pipe_frac_of_burst": None if achieved is None else round(3 * achieved / burst, 4),
                 "ms_per_step": round(attn["ms"] / args.steps, 3),
                 "traffic": profiled_traffic("sdpa_fwd_tc_block4.md", "traffic_bytes_per_launch_in_step")}
    roof_gemm = {"kernel": "nf24_gemm_tc (NF24 GEMM, all tensor-core Linears of the step)",
                 "bound": "tensor",
                 "achieved": None if g_achieved is None else round(g_achieved, 1),
                 "peak": peak, "unit": "TFLOP/s",
                 "frac": None if g_achieved is None else round(g_achieved / peak, 4),
                 "peak_source": f"bf16_tflops_sustained, {peak_src} (of measured)",
                 "flops": "algorithmic 2*M*N*K per launch, summed over the step's Linears "
                          "(3 fp16 tensor passes each: S.hi, S.lo, T.hi)",
                 "tensor_pipe_frac": None if g_achieved is None else round(3 * g_achieved / peak, 4),
                 "tensor_pipe_frac_of_burst": None if g_achieved is None else round(3 * g_achieved / burst, 4),
                 "ms_per_step": round(gemm["ms"] / args.steps, 3),
                 "traffic": profiled_traffic("nf24_gemm_tc_gelu_split_block4.md", "traffic_bytes_per_launch"),
                 "traffic_launch": "fc1 of a block (the largest Linear; one ncu capture)"}
    roofs = [roof_gemm, roof_attn] if gemm["ms"] >= attn["ms"] else [roof_attn, roof_gemm]
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": False, "scaling": "weak" if parallel == "replicas" else "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian latent/camera/condition; random-init weights packed to NF24)",
        "config": {"workload": "s20 CFG flow sampling, synthetic 28-block NF24 flow model (BASELINE config 5)",
                   "blocks": spec.blocks, "linears": len(spec.linears()), "hidden": spec.hidden,
                   "heads": spec.heads, "mlp": spec.mlp, "latent_tokens": spec.latent_tokens,
                   "seq": spec.seq, "cond_tokens": Mc, "sampler_steps": SAMPLER_STEPS,
                   "guidance": 3.0, "shift": 3.0, "global_batch": f"{images} image(s) x CFG pair",
                   "parallelism": parallelism_label(split, T, images, args.tp_reduce, SP),
                   "launch": "host-issued kernels" if args.no_graph else "one CUDA graph per sampler step",
                   "condition_path_ms_per_image": round(cond_ms, 3),
                   "value_formula": "(ms_per_step x 20 + condition_path_ms_per_image) / images",
                   "l2": "no flush: every step streams 1.4 GB of NF24 weights and ~1 GB of "
                         "activations, far above the 126 MB L2"},
        "tflops_logical_per_gpu": round(flops["total"] / (ms_step / 1e3) / 1e12, 1),
        "roofline": roofs[0],
        "roofline_second": roofs[1],
        "kernels": kernels,
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "finite": finite,
        **({"parity": parity} if parity is not None else {}),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(spec)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        sampler.graph = None  # release graphs before the process group goes
        torch.cuda.synchronize()
        barrier()
        if hasattr(model, "close"):
            model.close()  # IPC mappings of the peer reduction
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
