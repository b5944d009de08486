"""NF24 int16 weight packer (load-time, host side).

Produces the on-disk/in-memory contract the GEMM consumes, unchanged from the
reference so that shards packed by either side are interchangeable:

* ``code01_t``  int16 ``[in, out]`` = ``4*q0 + q1``
* ``q2_t``      int8  ``[in, out]``
* ``scale``     f32   ``[out]``     = ``max|w_row| / 127 / 1024``

and ``W[n, k] ~= scale[n] * (256*code01_t[k, n] + q2_t[k, n])``.

Algorithm (scripts/native_linear_rnf8_avx512_patch.py:14-87 of the reference):
per output row the base step is ``s = max|w| / 127``; ``q0`` is the nearest
member of the integer alphabet ``unique(round(127 * NF8))`` (ties resolved by
``bucketize`` on the midpoints); the first residual is coded as
``q1 = clamp(floor(r1 / (s/4) + 0.5), -128, 127)`` and the second as
``q2 = clamp(floor(r2 / (s/1024) + 0.5), -128, 127)``.
The NF8 codebook is the 255 normal quantiles plus a duplicate zero, normalised
to max 1 (scripts/native_linear_nf8_avx512_patch.py:12-20).

The steps are kept in the same order and precision as the reference because
the codes must be bit-identical; tests/test_pack.py pins them against golden
codes produced by the reference packer.
"""
from __future__ import annotations

import math
from typing import Any


def make_nf8_codebook(torch):
    """256-entry symmetric normal-float codebook (float32, sorted)."""
    p = (torch.arange(255, dtype=torch.float64) + 0.5) / 255.0
    levels = math.sqrt(2.0) * torch.erfinv(2.0 * p - 1.0)
    levels = levels / levels.abs().max()
    with_zero = torch.cat((levels, torch.zeros(1, dtype=torch.float64)))
    return torch.sort(with_zero)[0].float().contiguous()


def _stage_stats(torch, remaining, unclamped) -> dict[str, Any]:
    return {
        "residual_rmse": float(torch.sqrt(torch.mean(remaining * remaining)).item()),
        "residual_max_abs": float(remaining.abs().max().item()),
        "saturated_values": 0 if unclamped is None
        else int(((unclamped < -128) | (unclamped > 127)).sum().item()),
    }


def quantize_nf24_i16_per_output_channel(weight, codebook=None):
    """Pack an ``[out, in]`` float32 CPU weight into the NF24 int16 layout.

    Returns ``([code01_t, q2_t, q2_t], [scale, scale, scale], error)`` — the same
    triple-of-stages shape the reference's patch layer binds (codes1 and codes2
    both alias ``q2_t``; the three scales alias one tensor).
    """
    import torch

    if weight.device.type != "cpu" or weight.dtype != torch.float32 or weight.ndim != 2:
        raise ValueError("NF24 packing requires a CPU float32 2D weight")
    return quantize_nf24_i16_any_device(weight, codebook)


def quantize_nf24_i16_any_device(weight, codebook=None, stats: bool = True):
    """Same packing on any device.  Every step is an exactly rounded elementwise op, a
    comparison or a sort, so CUDA and CPU produce bit-identical codes (checked by
    tests/test_model_gpu.py); used to pack synthetic weights where they are generated."""
    import torch

    if weight.dtype != torch.float32 or weight.ndim != 2:
        raise ValueError("NF24 packing requires a float32 2D weight")
    if codebook is None:
        codebook = make_nf8_codebook(torch)
    codebook = codebook.to(weight.device)
    w = weight.detach().contiguous()
    tiny = torch.finfo(torch.float32).tiny
    # the per-row step is divided on the host: CUDA tensor-by-scalar division is not
    # always correctly rounded, and every code depends on this value
    step0 = (w.abs().amax(dim=1).clamp_min(tiny).cpu() / 127.0).to(w.device).contiguous()

    alphabet = torch.unique(torch.round(codebook * 127.0).clamp_(-127, 127)).to(torch.float32)
    mids = ((alphabet[:-1] + alphabet[1:]) * 0.5).contiguous()
    q0 = alphabet[torch.bucketize(w / step0[:, None], mids)].to(torch.int8)
    r1 = w - q0.to(torch.float32) * step0[:, None]

    step1 = step0 / 4.0
    q1_raw = torch.floor(r1 / step1[:, None] + 0.5)
    q1 = q1_raw.clamp(-128, 127).to(torch.int8)
    r2 = r1 - q1.to(torch.float32) * step1[:, None]

    scale = (step0 / 1024.0).contiguous()
    q2_raw = torch.floor(r2 / scale[:, None] + 0.5)
    q2 = q2_raw.clamp(-128, 127).to(torch.int8)
    r3 = r2 - q2.to(torch.float32) * scale[:, None]

    code01_t = (q0.t().to(torch.int16) * 4 + q1.t().to(torch.int16)).contiguous()
    q2_t = q2.t().contiguous()
    if not stats:
        return [code01_t, q2_t, q2_t], [scale, scale, scale], None
    stages = []
    for idx, (rem, name, raw) in enumerate(
        ((r1, "nf8_derived_int8_alphabet", None),
         (r2, "shared_scale_int8_radix4", q1_raw),
         (r3, "shared_scale_int8_radix256", q2_raw)), start=1):
        stages.append({"stage": idx, "quantizer": name, **_stage_stats(torch, rem, raw)})
    rms = float(torch.sqrt(torch.mean(w * w)).item())
    error = {
        "weight_rmse": stages[-1]["residual_rmse"],
        "weight_max_abs": stages[-1]["residual_max_abs"],
        "weight_rms": rms,
        "weight_relative_rmse": stages[-1]["residual_rmse"] / max(rms, 1.0e-30),
        "residual_mode": "nf24_i16",
        "storage_layout": "int16(q0*4+q1) + int8(q2)",
        "nf8_derived_alphabet_size": int(alphabet.numel()),
        "stages": stages,
    }
    return [code01_t, q2_t, q2_t], [scale, scale, scale], error


def dequantize_nf24_i16(code01_t, q2_t, scale):
    """Float32 ``[out, in]`` weight the codes stand for: ``(256*q01 + q2) * scale``."""
    import torch

    combined = code01_t.to(torch.int32) * 256 + q2_t.to(torch.int32)
    return (combined.to(torch.float32) * scale[None, :]).t().contiguous()
