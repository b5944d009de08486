"""The attention softmax's FMA-pipe 2^x (csrc/sdpa.cu exp2_poly2), checked on the CPU.

The coefficients in the kernel source are those csrc/gen_exp2_poly.py computes (Remez
minimax of the relative error of 2^f on [-1/2, 1/2], degree 5); evaluated as the kernel
does — clamp at -125, j = round-to-nearest(x) via the 1.5 * 2^23 addition, f = x - j,
float32 Horner with fused multiply-adds, 2^j added to the exponent field — the relative
error against exp2 stays within 2.5e-7 over the softmax's whole argument range, the order
of the MUFU ex2.approx it stands in for.
"""
import re
import sys
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parent.parent / "triposplat-cpu-avx512_b200" / "csrc"


def _kernel_coefficients():
    src = (CSRC / "sdpa.cu").read_text()
    body = src[src.index("void exp2_poly2"):]
    body = body[:body.index("\n}\n")]
    hexes = re.findall(r"f2pack\((0x[0-9a-fp.+-]+)f, \1f\)", body)
    return [np.float32(float.fromhex(h)) for h in hexes]  # highest degree first


def _fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def _exp2_poly(x):
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)
    c = _kernel_coefficients()
    r = np.full(x.shape, c[0], np.float32)
    for ck in c[1:]:
        r = _fma32(r, f, np.full(x.shape, ck, np.float32))
    bits = (r.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_kernel_coefficients_are_the_generated_minimax():
    sys.path.insert(0, str(CSRC))
    import gen_exp2_poly

    gen = gen_exp2_poly.remez_exp2(5).astype(np.float32)[::-1]
    assert [float(v) for v in _kernel_coefficients()] == [float(v) for v in gen]


def test_relative_error_over_the_softmax_range():
    x = np.concatenate([np.linspace(-125.0, 16.0, 1 << 22, dtype=np.float32),
                        np.linspace(-1.0, 1.0, 1 << 20, dtype=np.float32)])
    got = _exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert np.isfinite(got).all() and rel.max() <= 2.5e-7, rel.max()
    # below the clamp the result is 2^-125 order, far under what the fp16 P planes keep
    low = _exp2_poly(np.array([-200.0, -1e30], np.float32))
    assert (low > 0).all() and (low < 2.0 ** -124).all()
