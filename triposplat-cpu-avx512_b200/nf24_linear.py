"""Functional NF24 Linear on CUDA tensors, through the C-ABI.

``nf24_linear(x, code01_t, q2_t, scale, bias)`` is ``F.linear(x, W)`` with
``W = dequant(codes)``; it calls ``triposplat_gemm_rnf8_avx512`` (N % 16 == 0),
``..._tail`` (any N) or ``..._range`` (a column window), exactly as the
reference's patched ``nn.Linear.forward`` selects its kernel
(scripts/native_linear_rnf8_avx512_patch.py:309-361).
"""
from __future__ import annotations

import ctypes

import _native

_CODEBOOK = {}


def _codebook(device):
    import torch

    key = str(device)
    if key not in _CODEBOOK:
        # the NF24 kernel never reads it; the ABI still wants a non-null pointer
        _CODEBOOK[key] = torch.zeros(256, dtype=torch.float32, device=device)
    return _CODEBOOK[key]


def nf24_linear(x, code01_t, q2_t, scale, bias, *, out=None, start: int = 0,
                count: int | None = None, lib=None):
    import torch

    lib = lib or _native.load()
    K, N = int(code01_t.shape[0]), int(code01_t.shape[1])
    if int(x.shape[-1]) != K:
        raise ValueError(f"input features {x.shape[-1]} != {K}")
    if x.dtype != torch.float32:
        raise ValueError("NF24 Linear takes float32 activations")
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    _native.require_cuda(x2, code01_t, q2_t, scale, bias, what="nf24_linear operand")
    M = int(x2.shape[0])
    ranged = start != 0 or count is not None
    count = N - start if count is None else int(count)
    if out is None:
        out = torch.empty((M, count), dtype=torch.float32, device=x.device)
    elif not out.is_contiguous() or out.numel() != M * count or out.dtype != torch.float32:
        raise ValueError("out must be a contiguous float32 tensor of M x count elements")
    cb = _codebook(x.device)
    _native.use_current_stream(lib)
    ptrs = (x2.data_ptr(), code01_t.data_ptr(), q2_t.data_ptr(), q2_t.data_ptr(),
            scale.data_ptr(), scale.data_ptr(), scale.data_ptr(), cb.data_ptr(),
            bias.data_ptr(), out.data_ptr())
    if ranged:
        st = lib.triposplat_gemm_rnf8_avx512_range(*ptrs, M, K, N, start, count, K, count, 0, 3)
    elif N % 16:
        st = lib.triposplat_gemm_rnf8_avx512_tail(*ptrs, M, K, N, K, N, 0, 3)
    else:
        st = lib.triposplat_gemm_rnf8_avx512(*ptrs, M, K, N, K, N, 0, 3)
    if st != 0:
        raise RuntimeError(f"NF24 GEMM returned status {st} for M={M} K={K} N={N}: "
                           f"{lib.triposplat_b200_last_error().decode()}")
    return out.view(*x.shape[:-1], count)
