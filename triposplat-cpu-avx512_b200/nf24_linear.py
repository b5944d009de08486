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


def _status(lib, st, what):
    if st != 0:
        raise RuntimeError(f"{what} returned status {st}: {lib.triposplat_b200_last_error().decode()}")


def nf24_mlp_gelu(x, w1, w2, *, out=None, chunk_rows: int | None = None, hidden=None, lib=None):
    """fc2(GELU_tanh(fc1(x))) with NF24 weights through the reference's fused MLP entry
    (``triposplat_mlp_nf24_gelu_f32_avx512``, scripts/native_nf24_mlp_avx512.c:143-205; with
    ``chunk_rows`` the chunked entry, scripts/native_nf24_mlp_chunked_avx512.c:3-60, whose
    hidden buffer [>= chunk_rows, 4096] is ``hidden`` or allocated here).

    x: [M, 1024] float32 rows, any row stride >= 1024 (a 2-D view with unit column stride);
    w1 / w2: (code01_t, q2_t, scale, bias) of the 1024 -> 4096 and 4096 -> 1024 Linears;
    out: optional [M, 1024] float32 2-D view (row stride >= 1024)."""
    import torch

    lib = lib or _native.load()
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype != torch.float32:
        raise ValueError("x must be a 2-D float32 tensor with unit column stride")
    M = int(x.shape[0])
    (c1, q1, s1, b1), (c2, q2, s2, b2) = w1, w2
    K, H, N = int(c1.shape[0]), int(c1.shape[1]), int(c2.shape[1])
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    if out.dim() != 2 or out.stride(1) != 1 or out.dtype != torch.float32:
        raise ValueError("out must be a 2-D float32 tensor with unit column stride")
    if x.device.type != "cuda" or out.device.type != "cuda":
        raise ValueError("nf24_mlp_gelu: x and out must be CUDA tensors")
    _native.require_cuda(c1, q1, s1, b1, c2, q2, s2, b2, hidden, what="nf24_mlp_gelu operand")
    _native.use_current_stream(lib)
    ptrs = (x.data_ptr(), c1.data_ptr(), q1.data_ptr(), s1.data_ptr(), b1.data_ptr(),
            c2.data_ptr(), q2.data_ptr(), s2.data_ptr(), b2.data_ptr())
    if chunk_rows is None:
        st = lib.triposplat_mlp_nf24_gelu_f32_avx512(*ptrs, out.data_ptr(), M, K, H, N,
                                                     int(x.stride(0)), int(out.stride(0)), 0)
    else:
        if hidden is None:
            hidden = torch.empty((int(chunk_rows), H), dtype=torch.float32, device=x.device)
        st = lib.triposplat_mlp_nf24_gelu_chunked_f32_avx512(
            *ptrs, hidden.data_ptr(), out.data_ptr(), M, K, H, N, int(x.stride(0)),
            int(out.stride(0)), int(hidden.shape[0]), int(chunk_rows), 0)
    _status(lib, st, "NF24 MLP")
    return out


def nf24_qkv_rope_rmsnorm_pack(x, code01_t, q2_t, scale, bias, freqs, q_gamma, k_gamma, *,
                               batch: int, heads: int, L_padded: int | None = None, lib=None):
    """The QKV projection with its RoPE / per-head RMSNorm / pack epilogue through
    ``triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512``
    (scripts/gemm_nf24_qkv_direct_avx512.c:87-199).

    x: [batch * L, K] contiguous float32; weight [K, 3 * heads * 64]; freqs
    [1 or batch, L, heads, 64] (interleaved cos / sin).  Returns q [B, H, L, 64] and the
    packed k / v [B, H, 64, L_padded] (zero tail)."""
    import torch

    lib = lib or _native.load()
    if not x.is_contiguous() or x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError("x must be a contiguous 2-D float32 tensor")
    M, K = (int(d) for d in x.shape)
    B, H, D = int(batch), int(heads), 64
    if M % B:
        raise ValueError("rows are not a multiple of the batch")
    L = M // B
    N = int(code01_t.shape[1])
    Lp = ((L + 15) // 16) * 16 if L_padded is None else int(L_padded)
    dev = x.device
    q = torch.empty((B, H, L, D), dtype=torch.float32, device=dev)
    pk = torch.empty((B, H, D, Lp), dtype=torch.float32, device=dev)
    pv = torch.empty((B, H, D, Lp), dtype=torch.float32, device=dev)
    _native.require_cuda(x, code01_t, q2_t, scale, bias, freqs, q_gamma, k_gamma,
                         what="nf24_qkv_rope_rmsnorm_pack operand")
    cb = _codebook(dev)
    _native.use_current_stream(lib)
    st = lib.triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512(
        x.data_ptr(), code01_t.data_ptr(), q2_t.data_ptr(), q2_t.data_ptr(), scale.data_ptr(),
        scale.data_ptr(), scale.data_ptr(), cb.data_ptr(), bias.data_ptr(), freqs.data_ptr(),
        q_gamma.data_ptr(), k_gamma.data_ptr(), q.data_ptr(), pk.data_ptr(), pv.data_ptr(),
        B, L, K, N, H, D, Lp, int(freqs.shape[0]), 0, 3)
    _status(lib, st, "NF24 QKV projection")
    return q, pk, pv
