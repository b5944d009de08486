"""Exact SDPA through the C-ABI, mirroring the reference's ``native_sdpa_ctypes``.

``native_sdpa_f32(q, k, v, key_bias=None)`` has the reference's signature,
argument checks and error behaviour (scripts/native_sdpa_ctypes.py:23-76):
``[B,H,L,64]`` tensors, an optional key bias of ``Lk`` elements shared by every
(b, h), a RuntimeError on any non-zero status.  The tensors are CUDA tensors
and the library / symbol come from ``TRIPOSPLAT_NATIVE_SDPA_LIBRARY`` /
``TRIPOSPLAT_NATIVE_SDPA_SYMBOL`` exactly as in the reference (defaulting to
this package's library and ``triposplat_sdpa_f32_avx512_exact_q8t512``).

Extensions with no reference counterpart: a per-(b, h) bias of shape
``[B, H, Lk]`` and a BLHD output (``out_blhd=True``), both through
``triposplat_sdpa_f32_cuda_bias_bh``.
"""
from __future__ import annotations

import ctypes
import os
from functools import lru_cache
from pathlib import Path

import _native

DEFAULT_SYMBOL = "triposplat_sdpa_f32_avx512_exact_q8t512"


@lru_cache(maxsize=4)
def _load_kernel(path: str, symbol: str):
    lib = _native.load(path)
    fn = getattr(lib, symbol)
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 8
    fn.restype = ctypes.c_int
    return lib, fn


def native_sdpa_f32(q, k, v, *, key_bias=None, library=None, symbol=None, threads=None,
                    out_blhd: bool = False):
    import torch

    if q.device.type != "cuda" or k.device.type != "cuda" or v.device.type != "cuda":
        raise ValueError("CUDA SDPA takes CUDA tensors")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q/k/v must be [B,H,L,D]")
    if q.shape[:2] != k.shape[:2] or k.shape != v.shape:
        raise ValueError(f"unsupported q/k/v shapes: q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if int(q.shape[-1]) != 64 or int(k.shape[-1]) != 64:
        raise ValueError("exact SDPA requires head_dim=64")
    orig_dtype = q.dtype
    q_f = q.to(dtype=torch.float32).contiguous()
    k_f = k.to(dtype=torch.float32).contiguous()
    v_f = v.to(dtype=torch.float32).contiguous()
    B, H, Lq, Lk = int(q_f.shape[0]), int(q_f.shape[1]), int(q_f.shape[2]), int(k_f.shape[2])
    bias_f = None
    per_bh = False
    if key_bias is not None:
        if key_bias.device.type != "cuda":
            raise ValueError("key bias must be a CUDA tensor")
        if int(key_bias.numel()) == Lk:
            bias_f = key_bias.to(dtype=torch.float32).reshape(-1).contiguous()
        elif tuple(key_bias.shape) == (B, H, Lk):
            bias_f = key_bias.to(dtype=torch.float32).contiguous()
            per_bh = True
        else:
            raise ValueError(f"key bias length mismatch: bias={key_bias.numel()} keys={Lk}")
    shape = (B, Lq, H, 64) if out_blhd else (B, H, Lq, 64)
    out = torch.empty(shape, dtype=torch.float32, device=q.device)
    lib_path = _native.library_path(library or os.environ.get("TRIPOSPLAT_NATIVE_SDPA_LIBRARY"))
    symbol_name = symbol or os.environ.get("TRIPOSPLAT_NATIVE_SDPA_SYMBOL", DEFAULT_SYMBOL)
    lib, fn = _load_kernel(str(lib_path), symbol_name)
    _native.use_current_stream(lib)
    if per_bh or out_blhd:
        status = int(lib.triposplat_sdpa_f32_cuda_bias_bh(
            q_f.data_ptr(), k_f.data_ptr(), v_f.data_ptr(),
            None if bias_f is None else bias_f.data_ptr(), Lk if per_bh else 0,
            out.data_ptr(), B, H, Lq, Lk, int(out_blhd)))
    else:
        status = int(fn(
            q_f.data_ptr(), k_f.data_ptr(), v_f.data_ptr(),
            0 if bias_f is None else bias_f.data_ptr(), out.data_ptr(),
            B, H, Lq, Lk, 64, int(bias_f is not None),
            0 if bias_f is None else int(bias_f.numel()), int(threads or 0)))
    if status != 0:
        raise RuntimeError(
            f"CUDA exact SDPA returned status {status}; "
            f"q={tuple(q_f.shape)} k={tuple(k_f.shape)} bias={bias_f is not None}")
    return out.to(dtype=orig_dtype)


def native_sdpa_packed_blhd(q, packed_k, packed_v, Lk: int, *, key_bias=None, library=None):
    """Packed K/V ``[B,H,64,Lkp]`` in, ``[B,Lq,H,64]`` out
    (scripts/native_sdpa_avx512_exact_q8t512_packed.c:3-158)."""
    import torch

    B, H, Lq = int(q.shape[0]), int(q.shape[1]), int(q.shape[2])
    Lkp = int(packed_k.shape[-1])
    _native.require_cuda(q, packed_k, packed_v, key_bias, what="packed SDPA operand")
    out = torch.empty((B, Lq, H, 64), dtype=torch.float32, device=q.device)
    lib = _native.load(library)
    _native.use_current_stream(lib)
    st = int(lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
        q.data_ptr(), packed_k.data_ptr(), packed_v.data_ptr(),
        0 if key_bias is None else key_bias.data_ptr(), out.data_ptr(),
        B, H, Lq, int(Lk), 64, Lkp, int(key_bias is not None),
        0 if key_bias is None else int(key_bias.numel()), 0))
    if st != 0:
        raise RuntimeError(f"CUDA packed SDPA returned status {st}")
    return out
