"""Prologue / epilogue kernels on CUDA tensors, through the reference-named C-ABI.

Each function mirrors the computation the reference's strict patch performs with
its AVX-512 kernel (scripts/native_norm_rope_avx512_patch.py,
native_gelu_avx512_patch.py, native_silu_avx512_patch.py,
native_block_elementwise_avx512_patch.py, native_sampler_avx512_backend.py,
native_qkv_packed_attention_patch_v3.py) and raises on any non-zero status.
"""
from __future__ import annotations

import _native


def _lib():
    lib = _native.load()
    _native.use_current_stream(lib)
    return lib


def _ok(status, name):
    if int(status) != 0:
        raise RuntimeError(f"{name} returned status {status}")


def _f32(t, name):
    import torch

    if t.device.type != "cuda" or t.dtype != torch.float32:
        raise ValueError(f"{name}: expected a CUDA float32 tensor")
    return t if t.is_contiguous() else t.contiguous()


def layernorm(x, weight=None, bias=None, eps: float = 1e-6, out=None):
    import torch

    x = _f32(x, "layernorm")
    cols = int(x.shape[-1])
    out = torch.empty_like(x) if out is None else out
    aff = weight is not None
    _ok(_lib().triposplat_layernorm_f32_avx512(
        x.data_ptr(), weight.data_ptr() if aff else None, bias.data_ptr() if aff else None,
        out.data_ptr(), x.numel() // cols, cols, float(eps), int(aff), 0), "layernorm")
    return out


def multihead_rmsnorm(x, gamma, eps: float = 1e-12, out=None):
    import torch

    x = _f32(x, "multihead_rmsnorm")
    heads, dim = int(gamma.shape[0]), int(gamma.shape[1])
    out = torch.empty_like(x) if out is None else out
    _ok(_lib().triposplat_multihead_rmsnorm_f32_avx512(
        x.data_ptr(), gamma.data_ptr(), out.data_ptr(), x.numel() // (heads * dim), heads, dim,
        float(eps), 0), "multihead_rmsnorm")
    return out


def rope_complex(x, freqs, out=None):
    import torch

    x = _f32(x, "rope")
    dim = int(x.shape[-1])
    out = torch.empty_like(x) if out is None else out
    _ok(_lib().triposplat_rope_complex_f32_avx512(
        x.data_ptr(), _f32(freqs, "rope freqs").data_ptr(), out.data_ptr(), x.numel() // dim, dim, 0),
        "rope")
    return out


def gelu_tanh(x, out=None):
    import torch

    x = _f32(x, "gelu")
    out = torch.empty_like(x) if out is None else out
    _ok(_lib().triposplat_gelu_tanh_f32_avx512(x.data_ptr(), out.data_ptr(), x.numel(), 0), "gelu")
    return out


def silu(x, out=None):
    import torch

    x = _f32(x, "silu")
    out = torch.empty_like(x) if out is None else out
    _ok(_lib().triposplat_silu_f32_avx512(x.data_ptr(), out.data_ptr(), x.numel(), 0), "silu")
    return out


def modulate_inplace(h, scale, shift):
    """h[b, l, c] = h * (1 + scale[b, c]) + shift[b, c]"""
    B, L, C = (int(s) for s in h.shape)
    _ok(_lib().triposplat_modulate_inplace_f32_avx512(
        _f32(h, "modulate").data_ptr(), _f32(scale, "scale").data_ptr(),
        _f32(shift, "shift").data_ptr(), B, L, C, 0), "modulate")
    return h


def gated_residual_inplace(base, delta, gate):
    """delta *= gate[b]; base += delta"""
    B, L, C = (int(s) for s in base.shape)
    _ok(_lib().triposplat_gated_residual_inplace_f32_avx512(
        _f32(base, "base").data_ptr(), _f32(delta, "delta").data_ptr(),
        _f32(gate, "gate").data_ptr(), B, L, C, 0), "gated_residual")
    return base


def add_inplace(base, delta):
    _ok(_lib().triposplat_add_inplace_f32_avx512(
        _f32(base, "base").data_ptr(), _f32(delta, "delta").data_ptr(), base.numel(), 0), "add")
    return base


def cfg_combine_inplace(positive, negative, guidance):
    B = int(positive.shape[0])
    _ok(_lib().triposplat_cfg_combine_inplace_f32_avx512(
        _f32(positive, "positive").data_ptr(), _f32(negative, "negative").data_ptr(),
        _f32(guidance, "guidance").data_ptr(), B, positive.numel() // B, 0), "cfg_combine")
    return positive


def euler_update_inplace(sample, prediction, dt):
    B = int(sample.shape[0])
    _ok(_lib().triposplat_euler_update_inplace_f32_avx512(
        _f32(sample, "sample").data_ptr(), _f32(prediction, "prediction").data_ptr(),
        _f32(dt, "dt").data_ptr(), B, sample.numel() // B, 0), "euler_update")
    return sample


def qkv_rope_rmsnorm_pack(qkv, freqs, q_gamma, k_gamma, L_padded=None):
    """qkv [B,L,3,H,64] -> q [B,H,L,64], packed k/v [B,H,64,Lp]."""
    import torch

    qkv = _f32(qkv, "qkv")
    B, L, _, H, D = (int(s) for s in qkv.shape)
    Lp = ((L + 15) // 16) * 16 if L_padded is None else int(L_padded)
    q = torch.empty((B, H, L, D), dtype=torch.float32, device=qkv.device)
    pk = torch.empty((B, H, D, Lp), dtype=torch.float32, device=qkv.device)
    pv = torch.empty((B, H, D, Lp), dtype=torch.float32, device=qkv.device)
    _ok(_lib().triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(
        qkv.data_ptr(), _f32(freqs, "freqs").data_ptr(), q_gamma.data_ptr(), k_gamma.data_ptr(),
        q.data_ptr(), pk.data_ptr(), pv.data_ptr(), B, L, H, D, Lp, int(freqs.shape[0]), 0),
        "qkv_rope_rmsnorm_pack")
    return q, pk, pv


def q_kv_selected_rope_rmsnorm_pack(q, kv, freqs, selected, q_gamma, k_gamma, Lk_padded=None):
    """q [B,Lq,H,64] (rows chosen by `selected` for RoPE), kv [B,Lk,2,H,64]."""
    import torch

    B, Lq, H, D = (int(s) for s in q.shape)
    Lk = int(kv.shape[1])
    Lp = ((Lk + 15) // 16) * 16 if Lk_padded is None else int(Lk_padded)
    qo = torch.empty((B, H, Lq, D), dtype=torch.float32, device=q.device)
    pk = torch.empty((B, H, D, Lp), dtype=torch.float32, device=q.device)
    pv = torch.empty((B, H, D, Lp), dtype=torch.float32, device=q.device)
    _ok(_lib().triposplat_q_kv_selected_rope_rmsnorm_pack_f32_avx512_v2(
        _f32(q, "q").data_ptr(), _f32(kv, "kv").data_ptr(), _f32(freqs, "freqs").data_ptr(),
        selected.data_ptr(), q_gamma.data_ptr(), k_gamma.data_ptr(), qo.data_ptr(), pk.data_ptr(),
        pv.data_ptr(), B, Lq, Lk, H, D, Lp, int(freqs.shape[0]), 0), "q_kv_selected_pack")
    return qo, pk, pv
