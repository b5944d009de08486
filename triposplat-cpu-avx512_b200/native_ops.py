"""Prologue / epilogue kernels on CUDA tensors, through the reference-named C-ABI.

Each function mirrors the computation the reference's strict patch performs with
its AVX-512 kernel (scripts/native_norm_rope_avx512_patch.py,
native_gelu_avx512_patch.py, native_silu_avx512_patch.py,
native_block_elementwise_avx512_patch.py, native_sampler_avx512_backend.py,
native_qkv_packed_attention_patch_v3.py, native_embeddings_avx512_patch.py,
native_repo_avx512_patch.py) and raises on any non-zero status.
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


def timestep_embedding(timesteps, frequencies, output_dim=None):
    """[batch] timesteps, [half] frequencies -> [batch, output_dim] = [cos | sin | 0 ...]
    (scripts/native_embeddings_avx512_patch.py:76-97)."""
    import torch

    t, f = _f32(timesteps, "timestep_embedding"), _f32(frequencies, "timestep_embedding")
    half = int(f.numel())
    output_dim = 2 * half if output_dim is None else int(output_dim)
    out = torch.empty((int(t.numel()), output_dim), dtype=torch.float32, device=t.device)
    _ok(_lib().triposplat_timestep_embedding_f32_avx512(
        t.data_ptr(), f.data_ptr(), out.data_ptr(), int(t.numel()), half, output_dim, 0),
        "timestep_embedding")
    return out


def pcd_position_embedding(positions, frequencies, channels, double_pi=False):
    """positions [..., dims] -> [..., channels]: per axis [sin | cos] of x*f(*2)*pi, zero pad
    (scripts/native_embeddings_avx512_patch.py, point-cloud position embedder)."""
    import torch

    x, f = _f32(positions, "pcd_position_embedding"), _f32(frequencies, "pcd_position_embedding")
    dims = int(x.shape[-1])
    rows = x.numel() // dims
    out = torch.empty((*x.shape[:-1], int(channels)), dtype=torch.float32, device=x.device)
    _ok(_lib().triposplat_pcd_position_embedding_f32_avx512(
        x.data_ptr(), f.data_ptr(), out.data_ptr(), rows, dims, int(f.numel()), int(channels),
        int(bool(double_pi)), 0), "pcd_position_embedding")
    return out


def mul_inplace(lhs, rhs):
    """lhs *= rhs (the RePo gate * content product, scripts/native_repo_avx512_patch.py:55-66)."""
    lhs, rhs = _f32(lhs, "mul_inplace"), _f32(rhs, "mul_inplace")
    if lhs.shape != rhs.shape:
        raise ValueError("mul_inplace: shapes differ")
    _ok(_lib().triposplat_mul_inplace_f32_avx512(lhs.data_ptr(), rhs.data_ptr(), lhs.numel(), 0),
        "mul_inplace")
    return lhs


def repo_phasor(delta, frequencies):
    """RePo 3-D rotary phasors (scripts/native_repo_avx512_patch.py:68-105): delta
    [B, L, 3 * heads] and the three per-axis frequency vectors f_a -> complex64
    [B, L, heads, sum(dims)] with angle (x*tanh(f) + x*(f - tanh(f))) * pi per axis."""
    import torch

    d = _f32(delta, "repo_phasor")
    if d.ndim != 3 or int(d.shape[-1]) % 3:
        raise ValueError("repo_phasor: delta must be [B, L, 3 * heads]")
    parts = []
    for f in frequencies:
        f = _f32(f.reshape(-1), "repo_phasor")
        ft = torch.tanh(f).contiguous()
        parts.append((ft, (f - ft).contiguous()))
    dims = [int(p[0].numel()) for p in parts]
    B, L, heads = int(d.shape[0]), int(d.shape[1]), int(d.shape[2]) // 3
    out = torch.empty((B, L, heads, sum(dims)), dtype=torch.complex64, device=d.device)
    _ok(_lib().triposplat_repo_phasor_f32_avx512(
        d.data_ptr(), parts[0][0].data_ptr(), parts[0][1].data_ptr(), dims[0],
        parts[1][0].data_ptr(), parts[1][1].data_ptr(), dims[1],
        parts[2][0].data_ptr(), parts[2][1].data_ptr(), dims[2],
        out.data_ptr(), B * L * heads, 0), "repo_phasor")
    return out
