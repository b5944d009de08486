"""The reference's patch layer on CUDA: the patched modules run this library's kernels.

1. The reference's prepacked smoke test (scripts/smoke_nf24_prepacked.py:17-95) on the GPU:
   a ToyModel checkpoint is packed, resumed, loaded onto the device, patched with
   ``apply_triposplat_native_rnf8_avx512_patch`` and compared with the float model
   (gate: rmse < 1e-4, max_abs < 5e-4, fallbacks 0, checkpoint never loaded).
2. A small flow model with the upstream class names the reference's patchers key on
   (``UnifiedTransformerBlock``, ``RopeMultiHeadAttention``, ``MultiHeadRMSNorm``, GELU(tanh),
   SiLU, LayerNorm, the ``apply_rotary_emb`` of a ``model`` module and the attention helpers
   of a ``triposplat_attention_patch`` module), written here in plain PyTorch.  With every
   patcher applied the CUDA forward, the key-bias helper and the selected-query helper are
   compared against the same PyTorch code run in float64 on the dequantised weights
   (relative rmse <= 1e-5), with zero fallbacks.
"""
import math
import tempfile
import types
from pathlib import Path

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


class ToyModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(96, 64, bias=True)
        self.norm = nn.LayerNorm(64)
        self.fc2 = nn.Linear(64, 17, bias=False)

    def forward(self, x):
        return self.fc2(torch.tanh(self.norm(self.fc1(x))))


def test_prepacked_toy_model_round_trip_on_cuda():
    from safetensors.torch import save_file

    from native_patches import apply_triposplat_native_rnf8_avx512_patch
    from nf24_shards import load_nf24_i16_prepacked_model, pack_nf24_i16_checkpoint

    torch.manual_seed(0)
    source = ToyModel().eval()
    x = torch.randn(25, 96, dtype=torch.float32)
    reference = source(x).detach()
    with tempfile.TemporaryDirectory(prefix="triposplat-nf24-cuda-") as tmp:
        root = Path(tmp)
        ckpt = root / "toy.safetensors"
        save_file(source.state_dict(), ckpt.as_posix())
        manifest = pack_nf24_i16_checkpoint(ckpt, root / "packed", expected_linear_count=2)
        assert pack_nf24_i16_checkpoint(ckpt, root / "packed", expected_linear_count=2) == manifest
        loaded = load_nf24_i16_prepacked_model(root / "packed", ToyModel, verify_checksums=True,
                                               device="cuda").eval()
        meta = apply_triposplat_native_rnf8_avx512_patch(
            loaded, enabled=True, include_regex=r".*", threads=2, strict=True, stages=3,
            residual_mode="nf24_i16")
        with torch.inference_mode():
            observed = loaded(x.cuda()).cpu()
    diff = observed - reference
    rmse = torch.sqrt(torch.mean(diff.square())).item()
    max_abs = diff.abs().max().item()
    assert manifest["linear_count"] == 2
    assert meta["selected_count"] == 2
    assert meta["runtime"]["fallbacks"] == 0 and meta["runtime"]["calls"] == 2
    assert meta["prepacked_load"]["source_checkpoint_loaded"] is False
    assert rmse < 1.0e-4 and max_abs < 5.0e-4, (rmse, max_abs)


# ---------------------------------------------------------------------------------------
# a small flow model in the upstream module structure, in plain PyTorch
# ---------------------------------------------------------------------------------------
def _apply_rotary_emb(x, freqs):
    """x [.., L, H, D] real, freqs [Fb, L, H, D/2] complex: interleaved complex rotation."""
    xc = torch.view_as_complex(x.reshape(*x.shape[:-1], -1, 2).to(torch.float64).contiguous())
    out = torch.view_as_real(xc * freqs.to(torch.complex128)).flatten(-2)
    return out.to(x.dtype)


def _sdpa(q, k, v, bias=None):
    """q [B, Lq, H, D], k / v [B, Lk, H, D] -> [B, Lq, H, D]; scale 1/8, optional [Lk] bias."""
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * 0.125
    if bias is not None:
        s = s + bias.to(s.dtype)
    return torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, dim=-1), v)


def _make_modules():
    mdl = types.ModuleType("model")
    mdl.apply_rotary_emb = _apply_rotary_emb
    tap = types.ModuleType("triposplat_attention_patch")

    def qk(attn, x, rope_emb, freqs_q=None):
        b, length, c = x.shape
        qkv = attn.qkv(x).view(b, length, 3, attn.num_heads, attn.head_dim)
        q, k, v = qkv.unbind(2)
        q = attn.q_norm(mdl.apply_rotary_emb(q.contiguous(), rope_emb if freqs_q is None else freqs_q))
        k = attn.k_norm(mdl.apply_rotary_emb(k.contiguous(), rope_emb))
        return q, k, v

    def standard(attn, x, rope_emb, *, backend="default", compute_dtype="model", query_chunk_size=128,
                 contiguous_qkv=True, timing_callback=None):
        q, k, v = qk(attn, x, rope_emb)
        return attn.out(_sdpa(q, k, v).reshape(x.shape))

    def key_bias(attn, x, rope_emb, key_bias, *, backend="default", timing_callback=None):
        q, k, v = qk(attn, x, rope_emb)
        return attn.out(_sdpa(q, k, v, key_bias.reshape(-1)).reshape(x.shape))

    def selected(attn, x, selected_idx, rope_emb, *, backend, compute_dtype, query_chunk_size,
                 round_qkv_to_fp16=False, round_v_to_fp16=False, round_attn_core_to_fp16=False,
                 half_sequence=False, key_bias=None, timing_callback=None):
        q, k, v = qk(attn, x, rope_emb)
        q = q[:, selected_idx]
        o = _sdpa(q, k, v)
        return attn.out(o.reshape(x.shape[0], -1, x.shape[-1]))

    def modulate(h, scale, shift):
        h.mul_(1 + scale.unsqueeze(1))
        h.add_(shift.unsqueeze(1))
        return h

    def residual(x, h, gate):
        h.mul_(gate.unsqueeze(1))
        x.add_(h)
        return x

    tap._rope_self_attention_standard = standard
    tap._rope_self_attention_with_key_bias = key_bias
    tap._rope_self_attention_selected_rows = selected
    tap._modulate_inplace_preserve_order = modulate
    tap._residual_gate_inplace_preserve_order = residual
    return mdl, tap


class MultiHeadRMSNorm(nn.Module):
    def __init__(self, heads, dim):
        super().__init__()
        self.gamma = nn.Parameter(1.0 + 0.02 * torch.randn(heads, dim))

    def forward(self, x):
        n = x.norm(dim=-1, keepdim=True).clamp_min(1e-12)
        return x * (math.sqrt(x.shape[-1]) / n) * self.gamma


class RopeMultiHeadAttention(nn.Module):
    def __init__(self, c, heads, tap):
        super().__init__()
        self._type, self.use_rope, self.qk_rms_norm = "self", True, True
        self.num_heads, self.head_dim = heads, c // heads
        self.qkv = nn.Linear(c, 3 * c)
        self.out = nn.Linear(c, c)
        self.q_norm = MultiHeadRMSNorm(heads, self.head_dim)
        self.k_norm = MultiHeadRMSNorm(heads, self.head_dim)
        self._tap = tap  # the helper module this model calls (float32 CUDA or float64 reference)

    def forward(self, x, rope_emb=None):
        return self._tap._rope_self_attention_standard(self, x, rope_emb, backend="native_avx512_exact",
                                                       compute_dtype="model")


class Mlp(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.fc1 = nn.Linear(c, 4 * c)
        self.act = nn.GELU(approximate="tanh")
        self.fc2 = nn.Linear(4 * c, c)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


class UnifiedTransformerBlock(nn.Module):
    def __init__(self, c, heads, tap):
        super().__init__()
        self.modulation, self.share_mod = True, False
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(c, 6 * c))
        self.shift_table = nn.Parameter(0.02 * torch.randn(2, 6 * c))  # [B, 6C], as mod
        self.norm1 = nn.LayerNorm(c, elementwise_affine=False, eps=1e-6)
        self.norm2 = nn.LayerNorm(c, elementwise_affine=False, eps=1e-6)
        self.attn = RopeMultiHeadAttention(c, heads, tap)
        self.mlp = Mlp(c)
        self._tap = tap

    def forward(self, x, mod=None, rotary_emb=None):
        mod = self.adaLN_modulation(mod) + self.shift_table
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (c.contiguous() for c in mod.chunk(6, 1))
        h = self._tap._modulate_inplace_preserve_order(self.norm1(x), scale_msa, shift_msa)
        x = self._tap._residual_gate_inplace_preserve_order(x, self.attn(h, rope_emb=rotary_emb), gate_msa)
        h = self._tap._modulate_inplace_preserve_order(self.norm2(x), scale_mlp, shift_mlp)
        return self._tap._residual_gate_inplace_preserve_order(x, self.mlp(h), gate_mlp)


class SmallFlow(nn.Module):
    def __init__(self, c, heads, tap, blocks=2):
        super().__init__()
        self.blocks = nn.ModuleList([UnifiedTransformerBlock(c, heads, tap) for _ in range(blocks)])
        self.final_norm = nn.LayerNorm(c, eps=1e-6)
        self.head = nn.Linear(c, 7)

    def forward(self, x, temb, freqs):
        for blk in self.blocks:
            x = blk(x, temb, freqs)
        return self.head(self.final_norm(x))


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt())


def test_all_patchers_on_a_small_flow_model():
    import native_patches as npt
    from nf24_pack import dequantize_nf24_i16

    C, H, L, B = 128, 2, 40, 2
    mdl, tap = _make_modules()
    mdl64, tap64 = _make_modules()
    torch.manual_seed(3)
    gpu = SmallFlow(C, H, tap).eval().cuda()
    torch.manual_seed(3)
    ref = SmallFlow(C, H, tap64).eval()  # same initial weights; float64 reference below
    x = torch.randn(B, L, C)
    temb = torch.randn(B, C)
    ang = torch.randn(1, L, H, 32, dtype=torch.float64)
    freqs = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    key_bias = torch.randn(L)
    sel = torch.tensor([0, 3, 4, 17, 39], dtype=torch.int64)

    metas = {
        "linear": npt.apply_triposplat_native_rnf8_avx512_patch(gpu, enabled=True, stages=3,
                                                                residual_mode="nf24_i16"),
        "norm": npt.apply_triposplat_native_norm_rope_avx512_patch(gpu, enabled=True, rope_module=mdl),
        "gelu": npt.apply_triposplat_native_gelu_avx512_patch(gpu, enabled=True),
        "silu": npt.apply_triposplat_native_silu_avx512_patch(gpu, enabled=True),
        "block": npt.apply_triposplat_native_block_elementwise_avx512_patch(gpu, enabled=True,
                                                                            attention_module=tap),
        "attn": npt.apply_triposplat_native_qkv_packed_attention_helpers_patch(gpu, attention_module=tap),
    }
    assert metas["attn"]["selected_count"] == 2 and metas["block"]["selected_count"] == 2
    assert metas["linear"]["selected_count"] == 2 * 5 + 1

    # float64 reference on the weights the codes stand for
    ref = ref.double()
    for name, m in gpu.named_modules():
        if isinstance(m, nn.Linear):
            w = dequantize_nf24_i16(m._native_rnf8_codes0_t, m._native_rnf8_codes2_t, m._native_rnf8_scales0)
            ref.get_submodule(name).weight.data = w.cpu().double()
    with torch.inference_mode():
        got = gpu(x.cuda(), temb.cuda(), freqs.cuda())
        want = ref(x.double(), temb.double(), freqs)
        attn_g, attn_r = gpu.blocks[0].attn, ref.blocks[0].attn
        xa = torch.randn(B, L, C)
        kb_g = tap._rope_self_attention_with_key_bias(attn_g, xa.cuda(), freqs.cuda(), key_bias.cuda(),
                                                      backend="native_avx512_exact")
        kb_r = tap64._rope_self_attention_with_key_bias(attn_r, xa.double(), freqs, key_bias.double())
        se_g = tap._rope_self_attention_selected_rows(attn_g, xa.cuda(), sel.cuda(), freqs.cuda(),
                                                      backend="native_avx512_exact", compute_dtype="model",
                                                      query_chunk_size=128)
        se_r = tap64._rope_self_attention_selected_rows(attn_r, xa.double(), sel, freqs,
                                                        backend="default", compute_dtype="model",
                                                        query_chunk_size=128)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(got).all())
    assert _rel(got, want) <= 1e-5, _rel(got, want)
    assert _rel(kb_g, kb_r) <= 1e-5 and _rel(se_g, se_r) <= 1e-5
    rt = metas["attn"]["runtime"]
    assert rt["calls"] == 4 and rt["key_bias_calls"] == 1 and rt["selected_row_calls"] == 1
    assert rt["fallbacks"] == 0
    assert metas["linear"]["runtime"]["fallbacks"] == 0 and metas["linear"]["runtime"]["range_calls"] == 2
    assert metas["norm"]["runtime"]["layernorm"]["calls"] == 2 * 2 + 1
    assert metas["norm"]["runtime"]["rmsnorm"]["calls"] == 0  # the packed helpers fuse RoPE + RMSNorm
    assert metas["gelu"]["runtime"]["calls"] == 2 and metas["silu"]["runtime"]["calls"] == 2
    blk = metas["block"]["runtime"]
    assert blk["modulate"]["calls"] == 4 and blk["residual"]["calls"] == 4
    assert all(v["fallbacks"] == 0 for v in blk.values())


def test_rope_and_rmsnorm_patches_match_torch():
    """The RoPE and multi-head RMSNorm patches on their own (the path the packed helpers
    bypass), against the float64 PyTorch functions."""
    import native_patches as npt

    mdl, _ = _make_modules()
    torch.manual_seed(4)
    norm = MultiHeadRMSNorm(2, 64).cuda()
    m = nn.ModuleDict({"norm": norm})
    meta = npt.apply_triposplat_native_norm_rope_avx512_patch(m, enabled=True, rope_module=mdl)
    x = torch.randn(3, 11, 2, 64)
    ang = torch.randn(1, 11, 2, 32, dtype=torch.float64)
    freqs = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    with torch.inference_mode():
        r = mdl.apply_rotary_emb(x.cuda(), freqs.cuda())
        n = norm(x.cuda())
    r_ref = _apply_rotary_emb(x.double(), freqs)
    g = norm.gamma.detach().cpu().double()
    xd = x.double()
    n_ref = xd * (8.0 / xd.norm(dim=-1, keepdim=True).clamp_min(1e-12)) * g
    assert _rel(r, r_ref) <= 1e-6 and _rel(n, n_ref) <= 1e-6
    assert meta["runtime"]["rope"]["calls"] == 1 and meta["runtime"]["rope"]["freq_copies"] == 1
    assert meta["runtime"]["rmsnorm"]["calls"] == 1
