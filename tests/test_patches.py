"""The reference's patch layer on this library, host side (CPU only, no kernel runs):
the checkpoint packer reproduces the reference packer's directory, the prepacked loader
fills a model the way the reference's loader does, and the module patchers keep the
reference's argument checks, library checks and strict violations
(scripts/native_linear_rnf8_avx512_patch.py:145-463, native_linear_nf24_prepacked.py:202-437,
native_gelu_avx512_patch.py, native_silu_avx512_patch.py, native_norm_rope_avx512_patch.py)."""
import json
import types
from pathlib import Path

import pytest
import torch
import torch.nn as nn

GOLDEN = Path(__file__).resolve().parent / "golden"


class _ShardModel(nn.Module):
    """The module tree of tests/golden/shards_src.safetensors."""

    def __init__(self):
        super().__init__()
        self.blocks = nn.ModuleList([nn.Module()])
        blk = self.blocks[0]
        blk.attn = nn.Module()
        blk.attn.qkv = nn.Linear(64, 96)
        blk.mlp = nn.Module()
        blk.mlp.fc1 = nn.Linear(96, 48)
        blk.norm = nn.Module()
        blk.norm.gamma = nn.Parameter(torch.ones(64))
        self.head = nn.Linear(48, 16, bias=False)
        self.pos_table = nn.Parameter(torch.zeros(8, 64))


def test_checkpoint_packer_reproduces_reference_directory(tmp_path):
    """Same manifest as the reference packer's directory (tests/golden/shards_ref), file
    hashes included; a second call resumes from the complete directory."""
    from nf24_shards import pack_nf24_i16_checkpoint

    src = GOLDEN / "shards_src.safetensors"
    man = pack_nf24_i16_checkpoint(src, tmp_path / "p", expected_linear_count=3)
    ref = json.loads((GOLDEN / "shards_ref" / "manifest.json").read_text())
    assert man == ref
    assert pack_nf24_i16_checkpoint(src, tmp_path / "p", expected_linear_count=3) == man
    with pytest.raises(RuntimeError, match="expected 206 Linear weights"):
        pack_nf24_i16_checkpoint(src, tmp_path / "q")


def test_prepacked_loader_fills_model_from_reference_shards():
    from nf24_shards import load_nf24_i16_prepacked_model, load_nf24_shards

    model = load_nf24_i16_prepacked_model(GOLDEN / "shards_ref", _ShardModel, verify_checksums=True,
                                          device="cpu")
    sh = load_nf24_shards(GOLDEN / "shards_ref", device="cpu")
    for name in ("blocks.0.attn.qkv", "blocks.0.mlp.fc1", "head"):
        mod = model.get_submodule(name)
        assert torch.equal(mod._native_rnf8_codes0_t, sh.linears[name].code01)
        assert torch.equal(mod._native_rnf8_codes2_t, sh.linears[name].q2)
        assert torch.equal(mod._native_rnf8_scales0, sh.linears[name].scale)
        assert mod.weight.numel() == 0
    assert torch.equal(model.pos_table, sh.non_linear["pos_table"])
    load = model._native_rnf8_prepacked_load
    assert load["source_checkpoint_loaded"] is False and load["linear_count"] == 3
    assert load["checksums_verified"] is True

    class Extra(_ShardModel):
        def __init__(self):
            super().__init__()
            self.extra = nn.Linear(4, 4)
    with pytest.raises(RuntimeError, match="Linear mismatch"):
        load_nf24_i16_prepacked_model(GOLDEN / "shards_ref", Extra, device="cpu")


def test_linear_patch_argument_and_library_checks():
    from native_patches import apply_triposplat_native_rnf8_avx512_patch as patch

    m = nn.Sequential(nn.Linear(32, 16))
    assert patch(m) == {"enabled": False}
    with pytest.raises(ValueError, match="strict=True"):
        patch(m, enabled=True, strict=False)
    with pytest.raises(ValueError, match="exactly 3 stages"):
        patch(m, enabled=True, stages=2, residual_mode="nf24_i16")
    with pytest.raises(RuntimeError, match="requested=nf8, library=nf24_i16"):
        patch(m, enabled=True, stages=3, residual_mode="nf8")
    with pytest.raises(FileNotFoundError):
        patch(m, enabled=True, stages=3, residual_mode="nf24_i16", library_path="/nonexistent/lib.so")


def test_linear_patch_packs_and_enforces_strict_inputs():
    """Packing on the host gives the packer's codes; a CPU input is a strict violation (the
    kernels take CUDA tensors), exactly as the reference refuses a non-CPU input."""
    from native_patches import apply_triposplat_native_rnf8_avx512_patch as patch
    from nf24_pack import quantize_nf24_i16_per_output_channel

    torch.manual_seed(0)
    m = nn.Sequential(nn.Linear(32, 16), nn.Linear(16, 5, bias=False))
    w0 = m[0].weight.detach().clone()
    meta = patch(m, enabled=True, stages=3, residual_mode="nf24_i16")
    assert meta["selected_count"] == 2 and meta["skipped_count"] == 0
    assert meta["row_tile"] > 0 and meta["float32_weight_retained"] is False
    assert meta["selected_dims"] == {"0": "32x16", "1": "16x5"}
    codes, scales, _ = quantize_nf24_i16_per_output_channel(w0)
    assert torch.equal(m[0]._native_rnf8_codes0_t, codes[0])
    assert torch.equal(m[0]._native_rnf8_scales0, scales[0])
    assert m[0].weight.numel() == 0 and torch.count_nonzero(m[1]._native_rnf8_bias) == 0
    with torch.inference_mode(), pytest.raises(RuntimeError, match="input_cpu"):
        m(torch.randn(3, 32))
    with pytest.raises(RuntimeError, match="grad_enabled"):
        m(torch.randn(3, 32))
    with pytest.raises(ValueError, match="output range"):
        m[0]._native_avx512_forward_range(torch.randn(3, 32), 8, 16)


def test_linear_patch_include_exclude_strictness():
    from native_patches import apply_triposplat_native_rnf8_avx512_patch as patch

    m = nn.Sequential(nn.Linear(8, 16), nn.Linear(16, 16))
    with pytest.raises(ValueError, match="left 1 Linear modules unquantized"):
        patch(m, enabled=True, stages=3, residual_mode="nf24_i16", include_regex=r"^0$")


def test_activation_and_norm_patchers_select_and_check():
    from native_patches import (apply_triposplat_native_gelu_avx512_patch,
                                apply_triposplat_native_norm_rope_avx512_patch,
                                apply_triposplat_native_silu_avx512_patch)

    class MultiHeadRMSNorm(nn.Module):
        def __init__(self):
            super().__init__()
            self.gamma = nn.Parameter(torch.ones(2, 64))

    m = nn.Sequential(nn.GELU(approximate="tanh"), nn.SiLU(), nn.LayerNorm(64), MultiHeadRMSNorm())
    g = apply_triposplat_native_gelu_avx512_patch(m, enabled=True)
    assert g["selected"] == ["0"] and g["runtime"]["fallbacks"] == 0
    s = apply_triposplat_native_silu_avx512_patch(m, enabled=True)
    assert s["selected"] == ["1"]
    rope_mod = types.SimpleNamespace(apply_rotary_emb=lambda x, f: x)
    n = apply_triposplat_native_norm_rope_avx512_patch(m, enabled=True, rope_module=rope_mod)
    assert n["layernorm_selected"] == ["2"] and n["rmsnorm_selected"] == ["3"] and n["rope_patched"]
    assert rope_mod.apply_rotary_emb.__name__ == "native_rope"
    with torch.inference_mode(), pytest.raises(RuntimeError, match="strict violation.*input_cpu"):
        m[0](torch.randn(4, 64))
    with pytest.raises(ValueError, match="approximate=tanh"):
        apply_triposplat_native_gelu_avx512_patch(nn.Sequential(nn.GELU()), enabled=True)
    assert apply_triposplat_native_silu_avx512_patch(m) == {"enabled": False}
