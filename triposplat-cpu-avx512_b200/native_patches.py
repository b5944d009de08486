"""The reference's module patchers, on CUDA tensors, over ``libtriposplat_b200.so``.

Each ``apply_triposplat_native_*_patch(flow_model, ...)`` keeps the reference function's
name, keyword arguments, strict checks, error messages' meaning and returned metadata dict
(with its ``runtime`` counters, ``fallbacks`` included), so a pipeline that patches its
model with the reference's functions switches to the GPU by importing them from here:

* ``apply_triposplat_native_rnf8_avx512_patch`` — every ``nn.Linear`` runs the NF24 GEMM
  (scripts/native_linear_rnf8_avx512_patch.py:145-463): the library's residual mode must
  equal the requested one (this library implements ``nf24_i16``, mode 4, 3 stages), float
  weights are packed by the reference's packing steps (``nf24_pack``) or taken from a
  prepacked load (``nf24_shards.load_nf24_i16_prepacked_model``), the float weights are
  released, ``forward`` and ``_native_avx512_forward_range`` call the full / tail / range
  entry points;
* ``apply_triposplat_native_norm_rope_avx512_patch`` — ``nn.LayerNorm``, modules of class
  ``MultiHeadRMSNorm`` and the model module's ``apply_rotary_emb``
  (scripts/native_norm_rope_avx512_patch.py:10-156);
* ``apply_triposplat_native_gelu_avx512_patch`` — ``nn.GELU(approximate="tanh")``
  (scripts/native_gelu_avx512_patch.py:11-101);
* ``apply_triposplat_native_silu_avx512_patch`` — ``nn.SiLU``
  (scripts/native_silu_avx512_patch.py:6-35);
* ``apply_triposplat_native_block_elementwise_avx512_patch`` — modulate / gated residual
  / add of ``UnifiedTransformerBlock`` (scripts/native_block_elementwise_avx512_patch.py:6-60);
* ``apply_triposplat_native_qkv_packed_attention_helpers_patch`` — the attention helpers
  through RoPE + RMSNorm + pack and the packed exact SDPA
  (scripts/native_qkv_packed_attention_patch_v3.py:9-335).

Differences, all deliberate: tensors must be CUDA float32 (the reference's ``cpu`` checks
become ``cuda`` checks, with the same strict-violation reasons); kernels are queued on
PyTorch's current stream, so ``runtime["seconds"]`` counts host time to enqueue (call
``torch.cuda.synchronize()`` around a region for device time); ``threads`` is accepted and
ignored; ``library_path`` defaults to this package's library, and a library that is not
this CUDA build (no ``triposplat_b200_abi_version`` symbol) is refused rather than handed
device pointers.  The upstream modules the reference patches by import (``model`` for
``apply_rotary_emb``, ``triposplat_attention_patch`` for the block and attention helpers)
are imported by the same names unless passed in (``rope_module=`` /
``attention_module=``).
"""
from __future__ import annotations

import importlib
import math
import re
import time
import types
from typing import Any

import _native
from nf24_pack import make_nf8_codebook, quantize_nf24_i16_any_device

RESIDUAL_MODES = {0: "nf8", 1: "symmetric_int8", 4: "nf24_i16"}


def _library(library_path):
    """This package's CUDA library (or the one at ``library_path``, which must be a build
    of it: it is called with device pointers)."""
    path = _native.library_path(library_path)
    if not path.is_file():
        raise FileNotFoundError(path)
    lib = _native.load(path)
    if getattr(lib, "triposplat_b200_abi_version", None) is None:
        raise RuntimeError(f"{path} is not a CUDA build of the TripoSplat kernels")
    return lib, path


def _is_cuda_f32(t) -> bool:
    import torch

    return torch.is_tensor(t) and t.device.type == "cuda" and t.dtype == torch.float32


def _last_error(lib) -> str:
    return lib.triposplat_b200_last_error().decode(errors="replace")


# --------------------------------------------------------------------------------------
# NF24 Linear
# --------------------------------------------------------------------------------------
def apply_triposplat_native_rnf8_avx512_patch(
    flow_model,
    *,
    enabled: bool = False,
    include_regex: str | None = None,
    exclude_regex: str | None = None,
    library_path: str | None = None,
    optimized_library_path: str | None = None,
    optimized_shapes: tuple[tuple[int, int], ...] = (),
    threads: int = 2,
    strict: bool = True,
    stages: int = 2,
    residual_mode: str = "nf8",
    device=None,
) -> dict[str, Any]:
    """Patch every selected ``nn.Linear`` of ``flow_model`` to the CUDA NF24 GEMM.

    ``device`` (no reference counterpart): where the packed buffers go; by default they
    stay where the weight was (move the model with ``.cuda()`` before running it)."""
    if not enabled:
        return {"enabled": False}
    if not strict:
        raise ValueError("residual NF8 releases float32 weights and requires strict=True")
    if stages not in (2, 3):
        raise ValueError("residual NF8 stages must be 2 or 3")
    if residual_mode not in ("nf8", "symmetric_int8", "nf24_i16"):
        raise ValueError(f"unsupported residual quantizer: {residual_mode}")
    if residual_mode == "nf24_i16" and stages != 3:
        raise ValueError("NF24 int16 layout requires exactly 3 stages")

    import torch
    import torch.nn as nn

    include = re.compile(include_regex) if include_regex else None
    exclude = re.compile(exclude_regex) if exclude_regex else None
    lib, lib_path = _library(library_path)
    row_tile = int(lib.triposplat_gemm_rnf8_avx512_row_tile())
    mode_id = int(lib.triposplat_gemm_rnf8_avx512_residual_mode())
    library_residual_mode = RESIDUAL_MODES.get(mode_id)
    if library_residual_mode is None:
        raise RuntimeError(f"unsupported residual mode id from library: {mode_id}")
    if library_residual_mode != residual_mode:
        raise RuntimeError(
            f"residual quantizer/library mismatch: requested={residual_mode}, "
            f"library={library_residual_mode}")
    full_kernel = lib.triposplat_gemm_rnf8_avx512
    tail_kernel = lib.triposplat_gemm_rnf8_avx512_tail
    range_kernel = lib.triposplat_gemm_rnf8_avx512_range

    optimized_shapes_set = {tuple(int(v) for v in shape) for shape in optimized_shapes}
    optimized_full_kernel = None
    optimized_lib_path = None
    if optimized_library_path is not None:
        optimized_lib, optimized_lib_path = _library(optimized_library_path)
        optimized_mode = RESIDUAL_MODES.get(int(optimized_lib.triposplat_gemm_rnf8_avx512_residual_mode()))
        if optimized_mode != residual_mode:
            raise RuntimeError(
                f"optimized residual quantizer/library mismatch: requested={residual_mode}, "
                f"library={optimized_mode}")
        optimized_full_kernel = optimized_lib.triposplat_gemm_rnf8_avx512

    runtime = {"calls": 0, "range_calls": 0, "optimized_calls": 0, "rows": 0, "seconds": 0.0,
               "contiguous_copies": 0, "fallbacks": 0, "per_module": {}}
    selected, selected_dims, skipped, packing = [], {}, [], {}
    codebook = make_nf8_codebook(torch)
    prepacked_manifest = getattr(flow_model, "_native_rnf8_prepacked_manifest", None)
    if prepacked_manifest is not None and (stages != 3 or residual_mode != "nf24_i16"):
        raise ValueError("prepacked NF24 int16 requires stages=3 and residual_mode=nf24_i16")
    original_bytes = packed_bytes = weight_elements = 0
    weighted_squared_error = 0.0
    max_abs_error = 0.0

    def matches(name: str) -> bool:
        return not ((include is not None and include.search(name) is None)
                    or (exclude is not None and exclude.search(name) is not None))

    def prepare_input(module, x, module_name: str):
        if torch.is_grad_enabled():
            raise RuntimeError(f"residual NF8 strict violation for {module_name}: grad_enabled")
        if x.device.type != "cuda" or x.dtype != torch.float32:
            raise RuntimeError(f"residual NF8 strict violation for {module_name}: input_{x.device.type}_{x.dtype}")
        if int(x.shape[-1]) != int(module.in_features):
            raise RuntimeError(f"residual NF8 strict violation for {module_name}: input_feature_mismatch")
        if module._native_rnf8_codes0_t.device != x.device:
            raise RuntimeError(f"residual NF8 strict violation for {module_name}: "
                               f"weights_on_{module._native_rnf8_codes0_t.device}")
        x2 = x.reshape(-1, int(module.in_features))
        if not x2.is_contiguous():
            x2 = x2.contiguous()
            runtime["contiguous_copies"] += 1
        return x2

    def pointers(module):
        return (module._native_rnf8_codes0_t.data_ptr(), module._native_rnf8_codes1_t.data_ptr(),
                module._native_rnf8_codes2_t.data_ptr(), module._native_rnf8_scales0.data_ptr(),
                module._native_rnf8_scales1.data_ptr(), module._native_rnf8_scales2.data_ptr(),
                module._native_rnf8_codebook.data_ptr(), module._native_rnf8_bias.data_ptr())

    def record(name, rows, elapsed, is_range, optimized=False):
        runtime["calls"] += 1
        runtime["range_calls"] += int(is_range)
        runtime["optimized_calls"] += int(optimized)
        runtime["rows"] += rows
        runtime["seconds"] += elapsed
        item = runtime["per_module"].setdefault(
            name, {"calls": 0, "range_calls": 0, "optimized_calls": 0, "rows": 0, "seconds": 0.0})
        item["calls"] += 1
        item["range_calls"] += int(is_range)
        item["optimized_calls"] += int(optimized)
        item["rows"] += rows
        item["seconds"] += elapsed

    def make_forward(module_name: str):
        def forward(self, x):
            x2 = prepare_input(self, x, module_name)
            rows = int(x2.shape[0])
            out = torch.empty((rows, int(self.out_features)), dtype=torch.float32, device=x.device)
            shape = (int(self.in_features), int(self.out_features))
            use_optimized = (optimized_full_kernel is not None and shape in optimized_shapes_set
                             and shape[1] % 16 == 0)
            kernel = optimized_full_kernel if use_optimized else (tail_kernel if shape[1] % 16 else full_kernel)
            started = time.perf_counter()
            _native.use_current_stream(lib)
            status = int(kernel(x2.data_ptr(), *pointers(self), out.data_ptr(), rows, shape[0], shape[1],
                                shape[0], shape[1], int(threads), int(stages)))
            elapsed = time.perf_counter() - started
            if status != 0:
                runtime["fallbacks"] += 1
                raise RuntimeError(f"residual NF8 kernel returned {status} for {module_name}: {_last_error(lib)}")
            record(module_name, rows, elapsed, False, use_optimized)
            return out.view(*x.shape[:-1], int(self.out_features))
        return forward

    def make_range_forward(module_name: str):
        def range_forward(self, x, output_start: int, output_count: int):
            start, count = int(output_start), int(output_count)
            if start < 0 or count <= 0 or start + count > int(self.out_features):
                raise ValueError(f"invalid residual NF8 output range for {module_name}")
            x2 = prepare_input(self, x, module_name)
            rows = int(x2.shape[0])
            out = torch.empty((rows, count), dtype=torch.float32, device=x.device)
            K, N = int(self.in_features), int(self.out_features)
            started = time.perf_counter()
            _native.use_current_stream(lib)
            status = int(range_kernel(x2.data_ptr(), *pointers(self), out.data_ptr(), rows, K, N, start,
                                      count, K, count, int(threads), int(stages)))
            elapsed = time.perf_counter() - started
            if status != 0:
                runtime["fallbacks"] += 1
                raise RuntimeError(f"residual NF8 range kernel returned {status} for {module_name}: "
                                   f"{_last_error(lib)}")
            record(module_name, rows, elapsed, True)
            return out.view(*x.shape[:-1], count)
        return range_forward

    for name, module in flow_model.named_modules():
        if not isinstance(module, nn.Linear):
            continue
        if not matches(name):
            skipped.append(name)
            continue
        if prepacked_manifest is None:
            if module.weight.dtype != torch.float32 or module.weight.device.type not in ("cpu", "cuda"):
                raise ValueError(f"residual NF8 requires float32 weight on cpu or cuda: {name}")
            dev = torch.device(device) if device is not None else module.weight.device
            codes, scales, error = quantize_nf24_i16_any_device(module.weight.detach().to(dev), codebook)
            bias = (torch.zeros(int(module.out_features), dtype=torch.float32, device=dev)
                    if module.bias is None else module.bias.detach().to(dev).contiguous())
            module.register_buffer("_native_rnf8_codes0_t", codes[0], persistent=False)
            module.register_buffer("_native_rnf8_codes1_t", codes[1], persistent=False)
            module.register_buffer("_native_rnf8_codes2_t", codes[2], persistent=False)
            module.register_buffer("_native_rnf8_scales0", scales[0], persistent=False)
            module.register_buffer("_native_rnf8_scales1", scales[1], persistent=False)
            module.register_buffer("_native_rnf8_scales2", scales[2], persistent=False)
            module.register_buffer("_native_rnf8_bias", bias, persistent=False)
        else:
            item = prepacked_manifest["linears"].get(name)
            if item is None:
                raise ValueError(f"prepacked checkpoint has no Linear entry: {name}")
            codes = [module._native_rnf8_codes0_t, module._native_rnf8_codes1_t, module._native_rnf8_codes2_t]
            scales = [module._native_rnf8_scales0, module._native_rnf8_scales1, module._native_rnf8_scales2]
            bias = module._native_rnf8_bias
            error = item["quantization"]
            dev = codes[0].device
        module.register_buffer("_native_rnf8_codebook", codebook.clone().to(dev), persistent=False)
        module.weight = nn.Parameter(torch.empty(0, dtype=torch.float32), requires_grad=False)
        if module.bias is not None:
            module.bias = nn.Parameter(torch.empty(0, dtype=torch.float32), requires_grad=False)
        module.forward = types.MethodType(make_forward(name), module)
        module._native_avx512_forward_range = types.MethodType(make_range_forward(name), module)

        count = int(codes[0].numel())
        original = count * 4 + int(bias.numel()) * 4
        packed = count * 3 + int(scales[0].numel()) * 4 + int(bias.numel()) * 4 + 1024
        original_bytes += original
        packed_bytes += packed
        weight_elements += count
        weighted_squared_error += error["weight_rmse"] ** 2 * count
        max_abs_error = max(max_abs_error, error["weight_max_abs"])
        packing[name] = {**error, "weight_elements": count, "original_bytes": original, "packed_bytes": packed}
        selected.append(name)
        selected_dims[name] = f"{int(module.in_features)}x{int(module.out_features)}"

    if skipped:
        raise ValueError(f"residual NF8 strict mode left {len(skipped)} Linear modules unquantized")
    return {
        "enabled": bool(selected),
        "kind": "native_nf24_i16_cuda_linear_patch",
        "residual_stages": int(stages),
        "first_stage_quantizer": "nf8_derived_int8_alphabet",
        "residual_quantizer": residual_mode,
        "bits_per_weight": 24,
        "activation_dtype": "float32",
        "float32_weight_retained": False,
        "library_path": lib_path.as_posix(),
        "optimized_library_path": None if optimized_lib_path is None else optimized_lib_path.as_posix(),
        "optimized_shapes": [list(s) for s in sorted(optimized_shapes_set)],
        "row_tile": row_tile,
        "symbols": ["triposplat_gemm_rnf8_avx512", "triposplat_gemm_rnf8_avx512_range",
                    "triposplat_gemm_rnf8_avx512_tail", "triposplat_gemm_rnf8_avx512_row_tile",
                    "triposplat_gemm_rnf8_avx512_residual_mode"],
        "threads": int(threads),
        "strict": True,
        "prepacked_load": getattr(flow_model, "_native_rnf8_prepacked_load", {"enabled": False}),
        "selected_count": len(selected),
        "selected": selected,
        "selected_dims": selected_dims,
        "skipped_count": 0,
        "original_bytes": original_bytes,
        "packed_bytes": packed_bytes,
        "storage_ratio": packed_bytes / max(original_bytes, 1),
        "aggregate_weight_rmse": math.sqrt(weighted_squared_error / max(weight_elements, 1)),
        "aggregate_weight_max_abs": max_abs_error,
        "packing": packing,
        "runtime": runtime,
        "semantics": "All selected Linear weights are NF24 int16 codes decoded inside the B200 "
                     "tensor-core GEMM (exact fp16 operands, fp32 accumulation).",
    }


# --------------------------------------------------------------------------------------
# LayerNorm / multi-head RMSNorm / RoPE
# --------------------------------------------------------------------------------------
def apply_triposplat_native_norm_rope_avx512_patch(
    flow_model,
    *,
    enabled: bool = False,
    library_path: str | None = None,
    threads: int = 2,
    strict: bool = True,
    rope_module=None,
) -> dict[str, Any]:
    """``rope_module`` (no reference counterpart): the module whose ``apply_rotary_emb`` is
    replaced; the reference imports it as ``model``."""
    if not enabled:
        return {"enabled": False}

    import torch
    import torch.nn as nn

    triposplat_model = rope_module if rope_module is not None else importlib.import_module("model")
    lib, lib_path = _library(library_path)
    layernorm_kernel = lib.triposplat_layernorm_f32_avx512
    rmsnorm_kernel = lib.triposplat_multihead_rmsnorm_f32_avx512
    rope_kernel = lib.triposplat_rope_complex_f32_avx512

    runtime = {
        "layernorm": {"calls": 0, "rows": 0, "seconds": 0.0, "fallbacks": 0},
        "rmsnorm": {"calls": 0, "vectors": 0, "seconds": 0.0, "fallbacks": 0},
        "rope": {"calls": 0, "vectors": 0, "seconds": 0.0, "fallbacks": 0, "input_copies": 0,
                 "freq_copies": 0},
    }
    layernorm_selected, rmsnorm_selected, skipped = [], [], []

    def strict_error(kind, name, reason):
        runtime[kind]["fallbacks"] += 1
        if strict:
            raise RuntimeError(f"native CUDA {kind} strict violation for {name}: {reason}")

    def run(kernel, args, what):
        _native.use_current_stream(lib)
        started = time.perf_counter()
        status = int(kernel(*args))
        elapsed = time.perf_counter() - started
        if status != 0:
            raise RuntimeError(f"{what} returned {status}: {_last_error(lib)}")
        return elapsed

    def make_layernorm_forward(module_name):
        def forward(self, x):
            reason = None
            if torch.is_grad_enabled():
                reason = "grad_enabled"
            elif not _is_cuda_f32(x):
                reason = f"input_{x.device.type}_{x.dtype}"
            elif len(self.normalized_shape) != 1 or int(x.shape[-1]) != int(self.normalized_shape[0]):
                reason = "shape"
            if reason is not None:
                strict_error("layernorm", module_name, reason)
                return self._original_forward_native_norm_rope(x)
            source = x if x.is_contiguous() else x.contiguous()
            cols = int(source.shape[-1])
            rows = int(source.numel() // cols)
            out = torch.empty_like(source)
            has_affine = self.weight is not None
            w = self.weight.data_ptr() if has_affine else None
            b = self.bias.data_ptr() if has_affine and self.bias is not None else None
            if has_affine and b is None:
                raise RuntimeError(f"native LayerNorm for {module_name}: affine LayerNorm without bias")
            elapsed = run(layernorm_kernel, (source.data_ptr(), w, b, out.data_ptr(), rows, cols,
                                             float(self.eps), int(has_affine), int(threads)),
                          f"native LayerNorm for {module_name}")
            runtime["layernorm"]["calls"] += 1
            runtime["layernorm"]["rows"] += rows
            runtime["layernorm"]["seconds"] += elapsed
            return out.view_as(x)
        return forward

    def make_rmsnorm_forward(module_name):
        def forward(self, x):
            heads, dim = (int(v) for v in self.gamma.shape)
            reason = None
            if torch.is_grad_enabled():
                reason = "grad_enabled"
            elif not _is_cuda_f32(x):
                reason = f"input_{x.device.type}_{x.dtype}"
            elif tuple(int(v) for v in x.shape[-2:]) != (heads, dim):
                reason = "shape"
            if reason is not None:
                strict_error("rmsnorm", module_name, reason)
                return self._original_forward_native_norm_rope(x)
            source = x if x.is_contiguous() else x.contiguous()
            gamma = self.gamma.detach().contiguous()
            outer = int(source.numel() // (heads * dim))
            out = torch.empty_like(source)
            elapsed = run(rmsnorm_kernel, (source.data_ptr(), gamma.data_ptr(), out.data_ptr(), outer,
                                           heads, dim, 1.0e-12, int(threads)),
                          f"native RMSNorm for {module_name}")
            runtime["rmsnorm"]["calls"] += 1
            runtime["rmsnorm"]["vectors"] += outer * heads
            runtime["rmsnorm"]["seconds"] += elapsed
            return out.view_as(x)
        return forward

    for name, module in flow_model.named_modules():
        if isinstance(module, nn.LayerNorm):
            if len(module.normalized_shape) != 1:
                skipped.append(name)
                continue
            module._original_forward_native_norm_rope = module.forward
            module.forward = types.MethodType(make_layernorm_forward(name), module)
            layernorm_selected.append(name)
        elif module.__class__.__name__ == "MultiHeadRMSNorm":
            if not hasattr(module, "gamma") or module.gamma.ndim != 2:
                skipped.append(name)
                continue
            module._original_forward_native_norm_rope = module.forward
            module.forward = types.MethodType(make_rmsnorm_forward(name), module)
            rmsnorm_selected.append(name)
    if strict and skipped:
        raise ValueError(f"native norm strict mode left {len(skipped)} norm modules unpatched: {skipped[:8]}")

    original_rope = triposplat_model.apply_rotary_emb

    def native_rope(hidden_states, freqs):
        reason = None
        if torch.is_grad_enabled():
            reason = "grad_enabled"
        elif not _is_cuda_f32(hidden_states):
            reason = f"input_{hidden_states.device.type}_{hidden_states.dtype}"
        elif freqs.device.type != "cuda" or freqs.dtype != torch.complex64:
            reason = f"freq_{freqs.device.type}_{freqs.dtype}"
        elif int(hidden_states.shape[-1]) != 2 * int(freqs.shape[-1]):
            reason = "shape"
        if reason is not None:
            strict_error("rope", "model.apply_rotary_emb", reason)
            return original_rope(hidden_states, freqs)
        source = hidden_states
        if not source.is_contiguous():
            source = source.contiguous()
            runtime["rope"]["input_copies"] += 1
        dim = int(source.shape[-1])
        freq_float = torch.view_as_real(freqs).reshape(*freqs.shape[:-1], dim)
        if freq_float.numel() != source.numel():
            try:  # the kernel reads one frequency vector per input vector
                freq_float = freq_float.expand(*source.shape)
            except RuntimeError:
                strict_error("rope", "model.apply_rotary_emb", "freq_shape")
                return original_rope(hidden_states, freqs)
        if not freq_float.is_contiguous():
            freq_float = freq_float.contiguous()
            runtime["rope"]["freq_copies"] += 1
        vectors = int(source.numel() // dim)
        out = torch.empty_like(source)
        elapsed = run(rope_kernel, (source.data_ptr(), freq_float.data_ptr(), out.data_ptr(), vectors, dim,
                                    int(threads)), "native RoPE")
        runtime["rope"]["calls"] += 1
        runtime["rope"]["vectors"] += vectors
        runtime["rope"]["seconds"] += elapsed
        return out.view_as(hidden_states)

    def native_functional_layernorm(x, eps=1.0e-5):
        reason = None
        if torch.is_grad_enabled():
            reason = "grad_enabled"
        elif not _is_cuda_f32(x):
            reason = f"input_{x.device.type}_{x.dtype}"
        elif x.ndim < 1 or int(x.shape[-1]) <= 0:
            reason = "shape"
        if reason is not None:
            strict_error("layernorm", "functional_final_layernorm", reason)
            return torch.nn.functional.layer_norm(x.float(), x.shape[-1:], eps=float(eps)).type_as(x)
        source = x if x.is_contiguous() else x.contiguous()
        cols = int(source.shape[-1])
        rows = int(source.numel() // cols)
        out = torch.empty_like(source)
        elapsed = run(layernorm_kernel, (source.data_ptr(), None, None, out.data_ptr(), rows, cols,
                                         float(eps), 0, int(threads)), "native functional LayerNorm")
        runtime["layernorm"]["calls"] += 1
        runtime["layernorm"]["rows"] += rows
        runtime["layernorm"]["seconds"] += elapsed
        return out.view_as(x)

    flow_model._native_avx512_functional_layernorm = native_functional_layernorm
    triposplat_model.apply_rotary_emb = native_rope
    return {
        "enabled": True, "kind": "native_f32_cuda_layernorm_rmsnorm_rope_patch",
        "library_path": lib_path.as_posix(),
        "symbols": ["triposplat_layernorm_f32_avx512", "triposplat_multihead_rmsnorm_f32_avx512",
                    "triposplat_rope_complex_f32_avx512"],
        "threads": int(threads), "strict": bool(strict),
        "layernorm_selected_count": len(layernorm_selected), "layernorm_selected": layernorm_selected,
        "rmsnorm_selected_count": len(rmsnorm_selected), "rmsnorm_selected": rmsnorm_selected,
        "skipped_count": len(skipped), "skipped": skipped, "rope_patched": True, "runtime": runtime,
    }


# --------------------------------------------------------------------------------------
# GELU(tanh) and SiLU
# --------------------------------------------------------------------------------------
def apply_triposplat_native_gelu_avx512_patch(
    flow_model,
    *,
    enabled: bool = False,
    include_regex: str | None = None,
    exclude_regex: str | None = None,
    library_path: str | None = None,
    threads: int = 2,
    strict: bool = True,
) -> dict[str, Any]:
    if not enabled:
        return {"enabled": False}

    import torch
    import torch.nn as nn

    include = re.compile(include_regex) if include_regex else None
    exclude = re.compile(exclude_regex) if exclude_regex else None
    lib, lib_path = _library(library_path)
    kernel = lib.triposplat_gelu_tanh_f32_avx512
    runtime = {"calls": 0, "elements": 0, "seconds": 0.0, "fallbacks": 0, "fallback_reasons": {},
               "per_module": {}}
    selected, skipped = [], []

    def matches(name):
        return not ((include is not None and include.search(name) is None)
                    or (exclude is not None and exclude.search(name) is not None))

    def make_forward(module_name):
        def patched_forward(self, x):
            reason = None
            if torch.is_grad_enabled():
                reason = "grad_enabled"
            elif not _is_cuda_f32(x):
                reason = f"input_{x.device.type}_{x.dtype}"
            elif getattr(self, "approximate", "none") != "tanh":
                reason = f"approximate_{getattr(self, 'approximate', 'none')}"
            if reason is not None:
                runtime["fallbacks"] += 1
                runtime["fallback_reasons"][reason] = int(runtime["fallback_reasons"].get(reason, 0)) + 1
                if strict:
                    raise RuntimeError(f"native CUDA GELU strict violation for {module_name}: {reason}")
                return self._original_forward_native_gelu_avx512(x)
            source = x if x.is_contiguous() else x.contiguous()
            out = torch.empty_like(source)
            _native.use_current_stream(lib)
            started = time.perf_counter()
            status = int(kernel(source.data_ptr(), out.data_ptr(), source.numel(), int(threads)))
            elapsed = time.perf_counter() - started
            if status != 0:
                raise RuntimeError(f"native CUDA GELU returned {status} for {module_name}: {_last_error(lib)}")
            runtime["calls"] += 1
            runtime["elements"] += int(source.numel())
            runtime["seconds"] += elapsed
            item = runtime["per_module"].setdefault(module_name, {"calls": 0, "elements": 0, "seconds": 0.0})
            item["calls"] += 1
            item["elements"] += int(source.numel())
            item["seconds"] += elapsed
            return out.view_as(x)
        return patched_forward

    for name, module in flow_model.named_modules():
        if not isinstance(module, nn.GELU):
            continue
        if not matches(name):
            skipped.append(name)
            continue
        if getattr(module, "approximate", "none") != "tanh":
            if strict:
                raise ValueError(f"native CUDA GELU requires approximate=tanh: {name}")
            skipped.append(name)
            continue
        module._original_forward_native_gelu_avx512 = module.forward
        module.forward = types.MethodType(make_forward(name), module)
        selected.append(name)
    if strict and skipped:
        raise ValueError(f"native CUDA GELU strict mode left {len(skipped)} GELU modules unpatched")
    return {
        "enabled": bool(selected), "kind": "native_f32_cuda_gelu_tanh_patch",
        "library_path": lib_path.as_posix(), "symbol": "triposplat_gelu_tanh_f32_avx512",
        "threads": int(threads), "strict": bool(strict), "selected_count": len(selected),
        "selected": selected, "skipped_count": len(skipped), "skipped": skipped, "runtime": runtime,
    }


def apply_triposplat_native_silu_avx512_patch(
    flow_model,
    *,
    enabled: bool = False,
    library_path: str | None = None,
    threads: int = 2,
    strict: bool = True,
) -> dict[str, Any]:
    if not enabled:
        return {"enabled": False}

    import torch
    import torch.nn as nn

    lib, lib_path = _library(library_path)
    kernel = lib.triposplat_silu_f32_avx512
    runtime = {"calls": 0, "elements": 0, "seconds": 0.0, "fallbacks": 0, "per_module": {}}
    selected = []

    def make_forward(name):
        def forward(self, x):
            reason = None
            if torch.is_grad_enabled():
                reason = "grad_enabled"
            elif not _is_cuda_f32(x):
                reason = f"input_{x.device.type}_{x.dtype}"
            if reason is not None:
                runtime["fallbacks"] += 1
                if strict:
                    raise RuntimeError(f"native CUDA SiLU strict violation for {name}: {reason}")
                return self._original_forward_native_silu_avx512(x)
            source = x if x.is_contiguous() else x.contiguous()
            out = torch.empty_like(source)
            _native.use_current_stream(lib)
            started = time.perf_counter()
            status = int(kernel(source.data_ptr(), out.data_ptr(), source.numel(), int(threads)))
            elapsed = time.perf_counter() - started
            if status:
                raise RuntimeError(f"native CUDA SiLU returned {status} for {name}: {_last_error(lib)}")
            runtime["calls"] += 1
            runtime["elements"] += int(source.numel())
            runtime["seconds"] += elapsed
            item = runtime["per_module"].setdefault(name, {"calls": 0, "elements": 0, "seconds": 0.0})
            item["calls"] += 1
            item["elements"] += int(source.numel())
            item["seconds"] += elapsed
            return out.view_as(x)
        return forward

    for name, module in flow_model.named_modules():
        if not isinstance(module, nn.SiLU):
            continue
        module._original_forward_native_silu_avx512 = module.forward
        module.forward = types.MethodType(make_forward(name), module)
        selected.append(name)
    return {"enabled": bool(selected), "kind": "native_f32_cuda_silu_patch", "library_path": lib_path.as_posix(),
            "symbol": "triposplat_silu_f32_avx512", "threads": int(threads), "strict": bool(strict),
            "selected_count": len(selected), "selected": selected, "runtime": runtime}


# --------------------------------------------------------------------------------------
# Block elementwise (modulate, gated residual, add)
# --------------------------------------------------------------------------------------
def apply_triposplat_native_block_elementwise_avx512_patch(
    flow_model,
    *,
    enabled: bool = False,
    library_path: str | None = None,
    threads: int = 2,
    strict: bool = True,
    attention_module=None,
) -> dict[str, Any]:
    """``attention_module`` (no reference counterpart): the module whose
    ``_modulate_inplace_preserve_order`` / ``_residual_gate_inplace_preserve_order`` are
    replaced; the reference imports it as ``triposplat_attention_patch``."""
    if not enabled:
        return {"enabled": False}

    import torch

    tap = attention_module if attention_module is not None else importlib.import_module(
        "triposplat_attention_patch")
    lib, lib_path = _library(library_path)
    mod_k = lib.triposplat_modulate_inplace_f32_avx512
    res_k = lib.triposplat_gated_residual_inplace_f32_avx512
    add_k = lib.triposplat_add_inplace_f32_avx512
    runtime = {k: {"calls": 0, "elements": 0, "seconds": 0.0, "fallbacks": 0}
               for k in ("modulate", "residual", "add")}

    def valid(t):
        return _is_cuda_f32(t) and t.is_contiguous()

    def call(kind, kernel, args, elements):
        _native.use_current_stream(lib)
        started = time.perf_counter()
        status = int(kernel(*args))
        elapsed = time.perf_counter() - started
        if status:
            raise RuntimeError(f"native {kind} returned {status}: {_last_error(lib)}")
        runtime[kind]["calls"] += 1
        runtime[kind]["elements"] += elements
        runtime[kind]["seconds"] += elapsed

    def modulate(h, scale, shift):
        if not (valid(h) and valid(scale) and valid(shift)):
            runtime["modulate"]["fallbacks"] += 1
            if strict:
                raise RuntimeError("native modulate strict violation")
            return tap._native_original_modulate(h, scale, shift)
        b, r, c = int(h.shape[0]), int(h.shape[-2]), int(h.shape[-1])
        call("modulate", mod_k, (h.data_ptr(), scale.data_ptr(), shift.data_ptr(), b, r, c, int(threads)),
             h.numel())
        return h

    def residual(x, h, gate):
        if not (valid(x) and valid(h) and valid(gate)):
            runtime["residual"]["fallbacks"] += 1
            if strict:
                raise RuntimeError("native residual strict violation")
            return tap._native_original_residual(x, h, gate)
        b, r, c = int(x.shape[0]), int(x.shape[-2]), int(x.shape[-1])
        call("residual", res_k, (x.data_ptr(), h.data_ptr(), gate.data_ptr(), b, r, c, int(threads)),
             x.numel())
        return x

    def add_inplace(x, h):
        if not (valid(x) and valid(h) and x.shape == h.shape):
            runtime["add"]["fallbacks"] += 1
            if strict:
                raise RuntimeError("native add strict violation")
            x.add_(h)
            return x
        call("add", add_k, (x.data_ptr(), h.data_ptr(), x.numel(), int(threads)), x.numel())
        return x

    tap._native_original_modulate = tap._modulate_inplace_preserve_order
    tap._native_original_residual = tap._residual_gate_inplace_preserve_order
    tap._modulate_inplace_preserve_order = modulate
    tap._residual_gate_inplace_preserve_order = residual
    selected = []

    def make_forward(name):
        def forward(self, x, mod=None, rotary_emb=None):
            if self.modulation:
                if not self.share_mod:
                    mod = self.adaLN_modulation(mod)
                if getattr(self, "shift_table", None) is not None:
                    mod = mod.contiguous().clone()
                    add_inplace(mod, self.shift_table.type(mod.dtype).contiguous())
                shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (
                    c.contiguous() for c in mod.chunk(6, dim=1))
                h = modulate(self.norm1(x), scale_msa, shift_msa)
                h = self.attn(h, rope_emb=rotary_emb)
                x = residual(x, h, gate_msa)
                h = modulate(self.norm2(x), scale_mlp, shift_mlp)
                return residual(x, self.mlp(h), gate_mlp)
            x = add_inplace(x, self.attn(self.norm1(x), rope_emb=rotary_emb))
            return add_inplace(x, self.mlp(self.norm2(x)))
        return forward

    for name, module in flow_model.named_modules():
        if module.__class__.__name__ != "UnifiedTransformerBlock":
            continue
        module._native_avx512_add_inplace = add_inplace
        module._native_avx512_modulate_inplace = modulate
        module._original_forward_native_block_elementwise = module.forward
        module.forward = types.MethodType(make_forward(name), module)
        selected.append(name)
    flow_model._native_avx512_add_inplace = add_inplace
    flow_model._native_avx512_modulate_inplace = modulate
    return {"enabled": True, "kind": "native_f32_cuda_block_elementwise_patch",
            "library_path": lib_path.as_posix(), "threads": int(threads), "strict": bool(strict),
            "selected_count": len(selected), "selected": selected, "runtime": runtime}


# --------------------------------------------------------------------------------------
# Packed attention helpers (RoPE + RMSNorm + pack -> packed exact SDPA)
# --------------------------------------------------------------------------------------
def apply_triposplat_native_qkv_packed_attention_helpers_patch(
    flow_model,
    *,
    postprocess_library: str | None = None,
    sdpa_library: str | None = None,
    threads: int = 2,
    include_regex: str = r"^blocks[.][0-9]+[.]attn$",
    strict: bool = True,
    attention_module=None,
):
    """``attention_module`` (no reference counterpart): the module holding the attention
    helpers; the reference imports it as ``triposplat_attention_patch``."""
    import torch

    tap = attention_module if attention_module is not None else importlib.import_module(
        "triposplat_attention_patch")
    post_lib, postprocess_path = _library(postprocess_library)
    sdpa_lib, sdpa_path = _library(sdpa_library)
    postprocess = post_lib.triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2
    postprocess_selected = post_lib.triposplat_q_kv_selected_rope_rmsnorm_pack_f32_avx512_v2
    sdpa = sdpa_lib.triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd

    include = re.compile(include_regex)
    selected_names, selected_ids = [], set()
    for name, module in flow_model.named_modules():
        if module.__class__.__name__ != "RopeMultiHeadAttention" or include.search(name) is None:
            continue
        if module._type == "self" and module.use_rope and module.qk_rms_norm and module.head_dim == 64:
            selected_names.append(name)
            selected_ids.add(id(module))
    if strict and not selected_names:
        raise RuntimeError(f"packed Attention helper patch selected no modules with {include_regex!r}")

    workspace = {}
    runtime = {"calls": 0, "selected_row_calls": 0, "key_bias_calls": 0, "postprocess_seconds": 0.0,
               "sdpa_seconds": 0.0, "workspace_allocations": 0, "workspace_capacity_bytes": 0,
               "qkv_input_copies": 0, "frequency_copies": 0, "selected_index_copies": 0, "fallbacks": 0}

    def acquire(name, elements, device):
        tensor = workspace.get(name)
        if tensor is None or tensor.numel() < elements or tensor.device != device:
            tensor = torch.empty(elements, dtype=torch.float32, device=device)
            workspace[name] = tensor
            runtime["workspace_allocations"] += 1
            runtime["workspace_capacity_bytes"] = sum(v.numel() * 4 for v in workspace.values())
        return tensor[:elements]

    def stage(timing_callback, name, function, shape):
        if timing_callback is None:
            return function()
        started = time.perf_counter()
        try:
            return function()
        finally:
            timing_callback(name, time.perf_counter() - started, shape=shape)

    def frequency_view(rope_emb, b, length, heads, dim):
        frequency = torch.view_as_real(rope_emb).reshape(*rope_emb.shape[:-1], dim)
        if not frequency.is_contiguous():
            frequency = frequency.contiguous()
            runtime["frequency_copies"] += 1
        frequency_batches = int(frequency.shape[0])
        if frequency_batches not in (1, b) or frequency.numel() != frequency_batches * length * heads * dim:
            raise RuntimeError(f"packed Attention frequency mismatch: {tuple(rope_emb.shape)}")
        return frequency, frequency_batches

    def launch(kernel, args, what):
        _native.use_current_stream(post_lib)
        if sdpa_lib is not post_lib:
            _native.use_current_stream(sdpa_lib)
        started = time.perf_counter()
        status = int(kernel(*args))
        elapsed = time.perf_counter() - started
        if status != 0:
            raise RuntimeError(f"{what} returned {status}: {_last_error(post_lib)}")
        return elapsed

    def usable(attn, x, rope_emb):
        return (id(attn) in selected_ids and _is_cuda_f32(x) and rope_emb is not None
                and rope_emb.device.type == "cuda" and rope_emb.dtype == torch.complex64)

    def run(attn, x, rope_emb, key_bias, timing_callback):
        b, length, channels = (int(v) for v in x.shape)
        heads, dim = int(attn.num_heads), int(attn.head_dim)
        if not usable(attn, x, rope_emb):
            return None
        length_padded = (length + 15) & ~15
        qkv = stage(timing_callback, "attention.qkv_projection", lambda: attn.qkv(x), [b, length, 3 * channels])
        if not qkv.is_contiguous():
            qkv = qkv.contiguous()
            runtime["qkv_input_copies"] += 1
        frequency, frequency_batches = frequency_view(rope_emb, b, length, heads, dim)
        dev = x.device
        q = acquire("q", b * heads * length * dim, dev).view(b, heads, length, dim)
        packed_elements = b * heads * dim * length_padded
        packed_k = acquire("k", packed_elements, dev).view(b, heads, dim, length_padded)
        packed_v = acquire("v", packed_elements, dev).view(b, heads, dim, length_padded)
        output = acquire("out", b * length * heads * dim, dev).view(b, length, heads, dim)
        elapsed = launch(postprocess, (qkv.data_ptr(), frequency.data_ptr(), attn.q_norm.gamma.data_ptr(),
                                       attn.k_norm.gamma.data_ptr(), q.data_ptr(), packed_k.data_ptr(),
                                       packed_v.data_ptr(), b, length, heads, dim, length_padded,
                                       frequency_batches, int(threads)), "packed QKV postprocess")
        runtime["postprocess_seconds"] += elapsed
        if timing_callback is not None:
            timing_callback("attention.rope_qknorm_layout_pack", elapsed, shape=[b, heads, length, dim])
        bias_pointer, has_bias, bias_length = None, 0, 0
        if key_bias is not None:
            bias = key_bias.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
            if bias.numel() != length:
                raise RuntimeError(f"packed Attention key bias mismatch: {bias.numel()} != {length}")
            bias_pointer, has_bias, bias_length = bias.data_ptr(), 1, length
            runtime["key_bias_calls"] += 1
        elapsed = launch(sdpa, (q.data_ptr(), packed_k.data_ptr(), packed_v.data_ptr(), bias_pointer,
                                output.data_ptr(), b, heads, length, length, dim, length_padded, has_bias,
                                bias_length, int(threads)), "packed SDPA")
        runtime["sdpa_seconds"] += elapsed
        if timing_callback is not None:
            timing_callback("attention.sdpa", elapsed, shape=[b, heads, length, dim])
        runtime["calls"] += 1
        return stage(timing_callback, "attention.out_projection",
                     lambda: attn.out(output.view(b, length, channels)), [b, length, channels])

    def run_selected(attn, x, selected_idx, rope_emb, timing_callback):
        b, length, channels = (int(v) for v in x.shape)
        selected_length = int(selected_idx.numel())
        heads, dim = int(attn.num_heads), int(attn.head_dim)
        native_range = getattr(attn.qkv, "_native_avx512_forward_range", None)
        if (not usable(attn, x, rope_emb) or native_range is None or selected_idx.device.type != "cuda"
                or selected_idx.dtype != torch.int64):
            return None
        if not selected_idx.is_contiguous():
            selected_idx = selected_idx.contiguous()
            runtime["selected_index_copies"] += 1
        x_selected = stage(timing_callback, "attention.selected_index", lambda: x.index_select(1, selected_idx),
                           [b, selected_length, channels])
        q = stage(timing_callback, "attention.q_projection", lambda: native_range(x_selected, 0, channels),
                  [b, selected_length, channels])
        kv = stage(timing_callback, "attention.kv_projection", lambda: native_range(x, channels, 2 * channels),
                   [b, length, 2 * channels])
        if not q.is_contiguous():
            q = q.contiguous()
            runtime["qkv_input_copies"] += 1
        if not kv.is_contiguous():
            kv = kv.contiguous()
            runtime["qkv_input_copies"] += 1
        frequency, frequency_batches = frequency_view(rope_emb, b, length, heads, dim)
        length_padded = (length + 15) & ~15
        dev = x.device
        q_packed = acquire("q", b * heads * selected_length * dim, dev).view(b, heads, selected_length, dim)
        packed_elements = b * heads * dim * length_padded
        packed_k = acquire("k", packed_elements, dev).view(b, heads, dim, length_padded)
        packed_v = acquire("v", packed_elements, dev).view(b, heads, dim, length_padded)
        output = acquire("out", b * selected_length * heads * dim, dev).view(b, selected_length, heads, dim)
        elapsed = launch(postprocess_selected,
                         (q.data_ptr(), kv.data_ptr(), frequency.data_ptr(), selected_idx.data_ptr(),
                          attn.q_norm.gamma.data_ptr(), attn.k_norm.gamma.data_ptr(), q_packed.data_ptr(),
                          packed_k.data_ptr(), packed_v.data_ptr(), b, selected_length, length, heads, dim,
                          length_padded, frequency_batches, int(threads)), "selected packed Q/KV postprocess")
        runtime["postprocess_seconds"] += elapsed
        if timing_callback is not None:
            timing_callback("attention.rope_qknorm_layout_pack", elapsed,
                            shape={"q": [b, heads, selected_length, dim], "k": [b, heads, length, dim]})
        elapsed = launch(sdpa, (q_packed.data_ptr(), packed_k.data_ptr(), packed_v.data_ptr(), None,
                                output.data_ptr(), b, heads, selected_length, length, dim, length_padded, 0, 0,
                                int(threads)), "selected packed SDPA")
        runtime["sdpa_seconds"] += elapsed
        if timing_callback is not None:
            timing_callback("attention.sdpa", elapsed,
                            shape={"q": [b, heads, selected_length, dim], "k": [b, heads, length, dim]})
        runtime["calls"] += 1
        runtime["selected_row_calls"] += 1
        return stage(timing_callback, "attention.out_projection",
                     lambda: attn.out(output.view(b, selected_length, channels)), [b, selected_length, channels])

    original_standard = tap._rope_self_attention_standard
    original_key_bias = tap._rope_self_attention_with_key_bias
    original_selected = tap._rope_self_attention_selected_rows

    def packed_standard(attn, x, rope_emb, *, backend="default", compute_dtype="model", query_chunk_size=128,
                        contiguous_qkv=True, timing_callback=None):
        if backend == "native_avx512_exact" and compute_dtype == "model":
            result = run(attn, x, rope_emb, None, timing_callback)
            if result is not None:
                return result
        runtime["fallbacks"] += 1
        if strict and id(attn) in selected_ids:
            raise RuntimeError("selected standard Attention fell back from packed path")
        return original_standard(attn, x, rope_emb, backend=backend, compute_dtype=compute_dtype,
                                 query_chunk_size=query_chunk_size, contiguous_qkv=contiguous_qkv,
                                 timing_callback=timing_callback)

    def packed_key_bias(attn, x, rope_emb, key_bias, *, backend="default", timing_callback=None):
        if backend == "native_avx512_exact":
            result = run(attn, x, rope_emb, key_bias, timing_callback)
            if result is not None:
                return result
        runtime["fallbacks"] += 1
        if strict and id(attn) in selected_ids:
            raise RuntimeError("selected key-bias Attention fell back from packed path")
        return original_key_bias(attn, x, rope_emb, key_bias, backend=backend, timing_callback=timing_callback)

    def packed_selected(attn, x, selected_idx, rope_emb, *, backend, compute_dtype, query_chunk_size,
                        round_qkv_to_fp16=False, round_v_to_fp16=False, round_attn_core_to_fp16=False,
                        half_sequence=False, key_bias=None, timing_callback=None):
        exact = (backend == "native_avx512_exact" and compute_dtype == "model" and not round_qkv_to_fp16
                 and not round_v_to_fp16 and not round_attn_core_to_fp16 and not half_sequence
                 and key_bias is None)
        if exact:
            result = run_selected(attn, x, selected_idx, rope_emb, timing_callback)
            if result is not None:
                return result
            runtime["fallbacks"] += 1
            if strict and id(attn) in selected_ids:
                raise RuntimeError("selected-row Attention fell back from packed path")
        return original_selected(attn, x, selected_idx, rope_emb, backend=backend, compute_dtype=compute_dtype,
                                 query_chunk_size=query_chunk_size, round_qkv_to_fp16=round_qkv_to_fp16,
                                 round_v_to_fp16=round_v_to_fp16,
                                 round_attn_core_to_fp16=round_attn_core_to_fp16, half_sequence=half_sequence,
                                 key_bias=key_bias, timing_callback=timing_callback)

    tap._rope_self_attention_standard = packed_standard
    tap._rope_self_attention_with_key_bias = packed_key_bias
    tap._rope_self_attention_selected_rows = packed_selected
    return {
        "enabled": bool(selected_names),
        "kind": "native_attention_helpers_qkv_packed_exact_cuda",
        "postprocess_library": postprocess_path.as_posix(),
        "sdpa_library": sdpa_path.as_posix(),
        "threads": int(threads),
        "include_regex": include_regex,
        "selected_count": len(selected_names),
        "selected": selected_names,
        "runtime": runtime,
        "coverage": "positive standard, negative key-bias, and final positive selected-query helpers",
        "semantics": "RoPE -> per-head RMSNorm -> packed K/V, then the exact online-softmax SDPA "
                     "(split-fp16 tensor-core products, fp32 softmax); Q only for consumed rows in "
                     "the selected-query helper.",
    }


__all__ = [
    "apply_triposplat_native_rnf8_avx512_patch",
    "apply_triposplat_native_norm_rope_avx512_patch",
    "apply_triposplat_native_gelu_avx512_patch",
    "apply_triposplat_native_silu_avx512_patch",
    "apply_triposplat_native_block_elementwise_avx512_patch",
    "apply_triposplat_native_qkv_packed_attention_helpers_patch",
]
