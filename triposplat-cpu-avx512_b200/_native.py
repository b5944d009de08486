"""Loader and thin ctypes bindings for ``libtriposplat_b200.so``.

The library is the product: every hot-path call in this package goes through it.
There is no CPU or PyTorch fallback — if the library is missing or no CUDA
device is present, ``load()`` raises.
"""
from __future__ import annotations

import ctypes
import os
from functools import lru_cache
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEFAULT_LIBRARY = HERE / "libtriposplat_b200.so"

VP = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float
U64P = ctypes.POINTER(ctypes.c_uint64)

# name -> (argtypes, restype); mirrors include/triposplat_b200.h
SIGNATURES: dict[str, tuple[list, object]] = {
    # runtime
    "triposplat_b200_set_stream": ([VP], None),
    "triposplat_b200_get_stream": ([], VP),
    "triposplat_b200_status": ([], I),
    "triposplat_b200_clear_status": ([], None),
    "triposplat_b200_workspace_reserve": ([ctypes.c_uint64], I),
    "triposplat_b200_workspace_stats": ([U64P, U64P], I),
    "triposplat_b200_workspace_release": ([], None),
    "triposplat_b200_abi_version": ([], I),
    "triposplat_b200_launch_count": ([], ctypes.c_uint64),
    "triposplat_b200_last_error": ([], ctypes.c_char_p),
    "triposplat_b200_profile_enable": ([I], None),
    "triposplat_b200_profile_collect": ([U64P, ctypes.POINTER(ctypes.c_double), I], I),
    "triposplat_b200_profile_collect2": ([U64P, ctypes.POINTER(ctypes.c_double), I, I], I),
    # NF24 GEMM
    "triposplat_gemm_rnf8_avx512": ([VP] * 10 + [I] * 7, I),
    "triposplat_gemm_rnf8_avx512_range": ([VP] * 10 + [I] * 9, I),
    "triposplat_gemm_rnf8_avx512_tail": ([VP] * 10 + [I] * 7, I),
    "triposplat_gemm_rnf8_avx512_row_tile": ([], I),
    "triposplat_gemm_rnf8_avx512_residual_mode": ([], I),
    # fused MLP / QKV projection
    "triposplat_mlp_nf24_gelu_f32_avx512": ([VP] * 10 + [I] * 7, I),
    "triposplat_mlp_nf24_gelu_chunked_f32_avx512": ([VP] * 11 + [I] * 9, I),
    "triposplat_mlp_nf24_row_tile": ([], I),
    "triposplat_mlp_nf24_hidden_workspace_bytes_per_thread": ([], I),
    "triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512": ([VP] * 15 + [I] * 10, I),
    "triposplat_gemm_nf24_qkv_direct_row_tile": ([], I),
    "triposplat_gemm_nf24_qkv_direct_residual_mode": ([], I),
    "triposplat_gemm_nf24_qkv_direct_tile_bytes": ([], I),
    "triposplat_gemm_nf24_noalloc": ([VP] * 10 + [I] * 7, I),
    "triposplat_b200_split_bytes": ([I, I], ctypes.c_uint64),
    "triposplat_b200_split_f32": ([VP, I, I, I, VP], I),
    "triposplat_b200_ln_modulate_split": ([VP, I, I, F, VP, VP, I, I, VP], I),
    "triposplat_b200_ln_modulate_split_bound": ([VP, I, I, F, VP, VP, I, I, VP, VP, I, F, F], I),
    "triposplat_b200_gemm_nf24_split": ([VP, I, I] + [VP] * 5 + [I, I, I, VP, I, I], I),
    "triposplat_b200_gemm_nf24_split_range": ([VP, I, I] + [VP] * 5 + [I] * 5 + [VP, I, I], I),
    "triposplat_b200_nf24_codes_to_nk": ([VP, VP, I, I, VP, VP], I),
    "triposplat_b200_ipc_alloc": ([ctypes.c_uint64, VP, VP], I),
    "triposplat_b200_ipc_free": ([VP], I),
    "triposplat_b200_ipc_open": ([VP, VP], I),
    "triposplat_b200_ipc_close": ([VP], I),
    "triposplat_b200_peer_barrier": ([VP, I, I, VP], I),
    "triposplat_b200_peer_reduce_residual_f32": ([VP, I, VP, I64, I, I, VP, I, I64], I),
    "triposplat_b200_gemm_nf24_split_nk": ([VP, I, I, VP, VP, I] + [VP] * 3 + [I] * 5 + [VP, I, I], I),
    # exact SDPA
    "triposplat_sdpa_f32_avx512_exact_q8t512": ([VP] * 5 + [I] * 8, I),
    "triposplat_sdpa_f32_avx512_exact_q8": ([VP] * 5 + [I] * 8, I),
    "triposplat_sdpa_f32": ([VP] * 5 + [I] * 8, I),
    "triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd": ([VP] * 5 + [I] * 9, I),
    "triposplat_sdpa_f32_cuda_bias_bh": ([VP] * 4 + [ctypes.c_longlong, VP] + [I] * 5, I),
    "triposplat_sdpa_packed_output_is_blhd": ([], I),
    "triposplat_b200_attn_q_planes_bytes": ([I, I], ctypes.c_uint64),
    "triposplat_b200_attn_kv_planes_bytes": ([I, I], ctypes.c_uint64),
    "triposplat_b200_qkv_split_rows_f32": ([VP] * 4 + [I] * 6 + [VP, VP], I),
    "triposplat_b200_kv_planes_gather": ([VP, VP, I, I, I, I], I),
    "triposplat_b200_attend_rows_f32": ([VP, VP, VP, I, I, I, I], I),
    "triposplat_b200_attend_rows_split": ([VP, VP, I, I, I, I, VP], I),
    "triposplat_b200_kv_split_f32": ([VP, VP, I, I, I, VP], I),
    "triposplat_b200_q_split_f32": ([VP, VP, I, I, I, VP], I),
    "triposplat_sdpa_key_tile": ([], I),
    "triposplat_sdpa_query_block": ([], I),
    "triposplat_sdpa_q8t512_profile_reset": ([], None),
    "triposplat_sdpa_q8t512_profile_get": ([U64P] * 5, I),
    "triposplat_sdpa_q8t512_workspace_stats": ([U64P, U64P], I),
    "triposplat_sdpa_q8t512_workspace_release": ([], None),
    # prologue / epilogue kernels
    "triposplat_layernorm_f32_avx512": ([VP] * 4 + [I64, I, F, I, I], I),
    "triposplat_multihead_rmsnorm_f32_avx512": ([VP] * 3 + [I64, I, I, F, I], I),
    "triposplat_rope_complex_f32_avx512": ([VP] * 3 + [I64, I, I], I),
    "triposplat_gelu_tanh_f32_avx512": ([VP] * 2 + [I64, I], I),
    "triposplat_silu_f32_avx512": ([VP] * 2 + [I64, I], I),
    "triposplat_modulate_inplace_f32_avx512": ([VP] * 3 + [I] * 4, I),
    "triposplat_gated_residual_inplace_f32_avx512": ([VP] * 3 + [I] * 4, I),
    "triposplat_add_inplace_f32_avx512": ([VP] * 2 + [I64, I], I),
    "triposplat_cfg_combine_inplace_f32_avx512": ([VP] * 3 + [I, I64, I], I),
    "triposplat_euler_update_inplace_f32_avx512": ([VP] * 3 + [I, I64, I], I),
    "triposplat_ab2_update_inplace_f32_avx512": ([VP] * 5 + [I, I64, I], I),
    "triposplat_b200_cfg_euler_update_f32": ([VP] * 5 + [I, I64], I),
    "triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2": ([VP] * 7 + [I] * 7, I),
    "triposplat_qkv_rope_rmsnorm_pack_f32_avx512": ([VP] * 7 + [I] * 7, I),
    "triposplat_qkv_postprocess_token_tile": ([], I),
    "triposplat_qkv_postprocess_v2_tail_only_clear": ([], I),
    "triposplat_q_kv_selected_rope_rmsnorm_pack_f32_avx512_v2": ([VP] * 9 + [I] * 8, I),
    "triposplat_b200_q_kv_rmsnorm_pack_f32": ([VP] * 7 + [I] * 5, I),
    "triposplat_b200_qkv_rope_rmsnorm_sdpa_f32": ([VP] * 5 + [I] * 5, I),
    "triposplat_b200_q_kv_rmsnorm_sdpa_f32": ([VP] * 5 + [I] * 4, I),
    "triposplat_b200_qkv_rope_rmsnorm_sdpa_split": ([VP] * 4 + [I] * 4 + [VP], I),
    "triposplat_b200_q_kv_rmsnorm_sdpa_split": ([VP] * 4 + [I] * 4 + [VP], I),
    "triposplat_timestep_embedding_f32_avx512": ([VP] * 3 + [I] * 4, I),
    "triposplat_pcd_position_embedding_f32_avx512": ([VP] * 3 + [I64] + [I] * 5, I),
    "triposplat_mul_inplace_f32_avx512": ([VP, VP, I64, I], I),
    "triposplat_repo_phasor_f32_avx512": ([VP, VP, VP, I, VP, VP, I, VP, VP, I, VP, I64, I], I),
}


def library_path(path: str | os.PathLike | None = None) -> Path:
    p = Path(path or os.environ.get("TRIPOSPLAT_B200_LIBRARY", DEFAULT_LIBRARY))
    return p.resolve()


@lru_cache(maxsize=4)
def _load(path: str) -> ctypes.CDLL:
    if not Path(path).is_file():
        raise FileNotFoundError(
            f"{path} is missing: build it with `python triposplat-cpu-avx512_b200/build_lib.py`")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.argtypes = args
        fn.restype = res
    return lib


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    return _load(str(library_path(path)))


def bind(lib: ctypes.CDLL, name: str, args, res=I):
    fn = getattr(lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


def use_current_stream(lib: ctypes.CDLL) -> None:
    """Queue the library's next launches on PyTorch's current CUDA stream."""
    import torch

    lib.triposplat_b200_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def check_status(lib: ctypes.CDLL) -> None:
    st = int(lib.triposplat_b200_status())
    if st != 0:
        raise RuntimeError(f"a CUDA kernel of libtriposplat_b200 gave up on a wait (device status {st})")


def require_cuda(*tensors, what: str = "tensor") -> None:
    import torch

    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"{what} must be a CUDA tensor, got {t.device}")
        if not t.is_contiguous():
            raise ValueError(f"{what} must be contiguous")
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device")


KERNEL_FAMILIES = ("gemm_tc", "gemm_split", "gemm_simt", "sdpa_attn", "sdpa_split", "elementwise",
                   "peer_wait", "peer_copy")


def profile_collect(lib, keep: bool = False) -> dict:
    n = len(KERNEL_FAMILIES)
    launches = (ctypes.c_uint64 * n)()
    ms = (ctypes.c_double * n)()
    st = lib.triposplat_b200_profile_collect2(launches, ms, n, int(keep))
    if st != 0:
        raise RuntimeError(f"profile_collect returned {st}")
    return {k: {"launches": int(launches[i]), "ms": float(ms[i])} for i, k in enumerate(KERNEL_FAMILIES)}
