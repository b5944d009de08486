"""The NF24 packer restatement reproduces the reference packer's codes exactly
(golden codes were made by scripts/native_linear_rnf8_avx512_patch.py:75-87)."""
import numpy as np
import pytest
import torch

from nf24_pack import dequantize_nf24_i16, make_nf8_codebook, quantize_nf24_i16_per_output_channel
from conftest import GOLDEN


def test_codebook_matches_reference():
    np.testing.assert_array_equal(make_nf8_codebook(torch).numpy(), np.load(GOLDEN / "nf8_codebook.npy"))


@pytest.mark.parametrize("case", ["gemm_25x96x64", "gemm_3x96x5_tail", "gemm_130x256x144",
                                  "gemm_33x160x96_range32_48"])
def test_pack_bit_exact(golden, case):
    g = golden(case)
    codes, scales, err = quantize_nf24_i16_per_output_channel(torch.from_numpy(g["w"]))
    np.testing.assert_array_equal(codes[0].numpy(), g["code01_t"])
    np.testing.assert_array_equal(codes[1].numpy(), g["q2_t"])
    np.testing.assert_array_equal(scales[0].numpy(), g["scale"])
    assert codes[1] is codes[2] and scales[0] is scales[1] is scales[2]
    w_hat = dequantize_nf24_i16(codes[0], codes[1], scales[0])
    assert float((w_hat - torch.from_numpy(g["w"])).abs().max()) <= err["weight_max_abs"] * 1.0001 + 1e-12


def test_pack_code_range():
    torch.manual_seed(0)
    w = torch.randn(512, 1024) * 0.02
    codes, _, err = quantize_nf24_i16_per_output_channel(w)
    # by construction |4*q0 + q1| <= 4*127 + 128; the GEMM's exact fp16 decode needs |q01| <= 1023
    assert int(codes[0].abs().max()) <= 636
    assert err["weight_relative_rmse"] < 1e-5
