"""FP8 per-token quantiser on the GPU vs the CPU oracle and the reference's golden vectors (bit-exact)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import fp8
from tests.helpers import bits_of, codes_of, outlier_activations, to_bf16_tensor
from vflash_b200.kernels import quantize_fp8_rows
from vflash_b200.native.h3_fp8_activation import quantize_activation

pytestmark = pytest.mark.gpu
DEV = "cuda"


def check_against_oracle(x: torch.Tensor, pad_to: int = 16):
    codes, scales = quantize_fp8_rows(x, pad_to=pad_to)
    want_codes, want_scales = fp8.quantize_activation(bits_of(x), pad_to=pad_to)
    np.testing.assert_array_equal(codes_of(codes), want_codes)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), want_scales.view(np.uint32))


@pytest.mark.parametrize("name", ["outliers", "wide", "k16", "k24", "k40", "ties", "subnormal", "zeros"])
def test_golden_vectors_bit_exact(golden, name):
    x = to_bf16_tensor(golden[f"q_{name}_x"], DEV)
    codes, scales = quantize_fp8_rows(x)
    np.testing.assert_array_equal(codes_of(codes), golden[f"q_{name}_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden[f"q_{name}_scales"])


@pytest.mark.parametrize("rows", [1, 16, 17])
def test_strided_value_half_and_guard_lanes(golden, rows):
    base = to_bf16_tensor(golden[f"q_strided{rows}_base"], DEV)
    before = bits_of(base).copy()
    codes, scales = quantize_activation(base[:, :64])
    np.testing.assert_array_equal(codes_of(codes), golden[f"q_strided{rows}_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden[f"q_strided{rows}_scales"])
    np.testing.assert_array_equal(bits_of(base), before)  # input and NaN guard lanes untouched


@pytest.mark.parametrize("rows,cols", [(4099, 4096), (33, 5376), (20, 14336), (9, 16384), (5, 32768),
                                       (300, 24), (7, 1001), (130, 8)])
def test_seeded_shapes_bit_exact(rows, cols):
    check_against_oracle(outlier_activations(rows, cols, 1000 + cols).to(DEV))


def test_unaligned_view_takes_the_scalar_path_bit_exact():
    x = outlier_activations(19, 513, 9).to(DEV)
    check_against_oracle(x[:, 1:])  # 2-byte offset rows: no 16-byte vector loads


def test_every_bf16_value_bit_exact():
    # All 65536 bf16 bit patterns (NaN/inf replaced by 0), 256 per row: every
    # exponent range meets a different scale.
    patterns = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    values = fp8.bf16_value(patterns)
    patterns = np.where(np.isfinite(values), patterns, 0).astype(np.uint16)
    check_against_oracle(to_bf16_tensor(patterns.reshape(256, 256), DEV))


def test_every_bf16_value_at_unit_scale_bit_exact():
    # Rows whose amax is exactly 448 get scale 1, so every bf16 value in
    # [-448, 448] goes through the e4m3 rounding unscaled.
    values = fp8.bf16_value(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    inside = np.sort(values[np.isfinite(values) & (np.abs(values) <= 448)])
    cols = 256
    rows = -(-inside.size // (cols - 1))
    grid = np.zeros((rows, cols), np.float32)
    flat = np.zeros(rows * (cols - 1), np.float32)
    flat[: inside.size] = inside
    grid[:, 1:] = flat.reshape(rows, cols - 1)
    grid[:, 0] = 448.0
    check_against_oracle(to_bf16_tensor(fp8.bf16_bits(grid), DEV))


def test_non_finite_rows_against_the_reference(golden):
    # Rows holding +-inf (scale inf: finite values -> signed zero codes, infinities -> NaN),
    # NaN (scale 1) and -0, frozen from the reference's CPU quantiser.  Scales and every non-NaN
    # code are bit-exact.  A NaN code's sign bit is the platform's: x86 arithmetic returns a
    # negative default NaN for inf / inf and keeps a NaN operand's sign, CUDA arithmetic returns
    # the canonical positive NaN, so the reference itself gives 0xff on the CPU where a CUDA
    # run of the same expression gives 0x7f.  Both bytes decode to NaN; here they must sit at
    # the same places.  A row holding both a NaN and an infinity has scale 1, and its +-inf
    # must clamp to +-448 as in the reference (not turn into NaN).
    x = to_bf16_tensor(golden["q_specials_x"], DEV)
    codes, scales = quantize_fp8_rows(x)
    got, want = codes_of(codes), golden["q_specials_codes"]
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), golden["q_specials_scales"].view(np.uint32))
    got_nan, want_nan = (got & 0x7F) == 0x7F, (want & 0x7F) == 0x7F
    np.testing.assert_array_equal(got_nan, want_nan)
    np.testing.assert_array_equal(got[~got_nan], want[~want_nan])
    assert want_nan.any()


def test_nan_row_gets_unit_scale_like_torch():
    x = outlier_activations(4, 64, 3)
    x[2, 5] = float("nan")
    check_against_oracle(x.to(DEV))


def test_row_offsets_beyond_int32():
    # A strided view whose row stride x rows exceeds 2**31 elements
    # (the long-video FFN value half); offsets must be computed in 64 bits.
    cols = 256
    stride = 2**30 + 128
    rows = 3
    storage = torch.zeros((rows - 1) * stride + cols, dtype=torch.bfloat16, device=DEV)
    view = storage.as_strided((rows, cols), (stride, 1))
    src = outlier_activations(rows, cols, 77).to(DEV)
    view.copy_(src)
    codes, scales = quantize_fp8_rows(view)
    ref_codes, ref_scales = quantize_fp8_rows(src.contiguous())
    assert torch.equal(codes.view(torch.uint8), ref_codes.view(torch.uint8))
    assert torch.equal(scales, ref_scales)
    del storage


@pytest.mark.parametrize("cols", [4096, 1001])
def test_row_maxima_and_given_maxima_reproduce_the_full_quantiser(cols):
    from vflash_b200.kernels import row_absmax

    x = outlier_activations(300, cols, 4).to(DEV)
    x[7, 3] = float("nan")
    amax = row_absmax(x)
    want = x.float().abs().amax(dim=1)
    assert torch.equal(torch.isnan(amax), torch.isnan(want))
    assert torch.equal(amax[~torch.isnan(amax)], want[~torch.isnan(want)])
    codes, scales = quantize_fp8_rows(x)
    codes2, scales2 = quantize_fp8_rows(x, amax=amax)
    assert torch.equal(codes.view(torch.uint8), codes2.view(torch.uint8))
    assert torch.equal(scales, scales2)
    # a column slice quantised with the full row's maxima gives the full row's codes
    half = (cols // 2) // 8 * 8 or cols
    codes3, scales3 = quantize_fp8_rows(x[:, :half], amax=amax)
    assert torch.equal(codes3.view(torch.uint8), codes.view(torch.uint8)[:, :half])
    assert torch.equal(scales3, scales)


def test_drop_in_refuses_unbounded_widths():
    with pytest.raises(ValueError, match="SM100"):
        quantize_activation(torch.zeros(4, 8, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError, match="SM100"):
        quantize_activation(torch.zeros(4, 64, dtype=torch.float32, device=DEV))


def test_reference_named_torch_quantiser_matches_the_oracle():
    from vflash_b200.native.h3_fp8_linear import _quantize_activation_torch

    x = outlier_activations(37, 320, 21).to(DEV)
    codes, scales = _quantize_activation_torch(x)
    want_codes, want_scales = fp8.quantize_activation(bits_of(x))
    np.testing.assert_array_equal(codes_of(codes), want_codes)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), want_scales.view(np.uint32))
