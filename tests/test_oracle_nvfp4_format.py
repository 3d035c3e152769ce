"""The NVFP4 oracle's building blocks against the format definitions (CPU only).

The 128x4 scale layout (SF offset = mTile * (numKTiles * 512) + kTile * 512 +
(m % 32) * 16 + ((m % 128) / 32) * 4 + (k % 4)), e2m1 rounding to nearest even
with saturation at +-6, the nibble order of packed codes (element 2i in the
low nibble) and the error a quantise -> dequantise round trip may leave.  The
oracle is pinned to FlashInfer's own codes by the golden tests; these check
the pieces those tests rely on, at sizes and values the fixtures do not reach.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import nvfp4


@pytest.mark.parametrize("rows_pad,groups_pad", [(128, 4), (256, 8), (384, 12), (128, 256)])
def test_scale_offsets_are_a_permutation(rows_pad, groups_pad):
    off = nvfp4.sf_offsets(rows_pad, groups_pad).reshape(-1)
    assert np.array_equal(np.sort(off), np.arange(rows_pad * groups_pad))


def test_scale_offsets_follow_the_128x4_block_definition():
    rows_pad, groups_pad = 384, 12
    off = nvfp4.sf_offsets(rows_pad, groups_pad)
    k_tiles = groups_pad // 4
    rng = np.random.default_rng(3)
    for m, k in zip(rng.integers(0, rows_pad, 200), rng.integers(0, groups_pad, 200)):
        expected = (m // 128) * (k_tiles * 512) + (k // 4) * 512 + (m % 32) * 16 + ((m % 128) // 32) * 4 + k % 4
        assert off[m, k] == expected
    # one 128-row x 4-group block is one contiguous 512-byte run
    block = off[128:256, 4:8].reshape(-1)
    assert block.min() == 1 * k_tiles * 512 + 512 and block.max() == block.min() + 511


def test_scale_swizzle_round_trips():
    rng = np.random.default_rng(5)
    sf = rng.integers(0, 256, size=(256, 8), dtype=np.uint8)
    flat = nvfp4.sf_swizzle(sf)
    assert flat.shape == (256 * 8,)
    assert np.array_equal(nvfp4.sf_unswizzle(flat, 256, 8), sf)


def test_e2m1_encoder_rounds_ties_to_even_and_saturates():
    values = np.array([0.0, 0.25, 0.26, 0.5, 0.75, 1.0, 1.25, 1.5, 1.75, 2.0, 2.5, 3.0, 3.5, 4.0, 5.0, 5.01,
                       6.0, 7.0, 1e30, np.inf], dtype=np.float32)
    # e2m1 magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 are codes 0..7; ties go to the even code
    expected = np.array([0, 0, 1, 1, 2, 2, 2, 3, 4, 4, 4, 5, 6, 6, 6, 7, 7, 7, 7, 7], dtype=np.uint8)
    assert np.array_equal(nvfp4.e2m1_encode(values), expected)
    assert np.array_equal(nvfp4.e2m1_encode(-values), expected | 8)


def test_e2m1_codes_round_trip():
    codes = np.arange(16, dtype=np.uint8)
    assert np.array_equal(nvfp4.e2m1_encode(nvfp4.e2m1_decode(codes)), codes)


def test_packing_puts_the_even_element_in_the_low_nibble():
    codes = np.array([[1, 2, 15, 8]], dtype=np.uint8)
    packed = nvfp4.pack(codes)
    assert packed.tolist() == [[0x21, 0x8F]]
    assert np.array_equal(nvfp4.unpack(packed), codes)


def test_round_trip_error_is_within_one_scaled_step_of_each_block():
    rng = np.random.default_rng(11)
    rows, cols = 256, 512
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[rng.integers(0, rows, 40), rng.integers(0, cols, 40)] *= 20.0
    gsf = np.float32(448.0 * 6.0 / np.abs(x).max())
    packed, sf = nvfp4.quantize(x, float(gsf))
    deq = nvfp4.dequantize(packed, sf, rows, cols) / gsf  # codes x block scales, then the global scale
    block_amax = np.abs(x).reshape(rows, cols // 16, 16).max(axis=2)
    # RN on the e2m1 grid leaves at most half of its widest gap (4 -> 6) = 1 scaled unit; the
    # block's scale is amax / 6 rounded to e4m3 (at most 2^-4 relative above it)
    bound = np.repeat(block_amax / 6.0 * (1.0 + 2.0**-4) * (1.0 + 1e-3), 16, axis=1)
    assert np.all(np.abs(x - deq) <= bound + 1e-6)
    # and nothing is lost wholesale: the round trip keeps most of the signal
    rel = np.linalg.norm(x - deq) / np.linalg.norm(x)
    assert rel < 0.12
