"""NVFP4 drop-in plumbing (ported from the reference's tests/test_h3_nvfp4_linear.py)
and the CPU oracle's format codecs.  CPU only; the operators are mocked."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4
from vflash_b200.native import h3_nvfp4_linear as nv


def weights(scale=4.0):
    return nv.NVFP4Weight(
        torch.zeros((128, 32), dtype=torch.uint8),
        torch.zeros((128, 4), dtype=torch.uint8),
        torch.tensor(2.0, dtype=torch.float32),
        torch.tensor(scale, dtype=torch.float32),
    )


def test_calibrated_input_scale_and_weight_alpha_reach_the_same_kernel(monkeypatch):
    seen = {}
    w = weights()

    def quantize(x, sf, **kwargs):
        seen["input"] = x
        assert sf is w.input_scale
        assert kwargs == {"sfLayout": "128x4", "do_shuffle": False}
        return torch.zeros((6, 32), dtype=torch.uint8), torch.zeros((128, 4), dtype=torch.uint8)

    def matmul(a, b, a_scale, b_scale, alpha, dtype, out, **kwargs):
        assert b.data_ptr() == w.packed.data_ptr() and b.shape == (32, 128)
        assert b_scale.data_ptr() == w.scales.data_ptr() and b_scale.shape == (4, 128)
        assert dtype == torch.bfloat16 and out is None
        assert alpha.item() == 0.5
        assert kwargs == dict(block_size=16, use_8x4_sf_layout=False, backend="cutlass", use_nvfp4=True)
        return torch.full((6, 128), 3.0, dtype=torch.bfloat16)

    monkeypatch.setattr(nv, "_require_device", lambda _: None)
    monkeypatch.setattr(nv, "_operators", lambda: ("128x4", quantize, matmul))
    engine = nv.NVFP4Execution()
    value = torch.ones((2, 3, 64), dtype=torch.float32)
    output = engine.linear(value, w, torch.ones(128, dtype=torch.bfloat16))
    assert seen["input"].dtype == torch.bfloat16
    assert output.shape == (2, 3, 128) and torch.equal(output, torch.full_like(output, 4.0))
    assert engine.calls == 1 and engine.rows == 6


def test_unsupported_device_refuses_before_backend_use(monkeypatch):
    def unexpected():
        raise AssertionError("backend should not be touched")

    monkeypatch.setattr(nv, "_operators", unexpected)
    with pytest.raises(ValueError, match="SM100"):
        nv.NVFP4Execution().linear(torch.ones((1, 64), dtype=torch.bfloat16), weights())


@pytest.mark.parametrize("scale", [0.0, -1.0, float("nan"), float("inf")])
def test_invalid_calibration_cannot_become_a_valid_model(scale):
    with pytest.raises(ValueError, match="positive and finite"):
        weights(scale)


def test_unpadded_quantizer_does_not_silently_select_another_arithmetic(monkeypatch):
    monkeypatch.setattr(nv, "_require_device", lambda _: None)

    def quantize(*args, **kwargs):
        return torch.zeros((3, 32), dtype=torch.uint8), torch.zeros((3, 4), dtype=torch.uint8)

    def unexpected(*args, **kwargs):
        raise AssertionError("kernel must not consume invalid scale layout")

    monkeypatch.setattr(nv, "_operators", lambda: ("128x4", quantize, unexpected))
    engine = nv.NVFP4Execution()
    with pytest.raises(ValueError, match="scale padding"):
        engine.linear(torch.ones((3, 64), dtype=torch.bfloat16), weights())
    assert engine.calls == 0


def test_native_operators_keep_the_reference_call_contract():
    layout, quantize, matmul = nv._operators()
    assert layout == "128x4"
    with pytest.raises(ValueError, match="128x4"):
        quantize(torch.zeros(1, 16, dtype=torch.bfloat16), torch.tensor(1.0), sfLayout="8x4",
                 do_shuffle=False)
    with pytest.raises(ValueError, match="block-16"):
        matmul(None, None, None, None, None, torch.bfloat16, None, block_size=32,
               use_8x4_sf_layout=False, backend="cutlass", use_nvfp4=True)


def test_e2m1_codec_round_trips_and_rounds_to_even():
    codes = np.arange(16, dtype=np.uint8)
    values = nvfp4.e2m1_decode(codes)
    np.testing.assert_array_equal(nvfp4.e2m1_encode(values)[values != 0], codes[values != 0])
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.75, 100.0], dtype=np.float32)
    np.testing.assert_array_equal(nvfp4.e2m1_decode(nvfp4.e2m1_encode(ties)),
                                  [0, 1, 1, 2, 2, 4, 4, 6, -1, 6])


def test_packing_puts_even_elements_in_the_low_nibble():
    codes = np.array([[1, 2, 3, 4]], dtype=np.uint8)
    np.testing.assert_array_equal(nvfp4.pack(codes), [[0x21, 0x43]])
    np.testing.assert_array_equal(nvfp4.unpack(nvfp4.pack(codes)), codes)


def test_128x4_layout_is_a_permutation():
    rows_pad, groups_pad = nvfp4.sf_padded_shape(200, 10)
    assert (rows_pad, groups_pad) == (256, 12)
    offsets = nvfp4.sf_offsets(rows_pad, groups_pad)
    assert np.array_equal(np.sort(offsets.ravel()), np.arange(rows_pad * groups_pad))
    # the formula of the layout: rows 0/32/64/96 of a k-tile share one 16-byte line
    assert offsets[0, 0] == 0 and offsets[32, 0] == 4 and offsets[1, 0] == 16 and offsets[0, 3] == 3
    assert offsets[0, 4] == 512 and offsets[128, 0] == 512 * (groups_pad // 4)
    matrix = np.random.default_rng(0).integers(0, 255, (rows_pad, groups_pad), dtype=np.uint8)
    np.testing.assert_array_equal(nvfp4.sf_unswizzle(nvfp4.sf_swizzle(matrix), rows_pad, groups_pad), matrix)


def test_quantiser_known_answer():
    # one 16-element block with amax 6 and gsf 1: sf = e4m3(1.0) = 0x38,
    # scale = 1, codes are the e2m1 encodings of the values themselves
    x = np.array([[6, -6, 0.5, 1, 1.5, 2, 3, 4, -0.5, -1, 0, 0.25, 0.75, 5, -5, 2.5]], dtype=np.float32)
    packed, sf = nvfp4.quantize(x, 1.0)
    assert sf[0] == 0x38 and sf.size == 128 * 4 and (sf[1:] == 0).all()
    decoded = nvfp4.e2m1_decode(nvfp4.unpack(packed))[0]
    np.testing.assert_array_equal(decoded, [6, -6, 0.5, 1, 1.5, 2, 3, 4, -0.5, -1, 0, 0, 1, 4, -4, 2])


def test_dequantise_matmul_agrees_with_exact_emulation():
    rng = np.random.default_rng(1)
    x = rng.normal(size=(64, 128)).astype(np.float32)
    w = (rng.normal(size=(128, 128)) * 0.02).astype(np.float32)
    gx, gw = 448 * 6 / np.abs(x).max(), 448 * 6 / np.abs(w).max()
    ap, asf = nvfp4.quantize(x, gx)
    wp, wsf = nvfp4.quantize(w, gw)
    alpha = np.float32(1 / gw) / np.float32(gx)
    y = nvfp4.w4a4_reference(ap, asf, wp, wsf, alpha)
    y32 = nvfp4.dequant_matmul_f32(ap, asf, wp, wsf, alpha)
    assert np.linalg.norm(y - y32) / np.linalg.norm(y32) < 5e-3
    # and the quantised product approximates the unquantised one
    assert np.linalg.norm(y32 - x @ w.T) / np.linalg.norm(x @ w.T) < 0.2
