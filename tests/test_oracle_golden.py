"""Pin the CPU oracle against golden vectors frozen from the reference itself.

The fixtures come from tests/golden/make_golden.py, which imports Hansimov/vflash's
own ``_quantize_activation_torch`` and ``RowFP8Execution`` (CPU paths).
Quantisation must match bit for bit; linear outputs and transcendental
epilogues within the stated tolerances.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import epilogues as ep
from oracle import fp8

QUANT_CASES = ["outliers", "wide", "k16", "k24", "k40", "ties", "subnormal", "zeros", "specials"]


@pytest.mark.parametrize("name", QUANT_CASES)
def test_quantizer_matches_reference_bit_for_bit(golden, name):
    codes, scales = fp8.quantize_activation(golden[f"q_{name}_x"])
    np.testing.assert_array_equal(codes, golden[f"q_{name}_codes"])
    np.testing.assert_array_equal(scales.view(np.uint32), golden[f"q_{name}_scales"].view(np.uint32))


@pytest.mark.parametrize("rows", [1, 16, 17])
def test_strided_value_half_matches_reference(golden, rows):
    # tests/test_fp8_linear.py:99-120 of the reference: the value half of a
    # packed FFN projection (doubled row stride), a zero row and a bf16.tiny row.
    base = golden[f"q_strided{rows}_base"]
    codes, scales = fp8.quantize_activation(base[:, :64])
    np.testing.assert_array_equal(codes, golden[f"q_strided{rows}_codes"])
    np.testing.assert_array_equal(scales, golden[f"q_strided{rows}_scales"])
    padded = (rows + 15) // 16 * 16
    assert codes.shape == (padded, 64) and scales.shape == (padded, 1)
    assert scales[0, 0] == 1 and (codes[0] == 0).all()
    assert (codes[rows:] == 0).all() and (scales[rows:] == 1).all()


def test_e4m3_codec_round_trips_every_finite_code():
    codes = np.arange(256, dtype=np.uint8)
    values = fp8.e4m3_decode(codes)
    finite = ~np.isnan(values)
    np.testing.assert_array_equal(fp8.e4m3_encode(values[finite]), codes[finite])
    assert np.isnan(values[0x7F]) and np.isnan(values[0xFF])
    assert values[0x7E] == 448 and values[0x01] == 2.0**-9


def test_e4m3_encoder_rounds_to_nearest_even_against_torch():
    torch = pytest.importorskip("torch")
    gen = np.random.default_rng(5)
    x = np.concatenate([
        gen.normal(0, 50, 20000), gen.normal(0, 0.01, 20000),
        (np.arange(-3600, 3601) / 8.0),
    ]).astype(np.float32)
    x = np.clip(x, -448, 448)
    expected = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(fp8.e4m3_encode(x), expected)


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(6).normal(0, 1e3, 50000).astype(np.float32)
    expected = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(fp8.bf16_bits(x), expected)


def test_weight_only_linear_matches_reference(golden):
    torch = pytest.importorskip("torch")
    for case in ("wo_small", "wo_mid"):
        x = torch.from_numpy(golden[f"{case}_x"].view(np.int16)).view(torch.bfloat16)
        codes = torch.from_numpy(golden[f"{case}_codes"]).view(torch.float8_e4m3fn)
        scales = torch.from_numpy(golden[f"{case}_scales"])
        bias = torch.from_numpy(golden[f"{case}_bias"].view(np.int16)).view(torch.bfloat16)
        y = fp8.weight_only_linear(x, codes, scales, bias)
        expected = fp8.bf16_value(golden[f"{case}_y"])
        actual = y.float().numpy()
        # oneDNN's bf16 GEMM may block its reduction differently on another
        # host CPU; the result must still agree to bf16 precision.
        assert fp8.rel_l2(actual, expected) <= 4e-3, case


def test_weight_quantiser_matches_reference_expression(golden):
    # make_golden.py quantised the mid-size weight with the reference's own
    # activation expression per output row; the oracle's weight quantiser is
    # that expression without row padding.
    w = fp8.bf16_value(golden["wo_mid_w"])
    codes, scales = fp8.quantize_weight(w)
    np.testing.assert_array_equal(codes, golden["wo_mid_codes"])
    np.testing.assert_array_equal(scales, golden["wo_mid_scales"])


def test_strict_epilogues_match_eager_compositions(golden):
    np.testing.assert_array_equal(ep.silu_mul(golden["silu_packed"]), golden["silu_out"])
    np.testing.assert_array_equal(
        ep.gate_residual(golden["gr_residual"], golden["gr_gate"], golden["gr_projected"]),
        golden["gr_out"])
    np.testing.assert_array_equal(
        ep.qkv_direct_merge(golden["qkv_base"], golden["qkv_adapters"], golden["qkv_scalings"]),
        golden["qkv_out"])
    # tanh differs in the last fp32 bit between libraries (and where 1 + tanh
    # cancels, one library returns exactly 0): one bf16 ulp or 1e-6 absolute.
    got = fp8.bf16_value(ep.gelu_tanh(golden["gelu_y"]))
    want = fp8.bf16_value(golden["gelu_out"])
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() < 0.02


def test_w8a8_emulation_agrees_with_dequantised_matmul(golden):
    x = golden["wo_mid_x"]
    a_codes, a_scale = fp8.quantize_activation(x)
    y = fp8.w8a8_reference(a_codes[:33], a_scale[:33], golden["wo_mid_codes"], golden["wo_mid_scales"])
    f32 = fp8.dequant_matmul_f32(a_codes[:33], a_scale[:33], golden["wo_mid_codes"], golden["wo_mid_scales"])
    assert fp8.rel_l2(y, f32) < 5e-3


def test_oracle_modulate_matches_eager_torch_composition():
    # the reference kernel reproduces three eager bf16 TensorIterator kernels
    import torch

    from oracle import epilogues
    from tests.helpers import bits_of

    gen = torch.Generator().manual_seed(71)
    x = torch.randn(2, 5, 64, generator=gen).to(torch.bfloat16)
    scale = (torch.randn(5, 64, generator=gen) * 0.3).to(torch.bfloat16)
    shift = (torch.randn(5, 64, generator=gen) * 0.3).to(torch.bfloat16)
    eager = x * (1.0 + scale) + shift
    got = epilogues.modulate(bits_of(x), bits_of(scale), bits_of(shift))
    np.testing.assert_array_equal(got, bits_of(eager))


def test_oracle_rms_norm_matches_torch_cpu_within_one_ulp():
    import torch

    from oracle import epilogues
    from tests.helpers import bits_of

    gen = torch.Generator().manual_seed(72)
    x = (torch.randn(33, 4096, generator=gen) * 3).to(torch.bfloat16)
    w = (1 + torch.randn(4096, generator=gen) * 0.1).to(torch.bfloat16)
    ref = torch.nn.functional.rms_norm(x, (4096,), w, 1e-6)
    got = fp8.bf16_value(epilogues.rms_norm(bits_of(x), bits_of(w), 1e-6))
    want = ref.float().numpy()
    diff = np.abs(got - want)
    ulp = np.abs(want) * 2.0 ** -7
    assert (diff <= ulp).all()
    assert (diff == 0).mean() > 0.99


def test_oracle_rotary_matches_the_reference_eager_expression():
    # _apply_rotary (h3_native_denoiser.py:246-256) in eager bf16 torch, written out here
    import torch

    from oracle import epilogues
    from tests.helpers import bits_of

    gen = torch.Generator().manual_seed(73)
    for rd in (128, 64):
        x = torch.randn(2, 7, 3, 128, generator=gen).to(torch.bfloat16)
        cos = torch.randn(7, rd, generator=gen).to(torch.bfloat16)
        sin = torch.randn(7, rd, generator=gen).to(torch.bfloat16)
        rot, passthrough = x[..., :rd], x[..., rd:]
        first, second = rot.chunk(2, dim=-1)
        rotated = torch.cat((-second, first), dim=-1)
        c, s = cos[None, :, None, :], sin[None, :, None, :]
        eager = torch.cat((rot * c + rotated * s, passthrough), dim=-1)
        np.testing.assert_array_equal(epilogues.rotary(bits_of(x), bits_of(cos), bits_of(sin)), bits_of(eager))


@pytest.mark.parametrize("chunks", [1, 2])
def test_oracle_pack_qkv_matches_the_reference_layout(golden, chunks):
    q, k, v = golden[f"pack{chunks}_qkv"]
    np.testing.assert_array_equal(ep.pack_qkv(q, k, v, chunks), golden[f"pack{chunks}_out"])
    with pytest.raises(ValueError, match="destinations"):
        ep.pack_qkv(q[:, :, :6], k[:, :, :6], v[:, :, :6], 4)


def test_oracle_f64_to_bf16_rounds_once():
    # values at, just above and just below bf16 midpoints: a float32 detour that
    # rounds to nearest would land on the midpoint and round the tie wrongly
    from oracle.epilogues import f64_to_bf16_bits

    b = np.random.default_rng(0).integers(0, 0x7F00, 4096).astype(np.uint16)
    lo, hi = fp8.bf16_value(b).astype(np.float64), fp8.bf16_value(b + 1).astype(np.float64)
    mid, step = (lo + hi) / 2, hi - lo
    np.testing.assert_array_equal(f64_to_bf16_bits(mid), np.where(b & 1, b + 1, b).astype(np.uint16))
    np.testing.assert_array_equal(f64_to_bf16_bits(mid + step * 1e-9), (b + 1).astype(np.uint16))
    np.testing.assert_array_equal(f64_to_bf16_bits(mid - step * 1e-9), b)
    np.testing.assert_array_equal(f64_to_bf16_bits(-mid - step * 1e-9), (b + 1).astype(np.uint16) | 0x8000)


# --- NVFP4: the CPU restatement against FlashInfer's own outputs -------------
# tests/golden/nvfp4_flashinfer.npz holds FlashInfer's nvfp4_quantize and
# mm_fp4 results for seeded inputs, recorded on a B200 by
# tests/golden/make_nvfp4_golden.py (the reference's NVFP4 backend,
# h3_nvfp4_linear.py:102, 118-130).  The restatement uses exact reciprocals
# where FlashInfer uses rcp.approx, so it is held to >= 99.5 % of codes and
# scales identical, every differing code one e2m1 step away.

def _nvfp4_golden():
    import numpy as np

    from tests.conftest import GOLDEN

    return dict(np.load(GOLDEN / "nvfp4_flashinfer.npz"))


@pytest.mark.parametrize("case_name", ["c3_act", "c3_weight", "outliers_edges", "h3_width"])
def test_nvfp4_oracle_agrees_with_flashinfer_codes(case_name):
    import numpy as np

    from oracle import nvfp4
    from tests.golden.make_nvfp4_golden import DTYPES, QUANT_CASES, case_input, global_scale

    golden = _nvfp4_golden()
    name, rows, cols, seed, std, outliers, edges, tags = next(c for c in QUANT_CASES if c[0] == case_name)
    x = case_input(rows, cols, seed, std, outliers, edges)
    for tag in tags:
        values = x.to(DTYPES[tag]).float().numpy()
        gsf = float(golden[f"{name}.{tag}.gsf"])
        assert np.float32(gsf) == global_scale(x.to(DTYPES[tag])).numpy()  # the same expression on the host
        codes, sf = nvfp4.quantize(values, gsf)
        got = nvfp4.unpack(codes)
        want = nvfp4.unpack(golden[f"{name}.{tag}.codes"])
        assert got.shape == want.shape
        assert (got != want).mean() <= 5e-3
        step = np.abs(nvfp4.e2m1_decode(got) - nvfp4.e2m1_decode(want))
        assert step.max() <= 2.0  # one e2m1 step at most (the widest is 4 -> 6)
        assert (sf != golden[f"{name}.{tag}.sf"]).mean() <= 5e-3
        # the padding of the 128x4 layout is zero in both
        offsets = nvfp4.sf_offsets(*nvfp4.sf_padded_shape(rows, cols // 16))
        pad = np.ones(offsets.shape, bool)
        pad[:rows, : cols // 16] = False
        assert (golden[f"{name}.{tag}.sf"][offsets[pad]] == 0).all()


def test_nvfp4_oracle_emulates_mm_fp4_on_flashinfer_codes():
    import numpy as np

    from oracle import fp8, nvfp4
    from tests.golden.make_nvfp4_golden import LINEAR_CASE

    g = _nvfp4_golden()
    want = fp8.bf16_value(g["linear.mm_fp4"])
    got = nvfp4.w4a4_reference(g["linear.a_codes"], g["linear.a_sf"].reshape(-1), g["linear.w_codes"],
                               g["linear.w_sf"].reshape(-1), float(g["linear.alpha"]))
    assert got.shape == (LINEAR_CASE["rows"], LINEAR_CASE["n"])
    assert fp8.rel_l2(got, want) <= 1e-2
    # the exact emulation rounds once; the library kernel's fp32 accumulation order differs
    assert (got == want).mean() >= 0.95
    # the reference adds the bias as a separate bf16 op
    from tests.golden.make_nvfp4_golden import linear_inputs

    _x, _w, bias = linear_inputs()
    bias_bits = fp8.bf16_bits(bias.float().numpy())
    composed = fp8.bf16_round(want + fp8.bf16_value(bias_bits))
    np.testing.assert_array_equal(composed, fp8.bf16_value(g["linear.out"]))
