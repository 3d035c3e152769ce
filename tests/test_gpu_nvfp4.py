"""NVFP4 quantiser and block-scaled GEMM on the GPU.

Bars:
* quantiser codes and 128x4 scales bit-exact against FlashInfer's own
  nvfp4_quantize (the reference's NVFP4 backend), frozen on a B200 by
  tests/golden/make_nvfp4_golden.py into tests/golden/nvfp4_flashinfer.npz
  (bf16 and fp16; config 3 rows, the H3 width, ragged rows, outliers and
  edge blocks); against the CPU oracle (exact reciprocals instead of
  rcp.approx) at least 99.5 % identical, every difference one code step;
* GEMM on FlashInfer's own codes vs FlashInfer mm_fp4 from the same file:
  rel-L2 <= 1e-2, and NVFP4Execution.linear vs the reference's composition
  (nvfp4_quantize, mm_fp4 with alpha / input_scale, + bias) rel-L2 <= 1e-2;
* GEMM vs the exact fp64 emulation of mm_fp4 on the same codes: identical
  bf16 except rare one-ulp flips; vs the fp32 dequantise-then-matmul
  rel-L2 <= 2e-2.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8, nvfp4
from tests.golden.make_nvfp4_golden import DTYPES, LINEAR_CASE, QUANT_CASES, case_input, linear_inputs
from tests.helpers import bf16_close, bits_of, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import Epilogue, nvfp4_gemm, nvfp4_quantize
from vflash_b200.native.h3_nvfp4_linear import NVFP4Execution, NVFP4Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "nvfp4_flashinfer.npz"


@pytest.fixture(scope="module")
def flashinfer_golden():
    return dict(np.load(GOLDEN))


def global_scale(x: torch.Tensor) -> torch.Tensor:
    return (448.0 * 6.0 / x.float().abs().max()).to(torch.float32).reshape(())


def weight_case(n, k, seed, device=DEV):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).to(torch.bfloat16).to(device)
    gsf = global_scale(w)
    packed, scales = nvfp4_quantize(w, gsf)
    return w, packed, scales.view(n, k // 16), (1.0 / gsf).to(torch.float32)


def test_quantizer_structure_and_padding():
    x = outlier_activations(200, 96, 3).to(DEV)
    codes, sf = nvfp4_quantize(x, global_scale(x))
    assert codes.shape == (200, 48) and sf.shape == (256, 8)
    offsets = nvfp4.sf_offsets(256, 8)
    flat = sf.cpu().numpy().reshape(-1)
    pad_rows = flat[offsets[200:].ravel()]
    pad_cols = flat[offsets[:, 6:].ravel()]
    assert (pad_rows == 0).all() and (pad_cols == 0).all()


@pytest.mark.parametrize("rows,cols", [(300, 4096), (129, 5376), (7, 64)])
def test_quantizer_agrees_with_oracle(rows, cols):
    x = outlier_activations(rows, cols, rows + cols).to(DEV)
    gsf = global_scale(x)
    codes, sf = nvfp4_quantize(x, gsf)
    want_codes, want_sf = nvfp4.quantize(fp8.bf16_value(bits_of(x)), float(gsf))
    got_codes = nvfp4.unpack(codes.cpu().numpy())
    exp_codes = nvfp4.unpack(want_codes)
    # the oracle uses exact reciprocals where the reference uses rcp.approx:
    # values within an ulp of a rounding boundary may land one code apart
    assert (got_codes != exp_codes).mean() < 5e-3
    diff = np.abs(nvfp4.e2m1_decode(got_codes) - nvfp4.e2m1_decode(exp_codes))
    assert diff.max() <= 2.0  # one e2m1 step at most (the widest step is 4 -> 6)
    assert (sf.cpu().numpy().reshape(-1) != want_sf).mean() < 5e-3


@pytest.mark.parametrize("case,tag", [(c[0], t) for c in QUANT_CASES for t in c[-1]])
def test_quantizer_bit_exact_against_flashinfer(flashinfer_golden, case, tag):
    name, rows, cols, seed, std, outliers, edges, _tags = next(c for c in QUANT_CASES if c[0] == case)
    x = case_input(rows, cols, seed, std, outliers, edges).to(DEV).to(DTYPES[tag])
    gsf = torch.from_numpy(flashinfer_golden[f"{name}.{tag}.gsf"]).to(DEV).reshape(())
    assert torch.equal(gsf, global_scale(x))  # the same global scale FlashInfer was given
    codes, sf = nvfp4_quantize(x, gsf)
    want_codes = flashinfer_golden[f"{name}.{tag}.codes"]
    want_sf = flashinfer_golden[f"{name}.{tag}.sf"]
    assert codes.shape == want_codes.shape
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(sf.reshape(-1).cpu().numpy(), want_sf)


SHAPES = [(1, 128, 64), (100, 256, 256), (257, 384, 320), (300, 512, 4096), (64, 1024, 1024)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_matches_exact_emulation(m, n, k):
    x = outlier_activations(m, k, m + k).to(DEV)
    gsf = global_scale(x)
    a_codes, a_sf = nvfp4_quantize(x, gsf)
    _w, w_packed, w_scales, w_alpha = weight_case(n, k, n + k)
    alpha = (w_alpha / gsf).to(torch.float32)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(5)) * 0.01).to(torch.bfloat16).to(DEV)
    y = nvfp4_gemm(a_codes, a_sf, w_packed, w_scales, alpha, bias)
    args = (a_codes.cpu().numpy(), a_sf.cpu().numpy().reshape(-1), w_packed.cpu().numpy(),
            w_scales.cpu().numpy().reshape(-1), float(alpha))
    want = nvfp4.w4a4_reference(*args, bias=fp8.bf16_value(bits_of(bias)))
    pre_bias = np.abs(nvfp4.w4a4_reference(*args)) * 2.0**-7
    bf16_close(fp8.bf16_value(bits_of(y)), want, max_mismatch=2e-3, atol=pre_bias)
    ref32 = nvfp4.dequant_matmul_f32(*args)
    got = y.float().cpu().numpy() - fp8.bf16_value(bits_of(bias))
    assert fp8.rel_l2(got, ref32) <= 2e-2


def test_gemm_qkv_planes_equal_plain_output():
    m, n, k = 200, 384, 512
    x = outlier_activations(m, k, 1).to(DEV)
    gsf = global_scale(x)
    a_codes, a_sf = nvfp4_quantize(x, gsf)
    _w, w_packed, w_scales, w_alpha = weight_case(n, k, 2)
    alpha = (w_alpha / gsf).to(torch.float32)
    y = nvfp4_gemm(a_codes, a_sf, w_packed, w_scales, alpha)
    planes = nvfp4_gemm(a_codes, a_sf, w_packed, w_scales, alpha, planes=3)
    for i in range(3):
        assert torch.equal(planes[i], y[:, i * 128:(i + 1) * 128])


def _dequant_gpu(codes: torch.Tensor, sf: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """fp32 dequantisation on the GPU (test-side restatement of the formats)."""
    table = torch.tensor(nvfp4.E2M1_VALUES, device=codes.device)
    lo, hi = codes & 0xF, codes >> 4
    nib = torch.stack([lo, hi], dim=-1).reshape(rows, cols).long()
    vals = table[nib & 7] * torch.where(nib >= 8, -1.0, 1.0)
    rows_pad, groups_pad = nvfp4.sf_padded_shape(rows, cols // 16)
    offsets = torch.from_numpy(nvfp4.sf_offsets(rows_pad, groups_pad)[:rows, : cols // 16]).to(codes.device)
    sf_bytes = sf.reshape(-1)[offsets].cpu().numpy()
    sf_vals = torch.from_numpy(fp8.e4m3_decode(sf_bytes)).to(codes.device)
    return vals * sf_vals.repeat_interleave(16, dim=1)


@pytest.mark.parametrize("n", [4096, 16384])
def test_c3_shapes_vs_fp32_dequant(n):
    m, k = 32760, 4096
    x = outlier_activations(m, k, 1003).to(DEV)
    gsf = global_scale(x)
    a_codes, a_sf = nvfp4_quantize(x, gsf)
    _w, w_packed, w_scales, w_alpha = weight_case(n, k, 2003 + n)
    alpha = (w_alpha / gsf).to(torch.float32)
    y = nvfp4_gemm(a_codes, a_sf, w_packed, w_scales, alpha)
    a32 = _dequant_gpu(a_codes, a_sf, m, k)
    w32 = _dequant_gpu(w_packed, w_scales, n, k)
    ref = (a32 @ w32.t()) * alpha
    rel = ((y.float() - ref).norm() / ref.norm()).item()
    assert rel <= 2e-2, rel


def test_gemm_on_flashinfer_codes_vs_mm_fp4(flashinfer_golden):
    g = flashinfer_golden
    n, k = LINEAR_CASE["n"], LINEAR_CASE["k"]
    a_codes = torch.from_numpy(g["linear.a_codes"]).to(DEV)
    a_sf = torch.from_numpy(g["linear.a_sf"]).to(DEV)
    w_codes = torch.from_numpy(g["linear.w_codes"]).to(DEV)
    w_sf = torch.from_numpy(g["linear.w_sf"]).to(DEV).view(n, k // 16)
    alpha = torch.from_numpy(g["linear.alpha"]).to(DEV).reshape(())
    y = nvfp4_gemm(a_codes, a_sf, w_codes, w_sf, alpha).float()
    ref = torch.from_numpy(g["linear.mm_fp4"].view(np.int16)).view(torch.bfloat16).to(DEV).float()
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel <= 1e-2, rel


def test_execution_linear_vs_reference_composition(flashinfer_golden):
    """NVFP4Execution.linear against nvfp4_quantize -> mm_fp4(alpha / input_scale) -> + bias (FlashInfer)."""
    g = flashinfer_golden
    n, k = LINEAR_CASE["n"], LINEAR_CASE["k"]
    x, _w, bias = (t.to(DEV) for t in linear_inputs())
    weight = NVFP4Weight(torch.from_numpy(g["linear.w_codes"]).to(DEV),
                         torch.from_numpy(g["linear.w_sf"]).to(DEV).view(n, k // 16),
                         torch.from_numpy(g["linear.alpha_w"]).to(DEV).reshape(()),
                         torch.from_numpy(g["linear.input_scale"]).to(DEV).reshape(()))
    y = NVFP4Execution().linear(x, weight, bias).float()
    ref = torch.from_numpy(g["linear.out"].view(np.int16)).view(torch.bfloat16).to(DEV).float()
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel <= 1e-2, rel
    # the activation codes it ran on are FlashInfer's own
    codes, sf = nvfp4_quantize(x, weight.input_scale)
    np.testing.assert_array_equal(codes.cpu().numpy(), g["linear.a_codes"])
    np.testing.assert_array_equal(sf.reshape(-1).cpu().numpy(), g["linear.a_sf"].reshape(-1))


def nvfp4_case(m, n, k, seed):
    x = outlier_activations(m, k, seed).to(DEV)
    gsf = global_scale(x)
    a_codes, a_sf = nvfp4_quantize(x, gsf)
    _w, w_packed, w_scales, w_alpha = weight_case(n, k, seed + 1)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(seed + 2)) * 0.01).to(torch.bfloat16).to(DEV)
    return a_codes, a_sf, w_packed, w_scales, w_alpha, gsf, bias


def test_alpha_divided_on_the_device_equals_the_divided_scalar():
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(300, 384, 512, 61)
    want = nvfp4_gemm(a_codes, a_sf, wp, ws, (w_alpha / gsf).to(torch.float32), bias)
    got = nvfp4_gemm(a_codes, a_sf, wp, ws, w_alpha.reshape(()), alpha_div=gsf, epilogue=Epilogue(bias=bias))
    assert torch.equal(got, want)


def test_qkv_planes_and_direct_merge_bit_exact_nvfp4():
    m, h, k = 200, 256, 512
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(m, 3 * h, k, 71)
    alpha = (w_alpha / gsf).to(torch.float32)
    base = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, bias)
    gen = torch.Generator().manual_seed(5)
    adapters = tuple(torch.randn(m, h, generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
    scalings = (0.0625, 0.5, -1.25)
    merged = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha,
                        epilogue=Epilogue(bias=bias, planes=3, adapters=adapters, scalings=scalings))
    want = ep.qkv_direct_merge(bits_of(base), np.stack([bits_of(a) for a in adapters]), scalings)
    for i in range(3):
        np.testing.assert_array_equal(bits_of(merged[i]), want[:, i * h:(i + 1) * h])


def test_gelu_epilogue_vs_oracle_nvfp4():
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(257, 512, 384 + 128, 81)
    alpha = (w_alpha / gsf).to(torch.float32)
    base = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, bias)
    fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=_lib.EPI_GELU_TANH, bias=bias))
    want = fp8.bf16_value(ep.gelu_tanh(bits_of(base)))
    got = fp8.bf16_value(bits_of(fused))
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() < 1e-2


@pytest.mark.parametrize("f", [128, 384])
def test_swiglu_epilogue_vs_oracle_nvfp4(f):
    m, k = 301, 256
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(m, 2 * f, k, 91 + f)
    alpha = (w_alpha / gsf).to(torch.float32)
    packed = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, bias)
    fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=_lib.EPI_SWIGLU, bias=bias))
    assert fused.shape == (m, f)
    want = fp8.bf16_value(ep.silu_mul(bits_of(packed)))
    got = fp8.bf16_value(bits_of(fused))
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() < 1e-2


@pytest.mark.parametrize("with_gate", [True, False])
def test_residual_epilogue_bit_exact_nvfp4(with_gate):
    batch, tokens, n, k = 2, 75, 256, 256
    m = batch * tokens
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(m, n, k, 101)
    alpha = (w_alpha / gsf).to(torch.float32)
    base = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, bias)
    gen = torch.Generator().manual_seed(23)
    residual = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(DEV)
    gate = torch.randn(tokens, n, generator=gen).to(torch.bfloat16).to(DEV) if with_gate else None
    fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha,
                       epilogue=Epilogue(kind=_lib.EPI_RESIDUAL, bias=bias, residual=residual, gate=gate,
                                         tokens=tokens))
    if with_gate:
        want = ep.gate_residual(bits_of(residual).reshape(batch, tokens, n), bits_of(gate),
                                bits_of(base).reshape(batch, tokens, n)).reshape(m, n)
    else:
        want = fp8.bf16_bits(fp8.bf16_value(bits_of(residual)) + fp8.bf16_value(bits_of(base)))
    np.testing.assert_array_equal(bits_of(fused), want)


@pytest.mark.parametrize("kind", ["gelu", "swiglu", "residual", "merge"])
def test_epilogues_over_many_tiles_per_pair(kind):
    """Every CTA pair runs several tiles, so both accumulators (even and odd
    tiles, which share 64 TMEM columns and hand them over differently) carry
    each epilogue: 16 row blocks x 10 tiles of 256 columns = 160 tiles."""
    m, n, k = 4096 - 37, 2560, 256
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(m, n, k, 131)
    alpha = (w_alpha / gsf).to(torch.float32)
    base = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, bias)
    gen = torch.Generator().manual_seed(29)
    if kind == "gelu":
        fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=_lib.EPI_GELU_TANH, bias=bias))
        want = fp8.bf16_value(ep.gelu_tanh(bits_of(base)))
        got = fp8.bf16_value(bits_of(fused))
        np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
        assert (got != want).mean() < 1e-2
    elif kind == "swiglu":
        fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=_lib.EPI_SWIGLU, bias=bias))
        assert fused.shape == (m, n // 2)
        want = fp8.bf16_value(ep.silu_mul(bits_of(base)))
        got = fp8.bf16_value(bits_of(fused))
        np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
        assert (got != want).mean() < 1e-2
    elif kind == "residual":
        residual = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(DEV)
        fused = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha,
                           epilogue=Epilogue(kind=_lib.EPI_RESIDUAL, bias=bias, residual=residual))
        want = fp8.bf16_bits(fp8.bf16_value(bits_of(residual)) + fp8.bf16_value(bits_of(base)))
        np.testing.assert_array_equal(bits_of(fused), want)
    else:
        h = 896  # three planes: N = 2688 = 21 x 128, 11 tiles of 256 columns per row block
        n3 = 3 * h
        a3, s3, wp3, ws3, w3, g3, b3 = nvfp4_case(m, n3, k, 137)
        alpha3 = (w3 / g3).to(torch.float32)
        base3 = nvfp4_gemm(a3, s3, wp3, ws3, alpha3, b3)
        adapters = tuple(torch.randn(m, h, generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
        scalings = (0.0625, 0.5, -1.25)
        merged = nvfp4_gemm(a3, s3, wp3, ws3, alpha3,
                            epilogue=Epilogue(bias=b3, planes=3, adapters=adapters, scalings=scalings))
        want = ep.qkv_direct_merge(bits_of(base3), np.stack([bits_of(a) for a in adapters]), scalings)
        for i in range(3):
            np.testing.assert_array_equal(bits_of(merged[i]), want[:, i * h:(i + 1) * h])


@pytest.mark.parametrize("kind", ["store", "gelu", "swiglu"])
@pytest.mark.parametrize("m", [130, 4096 - 37])
def test_quantised_output_equals_the_quantiser_of_the_bf16_output(kind, m):
    """vfb_nvfp4_gemm_quant: codes and 128x4 scales (padding rows included)
    equal nvfp4_quantize of the bf16 result the same epilogue stores."""
    n, k = 2560, 256
    a_codes, a_sf, wp, ws, w_alpha, gsf, bias = nvfp4_case(m, n, k, 151)
    alpha = (w_alpha / gsf).to(torch.float32)
    epi = {"store": _lib.EPI_STORE, "gelu": _lib.EPI_GELU_TANH, "swiglu": _lib.EPI_SWIGLU}[kind]
    y = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=epi, bias=bias))
    next_scale = global_scale(y)
    want_codes, want_sf = nvfp4_quantize(y, next_scale)
    codes, sf = nvfp4_gemm(a_codes, a_sf, wp, ws, alpha, epilogue=Epilogue(kind=epi, bias=bias),
                           quantize_output=next_scale)
    assert codes.shape == want_codes.shape and sf.shape == want_sf.shape
    assert torch.equal(codes, want_codes)
    assert torch.equal(sf, want_sf)


@pytest.mark.parametrize("activation", ["gelu_tanh", "swiglu"])
@pytest.mark.parametrize("with_residual", [False, True])
def test_execution_ffn_equals_the_two_linears(activation, with_residual):
    """NVFP4Execution.ffn: the intermediate never exists in bf16, and the
    result is the unfused linear(gelu_linear(...)) / swiglu chain bit for bit."""
    h, f, tokens = 512, 768, 150
    n_up = 2 * f if activation == "swiglu" else f
    _w, up_packed, up_scales, up_alpha = weight_case(n_up, h, 161)
    _w, down_packed, down_scales, down_alpha = weight_case(h, f, 162)
    x = outlier_activations(2 * tokens, h, 163).to(DEV).view(2, tokens, h)
    up = NVFP4Weight(up_packed, up_scales, up_alpha.reshape(()), global_scale(x))
    engine = NVFP4Execution()
    first = engine.swiglu_linear if activation == "swiglu" else engine.gelu_linear
    gen = torch.Generator().manual_seed(164)
    up_bias = (torch.randn(n_up, generator=gen) * 0.01).to(torch.bfloat16).to(DEV)
    down_bias = (torch.randn(h, generator=gen) * 0.01).to(torch.bfloat16).to(DEV)
    mid = first(x, up, up_bias)
    down = NVFP4Weight(down_packed, down_scales, down_alpha.reshape(()), global_scale(mid))
    if with_residual:
        residual = outlier_activations(2 * tokens, h, 165).to(DEV).view(2, tokens, h)
        gate = outlier_activations(tokens, h, 166).to(DEV)
        want = engine.gate_residual_linear(mid, down, residual, gate, down_bias)
        got = engine.ffn(x, up, down, activation=activation, up_bias=up_bias, down_bias=down_bias,
                         residual=residual, gate=gate)
    else:
        want = engine.linear(mid, down, down_bias)
        got = engine.ffn(x, up, down, activation=activation, up_bias=up_bias, down_bias=down_bias)
    assert got.shape == want.shape
    assert torch.equal(got, want)


def test_execution_fused_entry_points_equal_linear_then_step():
    n, k = 384, 512
    _w, packed, scales, w_alpha = weight_case(n, k, 111)
    x = outlier_activations(2 * 75, k, 112).to(DEV).view(2, 75, k)
    weight = NVFP4Weight(packed, scales, w_alpha.reshape(()), global_scale(x))
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(113)) * 0.01).to(torch.bfloat16).to(DEV)
    engine = NVFP4Execution()
    y = engine.linear(x, weight, bias)
    # GELU
    g = engine.gelu_linear(x, weight, bias)
    want = fp8.bf16_value(ep.gelu_tanh(bits_of(y.reshape(-1, n))))
    np.testing.assert_allclose(fp8.bf16_value(bits_of(g.reshape(-1, n))), want, rtol=2.0**-7, atol=1e-6)
    # gated residual
    residual = outlier_activations(150, n, 114).to(DEV).view(2, 75, n)
    gate = outlier_activations(75, n, 115).to(DEV)
    r = engine.gate_residual_linear(x, weight, residual, gate, bias)
    want = ep.gate_residual(bits_of(residual), bits_of(gate), bits_of(y))
    np.testing.assert_array_equal(bits_of(r), want)
    # merged QKV planes = chunk(3) of the plain output
    q, kk, v = engine.qkv_linear(x, weight, bias)
    for plane, ref in zip((q, kk, v), y.chunk(3, dim=-1)):
        assert torch.equal(plane, ref)
    assert engine.calls == 4 and engine.rows == 4 * 150


def test_execution_linear_end_to_end():
    n, k = 256, 512
    _w, packed, scales, w_alpha = weight_case(n, k, 31)
    x = outlier_activations(2 * 75, k, 32).to(DEV).view(2, 75, k)
    input_scale = global_scale(x)
    weight = NVFP4Weight(packed, scales, w_alpha.reshape(()), input_scale)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(33)).to(torch.bfloat16).to(DEV)
    engine = NVFP4Execution()
    y = engine.linear(x, weight, bias)
    assert y.shape == (2, 75, n) and engine.calls == 1 and engine.rows == 150
    a_codes, a_sf = nvfp4_quantize(x.view(-1, k), input_scale)
    plain = nvfp4_gemm(a_codes, a_sf, packed, scales, weight.alpha / weight.input_scale)
    assert torch.equal(y.view(-1, n), plain + bias)
    # fp32 inputs are cast to bf16 first, as the reference does
    y32 = engine.linear(x.float(), weight, bias)
    assert torch.equal(y32, y)
