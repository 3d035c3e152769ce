"""NVFP4 quantiser and block-scaled GEMM on the GPU.

Bars:
* quantiser codes and 128x4 scales bit-exact against FlashInfer's own
  nvfp4_quantize (the reference's NVFP4 backend), when its prebuilt module is
  present (tests/golden/build_flashinfer_reference.py); against the CPU oracle
  (exact reciprocals instead of rcp.approx) at least 99.9 % identical, every
  difference one code step;
* GEMM vs the exact fp64 emulation of mm_fp4 on the same codes: identical
  bf16 except rare one-ulp flips; vs the fp32 dequantise-then-matmul
  rel-L2 <= 2e-2; vs FlashInfer mm_fp4 (when built) rel-L2 <= 1e-2.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8, nvfp4
from tests.helpers import bf16_close, bits_of, outlier_activations
from vflash_b200.kernels import nvfp4_gemm, nvfp4_quantize
from vflash_b200.native.h3_nvfp4_linear import NVFP4Execution, NVFP4Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"
FI_CACHE = Path(__file__).resolve().parent / ".flashinfer_ref"


def flashinfer_module(kind: str):
    built = list(FI_CACHE.glob(f"**/cached_ops/{kind}*/*.so"))
    if not built:
        pytest.skip(f"FlashInfer {kind} module not prebuilt (tests/golden/build_flashinfer_reference.py)")
    import flashinfer

    return flashinfer


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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quantizer_bit_exact_against_flashinfer(dtype):
    fi = flashinfer_module("fp4_quantization")
    x = outlier_activations(333, 4096, 11).to(DEV).to(dtype)
    # edge blocks: all-zero, tiny (subnormal in bf16) and exact ties
    x[0, :16] = 0
    x[1, :16] = torch.tensor(2.0**-130, dtype=torch.float32).to(dtype)
    x[2, :32] = torch.tensor([6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0] * 4, dtype=dtype)
    gsf = global_scale(x)
    codes, sf = nvfp4_quantize(x, gsf)
    ref_codes, ref_sf = fi.nvfp4_quantize(x, gsf, sfLayout=fi.SfLayout.layout_128x4, do_shuffle=False)
    ref_codes = ref_codes.contiguous().view(torch.uint8)
    assert torch.equal(codes, ref_codes.view(codes.shape))
    assert torch.equal(sf.reshape(-1), ref_sf.contiguous().view(torch.uint8).reshape(-1))


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


def test_gemm_vs_flashinfer_mm_fp4():
    fi = flashinfer_module("fp4_gemm")
    m, n, k = 1000, 1024, 2048
    x = outlier_activations(m, k, 21).to(DEV)
    gsf = global_scale(x)
    a_codes, a_sf = nvfp4_quantize(x, gsf)
    _w, w_packed, w_scales, w_alpha = weight_case(n, k, 22)
    alpha = (w_alpha / gsf).to(torch.float32)
    y = nvfp4_gemm(a_codes, a_sf, w_packed, w_scales, alpha)
    ref = fi.mm_fp4(a_codes, w_packed.T, a_sf, w_scales.T, alpha, torch.bfloat16, None,
                    block_size=16, use_8x4_sf_layout=False, backend="cutlass", use_nvfp4=True)
    rel = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel <= 1e-2, rel


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
