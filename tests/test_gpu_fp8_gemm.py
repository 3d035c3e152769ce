"""tcgen05 FP8 GEMM and its fused epilogues on the GPU vs the oracle.

Bars (stated per test):
* vs the exact fp64 emulation of ``torch._scaled_mm`` rowwise + bias
  (oracle.fp8.w8a8_reference): identical bf16 except rare one-ulp flips from
  fp32 accumulation order;
* vs ``torch._scaled_mm`` itself (the reference's W8A8 GEMM, cuBLASLt on this
  box): rel-L2 <= 1e-2;
* vs the fp32 dequantise-then-matmul: rel-L2 <= 2e-2;
* fused epilogues vs the oracle's strict-BF16 step applied to this GEMM's own
  plain output: bit-exact for add/multiply epilogues, one bf16 ulp (or 1e-6
  absolute) for the transcendental ones (expf / tanhf differ by an fp32 ulp).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8
from tests.helpers import bf16_close, bits_of, codes_of, fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_case(m, n, k, seed, bias=True):
    x = outlier_activations(m, k, 1000 + seed).to(DEV)
    w, ws = fp8_weight(n, k, 2000 + seed)
    b = (torch.randn(n, generator=torch.Generator().manual_seed(3000 + seed)) * 0.01).to(torch.bfloat16)
    return x, w.to(DEV), ws.to(DEV), (b.to(DEV) if bias else None)


def plain(x, w, ws, bias=None):
    codes, scales = quantize_fp8_rows(x)
    return codes, scales, fp8_gemm(codes, scales, x.shape[0], w, ws, Epilogue(bias=bias))


SHAPES = [
    (1, 32, 16), (17, 256, 64), (128, 256, 128), (129, 288, 208), (300, 544, 1024),
    (127, 512, 4096), (256, 4096, 256), (1000, 768, 2048), (333, 12288 // 8, 4096),
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_matches_exact_emulation(m, n, k):
    x, w, ws, b = make_case(m, n, k, seed=m + n + k)
    codes, scales, y = plain(x, w, ws, b)
    args = (codes_of(codes)[:m], scales.cpu().numpy()[:m], codes_of(w), ws.cpu().numpy())
    want = fp8.w8a8_reference(*args, bits_of(b))
    # a one-ulp flip of bf16(acc) before the bias add can survive a cancellation
    pre_bias_ulp = np.abs(fp8.w8a8_reference(*args)) * 2.0**-7
    bf16_close(fp8.bf16_value(bits_of(y)), want, max_mismatch=2e-3, atol=pre_bias_ulp)


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (32760, 1536, 4096)])
def test_gemm_vs_scaled_mm_and_fp32_dequant(m, n, k):
    x, w, ws, b = make_case(m, n, k, seed=7)
    codes, scales, y = plain(x, w, ws, None)
    ref = torch._scaled_mm(codes, w.t(), scale_a=scales, scale_b=ws.t(), out_dtype=torch.bfloat16)
    if isinstance(ref, tuple):
        ref = ref[0]
    ref = ref[:m].float()
    rel = ((y.float() - ref).norm() / ref.norm()).item()
    assert rel <= 1e-2, rel
    deq = (codes[:m].float() * scales[:m]) @ (w.float() * ws).t()
    rel32 = ((y.float() - deq).norm() / deq.norm()).item()
    assert rel32 <= 2e-2, rel32


def test_tail_rows_are_not_written():
    m, n, k = 130, 256, 256
    x, w, ws, _ = make_case(m, n, k, seed=3, bias=False)
    codes, scales = quantize_fp8_rows(x)
    out = torch.full((m + 10, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    fp8_gemm(codes, scales, m, w, ws, Epilogue(), out=out[:m])
    assert torch.isnan(out[m:].float()).all()
    assert not torch.isnan(out[:m].float()).any()


def test_qkv_planes_and_direct_merge_bit_exact():
    m, h, k = 200, 256, 512
    x, w, ws, b = make_case(m, 3 * h, k, seed=11)
    codes, scales, base = plain(x, w, ws, b)
    planes = fp8_gemm(codes, scales, m, w, ws, Epilogue(bias=b, planes=3))
    for i in range(3):
        assert torch.equal(planes[i], base[:, i * h:(i + 1) * h])
    gen = torch.Generator().manual_seed(5)
    adapters = tuple(torch.randn(m, h, generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
    scalings = (0.0625, 0.5, -1.25)
    merged = fp8_gemm(codes, scales, m, w, ws,
                      Epilogue(bias=b, planes=3, adapters=adapters, scalings=scalings))
    want = ep.qkv_direct_merge(bits_of(base), np.stack([bits_of(a) for a in adapters]), scalings)
    for i in range(3):
        np.testing.assert_array_equal(bits_of(merged[i]), want[:, i * h:(i + 1) * h])


def test_gelu_epilogue_vs_oracle():
    m, n, k = 257, 512, 384
    x, w, ws, b = make_case(m, n, k, seed=13)
    codes, scales, base = plain(x, w, ws, b)
    fused = fp8_gemm(codes, scales, m, w, ws, Epilogue(kind=_lib.EPI_GELU_TANH, bias=b))
    want = fp8.bf16_value(ep.gelu_tanh(bits_of(base)))
    got = fp8.bf16_value(bits_of(fused))
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() < 1e-2


@pytest.mark.parametrize("f", [128, 160, 512])
def test_swiglu_epilogue_vs_oracle(f):
    m, k = 301, 256
    x, w, ws, b = make_case(m, 2 * f, k, seed=17 + f)
    codes, scales, packed = plain(x, w, ws, b)
    fused = fp8_gemm(codes, scales, m, w, ws, Epilogue(kind=_lib.EPI_SWIGLU, bias=b))
    assert fused.shape == (m, f)
    want = fp8.bf16_value(ep.silu_mul(bits_of(packed)))
    got = fp8.bf16_value(bits_of(fused))
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() < 1e-2


@pytest.mark.parametrize("with_gate", [True, False])
def test_residual_epilogue_bit_exact(with_gate):
    batch, tokens, n, k = 2, 75, 256, 256
    m = batch * tokens
    x, w, ws, b = make_case(m, n, k, seed=19)
    codes, scales, base = plain(x, w, ws, b)
    gen = torch.Generator().manual_seed(23)
    residual = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(DEV)
    gate = torch.randn(tokens, n, generator=gen).to(torch.bfloat16).to(DEV) if with_gate else None
    fused = fp8_gemm(codes, scales, m, w, ws,
                     Epilogue(kind=_lib.EPI_RESIDUAL, bias=b, residual=residual, gate=gate,
                              tokens=tokens))
    if with_gate:
        want = ep.gate_residual(bits_of(residual).reshape(batch, tokens, n), bits_of(gate),
                                bits_of(base).reshape(batch, tokens, n)).reshape(m, n)
    else:
        want = fp8.bf16_bits(fp8.bf16_value(bits_of(residual)) + fp8.bf16_value(bits_of(base)))
    np.testing.assert_array_equal(bits_of(fused), want)


def test_device_status_stays_clean():
    m, n, k = 640, 1024, 1024
    x, w, ws, b = make_case(m, n, k, seed=29)
    plain(x, w, ws, b)
    assert _lib.device_status(clear=True) == _lib.VFB_OK


@pytest.mark.parametrize("k", [16, 32, 4096])
def test_known_answer_ones_times_ones_is_k(k):
    # reference tests/test_fp8_loaders.py:31-47 (K = 16 there), on the W8A8 path
    from vflash_b200.native.h3_fp8_linear import RowFP8Execution

    codes = torch.ones(32, k).to(torch.float8_e4m3fn).to(DEV)  # the GEMM needs N % 32 == 0
    scales = torch.ones(32, 1, device=DEV)
    x = torch.ones(2, k, dtype=torch.bfloat16, device=DEV)
    out = RowFP8Execution("w8a8").linear(x, codes, scales)
    assert torch.equal(out, torch.full((2, 32), float(k), dtype=torch.bfloat16, device=DEV))
