"""Rotary embedding (bit-exact) and QK-norm + rotary fused into the QKV GEMM epilogue.

The fused epilogue takes rstd from an fp32 sum of the head's squares in its
own order; the oracle sums in float64.  Where the two rstd differ by an fp32
ulp a bf16 rounding of the normalised value can flip, so the Q and K planes
are compared with a tolerance (at most 1 % of the values differ, rel-L2 <=
1e-3, no difference above 2^-5 of the plane's largest magnitude).  The V plane and
everything upstream of the norm are bit-identical to the unfused path.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8
from tests.helpers import bits_of, fp8_weight, outlier_activations
from vflash_b200.native.h3_fp8_linear import QKNormRope, RowFP8Execution
from vflash_b200.native.h3_fused_ops import triton_strict_bf16_rotary

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rope_tables(tokens, rd, seed):
    pos = torch.arange(tokens, dtype=torch.float32)[:, None]
    freq = 1.0 / (10000 ** (torch.arange(rd // 2, dtype=torch.float32) / (rd // 2)))
    ang = torch.cat([pos * freq, pos * freq], dim=1) + seed * 1e-3
    return ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)


@pytest.mark.parametrize("rd", [128, 64, 32])
def test_rotary_bit_exact(rd):
    x = torch.randn(2, 37, 4, 128, generator=torch.Generator().manual_seed(rd)).to(torch.bfloat16)
    cos, sin = rope_tables(37, rd, 1)
    got = triton_strict_bf16_rotary(x.to(DEV), cos.to(DEV), sin.to(DEV))
    np.testing.assert_array_equal(bits_of(got), ep.rotary(bits_of(x), bits_of(cos), bits_of(sin)))


def test_rotary_strided_tables():
    x = torch.randn(1, 9, 2, 128, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    cos, sin = rope_tables(9, 128, 2)
    wide_c = torch.zeros(9, 160, dtype=torch.bfloat16)
    wide_s = torch.zeros(9, 160, dtype=torch.bfloat16)
    wide_c[:, :128], wide_s[:, :128] = cos, sin
    got = triton_strict_bf16_rotary(x.to(DEV), wide_c.to(DEV)[:, :128], wide_s.to(DEV)[:, :128])
    np.testing.assert_array_equal(bits_of(got), ep.rotary(bits_of(x), bits_of(cos), bits_of(sin)))


def oracle_qk(planes_bits, batch, tokens, heads, q_norm, k_norm, cos, sin, eps):
    out = []
    for i, w in ((0, q_norm), (1, k_norm)):
        h = planes_bits[i].reshape(batch, tokens, heads, 128)
        n = ep.rms_norm(h, None if w is None else bits_of(w), eps)
        out.append(ep.rotary(n, bits_of(cos), bits_of(sin)))
    return out


def assert_close_planes(got, want):
    g = fp8.bf16_value(bits_of(got)).astype(np.float64).reshape(-1)
    w = fp8.bf16_value(want).astype(np.float64).reshape(-1)
    diff = np.abs(g - w)
    assert (diff > 0).mean() <= 1e-2, f"{(diff > 0).mean():.2e} differ"
    assert np.linalg.norm(g - w) <= 1e-3 * np.linalg.norm(w)
    assert diff.max() <= 2.0 ** -5 * np.abs(w).max()


@pytest.mark.parametrize("batch,tokens,heads,k", [(2, 150, 2, 512), (1, 4096, 4, 1024), (3, 17, 1, 256)])
@pytest.mark.parametrize("with_weights", [True, False])
def test_fused_qk_norm_rope_matches_oracle_and_unfused(batch, tokens, heads, k, with_weights):
    rows, width = batch * tokens, heads * 128
    x = outlier_activations(rows, k, 30 + heads).reshape(batch, tokens, k).to(DEV)
    codes, scale = fp8_weight(3 * width, k, 31)
    codes, scale = codes.to(DEV), scale.to(DEV)
    bias = (torch.randn(3 * width, generator=torch.Generator().manual_seed(32)) * 0.01).to(torch.bfloat16).to(DEV)
    gen = torch.Generator().manual_seed(33)
    qn = (1 + torch.randn(128, generator=gen) * 0.1).to(torch.bfloat16) if with_weights else None
    kn = (1 + torch.randn(128, generator=gen) * 0.1).to(torch.bfloat16) if with_weights else None
    cos, sin = rope_tables(tokens, 128, 5)
    execution = RowFP8Execution("w8a8")
    rope = QKNormRope(None if qn is None else qn.to(DEV), None if kn is None else kn.to(DEV),
                      cos.to(DEV), sin.to(DEV), 1e-5)
    q, kk, v = execution.qkv_linear(x, codes, scale, bias, qk_norm_rope=rope)
    q0, k0, v0 = execution.qkv_linear(x, codes, scale, bias)
    assert torch.equal(v, v0)
    want_q, want_k = oracle_qk([bits_of(q0), bits_of(k0)], batch, tokens, heads, qn, kn, cos, sin, 1e-5)
    assert_close_planes(q, want_q)
    assert_close_planes(kk, want_k)
    # the reference's own GPU chain: torch rms_norm per head, then the strict rotary
    qh = q0.reshape(batch, tokens, heads, 128)
    chain = triton_strict_bf16_rotary(
        torch.nn.functional.rms_norm(qh, (128,), None if qn is None else qn.to(DEV), 1e-5), cos.to(DEV), sin.to(DEV))
    assert_close_planes(q, bits_of(chain))


def test_fused_rejects_heads_that_are_not_128_wide():
    x = torch.zeros(1, 8, 256, dtype=torch.bfloat16, device=DEV)
    codes, scale = fp8_weight(3 * 96, 256, 1)
    cos, sin = rope_tables(8, 128, 0)
    with pytest.raises(ValueError, match="128-wide heads"):
        RowFP8Execution("w8a8").qkv_linear(x, codes.to(DEV), scale.to(DEV),
                                           qk_norm_rope=QKNormRope(None, None, cos.to(DEV), sin.to(DEV)))
    codes, scale = fp8_weight(3 * 128, 256, 1)
    with pytest.raises(ValueError, match="per token"):
        RowFP8Execution("w8a8").qkv_linear(x, codes.to(DEV), scale.to(DEV),
                                           qk_norm_rope=QKNormRope(None, None, cos[:3].to(DEV), sin[:3].to(DEV)))
