"""Strict-BF16 elementwise drop-ins on the GPU vs the oracle and the reference's eager goldens.

Add/multiply steps must match the oracle bit for bit; steps with silu round
expf differently in the last fp32 bit, so they may differ by one bf16 ulp in a
small fraction of elements.  The fused GEMM epilogues must equal the
standalone ops applied to the same GEMM's plain output bit for bit (same
device arithmetic, one HBM pass fewer).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8
from tests.helpers import bits_of, fp8_weight, outlier_activations, to_bf16_tensor
from vflash_b200 import _lib
from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows
from vflash_b200.native import h3_fused_ops as fused

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand_bf16(shape, seed, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=gen) * scale).to(torch.bfloat16).to(DEV)


def close_1ulp(got_bits, want_bits, max_frac=1e-2):
    got, want = fp8.bf16_value(got_bits), fp8.bf16_value(want_bits)
    np.testing.assert_allclose(got, want, rtol=2.0**-7, atol=1e-6)
    assert (got != want).mean() <= max_frac


def test_goldens_from_reference_eager_compositions(golden):
    packed = to_bf16_tensor(golden["silu_packed"], DEV)
    close_1ulp(bits_of(fused.triton_strict_bf16_silu_mul(packed)), golden["silu_out"])
    residual = to_bf16_tensor(golden["gr_residual"], DEV)
    gate = to_bf16_tensor(golden["gr_gate"], DEV)
    projected = to_bf16_tensor(golden["gr_projected"], DEV)
    out = fused.triton_strict_bf16_gate_residual(residual, gate, projected)
    np.testing.assert_array_equal(bits_of(out), golden["gr_out"])
    base = to_bf16_tensor(golden["qkv_base"], DEV)
    adapters = tuple(to_bf16_tensor(a, DEV) for a in golden["qkv_adapters"])
    scalings = tuple(float(s) for s in golden["qkv_scalings"])
    merged = fused.triton_strict_bf16_qkv_direct_merge(base, adapters, scalings=scalings)
    assert merged is base
    np.testing.assert_array_equal(bits_of(base), golden["qkv_out"])


@pytest.mark.parametrize("shape", [(2, 75, 512), (1, 33, 7168 * 2), (3, 5, 48)])
def test_silu_mul(shape):
    packed = rand_bf16(shape, 1, 3.0)
    close_1ulp(bits_of(fused.triton_strict_bf16_silu_mul(packed)), ep.silu_mul(bits_of(packed)))


@pytest.mark.parametrize("reuse", [False, True])
def test_ffn_adapter_silu(reuse):
    base = rand_bf16((2, 41, 2 * 384), 2, 2.0)
    adapter = rand_bf16((2, 41, 2 * 384), 3, 2.0)
    want = ep.ffn_adapter_silu(bits_of(base), bits_of(adapter), 0.0625)
    gate_before = bits_of(base[..., 384:]).copy()
    out = fused.triton_strict_bf16_ffn_adapter_silu(base, adapter, scaling=0.0625, block_size=1024,
                                                    reuse_base=reuse)
    close_1ulp(bits_of(out), want)
    if reuse:
        assert out.data_ptr() == base.data_ptr() and out.stride(-2) == 2 * 384
        np.testing.assert_array_equal(bits_of(base[..., 384:]), gate_before)


def test_gate_residual_with_strided_gate():
    residual = rand_bf16((3, 50, 256), 4)
    projected = rand_bf16((3, 50, 256), 5)
    gate_store = rand_bf16((50, 512), 6)
    gate = gate_store[:, 128:384]  # token stride 512, unit hidden stride
    out = fused.triton_strict_bf16_gate_residual(residual, gate, projected)
    want = ep.gate_residual(bits_of(residual), bits_of(gate), bits_of(projected))
    np.testing.assert_array_equal(bits_of(out), want)


def test_adapter_merges_and_adapter_gate_residual():
    base = rand_bf16((2, 30, 3 * 128), 7)
    adapter = rand_bf16((2, 30, 3 * 128), 8)
    out = fused.triton_strict_bf16_adapter_merge(base, adapter, scaling=0.3)
    np.testing.assert_array_equal(bits_of(out), ep.adapter_merge(bits_of(base), bits_of(adapter), (0.3,)))
    scalings = (0.0625, -0.5, 2.0)
    out = fused.triton_strict_bf16_qkv_adapter_merge(base, adapter, scalings=scalings)
    np.testing.assert_array_equal(bits_of(out), ep.adapter_merge(bits_of(base), bits_of(adapter), scalings))
    residual = rand_bf16((2, 30, 384), 9)
    gate = rand_bf16((30, 384), 10)
    out = fused.triton_strict_bf16_adapter_gate_residual(base, adapter, residual, gate, scaling=0.25)
    want = ep.adapter_gate_residual(bits_of(base), bits_of(adapter), bits_of(residual), bits_of(gate), 0.25)
    np.testing.assert_array_equal(bits_of(out), want)


def _gemm_case(m, n, k, seed):
    x = outlier_activations(m, k, seed).to(DEV)
    w, ws = fp8_weight(n, k, seed + 1)
    b = (torch.randn(n, generator=torch.Generator().manual_seed(seed + 2)) * 0.01).to(torch.bfloat16)
    codes, scales = quantize_fp8_rows(x)
    return codes, scales, w.to(DEV), ws.to(DEV), b.to(DEV)


def test_fused_epilogues_equal_standalone_ops_bit_for_bit():
    m, k, f = 300, 512, 256
    codes, scales, w, ws, b = _gemm_case(m, 2 * f, k, 31)
    packed = fp8_gemm(codes, scales, m, w, ws, Epilogue(bias=b))
    fused_swiglu = fp8_gemm(codes, scales, m, w, ws, Epilogue(kind=_lib.EPI_SWIGLU, bias=b))
    standalone = fused.triton_strict_bf16_silu_mul(packed.view(1, m, 2 * f))
    assert torch.equal(fused_swiglu, standalone.view(m, f))

    tokens = 100
    residual = rand_bf16((3, tokens, 2 * f), 12)
    gate = rand_bf16((tokens, 2 * f), 13)
    fused_res = fp8_gemm(codes, scales, m, w, ws,
                         Epilogue(kind=_lib.EPI_RESIDUAL, bias=b, residual=residual.view(m, 2 * f),
                                  gate=gate, tokens=tokens))
    standalone = fused.triton_strict_bf16_gate_residual(residual, gate, packed.view(3, tokens, 2 * f))
    assert torch.equal(fused_res, standalone.view(m, 2 * f))

    h = 128
    codes, scales, w, ws, b = _gemm_case(m, 3 * h, k, 41)
    base = fp8_gemm(codes, scales, m, w, ws, Epilogue(bias=b))
    adapters = tuple(rand_bf16((1, m, h), 50 + i) for i in range(3))
    scalings = (0.0625, 0.0625, 0.0625)
    planes = fp8_gemm(codes, scales, m, w, ws,
                      Epilogue(bias=b, planes=3, adapters=tuple(a.view(m, h) for a in adapters),
                               scalings=scalings))
    merged = fused.triton_strict_bf16_qkv_direct_merge(base.view(1, m, 3 * h), adapters, scalings=scalings)
    for i in range(3):
        assert torch.equal(planes[i], merged.view(m, 3 * h)[:, i * h:(i + 1) * h])
