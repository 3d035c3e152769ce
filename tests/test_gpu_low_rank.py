"""Low-rank adapter products on the tcgen05 pipeline (vfb_bf16_gemm) and the QKV path that uses them.

Bars:
* ``bf16_gemm`` vs the oracle's bf16(exact A @ W^T): at most 2 % of the
  outputs differ and each by one bf16 step (fp32 accumulation in another
  order), and likewise vs torch's cuBLAS ``functional.linear``;
* ``qkv_linear(residuals=...)`` is bit-identical to the same projection fed
  the adapters that ``qkv_low_rank`` returns, whose three branches equal
  ``low_rank`` branch by branch (one concatenated down GEMM vs one per
  branch: the same dot products).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8
from tests.helpers import bits_of, fp8_weight, outlier_activations
from vflash_b200.kernels import KernelInputError, bf16_gemm
from vflash_b200.native.h3_fp8_linear import RowFP8Execution

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(shape, seed, std=1.0):
    return (torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16)


def assert_close_to_exact(got_bits, a, w, want_bits=None, frac=2e-2):
    """``got`` vs bf16(exact a @ w^T): at most ``frac`` of the outputs differ, each
    by at most one bf16 step or 2^-20 of the sum of |products| (fp32 accumulation
    in another order; near-zero sums after cancellation carry that absolute error).
    """
    a64 = fp8.bf16_value(bits_of(a)).astype(np.float64)
    w64 = fp8.bf16_value(bits_of(w)).astype(np.float64)
    want_bits = ep.bf16_linear(bits_of(a), bits_of(w)) if want_bits is None else want_bits
    got = fp8.bf16_value(got_bits).astype(np.float64)
    want = fp8.bf16_value(want_bits).astype(np.float64)
    differ = got_bits != want_bits
    assert differ.mean() <= frac, f"{differ.mean():.3%} differ"
    step = np.abs(want) * 2.0 ** -7  # one bf16 step (8-bit significand) at |want|, at most
    bound = np.maximum(step, 2.0 ** -20 * (np.abs(a64) @ np.abs(w64).T))
    excess = np.abs(got - want) - bound
    assert excess.max(initial=0) <= 0, f"worst excess {excess.max():.3e}"


@pytest.mark.parametrize("m,n,k", [(150, 96, 4096), (300, 4096, 32), (129, 512, 16), (7, 40, 64),
                                   (1000, 128, 5376), (257, 264, 256)])
def test_bf16_gemm_matches_exact_rounding(m, n, k):
    a, w = bf16((m, k), m + k), bf16((n, k), n + k, std=0.05)
    got = bf16_gemm(a.to(DEV), w.to(DEV))
    assert got.shape == (m, n)
    assert_close_to_exact(bits_of(got), a, w)
    # cuBLAS (the reference's functional.linear) sits within the same bound
    cublas = torch.nn.functional.linear(a.to(DEV), w.to(DEV))
    assert_close_to_exact(bits_of(cublas), a, w)


def test_bf16_gemm_strided_operands_and_output():
    a_wide, w = bf16((200, 320), 1), bf16((64, 256), 2, std=0.05)
    a = a_wide[:, 64:]  # row stride 320, starts 128 bytes in
    out_wide = torch.zeros(200, 192, dtype=torch.bfloat16, device=DEV)
    view = out_wide[:, 64:128]
    got = bf16_gemm(a_wide.to(DEV)[:, 64:], w.to(DEV), out=view)
    assert got.data_ptr() == view.data_ptr()
    assert_close_to_exact(bits_of(view), a.contiguous(), w)
    assert not out_wide[:, :64].any() and not out_wide[:, 128:].any()
    with pytest.raises(KernelInputError):
        bf16_gemm(a.to(DEV), bf16((64, 250), 3).to(DEV))


@dataclass(frozen=True)
class Residual:
    down: torch.Tensor
    up: torch.Tensor
    scaling: float


def test_low_rank_and_qkv_residuals():
    batch, tokens, hidden, width, rank = 2, 150, 512, 256, 32
    x = outlier_activations(batch * tokens, hidden, 80).reshape(batch, tokens, hidden).to(DEV)
    codes, scale = fp8_weight(3 * width, hidden, 81)
    codes, scale = codes.to(DEV), scale.to(DEV)
    residuals = tuple(Residual(bf16((rank, hidden), 90 + i, 0.05).to(DEV), bf16((width, rank), 95 + i, 0.05).to(DEV),
                               s) for i, s in enumerate((0.5, -1.0, 0.125)))
    ex = RowFP8Execution("w8a8")
    single = [ex.low_rank(x, r.down, r.up) for r in residuals]
    for r, got in zip(residuals, single):
        xm = x.reshape(-1, hidden)
        low = bf16_gemm(xm, r.down)
        assert_close_to_exact(bits_of(low), xm.cpu(), r.down.cpu())
        # the up product of the kernel's own low-rank rows, then the whole chain vs the oracle
        assert_close_to_exact(bits_of(got.reshape(-1, width)), low.cpu(), r.up.cpu())
        want = ep.low_rank(bits_of(xm), bits_of(r.down), bits_of(r.up))
        g, w_ = fp8.bf16_value(bits_of(got.reshape(-1, width))), fp8.bf16_value(want)
        assert np.linalg.norm(g - w_) <= 1e-2 * np.linalg.norm(w_)
    fused = ex.qkv_low_rank(x, residuals)
    for a, b in zip(fused, single):
        assert torch.equal(a.reshape(b.shape), b)
    planes = ex.qkv_linear(x, codes, scale, residuals=residuals)
    merged = ex.qkv_linear(x, codes, scale, adapters=tuple(a.reshape(batch, tokens, width) for a in fused),
                           scalings=tuple(r.scaling for r in residuals))
    for p, q in zip(planes, merged):
        assert torch.equal(p, q)
    # the reference composition: value + bf16(unscaled * scaling), eager bf16
    base = ex.qkv_linear(x, codes, scale)
    for p, b, a, r in zip(planes, base, single, residuals):
        assert torch.equal(p, b + a * r.scaling)
