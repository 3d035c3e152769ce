"""AdaLN modulate (bit-exact) and the fused RMSNorm + modulate + FP8 quantiser on the GPU.

The fused kernel's rstd is an fp32 sum of squares in the kernel's own order
(the oracle sums in float64), so a bf16 rounding of the normalised value can
flip where the two rstd differ by an fp32 ulp; codes may then differ by one
e4m3 step.  Tolerance: at most 2e-3 of the codes differ, each by one step,
and row scales agree within one bf16 ulp of the row maximum.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from oracle import fp8
from tests.helpers import bits_of, codes_of, outlier_activations
from vflash_b200.kernels import quantize_fp8_norm_modulate, quantize_fp8_rows
from vflash_b200.native.h3_fp8_linear import NormModulate, RowFP8Execution
from vflash_b200.native.h3_fused_ops import H3FusedOpsError, triton_strict_bf16_modulate

pytestmark = pytest.mark.gpu
DEV = "cuda"


def modifiers(tokens, hidden, seed, std=0.3):
    gen = torch.Generator().manual_seed(seed)
    scale = (torch.randn(tokens, hidden, generator=gen) * std).to(torch.bfloat16)
    shift = (torch.randn(tokens, hidden, generator=gen) * std).to(torch.bfloat16)
    return scale, shift


@pytest.mark.parametrize("batch,tokens,hidden", [(1, 4096, 4096), (2, 37, 5376), (3, 5, 8)])
def test_modulate_bit_exact(batch, tokens, hidden):
    x = outlier_activations(batch * tokens, hidden, 3).reshape(batch, tokens, hidden)
    scale, shift = modifiers(tokens, hidden, 4)
    got = triton_strict_bf16_modulate(x.to(DEV), scale.to(DEV), shift.to(DEV))
    want = ep.modulate(bits_of(x), bits_of(scale), bits_of(shift))
    np.testing.assert_array_equal(bits_of(got), want)


def test_modulate_broadcast_token_row():
    x = outlier_activations(64, 256, 5).reshape(1, 64, 256)
    scale, shift = modifiers(1, 256, 6)
    got = triton_strict_bf16_modulate(x.to(DEV), scale.to(DEV).expand(64, 256), shift.to(DEV).expand(64, 256))
    want = ep.modulate(bits_of(x), np.broadcast_to(bits_of(scale), (64, 256)),
                       np.broadcast_to(bits_of(shift), (64, 256)))
    np.testing.assert_array_equal(bits_of(got), want)


def test_modulate_rejects_mismatched_modifier():
    x = torch.zeros(1, 4, 16, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(H3FusedOpsError, match="shape differs"):
        triton_strict_bf16_modulate(x, torch.zeros(3, 16, dtype=torch.bfloat16, device=DEV),
                                    torch.zeros(4, 16, dtype=torch.bfloat16, device=DEV))


def oracle_codes(x, w, scale, shift, eps, tokens):
    rows = x.shape[0]
    reps = rows // tokens
    normed = ep.rms_norm(bits_of(x), None if w is None else bits_of(w), eps)
    mod = ep.modulate(normed.reshape(reps, tokens, -1), bits_of(scale), bits_of(shift)).reshape(rows, -1)
    return fp8.quantize_activation(mod)


def assert_codes_close(got_codes, got_scales, want_codes, want_scales):
    g = codes_of(got_codes)
    assert g.shape == want_codes.shape
    diff = g != want_codes
    assert diff.mean() <= 2e-3, f"{diff.mean():.2e} of codes differ"
    if diff.any():
        gv = fp8.e4m3_decode(g[diff]).astype(np.float64)
        wv = fp8.e4m3_decode(want_codes[diff]).astype(np.float64)
        # one e4m3 step: at most 1/8 of the larger magnitude (or one subnormal step)
        assert (np.abs(gv - wv) <= np.maximum(np.abs(wv), np.abs(gv)) / 8 + 2.0 ** -9).all()
    gs = got_scales.cpu().numpy().reshape(-1)
    ws = want_scales.reshape(-1)
    np.testing.assert_allclose(gs, ws, rtol=2.0 ** -7, atol=0)


@pytest.mark.parametrize("rows,hidden,tokens", [(4096, 4096, 4096), (300, 5376, 100), (17, 8, 17),
                                                 (64, 16384, 1)])
def test_fused_norm_modulate_quant_vs_oracle(rows, hidden, tokens):
    x = (outlier_activations(rows, hidden, 11).float() * 2.5).to(torch.bfloat16)
    gen = torch.Generator().manual_seed(12)
    w = (1 + torch.randn(hidden, generator=gen) * 0.1).to(torch.bfloat16)
    scale, shift = modifiers(tokens, hidden, 13)
    codes, scales = quantize_fp8_norm_modulate(x.to(DEV), w.to(DEV), 1e-6, scale.to(DEV), shift.to(DEV))
    want_codes, want_scales = oracle_codes(x, w, scale, shift, 1e-6, tokens)
    assert_codes_close(codes, scales, want_codes, want_scales)


def test_fused_edge_rows_zero_nan_and_no_weight():
    x = outlier_activations(48, 256, 14)
    x[3] = 0.0                       # rstd = 1/sqrt(eps): the row becomes the shift
    x[7, 9] = float("nan")           # a NaN row stays NaN with unit scale
    scale, shift = modifiers(48, 256, 15)
    codes, scales = quantize_fp8_norm_modulate(x.to(DEV), None, 1e-5, scale.to(DEV), shift.to(DEV))
    want_codes, want_scales = oracle_codes(x, None, scale, shift, 1e-5, 48)
    g = codes_of(codes)
    np.testing.assert_array_equal(g[3], want_codes[3])
    assert ((g[7] & 0x7F) == 0x7F).all() and scales[7].item() == 1.0  # NaN codes, any sign
    keep = np.ones(g.shape[0], bool)
    keep[7] = False
    kt = torch.from_numpy(keep).to(codes.device)
    assert_codes_close(codes[kt], scales[kt], want_codes[keep], want_scales[keep])


def test_fused_matches_the_unfused_gpu_chain():
    rows, hidden = 2048, 4096
    x = outlier_activations(rows, hidden, 16).to(DEV)
    w = (1 + torch.randn(hidden, generator=torch.Generator().manual_seed(17)) * 0.1).to(torch.bfloat16).to(DEV)
    scale, shift = (t.to(DEV) for t in modifiers(rows, hidden, 18))
    normed = torch.nn.functional.rms_norm(x, (hidden,), w, 1e-6)
    chain = triton_strict_bf16_modulate(normed.reshape(1, rows, hidden), scale, shift).reshape(rows, hidden)
    want_codes, want_scales = quantize_fp8_rows(chain)
    codes, scales = quantize_fp8_norm_modulate(x, w, 1e-6, scale, shift)
    assert_codes_close(codes, scales, codes_of(want_codes), want_scales.cpu().numpy())


def test_execution_prologue_equals_quantising_the_modulated_input():
    rows, hidden, n = 512, 1024, 3 * 256
    x = outlier_activations(rows, hidden, 19).to(DEV).reshape(2, rows // 2, hidden)
    w = torch.ones(hidden, dtype=torch.bfloat16, device=DEV)
    scale, shift = (t.to(DEV) for t in modifiers(rows // 2, hidden, 20))
    codes, wscale = quantize_fp8_rows((torch.randn(n, hidden, generator=torch.Generator().manual_seed(21))
                                       * 0.02).to(torch.bfloat16).to(DEV), pad_to=1)
    execution = RowFP8Execution("w8a8")
    prologue = NormModulate(w, scale, shift, 1e-6)
    q, k, v = execution.qkv_linear(x, codes, wscale, prologue=prologue)
    normed = torch.nn.functional.rms_norm(x, (hidden,), w, 1e-6)
    q2, k2, v2 = execution.qkv_linear(triton_strict_bf16_modulate(normed, scale, shift), codes, wscale)
    for a, b in ((q, q2), (k, k2), (v, v2)):
        rel = ((a.float() - b.float()).norm() / b.float().norm()).item()
        assert rel <= 1e-3, rel
    lin = execution.linear(x, codes, wscale, prologue=prologue)
    assert torch.equal(lin[..., :256], q)
    with pytest.raises(ValueError, match="tokens differ"):
        execution.linear(x, codes, wscale, prologue=NormModulate(w, scale[:3], shift[:3]))
    with pytest.raises(ValueError, match="w8a8"):
        RowFP8Execution("weight-only").linear(x, codes, wscale, prologue=prologue)
