"""RMSNorm + AdaLN modulate + NVFP4 quantisation in one pass (the pre-GEMM fusion for NVFP4 linears).

The fused kernel's row sum of squares is an fp32 reduction in the kernel's
own order.  On inputs whose squares sum exactly in fp32 (values in
{0, +-0.5, +-1, +-2}) every order gives the same sum, so the kernel must
match the oracle's norm and modulate bit for bit, and its codes and scales
must equal the NVFP4 quantiser's on the oracle's modulated tensor.  On
general inputs an rstd one fp32 ulp away can move a bf16 rounding, so the
comparison with torch's rms_norm chain allows a small fraction of codes and
scales to differ.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from tests.helpers import bits_of, outlier_activations
from vflash_b200.kernels import nvfp4_norm_modulate_quantize, nvfp4_quantize
from vflash_b200.native.h3_fp8_linear import NormModulate
from vflash_b200.native.h3_fused_ops import triton_strict_bf16_modulate
from vflash_b200.native.h3_nvfp4_linear import NVFP4Execution, NVFP4Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"


def exact_sum_input(rows, hidden, seed):
    gen = torch.Generator().manual_seed(seed)
    choices = torch.tensor([0.0, 0.5, -0.5, 1.0, -1.0, 2.0, -2.0])
    return choices[torch.randint(0, len(choices), (rows, hidden), generator=gen)].to(torch.bfloat16)


def modifiers(tokens, hidden, seed, std=0.3):
    gen = torch.Generator().manual_seed(seed)
    scale = (torch.randn(tokens, hidden, generator=gen) * std).to(torch.bfloat16)
    shift = (torch.randn(tokens, hidden, generator=gen) * std).to(torch.bfloat16)
    return scale, shift


def oracle_modulated(x, w, scale, shift, eps, tokens):
    rows = x.shape[0]
    normed = ep.rms_norm(bits_of(x), None if w is None else bits_of(w), eps)
    mod = ep.modulate(normed.reshape(rows // tokens, tokens, -1), bits_of(scale), bits_of(shift))
    return torch.from_numpy(mod.reshape(rows, -1).view(np.int16)).view(torch.bfloat16)


def global_scale(t):
    return (448.0 * 6.0 / t.float().abs().max()).to(torch.float32).reshape(())


@pytest.mark.parametrize("rows,hidden,tokens,with_weight", [(300, 4096, 100, True), (64, 5376, 1, False),
                                                            (129, 16384, 129, True), (7, 64, 7, True)])
def test_bit_exact_on_exact_sums(rows, hidden, tokens, with_weight):
    x = exact_sum_input(rows, hidden, 31)
    gen = torch.Generator().manual_seed(32)
    w = (1 + torch.randn(hidden, generator=gen) * 0.1).to(torch.bfloat16) if with_weight else None
    scale, shift = modifiers(tokens, hidden, 33)
    mod = oracle_modulated(x, w, scale, shift, 1e-6, tokens).to(DEV)
    gsf = global_scale(mod)
    want_codes, want_sf = nvfp4_quantize(mod, gsf)
    codes, sf = nvfp4_norm_modulate_quantize(x.to(DEV), None if w is None else w.to(DEV), 1e-6,
                                             scale.to(DEV), shift.to(DEV), gsf)
    assert codes.shape == want_codes.shape and sf.shape == want_sf.shape
    assert torch.equal(codes, want_codes)
    assert torch.equal(sf, want_sf)  # padding rows included


def test_close_to_the_torch_chain_on_general_inputs():
    rows, hidden = 2048, 4096
    x = outlier_activations(rows, hidden, 34).to(DEV)
    w = (1 + torch.randn(hidden, generator=torch.Generator().manual_seed(35)) * 0.1).to(torch.bfloat16).to(DEV)
    scale, shift = (t.to(DEV) for t in modifiers(rows, hidden, 36))
    normed = torch.nn.functional.rms_norm(x, (hidden,), w, 1e-6)
    chain = triton_strict_bf16_modulate(normed.reshape(1, rows, hidden), scale, shift).reshape(rows, hidden)
    gsf = global_scale(chain)
    want_codes, want_sf = nvfp4_quantize(chain, gsf)
    codes, sf = nvfp4_norm_modulate_quantize(x, w, 1e-6, scale, shift, gsf)
    assert (codes != want_codes).float().mean().item() <= 2e-2
    assert (sf != want_sf).float().mean().item() <= 1e-2


def test_zero_row_becomes_the_quantised_shift():
    rows, hidden = 130, 256
    x = exact_sum_input(rows, hidden, 37)
    x[5] = 0.0  # rstd = 1/sqrt(eps): the normalised row is 0, the output the shift
    scale, shift = modifiers(rows, hidden, 38)
    mod = oracle_modulated(x, None, scale, shift, 1e-5, rows).to(DEV)
    assert torch.equal(mod[5], shift[5].to(DEV))
    gsf = global_scale(mod)
    want = nvfp4_quantize(mod, gsf)
    got = nvfp4_norm_modulate_quantize(x.to(DEV), None, 1e-5, scale.to(DEV), shift.to(DEV), gsf)
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])


def weight_case(n, k, seed):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).to(torch.bfloat16).to(DEV)
    gsf = global_scale(w)
    packed, scales = nvfp4_quantize(w, gsf)
    return packed, scales.view(n, k // 16).contiguous(), (1.0 / gsf).to(torch.float32)


def test_execution_prologue_equals_the_linear_of_the_modulated_input():
    batch, tokens, hidden, n, f = 2, 75, 512, 384, 768
    x = exact_sum_input(batch * tokens, hidden, 39)
    w = (1 + torch.randn(hidden, generator=torch.Generator().manual_seed(40)) * 0.1).to(torch.bfloat16)
    scale, shift = modifiers(tokens, hidden, 41)
    mod = oracle_modulated(x, w, scale, shift, 1e-6, tokens).to(DEV).view(batch, tokens, hidden)
    xd = x.to(DEV).view(batch, tokens, hidden)
    prologue = NormModulate(w.to(DEV), scale.to(DEV), shift.to(DEV), 1e-6)
    packed, wscales, alpha = weight_case(n, hidden, 42)
    weight = NVFP4Weight(packed, wscales, alpha.reshape(()), global_scale(mod))
    engine = NVFP4Execution()
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(43)) * 0.01).to(torch.bfloat16).to(DEV)
    assert torch.equal(engine.linear(xd, weight, bias, prologue=prologue), engine.linear(mod, weight, bias))
    q, k, v = engine.qkv_linear(xd, weight, bias, prologue=prologue)
    q2, k2, v2 = engine.qkv_linear(mod, weight, bias)
    assert torch.equal(q, q2) and torch.equal(k, k2) and torch.equal(v, v2)
    # the FFN with the prologue on its input
    up_packed, up_scales, up_alpha = weight_case(f, hidden, 44)
    up = NVFP4Weight(up_packed, up_scales, up_alpha.reshape(()), global_scale(mod))
    mid = engine.gelu_linear(mod, up)
    down_packed, down_scales, down_alpha = weight_case(hidden, f, 45)
    down = NVFP4Weight(down_packed, down_scales, down_alpha.reshape(()), global_scale(mid))
    assert torch.equal(engine.ffn(xd, up, down, prologue=prologue), engine.ffn(mod, up, down))
    with pytest.raises(ValueError):
        engine.linear(xd.float(), weight, bias, prologue=prologue)
