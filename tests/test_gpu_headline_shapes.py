"""Parity at the benchmark's full shapes against the reference's own GPU composition.

Config 1 (merged QKV, M=32760, N=12288, K=4096, bias, Q/K/V planes) and
config 2 (FFN, M=32760, H=4096, F=16384, GELU-tanh or SwiGLU, residual) run
through the public drop-in (``RowFP8Execution.qkv_linear`` / ``.ffn``) and are
compared with the chain the reference runs for the same layer
(src/vflash/native/h3_fp8_linear.py:92-121 per linear; the activation steps
of h3_fused_ops.py:185-224 and the residual add):

  per-token quantiser (_quantize_activation_torch's expression, h3_fp8_linear.py:18-31,
  evaluated by torch on the GPU) -> torch._scaled_mm rowwise (cuBLASLt) -> + bias
  -> F.gelu(approximate="tanh") | value * bf16(silu(gate)) -> quantiser again
  -> torch._scaled_mm -> + residual

Bars: rel-L2 <= 1e-2 against that chain (bf16 tolerance of the north star);
rel-L2 <= 2e-2 against the same quantised operands dequantised and multiplied
in fp32; activation codes and scales bit-exact against the quantiser
expression, for the input and for the intermediate.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import outlier_activations
from vflash_b200.native.h3_fp8_linear import RowFP8Execution

pytestmark = pytest.mark.gpu
DEV = "cuda"
TINY = torch.finfo(torch.float32).tiny


def torch_quantize(matrix: torch.Tensor):
    """The reference's portable quantiser expression (h3_fp8_linear.py:18-31), on the device, unpadded.

    The reference evaluates ``maxima / 448.0`` on the host (IEEE division);
    torch on CUDA turns a division by a Python scalar into a multiplication
    by its reciprocal, which differs by an ulp for some maxima, so the
    divisor is a device tensor here to keep the IEEE quotient.
    """
    floats = matrix.float()
    maxima = floats.abs().amax(dim=1, keepdim=True)
    scale = torch.where(maxima > 0, (maxima / torch.full_like(maxima, 448.0)).clamp_min(TINY),
                        torch.ones_like(maxima))
    return (floats / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), scale


def weight(n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    return torch_quantize(w)


def scaled_mm(codes, scales, w, ws):
    out = torch._scaled_mm(codes, w.t(), scale_a=scales, scale_b=ws.t(), out_dtype=torch.bfloat16)
    return out[0] if isinstance(out, tuple) else out


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def dequant(codes, scales):
    return codes.float() * scales


def test_config1_merged_qkv_full_shape():
    m, k, n = 32760, 4096, 12288
    x = outlier_activations(m, k, 1001).to(DEV)
    w, ws = weight(n, k, 2010)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(3001)) * 0.01).to(torch.bfloat16).to(DEV)
    q, kk, v = RowFP8Execution("w8a8").qkv_linear(x, w, ws, bias)
    got = torch.cat([t.reshape(m, -1) for t in (q, kk, v)], dim=1)
    codes, scales = torch_quantize(x)
    chain = scaled_mm(codes, scales, w, ws) + bias
    assert rel(got, chain) <= 1e-2
    deq = dequant(codes, scales) @ dequant(w, ws).t() + bias.float()
    assert rel(got, deq) <= 2e-2
    # the planes are the chain's .chunk(3) views
    for plane, ref in zip((q, kk, v), chain.chunk(3, dim=-1)):
        assert plane.reshape(m, -1).shape == ref.shape
        assert rel(plane.reshape(m, -1), ref) <= 1e-2


@pytest.mark.parametrize("activation", ["gelu_tanh", "swiglu"])
def test_config2_ffn_full_shape(activation):
    m, h, f = 32760, 4096, 16384
    x = outlier_activations(m, h, 1002).to(DEV)
    n_up = 2 * f if activation == "swiglu" else f
    up, ups = weight(n_up, h, 2020)
    down, downs = weight(h, f, 2021)
    ex = RowFP8Execution("w8a8")
    got = ex.ffn(x, up, ups, down, downs, activation=activation, residual=x)

    # the reference's chain, step by step
    xc, xs = torch_quantize(x)
    y_up = scaled_mm(xc, xs, up, ups)
    if activation == "swiglu":
        value, gate = y_up[:, :f], y_up[:, f:]
        mid = value * torch.nn.functional.silu(gate)
    else:
        mid = torch.nn.functional.gelu(y_up, approximate="tanh")
    mc, ms = torch_quantize(mid)
    chain = x + scaled_mm(mc, ms, down, downs)
    assert rel(got, chain) <= 1e-2

    # the same quantisation steps, products in fp32
    up32 = dequant(xc, xs) @ dequant(up, ups).t()
    if activation == "swiglu":
        mid32 = up32[:, :f] * torch.nn.functional.silu(up32[:, f:])
    else:
        mid32 = torch.nn.functional.gelu(up32, approximate="tanh")
    del up32
    mc32, ms32 = torch_quantize(mid32)
    deq = x.float() + dequant(mc32, ms32) @ dequant(down, downs).t()
    del mid32, mc32
    assert rel(got, deq) <= 2e-2

    # the library's intermediate (its up GEMM with the activation epilogue) is
    # the chain's within bf16 tolerance, and its requantisation is the
    # quantiser expression bit for bit
    lin = ex.swiglu_linear if activation == "swiglu" else ex.gelu_linear
    ours_mid = lin(x, up, ups).reshape(m, f)
    assert rel(ours_mid, mid) <= 1e-2
    codes, scales = ex_quantize(ours_mid)
    want_codes, want_scales = torch_quantize(ours_mid)
    assert torch.equal(codes[:m].view(torch.uint8), want_codes.view(torch.uint8))
    assert torch.equal(scales[:m], want_scales)


def ex_quantize(matrix):
    from vflash_b200.kernels import quantize_fp8_rows

    return quantize_fp8_rows(matrix)
