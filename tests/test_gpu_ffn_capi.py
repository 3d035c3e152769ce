"""The FP8 FFN entry points equal the step-by-step composition bit for bit.

The composition is the chain the reference runs for the block's FFN, each
step through this library's own separately tested entry points: the
per-token quantiser, the up GEMM with the activation epilogue (GELU-tanh or
SwiGLU), the quantiser again on the bf16 intermediate, and the down GEMM
with bias / gated residual.  vfb_fp8_ffn (RowFP8Execution.ffn) sequences
those launches in one call; vfb_fp8_ffn_one_kernel runs the up GEMM, the
requantisation and the down GEMM as one persistent kernel and must give the
same bits: the same MMA tiles in the same K order, the same epilogue
arithmetic and the same quotient per code.  Shapes cover several row-block
groups of its schedule, ragged rows, partial down tiles, and widths the
one-kernel path does not tile (it then runs the launches).
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import (Epilogue, KernelInputError, fp8_ffn, fp8_gemm, quantize_fp8_norm_modulate,
                                 quantize_fp8_rows)
from vflash_b200.native.h3_fp8_linear import NormModulate, RowFP8Execution

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(shape, seed, std=1.0):
    return (torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16).to(DEV)


def composition(codes, scales, rows, up, up_s, down, down_s, kind, up_bias, down_bias, residual, gate):
    mid = fp8_gemm(codes, scales, rows, up, up_s, Epilogue(kind=kind, bias=up_bias))
    mid_codes, mid_scales = quantize_fp8_rows(mid)
    if residual is None:
        ep = Epilogue(bias=down_bias)
    else:
        ep = Epilogue(kind=_lib.EPI_RESIDUAL, bias=down_bias, residual=residual, gate=gate,
                      tokens=0 if gate is None else gate.shape[0])
    return fp8_gemm(mid_codes, mid_scales, rows, down, down_s, ep)


def case(rows, hidden, width, activation, with_residual, seed=7):
    x = outlier_activations(rows, hidden, rows + hidden).to(DEV)
    n_up = 2 * width if activation == "swiglu" else width
    up, up_s = fp8_weight(n_up, hidden, seed)
    down, down_s = fp8_weight(hidden, width, seed + 1)
    return dict(x=x, up=up.to(DEV), up_s=up_s.to(DEV), down=down.to(DEV), down_s=down_s.to(DEV),
                up_bias=bf16((n_up,), seed + 2, 0.01), down_bias=bf16((hidden,), seed + 3, 0.01),
                residual=bf16((rows, hidden), seed + 4) if with_residual else None,
                gate=bf16((rows % 7 + 1, hidden), seed + 5, 0.5) if with_residual else None)


SHAPES = [
    (150, 256, 512),     # one row block
    (17, 512, 1024),     # fewer rows than a tile
    (1000, 1024, 4096),  # one group of four row blocks
    (2100, 512, 768),    # three groups, the last partial; three up tiles per row block
    (4500, 672, 1024),   # five groups; H = 672: a partial down tile
    (300, 256, 288),     # widths the fused kernel does not tile: the three-launch path
]


@pytest.mark.parametrize("rows,hidden,width", SHAPES)
@pytest.mark.parametrize("activation", ["gelu_tanh", "swiglu"])
@pytest.mark.parametrize("with_residual", [False, True])
def test_ffn_entry_points_equal_step_by_step_composition(rows, hidden, width, activation, with_residual):
    c = case(rows, hidden, width, activation, with_residual)
    kind = _lib.EPI_SWIGLU if activation == "swiglu" else _lib.EPI_GELU_TANH
    codes, scales = quantize_fp8_rows(c["x"])
    want = composition(codes, scales, rows, c["up"], c["up_s"], c["down"], c["down_s"], kind, c["up_bias"],
                       c["down_bias"], c["residual"], c["gate"])
    for one_kernel in (False, True):
        got = fp8_ffn(c["x"], c["up"], c["up_s"], c["down"], c["down_s"], activation=kind, up_bias=c["up_bias"],
                      down_bias=c["down_bias"], residual=c["residual"], gate=c["gate"], one_kernel=one_kernel)
        assert torch.equal(got, want), f"one_kernel={one_kernel}"
        ex = RowFP8Execution("w8a8")
        via_api = ex.ffn(c["x"], c["up"], c["up_s"], c["down"], c["down_s"], activation=activation,
                         up_bias=c["up_bias"], down_bias=c["down_bias"], residual=c["residual"], gate=c["gate"],
                         one_kernel=one_kernel)
        assert torch.equal(via_api, want), f"one_kernel={one_kernel}"
        assert ex.calls["w8a8"] == 2
    assert _lib.device_status(clear=True) == _lib.VFB_OK


@pytest.mark.parametrize("activation", ["gelu_tanh", "swiglu"])
def test_fused_ffn_after_the_norm_modulate_prologue(activation):
    rows, hidden, width, tokens = 1100, 512, 1024, 275
    c = case(rows, hidden, width, activation, with_residual=True, seed=30)
    norm_w = bf16((hidden,), 40, 0.1) + 1
    scale, shift = bf16((tokens, hidden), 41, 0.3), bf16((tokens, hidden), 42, 0.3)
    kind = _lib.EPI_SWIGLU if activation == "swiglu" else _lib.EPI_GELU_TANH
    codes, scales = quantize_fp8_norm_modulate(c["x"], norm_w, 1e-6, scale, shift)
    want = composition(codes, scales, rows, c["up"], c["up_s"], c["down"], c["down_s"], kind, c["up_bias"],
                       c["down_bias"], c["residual"], c["gate"])
    got = RowFP8Execution("w8a8").ffn(
        c["x"], c["up"], c["up_s"], c["down"], c["down_s"], activation=activation, up_bias=c["up_bias"],
        down_bias=c["down_bias"], residual=c["residual"], gate=c["gate"],
        prologue=NormModulate(norm_w, scale, shift, 1e-6))
    assert torch.equal(got, want)


def test_one_kernel_ffn_repeats_bit_for_bit():
    """The one-kernel path's work order is dynamic (pairs take items from a counter); the results are not."""
    c = case(3000, 512, 2048, "gelu_tanh", with_residual=True, seed=50)
    runs = [fp8_ffn(c["x"], c["up"], c["up_s"], c["down"], c["down_s"], residual=c["residual"], one_kernel=True)
            for _ in range(3)]
    assert torch.equal(runs[0], runs[1]) and torch.equal(runs[0], runs[2])
    assert _lib.device_status(clear=True) == _lib.VFB_OK


def test_c_entry_rejects_a_short_workspace():
    x = outlier_activations(64, 256, 1).to(DEV)
    up, up_s = fp8_weight(512, 256, 2)
    down, down_s = fp8_weight(256, 512, 3)
    lib = _lib.load()
    need = lib.vfb_fp8_ffn_workspace_bytes(64, 256, 512)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    out = torch.empty(64, 256, dtype=torch.bfloat16, device=DEV)
    rc = lib.vfb_fp8_ffn(x.data_ptr(), 64, 256, 256, up.to(DEV).data_ptr(), up_s.to(DEV).data_ptr(), 512,
                         down.to(DEV).data_ptr(), down_s.to(DEV).data_ptr(), _lib.EPI_GELU_TANH, None, None,
                         None, 0, None, 0, 0, out.data_ptr(), 256, ws.data_ptr(), need - 256,
                         _lib.stream_handle(torch.device(DEV)))
    assert rc == _lib.VFB_EINVAL and "workspace" in _lib.last_error()
    with pytest.raises(KernelInputError):
        fp8_ffn(x, up.to(DEV), up_s.to(DEV), down.to(DEV)[:, :256].contiguous(), down_s.to(DEV))
