"""The fused FP8 FFN through its single C entry point (vfb_fp8_ffn) equals RowFP8Execution.ffn bit for bit.

Both run the same four kernels (quantiser, up GEMM + activation, requantiser,
down GEMM + bias / gated residual); the C entry sequences them on the
caller's stream with its intermediates in a caller-owned workspace.  The
Python path is itself checked against the oracle in test_gpu_fp8_gemm.py.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import KernelInputError, fp8_ffn
from vflash_b200.native.h3_fp8_linear import RowFP8Execution

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(shape, seed, std=1.0):
    return (torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("rows,hidden,width", [(150, 256, 512), (17, 512, 1024), (1000, 1024, 4096)])
@pytest.mark.parametrize("activation", ["gelu_tanh", "swiglu"])
@pytest.mark.parametrize("with_residual", [False, True])
def test_c_entry_equals_python_composition(rows, hidden, width, activation, with_residual):
    x = outlier_activations(rows, hidden, rows + hidden).to(DEV)
    n_up = 2 * width if activation == "swiglu" else width
    up, up_s = fp8_weight(n_up, hidden, 7)
    down, down_s = fp8_weight(hidden, width, 8)
    up, up_s, down, down_s = up.to(DEV), up_s.to(DEV), down.to(DEV), down_s.to(DEV)
    up_bias, down_bias = bf16((n_up,), 9, 0.01), bf16((hidden,), 10, 0.01)
    residual = bf16((rows, hidden), 11) if with_residual else None
    gate = bf16((rows % 7 + 1, hidden), 12, 0.5) if with_residual else None
    ex = RowFP8Execution("w8a8")
    want = ex.ffn(x, up, up_s, down, down_s, activation=activation, up_bias=up_bias, down_bias=down_bias,
                  residual=residual, gate=gate)
    kind = _lib.EPI_SWIGLU if activation == "swiglu" else _lib.EPI_GELU_TANH
    got = fp8_ffn(x, up, up_s, down, down_s, activation=kind, up_bias=up_bias, down_bias=down_bias,
                  residual=residual, gate=gate)
    assert torch.equal(got, want)
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
