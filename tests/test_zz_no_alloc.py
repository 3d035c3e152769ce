"""vfb_fp8_ffn_noalloc: the fused FP8 FFN for callers that cannot allocate device memory.

A process that embeds the library in a runtime which already owns the GPU's
memory, or code that may not take cudaMalloc's implicit synchronisation,
cannot hand vfb_fp8_ffn a workspace; vfb_fp8_ffn_noalloc keeps the
intermediates in the library's own fixed 64 MiB device array instead.  Its
output must equal vfb_fp8_ffn's bit for bit (the same kernels run), on two
calls in a row that share the array, and shapes that need more than the
array must be refused before anything runs.

This file is named to be collected last, so a run that stops at the first
failure has run every other test before it.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import fp8_ffn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(shape, seed, std=1.0):
    return (torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16).to(DEV)


def case(rows, hidden, width, activation, seed, with_residual):
    x = outlier_activations(rows, hidden, seed).to(DEV)
    n_up = 2 * width if activation == _lib.EPI_SWIGLU else width
    up, up_s = fp8_weight(n_up, hidden, seed + 1)
    down, down_s = fp8_weight(hidden, width, seed + 2)
    args = dict(x=x, up=up.to(DEV), up_scales=up_s.to(DEV), down=down.to(DEV), down_scales=down_s.to(DEV),
                activation=activation, up_bias=bf16((n_up,), seed + 3, 0.01),
                down_bias=bf16((hidden,), seed + 4, 0.01),
                residual=bf16((rows, hidden), seed + 5) if with_residual else None,
                gate=bf16((5, hidden), seed + 6, 0.5) if with_residual else None)
    return args


def call_noalloc(a) -> torch.Tensor:
    """The new entry point through the C ABI; only the output buffer is the caller's."""
    lib = _lib.load()
    x, up, down, residual, gate = a["x"], a["up"], a["down"], a["residual"], a["gate"]
    rows, hidden = x.shape
    out = torch.empty(rows, hidden, dtype=torch.bfloat16, device=DEV)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    rc = lib.vfb_fp8_ffn_noalloc(
        x.data_ptr(), rows, hidden, x.stride(0), up.data_ptr(), a["up_scales"].data_ptr(), up.shape[0],
        down.data_ptr(), a["down_scales"].data_ptr(), a["activation"], ptr(a["up_bias"]), ptr(a["down_bias"]),
        ptr(residual), 0 if residual is None else residual.stride(0), ptr(gate),
        0 if gate is None else gate.stride(0), 0 if gate is None else gate.shape[0], out.data_ptr(), hidden,
        _lib.stream_handle(torch.device(DEV)))
    _lib.check(rc, "vfb_fp8_ffn_noalloc")
    return out


def test_noalloc_equals_the_workspace_entry_on_two_calls_in_a_row():
    first = case(150, 256, 512, _lib.EPI_GELU_TANH, 10, with_residual=True)
    second = case(333, 512, 1024, _lib.EPI_SWIGLU, 20, with_residual=False)
    got_first = call_noalloc(first)
    got_second = call_noalloc(second)  # reuses the array the first call wrote
    torch.cuda.synchronize()
    assert torch.equal(got_first, fp8_ffn(**first))
    assert torch.equal(got_second, fp8_ffn(**second))
    # and the first shapes again, after the larger call left its contents behind
    assert torch.equal(call_noalloc(first), got_first)
    assert _lib.device_status(clear=True) == _lib.VFB_OK


def test_noalloc_refuses_shapes_beyond_its_array():
    lib = _lib.load()
    rows, hidden, width = 4096, 4096, 16384
    need = lib.vfb_fp8_ffn_workspace_bytes(rows, hidden, width)
    assert need > 64 << 20
    rc = lib.vfb_fp8_ffn_noalloc(None, rows, hidden, hidden, None, None, width, None, None, _lib.EPI_GELU_TANH,
                                 None, None, None, 0, None, 0, 0, None, hidden,
                                 _lib.stream_handle(torch.device(DEV)))
    assert rc == _lib.VFB_EINVAL
    assert "scratch" in _lib.last_error() and str(need) in _lib.last_error()
