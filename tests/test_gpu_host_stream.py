"""Row-chunked host pipeline: equal to one call on all rows, bit for bit."""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200.native.h3_fp8_linear import RowFP8Execution
from vflash_b200.native.h3_host_stream import HostRowPipeline

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("rows,chunk", [(10001, 4096), (300, 4096), (4096, 1024), (33, 16)])
def test_pipelined_qkv_equals_one_call(rows, chunk):
    k, n = 512, 3 * 256
    codes, scale = fp8_weight(n, k, 7)
    codes, scale = codes.to(DEV), scale.to(DEV)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(8)) * 0.01).to(torch.bfloat16).to(DEV)
    x = outlier_activations(rows, k, 9)
    execution = RowFP8Execution("w8a8")
    want = execution.qkv_linear(x.to(DEV), codes, scale, bias)
    x_host = x.pin_memory()
    outs = [torch.empty((rows, n // 3), dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    pipe = HostRowPipeline(lambda xd: execution.qkv_linear(xd, codes, scale, bias), DEV, chunk_rows=chunk)
    for _ in range(2):  # slots and events are reused by a second call
        for o in outs:
            o.fill_(float("nan"))
        pipe(x_host, outs)
        torch.cuda.current_stream().synchronize()
        for got, ref in zip(outs, want):
            assert torch.equal(got, ref.cpu())


def test_rejects_pageable_host_buffers():
    pipe = HostRowPipeline(lambda xd: (xd,), DEV)
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="pinned"):
        pipe(x, [torch.zeros(4, 8, dtype=torch.bfloat16).pin_memory()])
