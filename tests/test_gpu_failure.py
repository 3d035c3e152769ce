"""Failure detection on the GPU without a fault: a bounded wait that runs out.

``vfb_wait_selftest`` waits on a barrier nothing completes; the wait must give
up after its limit, record VFB_ETIMEOUT in the device status word, and leave
the context usable (a GEMM afterwards gives the same bits as before).  Nothing here traps,
faults or hangs: the wait is bounded.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.native.h3_fp8_linear import RowFP8Execution

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports_status():
    _lib.device_status(clear=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    _lib.check(_lib.load().vfb_wait_selftest(50_000_000, _lib.stream_handle(torch.device("cuda"))),
               "vfb_wait_selftest")
    end.record()
    torch.cuda.synchronize()
    assert 45.0 <= start.elapsed_time(end) < 2000.0
    assert _lib.device_status(clear=True) == _lib.VFB_ETIMEOUT
    assert _lib.device_status(clear=True) == 0  # cleared


def test_context_stays_usable_after_a_timeout():
    x = outlier_activations(256, 512, 3).cuda()
    codes, scale = fp8_weight(256, 512, 4)
    execution = RowFP8Execution("w8a8")
    before = execution.linear(x, codes.cuda(), scale.cuda())
    _lib.load().vfb_wait_selftest(10_000_000, _lib.stream_handle(torch.device("cuda")))
    assert _lib.device_status(clear=True) == _lib.VFB_ETIMEOUT
    after = execution.linear(x, codes.cuda(), scale.cuda())
    assert torch.equal(before, after)
    assert _lib.device_status(clear=True) == 0


def test_selftest_rejects_out_of_range_limits():
    assert _lib.load().vfb_wait_selftest(10, None) == _lib.VFB_EINVAL
    assert _lib.load().vfb_wait_selftest(20_000_000_000, None) == _lib.VFB_EINVAL
