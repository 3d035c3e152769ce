"""The profiling cases run clean: status word zero and finite outputs (small row counts)."""

from __future__ import annotations

import pytest

from vflash_b200 import profile_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("argv", [
    ["fp8_gemm", "--rows", "300", "--repeats", "1"],
    ["fp8_gemm_gelu", "--rows", "300", "--repeats", "1"],
    ["ffn", "--rows", "300", "--repeats", "1"],
    ["ffn", "--rows", "300", "--repeats", "1", "--swiglu", "--one-kernel"],
    ["nvfp4_gemm", "--rows", "300", "--n", "256", "--repeats", "1"],
    ["bf16_up", "--rows", "300", "--repeats", "1"],
])
def test_profile_case_runs(argv):
    assert profile_cases.main(argv) == 0
