"""Drop-in API tests for RowFP8Execution / RowFP8Linear, ported from the reference's
tests/test_fp8_linear.py (Hansimov/vflash).  CPU-only: layout validation,
counters, observer, weight-only exactness and the W8A8 device refusal.
"""

from __future__ import annotations

import pytest
import torch

from vflash_b200.native.h3_fp8_linear import RowFP8Execution, RowFP8Linear


def weights():
    # tests/test_fp8_linear.py:13-16 of the reference
    codes = torch.arange(128).reshape(16, 8).to(torch.float8_e4m3fn)
    scales = torch.linspace(0.01, 0.1, 16).unsqueeze(1)
    return codes, scales


@pytest.mark.parametrize("shape", [(8,), (3, 8), (2, 3, 8), (0, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_weight_only_is_exact_restored_weight_expression(shape, dtype):
    codes, scales = weights()
    values = torch.randn(shape, dtype=dtype)
    bias = torch.randn(16, dtype=dtype)
    execution = RowFP8Execution()
    actual = execution.linear(values, codes, scales, bias)
    restored = (codes.float() * scales).to(dtype)
    expected = torch.nn.functional.linear(values, restored, bias)
    torch.testing.assert_close(actual, expected, rtol=0, atol=0)
    assert execution.calls == {"weight_only": 1, "w8a8": 0}


def test_module_assigns_weight_scales_without_bias_copy():
    codes, scales = weights()
    original = torch.nn.Linear(8, 16)
    execution = RowFP8Execution()
    module = RowFP8Linear(original, execution)
    assert module.bias is original.bias and module.weight.is_meta and module.row_scale.is_meta
    module.load_state_dict({"weight": codes, "row_scale": scales, "bias": original.bias}, assign=True)
    value = torch.randn(2, 8)
    torch.testing.assert_close(
        module(value), execution.linear(value, codes, scales, module.bias), rtol=0, atol=0)
    assert not module.weight.requires_grad


@pytest.mark.parametrize("backend", ["torch", "triton"])
def test_w8a8_cpu_fails_without_fallback(backend):
    codes, scales = weights()
    execution = RowFP8Execution("w8a8", activation_quantizer=backend)
    with pytest.raises(ValueError, match="SM100"):
        execution.linear(torch.ones(3, 8, dtype=torch.bfloat16), codes, scales)
    assert execution.calls == {"weight_only": 0, "w8a8": 0}


@pytest.mark.parametrize("method", ["qkv_linear", "gelu_linear", "swiglu_linear"])
def test_fused_entry_points_refuse_cpu_and_weight_only(method):
    codes = torch.zeros(96, 64, dtype=torch.float8_e4m3fn)
    scales = torch.ones(96, 1)
    value = torch.ones(3, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="w8a8"):
        getattr(RowFP8Execution(), method)(value, codes, scales)
    execution = RowFP8Execution("w8a8")
    with pytest.raises(ValueError, match="SM100"):
        getattr(execution, method)(value, codes, scales)
    assert execution.calls == {"weight_only": 0, "w8a8": 0}


@pytest.mark.parametrize("bad", ["codes", "scale_dtype", "scale_shape", "input_shape", "rank", "bias"])
def test_bad_layout_never_enters_gemm(bad, monkeypatch):
    codes, scales = weights()
    value = torch.ones(3, 8)
    bias = None
    if bad == "codes":
        codes = codes.float()
    elif bad == "scale_dtype":
        scales = scales.bfloat16()
    elif bad == "scale_shape":
        scales = scales.T
    elif bad == "input_shape":
        value = torch.ones(3, 7)
    elif bad == "rank":
        codes = codes.flatten()
    elif bad == "bias":
        bias = torch.ones(15)

    def forbidden(*args, **kwargs):
        pytest.fail("invalid layout reached GEMM")

    import vflash_b200.native.h3_fp8_linear as mod

    monkeypatch.setattr(torch.nn.functional, "linear", forbidden)
    monkeypatch.setattr(mod, "fp8_gemm", forbidden)
    monkeypatch.setattr(mod, "quantize_fp8_rows", forbidden)
    with pytest.raises(ValueError, match="declared"):
        RowFP8Execution().linear(value, codes, scales, bias)
    with pytest.raises(ValueError, match="declared"):
        RowFP8Execution("w8a8").linear(value, codes, scales, bias)


def test_executions_keep_precision_observation_and_counts_independent():
    codes, scales = weights()
    a, b = RowFP8Execution(), RowFP8Execution("w8a8")
    observed = []
    a.observer = lambda: observed.append(dict(a.calls))
    a.linear(torch.ones(8), codes, scales)
    assert observed == [{"weight_only": 0, "w8a8": 0}]
    assert b.mode == "w8a8" and b.calls == {"weight_only": 0, "w8a8": 0}
    with pytest.raises(ValueError):
        a.select("silent-fallback")
    assert a.mode == "weight-only"


def test_constructor_validation():
    with pytest.raises(ValueError, match="quantizer"):
        RowFP8Execution(activation_quantizer="numpy")
    with pytest.raises(ValueError, match="boolean"):
        RowFP8Execution(fast_accum=1)


def test_known_answer_ones_times_ones_is_sixteen():
    # reference tests/test_fp8_loaders.py:31-47: ones e4m3 codes, unit row scales, K = 16
    codes = torch.ones(4, 16).to(torch.float8_e4m3fn)
    scales = torch.ones(4, 1)
    out = RowFP8Execution("weight-only").linear(torch.ones(2, 16), codes, scales)
    assert torch.equal(out, torch.full((2, 4), 16.0))


def test_reference_named_torch_quantiser_refuses_the_host():
    from vflash_b200.native.h3_fp8_linear import _quantize_activation_torch

    with pytest.raises(ValueError, match="SM100"):
        _quantize_activation_torch(torch.zeros(4, 16, dtype=torch.bfloat16))
