"""Explicit NVFP4 arithmetic for the packed H3 QAD linear contract on SM100 (drop-in).

Mirrors Hansimov/vflash src/vflash/native/h3_nvfp4_linear.py: the frozen
``NVFP4Weight`` layout contract (packed e2m1 ``[N, K/2]`` with element 2i in
the low nibble, ue4m3 block scales ``[N, K/16]`` in the 128x4 layout, fp32
``alpha`` and ``input_scale`` scalars), ``NVFP4Execution.linear`` with its
validation, counters and single ``_require_device`` / ``_operators`` hooks.
``_operators()`` returns the native quantiser and GEMM behind the same
call signatures the reference uses for FlashInfer's ``nvfp4_quantize`` and
``mm_fp4`` (h3_nvfp4_linear.py:61-64, 102, 118-130), so callers and the
reference's tests see the same plumbing; the device gate is SM100.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import cache

import torch

from ..kernels import nvfp4_gemm, nvfp4_quantize

SF_LAYOUT_128x4 = "128x4"


@dataclass(frozen=True, eq=False)
class NVFP4Weight:
    packed: torch.Tensor
    scales: torch.Tensor
    alpha: torch.Tensor
    input_scale: torch.Tensor

    def __post_init__(self):
        if (
            self.packed.dtype != torch.uint8
            or self.packed.ndim != 2
            or min(self.packed.shape) < 1
            or self.packed.shape[0] % 128
            or self.packed.shape[1] % 32
            or self.scales.dtype != torch.uint8
            or self.scales.shape != (self.packed.shape[0], self.packed.shape[1] // 8)
            or not self.packed.is_contiguous()
            or not self.scales.is_contiguous()
        ):
            raise ValueError("NVFP4 requires declared packed codes and 128x4 block scales")
        for scalar in (self.alpha, self.input_scale):
            if scalar.dtype != torch.float32 or scalar.shape != torch.Size([]):
                raise ValueError("NVFP4 calibration and output alpha must be FP32 scalars")
            if scalar.device.type != "meta" and not bool(torch.isfinite(scalar) & (scalar > 0)):
                raise ValueError("NVFP4 scales must be positive and finite")
        if len({v.device for v in (self.packed, self.scales, self.alpha, self.input_scale)}) != 1:
            raise ValueError("NVFP4 tensors must share one explicit device")

    @property
    def in_features(self):
        return self.packed.shape[1] * 2

    @property
    def out_features(self):
        return self.packed.shape[0]


@cache
def _require_device(device):
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise ValueError("This NVFP4 execution requires an explicit SM100 CUDA device")


def _quantize(matrix, global_sf, *, sfLayout, do_shuffle):  # noqa: N803 - reference keyword names
    """``nvfp4_quantize`` contract: 128x4 scales, no shuffle."""
    if sfLayout != SF_LAYOUT_128x4 or do_shuffle:
        raise ValueError("only the 128x4 unshuffled scale layout is supported")
    return nvfp4_quantize(matrix, global_sf)


def _matmul(a, b, a_scale, b_scale, alpha, out_dtype, out, *, block_size, use_8x4_sf_layout,
            backend, use_nvfp4):
    """``mm_fp4`` contract: ``b``/``b_scale`` are the transposed weight views."""
    if (block_size != 16 or use_8x4_sf_layout or not use_nvfp4 or out_dtype != torch.bfloat16
            or out is not None or backend != "cutlass"):
        raise ValueError("only the NVFP4 block-16 128x4 bf16 contract is supported")
    return nvfp4_gemm(a, a_scale, b.T, b_scale.T, alpha)


def _operators():
    return SF_LAYOUT_128x4, _quantize, _matmul


class NVFP4Execution:
    """Frozen W4A4 execution on SM100; host clocks/counters remain diagnostic."""

    contract = "nvfp4-e2m1-block16-128x4-cutlass-v1"

    def __init__(self):
        self.calls = 0
        self.rows = 0
        self._ops = None

    def linear(self, values, weight: NVFP4Weight, bias=None):
        if (
            values.ndim < 1
            or values.shape[-1] != weight.in_features
            or values.dtype not in (torch.bfloat16, torch.float16, torch.float32)
            or values.device != weight.packed.device
        ):
            raise ValueError("NVFP4 input differs from its frozen matrix")
        if torch.is_grad_enabled() and values.requires_grad:
            raise ValueError("NVFP4 execution is inference-only")
        _require_device(values.device)
        if bias is not None and (
            bias.shape != (weight.out_features,)
            or bias.device != values.device
            or bias.dtype != torch.bfloat16
        ):
            raise ValueError("NVFP4 bias must match its BF16 output")
        if self._ops is None:
            self._ops = _operators()
        layout, quantize, matmul = self._ops
        shape = values.shape
        matrix = values.to(torch.bfloat16) if values.dtype == torch.float32 else values
        matrix = matrix.reshape(-1, weight.in_features)
        if matrix.shape[0] == 0:
            raise ValueError("NVFP4 input rows must be nonempty")
        codes, scales = quantize(matrix, weight.input_scale, sfLayout=layout, do_shuffle=False)
        padded_rows = matrix.shape[0] + (-matrix.shape[0]) % 128
        padded_columns = (weight.in_features // 16 + 3) // 4 * 4
        if (
            scales.dtype != torch.uint8
            or scales.device != matrix.device
            or scales.numel() != padded_rows * padded_columns
        ):
            raise ValueError("The quantizer omitted the required 128x4 scale padding")
        if codes.dtype != torch.uint8 or codes.shape != (matrix.shape[0], weight.in_features // 2):
            raise ValueError("The quantizer returned a different packed layout")
        output = matmul(
            codes,
            weight.packed.T,
            scales,
            weight.scales.T,
            weight.alpha / weight.input_scale,
            torch.bfloat16,
            None,
            block_size=16,
            use_8x4_sf_layout=False,
            backend="cutlass",
            use_nvfp4=True,
        )
        if output.dtype != torch.bfloat16 or output.shape != (matrix.shape[0], weight.out_features):
            raise ValueError("The NVFP4 kernel returned a different output layout")
        self.calls += 1
        self.rows += matrix.shape[0]
        output = output.reshape(*shape[:-1], weight.out_features)
        return output if bias is None else output + bias
