"""Bounded row FP8 activation quantisation on SM100 (drop-in for vflash's module).

Mirrors ``quantize_activation`` of Hansimov/vflash
(src/vflash/native/h3_fp8_activation.py:31-55): same input contract (CUDA
bf16 ``[M, K]``, unit column stride, 16 <= K <= 32768), same outputs (e4m3
codes ``[ceil16(M), K]`` and fp32 scales ``[ceil16(M), 1]``), same arithmetic
bit for bit, computed by the native kernel ``vfb_fp8_quant_rows``.
The device gate is SM100 instead of SM90/SM120.
"""

from __future__ import annotations

import torch

from ..kernels import quantize_fp8_rows


def quantize_activation(matrix):
    if (
        matrix.device.type != "cuda"
        or matrix.dtype != torch.bfloat16
        or matrix.ndim != 2
        or matrix.stride(1) != 1
        or not 16 <= matrix.shape[1] <= 32768
        or torch.cuda.get_device_capability(matrix.device) != (10, 0)
    ):
        raise ValueError("row FP8 activation requires a bounded SM100 BF16 matrix")
    return quantize_fp8_rows(matrix, pad_to=16)
