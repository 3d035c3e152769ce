"""Thin torch-facing wrappers over the C ABI (include/vflash_b200.h).

These functions validate tensors, allocate outputs with torch's caching
allocator, select the tensor's device and current stream, and call the native
library.  They never compute on the host and never fall back: a missing
library, a non-SM100 device or a rejected layout raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
BF16 = torch.bfloat16


class KernelInputError(ValueError):
    """A tensor handed to a native kernel violates its declared layout."""


def require_sm100(device: torch.device) -> None:
    """Raise unless ``device`` is a compute capability 10.0 CUDA device (B200)."""
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise KernelInputError("vflash_b200 kernels require an SM100 (B200) CUDA device")


def _aligned(t: torch.Tensor, nbytes: int = 16) -> bool:
    return t.data_ptr() % nbytes == 0


def padded_rows(rows: int, multiple: int = 16) -> int:
    return -(-rows // multiple) * multiple


def quantize_fp8_rows(matrix: torch.Tensor, *, pad_to: int = 16):
    """Per-token e4m3 codes ``[ceil(M/pad_to)*pad_to, K]`` and fp32 scales ``[.., 1]``.

    ``matrix`` is a bf16 ``[M, K]`` CUDA tensor with unit column stride (any
    row stride, e.g. the value half of a packed FFN projection).
    """
    if matrix.dtype != BF16 or matrix.ndim != 2 or matrix.stride(1) != 1 and matrix.shape[1] > 1:
        raise KernelInputError("FP8 activation quantisation needs a bf16 [M,K] matrix with unit column stride")
    rows, cols = matrix.shape
    if not 1 <= cols <= 32768:
        raise KernelInputError("FP8 activation quantisation needs 1 <= K <= 32768")
    padded = padded_rows(rows, pad_to)
    codes = torch.empty((padded, cols), device=matrix.device, dtype=FP8)
    scales = torch.empty((padded, 1), device=matrix.device, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(matrix.device):
        rc = lib.vfb_fp8_quant_rows(
            matrix.data_ptr() if rows else None, rows, cols, max(matrix.stride(0), cols),
            codes.data_ptr(), scales.data_ptr(), padded, _lib.stream_handle(matrix.device))
    _lib.check(rc, "vfb_fp8_quant_rows")
    return codes, scales


@dataclass
class Epilogue:
    """Options of the fused GEMM epilogue (see ``vfb_epilogue``)."""

    kind: int = _lib.EPI_STORE
    bias: torch.Tensor | None = None
    planes: int = 1                      # STORE/GELU: split N into this many output planes
    adapters: tuple | None = None        # STORE: one bf16 [M, N/planes] per plane (or None)
    scalings: tuple = (0.0, 0.0, 0.0)
    residual: torch.Tensor | None = None # RESIDUAL: bf16 [M, N]
    gate: torch.Tensor | None = None     # RESIDUAL: bf16 [tokens, N] with unit hidden stride
    tokens: int = 0


def fp8_gemm(a_codes: torch.Tensor, a_scales: torch.Tensor, rows: int, weight: torch.Tensor,
             w_scales: torch.Tensor, epilogue: Epilogue | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-scaled e4m3 GEMM ``bf16(sa * sw * A @ W^T)`` with a fused epilogue.

    ``a_codes`` e4m3 ``[>=rows, K]``, ``a_scales`` fp32 (>= rows entries),
    ``weight`` e4m3 ``[N, K]`` row-major, ``w_scales`` fp32 ``[N, 1]``.
    Returns bf16 ``[rows, N]`` (``[rows, N/2]`` for SWIGLU, ``[planes, rows,
    N/planes]`` when the output is split into planes).
    """
    ep = epilogue or Epilogue()
    n, k = weight.shape
    device = a_codes.device
    if (a_codes.dtype != FP8 or weight.dtype != FP8 or a_codes.ndim != 2 or a_codes.shape[1] != k
            or a_codes.stride(1) != 1 or weight.stride(1) != 1 or a_codes.shape[0] < rows):
        raise KernelInputError("FP8 GEMM operands differ from the declared e4m3 layout")
    if a_scales.dtype != torch.float32 or w_scales.dtype != torch.float32 or not w_scales.is_contiguous():
        raise KernelInputError("FP8 GEMM scales must be contiguous fp32")
    if not a_scales.is_contiguous() or a_scales.numel() < rows or w_scales.numel() != n:
        raise KernelInputError("FP8 GEMM scale vectors have the wrong length")
    if k % 16 or n % 32:
        raise KernelInputError("FP8 GEMM needs K % 16 == 0 and N % 32 == 0")
    for t in (a_codes, weight, w_scales):
        if t.device != device:
            raise KernelInputError("FP8 GEMM operands must share one device")
    if not (_aligned(a_codes) and _aligned(weight) and _aligned(w_scales)):
        raise KernelInputError("FP8 GEMM operands must be 16-byte aligned")

    e = _lib.Epilogue()
    e.kind = ep.kind
    if ep.bias is not None:
        if ep.bias.dtype != BF16 or ep.bias.shape != (n,) or not ep.bias.is_contiguous():
            raise KernelInputError("FP8 GEMM bias must be contiguous bf16 [N]")
        e.bias = ep.bias.data_ptr()
    if ep.kind == _lib.EPI_SWIGLU:
        width = n // 2
        shape = (rows, width)
    elif ep.planes > 1:
        width = n // ep.planes
        shape = (ep.planes, rows, width)
    else:
        width = n
        shape = (rows, n)
    if out is None:
        out = torch.empty(shape, device=device, dtype=BF16)
    elif out.shape != shape or out.dtype != BF16 or not out.is_contiguous():
        raise KernelInputError("FP8 GEMM output buffer has the wrong layout")
    e.out = out.data_ptr()
    e.ldo = width
    if ep.planes > 1 and ep.kind != _lib.EPI_SWIGLU:
        e.plane_width = width
        e.plane_stride = rows * width
    if ep.adapters is not None:
        for i, adapter in enumerate(ep.adapters):
            if adapter is None:
                continue
            if (adapter.dtype != BF16 or adapter.shape != (rows, width) or not adapter.is_contiguous()
                    or adapter.device != device):
                raise KernelInputError("adapters must be contiguous bf16 [rows, plane width]")
            e.adapter[i] = adapter.data_ptr()
        e.adapter_ld = width
        for i, s in enumerate(ep.scalings):
            e.scaling[i] = float(s)
    if ep.kind == _lib.EPI_RESIDUAL:
        r = ep.residual
        if r is None or r.dtype != BF16 or r.shape != (rows, n) or r.stride(1) != 1:
            raise KernelInputError("residual must be bf16 [rows, N] with unit column stride")
        e.residual = r.data_ptr()
        e.ldr = r.stride(0)
        if ep.gate is not None:
            g = ep.gate
            if g.dtype != BF16 or g.ndim != 2 or g.shape[1] != n or ep.tokens <= 0 or g.shape[0] != ep.tokens:
                raise KernelInputError("gate must be bf16 [tokens, N]")
            e.gate = g.data_ptr()
            e.gate_token_stride = g.stride(0)
            e.gate_hidden_stride = g.stride(1)
            e.tokens = ep.tokens
    if rows == 0:
        return out
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.vfb_fp8_gemm(
            a_codes.data_ptr(), a_codes.stride(0), a_scales.data_ptr(), weight.data_ptr(),
            weight.stride(0), w_scales.data_ptr(), rows, n, k, ctypes.byref(e),
            _lib.stream_handle(device))
    _lib.check(rc, "vfb_fp8_gemm")
    return out
