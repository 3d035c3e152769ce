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


def _check_fp8_input(matrix: torch.Tensor) -> tuple[int, int]:
    if matrix.dtype != BF16 or matrix.ndim != 2 or matrix.stride(1) != 1 and matrix.shape[1] > 1:
        raise KernelInputError("FP8 activation quantisation needs a bf16 [M,K] matrix with unit column stride")
    rows, cols = matrix.shape
    if not 1 <= cols <= 32768:
        raise KernelInputError("FP8 activation quantisation needs 1 <= K <= 32768")
    return rows, cols


def quantize_fp8_rows(matrix: torch.Tensor, *, pad_to: int = 16, amax: torch.Tensor | None = None):
    """Per-token e4m3 codes ``[ceil(M/pad_to)*pad_to, K]`` and fp32 scales ``[.., 1]``.

    ``matrix`` is a bf16 ``[M, K]`` CUDA tensor with unit column stride (any
    row stride, e.g. the value half of a packed FFN projection).  ``amax``
    (fp32 ``[M]``) supplies the row maxima instead of computing them — the
    full row's maxima when ``matrix`` is one rank's slice of a split row.
    """
    rows, cols = _check_fp8_input(matrix)
    padded = padded_rows(rows, pad_to)
    codes = torch.empty((padded, cols), device=matrix.device, dtype=FP8)
    scales = torch.empty((padded, 1), device=matrix.device, dtype=torch.float32)
    lib = _lib.load()
    x_ptr = matrix.data_ptr() if rows else None
    ldx = max(matrix.stride(0), cols)
    with torch.cuda.device(matrix.device):
        if amax is None:
            rc = lib.vfb_fp8_quant_rows(x_ptr, rows, cols, ldx, codes.data_ptr(), scales.data_ptr(),
                                        padded, _lib.stream_handle(matrix.device))
        else:
            if (amax.dtype != torch.float32 or amax.numel() != rows or not amax.is_contiguous()
                    or amax.device != matrix.device):
                raise KernelInputError("row maxima must be contiguous fp32 [M] on the input's device")
            rc = lib.vfb_fp8_quant_rows_amax(x_ptr, rows, cols, ldx, amax.data_ptr(), codes.data_ptr(),
                                             scales.data_ptr(), padded, _lib.stream_handle(matrix.device))
    _lib.check(rc, "vfb_fp8_quant_rows")
    return codes, scales


def _check_modifier(t: torch.Tensor, cols: int, device, name: str) -> None:
    if (t.dtype != BF16 or t.ndim != 2 or t.shape[1] != cols or t.stride(1) != 1 or t.device != device
            or t.shape[0] < 1):
        raise KernelInputError(f"{name} must be bf16 [tokens, K] with unit column stride")


def quantize_fp8_norm_modulate(matrix: torch.Tensor, norm_weight: torch.Tensor | None, eps: float,
                               scale: torch.Tensor, shift: torch.Tensor, *, pad_to: int = 16):
    """RMSNorm + AdaLN modulate + per-token e4m3 quantisation of ``matrix`` in one pass.

    ``matrix`` bf16 ``[M, K]`` (unit column stride), ``norm_weight`` bf16
    ``[K]`` or None, ``scale``/``shift`` bf16 ``[tokens, K]`` (row ``r`` of
    ``matrix`` uses row ``r % tokens``; a ``[1, K]`` row serves every token).
    Returns the codes and scales the quantiser would produce for
    ``bf16(bf16(rms_norm(x) * bf16(1 + scale)) + shift)``.
    """
    rows, cols = _check_fp8_input(matrix)
    device = matrix.device
    _check_modifier(scale, cols, device, "modulate scale")
    _check_modifier(shift, cols, device, "modulate shift")
    tokens = scale.shape[0]
    if shift.shape[0] != tokens:
        raise KernelInputError("modulate scale and shift cover different token counts")
    if norm_weight is not None and (norm_weight.dtype != BF16 or norm_weight.shape != (cols,)
                                    or not norm_weight.is_contiguous() or norm_weight.device != device):
        raise KernelInputError("norm weight must be contiguous bf16 [K]")
    padded = padded_rows(rows, pad_to)
    codes = torch.empty((padded, cols), device=device, dtype=FP8)
    scales = torch.empty((padded, 1), device=device, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.vfb_fp8_norm_modulate_quant(
            matrix.data_ptr() if rows else None, rows, cols, max(matrix.stride(0), cols),
            None if norm_weight is None else norm_weight.data_ptr(), float(eps), scale.data_ptr(),
            scale.stride(0) if tokens > 1 else 0, shift.data_ptr(), shift.stride(0) if tokens > 1 else 0,
            tokens, codes.data_ptr(), scales.data_ptr(), padded, _lib.stream_handle(device))
    _lib.check(rc, "vfb_fp8_norm_modulate_quant")
    return codes, scales


def row_absmax(matrix: torch.Tensor) -> torch.Tensor:
    """fp32 ``[M]`` row maxima of |x| (NaN for rows holding a NaN), as the quantiser computes them."""
    rows, cols = _check_fp8_input(matrix)
    amax = torch.empty(rows, device=matrix.device, dtype=torch.float32)
    if rows == 0:
        return amax
    lib = _lib.load()
    with torch.cuda.device(matrix.device):
        rc = lib.vfb_fp8_row_absmax(matrix.data_ptr(), rows, cols, max(matrix.stride(0), cols),
                                    amax.data_ptr(), _lib.stream_handle(matrix.device))
    _lib.check(rc, "vfb_fp8_row_absmax")
    return amax


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
    # QKV_NORM_ROPE (planes = 3, 128-column heads, rotary over the whole head)
    q_norm: torch.Tensor | None = None   # bf16 [128] or None
    k_norm: torch.Tensor | None = None   # bf16 [128] or None
    rope_cos: torch.Tensor | None = None # bf16 [tokens, 128], unit column stride
    rope_sin: torch.Tensor | None = None # bf16 [tokens, 128], same layout as rope_cos
    qk_eps: float = 1e-5
    # STORE / QKV_NORM_ROPE with planes = 3: store the planes in pack_qkv's
    # (chunks, 2, 3, rows, plane width / (2 * chunks)) wire layout instead
    wire_chunks: int = 0


def _build_epilogue(ep: Epilogue, rows: int, n: int, device, out: torch.Tensor | None):
    """The ``vfb_epilogue`` of ``ep`` for a GEMM with ``rows`` x ``n`` outputs, and its output tensor."""
    e = _lib.Epilogue()
    e.kind = ep.kind
    if ep.bias is not None:
        if ep.bias.dtype != BF16 or ep.bias.shape != (n,) or not ep.bias.is_contiguous():
            raise KernelInputError("FP8 GEMM bias must be contiguous bf16 [N]")
        e.bias = ep.bias.data_ptr()
    if ep.kind == _lib.EPI_SWIGLU:
        width = n // 2
        shape = (rows, width)
    elif ep.wire_chunks:
        c = ep.wire_chunks
        if (ep.kind not in (_lib.EPI_STORE, _lib.EPI_QKV_NORM_ROPE) or ep.planes != 3 or c < 0
                or (n // 3) % (2 * c) or (n // 3 // (2 * c)) % 32):
            raise KernelInputError("the wire layout splits three planes into 2 * chunks groups of 32k columns")
        width = n // 3
        shape = (c, 2, 3, rows, width // (2 * c))
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
    if ep.wire_chunks:
        e.wire_chunks = ep.wire_chunks
        e.ldo = shape[-1]
        e.plane_stride = rows * shape[-1]
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
    if ep.kind == _lib.EPI_QKV_NORM_ROPE:
        cos, sin = ep.rope_cos, ep.rope_sin
        if (cos is None or sin is None or cos.dtype != BF16 or sin.dtype != BF16 or cos.ndim != 2
                or cos.shape != sin.shape or cos.shape[1] != 128 or cos.stride(1) != 1 or sin.stride(1) != 1
                or cos.stride(0) != sin.stride(0) or cos.device != device or sin.device != device):
            raise KernelInputError("rotary cos/sin must be bf16 [tokens, 128] with one row stride")
        for name, w in (("q_norm", ep.q_norm), ("k_norm", ep.k_norm)):
            if w is not None and (w.dtype != BF16 or w.shape != (128,) or not w.is_contiguous()
                                  or w.device != device):
                raise KernelInputError(f"{name} must be contiguous bf16 [128]")
        if ep.planes != 3:
            raise KernelInputError("QK-norm + rotary writes the three Q, K, V planes")
        tokens = cos.shape[0]
        e.q_norm = None if ep.q_norm is None else ep.q_norm.data_ptr()
        e.k_norm = None if ep.k_norm is None else ep.k_norm.data_ptr()
        e.rope_cos = cos.data_ptr()
        e.rope_sin = sin.data_ptr()
        e.rope_token_stride = cos.stride(0) if tokens > 1 else 0
        e.qk_eps = float(ep.qk_eps)
        e.tokens = tokens
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
    return e, out


def fp8_gemm(a_codes: torch.Tensor, a_scales: torch.Tensor, rows: int, weight: torch.Tensor,
             w_scales: torch.Tensor, epilogue: Epilogue | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-scaled e4m3 GEMM ``bf16(sa * sw * A @ W^T)`` with a fused epilogue.

    ``a_codes`` e4m3 ``[>=rows, K]``, ``a_scales`` fp32 (>= rows entries),
    ``weight`` e4m3 ``[N, K]`` row-major, ``w_scales`` fp32 ``[N, 1]``.
    Returns bf16 ``[rows, N]`` (``[rows, N/2]`` for SWIGLU, ``[planes, rows,
    N/planes]`` when the output is split into planes, ``[chunks, 2, 3, rows,
    N/(6 chunks)]`` in the wire layout).
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

    e, out = _build_epilogue(ep, rows, n, device, out)
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


# ---------------------------------------------------------------------------
# NVFP4
# ---------------------------------------------------------------------------
def nvfp4_sf_shape(rows: int, cols: int) -> tuple[int, int]:
    """Padded 128x4 scale-factor shape for a [rows, cols] input: (ceil128(rows), ceil4(cols/16))."""
    return (-(-rows // 128) * 128, -(-(cols // 16) // 4) * 4)


def _ffn_operands(rows, hidden, device, up, up_scales, down, down_scales, activation, up_bias, down_bias,
                  residual, gate):
    n_up = up.shape[0]
    width = n_up // 2 if activation == _lib.EPI_SWIGLU else n_up
    if (up.dtype != FP8 or down.dtype != FP8 or up.ndim != 2 or up.shape[1] != hidden
            or down.shape != (hidden, width) or not up.is_contiguous() or not down.is_contiguous()
            or up_scales.numel() != n_up or down_scales.numel() != hidden
            or up_scales.dtype != torch.float32 or down_scales.dtype != torch.float32
            or not up_scales.is_contiguous() or not down_scales.is_contiguous()):
        raise KernelInputError("FP8 FFN operands differ from the declared layouts")
    for t in (up, down, up_scales, down_scales, up_bias, down_bias, residual, gate):
        if t is not None and t.device != device:
            raise KernelInputError("FP8 FFN operands must share one device")
    for name, b, n in (("up", up_bias, n_up), ("down", down_bias, hidden)):
        if b is not None and (b.dtype != BF16 or b.shape != (n,) or not b.is_contiguous()):
            raise KernelInputError(f"FP8 FFN {name} bias must be contiguous bf16 [{n}]")
    if residual is not None and (residual.dtype != BF16 or residual.shape != (rows, hidden)
                                 or residual.stride(1) != 1):
        raise KernelInputError("FP8 FFN residual must be bf16 [M, H] with unit column stride")
    if gate is not None and (gate.dtype != BF16 or gate.ndim != 2 or gate.shape[1] != hidden
                             or gate.stride(1) != 1):
        raise KernelInputError("FP8 FFN gate must be bf16 [tokens, H] with unit column stride")
    lib = _lib.load()
    need = lib.vfb_fp8_ffn_workspace_bytes(rows, hidden, width)
    if need < 0:
        raise KernelInputError("FP8 FFN shape is outside the supported range")
    workspace = torch.empty(need + 256, device=device, dtype=torch.uint8)
    base = workspace.data_ptr() + (-workspace.data_ptr()) % 256
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    tail = [up.data_ptr(), up_scales.data_ptr(), n_up, down.data_ptr(), down_scales.data_ptr(), activation,
            ptr(up_bias), ptr(down_bias), ptr(residual), 0 if residual is None else residual.stride(0),
            ptr(gate), 0 if gate is None else gate.stride(0), 0 if gate is None else gate.shape[0]]
    return lib, need, workspace, base, tail


def fp8_ffn(x: torch.Tensor, up: torch.Tensor, up_scales: torch.Tensor, down: torch.Tensor,
            down_scales: torch.Tensor, *, activation: int = _lib.EPI_GELU_TANH, up_bias=None, down_bias=None,
            residual=None, gate=None, one_kernel: bool = False) -> torch.Tensor:
    """The whole FP8 FFN through ``vfb_fp8_ffn`` (one C call, workspace from torch's allocator).

    ``x`` bf16 ``[M, H]`` (unit column stride), ``up`` e4m3 ``[F or 2F, H]``,
    ``down`` e4m3 ``[H, F]``, scales fp32 ``[N, 1]``; ``residual`` bf16
    ``[M, H]`` and ``gate`` bf16 ``[tokens, H]`` as the down GEMM's RESIDUAL
    epilogue.  ``one_kernel`` selects ``vfb_fp8_ffn_one_kernel`` (the same
    bits from one persistent launch).  Returns bf16 ``[M, H]``.
    """
    if x.dtype != BF16 or x.ndim != 2 or x.stride(1) != 1:
        raise KernelInputError("FP8 FFN input must be bf16 [M, H] with unit column stride")
    rows, hidden = x.shape
    device = x.device
    lib, need, workspace, base, tail = _ffn_operands(rows, hidden, device, up, up_scales, down, down_scales,
                                                     activation, up_bias, down_bias, residual, gate)
    out = torch.empty((rows, hidden), device=device, dtype=BF16)
    entry = lib.vfb_fp8_ffn_one_kernel if one_kernel else lib.vfb_fp8_ffn
    with torch.cuda.device(device):
        rc = entry(x.data_ptr(), rows, hidden, x.stride(0), *tail, out.data_ptr(), hidden, base, need,
                   _lib.stream_handle(device))
    _lib.check(rc, "vfb_fp8_ffn_one_kernel" if one_kernel else "vfb_fp8_ffn")
    return out


def fp8_ffn_quantized(codes: torch.Tensor, scales: torch.Tensor, rows: int, up: torch.Tensor,
                      up_scales: torch.Tensor, down: torch.Tensor, down_scales: torch.Tensor, *,
                      activation: int = _lib.EPI_GELU_TANH, up_bias=None, down_bias=None, residual=None,
                      gate=None) -> torch.Tensor:
    """``fp8_ffn`` on an input already quantised per token (``vfb_fp8_ffn_quantized``).

    ``codes`` e4m3 ``[>= rows, H]`` contiguous and ``scales`` fp32 (``>= rows``
    entries), e.g. from ``quantize_fp8_norm_modulate``.
    """
    if (codes.dtype != FP8 or codes.ndim != 2 or not codes.is_contiguous() or codes.shape[0] < rows
            or scales.dtype != torch.float32 or not scales.is_contiguous() or scales.numel() < rows
            or scales.device != codes.device):
        raise KernelInputError("FP8 FFN codes must be contiguous e4m3 [>= M, H] with fp32 scales")
    hidden = codes.shape[1]
    device = codes.device
    lib, need, workspace, base, tail = _ffn_operands(rows, hidden, device, up, up_scales, down, down_scales,
                                                     activation, up_bias, down_bias, residual, gate)
    out = torch.empty((rows, hidden), device=device, dtype=BF16)
    if rows == 0:
        return out
    with torch.cuda.device(device):
        rc = lib.vfb_fp8_ffn_quantized(codes.data_ptr(), scales.data_ptr(), rows, hidden, *tail, out.data_ptr(),
                                       hidden, base, need, _lib.stream_handle(device))
    _lib.check(rc, "vfb_fp8_ffn_quantized")
    return out


def bf16_gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``bf16(a @ w^T)``: bias-free ``functional.linear`` in bf16 on the tcgen05 pipeline.

    ``a`` bf16 ``[M, K]`` and ``w`` bf16 ``[N, K]``, unit column stride, row
    strides multiples of 8, 16-byte aligned; K % 8 == 0, N % 8 == 0.  ``out``
    (bf16 ``[M, N]``, unit column stride) may be a strided view, e.g. a
    column slice of a wider buffer.
    """
    if (a.dtype != BF16 or w.dtype != BF16 or a.ndim != 2 or w.ndim != 2 or a.shape[1] != w.shape[1]
            or a.stride(1) != 1 or w.stride(1) != 1 or a.device != w.device):
        raise KernelInputError("bf16 GEMM operands must be bf16 [M,K] and [N,K] with unit column stride")
    rows, k = a.shape
    n = w.shape[0]
    if k % 8 or n % 8 or a.stride(0) % 8 or w.stride(0) % 8 or not (_aligned(a) and _aligned(w)):
        raise KernelInputError("bf16 GEMM needs K % 8 == 0, N % 8 == 0 and 16-byte aligned rows")
    e = _lib.Epilogue()
    e.kind = _lib.EPI_STORE
    if out is None:
        out = torch.empty((rows, n), device=a.device, dtype=BF16)
    elif (out.dtype != BF16 or out.shape != (rows, n) or out.stride(1) != 1 or out.stride(0) % 8
          or not _aligned(out) or out.device != a.device):
        raise KernelInputError("bf16 GEMM output must be bf16 [M, N], unit column stride, aligned rows")
    e.out = out.data_ptr()
    e.ldo = out.stride(0)
    if rows == 0:
        return out
    lib = _lib.load()
    with torch.cuda.device(a.device):
        rc = lib.vfb_bf16_gemm(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), rows, n, k,
                               ctypes.byref(e), _lib.stream_handle(a.device))
    _lib.check(rc, "vfb_bf16_gemm")
    return out


def nvfp4_quantize(matrix: torch.Tensor, global_scale: torch.Tensor):
    """e2m1 codes ``[M, K/2]`` (uint8) and 128x4 ue4m3 scales ``[ceil128(M), ceil4(K/16)]`` (uint8).

    ``matrix`` is bf16 or fp16 ``[M, K]`` with unit column stride and K % 16 == 0;
    ``global_scale`` an fp32 scalar tensor on the same device.
    """
    if (matrix.dtype not in (BF16, torch.float16) or matrix.ndim != 2 or matrix.stride(1) != 1
            or matrix.shape[1] % 16):
        raise KernelInputError("NVFP4 quantisation needs a bf16/fp16 [M,K] matrix, K % 16 == 0")
    if (global_scale.dtype != torch.float32 or global_scale.numel() != 1
            or global_scale.device != matrix.device):
        raise KernelInputError("NVFP4 global scale must be an fp32 scalar on the input's device")
    rows, cols = matrix.shape
    codes = torch.empty((rows, cols // 2), device=matrix.device, dtype=torch.uint8)
    sf = torch.empty(nvfp4_sf_shape(rows, cols), device=matrix.device, dtype=torch.uint8)
    if rows == 0:
        return codes, sf
    lib = _lib.load()
    with torch.cuda.device(matrix.device):
        rc = lib.vfb_nvfp4_quant_rows(matrix.data_ptr(), 0 if matrix.dtype == BF16 else 1, rows, cols,
                                      matrix.stride(0), global_scale.data_ptr(), codes.data_ptr(),
                                      sf.data_ptr(), _lib.stream_handle(matrix.device))
    _lib.check(rc, "vfb_nvfp4_quant_rows")
    return codes, sf


def nvfp4_norm_modulate_quantize(matrix: torch.Tensor, norm_weight: torch.Tensor | None, eps: float,
                                 scale: torch.Tensor, shift: torch.Tensor, global_scale: torch.Tensor):
    """RMSNorm + AdaLN modulate + NVFP4 quantisation of ``matrix`` in one pass.

    The operands are those of ``quantize_fp8_norm_modulate``; ``global_scale``
    is the NVFP4 linear's input scale.  Returns what
    ``nvfp4_quantize(bf16(bf16(rms_norm(x) * bf16(1 + scale)) + shift),
    global_scale)`` returns; K % 64 == 0.
    """
    rows, cols = _check_fp8_input(matrix)
    device = matrix.device
    if cols % 64:
        raise KernelInputError("the NVFP4 prologue needs K % 64 == 0")
    _check_modifier(scale, cols, device, "modulate scale")
    _check_modifier(shift, cols, device, "modulate shift")
    tokens = scale.shape[0]
    if shift.shape[0] != tokens:
        raise KernelInputError("modulate scale and shift cover different token counts")
    if norm_weight is not None and (norm_weight.dtype != BF16 or norm_weight.shape != (cols,)
                                    or not norm_weight.is_contiguous() or norm_weight.device != device):
        raise KernelInputError("norm weight must be contiguous bf16 [K]")
    if (global_scale.dtype != torch.float32 or global_scale.numel() != 1 or global_scale.device != device):
        raise KernelInputError("NVFP4 global scale must be an fp32 scalar on the input's device")
    codes = torch.empty((rows, cols // 2), device=device, dtype=torch.uint8)
    sf = torch.empty(nvfp4_sf_shape(rows, cols), device=device, dtype=torch.uint8)
    if rows == 0:
        return codes, sf
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.vfb_nvfp4_norm_modulate_quant(
            matrix.data_ptr(), rows, cols, max(matrix.stride(0), cols),
            None if norm_weight is None else norm_weight.data_ptr(), float(eps), scale.data_ptr(),
            scale.stride(0) if tokens > 1 else 0, shift.data_ptr(), shift.stride(0) if tokens > 1 else 0,
            tokens, global_scale.data_ptr(), codes.data_ptr(), sf.data_ptr(), _lib.stream_handle(device))
    _lib.check(rc, "vfb_nvfp4_norm_modulate_quant")
    return codes, sf


def nvfp4_gemm(a_codes: torch.Tensor, a_sf: torch.Tensor, w_packed: torch.Tensor,
               w_scales: torch.Tensor, alpha: torch.Tensor, bias: torch.Tensor | None = None,
               planes: int = 1, *, alpha_div: torch.Tensor | None = None,
               epilogue: Epilogue | None = None, quantize_output: torch.Tensor | None = None):
    """``bf16(alpha * A @ W^T)`` (+ bias, + epilogue) for NVFP4 operands in the 128x4 scale layout.

    ``alpha`` (and ``alpha_div``, when given: the GEMM uses ``alpha / alpha_div``
    computed on the device) are fp32 scalar tensors.  ``epilogue`` selects the
    fused step after the bias (``Epilogue`` kinds STORE with planes and LoRA
    adapters, GELU_TANH, SWIGLU over the packed ``[2F, K/2]`` weight, or
    RESIDUAL); ``bias`` / ``planes`` are the plain-store shorthand.

    ``quantize_output`` (an fp32 scalar tensor, the next NVFP4 linear's input
    scale) returns the result as ``nvfp4_quantize(result, quantize_output)``
    would, bit for bit, without the bf16 tensor: ``(codes, scales)`` from
    ``vfb_nvfp4_gemm_quant`` (STORE with one plane, GELU_TANH or SWIGLU).
    """
    rows, half_k = a_codes.shape
    n = w_packed.shape[0]
    k = 2 * half_k
    if (a_codes.dtype != torch.uint8 or w_packed.dtype != torch.uint8 or w_packed.shape[1] != half_k
            or not a_codes.is_contiguous() or not w_packed.is_contiguous()):
        raise KernelInputError("NVFP4 GEMM codes must be contiguous uint8 [M,K/2] and [N,K/2]")
    ep = epilogue or Epilogue(bias=bias, planes=planes)
    if epilogue is not None and (bias is not None or planes != 1):
        raise KernelInputError("pass bias and planes inside the epilogue")
    if k % 64 or n % 128 or n % ep.planes or (n // ep.planes) % 32:
        raise KernelInputError("NVFP4 GEMM needs K % 64 == 0, N % 128 == 0")
    if ep.kind == _lib.EPI_SWIGLU and (n // 2) % 128:
        raise KernelInputError("NVFP4 SwiGLU needs the packed [2F, K/2] weight with F % 128 == 0")
    if ep.kind == _lib.EPI_QKV_NORM_ROPE or ep.wire_chunks:
        raise KernelInputError("NVFP4 GEMM has no QK-norm or wire-layout epilogue")
    pr, pc = nvfp4_sf_shape(rows, k)
    if (a_sf.dtype != torch.uint8 or a_sf.numel() != pr * pc or not a_sf.is_contiguous()
            or w_scales.dtype != torch.uint8 or w_scales.numel() != n * (k // 16)
            or not w_scales.is_contiguous()):
        raise KernelInputError("NVFP4 GEMM scales differ from the 128x4 layout")
    for name, scalar in (("alpha", alpha), ("alpha_div", alpha_div)):
        if scalar is not None and (scalar.dtype != torch.float32 or scalar.numel() != 1):
            raise KernelInputError(f"NVFP4 GEMM {name} must be an fp32 scalar tensor")
    device = a_codes.device
    for t in (a_sf, w_packed, w_scales, alpha, alpha_div):
        if t is not None and t.device != device:
            raise KernelInputError("NVFP4 GEMM operands must share one device")
    if quantize_output is not None:
        return _nvfp4_gemm_quant(a_codes, a_sf, w_packed, w_scales, alpha, alpha_div, ep, quantize_output)
    e, out = _build_epilogue(ep, rows, n, device, None)
    if rows == 0:
        return out
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.vfb_nvfp4_gemm_ex(a_codes.data_ptr(), a_sf.data_ptr(), w_packed.data_ptr(), w_scales.data_ptr(),
                                   alpha.data_ptr(), None if alpha_div is None else alpha_div.data_ptr(), rows, n,
                                   k, ctypes.byref(e), _lib.stream_handle(device))
    _lib.check(rc, "vfb_nvfp4_gemm_ex")
    return out


def _nvfp4_gemm_quant(a_codes, a_sf, w_packed, w_scales, alpha, alpha_div, ep: Epilogue, global_scale):
    """``nvfp4_gemm`` whose result leaves the kernel as NVFP4 codes and 128x4 scales."""
    rows, half_k = a_codes.shape
    n = w_packed.shape[0]
    device = a_codes.device
    if ep.kind not in (_lib.EPI_STORE, _lib.EPI_GELU_TANH, _lib.EPI_SWIGLU) or ep.planes != 1 or ep.adapters:
        raise KernelInputError("the NVFP4 output needs a STORE, GELU_TANH or SWIGLU epilogue with one plane")
    width = n // 2 if ep.kind == _lib.EPI_SWIGLU else n
    if width % 64:
        raise KernelInputError("the NVFP4 output width must be a multiple of 64")
    if (global_scale.dtype != torch.float32 or global_scale.numel() != 1 or global_scale.device != device):
        raise KernelInputError("NVFP4 global scale must be an fp32 scalar on the GEMM's device")
    e = _lib.Epilogue()
    e.kind = ep.kind
    if ep.bias is not None:
        if ep.bias.dtype != BF16 or ep.bias.shape != (n,) or not ep.bias.is_contiguous():
            raise KernelInputError("NVFP4 GEMM bias must be contiguous bf16 [N]")
        e.bias = ep.bias.data_ptr()
    codes = torch.empty((rows, width // 2), device=device, dtype=torch.uint8)
    sf = torch.empty(nvfp4_sf_shape(rows, width), device=device, dtype=torch.uint8)
    if rows == 0:
        return codes, sf
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.vfb_nvfp4_gemm_quant(a_codes.data_ptr(), a_sf.data_ptr(), w_packed.data_ptr(), w_scales.data_ptr(),
                                      alpha.data_ptr(), None if alpha_div is None else alpha_div.data_ptr(), rows, n,
                                      2 * half_k, ctypes.byref(e), global_scale.data_ptr(), codes.data_ptr(),
                                      sf.data_ptr(), _lib.stream_handle(device))
    _lib.check(rc, "vfb_nvfp4_gemm_quant")
    return codes, sf
