"""Strict-BF16 elementwise steps of the H3 block on SM100 (drop-in).

Mirrors the public functions of Hansimov/vflash's
src/vflash/native/h3_fused_ops.py — same names (the ``triton_`` prefix is
kept so existing callers need no change), signatures, validation order,
``H3FusedOpsError`` messages and BF16 rounding boundaries — with every launch
going to the native library (``vfb_*`` entry points of
include/vflash_b200.h).  Validation never touches a device, so CPU tensors
are rejected without initialising CUDA, as in the reference.

``block_size`` is accepted and validated for compatibility; the native
kernels size their own launches.  The contiguous last dimension must be a
multiple of 8 (every H3 width is).

The same arithmetic is also available fused into the FP8 GEMM epilogue
(``RowFP8Execution.qkv_linear`` / ``swiglu_linear`` / ``gate_residual_linear``),
which removes the extra HBM pass these standalone launches make.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

from .. import _lib


class H3FusedOpsError(ValueError):
    """A fused H3 invocation violates the fixed CUDA/BF16 contract."""


_BLOCK_SIZES = frozenset({128, 256, 512, 1024})


def _torch():
    try:
        import torch
    except ImportError as exc:  # pragma: no cover - runtime image contract
        raise H3FusedOpsError("the fused H3 backend requires PyTorch") from exc
    return torch


def _require_launchable(*tensors: Any) -> None:
    """Device and width gate applied after the reference's own validation."""
    torch = _torch()
    device = tensors[0].device
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise H3FusedOpsError("the fused H3 kernels require an SM100 (B200) CUDA device")
    for tensor in tensors:
        if tensor.shape[-1] % 8:
            raise H3FusedOpsError("the fused H3 kernels need a last dimension divisible by 8")


def _stream(device) -> int:
    return _lib.stream_handle(device)


def _validate_common(value: Any, modifier: Any, *, modifier_name: str, block_size: int) -> tuple[int, int, int]:
    torch = _torch()
    if block_size not in _BLOCK_SIZES:
        raise H3FusedOpsError(f"unsupported fused H3 block size: {block_size}")
    if not isinstance(value, torch.Tensor) or not isinstance(modifier, torch.Tensor):
        raise H3FusedOpsError("fused H3 inputs must be tensors")
    if value.device.type != "cuda" or modifier.device != value.device:
        raise H3FusedOpsError("fused H3 inputs must share one CUDA device")
    if value.dtype != torch.bfloat16 or modifier.dtype != torch.bfloat16:
        raise H3FusedOpsError("fused H3 inputs must use BF16")
    if value.ndim != 3 or modifier.ndim != 2:
        raise H3FusedOpsError(f"fused H3 value must be [B,S,H] and {modifier_name} must be [S,H]")
    batch, tokens, hidden_size = (int(item) for item in value.shape)
    if tuple(modifier.shape) != (tokens, hidden_size):
        raise H3FusedOpsError(f"fused H3 {modifier_name} shape differs from the activation")
    if not value.is_contiguous() or modifier.stride(-1) != 1:
        raise H3FusedOpsError("fused H3 activations require a contiguous hidden dimension")
    return batch, tokens, hidden_size


def _validate_matching_activation(value: Any, candidate: Any, *, candidate_name: str,
                                  block_size: int) -> tuple[int, int, int]:
    torch = _torch()
    if block_size not in _BLOCK_SIZES:
        raise H3FusedOpsError(f"unsupported fused H3 block size: {block_size}")
    if not isinstance(value, torch.Tensor) or not isinstance(candidate, torch.Tensor):
        raise H3FusedOpsError("fused H3 inputs must be tensors")
    if value.device.type != "cuda" or candidate.device != value.device:
        raise H3FusedOpsError("fused H3 inputs must share one CUDA device")
    if value.dtype != torch.bfloat16 or candidate.dtype != torch.bfloat16:
        raise H3FusedOpsError("fused H3 inputs must use BF16")
    if value.ndim != 3 or tuple(candidate.shape) != tuple(value.shape):
        raise H3FusedOpsError(f"fused H3 {candidate_name} must match the [B,S,H] activation")
    if not value.is_contiguous() or not candidate.is_contiguous():
        raise H3FusedOpsError("fused H3 activations must be contiguous")
    return tuple(int(item) for item in value.shape)


def _validate_scalings(scalings: tuple[float, ...], expected: int) -> tuple[float, ...]:
    if len(scalings) != expected or any(not math.isfinite(value) for value in scalings):
        raise H3FusedOpsError(f"fused H3 adapter requires {expected} finite scalings")
    return tuple(float(value) for value in scalings)


def _check(rc: int, what: str) -> None:
    if rc != _lib.VFB_OK:
        raise H3FusedOpsError(f"{what} failed: {_lib.last_error()}")


def triton_strict_bf16_gate_residual(residual: Any, gate: Any, projected: Any, *,
                                     block_size: int = 256) -> Any:
    """Compute ``residual + gate * projected`` with eager BF16 rounding."""
    batch, tokens, hidden_size = _validate_common(residual, gate, modifier_name="gate",
                                                  block_size=block_size)
    torch = _torch()
    if (
        not isinstance(projected, torch.Tensor)
        or projected.device != residual.device
        or projected.dtype != torch.bfloat16
        or tuple(projected.shape) != tuple(residual.shape)
        or not projected.is_contiguous()
    ):
        raise H3FusedOpsError("fused H3 projected activation differs from the residual")
    _require_launchable(residual)
    output = torch.empty_like(residual)
    with torch.cuda.device(residual.device):
        rc = _lib.load().vfb_gate_residual(
            residual.data_ptr(), gate.data_ptr(), gate.stride(0), projected.data_ptr(),
            batch * tokens, tokens, hidden_size, output.data_ptr(), _stream(residual.device))
    _check(rc, "vfb_gate_residual")
    return output


def triton_strict_bf16_modulate(value: Any, scale: Any, shift: Any, *, block_size: int = 256) -> Any:
    """Compute ``value * (1 + scale) + shift`` with eager BF16 rounding.

    Replaces src/vflash/native/h3_fused_ops.py:575-611 (kernel 52-122):
    ``bf16(bf16(value * bf16(1 + scale)) + shift)``, scale and shift ``[S,H]``
    indexed per token.
    """
    batch, tokens, hidden_size = _validate_common(value, scale, modifier_name="scale",
                                                  block_size=block_size)
    _validate_common(value, shift, modifier_name="shift", block_size=block_size)
    torch = _torch()
    _require_launchable(value)
    output = torch.empty_like(value)
    with torch.cuda.device(value.device):
        rc = _lib.load().vfb_modulate(
            value.data_ptr(), scale.data_ptr(), scale.stride(0), shift.data_ptr(), shift.stride(0),
            batch * tokens, tokens, hidden_size, output.data_ptr(), _stream(value.device))
    _check(rc, "vfb_modulate")
    return output


def triton_strict_bf16_rotary(value: Any, cos: Any, sin: Any, *, block_size: int = 256) -> Any:
    """Apply H3 split-half RoPE while preserving eager BF16 products.

    Replaces src/vflash/native/h3_fused_ops.py:1031-1085 (kernel 421-510):
    value ``[B,S,heads,head_dim]``, cos/sin ``[S,rotary_dim]``.
    """
    torch = _torch()
    if block_size not in _BLOCK_SIZES:
        raise H3FusedOpsError(f"unsupported fused H3 block size: {block_size}")
    if not all(isinstance(item, torch.Tensor) for item in (value, cos, sin)):
        raise H3FusedOpsError("fused H3 rotary inputs must be tensors")
    if value.device.type != "cuda" or cos.device != value.device or sin.device != value.device:
        raise H3FusedOpsError("fused H3 rotary inputs must share one CUDA device")
    if value.dtype != torch.bfloat16 or cos.dtype != value.dtype or sin.dtype != value.dtype:
        raise H3FusedOpsError("fused H3 rotary inputs must use BF16")
    if value.ndim != 4 or cos.ndim != 2 or tuple(sin.shape) != tuple(cos.shape):
        raise H3FusedOpsError("fused H3 rotary shapes are invalid")
    batch, tokens, heads, head_dim = (int(item) for item in value.shape)
    rotary_dim = int(cos.shape[1])
    if int(cos.shape[0]) != tokens or rotary_dim <= 0 or rotary_dim > head_dim or rotary_dim % 2:
        raise H3FusedOpsError("fused H3 rotary dimension is invalid")
    if not value.is_contiguous() or cos.stride(-1) != 1 or sin.stride(-1) != 1:
        raise H3FusedOpsError("fused H3 rotary inputs require contiguous hidden dimensions")
    _require_launchable(value)
    output = torch.empty_like(value)
    with torch.cuda.device(value.device):
        rc = _lib.load().vfb_rotary(
            value.data_ptr(), cos.data_ptr(), cos.stride(0), sin.data_ptr(), sin.stride(0), batch * tokens,
            tokens, heads, head_dim, rotary_dim, output.data_ptr(), _stream(value.device))
    _check(rc, "vfb_rotary")
    return output


def triton_strict_bf16_silu_mul(packed: Any, *, block_size: int = 256) -> Any:
    """Fuse H3 ``value * silu(gate)`` while retaining the eager BF16 round."""
    torch = _torch()
    if block_size not in _BLOCK_SIZES:
        raise H3FusedOpsError(f"unsupported fused H3 block size: {block_size}")
    if (
        not isinstance(packed, torch.Tensor)
        or packed.device.type != "cuda"
        or packed.dtype != torch.bfloat16
        or packed.ndim != 3
        or int(packed.shape[-1]) % 2
        or not packed.is_contiguous()
    ):
        raise H3FusedOpsError("fused H3 SiLU/mul requires contiguous CUDA BF16 [B,S,2H] input")
    hidden_size = int(packed.shape[-1]) // 2
    if hidden_size <= 0:
        raise H3FusedOpsError("fused H3 SiLU/mul hidden size must be positive")
    output = torch.empty((*packed.shape[:-1], hidden_size), device=packed.device, dtype=packed.dtype)
    _require_launchable(output)
    rows = output.numel() // hidden_size
    with torch.cuda.device(packed.device):
        rc = _lib.load().vfb_silu_mul(packed.data_ptr(), rows, hidden_size, output.data_ptr(),
                                      hidden_size, _stream(packed.device))
    _check(rc, "vfb_silu_mul")
    return output


def triton_strict_bf16_ffn_adapter_silu(base: Any, adapter: Any, *, scaling: float, block_size: int,
                                        reuse_base: bool = False) -> Any:
    """Merge the FFN adapter and SiLU without a merged [B,S,2F] temporary.

    The separate BF16 LoRA product, addition and SiLU round boundaries remain
    explicit.  ``reuse_base`` transfers ownership of a fresh base projection to
    the result: only its value half is overwritten, returning a strided view.
    """
    torch = _torch()
    if (
        not isinstance(base, torch.Tensor)
        or not isinstance(adapter, torch.Tensor)
        or base.device.type != "cuda"
        or adapter.device != base.device
        or base.dtype != torch.bfloat16
        or adapter.dtype != base.dtype
        or base.ndim != 3
        or tuple(adapter.shape) != tuple(base.shape)
        or not base.is_contiguous()
        or not adapter.is_contiguous()
        or any(size <= 0 for size in base.shape)
        or base.shape[-1] % 2
    ):
        raise H3FusedOpsError("FFN fusion requires matching contiguous CUDA BF16 [B,S,2F]")
    if (
        not isinstance(scaling, (float, int))
        or isinstance(scaling, bool)
        or not math.isfinite(scaling)
        or block_size != 1024
    ):
        raise H3FusedOpsError("FFN fusion requires finite scaling and block size 1024")
    if type(reuse_base) is not bool or (reuse_base and (base.requires_grad or adapter.requires_grad)):
        raise H3FusedOpsError("owned FFN reuse requires an inference-only boolean contract")
    width = base.shape[-1] // 2
    output = (
        base[..., :width]
        if reuse_base
        else torch.empty((*base.shape[:-1], width), device=base.device, dtype=base.dtype)
    )
    _require_launchable(base[..., :width])
    rows = base.numel() // base.shape[-1]
    out_ld = 2 * width if reuse_base else width
    with torch.cuda.device(base.device):
        rc = _lib.load().vfb_ffn_adapter_silu(base.data_ptr(), adapter.data_ptr(), rows, width,
                                              float(scaling), output.data_ptr(), out_ld,
                                              _stream(base.device))
    _check(rc, "vfb_ffn_adapter_silu")
    return output


def _merge(base, adapter, scalings, branches: int) -> Any:
    torch = _torch()
    output = torch.empty_like(base)
    _require_launchable(base)
    values = (ctypes.c_float * 3)(*(list(scalings) + [0.0] * (3 - len(scalings))))
    width = base.shape[-1]
    with torch.cuda.device(base.device):
        rc = _lib.load().vfb_adapter_merge(base.data_ptr(), adapter.data_ptr(),
                                           base.numel() // width, width, branches, values,
                                           output.data_ptr(), _stream(base.device))
    _check(rc, "vfb_adapter_merge")
    return output


def triton_strict_bf16_adapter_merge(base: Any, adapter: Any, *, scaling: float,
                                     block_size: int = 256) -> Any:
    """Fuse LoRA scaling and base addition with official BF16 boundaries."""
    _validate_matching_activation(base, adapter, candidate_name="adapter", block_size=block_size)
    (scaling,) = _validate_scalings((scaling,), 1)
    return _merge(base, adapter, (scaling,), 1)


def triton_strict_bf16_qkv_adapter_merge(base: Any, concatenated_adapter: Any, *,
                                         scalings: tuple[float, float, float],
                                         block_size: int = 256) -> Any:
    """Fuse three Q/K/V LoRA scaling/add branches after one contiguous pack."""
    _batch, _tokens, hidden_size = _validate_matching_activation(
        base, concatenated_adapter, candidate_name="concatenated QKV adapter", block_size=block_size)
    if hidden_size % 3:
        raise H3FusedOpsError("fused H3 QKV hidden size must be divisible by three")
    scales = _validate_scalings(scalings, 3)
    return _merge(base, concatenated_adapter, scales, 3)


def _shares_storage(left: Any, right: Any) -> bool:
    return left.untyped_storage().data_ptr() == right.untyped_storage().data_ptr()


def _validate_qkv_direct_merge(base: Any, adapters: tuple[Any, Any, Any],
                               scalings: tuple[float, float, float], *,
                               block_size: int) -> tuple[int, int, tuple[float, float, float]]:
    """Validate separate BF16 branches and exclusive ownership of the base storage."""
    torch = _torch()
    if (
        not isinstance(base, torch.Tensor)
        or base.dtype != torch.bfloat16
        or base.ndim != 3
        or any(size <= 0 for size in base.shape)
        or base.shape[-1] % 3
        or not base.is_contiguous()
        or base.requires_grad
        or not isinstance(adapters, tuple)
        or len(adapters) != 3
    ):
        raise H3FusedOpsError("base must be a contiguous inference BF16 [B,S,3H]")
    expected = (*base.shape[:-1], base.shape[-1] // 3)
    for adapter in adapters:
        if (
            not isinstance(adapter, torch.Tensor)
            or adapter.device != base.device
            or adapter.dtype != base.dtype
            or tuple(adapter.shape) != expected
            or not adapter.is_contiguous()
            or adapter.requires_grad
            or _shares_storage(base, adapter)
        ):
            raise H3FusedOpsError("adapters must be separate contiguous BF16 [B,S,H]")
    if (
        not isinstance(scalings, tuple)
        or len(scalings) != 3
        or any(not isinstance(value, (int, float)) or isinstance(value, bool)
               or not math.isfinite(value) for value in scalings)
        or block_size != 1024
    ):
        raise H3FusedOpsError("require three finite scalings and SM89 block size 1024")
    return base.numel() // 3, expected[-1], tuple(float(value) for value in scalings)


def triton_strict_bf16_qkv_direct_merge(base: Any, adapters: tuple[Any, Any, Any], *,
                                        scalings: tuple[float, float, float],
                                        block_size: int = 1024) -> Any:
    """Merge three LoRA branches into a fresh base; the caller relinquishes its old values."""
    _elements, width, scales = _validate_qkv_direct_merge(base, adapters, scalings,
                                                          block_size=block_size)
    if base.device.type != "cuda":
        raise H3FusedOpsError("the direct QKV merge requires CUDA BF16 tensors")
    torch = _torch()
    _require_launchable(adapters[0])
    values = (ctypes.c_float * 3)(*scales)
    rows = base.numel() // base.shape[-1]
    with torch.cuda.device(base.device):
        rc = _lib.load().vfb_qkv_direct_merge(base.data_ptr(), adapters[0].data_ptr(),
                                              adapters[1].data_ptr(), adapters[2].data_ptr(),
                                              rows, width, values, _stream(base.device))
    _check(rc, "vfb_qkv_direct_merge")
    return base


def triton_strict_bf16_adapter_gate_residual(base: Any, adapter: Any, residual: Any, gate: Any, *,
                                             scaling: float, block_size: int = 256) -> Any:
    """Fuse LoRA scale/add and output gate/residual with strict BF16 rounding."""
    _validate_matching_activation(base, adapter, candidate_name="adapter", block_size=block_size)
    batch, tokens, hidden_size = _validate_common(residual, gate, modifier_name="gate",
                                                  block_size=block_size)
    if tuple(base.shape) != tuple(residual.shape):
        raise H3FusedOpsError("fused H3 projection must match the residual")
    (scaling,) = _validate_scalings((scaling,), 1)
    torch = _torch()
    _require_launchable(residual)
    output = torch.empty_like(residual)
    with torch.cuda.device(residual.device):
        rc = _lib.load().vfb_adapter_gate_residual(
            base.data_ptr(), adapter.data_ptr(), residual.data_ptr(), gate.data_ptr(),
            gate.stride(0), batch * tokens, tokens, hidden_size, scaling, output.data_ptr(),
            _stream(residual.device))
    _check(rc, "vfb_adapter_gate_residual")
    return output
