"""ctypes binding of ``libvflash_b200.so`` (the C ABI declared in include/vflash_b200.h).

The library is loaded once per process.  There is no fallback: if the shared
object is missing or fails to load, every call raises ``NativeLibraryError``.
Tensors cross the boundary as raw device pointers, sizes and strides; the
current torch CUDA stream is passed explicitly.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIBRARY_PATH = Path(os.environ.get("VFLASH_B200_LIBRARY", Path(__file__).with_name("libvflash_b200.so")))

VFB_OK = 0
VFB_EINVAL = 1
VFB_ECUDA = 2
VFB_EDEVICE = 3
VFB_ETIMEOUT = 4

EPI_STORE = 0
EPI_GELU_TANH = 1
EPI_SWIGLU = 2
EPI_RESIDUAL = 3
EPI_QKV_NORM_ROPE = 4

# Every symbol include/vflash_b200.h declares, with its ctypes signature.
_c_int64 = ctypes.c_int64
_vp = ctypes.c_void_p


class Epilogue(ctypes.Structure):
    """Mirror of ``vfb_epilogue``."""

    _fields_ = [
        ("kind", ctypes.c_int32),
        ("wire_chunks", ctypes.c_int32),
        ("out", _vp),
        ("ldo", _c_int64),
        ("plane_width", _c_int64),
        ("plane_stride", _c_int64),
        ("bias", _vp),
        ("adapter", _vp * 3),
        ("adapter_ld", _c_int64),
        ("scaling", ctypes.c_float * 3),
        ("reserved1", ctypes.c_int32),
        ("residual", _vp),
        ("ldr", _c_int64),
        ("gate", _vp),
        ("gate_token_stride", _c_int64),
        ("gate_hidden_stride", _c_int64),
        ("tokens", _c_int64),
        ("q_norm", _vp),
        ("k_norm", _vp),
        ("rope_cos", _vp),
        ("rope_sin", _vp),
        ("rope_token_stride", _c_int64),
        ("qk_eps", ctypes.c_float),
        ("reserved2", ctypes.c_int32),
    ]


SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "vfb_last_error": (ctypes.c_char_p, []),
    "vfb_version": (ctypes.c_char_p, []),
    "vfb_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "vfb_wait_selftest": (ctypes.c_int, [_c_int64, _vp]),
    "vfb_fp8_quant_rows": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_row_absmax": (ctypes.c_int, [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp]),
    "vfb_fp8_quant_rows_amax": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_norm_modulate_quant": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, ctypes.c_float, _vp, _c_int64, _vp, _c_int64, _c_int64,
         _vp, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_gemm": (
        ctypes.c_int,
        [_vp, _c_int64, _vp, _vp, _c_int64, _vp, _c_int64, _c_int64, _c_int64,
         ctypes.POINTER(Epilogue), _vp],
    ),
    "vfb_fp8_ffn_workspace_bytes": (_c_int64, [_c_int64, _c_int64, _c_int64]),
    "vfb_fp8_ffn": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, ctypes.c_int32, _vp, _vp, _vp,
         _c_int64, _vp, _c_int64, _c_int64, _vp, _c_int64, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_ffn_one_kernel": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, ctypes.c_int32, _vp, _vp, _vp,
         _c_int64, _vp, _c_int64, _c_int64, _vp, _c_int64, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_ffn_quantized": (
        ctypes.c_int,
        [_vp, _vp, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, ctypes.c_int32, _vp, _vp, _vp,
         _c_int64, _vp, _c_int64, _c_int64, _vp, _c_int64, _vp, _c_int64, _vp],
    ),
    "vfb_fp8_ffn_noalloc": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, ctypes.c_int32, _vp, _vp, _vp,
         _c_int64, _vp, _c_int64, _c_int64, _vp, _c_int64, _vp],
    ),
    "vfb_bf16_gemm": (
        ctypes.c_int,
        [_vp, _c_int64, _vp, _c_int64, _c_int64, _c_int64, _c_int64, ctypes.POINTER(Epilogue), _vp],
    ),
    "vfb_nvfp4_quant_rows": (
        ctypes.c_int, [_vp, ctypes.c_int32, _c_int64, _c_int64, _c_int64, _vp, _vp, _vp, _vp]),
    "vfb_nvfp4_norm_modulate_quant": (
        ctypes.c_int,
        [_vp, _c_int64, _c_int64, _c_int64, _vp, ctypes.c_float, _vp, _c_int64, _vp, _c_int64, _c_int64,
         _vp, _vp, _vp, _vp],
    ),
    "vfb_nvfp4_gemm": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp]),
    "vfb_nvfp4_gemm_ex": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, ctypes.POINTER(Epilogue), _vp],
    ),
    "vfb_nvfp4_gemm_quant": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, ctypes.POINTER(Epilogue), _vp, _vp, _vp,
         _vp],
    ),
    "vfb_silu_mul": (ctypes.c_int, [_vp, _c_int64, _c_int64, _vp, _c_int64, _vp]),
    "vfb_ffn_adapter_silu": (
        ctypes.c_int, [_vp, _vp, _c_int64, _c_int64, ctypes.c_float, _vp, _c_int64, _vp]),
    "vfb_gate_residual": (
        ctypes.c_int, [_vp, _vp, _c_int64, _vp, _c_int64, _c_int64, _c_int64, _vp, _vp]),
    "vfb_modulate": (
        ctypes.c_int, [_vp, _vp, _c_int64, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _vp, _vp]),
    "vfb_rotary": (
        ctypes.c_int, [_vp, _vp, _c_int64, _vp, _c_int64, _c_int64, _c_int64, _c_int64, _c_int64, _c_int64,
                       _vp, _vp]),
    "vfb_adapter_gate_residual": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64, ctypes.c_float, _vp, _vp]),
    "vfb_adapter_merge": (
        ctypes.c_int, [_vp, _vp, _c_int64, _c_int64, ctypes.c_int32, ctypes.POINTER(ctypes.c_float),
                       _vp, _vp]),
    "vfb_qkv_direct_merge": (
        ctypes.c_int, [_vp, _vp, _vp, _vp, _c_int64, _c_int64, ctypes.POINTER(ctypes.c_float), _vp]),
}


class NativeLibraryError(RuntimeError):
    """The native library is missing, failed to load, or a call failed."""


_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library (once) and bind every declared symbol."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not LIBRARY_PATH.exists():
                raise NativeLibraryError(
                    f"{LIBRARY_PATH} is missing; build it with `python -m vflash_b200.build`"
                )
            try:
                handle = ctypes.CDLL(str(LIBRARY_PATH))
            except OSError as exc:
                raise NativeLibraryError(f"cannot load {LIBRARY_PATH}: {exc}") from exc
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _handle = handle
    return _handle


def last_error() -> str:
    return load().vfb_last_error().decode()


def check(rc: int, what: str) -> None:
    if rc != VFB_OK:
        raise NativeLibraryError(f"{what} failed (code {rc}): {last_error()}")


def ptr(tensor) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_handle(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def device_status(clear: bool = True) -> int:
    """Device-side status word of the current device (VFB_ETIMEOUT after an expired wait)."""
    value = ctypes.c_int(0)
    check(load().vfb_device_status(ctypes.byref(value), int(clear)), "vfb_device_status")
    return value.value
