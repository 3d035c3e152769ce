"""The C-ABI library builds, loads and exports every symbol include/vflash_b200.h declares.

No compute call is made here; only argument validation that returns before
touching a device.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from vflash_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "vflash_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vfb_\w+)\s*\(", text)))


def exported_symbols(path: Path) -> set[str]:
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    exported = exported_symbols(_lib.LIBRARY_PATH)
    for name in declared_symbols():
        assert name in exported, name
        assert getattr(lib, name) is not None
    # nothing else leaks from the shared object's C ABI namespace
    assert {s for s in exported if s.startswith("vfb_")} == set(declared_symbols())


def test_version_and_error_strings():
    assert _lib.load().vfb_version().decode().startswith("vflash_b200")
    assert isinstance(_lib.last_error(), str)


def test_epilogue_struct_layout_matches_header():
    # 8-byte aligned fields as declared in vfb_epilogue
    assert ctypes.sizeof(_lib.Epilogue) == 4 + 4 + 8 * 5 + 8 * 3 + 8 + 4 * 3 + 4 + 8 * 6 + 8 * 5 + 4 + 4
    assert _lib.Epilogue.adapter.offset == 48
    assert _lib.Epilogue.residual.offset == 96
    assert _lib.Epilogue.q_norm.offset == 144
    assert _lib.Epilogue.wire_chunks.offset == 4


@pytest.mark.parametrize(
    "args",
    [
        (None, 4, 0, 4, None, None, 16, None),  # K = 0
        (None, 4, 40000, 40000, None, None, 16, None),  # K > 32768
        (None, 4, 64, 32, None, None, 16, None),  # ldx < K
        (None, 20, 64, 64, None, None, 16, None),  # M_pad < M
    ],
)
def test_quantiser_rejects_bad_shapes_before_any_launch(args):
    rc = _lib.load().vfb_fp8_quant_rows(*args)
    assert rc == _lib.VFB_EINVAL
    assert "vfb_fp8_quant_rows" in _lib.last_error()


def test_gemm_rejects_bad_shapes_before_any_launch():
    lib = _lib.load()
    ep = _lib.Epilogue()
    ep.kind = _lib.EPI_STORE
    assert lib.vfb_fp8_gemm(None, 64, None, None, 64, None, 4, 48, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert "N % 32" in _lib.last_error()
    ep.kind = 9
    assert lib.vfb_fp8_gemm(None, 64, None, None, 64, None, 4, 64, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert "unknown epilogue" in _lib.last_error()
    assert lib.vfb_fp8_gemm(None, 64, None, None, 64, None, 4, 64, 64, None, None) == _lib.VFB_EINVAL


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIBRARY_PATH", tmp_path / "absent.so")
    monkeypatch.setattr(_lib, "_handle", None)
    with pytest.raises(_lib.NativeLibraryError, match="missing"):
        _lib.load()


def test_new_entry_points_reject_bad_arguments_before_any_launch():
    lib = _lib.load()
    # fused norm + modulate + quantise: K % 8, tokens, eps, M_pad
    assert lib.vfb_fp8_norm_modulate_quant(None, 4, 12, 12, None, 1e-6, None, 0, None, 0, 1, None, None, 16,
                                           None) == _lib.VFB_EINVAL
    assert "vfb_fp8_norm_modulate_quant" in _lib.last_error()
    assert lib.vfb_fp8_norm_modulate_quant(None, 4, 64, 64, None, 1e-6, None, 0, None, 0, 0, None, None, 16,
                                           None) == _lib.VFB_EINVAL
    assert lib.vfb_fp8_norm_modulate_quant(None, 4, 64, 64, None, -1.0, None, 0, None, 0, 1, None, None, 16,
                                           None) == _lib.VFB_EINVAL
    assert lib.vfb_fp8_norm_modulate_quant(None, 20, 64, 64, None, 1e-6, None, 0, None, 0, 1, None, None, 16,
                                           None) == _lib.VFB_EINVAL
    # modulate / rotary: widths, tokens, rotary dimension
    assert lib.vfb_modulate(None, None, 0, None, 0, 4, 1, 12, None, None) == _lib.VFB_EINVAL
    assert lib.vfb_modulate(None, None, 0, None, 0, 4, 0, 16, None, None) == _lib.VFB_EINVAL
    assert lib.vfb_rotary(None, None, 0, None, 0, 4, 1, 2, 128, 130, None, None) == _lib.VFB_EINVAL
    assert lib.vfb_rotary(None, None, 0, None, 0, 4, 1, 2, 128, 63, None, None) == _lib.VFB_EINVAL
    assert "rotary_dim" in _lib.last_error()
    # bounded-wait self-test: limit range
    assert lib.vfb_wait_selftest(10, None) == _lib.VFB_EINVAL
    # QKV + QK-norm + rotary epilogue needs its tables
    ep = _lib.Epilogue()
    ep.kind = _lib.EPI_QKV_NORM_ROPE
    assert lib.vfb_fp8_gemm(None, 64, None, None, 64, None, 4, 384, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    # the pack_qkv wire layout only for STORE / QKV_NORM_ROPE, and a bounded chunk count
    for kind, chunks in ((_lib.EPI_GELU_TANH, 1), (_lib.EPI_RESIDUAL, 2), (_lib.EPI_STORE, -1),
                         (_lib.EPI_STORE, 4096)):
        ep = _lib.Epilogue()
        ep.kind, ep.wire_chunks = kind, chunks
        buf = ctypes.create_string_buffer(64)
        ptr = (ctypes.addressof(buf) + 15) // 16 * 16
        ep.out, ep.ldo = ptr, 64
        assert lib.vfb_fp8_gemm(ptr, 64, ptr, ptr, 64, ptr, 4, 384, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
        assert "wire_chunks" in _lib.last_error()


def test_bf16_gemm_rejects_bad_arguments_before_any_launch():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(64)
    ptr = (ctypes.addressof(buf) + 15) // 16 * 16
    ep = _lib.Epilogue()
    ep.kind, ep.out, ep.ldo = _lib.EPI_STORE, ptr, 64
    # K % 8, strides
    assert lib.vfb_bf16_gemm(ptr, 64, ptr, 64, 4, 64, 12, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert lib.vfb_bf16_gemm(ptr, 12, ptr, 64, 4, 64, 8, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert "vfb_bf16_gemm" in _lib.last_error()
    # N % 8
    assert lib.vfb_bf16_gemm(ptr, 64, ptr, 64, 4, 60, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    # plain STORE only: no bias, adapters, planes or other kinds
    for field, value in (("bias", ptr), ("plane_width", 32), ("wire_chunks", 1), ("kind", _lib.EPI_GELU_TANH)):
        bad = _lib.Epilogue()
        bad.kind, bad.out, bad.ldo = _lib.EPI_STORE, ptr, 64
        setattr(bad, field, value)
        assert lib.vfb_bf16_gemm(ptr, 64, ptr, 64, 4, 64, 64, ctypes.byref(bad), None) == _lib.VFB_EINVAL
        assert "vfb_bf16_gemm" in _lib.last_error()


def test_ffn_workspace_and_argument_checks_before_any_launch():
    lib = _lib.load()
    # x codes, x scales, mid, mid codes, mid scales, then the fused kernel's row
    # maxima and counters (1 + 2 per 256-row block); 256-byte aligned regions
    assert lib.vfb_fp8_ffn_workspace_bytes(10, 64, 64) == 1024 + 256 + 1280 + 1024 + 256 + 256
    assert lib.vfb_fp8_ffn_workspace_bytes(32760, 4096, 16384) == (
        32768 * 4096 + 32768 * 4 + 32760 * 16384 * 2 + 32768 * 16384 + 32768 * 4
        + (32760 * 4 + (1 + 2 * 128) * 4 + 255) // 256 * 256)
    for bad in ((10, 48, 64), (10, 64, 40), (-1, 64, 64), (10, 65536, 64)):
        assert lib.vfb_fp8_ffn_workspace_bytes(*bad) == -1
    buf = ctypes.create_string_buffer(8192)
    ptr = (ctypes.addressof(buf) + 255) // 256 * 256
    args = [ptr, 10, 64, 64, ptr, ptr, 64, ptr, ptr, _lib.EPI_GELU_TANH, None, None, None, 0, None, 0, 0,
            ptr, 64, ptr, 4096, None]
    bad_activation = list(args)
    bad_activation[9] = _lib.EPI_RESIDUAL
    assert lib.vfb_fp8_ffn(*bad_activation) == _lib.VFB_EINVAL and "activation" in _lib.last_error()
    odd_swiglu = list(args)
    odd_swiglu[9], odd_swiglu[6] = _lib.EPI_SWIGLU, 66
    assert lib.vfb_fp8_ffn(*odd_swiglu) == _lib.VFB_EINVAL
    short = list(args)
    short[20] = 4095
    assert lib.vfb_fp8_ffn(*short) == _lib.VFB_EINVAL and "workspace" in _lib.last_error()
    misaligned = list(args)
    misaligned[19] = ptr + 16
    assert lib.vfb_fp8_ffn(*misaligned) == _lib.VFB_EINVAL
    gate_alone = list(args)
    gate_alone[14], gate_alone[15], gate_alone[16] = ptr, 64, 1
    assert lib.vfb_fp8_ffn(*gate_alone) == _lib.VFB_EINVAL and "gate" in _lib.last_error()


def test_noalloc_row_limit_at_the_h3_ffn_shape():
    """vfb_fp8_ffn_noalloc's fixed 64 MiB array holds the intermediates of at most 1,382 rows at
    the H3 FFN shape (hidden 5376, F 14336); one more row is refused before any device work."""
    lib = _lib.load()
    scratch = 64 << 20
    assert lib.vfb_fp8_ffn_workspace_bytes(1382, 5376, 14336) <= scratch
    assert lib.vfb_fp8_ffn_workspace_bytes(1383, 5376, 14336) > scratch
    rc = lib.vfb_fp8_ffn_noalloc(None, 1383, 5376, 5376, None, None, 14336, None, None, _lib.EPI_GELU_TANH, None,
                                 None, None, 0, None, 0, 0, None, 5376, None)
    assert rc == _lib.VFB_EINVAL and "scratch" in _lib.last_error()
    # a wrong activation is reported as such, before the size check
    rc = lib.vfb_fp8_ffn_noalloc(None, 1383, 5376, 5376, None, None, 14336, None, None, _lib.EPI_RESIDUAL, None,
                                 None, None, 0, None, 0, 0, None, 5376, None)
    assert rc == _lib.VFB_EINVAL and "activation" in _lib.last_error()


def test_nvfp4_output_and_prologue_entry_points_reject_bad_arguments_before_any_launch():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(256)
    ptr = (ctypes.addressof(buf) + 15) // 16 * 16
    alpha = ctypes.c_float(1.0)
    gsf = ctypes.c_float(1.0)

    def quant(ep, codes=ptr, sf=ptr, n=128):
        return lib.vfb_nvfp4_gemm_quant(ptr, ptr, ptr, ptr, ctypes.byref(alpha), None, 4, n, 64,
                                        ctypes.byref(ep), ctypes.byref(gsf), codes, sf, None)

    # the NVFP4 output: no RESIDUAL epilogue, one plane, no adapter merge
    ep = _lib.Epilogue()
    ep.kind = _lib.EPI_RESIDUAL
    assert quant(ep) == _lib.VFB_EINVAL and "NVFP4 output" in _lib.last_error()
    ep = _lib.Epilogue()
    ep.kind, ep.plane_width = _lib.EPI_STORE, 64
    assert quant(ep) == _lib.VFB_EINVAL and "one plane" in _lib.last_error()
    ep = _lib.Epilogue()
    ep.kind = _lib.EPI_GELU_TANH
    ep.adapter[0] = ptr
    assert quant(ep) == _lib.VFB_EINVAL and "adapter" in _lib.last_error()
    # codes and scales present and 16-byte aligned; N % 128
    ep = _lib.Epilogue()
    ep.kind = _lib.EPI_GELU_TANH
    assert quant(ep, codes=None) == _lib.VFB_EINVAL and "global scale" in _lib.last_error()
    assert quant(ep, sf=ptr + 8) == _lib.VFB_EINVAL
    assert quant(ep, n=192) == _lib.VFB_EINVAL and "vfb_nvfp4_gemm_quant" in _lib.last_error()
    ep.kind = _lib.EPI_SWIGLU
    assert quant(ep, n=128) == _lib.VFB_EINVAL and "SWIGLU" in _lib.last_error()

    # norm + modulate + NVFP4 quantise: K % 64, tokens, eps, alignment
    def prologue(k=64, ldx=64, tokens=1, eps=1e-6, x=ptr, codes=ptr):
        return lib.vfb_nvfp4_norm_modulate_quant(x, 4, k, ldx, None, eps, ptr, 0, ptr, 0, tokens,
                                                 ctypes.byref(gsf), codes, ptr, None)

    assert prologue(k=96, ldx=96) == _lib.VFB_EINVAL and "K %" in _lib.last_error()
    assert prologue(ldx=32) == _lib.VFB_EINVAL
    assert prologue(tokens=0) == _lib.VFB_EINVAL
    assert prologue(eps=-1.0) == _lib.VFB_EINVAL
    assert prologue(x=ptr + 2) == _lib.VFB_EINVAL and "aligned" in _lib.last_error()
    assert prologue(codes=ptr + 4) == _lib.VFB_EINVAL
    assert prologue(x=None) == _lib.VFB_EINVAL and "NULL" in _lib.last_error()


def test_fp8_swiglu_width_checks_come_before_the_device_probe():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(256)
    ptr = (ctypes.addressof(buf) + 15) // 16 * 16
    ep = _lib.Epilogue()
    ep.kind, ep.out, ep.ldo = _lib.EPI_SWIGLU, ptr, 64
    # packed width 2F with F % 32: N = 96 is refused
    assert lib.vfb_fp8_gemm(ptr, 64, ptr, ptr, 64, ptr, 4, 96, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert "SWIGLU" in _lib.last_error()
    # ldo below F = 64
    ep.ldo = 32
    assert lib.vfb_fp8_gemm(ptr, 64, ptr, ptr, 64, ptr, 4, 128, 64, ctypes.byref(ep), None) == _lib.VFB_EINVAL
    assert "ldo" in _lib.last_error()
