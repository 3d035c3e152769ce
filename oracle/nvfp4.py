"""CPU restatement of the NVFP4 linear path (test infrastructure only).

Reference: Hansimov/vflash src/vflash/native/h3_nvfp4_linear.py:77-139 calls
FlashInfer (``flashinfer-python==0.6.18``, pyproject.toml:24; not vendored in
the reference) for the arithmetic:

* ``nvfp4_quantize(x, gsf, sfLayout=128x4, do_shuffle=False)`` — per 16
  elements ``sf = e4m3_rn_satfinite(gsf * (amax * rcp(6)))``,
  ``scale = amax != 0 ? rcp(float(sf) * rcp(gsf)) : 0``,
  ``code = e2m1_rn_satfinite(x * scale)`` (FlashInfer's published
  quantization_utils.cuh:294-380, default recipe), with multiplies that flush
  subnormals (fast-math build).  ``rcp`` there is ``rcp.approx.ftz.f32``; this
  restatement uses correctly rounded fp32 reciprocals, so a value within an
  ulp of an e2m1 / e4m3 rounding boundary may round the other way here (about
  0.1 % of codes on seeded N(0,1) data, one code step each).  Bit parity is
  therefore pinned on the GPU against FlashInfer itself (bit-exact, bf16 and
  fp16 inputs); this oracle is held to >= 99.5 % agreement.
* ``mm_fp4(...)`` — ``out = bf16(alpha * sum_k a(m,k) w(n,k))`` where
  ``a(m,k) = e2m1(code) * e4m3(sf[m, k/16])`` (likewise ``w``), then
  ``bf16(out + bias)`` as a separate add (h3_nvfp4_linear.py:139).

Formats, from their definitions: e2m1 = 1 sign bit, 2 exponent bits, 1
mantissa bit, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}; two codes per byte with
element 2i in the low nibble.  Scale factors are ue4m3 bytes in the 128x4
layout: for row m and 16-element group k,
``offset = (m//128)*(kt*512) + (k//4)*512 + (m%32)*16 + ((m%128)//32)*4 + k%4``
with ``kt = ceil(groups/4)``; rows are padded to 128 and groups to 4.
"""

from __future__ import annotations

import numpy as np

from .fp8 import bf16_round, e4m3_decode, e4m3_encode

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
FLT_MIN = np.float32(np.finfo(np.float32).tiny)


def _ftz(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return np.where(np.abs(x) < FLT_MIN, np.float32(0.0) * np.sign(x), x).astype(np.float32)


def mul_ftz(a, b) -> np.ndarray:
    """fp32 multiply with subnormal inputs and results flushed to zero."""
    return _ftz(_ftz(a) * _ftz(b))


def e2m1_encode(v: np.ndarray) -> np.ndarray:
    """float32 -> 4-bit e2m1 codes, round to nearest even, saturating to +-6."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v)
    idx = np.zeros(v.shape, dtype=np.uint8)
    # interval boundaries with ties going to the even mantissa
    idx = np.where(a > 0.25, 1, idx)
    idx = np.where(a >= 0.75, 2, idx)
    idx = np.where(a > 1.25, 3, idx)
    idx = np.where(a >= 1.75, 4, idx)
    idx = np.where(a > 2.5, 5, idx)
    idx = np.where(a >= 3.5, 6, idx)
    idx = np.where(a > 5.0, 7, idx)
    sign = (np.signbit(v)).astype(np.uint8) << 3
    return (idx.astype(np.uint8) | sign).astype(np.uint8)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    mag = E2M1_VALUES[c & 7]
    return np.where(c & 8, -mag, mag).astype(np.float32)


def pack(codes: np.ndarray) -> np.ndarray:
    """[R, K] 4-bit codes -> [R, K/2] bytes, element 2i in the low nibble."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = p >> 4
    return out


def sf_padded_shape(rows: int, groups: int) -> tuple[int, int]:
    return (-(-rows // 128) * 128, -(-groups // 4) * 4)


def sf_offsets(rows_pad: int, groups_pad: int) -> np.ndarray:
    """Byte offset of scale (m, k) in the 128x4 layout, as an [rows_pad, groups_pad] array."""
    m = np.arange(rows_pad, dtype=np.int64)[:, None]
    k = np.arange(groups_pad, dtype=np.int64)[None, :]
    kt = groups_pad // 4
    return (m // 128) * (kt * 512) + (k // 4) * 512 + (m % 32) * 16 + ((m % 128) // 32) * 4 + k % 4


def sf_swizzle(sf_matrix: np.ndarray) -> np.ndarray:
    """[rows_pad, groups_pad] row-major scales -> flat 128x4 layout."""
    rows_pad, groups_pad = sf_matrix.shape
    flat = np.zeros(rows_pad * groups_pad, dtype=np.uint8)
    flat[sf_offsets(rows_pad, groups_pad)] = sf_matrix
    return flat


def sf_unswizzle(flat: np.ndarray, rows_pad: int, groups_pad: int) -> np.ndarray:
    return np.asarray(flat, dtype=np.uint8).reshape(-1)[sf_offsets(rows_pad, groups_pad)]


def quantize(x: np.ndarray, gsf: float):
    """Restated nvfp4_quantize: returns (packed codes [M, K/2], scales flat 128x4 layout).

    ``x`` holds bf16/fp16-representable float32 values, shape [M, K], K % 16 == 0.
    """
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    groups = cols // 16
    gsf = np.float32(gsf)
    rcp6 = np.float32(1.0) / np.float32(6.0)
    rcp_gsf = np.float32(1.0) / gsf
    blocks = x.reshape(rows, groups, 16)
    amax = np.abs(blocks).max(axis=2)
    sf_value = mul_ftz(gsf, mul_ftz(amax, rcp6))
    sf = e4m3_encode(sf_value)
    with np.errstate(divide="ignore"):
        denom = mul_ftz(e4m3_decode(sf), rcp_gsf)
        scale = np.where(_ftz(amax) != 0, np.float32(1.0) / denom, np.float32(0.0)).astype(np.float32)
    codes = e2m1_encode(mul_ftz(blocks, scale[:, :, None])).reshape(rows, cols)
    rows_pad, groups_pad = sf_padded_shape(rows, groups)
    sf_full = np.zeros((rows_pad, groups_pad), dtype=np.uint8)
    sf_full[:rows, :groups] = sf
    return pack(codes), sf_swizzle(sf_full)


def dequantize(packed: np.ndarray, sf_flat: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """e2m1(code) * e4m3(scale) per element (no global scale), float64 [rows, cols]."""
    rows_pad, groups_pad = sf_padded_shape(rows, cols // 16)
    sf = e4m3_decode(sf_unswizzle(sf_flat, rows_pad, groups_pad)[:rows, : cols // 16]).astype(np.float64)
    vals = e2m1_decode(unpack(packed)).astype(np.float64)
    return vals * np.repeat(sf, 16, axis=1)


def w4a4_reference(a_packed, a_sf, w_packed, w_sf, alpha: float, bias=None):
    """Exact emulation of mm_fp4 + bias: bf16(alpha * sum) then bf16(+ bias); float32 values."""
    m, n, k = a_packed.shape[0], w_packed.shape[0], a_packed.shape[1] * 2
    acc = dequantize(a_packed, a_sf, m, k) @ dequantize(w_packed, w_sf, n, k).T
    y = bf16_round((np.float32(alpha) * acc.astype(np.float32)).astype(np.float32))
    if bias is not None:
        y = bf16_round(y + np.asarray(bias, np.float32).reshape(1, -1))
    return y


def dequant_matmul_f32(a_packed, a_sf, w_packed, w_sf, alpha: float) -> np.ndarray:
    """fp32 dequantise-then-matmul of the same quantised operands."""
    m, n, k = a_packed.shape[0], w_packed.shape[0], a_packed.shape[1] * 2
    a = dequantize(a_packed, a_sf, m, k).astype(np.float32)
    w = dequantize(w_packed, w_sf, n, k).astype(np.float32)
    return (np.float32(alpha) * (a @ w.T)).astype(np.float32)
