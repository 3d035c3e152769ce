"""CPU restatement of the reference FP8 row-scaled linear path (test infrastructure only).

Reference (Hansimov/vflash, paths relative to its repository root):
  * ``_quantize_activation_torch`` — src/vflash/native/h3_fp8_linear.py:18-31
    (the Triton ``_rows_fp8`` kernel, src/vflash/native/h3_fp8_activation.py:13-28,
    computes the same expression with ``div_rn``).
  * ``RowFP8Execution.linear`` weight-only branch — h3_fp8_linear.py:88-91.
  * W8A8 branch — h3_fp8_linear.py:92-121 (``torch._scaled_mm`` rowwise, then
    ``output + bias``).

The e4m3 and bf16 encoders below are written from the formats' definitions
(e4m3fn: 1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no infinity,
S.1111.111 = NaN, max 448; bf16: the upper 16 bits of an IEEE binary32,
rounded to nearest even), not from any library.
"""

from __future__ import annotations

import numpy as np

FLT_MIN = np.float32(np.finfo(np.float32).tiny)
E4M3_MAX = np.float32(448.0)


# ---------------------------------------------------------------------------
# bf16
# ---------------------------------------------------------------------------
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even, NaN kept quiet."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    b = f.view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), rounded)
    return rounded


def bf16_value(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """One eager BF16 rounding boundary: float32 -> nearest bf16 -> float32."""
    return bf16_value(bf16_bits(x))


# ---------------------------------------------------------------------------
# e4m3fn
# ---------------------------------------------------------------------------
def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn bytes, round to nearest even, saturating finite values to +-448."""
    f = np.asarray(x, dtype=np.float32)
    sign = (f.view(np.uint32) >> 31).astype(np.uint8) << 7
    a = np.abs(f).astype(np.float64)
    code = np.zeros(f.shape, dtype=np.uint8)
    # subnormals (and zero): multiples of 2^-9 below 2^-6
    sub = a < 2.0**-6
    code = np.where(sub, np.rint(a * 512.0).astype(np.int64), 0).astype(np.int64)
    # normals
    mant, ex = np.frexp(np.where(sub, 1.0, a))  # a = mant * 2^ex, mant in [0.5, 1)
    e = ex - 1  # a = (2*mant) * 2^e, 2*mant in [1, 2)
    q = np.rint((2.0 * mant - 1.0) * 8.0).astype(np.int64)
    carry = q == 8
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 0, q)
    normal = ((e + 7) << 3) | q
    normal = np.minimum(normal, 0x7E)  # saturate finite overflow to 448
    code = np.where(sub, code, normal)
    code = np.where(np.isinf(f), 0x7E, code)
    out = code.astype(np.uint8) | sign
    return np.where(np.isnan(f), np.uint8(0x7F) | sign, out).astype(np.uint8)


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 (0x7F / 0xFF decode to NaN)."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    value = np.where(e == 0, m * 2.0**-9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    value = np.where((c & 0x7F) == 0x7F, np.nan, value)
    return (sign * value).astype(np.float32)


# ---------------------------------------------------------------------------
# activation quantiser (h3_fp8_linear.py:18-31)
# ---------------------------------------------------------------------------
def quantize_activation(matrix_bf16_bits: np.ndarray, pad_to: int = 16):
    """Per-token e4m3 quantisation of a bf16 matrix given as uint16 bit patterns.

    Returns ``(codes uint8 [ceil(M/pad_to)*pad_to, K], scales float32 [.., 1])``:
      amax  = max |x| per row (fp32; NaN propagates as in torch.amax)
      scale = amax > 0 ? max(amax / 448, FLT_MIN) : 1
      codes = e4m3(clamp(x / scale, -448, 448))
    Padding rows are zero, so they get code 0 and scale 1.
    """
    x = bf16_value(np.asarray(matrix_bf16_bits, dtype=np.uint16))
    rows, cols = x.shape
    padded = -(-rows // pad_to) * pad_to if pad_to > 1 else rows
    if padded != rows:
        x = np.concatenate([x, np.zeros((padded - rows, cols), dtype=np.float32)], axis=0)
    nan_rows = np.isnan(x).any(axis=1, keepdims=True)
    amax = np.abs(x).max(axis=1, keepdims=True).astype(np.float32) if cols else np.zeros(
        (padded, 1), np.float32)
    amax = np.where(nan_rows, np.float32(np.nan), amax)
    with np.errstate(invalid="ignore", divide="ignore"):
        scale = np.where(amax > 0, np.maximum(amax / E4M3_MAX, FLT_MIN), np.float32(1.0))
        scale = scale.astype(np.float32)
        q = (x / scale).astype(np.float32)
    # torch.clamp keeps NaN
    q = np.where(q > E4M3_MAX, E4M3_MAX, q)
    q = np.where(q < -E4M3_MAX, -E4M3_MAX, q)
    return e4m3_encode(q), scale


def quantize_weight(weight_f32: np.ndarray):
    """Per-output-row e4m3 weight quantisation used for synthetic weights.

    The reference ships no weight quantiser (its FP8 weights arrive
    pre-quantised as ``<name>.weight`` + ``<name>.weight.row_scale``); this
    applies the activation formula above to each output row, without padding.
    Input is float32; it is first rounded to bf16 as a checkpoint would be.
    """
    bits = bf16_bits(np.asarray(weight_f32, dtype=np.float32))
    codes, scale = quantize_activation(bits, pad_to=1)
    return codes, scale


# ---------------------------------------------------------------------------
# linears
# ---------------------------------------------------------------------------
def weight_only_linear(value, codes, scale, bias=None):
    """``RowFP8Execution("weight-only").linear`` (h3_fp8_linear.py:88-91) on torch CPU.

    ``restored = (codes.float() * scale).to(value.dtype)``, then
    ``F.linear(value, restored, bias)``.  This is the reference's own CPU path
    and the timed CPU baseline.
    """
    import torch

    restored = (codes.float() * scale).to(value.dtype)
    return torch.nn.functional.linear(value, restored, bias)


def w8a8_reference(a_codes, a_scale, w_codes, w_scale, bias_bits=None):
    """Emulation of ``torch._scaled_mm`` rowwise + bias (h3_fp8_linear.py:109-121).

    out = bf16(sa[m] * sw[n] * sum_k a[m,k] w[n,k]) accumulated exactly (fp64),
    then bf16(out + bias).  Returns float32 values of the bf16 result.
    """
    a = e4m3_decode(a_codes).astype(np.float64)
    w = e4m3_decode(w_codes).astype(np.float64)
    acc = a @ w.T
    y = (acc.astype(np.float32) * np.asarray(a_scale, np.float32).reshape(-1, 1)
         * np.asarray(w_scale, np.float32).reshape(1, -1))
    y = bf16_round(y.astype(np.float32))
    if bias_bits is not None:
        y = bf16_round(y + bf16_value(bias_bits).reshape(1, -1))
    return y


def dequant_matmul_f32(a_codes, a_scale, w_codes, w_scale):
    """fp32 dequantise-then-matmul: (codes_a * sa) @ (codes_w * sw)^T."""
    a = e4m3_decode(a_codes) * np.asarray(a_scale, np.float32).reshape(-1, 1)
    w = e4m3_decode(w_codes) * np.asarray(w_scale, np.float32).reshape(-1, 1)
    return (a.astype(np.float32) @ w.astype(np.float32).T).astype(np.float32)


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    denom = np.linalg.norm(e)
    return float(np.linalg.norm(a - e) / (denom if denom > 0 else 1.0))
