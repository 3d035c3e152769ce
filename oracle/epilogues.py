"""CPU restatement of the strict-BF16 elementwise steps around the linears (test infrastructure only).

Each function keeps the rounding boundaries of the reference kernel it cites
(Hansimov/vflash, src/vflash/native/h3_fused_ops.py); inputs and outputs are
bf16 bit patterns (uint16) so that results can be compared bit for bit.
"""

from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits, bf16_round, bf16_value


def silu_f32(g: np.ndarray) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def gelu_tanh_f32(y: np.ndarray) -> np.ndarray:
    """0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3))) in fp32."""
    y = np.asarray(y, dtype=np.float32)
    k_beta = np.float32(0.7978845608028654)
    k_kappa = np.float32(0.044715)
    cube = y * y * y
    inner = k_beta * (y + k_kappa * cube)
    return (np.float32(0.5) * y * (np.float32(1.0) + np.tanh(inner))).astype(np.float32)


def silu_mul(packed_bits: np.ndarray) -> np.ndarray:
    """``strict_silu_mul_kernel`` (h3_fused_ops.py:185-224): value * bf16(silu(gate)).

    ``packed`` is [..., 2F]; value = first F columns, gate = last F.
    """
    packed = bf16_value(packed_bits)
    width = packed.shape[-1] // 2
    value, gate = packed[..., :width], packed[..., width:]
    return bf16_bits(value * bf16_round(silu_f32(gate)))


def gelu_tanh(y_bits: np.ndarray) -> np.ndarray:
    """torch ``F.gelu(y, approximate="tanh")`` on a bf16 linear output."""
    return bf16_bits(gelu_tanh_f32(bf16_value(y_bits)))


def gate_residual(residual_bits, gate_bits, projected_bits) -> np.ndarray:
    """``strict_gate_residual_kernel`` (h3_fused_ops.py:125-170): residual + bf16(gate * projected).

    residual/projected [B,S,H]; gate [S,H] broadcast over the batch.
    """
    residual = bf16_value(residual_bits)
    gate = bf16_value(gate_bits)
    projected = bf16_value(projected_bits)
    return bf16_bits(residual + bf16_round(gate * projected))


def qkv_direct_merge(base_bits, adapter_bits, scalings) -> np.ndarray:
    """``strict_qkv_direct_merge_kernel`` (h3_fused_ops.py:901-949).

    base [..., 3H]; adapters 3 x [..., H]; per branch b:
    base_b = bf16(base_b + bf16(adapter_b * scaling_b)).
    """
    base = bf16_value(base_bits).copy()
    width = base.shape[-1] // 3
    for b in range(3):
        adapter = bf16_value(adapter_bits[b])
        sl = slice(b * width, (b + 1) * width)
        base[..., sl] = base[..., sl] + bf16_round(adapter * np.float32(scalings[b]))
    return bf16_bits(base)


def ffn_adapter_silu(base_bits, adapter_bits, scaling) -> np.ndarray:
    """``strict_ffn_adapter_silu_kernel`` (h3_fused_ops.py:254-284).

    value = bf16(base_v + bf16(adapter_v * s)), gate = bf16(base_g + bf16(adapter_g * s)),
    out = bf16(value * bf16(silu(gate))).
    """
    base = bf16_value(base_bits)
    adapter = bf16_value(adapter_bits)
    width = base.shape[-1] // 2
    s = np.float32(scaling)
    value = bf16_round(base[..., :width] + bf16_round(adapter[..., :width] * s))
    gate = bf16_round(base[..., width:] + bf16_round(adapter[..., width:] * s))
    return bf16_bits(value * bf16_round(silu_f32(gate)))


def adapter_merge(base_bits, adapter_bits, scalings) -> np.ndarray:
    """``strict_adapter_merge_kernel`` (h3_fused_ops.py:298-339): base + bf16(adapter * s_branch).

    ``scalings`` has one entry per equal-width branch of the last dimension.
    """
    base = bf16_value(base_bits)
    adapter = bf16_value(adapter_bits)
    branches = len(scalings)
    width = base.shape[-1] // branches
    scale = np.repeat(np.asarray(scalings, dtype=np.float32), width)
    return bf16_bits(base + bf16_round(adapter * scale))


def adapter_gate_residual(base_bits, adapter_bits, residual_bits, gate_bits, scaling) -> np.ndarray:
    """``strict_adapter_gate_residual_kernel`` (h3_fused_ops.py:342-415).

    residual + bf16(gate * bf16(base + bf16(adapter * s))).
    """
    base = bf16_value(base_bits)
    adapter = bf16_value(adapter_bits)
    residual = bf16_value(residual_bits)
    gate = bf16_value(gate_bits)
    adapted = bf16_round(base + bf16_round(adapter * np.float32(scaling)))
    return bf16_bits(residual + bf16_round(gate * adapted))


def modulate(value_bits, scale_bits, shift_bits) -> np.ndarray:
    """``strict_modulate_kernel`` (h3_fused_ops.py:52-122): bf16(bf16(x * bf16(1 + scale)) + shift).

    value [B,S,H] (or [S,H]); scale/shift [S,H] broadcast over the batch.
    All arithmetic in fp32 with the kernel's three bf16 roundings.
    """
    value = bf16_value(value_bits)
    scale = bf16_value(scale_bits)
    shift = bf16_value(shift_bits)
    one_plus = bf16_round((np.float32(1.0) + scale).astype(np.float32))
    scaled = bf16_round((value * one_plus).astype(np.float32))
    return bf16_bits((scaled + shift).astype(np.float32))


def rms_norm(x_bits, weight_bits, eps: float) -> np.ndarray:
    """torch ``F.rms_norm`` on bf16 (``_rms_norm``, h3_native_denoiser.py:231-243).

    Follows torch's fused decomposition (fp32 upcast, ``rsqrt(mean(x^2) + eps)``,
    ``(x * rstd) * w`` in fp32, one rounding to bf16).  The mean of squares is
    summed in float64 and rounded to fp32, and the reciprocal square root is
    taken in float64 and rounded to fp32: the ideal values that a GPU
    reduction approximates to within an fp32 ulp.
    """
    x = bf16_value(x_bits).astype(np.float32)
    k = x.shape[-1]
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    mean = (ss.astype(np.float32) / np.float32(k)).astype(np.float32)
    mean_eps = (mean + np.float32(eps)).astype(np.float32)
    rstd = (1.0 / np.sqrt(mean_eps.astype(np.float64))).astype(np.float32)
    y = (x * rstd).astype(np.float32)
    if weight_bits is not None:
        y = (y * bf16_value(weight_bits).astype(np.float32)).astype(np.float32)
    return bf16_bits(y)


def rotary(value_bits, cos_bits, sin_bits) -> np.ndarray:
    """``strict_rotary_kernel`` (h3_fused_ops.py:421-510) / ``_apply_rotary`` (h3_native_denoiser.py:246-256).

    value [B,S,heads,head_dim]; cos/sin [S,rotary_dim].  On the first
    rotary_dim values of each head: bf16(bf16(x * cos) + bf16(partner * sin))
    with partner = cat(-second_half, first_half); the rest is copied.
    """
    value = bf16_value(value_bits)
    cos = bf16_value(cos_bits)[None, :, None, :]
    sin = bf16_value(sin_bits)[None, :, None, :]
    rd = cos.shape[-1]
    rot = value[..., :rd]
    first, second = rot[..., : rd // 2], rot[..., rd // 2:]
    partner = np.concatenate([-second, first], axis=-1)
    out = value.copy()
    out[..., :rd] = bf16_round(rot * cos) + bf16_round(partner * sin)
    return bf16_bits(out.astype(np.float32))


def pack_qkv(q, k, v, chunks: int) -> np.ndarray:
    """Destination-major QKV wire layout (src/vflash/native/h3_parallel_relayout.py:214-222).

    ``q``, ``k``, ``v`` are ``[B, rows, heads, D]`` arrays (any dtype, here
    bf16 bit patterns); heads split as (destination 2, chunk, heads per
    chunk), and the result is ``(chunk, destination, qkv, B, rows,
    heads / (2 chunks), D)``.  A pure permutation: values are moved, not
    changed.
    """
    b, rows, heads, d = q.shape
    if heads % (2 * chunks):
        raise ValueError("QKV heads must divide two destinations and all chunks")
    stacked = np.stack((q, k, v)).reshape(3, b, rows, 2, chunks, heads // (2 * chunks), d)
    return np.ascontiguousarray(stacked.transpose(4, 3, 0, 1, 2, 5, 6))


def bf16_linear(a_bits, w_bits) -> np.ndarray:
    """``functional.linear(a, w)`` in bf16 without bias: bf16(exact a @ w^T), as bf16 bits.

    The products and their sum are formed in float64 (exact for these sizes
    up to the final rounding), so a fp32-accumulating kernel may differ from
    this by one bf16 step where its sum lands next to a rounding boundary.
    Follows the low-rank products of _residual_linear_unscaled
    (src/vflash/native/h3_native_denoiser.py:288-299).
    """
    a = bf16_value(a_bits).astype(np.float64)
    w = bf16_value(w_bits).astype(np.float64)
    return f64_to_bf16_bits(a @ w.T)


def f64_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float64 -> bf16 bits with ONE round-to-nearest-even.

    Goes through float32 rounded to odd (an inexact result takes the odd one
    of its two float32 neighbours), which keeps the sticky information, so
    the final bf16 rounding equals a direct rounding of the float64 value.
    """
    x = np.asarray(x, dtype=np.float64)
    t = x.astype(np.float32)
    inexact = t.astype(np.float64) != x
    even = (t.view(np.uint32) & 1) == 0
    fix = inexact & even & np.isfinite(t)
    toward = np.where(x > t.astype(np.float64), np.float32(np.inf), np.float32(-np.inf))
    t = np.where(fix, np.nextafter(t, toward), t).astype(np.float32)
    return bf16_bits(t)


def low_rank(x_bits, down_bits, up_bits) -> np.ndarray:
    """Unscaled low-rank residual: bf16 rounding after each product (h3_native_denoiser.py:297-299)."""
    return bf16_linear(bf16_linear(x_bits, down_bits), up_bits)
