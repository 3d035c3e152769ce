"""Explicit approximate row-scaled E4M3 linear execution on SM100 (drop-in).

Mirrors ``RowFP8Execution`` / ``RowFP8Linear`` of Hansimov/vflash
(src/vflash/native/h3_fp8_linear.py:34-149): same constructor arguments,
attributes (``mode``, ``calls``, ``observer``, ``measure``), validation order
and error messages, same weight layout (e4m3 ``[N, K]`` + fp32 ``row_scale``
``[N, 1]``) and same output (bf16 ``[..., N]``).

* ``weight-only`` keeps the reference's restored-weight expression verbatim
  (h3_fp8_linear.py:88-91); it is the reference's explicit alternative mode,
  not the W8A8 hot path, and never runs in its place.
* ``w8a8`` runs the native SM100 path: the per-token e4m3 quantiser
  (``vfb_fp8_quant_rows``) and the tcgen05 GEMM (``vfb_fp8_gemm``) with the
  row x column scales and bias fused into its epilogue.  Both
  ``activation_quantizer`` values select the same native quantiser (the
  reference's two choices compute identical bits).  ``fast_accum`` is kept
  for compatibility: the tcgen05 path always accumulates in fp32 TMEM.
  Non-SM100 devices and non-bf16 inputs raise; nothing falls back.

New fused entry points (``qkv_linear``, ``gelu_linear``, ``swiglu_linear``,
``gate_residual_linear``, ``ffn``) run the same GEMM with the elementwise step
that the H3 block performs next fused into the epilogue; each keeps the BF16
rounding boundaries of the reference's separate launch.  ``linear``,
``qkv_linear``, ``gelu_linear``, ``swiglu_linear`` and ``ffn`` also take a
``prologue=NormModulate(...)``: the block's RMSNorm + AdaLN modulate
(src/vflash/native/h3_native_denoiser.py:534-541, 561-568) then runs inside
the activation quantiser (``vfb_fp8_norm_modulate_quant``) and ``value`` is
the un-normalised hidden state.
"""

from __future__ import annotations

from collections.abc import Callable
from contextlib import AbstractContextManager, nullcontext
from dataclasses import dataclass
from typing import Any

import torch

from .. import _lib
from ..kernels import (Epilogue, bf16_gemm, fp8_ffn, fp8_ffn_quantized, fp8_gemm, quantize_fp8_norm_modulate,
                       quantize_fp8_rows)


@dataclass(frozen=True)
class NormModulate:
    """RMSNorm + AdaLN modulate applied to a linear's input inside its quantiser.

    ``norm_weight`` bf16 ``[K]`` (or None), ``scale``/``shift`` bf16 ``[S, K]``
    indexed by token (``[1, K]`` for one modulation of every token), ``eps``
    the norm epsilon.  The quantised activation is that of
    ``bf16(bf16(rms_norm(value) * bf16(1 + scale)) + shift)``.
    """

    norm_weight: torch.Tensor | None
    scale: torch.Tensor
    shift: torch.Tensor
    eps: float = 1e-6


@dataclass(frozen=True)
class QKNormRope:
    """The block's QK-norm + rotary (h3_native_denoiser.py:409-419) fused into ``qkv_linear``.

    ``q_norm``/``k_norm`` bf16 ``[128]`` (or None), ``cos``/``sin`` bf16
    ``[S, 128]`` indexed by token (rotary over the whole 128-wide head), ``eps``
    the QK-norm epsilon.
    """

    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    cos: torch.Tensor
    sin: torch.Tensor
    eps: float = 1e-5


def _quantize_activation_torch(matrix):
    """The reference's per-token quantiser (h3_fp8_linear.py:18-31), same outputs, on SM100.

    Codes e4m3 ``[ceil16(M), K]`` and fp32 scales ``[ceil16(M), 1]`` of a bf16
    ``[M, K]`` matrix, computed by the native quantiser, which reproduces the
    reference expression bit for bit.  Raises for other devices (no host path).
    """
    if not isinstance(matrix, torch.Tensor) or not _on_sm100(matrix.device) or matrix.dtype != torch.bfloat16:
        raise ValueError("the FP8 activation quantiser requires an SM100 (B200) BF16 matrix")
    return quantize_fp8_rows(matrix, pad_to=16)


def _on_sm100(device: torch.device) -> bool:
    return device.type == "cuda" and torch.cuda.get_device_capability(device) == (10, 0)


class RowFP8Execution:
    """Own precision choice and counters without changing any process globals.

    Weight-only restores approximate weights for the ordinary GEMM. W8A8 uses
    BF16 input, E4M3 activations/weights and FP32 per-row scales on SM100.
    ``measure`` may supply asynchronous profiling scopes; this class inserts no
    synchronization, model reads, environment changes or device selection.
    """

    def __init__(
        self,
        mode: str = "weight-only",
        *,
        activation_quantizer: str = "torch",
        fast_accum: bool = False,
        measure: Callable[[str], AbstractContextManager[Any]] | None = None,
    ) -> None:
        if activation_quantizer not in ("torch", "triton"):
            raise ValueError("unknown FP8 activation quantizer")
        if type(fast_accum) is not bool:
            raise ValueError("fast_accum must be an explicit boolean")
        self.activation_quantizer = activation_quantizer
        self.fast_accum = fast_accum
        self.measure = measure if measure is not None else lambda _name: nullcontext()
        self.observer: Callable[[], None] | None = None
        self.calls = {"weight_only": 0, "w8a8": 0}
        self.select(mode)

    def select(self, mode: str) -> None:
        if mode not in ("weight-only", "w8a8"):
            raise ValueError("unknown FP8 execution mode")
        self.mode = mode

    # -- validation shared by every entry point (h3_fp8_linear.py:70-87) -------
    @staticmethod
    def _validate(value, weight, scale, bias) -> None:
        if (
            weight.ndim != 2
            or value.ndim < 1
            or min(weight.shape) <= 0
            or value.shape[-1] != weight.shape[1]
            or weight.dtype != torch.float8_e4m3fn
            or scale.dtype != torch.float32
            or scale.shape != (weight.shape[0], 1)
            or weight.device != value.device
            or scale.device != value.device
        ):
            raise ValueError("FP8 codes/scales differ from the declared layout")
        if bias is not None and (
            bias.shape != (weight.shape[0],)
            or bias.device != value.device
            or bias.dtype != value.dtype
        ):
            raise ValueError("FP8 bias differs from the declared output")

    @staticmethod
    def _require_w8a8_device(value) -> None:
        if value.dtype != torch.bfloat16 or not _on_sm100(value.device):
            raise ValueError("W8A8 requires SM100 (B200) BF16 inputs")

    def _observe(self) -> None:
        if self.observer is not None and sum(self.calls.values()) % 200 == 0:
            self.observer()

    def _quantize(self, matrix, prologue: NormModulate | None = None, shape=None):
        with self.measure("linear.activation_quantize"):
            if prologue is None:
                return quantize_fp8_rows(matrix, pad_to=16)
            tokens = prologue.scale.shape[0] if prologue.scale.ndim == 2 else 0
            if shape is not None and len(shape) >= 3 and tokens not in (1, shape[-2]):
                raise ValueError("FP8 prologue modulation tokens differ from the activation")
            if tokens < 1 or matrix.shape[0] % tokens:
                raise ValueError("FP8 prologue modulation tokens differ from the activation")
            return quantize_fp8_norm_modulate(matrix, prologue.norm_weight, prologue.eps, prologue.scale,
                                              prologue.shift, pad_to=16)

    def linear(self, value, weight, scale, bias=None, *, prologue: NormModulate | None = None):
        self._observe()
        self._validate(value, weight, scale, bias)
        if prologue is not None and self.mode != "w8a8":
            raise ValueError("fused FP8 prologues require the w8a8 mode")
        if self.mode == "weight-only":
            self.calls["weight_only"] += 1
            restored = (weight.float() * scale).to(value.dtype)
            return torch.nn.functional.linear(value, restored, bias)
        self._require_w8a8_device(value)
        self.calls["w8a8"] += 1
        shape = value.shape
        matrix = value.reshape(-1, shape[-1])
        rows = matrix.shape[0]
        codes, act_scale = self._quantize(matrix, prologue, shape)
        with self.measure("linear.fp8_gemm"):
            output = fp8_gemm(codes, act_scale, rows, weight, scale, Epilogue(bias=bias))
        return output.reshape(*shape[:-1], weight.shape[0])

    # -- fused entry points ------------------------------------------------------
    def _fused_prologue(self, value, weight, scale, bias):
        self._observe()
        self._validate(value, weight, scale, bias)
        if self.mode != "w8a8":
            raise ValueError("fused FP8 epilogues require the w8a8 mode")
        self._require_w8a8_device(value)
        self.calls["w8a8"] += 1
        matrix = value.reshape(-1, value.shape[-1])
        return value.shape, matrix, matrix.shape[0]

    def low_rank(self, value, down, up):
        """Unscaled low-rank residual ``linear(linear(value, down), up)`` in bf16.

        ``_residual_linear_unscaled`` (src/vflash/native/h3_native_denoiser.py:
        288-299) with both products on the tcgen05 pipeline (``vfb_bf16_gemm``):
        ``value`` bf16 ``[..., K]``, ``down`` ``[r, K]``, ``up`` ``[N, r]``;
        each product is rounded to bf16 as ``functional.linear`` rounds it.
        """
        shape, matrix = self._low_rank_input(value, down)
        low = bf16_gemm(matrix, down.to(device=value.device, dtype=torch.bfloat16).contiguous())
        out = bf16_gemm(low, up.to(device=value.device, dtype=torch.bfloat16).contiguous())
        return out.reshape(*shape[:-1], out.shape[-1])

    def qkv_low_rank(self, value, residuals) -> tuple:
        """The three QKV branches' unscaled low-rank outputs ``[rows, inner]``.

        The branches share their input, so their ``down`` matrices run as ONE
        GEMM over ``[3r, K]`` (the input is read once), then each branch's
        ``up`` reads its ``r`` columns of that product in place.
        """
        if len(residuals) != 3:
            raise ValueError("H3 QKV residual pack must contain three branches")
        downs = [r.down.to(device=value.device, dtype=torch.bfloat16) for r in residuals]
        rank = downs[0].shape[0]
        if any(d.shape != downs[0].shape for d in downs) or rank % 8:
            raise ValueError("QKV low-rank branches need one shared rank, a multiple of 8")
        _shape, matrix = self._low_rank_input(value, downs[0])
        low = bf16_gemm(matrix, torch.cat(downs, dim=0))
        return tuple(bf16_gemm(low[:, i * rank:(i + 1) * rank],
                               r.up.to(device=value.device, dtype=torch.bfloat16).contiguous())
                     for i, r in enumerate(residuals))

    @staticmethod
    def _low_rank_input(value, down):
        if value.dtype != torch.bfloat16 or value.shape[-1] != down.shape[-1] or value.device.type != "cuda":
            raise ValueError("low-rank branches take bf16 CUDA states matching their down matrix")
        matrix = value.reshape(-1, value.shape[-1])
        if matrix.stride(-1) != 1:
            matrix = matrix.contiguous()
        return value.shape, matrix

    def qkv_linear(self, value, weight, scale, bias=None, *, adapters=None, scalings=None,
                   prologue: NormModulate | None = None, qk_norm_rope: QKNormRope | None = None,
                   pack_chunks: int | None = None, head_dim: int = 128, residuals=None):
        """Merged QKV projection writing Q, K and V planes directly.

        With ``qk_norm_rope`` the Q and K planes also get the block's per-head
        RMSNorm and rotary embedding in the epilogue (one pass instead of
        ``_qk_norm_rotary``'s four launches).

        With ``pack_chunks`` the epilogue stores straight into the
        destination-major wire layout of ``pack_qkv(q, k, v, chunks=...)``
        (src/vflash/native/h3_parallel_relayout.py:214-256) and returns that
        one tensor, ``(chunks, 2, 3, *value.shape[:-1], heads / (2 chunks),
        head_dim)``, instead of the three planes: the pack pass before the
        sequence-head all-to-all disappears.

        ``residuals`` (three objects with ``down``, ``up`` and ``scaling``, as
        ``H3LowRankResidualWeights``) computes the branches' adapters with
        ``qkv_low_rank`` and merges them in the epilogue: the reference's
        ``_qkv_linear`` with residuals (h3_native_denoiser.py:301-316) end to
        end on the GPU, ``value`` being the projection's bf16 input.

        Equivalent to ``linear(value, weight, scale, bias).chunk(3, -1)``
        (src/vflash/native/h3_native_denoiser.py:541) followed, when
        ``adapters`` is given, by ``triton_strict_bf16_qkv_direct_merge``
        (src/vflash/native/h3_fused_ops.py:954-979): per branch
        ``bf16(base + bf16(adapter * scaling))``.  Returns three contiguous
        ``[..., N/3]`` tensors that are views of one ``[3, rows, N/3]`` buffer.
        """
        if residuals is not None:
            if adapters is not None or prologue is not None:
                raise ValueError("residuals replace adapters and need the materialised bf16 input")
            adapters = self.qkv_low_rank(value, residuals)
            scalings = tuple(float(r.scaling) for r in residuals)
        shape, matrix, rows = self._fused_prologue(value, weight, scale, bias)
        n = weight.shape[0]
        if n % 3:
            raise ValueError("merged QKV weight rows must be divisible by three")
        width = n // 3
        flat_adapters = None
        scales = (0.0, 0.0, 0.0)
        if adapters is not None:
            if (not isinstance(adapters, tuple) or len(adapters) != 3 or scalings is None
                    or len(scalings) != 3):
                raise ValueError("QKV merge requires three adapters and three scalings")
            flat_adapters = tuple(a.reshape(rows, width) for a in adapters)
            scales = tuple(float(s) for s in scalings)
        epilogue = Epilogue(bias=bias, planes=3, adapters=flat_adapters, scalings=scales)
        if pack_chunks is not None:
            if (not isinstance(pack_chunks, int) or pack_chunks < 1 or head_dim < 1
                    or width % (2 * pack_chunks * head_dim) or (width // (2 * pack_chunks)) % 32):
                raise ValueError("QKV heads must divide two destinations and all chunks")
            epilogue.wire_chunks = pack_chunks
        if qk_norm_rope is not None:
            tokens = qk_norm_rope.cos.shape[0] if qk_norm_rope.cos.ndim == 2 else 0
            if width % 128 or tokens < 1 or rows % tokens or (len(shape) >= 3 and tokens not in (1, shape[-2])):
                raise ValueError("FP8 QK-norm rotary needs 128-wide heads and cos/sin rows per token")
            epilogue.kind = _lib.EPI_QKV_NORM_ROPE
            epilogue.q_norm, epilogue.k_norm = qk_norm_rope.q_norm, qk_norm_rope.k_norm
            epilogue.rope_cos, epilogue.rope_sin = qk_norm_rope.cos, qk_norm_rope.sin
            epilogue.qk_eps = qk_norm_rope.eps
        codes, act_scale = self._quantize(matrix, prologue, shape)
        with self.measure("linear.fp8_gemm"):
            planes = fp8_gemm(codes, act_scale, rows, weight, scale, epilogue)
        if pack_chunks is not None:
            per_chunk = width // (2 * pack_chunks)
            return planes.view(pack_chunks, 2, 3, *shape[:-1], per_chunk // head_dim, head_dim)
        return tuple(planes[i].reshape(*shape[:-1], width) for i in range(3))

    def gelu_linear(self, value, weight, scale, bias=None, *, prologue: NormModulate | None = None):
        """``F.gelu(linear(...), approximate="tanh")`` with the GELU in the epilogue."""
        shape, matrix, rows = self._fused_prologue(value, weight, scale, bias)
        codes, act_scale = self._quantize(matrix, prologue, shape)
        with self.measure("linear.fp8_gemm"):
            out = fp8_gemm(codes, act_scale, rows, weight, scale,
                           Epilogue(kind=_lib.EPI_GELU_TANH, bias=bias))
        return out.reshape(*shape[:-1], weight.shape[0])

    def swiglu_linear(self, value, weight, scale, bias=None, *, prologue: NormModulate | None = None):
        """Packed FFN input projection with ``value * bf16(silu(gate))`` fused.

        ``weight`` is the packed ``[2F, K]`` ffn_in matrix (value rows first,
        src/vflash/native/h3_native_denoiser.py:369-373); the result equals
        ``triton_strict_bf16_silu_mul(linear(...))`` and has width F.
        """
        shape, matrix, rows = self._fused_prologue(value, weight, scale, bias)
        if weight.shape[0] % 64:
            raise ValueError("packed SwiGLU weight needs 2F rows with F % 32 == 0")
        codes, act_scale = self._quantize(matrix, prologue, shape)
        with self.measure("linear.fp8_gemm"):
            out = fp8_gemm(codes, act_scale, rows, weight, scale,
                           Epilogue(kind=_lib.EPI_SWIGLU, bias=bias))
        return out.reshape(*shape[:-1], weight.shape[0] // 2)

    def gate_residual_linear(self, value, weight, scale, residual, gate=None, bias=None):
        """``residual + bf16(gate * linear(...))`` fused (gate optional).

        Matches ``triton_strict_bf16_gate_residual`` (h3_fused_ops.py:614-657)
        applied to the linear output: ``residual`` is ``[B, S, N]`` and
        ``gate`` ``[S, N]`` indexed by token; without ``gate`` it is a plain
        BF16 residual add.
        """
        shape, matrix, rows = self._fused_prologue(value, weight, scale, bias)
        n = weight.shape[0]
        if residual.dtype != torch.bfloat16 or residual.shape != (*shape[:-1], n):
            raise ValueError("FP8 residual differs from the declared output")
        res = residual.reshape(rows, n)
        tokens = 0
        if gate is not None:
            if gate.dtype != torch.bfloat16 or gate.ndim != 2 or gate.shape[1] != n:
                raise ValueError("FP8 gate must be BF16 [S, N]")
            tokens = gate.shape[0]
            if len(shape) < 2 or shape[-2] != tokens:
                raise ValueError("FP8 gate tokens differ from the activation")
        codes, act_scale = self._quantize(matrix)
        with self.measure("linear.fp8_gemm"):
            out = fp8_gemm(codes, act_scale, rows, weight, scale,
                           Epilogue(kind=_lib.EPI_RESIDUAL, bias=bias, residual=res, gate=gate,
                                    tokens=tokens))
        return out.reshape(*shape[:-1], n)

    def ffn(self, value, up_weight, up_scale, down_weight, down_scale, *, activation="gelu_tanh",
            up_bias=None, down_bias=None, residual=None, gate=None, prologue: NormModulate | None = None,
            one_kernel: bool = False):
        """Fused FFN: up GEMM + activation -> per-token e4m3 requant -> down GEMM.

        ``activation`` is ``"gelu_tanh"`` (up weight ``[F, H]``) or ``"swiglu"``
        (packed up weight ``[2F, H]``).  The down GEMM's epilogue adds
        ``residual`` (and multiplies by ``gate`` first) when given.  The
        intermediate is requantised per token over its full row, exactly as
        the reference quantises the activation of the next linear
        (src/vflash/native/h3_fp8_activation.py:16-19).  One native call
        (``vfb_fp8_ffn``, or ``vfb_fp8_ffn_quantized`` after a fused
        ``prologue``) that runs the up GEMM, the requantisation and the down
        GEMM as three launches; ``one_kernel=True`` (no prologue) runs them as
        one persistent kernel (``vfb_fp8_ffn_one_kernel``, same bits, slower
        than the three launches on the B200 at every M measured).
        """
        if (
            down_weight.ndim != 2
            or down_weight.dtype != torch.float8_e4m3fn
            or down_scale.dtype != torch.float32
            or down_scale.shape != (down_weight.shape[0], 1)
            or down_weight.device != value.device
            or down_scale.device != value.device
        ):
            raise ValueError("FP8 codes/scales differ from the declared layout")
        if down_bias is not None and (
            down_bias.shape != (down_weight.shape[0],)
            or down_bias.device != value.device
            or down_bias.dtype != value.dtype
        ):
            raise ValueError("FP8 bias differs from the declared output")
        if activation not in ("gelu_tanh", "swiglu"):
            raise ValueError("unknown FFN activation")
        shape, matrix, rows = self._fused_prologue(value, up_weight, up_scale, up_bias)
        hidden = down_weight.shape[0]
        width = up_weight.shape[0] // 2 if activation == "swiglu" else up_weight.shape[0]
        if width != down_weight.shape[1]:
            raise ValueError("FFN down weight differs from the intermediate width")
        if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != (*shape[:-1], hidden)):
            raise ValueError("FP8 residual differs from the declared output")
        kind = _lib.EPI_SWIGLU if activation == "swiglu" else _lib.EPI_GELU_TANH
        args = dict(activation=kind, up_bias=up_bias, down_bias=down_bias,
                    residual=None if residual is None else residual.reshape(rows, hidden), gate=gate)
        self.calls["w8a8"] += 1  # the FFN's second linear
        if prologue is None:
            with self.measure("linear.fp8_gemm"):
                out = fp8_ffn(matrix, up_weight, up_scale, down_weight, down_scale, one_kernel=one_kernel, **args)
        else:
            if one_kernel:
                raise ValueError("the one-kernel FFN takes the unquantised input (no prologue)")
            codes, act_scale = self._quantize(matrix, prologue, shape)
            with self.measure("linear.fp8_gemm"):
                out = fp8_ffn_quantized(codes, act_scale, rows, up_weight, up_scale, down_weight, down_scale,
                                        **args)
        return out.reshape(*shape[:-1], hidden)


class RowFP8Linear(torch.nn.Module):
    """Meta-initialized Linear replacement; assign trusted codes and row_scale.

    The original bias is preserved. A loader must assign all meta tensors before
    execution, and retain the intended host/device placement of each module.
    (Hansimov/vflash src/vflash/native/h3_fp8_linear.py:124-149.)
    """

    def __init__(self, original: torch.nn.Linear, execution: RowFP8Execution):
        super().__init__()
        self.in_features = original.in_features
        self.out_features = original.out_features
        self.weight = torch.nn.Parameter(
            torch.empty(
                (self.out_features, self.in_features), device="meta", dtype=torch.float8_e4m3fn
            ),
            requires_grad=False,
        )
        self.register_buffer(
            "row_scale",
            torch.empty((self.out_features, 1), device="meta", dtype=torch.float32),
        )
        self.bias = original.bias
        self.execution = execution

    def forward(self, value):
        return self.execution.linear(value, self.weight, self.row_scale, self.bias)
