"""Explicit NVFP4 arithmetic for the packed H3 QAD linear contract on SM100 (drop-in).

Mirrors Hansimov/vflash src/vflash/native/h3_nvfp4_linear.py: the frozen
``NVFP4Weight`` layout contract (packed e2m1 ``[N, K/2]`` with element 2i in
the low nibble, ue4m3 block scales ``[N, K/16]`` in the 128x4 layout, fp32
``alpha`` and ``input_scale`` scalars), ``NVFP4Execution.linear`` with its
validation, counters and single ``_require_device`` / ``_operators`` hooks.
``_operators()`` returns the native quantiser and GEMM behind the same
call signatures the reference uses for FlashInfer's ``nvfp4_quantize`` and
``mm_fp4`` (h3_nvfp4_linear.py:61-64, 102, 118-130), so callers and the
reference's tests see the same plumbing; the device gate is SM100.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import cache

import torch

from .. import _lib
from ..kernels import Epilogue, nvfp4_gemm, nvfp4_norm_modulate_quantize, nvfp4_quantize
from .h3_fp8_linear import NormModulate

SF_LAYOUT_128x4 = "128x4"


@dataclass(frozen=True, eq=False)
class NVFP4Weight:
    packed: torch.Tensor
    scales: torch.Tensor
    alpha: torch.Tensor
    input_scale: torch.Tensor

    def __post_init__(self):
        if (
            self.packed.dtype != torch.uint8
            or self.packed.ndim != 2
            or min(self.packed.shape) < 1
            or self.packed.shape[0] % 128
            or self.packed.shape[1] % 32
            or self.scales.dtype != torch.uint8
            or self.scales.shape != (self.packed.shape[0], self.packed.shape[1] // 8)
            or not self.packed.is_contiguous()
            or not self.scales.is_contiguous()
        ):
            raise ValueError("NVFP4 requires declared packed codes and 128x4 block scales")
        for scalar in (self.alpha, self.input_scale):
            if scalar.dtype != torch.float32 or scalar.shape != torch.Size([]):
                raise ValueError("NVFP4 calibration and output alpha must be FP32 scalars")
            if scalar.device.type != "meta" and not bool(torch.isfinite(scalar) & (scalar > 0)):
                raise ValueError("NVFP4 scales must be positive and finite")
        if len({v.device for v in (self.packed, self.scales, self.alpha, self.input_scale)}) != 1:
            raise ValueError("NVFP4 tensors must share one explicit device")

    @property
    def in_features(self):
        return self.packed.shape[1] * 2

    @property
    def out_features(self):
        return self.packed.shape[0]


@cache
def _require_device(device):
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise ValueError("This NVFP4 execution requires an explicit SM100 CUDA device")


def _quantize(matrix, global_sf, *, sfLayout, do_shuffle):  # noqa: N803 - reference keyword names
    """``nvfp4_quantize`` contract: 128x4 scales, no shuffle."""
    if sfLayout != SF_LAYOUT_128x4 or do_shuffle:
        raise ValueError("only the 128x4 unshuffled scale layout is supported")
    return nvfp4_quantize(matrix, global_sf)


def _matmul(a, b, a_scale, b_scale, alpha, out_dtype, out, *, block_size, use_8x4_sf_layout,
            backend, use_nvfp4):
    """``mm_fp4`` contract: ``b``/``b_scale`` are the transposed weight views."""
    if (block_size != 16 or use_8x4_sf_layout or not use_nvfp4 or out_dtype != torch.bfloat16
            or out is not None or backend != "cutlass"):
        raise ValueError("only the NVFP4 block-16 128x4 bf16 contract is supported")
    return nvfp4_gemm(a, a_scale, b.T, b_scale.T, alpha)


def _operators():
    return SF_LAYOUT_128x4, _quantize, _matmul


class NVFP4Execution:
    """Frozen W4A4 execution on SM100; host clocks/counters remain diagnostic."""

    contract = "nvfp4-e2m1-block16-128x4-cutlass-v1"

    def __init__(self):
        self.calls = 0
        self.rows = 0
        self._ops = None

    def linear(self, values, weight: NVFP4Weight, bias=None, *, prologue: NormModulate | None = None):
        """``bf16(mm_fp4(nvfp4_quantize(values), W) * alpha / input_scale) + bias``.

        With the native operators the division of the two calibration scalars
        and the bias add run inside the GEMM's epilogue (one quantiser launch
        and one GEMM launch per call); operators supplied through
        ``_operators`` (e.g. a test's fakes) get the reference's call
        sequence and arguments (h3_nvfp4_linear.py:100-139).

        ``prologue`` (native operators only): ``values`` is the block's
        un-normalised hidden state, and the quantiser applies its RMSNorm and
        AdaLN modulate first, in the same pass (``vfb_nvfp4_norm_modulate_quant``);
        the result equals ``linear(modulated)`` bit for bit.
        """
        return self._run(values, weight, bias, Epilogue(bias=bias), prologue=prologue)

    def _quantize_input(self, matrix, weight: NVFP4Weight, prologue):
        if prologue is None:
            return nvfp4_quantize(matrix, weight.input_scale)
        return nvfp4_norm_modulate_quantize(matrix, prologue.norm_weight, prologue.eps, prologue.scale,
                                            prologue.shift, weight.input_scale)

    def _run(self, values, weight: NVFP4Weight, bias, epilogue: Epilogue, out_features=None, prologue=None):
        if (
            values.ndim < 1
            or values.shape[-1] != weight.in_features
            or values.dtype not in (torch.bfloat16, torch.float16, torch.float32)
            or values.device != weight.packed.device
        ):
            raise ValueError("NVFP4 input differs from its frozen matrix")
        if torch.is_grad_enabled() and values.requires_grad:
            raise ValueError("NVFP4 execution is inference-only")
        _require_device(values.device)
        if bias is not None and (
            bias.shape != (weight.out_features,)
            or bias.device != values.device
            or bias.dtype != torch.bfloat16
        ):
            raise ValueError("NVFP4 bias must match its BF16 output")
        if self._ops is None:
            self._ops = _operators()
        layout, quantize, matmul = self._ops
        shape = values.shape
        matrix = values.to(torch.bfloat16) if values.dtype == torch.float32 else values
        matrix = matrix.reshape(-1, weight.in_features)
        if matrix.shape[0] == 0:
            raise ValueError("NVFP4 input rows must be nonempty")
        if prologue is not None:
            if matmul is not _matmul or values.dtype != torch.bfloat16:
                raise ValueError("the NVFP4 norm/modulate prologue needs the native operators and bf16 input")
            codes, scales = self._quantize_input(matrix, weight, prologue)
        else:
            codes, scales = quantize(matrix, weight.input_scale, sfLayout=layout, do_shuffle=False)
        padded_rows = matrix.shape[0] + (-matrix.shape[0]) % 128
        padded_columns = (weight.in_features // 16 + 3) // 4 * 4
        if (
            scales.dtype != torch.uint8
            or scales.device != matrix.device
            or scales.numel() != padded_rows * padded_columns
        ):
            raise ValueError("The quantizer omitted the required 128x4 scale padding")
        if codes.dtype != torch.uint8 or codes.shape != (matrix.shape[0], weight.in_features // 2):
            raise ValueError("The quantizer returned a different packed layout")
        width = out_features or weight.out_features
        if matmul is _matmul:
            output = nvfp4_gemm(codes, scales, weight.packed, weight.scales, weight.alpha,
                                alpha_div=weight.input_scale, epilogue=epilogue)
            self.calls += 1
            self.rows += matrix.shape[0]
            if isinstance(output, torch.Tensor) and output.ndim == 3:  # Q, K, V planes
                return tuple(output[i].reshape(*shape[:-1], output.shape[-1]) for i in range(output.shape[0]))
            if output.dtype != torch.bfloat16 or output.shape != (matrix.shape[0], width):
                raise ValueError("The NVFP4 kernel returned a different output layout")
            return output.reshape(*shape[:-1], width)
        if epilogue.kind != _lib.EPI_STORE or epilogue.planes != 1 or epilogue.adapters is not None:
            raise ValueError("fused NVFP4 epilogues need the native operators")
        output = matmul(
            codes,
            weight.packed.T,
            scales,
            weight.scales.T,
            weight.alpha / weight.input_scale,
            torch.bfloat16,
            None,
            block_size=16,
            use_8x4_sf_layout=False,
            backend="cutlass",
            use_nvfp4=True,
        )
        if output.dtype != torch.bfloat16 or output.shape != (matrix.shape[0], weight.out_features):
            raise ValueError("The NVFP4 kernel returned a different output layout")
        self.calls += 1
        self.rows += matrix.shape[0]
        output = output.reshape(*shape[:-1], weight.out_features)
        return output if bias is None else output + bias

    # -- fused entry points (opt-in): the strict-BF16 step after the linear runs
    # in the GEMM's epilogue, as for RowFP8Execution
    def _check_bias(self, values, bias, n):
        if bias is not None and (bias.shape != (n,) or bias.device != values.device
                                 or bias.dtype != torch.bfloat16):
            raise ValueError("NVFP4 bias must match its BF16 output")

    def gelu_linear(self, values, weight: NVFP4Weight, bias=None, *, prologue: NormModulate | None = None):
        """``F.gelu(linear(values, weight, bias), approximate="tanh")`` with the GELU in the epilogue."""
        self._check_bias(values, bias, weight.out_features)
        return self._run(values, weight, bias, Epilogue(kind=_lib.EPI_GELU_TANH, bias=bias), prologue=prologue)

    def swiglu_linear(self, values, weight: NVFP4Weight, bias=None, *, prologue: NormModulate | None = None):
        """Packed FFN input ``[2F, K]`` with ``value * bf16(silu(gate))`` fused (h3_fused_ops.py:185-224)."""
        if weight.out_features % 256:
            raise ValueError("packed NVFP4 SwiGLU weight needs 2F rows with F % 128 == 0")
        self._check_bias(values, bias, weight.out_features)
        return self._run(values, weight, bias, Epilogue(kind=_lib.EPI_SWIGLU, bias=bias),
                         out_features=weight.out_features // 2, prologue=prologue)

    def gate_residual_linear(self, values, weight: NVFP4Weight, residual, gate=None, bias=None):
        """``residual + bf16(gate * linear(...))`` fused (h3_fused_ops.py:125-170); gate ``[tokens, N]``."""
        self._check_bias(values, bias, weight.out_features)
        n = weight.out_features
        if (residual.dtype != torch.bfloat16 or residual.shape != (*values.shape[:-1], n)
                or residual.device != values.device):
            raise ValueError("NVFP4 residual differs from the declared output")
        if gate is not None and (gate.dtype != torch.bfloat16 or gate.ndim != 2 or gate.shape[1] != n):
            raise ValueError("NVFP4 gate must be bf16 [tokens, N]")
        ep = Epilogue(kind=_lib.EPI_RESIDUAL, bias=bias, residual=residual.reshape(-1, n), gate=gate,
                      tokens=0 if gate is None else gate.shape[0])
        return self._run(values, weight, bias, ep)

    def qkv_linear(self, values, weight: NVFP4Weight, bias=None, *, adapters=None, scalings=None,
                   prologue: NormModulate | None = None):
        """Merged QKV: the Q, K, V planes of one GEMM, optionally each merged with its LoRA branch.

        ``adapters`` (three bf16 ``[..., N/3]`` tensors or None) and
        ``scalings`` follow triton_strict_bf16_qkv_direct_merge
        (h3_fused_ops.py:901-979): plane = bf16(plane + bf16(adapter * s)).
        """
        n = weight.out_features
        if n % 96:
            raise ValueError("merged NVFP4 QKV needs three planes of a multiple of 32 columns")
        self._check_bias(values, bias, n)
        flat = None
        if adapters is not None:
            if scalings is None or len(adapters) != 3 or len(scalings) != 3:
                raise ValueError("QKV adapters need three branches and three scalings")
            flat = tuple(None if a is None else a.reshape(-1, n // 3) for a in adapters)
        ep = Epilogue(bias=bias, planes=3, adapters=flat, scalings=tuple(scalings or (0.0, 0.0, 0.0)))
        return self._run(values, weight, bias, ep, prologue=prologue)

    def ffn(self, values, up: NVFP4Weight, down: NVFP4Weight, *, activation="gelu_tanh", up_bias=None,
            down_bias=None, residual=None, gate=None, prologue: NormModulate | None = None):
        """The QAD FFN ``down(act(up(values)))``, optionally with a gated residual.

        The same bits as ``linear(gelu_linear(values, up, up_bias), down, down_bias)``
        (``swiglu_linear`` for ``activation="swiglu"`` over the packed ``[2F, K]``
        up weight; ``gate_residual_linear`` when ``residual`` is given), but the
        up GEMM's epilogue quantises its bf16 result with ``down.input_scale``
        exactly as the down linear's quantiser would, so the intermediate never
        exists in bf16: three launches (quantiser, up GEMM, down GEMM) and no
        intermediate round trip through HBM.  ``prologue`` applies the block's
        norm and modulate to ``values`` inside the first quantiser.
        """
        if activation not in ("gelu_tanh", "swiglu"):
            raise ValueError("NVFP4 FFN activation must be gelu_tanh or swiglu")
        width = up.out_features // 2 if activation == "swiglu" else up.out_features
        if activation == "swiglu" and up.out_features % 256:
            raise ValueError("packed NVFP4 SwiGLU weight needs 2F rows with F % 128 == 0")
        if down.in_features != width or width % 64:
            raise ValueError("NVFP4 FFN weights differ: down.in_features must be the activation width")
        if (values.ndim < 1 or values.shape[-1] != up.in_features
                or values.dtype not in (torch.bfloat16, torch.float16, torch.float32)
                or values.device != up.packed.device or down.packed.device != up.packed.device):
            raise ValueError("NVFP4 input differs from its frozen matrix")
        if torch.is_grad_enabled() and values.requires_grad:
            raise ValueError("NVFP4 execution is inference-only")
        _require_device(values.device)
        self._check_bias(values, up_bias, up.out_features)
        self._check_bias(values, down_bias, down.out_features)
        n = down.out_features
        if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != (*values.shape[:-1], n)
                                     or residual.device != values.device):
            raise ValueError("NVFP4 residual differs from the declared output")
        if gate is not None and (residual is None or gate.dtype != torch.bfloat16 or gate.ndim != 2
                                 or gate.shape[1] != n):
            raise ValueError("NVFP4 gate must be bf16 [tokens, N] with a residual")
        if self._ops is None:
            self._ops = _operators()
        if self._ops[2] is not _matmul:
            raise ValueError("the fused NVFP4 FFN needs the native operators")
        shape = values.shape
        matrix = values.to(torch.bfloat16) if values.dtype == torch.float32 else values
        matrix = matrix.reshape(-1, up.in_features)
        if matrix.shape[0] == 0:
            raise ValueError("NVFP4 input rows must be nonempty")
        if prologue is not None and values.dtype != torch.bfloat16:
            raise ValueError("the NVFP4 norm/modulate prologue needs bf16 input")
        codes, scales = self._quantize_input(matrix, up, prologue)
        kind = _lib.EPI_SWIGLU if activation == "swiglu" else _lib.EPI_GELU_TANH
        mid_codes, mid_scales = nvfp4_gemm(codes, scales, up.packed, up.scales, up.alpha, alpha_div=up.input_scale,
                                           epilogue=Epilogue(kind=kind, bias=up_bias),
                                           quantize_output=down.input_scale)
        if residual is None:
            ep = Epilogue(bias=down_bias)
        else:
            ep = Epilogue(kind=_lib.EPI_RESIDUAL, bias=down_bias, residual=residual.reshape(-1, n), gate=gate,
                          tokens=0 if gate is None else gate.shape[0])
        out = nvfp4_gemm(mid_codes, mid_scales, down.packed, down.scales, down.alpha, alpha_div=down.input_scale,
                         epilogue=ep)
        self.calls += 2
        self.rows += 2 * matrix.shape[0]
        return out.reshape(*shape[:-1], n)
