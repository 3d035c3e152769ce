"""Generate the golden vectors in this directory from the reference implementation.

Run in a container that has the reference checkout (Hansimov/vflash):

    python tests/golden/make_golden.py --reference-src <vflash checkout>/src

It imports the reference's own CPU code and freezes its outputs:

* ``_quantize_activation_torch`` (src/vflash/native/h3_fp8_linear.py:18-31) on
  seeded inputs, including the padding / zero-row / bf16.tiny / strided-view
  cases of the reference test tests/test_fp8_linear.py:99-120, rounding ties
  and bf16 subnormals, non-finite and signed-zero rows -> e4m3 codes and fp32
  scales (bit-exact fixtures);
* ``RowFP8Execution("weight-only").linear`` (h3_fp8_linear.py:88-91) on the
  reference test's fixture weights (tests/test_fp8_linear.py:13-16) and on a
  seeded mid-size case;
* the eager BF16 compositions that the reference's strict fused kernels are
  written to reproduce (src/vflash/native/h3_fused_ops.py module docstring and
  kernels at 125-224, 901-949): value*silu(gate), residual + gate*projected,
  base + adapter*scaling, and torch's tanh-GELU on a linear output;
* ``pack_qkv_reference`` (src/vflash/native/h3_parallel_relayout.py:214-222),
  the destination-major wire layout of the QKV planes.

Nothing at test time reads the reference: the tests load the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bits(t):
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def u8(t):
    import torch

    return t.contiguous().view(torch.uint8).numpy().copy()


def outlier_matrix(rows, cols, seed):
    """N(0,1) with round(0.001*rows*cols) entries scaled x20, then bf16."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=gen)
    count = round(0.001 * rows * cols)
    if count:
        idx = torch.randperm(rows * cols, generator=torch.Generator().manual_seed(seed + 1))[:count]
        x.view(-1)[idx] *= 20
    return x.to(torch.bfloat16)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", required=True, help="the src/ directory of a vflash checkout")
    parser.add_argument("--out", default=str(HERE / "fp8_golden.npz"), help="where to write the fixture")
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    import torch
    from vflash.native.h3_fp8_linear import RowFP8Execution, _quantize_activation_torch

    out: dict[str, np.ndarray] = {}

    def quant_case(name, matrix):
        codes, scales = _quantize_activation_torch(matrix)
        out[f"q_{name}_x"] = bits(matrix)
        out[f"q_{name}_codes"] = u8(codes)
        out[f"q_{name}_scales"] = scales.numpy().copy()

    quant_case("outliers", outlier_matrix(37, 512, 1000))
    quant_case("wide", outlier_matrix(5, 4096, 1001))
    quant_case("k16", outlier_matrix(3, 16, 1002))
    quant_case("k24", outlier_matrix(18, 24, 1003))
    quant_case("k40", outlier_matrix(17, 40, 1004))
    for rows in (1, 16, 17):
        # tests/test_fp8_linear.py:99-120: value half of an FFN projection with
        # a doubled physical row stride; zero row; bf16.tiny row.
        base = torch.full((rows, 128), float("nan"), dtype=torch.bfloat16)
        values = base[:, :64]
        values.copy_(torch.linspace(-448, 448, 64))
        values[0].zero_()
        if rows > 1:
            values[1].fill_(torch.finfo(torch.bfloat16).tiny)
        codes, scales = _quantize_activation_torch(values)
        out[f"q_strided{rows}_base"] = bits(base)
        out[f"q_strided{rows}_codes"] = u8(codes)
        out[f"q_strided{rows}_scales"] = scales.numpy().copy()
    # rounding ties of e4m3 (normal and subnormal) with scale exactly 1 (amax 448)
    ties = torch.tensor(
        [448.0, 1.0625, 1.1875, -1.0625, 3.25, 2.0**-10, 3 * 2.0**-10, -5 * 2.0**-10,
         2.0**-6 * 1.0625, 240.0, 232.0, -0.0, 0.0, 7.5 * 2.0**-9, 0.015625, 300.0],
        dtype=torch.float32).to(torch.bfloat16).reshape(1, 16)
    quant_case("ties", ties)
    # bf16 subnormal magnitudes (amax / 448 underflows to the FLT_MIN clamp)
    sub = torch.tensor([2.0**-133, -(2.0**-130), 2.0**-127, 3 * 2.0**-133] * 4,
                       dtype=torch.float32).to(torch.bfloat16).reshape(2, 8)
    quant_case("subnormal", sub)
    quant_case("zeros", torch.zeros(3, 32, dtype=torch.bfloat16))
    # non-finite and signed-zero rows: an inf makes the row's scale inf (finite values -> 0,
    # infinities -> NaN), a NaN makes amax NaN and the scale 1, an all -0 row keeps -0 codes;
    # the largest bf16 magnitudes give a finite scale
    inf, nan = float("inf"), float("nan")
    specials = torch.tensor(
        [[1.0, inf, -2.0, 0.5] * 4,
         [-inf, 3.0, -0.0, 1e-3] * 4,
         [nan, 1.0, -448.0, 2.5] * 4,
         [inf, -inf, nan, 0.0] * 4,
         [3.3e38, -1.0, -0.0, 1e-38] * 4,
         [-0.0] * 16],
        dtype=torch.float32).to(torch.bfloat16)
    quant_case("specials", specials)

    # weight-only linear, reference fixture weights
    codes = torch.arange(128).reshape(16, 8).to(torch.float8_e4m3fn)
    scales = torch.linspace(0.01, 0.1, 16).unsqueeze(1)
    gen = torch.Generator().manual_seed(7)
    value = torch.randn(3, 8, generator=gen).to(torch.bfloat16)
    bias = torch.randn(16, generator=gen).to(torch.bfloat16)
    y = RowFP8Execution().linear(value, codes, scales, bias)
    out["wo_small_x"] = bits(value)
    out["wo_small_codes"] = u8(codes)
    out["wo_small_scales"] = scales.numpy().copy()
    out["wo_small_bias"] = bits(bias)
    out["wo_small_y"] = bits(y)
    # seeded mid-size case, weights quantised per output row
    x = outlier_matrix(33, 256, 1010)
    gen = torch.Generator().manual_seed(2010)
    w = (torch.randn(64, 256, generator=gen) * 0.02).to(torch.bfloat16)
    wc, ws = _quantize_activation_torch(w)
    wc, ws = wc[:64], ws[:64]
    bias = (torch.randn(64, generator=torch.Generator().manual_seed(3010)) * 0.01).to(torch.bfloat16)
    y = RowFP8Execution().linear(x, wc, ws, bias)
    out["wo_mid_x"] = bits(x)
    out["wo_mid_w"] = bits(w)
    out["wo_mid_codes"] = u8(wc)
    out["wo_mid_scales"] = ws.numpy().copy()
    out["wo_mid_bias"] = bits(bias)
    out["wo_mid_y"] = bits(y)

    # eager BF16 compositions reproduced by the strict fused kernels
    gen = torch.Generator().manual_seed(11)
    packed = (torch.randn(3, 7, 128, generator=gen) * 3).to(torch.bfloat16)
    value, gate = packed.chunk(2, dim=-1)
    out["silu_packed"] = bits(packed)
    out["silu_out"] = bits(value * torch.nn.functional.silu(gate))
    y = (torch.randn(9, 64, generator=gen) * 2).to(torch.bfloat16)
    out["gelu_y"] = bits(y)
    out["gelu_out"] = bits(torch.nn.functional.gelu(y, approximate="tanh"))
    residual = torch.randn(2, 5, 64, generator=gen).to(torch.bfloat16)
    gate = torch.randn(5, 64, generator=gen).to(torch.bfloat16)
    projected = torch.randn(2, 5, 64, generator=gen).to(torch.bfloat16)
    out["gr_residual"] = bits(residual)
    out["gr_gate"] = bits(gate)
    out["gr_projected"] = bits(projected)
    out["gr_out"] = bits(residual + gate * projected)
    base = torch.randn(2, 5, 96, generator=gen).to(torch.bfloat16)
    adapters = [torch.randn(2, 5, 32, generator=gen).to(torch.bfloat16) for _ in range(3)]
    scalings = (0.0625, 0.5, -1.25)
    merged = torch.cat([b + a * s for b, a, s in zip(base.chunk(3, dim=-1), adapters, scalings)], -1)
    out["qkv_base"] = bits(base)
    out["qkv_adapters"] = np.stack([bits(a) for a in adapters])
    out["qkv_scalings"] = np.asarray(scalings, dtype=np.float32)
    out["qkv_out"] = bits(merged)

    # the destination-major QKV wire layout (src/vflash/native/h3_parallel_relayout.py:214-222)
    from vflash.native.h3_parallel_relayout import pack_qkv_reference

    gen = torch.Generator().manual_seed(12)
    for chunks in (1, 2):
        qkv = [torch.randn(2, 3, 8, 4, generator=gen).to(torch.bfloat16) for _ in range(3)]
        out[f"pack{chunks}_qkv"] = np.stack([bits(t) for t in qkv])
        out[f"pack{chunks}_out"] = bits(pack_qkv_reference(*qkv, chunks=chunks))

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} with {len(out)} arrays")


if __name__ == "__main__":
    main()
