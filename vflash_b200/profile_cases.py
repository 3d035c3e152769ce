"""Small, self-checking runs of one hot-path kernel, for profilers.

``bench.py`` times the full configurations; a detailed profiler capture
replays each launch dozens of times, so it runs on a smaller case of the same
kernel.  This module runs such a case a fixed number of times on ``cuda:0``
with seeded synthetic inputs and exits non-zero when the library reports a
device error or the output is not finite::

    python -m vflash_b200.profile_cases fp8_gemm --rows 4096
    python -m vflash_b200.profile_cases fp8_gemm_gelu --rows 8192
    python -m vflash_b200.profile_cases ffn --rows 8192 [--swiglu] [--one-kernel]
    python -m vflash_b200.profile_cases nvfp4_gemm --rows 8192 --n 4096
    python -m vflash_b200.profile_cases bf16_up --rows 32760

Shapes other than the row count are those of the benchmark configurations:
the merged QKV projection (N = 12288, K = 4096), the FFN (H = 4096,
F = 16384; ``fp8_gemm_gelu`` is its up projection alone), the NVFP4
linear (K = 4096) and a rank-32 low-rank up product (bf16, K = 32,
N = 4096).
"""

from __future__ import annotations

import argparse
import sys

import torch

from . import _lib
from .kernels import Epilogue, bf16_gemm, fp8_ffn, fp8_gemm, nvfp4_gemm, nvfp4_quantize, quantize_fp8_rows


def _seeded(rows: int, cols: int, seed: int, std: float, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(rows, cols, generator=g, device=device) * std).to(torch.bfloat16)


def run(case: str, rows: int, repeats: int, n: int = 4096, swiglu: bool = False,
        one_kernel: bool = False) -> torch.Tensor:
    device = torch.device("cuda", 0)
    if case == "fp8_gemm":
        x = _seeded(rows, 4096, 1, 1.0, device)
        w, ws = quantize_fp8_rows(_seeded(12288, 4096, 2, 0.02, device), pad_to=1)
        bias = _seeded(1, 12288, 3, 0.01, device).reshape(-1)
        codes, scales = quantize_fp8_rows(x)
        for _ in range(repeats):
            y = fp8_gemm(codes, scales, rows, w, ws, Epilogue(bias=bias, planes=3))
    elif case == "fp8_gemm_gelu":
        # the FFN's up projection (F = 16384) with the GELU-tanh epilogue
        x = _seeded(rows, 4096, 1, 1.0, device)
        w, ws = quantize_fp8_rows(_seeded(16384, 4096, 2, 0.02, device), pad_to=1)
        codes, scales = quantize_fp8_rows(x)
        for _ in range(repeats):
            y = fp8_gemm(codes, scales, rows, w, ws, Epilogue(kind=_lib.EPI_GELU_TANH))
    elif case == "ffn":
        h, f = 4096, 16384
        x = _seeded(rows, h, 1, 1.0, device)
        n_up = 2 * f if swiglu else f
        up, ups = quantize_fp8_rows(_seeded(n_up, h, 2, 0.02, device), pad_to=1)
        down, downs = quantize_fp8_rows(_seeded(h, f, 3, 0.02, device), pad_to=1)
        kind = _lib.EPI_SWIGLU if swiglu else _lib.EPI_GELU_TANH
        for _ in range(repeats):
            y = fp8_ffn(x, up, ups, down, downs, activation=kind, residual=x, one_kernel=one_kernel)
    elif case == "nvfp4_gemm":
        x = _seeded(rows, 4096, 1, 1.0, device)
        w = _seeded(n, 4096, 2, 0.02, device)
        gsf_x = (448.0 * 6.0 / x.float().abs().max()).reshape(())
        gsf_w = (448.0 * 6.0 / w.float().abs().max()).reshape(())
        wp, wsc = nvfp4_quantize(w, gsf_w)
        alpha = ((1.0 / gsf_w) / gsf_x).to(torch.float32)
        ac, asf = nvfp4_quantize(x, gsf_x)
        for _ in range(repeats):
            y = nvfp4_gemm(ac, asf, wp, wsc.view(n, 4096 // 16), alpha)
    elif case == "bf16_up":
        # a low-rank adapter's up product: [rows, 32] x [4096, 32]^T, bound by its output writes
        lo = _seeded(rows, 32, 1, 1.0, device)
        up = _seeded(4096, 32, 2, 0.02, device)
        for _ in range(repeats):
            y = bf16_gemm(lo, up)
    else:
        raise ValueError(f"unknown case {case!r}")
    torch.cuda.synchronize(device)
    return y


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("case", choices=["fp8_gemm", "fp8_gemm_gelu", "ffn", "nvfp4_gemm", "bf16_up"])
    parser.add_argument("--rows", type=int, default=4096)
    parser.add_argument("--n", type=int, default=4096, help="NVFP4 output features")
    parser.add_argument("--repeats", type=int, default=3)
    parser.add_argument("--swiglu", action="store_true")
    parser.add_argument("--one-kernel", action="store_true")
    args = parser.parse_args(argv)
    y = run(args.case, args.rows, args.repeats, args.n, args.swiglu, args.one_kernel)
    status = _lib.device_status(clear=True)
    finite = bool(torch.isfinite(y.float()).all())
    print(f"{args.case} rows={args.rows} status={status} finite={finite}")
    return 0 if status == 0 and finite else 1


if __name__ == "__main__":
    sys.exit(main())
