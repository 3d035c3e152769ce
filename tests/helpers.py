"""Shared helpers for the parity tests: seeded inputs and numpy <-> torch conversion."""

from __future__ import annotations

import numpy as np
import torch

from oracle import fp8


def to_bf16_tensor(bits: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_fp8_tensor(codes: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(codes)).view(torch.float8_e4m3fn).to(device)


def codes_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def outlier_activations(rows: int, cols: int, seed: int) -> torch.Tensor:
    """bf16 N(0,1) with round(0.001*rows*cols) entries x20 (the benchmark's outlier rule)."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=gen)
    count = round(0.001 * rows * cols)
    if count:
        idx = torch.randperm(rows * cols, generator=torch.Generator().manual_seed(seed + 1))[:count]
        x.view(-1)[idx] *= 20
    return x.to(torch.bfloat16)


def fp8_weight(rows: int, cols: int, seed: int, std: float = 0.02):
    """Seeded N(0, std) weight quantised per output row -> (e4m3 [rows, cols], fp32 [rows, 1])."""
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(rows, cols, generator=gen) * std).float().numpy()
    codes, scales = fp8.quantize_weight(w)
    return to_fp8_tensor(codes), torch.from_numpy(scales)


def bf16_close(actual: np.ndarray, expected: np.ndarray, *, max_mismatch: float, ulps: int = 1,
               atol=0.0) -> None:
    """Values agree except a fraction ``max_mismatch`` that may differ by ``ulps`` bf16 ulp.

    ``atol`` (scalar or per element) widens the bound where an earlier rounding
    step feeds a cancellation, e.g. one ulp of the GEMM output before a bias add.
    """
    a = np.asarray(actual, np.float32)
    e = np.asarray(expected, np.float32)
    assert a.shape == e.shape
    assert np.array_equal(np.isnan(a), np.isnan(e))
    mismatch = (a != e) & ~np.isnan(e)
    frac = mismatch.mean() if a.size else 0.0
    assert frac <= max_mismatch, f"{frac:.2e} of values differ"
    if mismatch.any():
        ulp = np.maximum(np.abs(e[mismatch]), 2.0**-126) * 2.0**-7 * ulps * 1.0001
        tol = np.broadcast_to(np.asarray(atol, np.float32), e.shape)[mismatch]
        assert (np.abs(a[mismatch] - e[mismatch]) <= ulp + tol).all()
