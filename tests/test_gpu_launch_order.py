"""A GEMM launched right after the quantiser that writes its operand reads that output.

The GEMMs are launched as programmatic dependents of the previous kernel in
the stream, and the quantisers let their dependents be scheduled as soon as
they start: the GEMM's setup overlaps the quantiser's last wave and every
GEMM thread waits for the quantiser to complete before it reads or writes
global memory.  These tests run quantiser -> GEMM pairs back to back on one
stream, each pair overwriting the same code and scale buffers with a
different input, and compare every output with the one computed with the
quantiser finished (a device synchronisation) before the GEMM was launched.
A GEMM that read early would see the previous input's codes or partly
written ones.  The same sequence is also captured and replayed as a CUDA
graph.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200 import _lib
from vflash_b200.kernels import nvfp4_quantize

pytestmark = pytest.mark.gpu
DEV = "cuda"
M, K, N = 8192, 4096, 4096
ROUNDS = 4


def _check(rc, what):
    _lib.check(rc, what)


def fp8_pair(lib, x, codes, scales, w, ws, out, stream):
    _check(lib.vfb_fp8_quant_rows(x.data_ptr(), M, K, K, codes.data_ptr(), scales.data_ptr(), M, stream),
           "vfb_fp8_quant_rows")
    ep = _lib.Epilogue()
    ep.kind, ep.out, ep.ldo = _lib.EPI_STORE, out.data_ptr(), N
    _check(lib.vfb_fp8_gemm(codes.data_ptr(), K, scales.data_ptr(), w.data_ptr(), K, ws.data_ptr(), M, N, K,
                            ctypes.byref(ep), stream), "vfb_fp8_gemm")


def nvfp4_pair(lib, x, gsf, codes, sf, w, wsf, alpha, out, stream):
    _check(lib.vfb_nvfp4_quant_rows(x.data_ptr(), 0, M, K, K, gsf.data_ptr(), codes.data_ptr(), sf.data_ptr(),
                                    stream), "vfb_nvfp4_quant_rows")
    _check(lib.vfb_nvfp4_gemm(codes.data_ptr(), sf.data_ptr(), w.data_ptr(), wsf.data_ptr(), alpha.data_ptr(), M,
                              N, K, None, out.data_ptr(), 1, stream), "vfb_nvfp4_gemm")


def inputs():
    return [outlier_activations(M, K, 500 + i).to(DEV) for i in range(ROUNDS)]


def test_fp8_gemm_after_quantiser_back_to_back_and_in_a_graph():
    lib = _lib.load()
    stream = _lib.stream_handle(torch.device(DEV))
    xs = inputs()
    w, ws = fp8_weight(N, K, 71)
    w, ws = w.to(DEV), ws.to(DEV)
    codes = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=DEV)
    scales = torch.empty((M, 1), dtype=torch.float32, device=DEV)
    expected = []
    for x in xs:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
        _check(lib.vfb_fp8_quant_rows(x.data_ptr(), M, K, K, codes.data_ptr(), scales.data_ptr(), M, stream),
               "vfb_fp8_quant_rows")
        torch.cuda.synchronize()
        ep = _lib.Epilogue()
        ep.kind, ep.out, ep.ldo = _lib.EPI_STORE, out.data_ptr(), N
        _check(lib.vfb_fp8_gemm(codes.data_ptr(), K, scales.data_ptr(), w.data_ptr(), K, ws.data_ptr(), M, N, K,
                                ctypes.byref(ep), stream), "vfb_fp8_gemm")
        torch.cuda.synchronize()
        expected.append(out)
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device=DEV) for _ in xs]
    for _ in range(3):
        for x, out in zip(xs, outs):
            fp8_pair(lib, x, codes, scales, w, ws, out, stream)
        torch.cuda.synchronize()
        for out, ref in zip(outs, expected):
            assert torch.equal(out, ref)
        for out in outs:
            out.zero_()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            capture_stream = _lib.stream_handle(torch.device(DEV))
            for x, out in zip(xs, outs):
                fp8_pair(lib, x, codes, scales, w, ws, out, capture_stream)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        for out in outs:
            out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for out, ref in zip(outs, expected):
            assert torch.equal(out, ref)
    del graph
    assert _lib.device_status(clear=True) == 0


def test_nvfp4_gemm_after_quantiser_back_to_back():
    lib = _lib.load()
    stream = _lib.stream_handle(torch.device(DEV))
    xs = inputs()
    gsf = (448.0 * 6.0 / torch.stack([x.float().abs().max() for x in xs]).max()).to(torch.float32).reshape(())
    wt = (torch.randn(N, K, generator=torch.Generator().manual_seed(72)) * 0.02).to(torch.bfloat16).to(DEV)
    gsf_w = (448.0 * 6.0 / wt.float().abs().max()).reshape(()).to(torch.float32)
    w, wsf = nvfp4_quantize(wt, gsf_w)
    alpha = ((1.0 / gsf_w) / gsf).to(torch.float32).reshape(())
    codes = torch.empty((M, K // 2), dtype=torch.uint8, device=DEV)
    sf = torch.empty((M * K // 16,), dtype=torch.uint8, device=DEV)
    expected = []
    for x in xs:
        ref_codes, ref_sf = nvfp4_quantize(x, gsf)
        torch.cuda.synchronize()
        out = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
        _check(lib.vfb_nvfp4_gemm(ref_codes.data_ptr(), ref_sf.data_ptr(), w.data_ptr(), wsf.data_ptr(),
                                  alpha.data_ptr(), M, N, K, None, out.data_ptr(), 1, stream), "vfb_nvfp4_gemm")
        torch.cuda.synchronize()
        expected.append(out)
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device=DEV) for _ in xs]
    for _ in range(3):
        for x, out in zip(xs, outs):
            nvfp4_pair(lib, x, gsf, codes, sf, w, wsf, alpha, out, stream)
        torch.cuda.synchronize()
        for out, ref in zip(outs, expected):
            assert torch.equal(out, ref)
        for out in outs:
            out.zero_()
    assert _lib.device_status(clear=True) == 0
