"""The merged-QKV GEMM storing straight into pack_qkv's destination-major wire layout.

The wire layout moves values without changing them, so the bar is bit
identity: the packed output equals the oracle's pack_qkv (pinned on the
reference's pack_qkv_reference by the golden vectors) applied to the planar
Q, K, V outputs of the same call — plain, with the LoRA direct merge, and
with the QK-norm + rotary epilogue.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogues as ep
from tests.helpers import bits_of, fp8_weight, outlier_activations
from tests.test_gpu_qk_rope import rope_tables
from vflash_b200.kernels import KernelInputError
from vflash_b200.native.h3_fp8_linear import QKNormRope, RowFP8Execution

pytestmark = pytest.mark.gpu
DEV = "cuda"


def case(batch, tokens, heads, k, seed):
    width = heads * 128
    x = outlier_activations(batch * tokens, k, seed).reshape(batch, tokens, k).to(DEV)
    codes, scale = fp8_weight(3 * width, k, seed + 1)
    bias = (torch.randn(3 * width, generator=torch.Generator().manual_seed(seed + 2)) * 0.01).to(torch.bfloat16)
    return x, codes.to(DEV), scale.to(DEV), bias.to(DEV)


def packed_oracle(q, k, v, chunks):
    return ep.pack_qkv(*(bits_of(t.view(*t.shape[:-1], -1, 128)) for t in (q, k, v)), chunks)


@pytest.mark.parametrize("batch,tokens,heads,chunks", [(2, 150, 8, 1), (2, 150, 8, 2), (1, 300, 8, 4),
                                                      (3, 17, 4, 2), (1, 4096, 16, 2)])
def test_plain_store_packs_like_pack_qkv(batch, tokens, heads, chunks):
    x, w, s, bias = case(batch, tokens, heads, 256, 40 + heads)
    ex = RowFP8Execution("w8a8")
    q, k, v = ex.qkv_linear(x, w, s, bias)
    packed = ex.qkv_linear(x, w, s, bias, pack_chunks=chunks)
    assert packed.shape == (chunks, 2, 3, batch, tokens, heads // (2 * chunks), 128)
    assert packed.is_contiguous()
    np.testing.assert_array_equal(bits_of(packed), packed_oracle(q, k, v, chunks))


def test_adapters_and_qk_norm_rope_pack_like_pack_qkv():
    batch, tokens, heads, chunks = 2, 64, 4, 2
    x, w, s, bias = case(batch, tokens, heads, 512, 60)
    width = heads * 128
    gen = torch.Generator().manual_seed(61)
    adapters = tuple(torch.randn(batch, tokens, width, generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
    scalings = (0.25, -0.5, 1.0)
    ex = RowFP8Execution("w8a8")
    planes = ex.qkv_linear(x, w, s, bias, adapters=adapters, scalings=scalings)
    packed = ex.qkv_linear(x, w, s, bias, adapters=adapters, scalings=scalings, pack_chunks=chunks)
    np.testing.assert_array_equal(bits_of(packed), packed_oracle(*planes, chunks))
    cos, sin = rope_tables(tokens, 128, 3)
    qn = (1 + torch.randn(128, generator=gen) * 0.1).to(torch.bfloat16).to(DEV)
    kn = (1 + torch.randn(128, generator=gen) * 0.1).to(torch.bfloat16).to(DEV)
    rope = QKNormRope(qn, kn, cos.to(DEV), sin.to(DEV), 1e-5)
    planes = ex.qkv_linear(x, w, s, bias, qk_norm_rope=rope)
    packed = ex.qkv_linear(x, w, s, bias, qk_norm_rope=rope, pack_chunks=chunks)
    np.testing.assert_array_equal(bits_of(packed), packed_oracle(*planes, chunks))


def test_wire_layout_rejects_heads_that_do_not_split():
    x, w, s, bias = case(1, 32, 4, 256, 70)
    ex = RowFP8Execution("w8a8")
    with pytest.raises(ValueError, match="destinations"):
        ex.qkv_linear(x, w, s, bias, pack_chunks=4)
    with pytest.raises(ValueError, match="destinations"):
        ex.qkv_linear(x, w, s, bias, pack_chunks=0)
    from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows

    codes, scale = quantize_fp8_rows(x.view(32, 256))
    with pytest.raises(KernelInputError):
        fp8_gemm(codes, scale, 32, w, s, Epilogue(planes=1, wire_chunks=1))
