"""CPU validation of the strict-BF16 drop-ins (ported from the reference's
tests/test_qkv_direct_merge.py:180-211 and tests/test_ffn_fusion.py:134-141):
layouts, aliasing, grad and scalings are checked before any launch, and CPU
tensors are rejected without initialising CUDA."""

from __future__ import annotations

import pytest
import torch

from vflash_b200.native import h3_fused_ops as fused


def test_branch_metadata_and_cpu_launch_rejection():
    initialized = torch.cuda.is_initialized()
    base = torch.zeros((1, 3, 12), dtype=torch.bfloat16)
    adapters = tuple(torch.ones((1, 3, 4), dtype=torch.bfloat16) for _ in range(3))
    scales = (0.0625, 1.0, -0.3)
    assert fused._validate_qkv_direct_merge(base, adapters, scales, block_size=1024) == (12, 4, scales)
    alias = base.view(-1)[:12].view(1, 3, 4)
    for invalid in (base.float(), base.transpose(1, 2), base.clone().requires_grad_(True)):
        with pytest.raises(fused.H3FusedOpsError):
            fused._validate_qkv_direct_merge(invalid, adapters, scales, block_size=1024)
    grad_adapter = adapters[0].clone().requires_grad_(True)
    with pytest.raises(fused.H3FusedOpsError, match="separate"):
        fused._validate_qkv_direct_merge(base, (grad_adapter, *adapters[1:]), scales, block_size=1024)
    with pytest.raises(fused.H3FusedOpsError, match="separate"):
        fused._validate_qkv_direct_merge(base, (alias, *adapters[1:]), scales, block_size=1024)
    for invalid in ((0.0625,) * 2, (float("nan"), 1.0, 1.0), (True, 1.0, 1.0)):
        with pytest.raises(fused.H3FusedOpsError, match="scalings"):
            fused._validate_qkv_direct_merge(base, adapters, invalid, block_size=1024)
    with pytest.raises(fused.H3FusedOpsError, match="CUDA BF16"):
        fused.triton_strict_bf16_qkv_direct_merge(base, adapters, scalings=scales)
    assert torch.cuda.is_initialized() == initialized


def test_ffn_cpu_tensor_is_rejected_without_cuda_initialization():
    initialized = torch.cuda.is_initialized()
    value = torch.zeros((1, 3, 8), dtype=torch.bfloat16)
    with pytest.raises(fused.H3FusedOpsError, match="CUDA BF16"):
        fused.triton_strict_bf16_ffn_adapter_silu(value, value, scaling=0.0625, block_size=1024)
    assert torch.cuda.is_initialized() == initialized


def test_common_validation_messages():
    value = torch.zeros((2, 3, 8), dtype=torch.bfloat16)
    gate = torch.zeros((3, 8), dtype=torch.bfloat16)
    with pytest.raises(fused.H3FusedOpsError, match="block size"):
        fused.triton_strict_bf16_gate_residual(value, gate, value, block_size=100)
    with pytest.raises(fused.H3FusedOpsError, match="CUDA device"):
        fused.triton_strict_bf16_gate_residual(value, gate, value)
    with pytest.raises(fused.H3FusedOpsError, match="CUDA BF16"):
        fused.triton_strict_bf16_silu_mul(value)
    with pytest.raises(fused.H3FusedOpsError, match="CUDA device"):
        fused.triton_strict_bf16_adapter_merge(value, value, scaling=0.5)


def test_validate_common_shapes():
    value = torch.zeros((2, 3, 8), dtype=torch.bfloat16)
    assert fused._validate_scalings((1, 2.0, 3), 3) == (1.0, 2.0, 3.0)
    with pytest.raises(fused.H3FusedOpsError, match="finite"):
        fused._validate_scalings((float("inf"),), 1)
    with pytest.raises(fused.H3FusedOpsError, match="tensors"):
        fused._validate_matching_activation(value, object(), candidate_name="adapter", block_size=256)
