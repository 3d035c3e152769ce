"""A QAD NVFP4 checkpoint read into pinned memory, put on the GPU and run through NVFP4Execution."""

from __future__ import annotations

import pytest
import torch

from oracle import fp8, nvfp4
from tests.helpers import outlier_activations
from tests.test_qad_files import SHAPES, write
from vflash_b200.kernels import nvfp4_quantize
from vflash_b200.native.h3_nvfp4_linear import NVFP4Execution, NVFP4Weight
from vflash_b200.native.h3_weight_files import QAD_INPUT_SF, PinnedNVFP4Linears, qad_targets

pytestmark = pytest.mark.gpu
DEV = "cuda"


def quantized_checkpoint(blocks: int) -> dict[str, torch.Tensor]:
    """Packed tensors as a QAD export holds them: NVFP4 weights, alpha = 1 / global scale."""
    out = {}
    for i, prefix in enumerate(qad_targets(blocks).values()):
        n, k = SHAPES[prefix.split(".", 2)[2]]
        w = (torch.randn(n, k, generator=torch.Generator().manual_seed(100 + i)) * 0.02).to(torch.bfloat16).to(DEV)
        gsf = (448.0 * 6.0 / w.float().abs().max()).reshape(())
        packed, scales = nvfp4_quantize(w, gsf)
        out[prefix + "::_nvfp4_weight"] = packed.cpu()
        out[prefix + "::_nvfp4_weight_scale"] = scales.view(n, k // 16).cpu()
        out[prefix + "::_nvfp4_alpha"] = (1.0 / gsf).cpu()
        out[prefix + "::_weight_global_sf"] = gsf.cpu()
        if ".ff." in prefix:
            out[prefix + "::" + QAD_INPUT_SF] = torch.tensor(448.0 * 6.0 / 100.0)  # calibrated for |x| <= 100
    return out


def test_materialized_checkpoint_runs_like_directly_placed_weights(tmp_path):
    tensors = quantized_checkpoint(2)
    path = tmp_path / "qad.safetensors"
    write(path, tensors)
    linears = PinnedNVFP4Linears(path, blocks=2)
    assert all(w.packed.is_pinned() for w in linears.weights.values())
    placed = linears.materialize(DEV)
    torch.cuda.synchronize()
    engine = NVFP4Execution()
    for j, (name, prefix) in enumerate(qad_targets(2).items()):
        weight = placed[name]
        assert weight.packed.device.type == "cuda"
        direct = NVFP4Weight(tensors[prefix + "::_nvfp4_weight"].to(DEV),
                             tensors[prefix + "::_nvfp4_weight_scale"].to(DEV),
                             tensors[prefix + "::_nvfp4_alpha"].to(DEV),
                             (tensors[prefix + "::" + QAD_INPUT_SF] if ".ff." in prefix
                              else torch.ones((), dtype=torch.float32)).to(DEV))
        x = outlier_activations(150, weight.in_features, 200 + j).to(DEV)
        y = engine.linear(x, weight)
        assert torch.equal(y, engine.linear(x, direct)), name
        # the output follows the exact emulation of the same quantised operands
        a_codes, a_sf = nvfp4_quantize(x, weight.input_scale)
        want = nvfp4.w4a4_reference(a_codes.cpu().numpy(), a_sf.cpu().numpy().reshape(-1),
                                    weight.packed.cpu().numpy(), weight.scales.cpu().numpy().reshape(-1),
                                    float(weight.alpha / weight.input_scale))
        assert fp8.rel_l2(y.float().cpu().numpy(), want) <= 1e-2, name
