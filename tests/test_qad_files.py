"""Reading a QAD NVFP4 checkpoint (the reference's packed-file keys) into pinned memory."""

from __future__ import annotations

import pytest
import torch

from vflash_b200.native.h3_nvfp4_linear import NVFP4Weight
from vflash_b200.native.h3_pinned_arena import ALIGN, PinnedHostArena
from vflash_b200.native.h3_weight_files import (QAD_INPUT_SF, PinnedNVFP4Linears, qad_required_keys,
                                                qad_targets)

safetensors_torch = pytest.importorskip("safetensors.torch")

# (N, K) per linear, small multiples of the NVFP4 contract (N % 128, K/2 % 32)
SHAPES = {"attn.to_q": (128, 64), "attn.to_k": (128, 64), "attn.to_v": (128, 64),
          "attn.to_out": (128, 128), "ff.fc_in": (256, 64), "ff.fc_out": (128, 256)}


def qad_tensors(blocks: int, seed: int = 0) -> dict[str, torch.Tensor]:
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for prefix in qad_targets(blocks).values():
        n, k = SHAPES[prefix.split(".", 2)[2]]
        out[prefix + "::_nvfp4_weight"] = torch.randint(0, 256, (n, k // 2), generator=gen, dtype=torch.uint8)
        out[prefix + "::_nvfp4_weight_scale"] = torch.randint(0, 127, (n, k // 16), generator=gen, dtype=torch.uint8)
        out[prefix + "::_nvfp4_alpha"] = torch.rand((), generator=gen) + 1e-3
        out[prefix + "::_weight_global_sf"] = torch.rand((), generator=gen) + 1.0
        if ".ff." in prefix:
            out[prefix + "::" + QAD_INPUT_SF] = torch.rand((), generator=gen) + 1.0
    return out


def write(path, tensors):
    safetensors_torch.save_file(tensors, str(path), metadata={"format": "pt"})


def test_targets_and_keys_follow_the_reference_naming():
    targets = qad_targets(50)
    assert len(targets) == 300
    assert targets["transformer_blocks.7.attn.to_out.0"] == "transformer_blocks.7.attn.to_out"
    assert targets["transformer_blocks.49.ff.net.0.proj"] == "transformer_blocks.49.ff.fc_in"
    keys = qad_required_keys(targets.values())
    assert len(keys) == 300 * 4 + 100  # the FFN linears add their input scale


def test_pinned_weights_equal_the_file(tmp_path):
    tensors = qad_tensors(2)
    path = tmp_path / "qad.safetensors"
    write(path, tensors)
    linears = PinnedNVFP4Linears(path, blocks=2, arena=PinnedHostArena(1 << 20, pin_memory=False))
    assert len(linears.weights) == 12
    for name, prefix in qad_targets(2).items():
        w = linears.weights[name]
        assert isinstance(w, NVFP4Weight)
        assert torch.equal(w.packed, tensors[prefix + "::_nvfp4_weight"])
        assert torch.equal(w.scales, tensors[prefix + "::_nvfp4_weight_scale"])
        assert torch.equal(w.alpha, tensors[prefix + "::_nvfp4_alpha"])
        want_in = tensors[prefix + "::" + QAD_INPUT_SF] if ".ff." in prefix else torch.ones(())
        assert torch.equal(w.input_scale, want_in)
        for t in (w.packed, w.scales, w.alpha, w.input_scale):
            assert t.data_ptr() % ALIGN == 0


def test_materialize_views_one_allocation(tmp_path):
    tensors = qad_tensors(1, seed=3)
    path = tmp_path / "qad.safetensors"
    write(path, tensors)
    linears = PinnedNVFP4Linears(path, blocks=1, arena=PinnedHostArena(1 << 20, pin_memory=False))
    placed = linears.materialize("cpu")
    base = min(w.packed.data_ptr() for w in placed.values())
    for name, w in placed.items():
        host = linears.weights[name]
        for a, b in ((w.packed, host.packed), (w.scales, host.scales), (w.alpha, host.alpha),
                     (w.input_scale, host.input_scale)):
            assert torch.equal(a, b) and a.data_ptr() != b.data_ptr()
            assert (a.data_ptr() - base) % ALIGN == 0 and a.data_ptr() - base < linears.nbytes


def test_key_set_must_match_exactly(tmp_path):
    tensors = qad_tensors(1)
    missing = dict(tensors)
    missing.pop("transformer_blocks.0.ff.fc_out::" + QAD_INPUT_SF)
    write(tmp_path / "a.safetensors", missing)
    with pytest.raises(ValueError, match="must cover all 6 original main-block linears"):
        PinnedNVFP4Linears(tmp_path / "a.safetensors", blocks=1)
    extra = dict(tensors)
    extra["transformer_blocks.0.attn.to_q::" + QAD_INPUT_SF] = torch.ones(())
    write(tmp_path / "b.safetensors", extra)
    with pytest.raises(ValueError, match="must cover all"):
        PinnedNVFP4Linears(tmp_path / "b.safetensors", blocks=1)


def test_layout_mismatches_are_rejected(tmp_path):
    tensors = qad_tensors(1)
    bad = dict(tensors)
    bad["transformer_blocks.0.attn.to_q::_nvfp4_weight_scale"] = torch.zeros(128, 3, dtype=torch.uint8)
    write(tmp_path / "a.safetensors", bad)
    with pytest.raises(ValueError, match="_nvfp4_weight_scale"):
        PinnedNVFP4Linears(tmp_path / "a.safetensors", blocks=1)
    bad = dict(tensors)
    bad["transformer_blocks.0.attn.to_k::_nvfp4_alpha"] = torch.ones(1)
    write(tmp_path / "b.safetensors", bad)
    with pytest.raises(ValueError, match="_nvfp4_alpha"):
        PinnedNVFP4Linears(tmp_path / "b.safetensors", blocks=1)
    bad = dict(tensors)
    bad["transformer_blocks.0.ff.fc_in::_nvfp4_alpha"] = torch.zeros(())
    write(tmp_path / "c.safetensors", bad)
    with pytest.raises(ValueError, match="positive and finite"):
        PinnedNVFP4Linears(tmp_path / "c.safetensors", blocks=1, arena=PinnedHostArena(1 << 20, pin_memory=False))
    bad = dict(tensors)
    bad["transformer_blocks.0.ff.fc_in::_nvfp4_weight"] = torch.zeros(100, 32, dtype=torch.uint8)
    bad["transformer_blocks.0.ff.fc_in::_nvfp4_weight_scale"] = torch.zeros(100, 4, dtype=torch.uint8)
    write(tmp_path / "d.safetensors", bad)
    with pytest.raises(ValueError, match="declared packed codes"):
        PinnedNVFP4Linears(tmp_path / "d.safetensors", blocks=1, arena=PinnedHostArena(1 << 20, pin_memory=False))
