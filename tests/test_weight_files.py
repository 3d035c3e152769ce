"""Reading FP8 block files (the reference's safetensors layout) straight into pinned block buffers."""

from __future__ import annotations

import json
import struct

import pytest
import torch

from vflash_b200.native.h3_parallel import FP8Weight
from vflash_b200.native.h3_pinned_arena import ALIGN, BlockLayout, PinnedHostArena, pin_blocks
from vflash_b200.native.h3_weight_files import FP8_BLOCK_KEYS, pin_fp8_block_files, read_header

safetensors_torch = pytest.importorskip("safetensors.torch")

SHAPES = (("qkv", 96, 64), ("attention_out", 32, 32), ("ffn_in", 128, 32), ("ffn_out", 32, 128))


def random_block(seed: int) -> dict[str, FP8Weight]:
    gen = torch.Generator().manual_seed(seed)
    return {name: FP8Weight(torch.randint(0, 256, (n, k), generator=gen, dtype=torch.uint8)
                            .view(torch.float8_e4m3fn), torch.rand((n, 1), generator=gen) + 0.5)
            for name, n, k in SHAPES}


def write_block(path, block, extra=None):
    tensors = {}
    for name, w in block.items():
        tensors[FP8_BLOCK_KEYS[name]] = w.codes.contiguous()
        tensors[FP8_BLOCK_KEYS[name] + ".row_scale"] = w.row_scale.contiguous()
    tensors.update(extra or {})
    safetensors_torch.save_file(tensors, str(path), metadata={"format": "pt"})


@pytest.mark.parametrize("world", [1, 2, 4])
def test_file_reads_equal_in_memory_packing(tmp_path, world):
    layout = BlockLayout.for_shapes(SHAPES, multiple=ALIGN * world)
    blocks = [random_block(s) for s in range(3)]
    paths = []
    for i, b in enumerate(blocks):
        paths.append(tmp_path / f"block_{i}.safetensors")
        write_block(paths[-1], b, extra={"adapter.attn.q.down": torch.ones(2, 64, dtype=torch.bfloat16)})
    arena = PinnedHostArena(1 << 20, pin_memory=False)
    want = [pin_blocks(layout, blocks, arena, rank=r, world=world) for r in range(world)]
    got = [pin_fp8_block_files(paths, layout, arena, rank=r, world=world) for r in range(world)]
    for r in range(world):
        for g, w in zip(got[r], want[r]):
            assert torch.equal(g, w)
            assert g.data_ptr() % ALIGN == 0


def test_header_entries_and_payload_offset(tmp_path):
    path = tmp_path / "b.safetensors"
    write_block(path, random_block(1))
    offset, entries = read_header(path)
    assert set(entries) == {k for v in FP8_BLOCK_KEYS.values() for k in (v, v + ".row_scale")}
    assert entries["attn.qkv.weight"]["dtype"] == "F8_E4M3" and entries["attn.qkv.weight"]["shape"] == [96, 64]
    assert offset == 8 + struct.unpack("<Q", path.read_bytes()[:8])[0]


def raw_file(path, header: dict, payload: bytes):
    blob = json.dumps(header).encode()
    path.write_bytes(struct.pack("<Q", len(blob)) + blob + payload)


@pytest.mark.parametrize("case,match", [
    ("gap", "gaps or overlaps"),
    ("size", "differ from header"),
    ("shape", "differs from its shape"),
    ("dtype", "malformed"),
    ("truncated", "truncated"),
])
def test_malformed_headers_are_rejected(tmp_path, case, match):
    path = tmp_path / "bad.safetensors"
    if case == "truncated":
        path.write_bytes(b"\x01\x02")
    else:
        header = {"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]},
                  "b": {"dtype": "U8", "shape": [4], "data_offsets": [4, 8]}}
        payload = bytes(8)
        if case == "gap":
            header["b"]["data_offsets"] = [5, 9]
            payload = bytes(9)
        elif case == "size":
            payload = bytes(10)
        elif case == "shape":
            header["b"]["shape"] = [5]
        elif case == "dtype":
            header["b"]["dtype"] = "Q4"
        raw_file(path, header, payload)
    with pytest.raises(ValueError, match=match):
        read_header(path)


def test_wrong_dtype_or_missing_tensor_is_rejected(tmp_path):
    layout = BlockLayout.for_shapes(SHAPES)
    arena = PinnedHostArena(1 << 20, pin_memory=False)
    block = random_block(2)
    bad = dict(block)
    path = tmp_path / "b.safetensors"
    tensors = {FP8_BLOCK_KEYS[n]: w.codes for n, w in bad.items()}
    tensors.update({FP8_BLOCK_KEYS[n] + ".row_scale": w.row_scale for n, w in bad.items()})
    tensors["attn.out.weight.row_scale"] = tensors["attn.out.weight.row_scale"].to(torch.bfloat16)
    safetensors_torch.save_file(tensors, str(path))
    with pytest.raises(ValueError, match="expected F32"):
        pin_fp8_block_files([path], layout, arena)
    del tensors["attn.out.weight.row_scale"]
    safetensors_torch.save_file(tensors, str(path))
    with pytest.raises(ValueError, match="no tensor attn.out.weight.row_scale"):
        pin_fp8_block_files([path], layout, arena)


def test_block_files_may_carry_tensors_of_other_dtypes(tmp_path):
    layout = BlockLayout.for_shapes(SHAPES)
    block = random_block(7)
    path = tmp_path / "b.safetensors"
    write_block(path, block, extra={"x.f64": torch.ones(3, dtype=torch.float64),
                                    "x.flag": torch.tensor([True, False]), "x.i16": torch.arange(4, dtype=torch.int16)})
    arena = PinnedHostArena(1 << 20, pin_memory=False)
    got = pin_fp8_block_files([path], layout, arena)[0]
    want = pin_blocks(layout, [block], arena)[0]
    assert torch.equal(got, want)
