"""Framed zstd sidecars of safetensors payloads: the reference's format, validation and reads."""

from __future__ import annotations

import json

import pytest
import torch

from tests.test_weight_files import SHAPES, random_block, write_block
from vflash_b200.native.h3_pinned_arena import ALIGN, BlockLayout, PinnedHostArena
from vflash_b200.native.h3_weight_codec import (ZSTD_MAGIC, frame_parameters, pin_fp8_block_sidecars, prepare,
                                                read_into)
from vflash_b200.native.h3_buffered_weights import payload_header
from vflash_b200.native.h3_weight_files import pin_fp8_block_files

pytest.importorskip("safetensors.torch")
pa = pytest.importorskip("pyarrow")
if not pa.Codec.is_available("zstd"):
    pytest.skip("pyarrow without zstd", allow_module_level=True)


def source_file(tmp_path, seed=0, name="block.safetensors"):
    path = tmp_path / name
    write_block(path, random_block(seed), extra={"adapter.attn.q.down": torch.ones(2, 64, dtype=torch.bfloat16)})
    return path


def payload_of(path):
    offset, _ = payload_header(path)
    return path.read_bytes()[offset:], offset


def test_prepare_then_read_into_round_trips(tmp_path):
    src = source_file(tmp_path)
    manifest = prepare(src, tmp_path / "side", chunk_bytes=4096)
    payload, offset = payload_of(src)
    assert manifest["payload_bytes"] == len(payload) and len(manifest["frames"]) == -(-len(payload) // 4096)
    assert json.loads((tmp_path / "side" / "index.json").read_text()) == manifest
    for workers in (1, 4):
        target = bytearray(len(payload))
        info = read_into(tmp_path / "side", memoryview(target), source_name=src.name,
                         source_size=src.stat().st_size, header_bytes=offset, workers=workers)
        assert bytes(target) == payload
        assert info["frames"] == len(manifest["frames"]) and info["decoded_bytes"] == len(payload)


def test_prepare_refuses_existing_destination_and_bad_chunks(tmp_path):
    src = source_file(tmp_path)
    (tmp_path / "exists").mkdir()
    with pytest.raises(ValueError, match="new destination"):
        prepare(src, tmp_path / "exists")
    with pytest.raises(ValueError, match="bounded compression chunks"):
        prepare(src, tmp_path / "side", chunk_bytes=1024)


def test_read_into_checks_the_source_layout_and_the_index(tmp_path):
    src = source_file(tmp_path)
    prepare(src, tmp_path / "side", chunk_bytes=4096)
    payload, offset = payload_of(src)
    size = src.stat().st_size
    good = dict(source_name=src.name, source_size=size, header_bytes=offset)
    target = bytearray(len(payload))
    for bad in (dict(good, source_name="other.safetensors"), dict(good, source_size=size + 1),
                dict(good, header_bytes=offset + 8)):
        with pytest.raises(ValueError, match="source layout differs"):
            read_into(tmp_path / "side", target, **bad)
    with pytest.raises(ValueError, match="source layout differs"):
        read_into(tmp_path / "side", bytearray(len(payload) - 1), **good)
    with pytest.raises(ValueError, match="concurrency"):
        read_into(tmp_path / "side", target, workers=3, **good)
    index = tmp_path / "side" / "index.json"
    data = json.loads(index.read_text())
    data["frames"][1][0] += 1  # a gap between frames
    index.write_text(json.dumps(data))
    with pytest.raises(ValueError, match="overlap or exceed"):
        read_into(tmp_path / "side", target, **good)


def test_read_into_rejects_a_frame_that_differs_from_its_record(tmp_path):
    src = source_file(tmp_path)
    prepare(src, tmp_path / "side", chunk_bytes=4096)
    payload, offset = payload_of(src)
    good = dict(source_name=src.name, source_size=src.stat().st_size, header_bytes=offset)
    blob = tmp_path / "side" / "payload.zst"
    raw = bytearray(blob.read_bytes())
    raw[0] ^= 0xFF  # the first frame loses its magic number
    blob.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="not a zstd frame"):
        read_into(tmp_path / "side", bytearray(len(payload)), **good)
    blob.write_bytes(bytes(raw[:-1]))
    with pytest.raises(ValueError, match="size or type differs"):
        read_into(tmp_path / "side", bytearray(len(payload)), **good)


def test_frame_header_fields():
    magic = ZSTD_MAGIC.to_bytes(4, "little")
    # single segment, 1-byte content size: window = content
    assert frame_parameters(magic + bytes([0x20, 200, 0])) == (200, 200)
    # 2-byte content size is stored minus 256
    assert frame_parameters(magic + bytes([0x60, 0x00, 0x01, 0])) == (512, 512)
    # window descriptor: exponent 1, mantissa 2 -> 2048 + 2 * 256; 4-byte content size
    assert frame_parameters(magic + bytes([0x80, (1 << 3) | 2]) + (5000).to_bytes(4, "little")) == (5000, 2560)
    # no content size
    assert frame_parameters(magic + bytes([0x00, 0x00, 0, 0])) == (None, 1024)
    with pytest.raises(ValueError, match="dictionary"):
        frame_parameters(magic + bytes([0x21, 7, 9, 0]))
    with pytest.raises(ValueError, match="not a zstd frame"):
        frame_parameters(b"\x00" * 8)
    codec = pa.Codec("zstd", compression_level=3)
    data = bytes(range(256)) * 100
    assert frame_parameters(codec.compress(data, asbytes=True))[0] == len(data)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sidecar_blocks_equal_file_blocks(tmp_path, world):
    layout = BlockLayout.for_shapes(SHAPES, multiple=ALIGN * world)
    sources, pairs = [], []
    for i in range(3):
        src = source_file(tmp_path, seed=10 + i, name=f"block_{i}.safetensors")
        prepare(src, tmp_path / f"side_{i}", chunk_bytes=4096)
        sources.append(src)
        pairs.append((src, tmp_path / f"side_{i}"))
    arena = PinnedHostArena(1 << 20, pin_memory=False)
    for rank in range(world):
        want = pin_fp8_block_files(sources, layout, arena, rank=rank, world=world)
        got = pin_fp8_block_sidecars(pairs, layout, arena, rank=rank, world=world)
        for g, w in zip(got, want):
            assert torch.equal(g, w) and g.data_ptr() % ALIGN == 0


# the failure cases of the reference's own sidecar tests (tests/test_weight_codec.py
# of vflash), which need the zstandard module to run there


def sidecar_case(tmp_path):
    src = source_file(tmp_path)
    manifest = prepare(src, tmp_path / "side", chunk_bytes=4096)
    payload, offset = payload_of(src)
    return src, tmp_path / "side", payload, dict(source_name=src.name, source_size=src.stat().st_size,
                                                 header_bytes=offset), manifest


@pytest.mark.parametrize("change", ["overlap", "oversize", "source", "name", "truncated", "symlink"])
def test_inconsistent_or_unsafe_sidecars_are_refused(tmp_path, change):
    src, side, payload, layout, manifest = sidecar_case(tmp_path)
    if change == "overlap":
        manifest["frames"][1][0] -= 1
    elif change == "oversize":
        manifest["frames"][0][2] = 12 * 1024**3
    elif change == "source":
        manifest["source_size"] += 1
    elif change == "name":
        manifest["source_name"] = "another.safetensors"
    elif change == "truncated":
        with (side / "payload.zst").open("r+b") as handle:
            handle.truncate(5)
    else:
        (side / "payload.zst").rename(side / "real.zst")
        (side / "payload.zst").symlink_to(side / "real.zst")
    (side / "index.json").write_text(json.dumps(manifest))
    with pytest.raises((ValueError, OSError)):
        read_into(side, memoryview(bytearray(len(payload))), **layout)


def test_short_positioned_reads_and_early_end(tmp_path, monkeypatch):
    from vflash_b200.native import h3_weight_codec as codec

    src, side, payload, layout, _manifest = sidecar_case(tmp_path)
    real = codec.os.pread
    monkeypatch.setattr(codec.os, "pread", lambda fd, n, at: real(fd, min(n, 7), at))
    target = bytearray(len(payload))
    read_into(side, memoryview(target), **layout)
    assert bytes(target) == payload
    monkeypatch.setattr(codec.os, "pread", lambda *args: b"")
    with pytest.raises(ValueError, match="ended early"):
        read_into(side, memoryview(target), **layout)


def test_a_second_frame_inside_one_record_is_refused(tmp_path):
    src, side, payload, layout, manifest = sidecar_case(tmp_path)
    blob = side / "payload.zst"
    raw = blob.read_bytes()
    first = manifest["frames"][0][1]
    extra = pa.Codec("zstd", compression_level=3).compress(b"not a declared frame", asbytes=True)
    blob.write_bytes(raw[:first] + extra + raw[first:])
    manifest["frames"][0][1] += len(extra)
    for record in manifest["frames"][1:]:
        record[0] += len(extra)
    manifest["compressed_bytes"] += len(extra)
    (side / "index.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="beyond its one frame"):
        read_into(side, memoryview(bytearray(len(payload))), **layout)


@pytest.mark.parametrize("kind", ["symlink", "fifo", "list"])
def test_index_must_be_a_bounded_regular_object(tmp_path, kind):
    import os

    src, side, payload, layout, _manifest = sidecar_case(tmp_path)
    index = side / "index.json"
    if kind == "symlink":
        index.rename(side / "real.json")
        index.symlink_to(side / "real.json")
    elif kind == "fifo":
        index.unlink()
        os.mkfifo(index)
    else:
        index.write_text("[]")
    with pytest.raises((ValueError, OSError)):
        read_into(side, memoryview(bytearray(len(payload))), **layout)


def test_frame_length_walks_the_blocks():
    from vflash_b200.native.h3_weight_codec import frame_length

    codec = pa.Codec("zstd", compression_level=3)
    for data in (b"a", bytes(5000), bytes(range(256)) * 300):
        frame = codec.compress(data, asbytes=True)
        assert frame_length(frame) == len(frame)
        assert frame_length(frame + codec.compress(b"tail", asbytes=True)) == len(frame)
        with pytest.raises(ValueError, match="truncated"):
            frame_length(frame[:-1])


def test_prepare_accepts_any_dense_dtype_the_reference_accepts(tmp_path):
    path = tmp_path / "mixed.safetensors"
    from safetensors.torch import save_file

    save_file({"a": torch.arange(6, dtype=torch.float64), "b": torch.ones(3, dtype=torch.int16)}, str(path))
    manifest = prepare(path, tmp_path / "side", chunk_bytes=4096)
    payload, offset = payload_of(path)
    target = bytearray(len(payload))
    read_into(tmp_path / "side", memoryview(target), source_name=path.name, source_size=path.stat().st_size,
              header_bytes=offset)
    assert bytes(target) == payload and manifest["payload_bytes"] == len(payload)
