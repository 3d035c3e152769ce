"""Read FP8 block weights from the reference's safetensors files straight into the pinned arena.

Each H3 block file holds the four FP8 linears as ``X.weight`` (F8_E4M3
``[N, K]``) and ``X.weight.row_scale`` (F32 ``[N, 1]``), keys ``attn.qkv``,
``attn.out``, ``ffn.in`` and ``ffn.out`` (src/vflash/native/h3_fp8_runtime.py:
87-96).  The header is validated as the reference's dense safetensors
inspection does (src/vflash/native/h3_tensor_file.py:290-367: bounded header,
known dtypes, shapes matching byte ranges, payload ranges without gaps or
overlaps covering the file), then every tensor's bytes are read with
positioned reads directly into its field of the packed block in pinned host
memory (``BlockLayout``) — no intermediate buffer, no second copy.  With a
process group each rank reads only the byte range of every block that it
pins (its 1/n share for ``FP8BlockRing``'s all-gather).
"""

from __future__ import annotations

import json
import math
import os
import struct
from collections.abc import Iterable
from pathlib import Path

import torch

from .h3_pinned_arena import BlockLayout, PinnedHostArena

HEADER_LIMIT = 100 * 1024 * 1024
DTYPE_BYTES = {"F8_E4M3": 1, "F32": 4, "BF16": 2, "F16": 2, "U8": 1, "I8": 1, "I32": 4, "I64": 8}

# block linear -> safetensors key of its FP8 codes (the scales are key + ".row_scale")
FP8_BLOCK_KEYS = {"qkv": "attn.qkv.weight", "attention_out": "attn.out.weight",
                  "ffn_in": "ffn.in.weight", "ffn_out": "ffn.out.weight"}


def read_header(path: Path) -> tuple[int, dict[str, dict]]:
    """(payload offset, tensor entries) of a dense safetensors file, validated."""
    path = Path(path)
    size = path.stat().st_size
    with path.open("rb") as handle:
        prefix = handle.read(8)
        if len(prefix) != 8:
            raise ValueError(f"safetensors prefix is truncated: {path.name}")
        header_size = struct.unpack("<Q", prefix)[0]
        if header_size < 2 or header_size > HEADER_LIMIT or header_size > size - 8:
            raise ValueError(f"safetensors header size is invalid: {path.name}")
        try:
            header = json.loads(handle.read(header_size).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as exc:
            raise ValueError(f"safetensors header is invalid: {path.name}") from exc
    if not isinstance(header, dict):
        raise ValueError(f"safetensors header must be an object: {path.name}")
    entries = {}
    for name, row in header.items():
        if name == "__metadata__":
            continue
        if not isinstance(row, dict):
            raise ValueError(f"safetensors tensor entry is invalid: {name}")
        dtype, shape, offsets = row.get("dtype"), row.get("shape"), row.get("data_offsets")
        if dtype not in DTYPE_BYTES or not isinstance(shape, list) or any(
                not isinstance(d, int) or isinstance(d, bool) or d < 0 for d in shape):
            raise ValueError(f"unsupported or malformed tensor layout: {name}")
        if (not isinstance(offsets, list) or len(offsets) != 2
                or offsets[1] - offsets[0] != math.prod(shape) * DTYPE_BYTES[dtype] or offsets[0] < 0):
            raise ValueError(f"tensor byte range differs from its shape: {name}")
        entries[name] = {"dtype": dtype, "shape": shape, "begin": offsets[0], "end": offsets[1]}
    end = 0
    for begin, stop in sorted((e["begin"], e["end"]) for e in entries.values()):
        if begin != end:
            raise ValueError("checkpoint offsets have gaps or overlaps")
        end = stop
    offset = 8 + header_size
    if offset + end != size:
        raise ValueError("checkpoint bytes differ from header")
    return offset, entries


def _expect(entries: dict, key: str, dtype: str, shape: tuple[int, ...]) -> dict:
    entry = entries.get(key)
    if entry is None:
        raise ValueError(f"block file has no tensor {key}")
    if entry["dtype"] != dtype or tuple(entry["shape"]) != shape:
        raise ValueError(f"{key} is {entry['dtype']} {entry['shape']}, expected {dtype} {list(shape)}")
    return entry


def _pread_into(fd: int, view: memoryview, file_offset: int) -> None:
    done = 0
    while done < len(view):
        count = os.preadv(fd, [view[done:]], file_offset + done)
        if count <= 0:
            raise ValueError("weight file ended during a positioned read")
        done += count


def pin_fp8_block_files(paths: Iterable[Path], layout: BlockLayout, arena: PinnedHostArena, *,
                        rank: int = 0, world: int = 1) -> list[torch.Tensor]:
    """This rank's byte range of each packed block, read from its file into the arena.

    ``layout`` names its linears as ``FP8_BLOCK_KEYS``; each field (codes or
    row scales of one linear) is matched to its tensor by dtype and shape.
    """
    if layout.nbytes % world:
        raise ValueError("packed block size must divide evenly between the ranks")
    chunk = layout.nbytes // world
    lo, hi = rank * chunk, (rank + 1) * chunk
    out = []
    for path in paths:
        offset, entries = read_header(Path(path))
        host = arena.empty(chunk)
        host.zero_()  # padding between fields
        view = memoryview(host.numpy())
        try:
            with Path(path).open("rb", buffering=0) as handle:
                fd = handle.fileno()
                for field in layout.fields:
                    key = FP8_BLOCK_KEYS[field.name] + ("" if field.kind == "codes" else ".row_scale")
                    dtype = "F8_E4M3" if field.kind == "codes" else "F32"
                    entry = _expect(entries, key, dtype, field.shape)
                    begin, end = max(lo, field.offset), min(hi, field.offset + field.nbytes)
                    if begin >= end:
                        continue
                    _pread_into(fd, view[begin - lo:end - lo], offset + entry["begin"] + begin - field.offset)
        finally:
            view.release()
        out.append(host)
    return out
