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

``PinnedNVFP4Linears`` does the same for the packed NVFP4 file of a QAD
checkpoint (src/vflash/adapters/h3_qad.py:96-134): the reference's exact key
set, every linear read into one pinned chunk, one device allocation and one
copy per linear when the weights are put on the GPU.
"""

from __future__ import annotations

import contextlib
import json
import math
import os
import struct
from collections.abc import Iterable
from pathlib import Path

import torch

from .h3_pinned_arena import BlockLayout, PinnedHostArena

HEADER_LIMIT = 100 * 1024 * 1024
# element sizes of the safetensors dtypes (a block file may carry tensors of any of them)
DTYPE_BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "F8_E4M3": 1, "F8_E5M2": 1, "I64": 8, "I32": 4,
               "I16": 2, "I8": 1, "U64": 8, "U32": 4, "U16": 2, "U8": 1, "BOOL": 1}

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


# ---------------------------------------------------------------------------
# QAD NVFP4 checkpoints
# ---------------------------------------------------------------------------
# main-block linear (module name inside a transformer block) -> its prefix in
# the packed file (src/vflash/adapters/h3_qad.py:22-29)
QAD_LINEARS = {"attn.to_q": "attn.to_q", "attn.to_k": "attn.to_k", "attn.to_v": "attn.to_v",
               "attn.to_out.0": "attn.to_out", "ff.net.0.proj": "ff.fc_in", "ff.net.2": "ff.fc_out"}
# fields every packed linear carries; FFN linears add the calibrated input scale
# (h3_qad.py:106-118); the others run with a unit input scale (h3_qad.py:121-128)
QAD_FIELDS = ("_nvfp4_weight", "_nvfp4_weight_scale", "_nvfp4_alpha", "_weight_global_sf")
QAD_INPUT_SF = "_nvfp4_input_global_sf"


def qad_targets(blocks: int = 50, linears: dict[str, str] = QAD_LINEARS) -> dict[str, str]:
    """Module name -> packed-file prefix for every main-block linear (h3_qad.py:63-67)."""
    return {f"transformer_blocks.{i}.{name}": f"transformer_blocks.{i}.{source}"
            for i in range(blocks) for name, source in linears.items()}


def qad_required_keys(prefixes: Iterable[str]) -> set[str]:
    prefixes = list(prefixes)
    keys = {f"{p}::{f}" for p in prefixes for f in QAD_FIELDS}
    keys.update(f"{p}::{QAD_INPUT_SF}" for p in prefixes if ".ff." in p)
    return keys


def _aligned(n: int) -> int:
    return (n + 255) // 256 * 256


class PinnedNVFP4Linears:
    """Every packed NVFP4 linear of a QAD checkpoint, read once into pinned host memory.

    Replaces the reference's ``safe_open`` + ``get_tensor`` pass over the
    packed file (h3_qad.py:104-134) and its per-tensor ``.to(device)`` copies
    (h3_qad.py:151-168).  The key set must equal the reference's required set
    exactly; each linear's packed codes (U8 ``[N, K/2]``), block scales (U8
    ``[N, K/16]``, 128x4 order), ``alpha`` and input scale (F32 scalars; 1.0
    for the attention linears) are read with positioned reads into one
    256-byte aligned pinned chunk per linear.  ``weights`` holds host
    ``NVFP4Weight`` views (validated by its own contract); ``materialize``
    puts every linear on a device in one allocation with one asynchronous
    copy per linear, and returns device ``NVFP4Weight`` views of it.
    """

    def __init__(self, path, *, blocks: int = 50, linears: dict[str, str] = QAD_LINEARS,
                 arena: PinnedHostArena | None = None) -> None:
        from .h3_nvfp4_linear import NVFP4Weight

        path = Path(path)
        offset, entries = read_header(path)
        targets = qad_targets(blocks, linears)
        if set(entries) != qad_required_keys(targets.values()):
            raise ValueError(f"QAD must cover all {len(targets)} original main-block linears")
        plans = {}
        for name, prefix in targets.items():
            packed = entries[prefix + "::_nvfp4_weight"]
            if packed["dtype"] != "U8" or len(packed["shape"]) != 2:
                raise ValueError(f"{prefix}::_nvfp4_weight must be U8 [N, K/2]")
            n, half_k = packed["shape"]
            _expect(entries, prefix + "::_nvfp4_weight_scale", "U8", (n, half_k // 8))
            for field in ("_nvfp4_alpha", "_weight_global_sf") + ((QAD_INPUT_SF,) if ".ff." in prefix else ()):
                _expect(entries, f"{prefix}::{field}", "F32", ())
            sizes = (n * half_k, n * (half_k // 8), 4, 4)
            starts, at = [], 0
            for size in sizes:
                starts.append(at)
                at = _aligned(at + size)
            plans[name] = (prefix, n, half_k, starts, at)
        largest = max(plan[4] for plan in plans.values())
        self.arena = arena or PinnedHostArena(max(2 * 1024**3, 1 << (largest - 1).bit_length()))
        self.chunks: dict[str, torch.Tensor] = {}
        self.plans = plans
        self.weights: dict[str, NVFP4Weight] = {}
        with path.open("rb", buffering=0) as handle:
            fd = handle.fileno()
            for name, (prefix, n, half_k, starts, nbytes) in plans.items():
                chunk = self.arena.empty(nbytes)
                chunk.zero_()
                view = memoryview(chunk.numpy())
                try:
                    sources = ("_nvfp4_weight", "_nvfp4_weight_scale", "_nvfp4_alpha",
                               QAD_INPUT_SF if ".ff." in prefix else None)
                    for field, start in zip(sources, starts):
                        if field is None:
                            continue
                        entry = entries[f"{prefix}::{field}"]
                        _pread_into(fd, view[start:start + entry["end"] - entry["begin"]],
                                    offset + entry["begin"])
                finally:
                    view.release()
                if ".ff." not in prefix:
                    chunk[starts[3]:starts[3] + 4].view(torch.float32).fill_(1.0)
                self.chunks[name] = chunk
                self.weights[name] = self._views(chunk, n, half_k, starts)
        if arena is None:
            self.arena.close()

    @staticmethod
    def _views(chunk: torch.Tensor, n: int, half_k: int, starts: list[int]):
        from .h3_nvfp4_linear import NVFP4Weight

        return NVFP4Weight(chunk[starts[0]:starts[0] + n * half_k].view(n, half_k),
                           chunk[starts[1]:starts[1] + n * (half_k // 8)].view(n, half_k // 8),
                           chunk[starts[2]:starts[2] + 4].view(torch.float32).reshape(()),
                           chunk[starts[3]:starts[3] + 4].view(torch.float32).reshape(()))

    @property
    def nbytes(self) -> int:
        return sum(chunk.numel() for chunk in self.chunks.values())

    def materialize(self, device) -> dict:
        """Device ``NVFP4Weight`` views of every linear: one allocation, one copy per linear.

        The copies are enqueued on the current stream of ``device`` from
        pinned memory; kernels on that stream see the weights in order.
        """
        device = torch.device(device)
        slab = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        out, at = {}, 0
        with torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext():
            for name, chunk in self.chunks.items():
                target = slab[at:at + chunk.numel()]
                target.copy_(chunk, non_blocking=True)
                _prefix, n, half_k, starts, nbytes = self.plans[name]
                out[name] = self._views(target, n, half_k, starts)
                at += nbytes
        return out
