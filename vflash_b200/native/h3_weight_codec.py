"""Lossless framed zstd sidecars of safetensors payloads (drop-in for the reference's codec).

Mirrors Hansimov/vflash src/vflash/native/h3_weight_codec.py: a sidecar
directory holds ``payload.zst`` (the source file's payload after its header,
cut into independent zstd frames of at most ``chunk_bytes`` decoded bytes)
and ``index.json`` (format 1: source name and size, header bytes, payload
bytes, chunk bound, compressed bytes and one ``[offset, compressed,
decoded]`` record per frame, written last).  ``prepare`` (25-82) writes one
and checks every frame by decoding it; ``read_into`` (85-183) validates the
index against the caller's source layout exactly as the reference does and
decodes the frames in parallel into disjoint slices of a caller-owned buffer.

The zstd codec is pyarrow's (the reference uses the ``zstandard`` module,
which this image does not have; both produce and read standard RFC 8878
frames).  The frame header is parsed here (``frame_parameters``) so that a
frame's declared content size and window are checked before it is decoded,
as the reference checks ``zstandard.get_frame_parameters``, and its block
headers are walked (``frame_length``) so that a record holding anything
after its one frame is refused, as the reference's ``allow_extra_data=False``
refuses it.

``pin_fp8_block_sidecars`` feeds the FP8 block ring from sidecars: only the
frames that overlap this rank's share of each packed block are decoded, and
their bytes land in the block's fields in pinned memory.
"""

from __future__ import annotations

import json
import os
import stat
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CHUNK = 16 * 1024**2
MAX_FILE = 12 * 1024**3
ZSTD_MAGIC = 0xFD2FB528


def _codec(level: int | None = None):
    import pyarrow as pa

    if not pa.Codec.is_available("zstd"):
        raise RuntimeError("this pyarrow build has no zstd codec")
    return pa.Codec("zstd", compression_level=level) if level is not None else pa.Codec("zstd")


def identity(value):
    return value.st_dev, value.st_ino, value.st_size, value.st_mtime_ns, value.st_ctime_ns


def frame_parameters(frame: bytes) -> tuple[int | None, int]:
    """(content size or None, window size) from a zstd frame header (RFC 8878 section 3.1.1)."""
    if len(frame) < 6 or int.from_bytes(frame[:4], "little") != ZSTD_MAGIC:
        raise ValueError("compressed frame is not a zstd frame")
    descriptor = frame[4]
    fcs_flag, single_segment, dict_flag = descriptor >> 6, (descriptor >> 5) & 1, descriptor & 3
    if descriptor & 0x08:
        raise ValueError("compressed frame sets a reserved header bit")
    at = 5
    window = None
    if not single_segment:
        exponent, mantissa = frame[at] >> 3, frame[at] & 7
        base = 1 << (10 + exponent)
        window = base + (base // 8) * mantissa
        at += 1
    dict_bytes = (0, 1, 2, 4)[dict_flag]
    if dict_bytes and int.from_bytes(frame[at:at + dict_bytes], "little"):
        raise ValueError("compressed frame needs a dictionary")
    at += dict_bytes
    fcs_bytes = (1 if single_segment else 0, 2, 4, 8)[fcs_flag]
    if len(frame) < at + fcs_bytes:
        raise ValueError("compressed frame header is truncated")
    content = None
    if fcs_bytes:
        content = int.from_bytes(frame[at:at + fcs_bytes], "little") + (256 if fcs_bytes == 2 else 0)
    if single_segment:
        window = content
    return content, window


def frame_length(frame: bytes) -> int:
    """Bytes of the zstd frame that starts ``frame``: header, blocks, optional checksum (RFC 8878 3.1.1).

    Each block header is 3 bytes (little endian: bit 0 last block, bits 1-2
    type, bits 3-23 size); a raw or compressed block carries ``size`` bytes,
    an RLE block one byte, type 3 is reserved.
    """
    if len(frame) < 6 or int.from_bytes(frame[:4], "little") != ZSTD_MAGIC:
        raise ValueError("compressed frame is not a zstd frame")
    descriptor = frame[4]
    fcs_flag, single_segment, checksum, dict_flag = (descriptor >> 6, (descriptor >> 5) & 1,
                                                     (descriptor >> 2) & 1, descriptor & 3)
    at = (5 + (0 if single_segment else 1) + (0, 1, 2, 4)[dict_flag]
          + (1 if single_segment else 0, 2, 4, 8)[fcs_flag])
    while True:
        if len(frame) < at + 3:
            raise ValueError("compressed frame is truncated")
        header = int.from_bytes(frame[at:at + 3], "little")
        last, kind, size = header & 1, (header >> 1) & 3, header >> 3
        if kind == 3:
            raise ValueError("compressed frame has a reserved block type")
        at += 3 + (1 if kind == 1 else size)
        if last:
            break
    at += 4 if checksum else 0
    if len(frame) < at:
        raise ValueError("compressed frame is truncated")
    return at


def prepare(source: Path, destination: Path, *, chunk_bytes=CHUNK):
    """Create one new sidecar; compare each decoded frame with its input."""
    from .h3_buffered_weights import payload_header

    source, destination = Path(source), Path(destination)
    if type(chunk_bytes) is not int or not 4096 <= chunk_bytes <= CHUNK:
        raise ValueError("bounded compression chunks required")
    before = source.stat()
    offset, _ = payload_header(source)
    payload = before.st_size - offset
    if not 0 < payload <= MAX_FILE or destination.exists() or destination.is_symlink():
        raise ValueError("one bounded source and a new destination required")
    destination.mkdir(mode=0o700)
    codec = _codec(3)
    records = []
    with source.open("rb", buffering=0) as original, (destination / "payload.zst").open("xb") as output:
        if identity(os.fstat(original.fileno())) != identity(before):
            raise ValueError("source changed before compression")
        original.seek(offset)
        remaining = payload
        while remaining:
            data = original.read(min(remaining, chunk_bytes))
            if not data:
                raise ValueError("source ended during compression")
            compressed = codec.compress(data, asbytes=True)
            content, _window = frame_parameters(compressed)
            if (content != len(data) or frame_length(compressed) != len(compressed)
                    or codec.decompress(compressed, len(data), asbytes=True) != data):
                raise ValueError("compressed frame differs from its source")
            records.append([output.tell(), len(compressed), len(data)])
            output.write(compressed)
            remaining -= len(data)
        output.flush()
        os.fsync(output.fileno())
        if (identity(os.fstat(original.fileno())) != identity(before)
                or identity(source.stat()) != identity(before)):
            raise ValueError("source changed during compression")
    manifest = dict(format=1, source_name=source.name, source_size=before.st_size, header_bytes=offset,
                    payload_bytes=payload, chunk_bytes=chunk_bytes,
                    compressed_bytes=(destination / "payload.zst").stat().st_size, frames=records,
                    verified_roundtrip=True)
    # manifest last: a failed preparation is never a consumable sidecar
    with (destination / "index.json").open("x") as handle:
        json.dump(manifest, handle, separators=(",", ":"))
        handle.flush()
        os.fsync(handle.fileno())
    return manifest


def _read_index(directory: Path) -> dict:
    index = directory / "index.json"
    fd = os.open(index, os.O_RDONLY | os.O_NOFOLLOW | os.O_NONBLOCK)
    with os.fdopen(fd, "rb") as handle:
        before = os.fstat(handle.fileno())
        if not stat.S_ISREG(before.st_mode) or not 0 < before.st_size <= 1024**2:
            raise ValueError("bounded regular compression index required")
        raw = handle.read(1024**2 + 1)
        if (len(raw) != before.st_size or identity(os.fstat(handle.fileno())) != identity(before)
                or identity(index.stat()) != identity(before)):
            raise ValueError("compression index changed during read")
    data = json.loads(raw)
    if not isinstance(data, dict):
        raise ValueError("compression index must be an object")
    return data


def _frame_plan(data: dict, *, source_name, source_size, header_bytes, target_bytes) -> list[tuple]:
    """(compressed offset, compressed bytes, payload offset, decoded bytes) per frame, validated."""
    size = source_size - header_bytes
    if (data.get("format") != 1 or data.get("verified_roundtrip") is not True
            or data.get("source_name") != source_name or Path(source_name).name != source_name
            or data.get("source_size") != source_size or data.get("header_bytes") != header_bytes
            or data.get("payload_bytes") != size or target_bytes != size or not 0 < size <= MAX_FILE):
        raise ValueError("compression source layout differs")
    chunk = data.get("chunk_bytes")
    if type(chunk) is not int or not 4096 <= chunk <= CHUNK:
        raise ValueError("invalid compression chunk bound")
    frames = data.get("frames")
    if not isinstance(frames, list) or not 1 <= len(frames) <= MAX_FILE // 4096:
        raise ValueError("invalid compression frames")
    plan = []
    compressed_end = output_end = 0
    for row in frames:
        if not isinstance(row, list) or len(row) != 3 or any(type(x) is not int for x in row):
            raise ValueError("invalid compression frame record")
        begin, packed, decoded = row
        if (begin != compressed_end or not 0 < packed <= chunk + 1024**2 or not 0 < decoded <= chunk
                or output_end + decoded > size):
            raise ValueError("compression frames overlap or exceed bounds")
        plan.append((begin, packed, output_end, decoded))
        compressed_end += packed
        output_end += decoded
    if output_end != size or compressed_end != data.get("compressed_bytes"):
        raise ValueError("compression frames do not cover the declared payload")
    return plan


def _decode_frames(directory: Path, plan: list[tuple], compressed_bytes: int, sink, workers: int) -> None:
    """Decode every frame of ``plan`` and hand ``(payload offset, bytes)`` to ``sink``."""
    codec = _codec()
    path = directory / "payload.zst"
    fd = os.open(path, os.O_RDONLY | os.O_NOFOLLOW | os.O_NONBLOCK)
    try:
        before = os.fstat(fd)
        if not stat.S_ISREG(before.st_mode) or before.st_size != compressed_bytes:
            raise ValueError("compressed payload size or type differs")

        def read_frame(row):
            begin, packed, output, decoded = row
            pieces, remaining = [], packed
            while remaining:
                piece = os.pread(fd, remaining, begin)
                if not piece:
                    raise ValueError("compressed payload ended early")
                pieces.append(piece)
                begin += len(piece)
                remaining -= len(piece)
            frame = b"".join(pieces)
            content, window = frame_parameters(frame)
            if content != decoded or window is None or window > CHUNK:
                raise ValueError("compressed frame content/window exceeds declaration")
            if frame_length(frame) != packed:
                raise ValueError("compressed record holds data beyond its one frame")
            value = codec.decompress(frame, decoded, asbytes=True)
            if len(value) != decoded:
                raise ValueError("decoded frame size differs")
            sink(output, value)

        with ThreadPoolExecutor(max_workers=workers, thread_name_prefix="compressed-weight") as pool:
            list(pool.map(read_frame, plan))
        if identity(os.fstat(fd)) != identity(before) or identity(path.stat()) != identity(before):
            raise ValueError("compressed payload changed during read")
    finally:
        os.close(fd)


def read_into(directory: Path, target, *, source_name, source_size, header_bytes, workers=4):
    """Parallel independent frames fill disjoint slices of an owned CPU buffer."""
    if type(workers) is not int or workers not in (1, 2, 4, 8):
        raise ValueError("bounded compressed concurrency required")
    directory = Path(directory)
    data = _read_index(directory)
    plan = _frame_plan(data, source_name=source_name, source_size=source_size, header_bytes=header_bytes,
                       target_bytes=len(target))

    def sink(output, value):
        target[output:output + len(value)] = value

    _decode_frames(directory, plan, data["compressed_bytes"], sink, workers)
    return dict(compressed_bytes=data["compressed_bytes"], decoded_bytes=sum(r[3] for r in plan),
                frames=len(plan))


def pin_fp8_block_sidecars(blocks, layout, arena, *, rank: int = 0, world: int = 1, workers: int = 4):
    """This rank's byte range of each packed FP8 block, decoded from its sidecar.

    ``blocks`` yields ``(source safetensors path, sidecar directory)`` pairs;
    the header (and so every tensor's payload range) comes from the source
    file, the bytes from the sidecar.  Only the frames overlapping the fields
    of this rank's share are decoded, and each decoded frame is copied
    straight into the fields it covers.  Equal to ``pin_fp8_block_files`` on
    the source files.
    """
    import numpy as np

    from .h3_weight_files import FP8_BLOCK_KEYS, _expect, read_header

    if type(workers) is not int or workers not in (1, 2, 4, 8):
        raise ValueError("bounded compressed concurrency required")
    if layout.nbytes % world:
        raise ValueError("packed block size must divide evenly between the ranks")
    chunk = layout.nbytes // world
    lo, hi = rank * chunk, (rank + 1) * chunk
    out = []
    for source, directory in blocks:
        source, directory = Path(source), Path(directory)
        offset, entries = read_header(source)
        size = source.stat().st_size
        data = _read_index(directory)
        plan = _frame_plan(data, source_name=source.name, source_size=size, header_bytes=offset,
                           target_bytes=size - offset)
        # payload range -> block offset for every field byte this rank pins
        pieces = []
        for field in layout.fields:
            key = FP8_BLOCK_KEYS[field.name] + ("" if field.kind == "codes" else ".row_scale")
            entry = _expect(entries, key, "F8_E4M3" if field.kind == "codes" else "F32", field.shape)
            begin, end = max(lo, field.offset), min(hi, field.offset + field.nbytes)
            if begin < end:
                src = entry["begin"] + begin - field.offset
                pieces.append((src, src + end - begin, begin - lo))
        host = arena.empty(chunk)
        host.zero_()  # padding between fields
        view = host.numpy()
        needed = [r for r in plan if any(s < r[2] + r[3] and r[2] < e for s, e, _ in pieces)]

        def sink(output, value, pieces=pieces, view=view):
            frame = np.frombuffer(value, dtype=np.uint8)
            for s, e, dst in pieces:
                a, b = max(s, output), min(e, output + len(frame))
                if a < b:
                    view[dst + a - s:dst + b - s] = frame[a - output:b - output]

        _decode_frames(directory, needed, data["compressed_bytes"], sink, workers)
        out.append(host)
    return out
