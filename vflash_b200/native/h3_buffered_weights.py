"""Owned-buffer reads of immutable safetensors files (drop-in for the reference's buffered reader).

Mirrors Hansimov/vflash src/vflash/native/h3_buffered_weights.py:
``SequentialWeights`` is a ``safe_open``-like context manager that reads a
whole shard's payload into ONE host buffer (sequentially, with 1/2/4/8
parallel positioned reads, or by decoding its framed zstd sidecar) and hands
out tensors that are views of that buffer, so a tensor kept after the scope
keeps the whole buffer alive; ``host_headroom`` bounds the read by the host
memory available to this process; ``payload_header`` validates the header
as the reference's ``inspect_dense_safetensors`` (src/vflash/native/
h3_tensor_file.py:289-367) does, with the same error texts.

B200 addition (keyword-only, off by default): ``pin_memory=True`` reads the
payload straight into page-locked memory, so tensors taken from it reach the
GPU by asynchronous copies (``tensor.to(device, non_blocking=True)``) with no
staging copy.
"""

from __future__ import annotations

import json
import math
import os
import re
import stat
import struct
import time
from pathlib import Path

import torch

DTYPES = {
    "F32": torch.float32,
    "F16": torch.float16,
    "BF16": torch.bfloat16,
    "F8_E4M3": torch.float8_e4m3fn,
    "I64": torch.int64,
    "I32": torch.int32,
    "I16": torch.int16,
    "I8": torch.int8,
    "U8": torch.uint8,
    "BOOL": torch.bool,
}
HEADER_LIMIT = 100 * 1024 * 1024
_DTYPE_NAME = re.compile(r"[A-Z][A-Z0-9_]{0,15}")


class _HeaderError(Exception):
    pass


def identity(value):
    return value.st_dev, value.st_ino, value.st_size, value.st_mtime_ns, value.st_ctime_ns


def host_headroom():
    """Bytes of host memory this process may still use: MemAvailable, capped by its cgroup's limit."""
    available = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                available = int(line.split()[1]) * 1024
                break
    except OSError:
        pass
    try:
        maximum = Path("/sys/fs/cgroup/memory.max").read_text().strip()
        current = int(Path("/sys/fs/cgroup/memory.current").read_text())
        if maximum.isdigit():
            available = min(available, max(0, int(maximum) - current))
    except OSError:
        pass
    return available


def _inspect(path: Path):
    try:
        before = path.stat()
    except OSError as exc:
        raise _HeaderError from exc
    if not stat.S_ISREG(before.st_mode):
        raise _HeaderError
    try:
        with path.open("rb") as handle:
            if identity(os.fstat(handle.fileno())) != identity(before):
                raise _HeaderError
            prefix = handle.read(8)
            if len(prefix) != 8:
                raise _HeaderError
            header_size = struct.unpack("<Q", prefix)[0]
            if header_size < 2 or header_size > HEADER_LIMIT or header_size > before.st_size - 8:
                raise _HeaderError
            header = json.loads(handle.read(header_size).decode("utf-8"))
    except (OSError, UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise _HeaderError from exc
    if not isinstance(header, dict):
        raise _HeaderError
    data_size = before.st_size - 8 - header_size
    rows, spans = {}, []
    for name, value in header.items():
        if name == "__metadata__":
            if not isinstance(value, dict):
                raise _HeaderError
            continue
        if not isinstance(name, str) or not name or not isinstance(value, dict):
            raise _HeaderError
        dtype, shape, offsets = value.get("dtype"), value.get("shape"), value.get("data_offsets")
        if not isinstance(dtype, str) or not _DTYPE_NAME.fullmatch(dtype):
            raise _HeaderError
        if not isinstance(shape, list) or any(type(d) is not int or d < 0 for d in shape):
            raise _HeaderError
        if not isinstance(offsets, list) or len(offsets) != 2 or any(type(o) is not int for o in offsets):
            raise _HeaderError
        start, stop = offsets
        if start < 0 or stop < start or stop > data_size:
            raise _HeaderError
        spans.append((start, stop))
        rows[name] = {"dtype": dtype, "shape": tuple(shape), "data_offsets": (start, stop)}
    if not rows:
        raise _HeaderError
    reach = 0
    for start, stop in sorted(spans):
        if start < reach:
            raise _HeaderError
        reach = max(reach, stop)
    return rows, 8 + header_size, before


def payload_header(path):
    """(payload offset, tensor rows) of a dense safetensors shard, validated without reading its payload."""
    try:
        rows, offset, before = _inspect(Path(path))
    except _HeaderError as exc:
        raise ValueError("invalid immutable tensor header") from exc
    end = 0
    for start, stop in sorted(row["data_offsets"] for row in rows.values()):
        if start != end:
            raise ValueError("checkpoint offsets have gaps or overlaps")
        end = stop
    if offset + end != before.st_size:
        raise ValueError("checkpoint bytes differ from header")
    return offset, rows


class SequentialWeights:
    """Read one safetensors shard into one owned host buffer; tensors are views of it."""

    def __init__(self, path, *, framework="pt", device="cpu", observation=None, read_workers=1,
                 compressed_directory=None, pin_memory=False):
        if framework != "pt" or device != "cpu":
            raise ValueError("sequential model reads require CPU Torch storage")
        if type(read_workers) is not int or read_workers not in (1, 2, 4, 8):
            raise ValueError("weight read concurrency must be 1, 2, 4 or 8")
        if read_workers > 1 and not hasattr(os, "preadv"):
            raise ValueError("parallel weight reads require positioned vector I/O")
        self.read_workers = read_workers
        self.compressed_directory = compressed_directory
        self.path = Path(path)
        self.observation = observation
        self.pin_memory = bool(pin_memory)
        self.tensors = {}

    def __enter__(self):
        start = time.monotonic()
        before = self.path.stat()
        offset, entries = payload_header(self.path)
        size = before.st_size - offset
        if not 0 < size <= 12 * 1024**3 or host_headroom() < size + 2 * 1024**3:
            raise ValueError("sequential weight read exceeds its bounded host memory budget")
        specs = []
        for name, row in entries.items():
            dtype = DTYPES.get(row["dtype"])
            begin, end = row["data_offsets"]
            if (dtype is None or begin % dtype.itemsize
                    or end - begin != math.prod(row["shape"]) * dtype.itemsize):
                raise ValueError("unsupported or malformed sequential tensor layout")
            specs.append((name, dtype, row["shape"], begin, end))
        buffer = torch.empty(size, dtype=torch.uint8, device="cpu", pin_memory=self.pin_memory)
        view = memoryview(buffer.numpy())
        try:
            with self.path.open("rb", buffering=0) as stream:
                if identity(os.fstat(stream.fileno())) != identity(before):
                    raise ValueError("weight source changed before sequential read")
                if self.compressed_directory is not None:
                    from .h3_weight_codec import read_into

                    compressed = read_into(Path(self.compressed_directory), view, source_name=self.path.name,
                                           source_size=before.st_size, header_bytes=offset,
                                           workers=self.read_workers)
                    if self.observation is not None:
                        self.observation["compressed_bytes"] = (self.observation.get("compressed_bytes", 0)
                                                                + compressed["compressed_bytes"])
                elif self.read_workers == 1:
                    stream.seek(offset)
                    count = 0
                    while count < size:
                        got = stream.readinto(view[count:min(size, count + 8 * 1024**2)])
                        if not got:
                            raise ValueError("weight source ended during sequential read")
                        count += got
                else:
                    _parallel_read(stream.fileno(), view, offset, size, self.read_workers)
                if (identity(os.fstat(stream.fileno())) != identity(before)
                        or identity(self.path.stat()) != identity(before)):
                    raise ValueError("weight source changed during sequential read")
            self.tensors = {name: buffer[begin:end].view(dtype).reshape(shape)
                            for name, dtype, shape, begin, end in specs}
            if self.observation is not None:
                self.observation["files"] += 1
                self.observation["bytes"] += size
                self.observation["read_seconds"] += time.monotonic() - start
        except BaseException:
            # the traceback keeps this frame: drop the payload before re-raising
            self.tensors.clear()
            buffer = None
            raise
        finally:
            view.release()
        return self

    def keys(self):
        return self.tensors.keys()

    def get_tensor(self, name):
        return self.tensors[name]

    def __exit__(self, *args):
        # tensors already taken keep the buffer alive; the reader lets go of it
        self.tensors.clear()


def _parallel_read(fd: int, view: memoryview, offset: int, size: int, workers: int) -> None:
    """Disjoint byte ranges of the payload, one per worker, read with positioned reads into ``view``."""
    from concurrent.futures import ThreadPoolExecutor

    span = math.ceil(size / workers)

    def read_range(begin):
        end = min(size, begin + span)
        while begin < end:
            got = os.preadv(fd, [view[begin:min(end, begin + 8 * 1024**2)]], offset + begin)
            if not got:
                raise ValueError("weight source ended during parallel read")
            begin += got

    with ThreadPoolExecutor(max_workers=workers, thread_name_prefix="native-weight") as pool:
        list(pool.map(read_range, range(0, size, span)))
