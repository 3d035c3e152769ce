"""Pinned host arena and double-buffered FP8 weight streaming for the block stack.

``PinnedHostArena`` mirrors Hansimov/vflash src/vflash/native/h3_pinned_arena.py:8-79
(bump allocation of immutable host tensors inside power-of-two pinned slabs,
256-byte alignment, views keep their slab alive, close drops the allocator's
reference only).

``FP8BlockRing`` follows the two-slot ring of ``H3NativeDenoiserBF16Ring``
(src/vflash/native/h3_native_denoiser.py:1447-1927: a copy stream, ready and
compute-done events per slot, block i+2 copied into the slot block i used once
block i's compute has finished) for FP8 blocks, with two B200-specific
choices:

* every block is packed into ONE contiguous byte buffer (codes and row scales
  of its linears, 256-byte aligned), so a block crosses PCIe as one copy and
  a device slot is one allocation with fixed views;
* with a process group of n ranks (one per GPU), each rank pins and copies
  only its 1/n byte range of every block and an NCCL all-gather over NVLink
  assembles the block in every rank's slot: each block crosses PCIe once in
  total instead of once per GPU, and the pinned host memory of all ranks
  together holds one copy of the weights.

``resident=True`` instead keeps every block on the device after its first
copy (a stack of 48 H3 blocks is 9.7 GB of FP8 weights; B200 has 180 GB), and
``resident_blocks=R`` keeps the first R resident and streams the rest, and
``slots=S`` (default 2, as the reference) rotates the streamed blocks through
S device buffers, so each block's copy has S - 1 blocks of compute to land.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable
from dataclasses import dataclass
from typing import Any

import torch

from .h3_parallel import FP8Weight

ALIGN = 256


class PinnedHostArena:
    """Bump-allocate views across blocks without per-tensor power-of-two padding.

    Every returned tensor retains its allocation through Torch's own Storage;
    the allocator owns only the current slab, and closing drops that reference
    without invalidating live views.
    """

    def __init__(self, chunk_bytes: int = 2 * 1024**3, *, pin_memory: bool = True) -> None:
        if chunk_bytes < ALIGN or chunk_bytes & (chunk_bytes - 1):
            raise ValueError("host arena size must be a power of two of at least 256 bytes")
        self.chunk_bytes = chunk_bytes
        self.pin_memory = pin_memory
        self.allocation_count = 0
        self.payload_bytes = 0
        self._buffer: Any = None
        self._offset = 0
        self._closed = False

    def empty(self, nbytes: int) -> torch.Tensor:
        """A 256-byte aligned uint8 view of ``nbytes`` inside the current (or a new) slab."""
        if self._closed:
            raise RuntimeError("the host arena is closed")
        if nbytes <= 0 or nbytes > self.chunk_bytes:
            raise ValueError("a host tensor must fit entirely inside one arena slab")
        try:
            offset = (self._offset + ALIGN - 1) // ALIGN * ALIGN
            if self._buffer is None or offset + nbytes > self.chunk_bytes:
                # Pinned slabs are page aligned; pageable ones are over-allocated
                # by one line so the slab itself can start on a 256-byte boundary.
                extra = 0 if self.pin_memory else ALIGN
                raw = torch.empty(self.chunk_bytes + extra, dtype=torch.uint8, device="cpu",
                                  pin_memory=self.pin_memory)
                lead = (-raw.data_ptr()) % ALIGN
                if lead > extra:
                    raise RuntimeError("pinned host slab is not 256-byte aligned")
                self._buffer = raw.narrow(0, lead, self.chunk_bytes)
                self.allocation_count += 1
                offset = 0
            out = self._buffer.narrow(0, offset, nbytes)
            self._offset = offset + nbytes
            self.payload_bytes += nbytes
            return out
        except BaseException:
            self.close()
            raise

    def copy(self, source: torch.Tensor) -> torch.Tensor:
        """Synchronous CPU copy into one contiguous, dtype-aligned view."""
        if (
            not isinstance(source, torch.Tensor)
            or source.device.type != "cpu"
            or source.layout != torch.strided
            or source.requires_grad
        ):
            raise ValueError("the host arena requires dense CPU tensors without gradients")
        size = source.numel() * source.element_size()
        out = self.empty(size).view(source.dtype).reshape(source.shape)
        out.copy_(source)
        return out

    def close(self) -> None:
        self._buffer = None
        self._closed = True

    def __enter__(self) -> PinnedHostArena:
        return self

    def __exit__(self, *_: Any) -> None:
        self.close()


# ---------------------------------------------------------------------------
# packed FP8 blocks
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Field:
    name: str
    kind: str          # "codes" or "scale"
    offset: int
    shape: tuple[int, ...]
    dtype: torch.dtype

    @property
    def nbytes(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * torch.empty((), dtype=self.dtype).element_size()


@dataclass(frozen=True)
class BlockLayout:
    """Byte layout of one packed FP8 block: the codes and row scales of each linear."""

    fields: tuple[Field, ...]
    nbytes: int

    @staticmethod
    def for_shapes(shapes: Iterable[tuple[str, int, int]], multiple: int = ALIGN) -> BlockLayout:
        fields, offset = [], 0
        for name, n, k in shapes:
            for kind, shape, dtype in (("codes", (n, k), torch.float8_e4m3fn),
                                       ("scale", (n, 1), torch.float32)):
                offset = (offset + ALIGN - 1) // ALIGN * ALIGN
                f = Field(name, kind, offset, shape, dtype)
                fields.append(f)
                offset += f.nbytes
        total = (offset + multiple - 1) // multiple * multiple
        return BlockLayout(tuple(fields), total)

    def views(self, buffer: torch.Tensor) -> dict[str, FP8Weight]:
        parts: dict[str, dict[str, torch.Tensor]] = {}
        for f in self.fields:
            t = buffer.narrow(0, f.offset, f.nbytes).view(f.dtype).reshape(f.shape)
            parts.setdefault(f.name, {})[f.kind] = t
        return {name: FP8Weight(p["codes"], p["scale"]) for name, p in parts.items()}

    def pack(self, weights: dict[str, FP8Weight], out: torch.Tensor) -> None:
        """Copy ``weights`` (any device) into the packed byte buffer ``out``."""
        dest = self.views(out)
        for name, w in weights.items():
            dest[name].codes.copy_(w.codes)
            dest[name].row_scale.copy_(w.row_scale)


class FP8BlockRing:
    """Stream packed FP8 blocks host -> device through two slots, overlapped with compute.

    ``host_blocks`` are this rank's pinned byte buffers (the whole block, or
    with ``group`` its 1/n byte range); ``run(hidden, block_fn)`` applies
    ``block_fn(weights, hidden) -> hidden`` to every block in order on the
    current stream while the copy stream prefetches two blocks ahead.
    """

    def __init__(self, layout: BlockLayout, host_blocks: list[torch.Tensor], device: torch.device, *,
                 group=None, resident: bool = False, resident_blocks: int = 0, slots: int = 2,
                 profile: bool = False) -> None:
        import torch.distributed as dist

        self.layout = layout
        self.host_blocks = host_blocks
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if layout.nbytes % self.world:
            raise ValueError("packed block size must divide evenly between the ranks")
        self.chunk = layout.nbytes // self.world
        for b in host_blocks:
            if b.dtype != torch.uint8 or b.numel() != self.chunk:
                raise ValueError("host block buffers differ from the packed layout")
        n = len(host_blocks)
        # blocks [0, resident_count) stay on the device after their first copy;
        # the rest stream through two slots
        self.resident_count = n if resident else max(0, min(int(resident_blocks), n))
        self.resident = self.resident_count == n
        if slots < 2:
            raise ValueError("the ring needs at least two slots")
        # streamed blocks rotate through `slots` buffers: the copy of block i + slots
        # starts when block i's compute ends, so it has slots - 1 blocks of compute to land
        self.stream_slots = slots
        count = self.resident_count + min(slots, n - self.resident_count)
        self.slots = [torch.empty(layout.nbytes, dtype=torch.uint8, device=self.device)
                      for _ in range(count)]
        self.slot_views = [layout.views(s) for s in self.slots]
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.ready = [torch.cuda.Event() for _ in range(count)]
        self.done = [torch.cuda.Event() for _ in range(count)]
        self.loaded = [False] * count
        self.h2d_bytes = 0
        # profile=True: CUDA events around each block's host copy and all-gather on the copy stream
        self.profile = profile
        self.marks: list[tuple[torch.cuda.Event, torch.cuda.Event, torch.cuda.Event]] = []

    def _fetch(self, index: int, slot: int) -> None:
        """Queue block ``index`` into ``slot`` on the copy stream (after the slot's last use)."""
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.done[slot])
            marks = None
            if self.profile:
                marks = tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
                marks[0].record(self.copy_stream)
                self.marks.append(marks)
            assemble_block(self.slots[slot], self.host_blocks[index], rank=self.rank, world=self.world,
                           group=self.group, marks=marks)
            self.h2d_bytes += self.chunk
            self.ready[slot].record(self.copy_stream)

    def run(self, hidden: torch.Tensor, block_fn: Callable[[dict[str, FP8Weight], torch.Tensor], torch.Tensor],
            *, wait_ready: bool = True):
        """Apply ``block_fn`` block by block; ``wait_ready=False`` (resident and already loaded
        and synchronised only) skips the copy-stream events, as a CUDA graph capture needs."""
        compute = torch.cuda.current_stream(self.device)
        n = len(self.host_blocks)
        r = self.resident_count
        if not wait_ready and (r != n or not all(self.loaded)):
            raise ValueError("skipping the ready events needs every block resident and loaded")
        for i in range(r):
            if not self.loaded[i]:
                self._fetch(i, i)
                self.loaded[i] = True
        depth = self.stream_slots
        # the first streamed blocks load while the resident ones compute
        for j in range(min(depth, n - r)):
            self._fetch(r + j, r + j)
        for i in range(r):
            if wait_ready:
                compute.wait_event(self.ready[i])
            hidden = block_fn(self.slot_views[i], hidden)
        for i in range(r, n):
            slot = r + (i - r) % depth
            compute.wait_event(self.ready[slot])
            hidden = block_fn(self.slot_views[slot], hidden)
            self.done[slot].record(compute)
            if i + depth < n:
                self._fetch(i + depth, slot)
        return hidden

    def copy_times(self) -> tuple[float, float, int]:
        """Mean milliseconds per profiled block of the host copy and of the all-gather, and the block count.

        Synchronises the copy stream; clears the recorded events.
        """
        self.copy_stream.synchronize()
        h2d = [a.elapsed_time(b) for a, b, _ in self.marks]
        gather = [b.elapsed_time(c) for _, b, c in self.marks]
        count = len(self.marks)
        self.marks = []
        if not count:
            return 0.0, 0.0, 0
        return sum(h2d) / count, sum(gather) / count, count


def assemble_block(dest: torch.Tensor, host_chunk: torch.Tensor, *, rank: int = 0, world: int = 1,
                   group=None, marks=None) -> None:
    """Copy this rank's byte range of a packed block into ``dest``, then all-gather the rest.

    ``dest`` is the whole packed block on this rank's device; rank r's range
    is ``[r*chunk, (r+1)*chunk)``.  The all-gather is in place (the input is
    the output's own range), so it moves only the other ranks' bytes.
    ``marks`` (three timing events, the first already recorded) get the end
    of the host copy and the end of the all-gather recorded on the current
    stream.
    """
    import torch.distributed as dist

    chunk = host_chunk.numel()
    if dest.numel() != chunk * world:
        raise ValueError("block chunk sizes differ from the destination")
    stream = torch.cuda.current_stream(dest.device) if marks is not None else None
    if world == 1:
        dest.copy_(host_chunk, non_blocking=True)
        if marks is not None:
            marks[1].record(stream)
            marks[2].record(stream)
        return
    mine = dest.narrow(0, rank * chunk, chunk)
    mine.copy_(host_chunk, non_blocking=True)
    if marks is not None:
        marks[1].record(stream)
    dist.all_gather_into_tensor(dest, mine, group=group)
    if marks is not None:
        marks[2].record(stream)


def pin_blocks(layout: BlockLayout, blocks: Iterable[dict[str, FP8Weight]], arena: PinnedHostArena, *,
               rank: int = 0, world: int = 1) -> list[torch.Tensor]:
    """Pack each block and keep this rank's 1/world byte range of it in the pinned arena.

    Build the layout with ``multiple=256*world`` so every rank's range is a
    whole number of 256-byte lines.
    """
    if layout.nbytes % world:
        raise ValueError("packed block size must divide evenly between the ranks")
    chunk = layout.nbytes // world
    host = []
    staging = None
    for weights in blocks:
        device = next(iter(weights.values())).codes.device
        if staging is None or staging.device != device:
            staging = torch.zeros(layout.nbytes, dtype=torch.uint8, device=device)  # padding stays 0
        layout.pack(weights, staging)
        out = arena.empty(chunk)
        out.copy_(staging.narrow(0, rank * chunk, chunk))
        host.append(out)
    return host
