"""Row-chunked host <-> device pipeline for row-independent linears.

Every FP8/NVFP4 linear of this path maps each token row independently (the
activation scale is per token, ``src/vflash/native/h3_fp8_linear.py:18-31``,
and each output row depends only on its input row), so a host-resident
activation can be processed in row chunks with the host->device copy of chunk
c+1, the compute of chunk c and the device->host copy of chunk c-1 in flight
at once on three streams.  The result equals one call on all rows bit for bit.

PCIe is full duplex, so for an op whose output is larger than its input (the
merged QKV projection writes 3x its input bytes) the pipeline is bound by the
device->host copy alone instead of by the sum of both copies and the compute.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Sequence

import torch


def device_bus_id(device) -> str:
    """NVML-style PCI address (``DDDDDDDD:BB:DD.0``) of a CUDA device."""
    props = torch.cuda.get_device_properties(torch.device(device))
    return f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"


def cpu_set_for_bus_id(bus_id: str, nvml=None) -> set[int]:
    """CPUs local to the GPU at ``bus_id`` (NVML's CPU affinity), or an empty set if unknown.

    ``nvml`` defaults to the ``pynvml`` module; finding the device by PCI
    address keeps the mapping right under any ``CUDA_VISIBLE_DEVICES``.
    """
    if nvml is None:
        try:
            import pynvml as nvml
        except ImportError:
            return set()
    try:
        nvml.nvmlInit()
        try:
            handle = nvml.nvmlDeviceGetHandleByPciBusId(bus_id)
            masks = nvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        finally:
            nvml.nvmlShutdown()
    except Exception:
        return set()
    return {64 * w + b for w, mask in enumerate(masks) for b in range(64) if (int(mask) >> b) & 1}


def bind_host_to_device(device, nvml=None) -> set[int]:
    """Run this process on the CPUs local to ``device`` (returns them; no-op if unknown).

    Pinned buffers allocated afterwards are first touched by a thread on the
    GPU's own socket, so host<->device copies do not cross the socket link.
    Only this process's CPU affinity changes.
    """
    cpus = cpu_set_for_bus_id(device_bus_id(device), nvml) & set(os.sched_getaffinity(0))
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus


def plan_chunks(rows: int, chunk_rows: int, align: int = 16) -> list[tuple[int, int]]:
    """(begin, end) row ranges of at most ``chunk_rows`` rows; all but the last a multiple of ``align``."""
    if rows < 0 or chunk_rows < 1 or align < 1:
        raise ValueError("invalid chunk plan")
    step = max(align, chunk_rows // align * align)
    return [(b, min(rows, b + step)) for b in range(0, rows, step)]


class HostRowPipeline:
    """Apply ``fn`` to pinned host rows chunk by chunk, overlapping copies and compute.

    ``fn(x_dev) -> tuple of device tensors`` must map rows independently and
    return tensors whose first dimension is the chunk's rows (views of any
    layout are copied row-wise into the matching slice of ``outs``).  Two
    device input slots alternate; the compute of a chunk waits for its copy,
    the copy into a slot waits for the compute that last read it, and every
    output waits for its compute before its device->host copy, which keeps
    the output alive until it has been read (``record_stream``).
    """

    def __init__(self, fn: Callable[[torch.Tensor], Sequence[torch.Tensor]], device, *,
                 chunk_rows: int = 4096) -> None:
        self.fn = fn
        self.device = torch.device(device)
        self.chunk_rows = chunk_rows
        self.h2d = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        self._slots: list[torch.Tensor] = []
        self._loaded = [torch.cuda.Event(), torch.cuda.Event()]
        self._consumed = [torch.cuda.Event(), torch.cuda.Event()]
        self._copied_out = torch.cuda.Event()

    def _slot(self, index: int, like: torch.Tensor, rows: int) -> torch.Tensor:
        shape = (self.chunk_rows, *like.shape[1:])
        if len(self._slots) < 2 or self._slots[0].shape != shape or self._slots[0].dtype != like.dtype:
            self._slots = [torch.empty(shape, dtype=like.dtype, device=self.device) for _ in range(2)]
        return self._slots[index][:rows]

    def __call__(self, x_host: torch.Tensor, outs: Sequence[torch.Tensor]) -> Sequence[torch.Tensor]:
        if x_host.device.type != "cpu" or not x_host.is_pinned():
            raise ValueError("host rows must be a pinned CPU tensor")
        for out in outs:
            if out.device.type != "cpu" or not out.is_pinned() or out.shape[0] != x_host.shape[0]:
                raise ValueError("outputs must be pinned CPU tensors with the input's rows")
        compute = torch.cuda.current_stream(self.device)
        chunks = plan_chunks(x_host.shape[0], self.chunk_rows)
        for c, (begin, end) in enumerate(chunks):
            slot = c % 2
            dev_in = self._slot(slot, x_host, end - begin)
            with torch.cuda.stream(self.h2d):
                self.h2d.wait_event(self._consumed[slot])
                dev_in.copy_(x_host[begin:end], non_blocking=True)
                self._loaded[slot].record(self.h2d)
            compute.wait_event(self._loaded[slot])
            results = self.fn(dev_in)
            self._consumed[slot].record(compute)
            if len(results) != len(outs):
                raise ValueError("fn returned a different number of outputs")
            self.d2h.wait_stream(compute)
            with torch.cuda.stream(self.d2h):
                for res, out in zip(results, outs):
                    res.record_stream(self.d2h)
                    out[begin:end].copy_(res.reshape(out[begin:end].shape), non_blocking=True)
        self._copied_out.record(self.d2h)
        compute.wait_event(self._copied_out)
        return outs
