"""Owned-buffer shard reads: exact tensors, budgets, short reads, changed sources, sidecars, pinned buffers.

The cases follow the reference's own tests of its buffered reader
(vflash tests/test_buffered_weights.py); the pinned-memory variant is this
library's addition.
"""

from __future__ import annotations

import pytest
import torch

from vflash_b200.native import h3_buffered_weights as io
from vflash_b200.native.h3_buffered_weights import SequentialWeights, payload_header

save_file = pytest.importorskip("safetensors.torch").save_file


def tensors():
    return {
        "codes": torch.arange(24).reshape(3, 8).to(torch.float8_e4m3fn),
        "scale": torch.tensor([[0.1], [0.2], [0.3]]),
        "norm": torch.randn(8, generator=torch.Generator().manual_seed(0)).bfloat16(),
        "index": torch.arange(3),
        "flags": torch.tensor([True, False, True]),
        "empty": torch.empty((0, 3), dtype=torch.float16),
    }


@pytest.mark.parametrize("workers", [1, 2, 4, 8])
def test_values_lifetime_and_untouched_source(tmp_path, workers):
    path = tmp_path / "weights.safetensors"
    values = tensors()
    save_file(values, path)
    before = path.stat()
    observation = {"files": 0, "bytes": 0, "read_seconds": 0.0}
    with SequentialWeights(path, observation=observation, read_workers=workers) as source:
        loaded = {name: source.get_tensor(name) for name in source.keys()}
    assert set(loaded) == set(values)
    for name, got in loaded.items():
        assert got.dtype == values[name].dtype and got.shape == values[name].shape
        assert torch.equal(got.float(), values[name].float())
    assert observation["bytes"] == sum(t.numel() * t.element_size() for t in values.values())
    assert observation["files"] == 1
    after = path.stat()
    assert (before.st_size, before.st_mtime_ns, before.st_ctime_ns) == (after.st_size, after.st_mtime_ns,
                                                                        after.st_ctime_ns)


def test_memory_budget_and_truncated_payload(tmp_path, monkeypatch):
    path = tmp_path / "weights.safetensors"
    save_file({"w": torch.ones(4)}, path)
    monkeypatch.setattr(io, "host_headroom", lambda: 1)
    with pytest.raises(ValueError, match="memory budget"), SequentialWeights(path):
        pass
    monkeypatch.undo()
    with path.open("r+b") as handle:
        handle.truncate(path.stat().st_size - 1)
    with pytest.raises(ValueError, match="invalid immutable tensor header"), SequentialWeights(path):
        pass


def test_parallel_short_reads_and_end_of_file(tmp_path, monkeypatch):
    path = tmp_path / "weights.safetensors"
    values = torch.arange(3001, dtype=torch.int32)
    save_file({"w": values}, path)
    real = io.os.preadv
    monkeypatch.setattr(io.os, "preadv", lambda fd, buffers, offset: real(fd, [buffers[0][:7]], offset))
    with SequentialWeights(path, read_workers=4) as source:
        assert torch.equal(source.get_tensor("w"), values)
    monkeypatch.setattr(io.os, "preadv", lambda *args: 0)
    with pytest.raises(ValueError, match="ended during parallel"), SequentialWeights(path, read_workers=4):
        pass


def test_changed_source_and_bad_concurrency(tmp_path, monkeypatch):
    path = tmp_path / "weights.safetensors"
    save_file({"w": torch.ones(101)}, path)
    for workers in (0, True, 3, 16):
        with pytest.raises(ValueError, match="concurrency"):
            SequentialWeights(path, read_workers=workers)
    real = io.os.preadv

    def touch_while_reading(fd, buffers, offset):
        count = real(fd, buffers, offset)
        io.os.utime(path, ns=(path.stat().st_atime_ns, path.stat().st_mtime_ns + 1000))
        return count

    monkeypatch.setattr(io.os, "preadv", touch_while_reading)
    with pytest.raises(ValueError, match="source changed"), SequentialWeights(path, read_workers=2):
        pass


@pytest.mark.parametrize("compressed", [False, True])
@pytest.mark.parametrize("pinned", [False, True])
def test_tensors_outlive_the_scope_and_the_file(tmp_path, compressed, pinned):
    if pinned and not torch.cuda.is_available():
        # pinning needs a CUDA driver; without one the option is refused by torch
        pytest.skip("page-locked host memory needs a CUDA device")
    if compressed:
        pa = pytest.importorskip("pyarrow")
        if not pa.Codec.is_available("zstd"):
            pytest.skip("pyarrow without zstd")
        from vflash_b200.native.h3_weight_codec import prepare
    path = tmp_path / "weights.safetensors"
    values = {"codes": torch.arange(1024).remainder(41).to(torch.float8_e4m3fn), "scalar": torch.tensor(3.5),
              "empty": torch.empty((0, 7))}
    save_file(values, path)
    sidecar = tmp_path / "sidecar" if compressed else None
    if sidecar is not None:
        prepare(path, sidecar, chunk_bytes=4096)
    observation = {"files": 0, "bytes": 0, "read_seconds": 0.0}
    with SequentialWeights(path, compressed_directory=sidecar, read_workers=4, observation=observation,
                           pin_memory=pinned) as source:
        kept = {name: source.get_tensor(name) for name in values}
    path.unlink()
    for name, t in kept.items():
        assert torch.equal(t.reshape(-1).view(torch.uint8), values[name].reshape(-1).view(torch.uint8))
        assert t.is_pinned() == pinned or t.numel() == 0
    assert observation["files"] == 1
    assert ("compressed_bytes" in observation) is compressed


def test_a_failed_read_does_not_keep_the_payload(tmp_path, monkeypatch):
    import gc
    import weakref

    path = tmp_path / "weights.safetensors"
    save_file({"w": torch.ones(1000)}, path)
    original = io.torch.empty
    made = []

    def tracked(*args, **kwargs):
        value = original(*args, **kwargs)
        made.append(weakref.ref(value))
        return value

    monkeypatch.setattr(io.torch, "empty", tracked)
    monkeypatch.setattr(io.os, "preadv", lambda *args: 0)
    with pytest.raises(ValueError, match="ended during parallel") as failure, SequentialWeights(path, read_workers=4):
        pass
    gc.collect()
    assert failure.value.__traceback__ is not None
    assert made and all(ref() is None for ref in made)


def test_header_errors_use_the_reference_texts(tmp_path):
    path = tmp_path / "weights.safetensors"
    save_file({"a": torch.ones(4), "b": torch.zeros(2)}, path)
    offset, rows = payload_header(path)
    assert rows["a"]["shape"] == (4,) and rows["a"]["dtype"] == "F32" and offset > 8
    raw = path.read_bytes()
    (tmp_path / "short.safetensors").write_bytes(raw[:5])
    with pytest.raises(ValueError, match="invalid immutable tensor header"):
        payload_header(tmp_path / "short.safetensors")
    (tmp_path / "extra.safetensors").write_bytes(raw + b"\0" * 4)
    with pytest.raises(ValueError, match="differ from header"):
        payload_header(tmp_path / "extra.safetensors")


@pytest.mark.gpu
def test_pinned_read_copies_to_the_gpu_asynchronously(tmp_path):
    path = tmp_path / "weights.safetensors"
    values = {"codes": torch.arange(4096).remainder(97).to(torch.uint8).view(64, 64),
              "scale": torch.rand(64, 1, generator=torch.Generator().manual_seed(1))}
    save_file(values, path)
    with SequentialWeights(path, read_workers=2, pin_memory=True) as source:
        host = {name: source.get_tensor(name) for name in values}
    assert all(t.is_pinned() for t in host.values())
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        placed = {name: t.to("cuda", non_blocking=True) for name, t in host.items()}
    stream.synchronize()
    for name, t in placed.items():
        assert torch.equal(t.cpu(), values[name])
