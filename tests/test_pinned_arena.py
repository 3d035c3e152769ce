"""Pinned host arena, packed FP8 block layout and the per-rank block split (CPU, gloo).

The arena follows Hansimov/vflash src/vflash/native/h3_pinned_arena.py:8-79;
the tests restate that file's behaviour (alignment, slab rollover, lifetime,
rejections) with unpinned slabs, since pinning needs a GPU.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from vflash_b200.native.h3_parallel import FP8Weight
from vflash_b200.native.h3_pinned_arena import (
    ALIGN,
    BlockLayout,
    PinnedHostArena,
    assemble_block,
    pin_blocks,
)

SHAPES = (("qkv", 96, 64), ("attention_out", 32, 32), ("ffn_in", 128, 32), ("ffn_out", 32, 128))


def random_block(seed: int, shapes=SHAPES) -> dict[str, FP8Weight]:
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for name, n, k in shapes:
        codes = torch.randint(0, 256, (n, k), generator=gen, dtype=torch.uint8).view(torch.float8_e4m3fn)
        scale = torch.rand((n, 1), generator=gen) + 0.5
        out[name] = FP8Weight(codes, scale)
    return out


def test_copies_are_256_byte_aligned_and_share_a_slab():
    arena = PinnedHostArena(1 << 16, pin_memory=False)
    a = arena.copy(torch.arange(10, dtype=torch.int16))
    b = arena.copy(torch.arange(7, dtype=torch.float32).reshape(7, 1))
    c = arena.copy(torch.ones(3, 5, dtype=torch.bfloat16))
    for t in (a, b, c):
        assert t.data_ptr() % ALIGN == 0
        assert t.is_contiguous()
    assert arena.allocation_count == 1
    assert arena.payload_bytes == 20 + 28 + 30
    assert b.data_ptr() - a.data_ptr() == ALIGN and c.data_ptr() - b.data_ptr() == ALIGN
    assert torch.equal(a, torch.arange(10, dtype=torch.int16))
    assert torch.equal(b, torch.arange(7, dtype=torch.float32).reshape(7, 1))
    assert b.shape == (7, 1) and c.dtype == torch.bfloat16


def test_full_slab_rolls_over_and_views_outlive_close():
    arena = PinnedHostArena(1024, pin_memory=False)
    first = arena.copy(torch.full((600,), 3, dtype=torch.uint8))
    second = arena.copy(torch.full((600,), 4, dtype=torch.uint8))  # 768 + 600 > 1024: new slab
    exact = arena.copy(torch.full((1024,), 5, dtype=torch.uint8))   # a whole slab
    assert arena.allocation_count == 3
    arena.close()
    assert int(first.sum()) == 3 * 600 and int(second.sum()) == 4 * 600 and int(exact.sum()) == 5 * 1024
    with pytest.raises(RuntimeError, match="closed"):
        arena.copy(torch.zeros(4))


def test_context_manager_closes():
    with PinnedHostArena(256, pin_memory=False) as arena:
        arena.copy(torch.zeros(2))
    with pytest.raises(RuntimeError, match="closed"):
        arena.empty(16)


@pytest.mark.parametrize("size", [0, 255, 3 << 10, 1000])
def test_rejects_sizes_that_are_not_powers_of_two_of_at_least_256(size):
    with pytest.raises(ValueError, match="power of two"):
        PinnedHostArena(size, pin_memory=False)


def test_rejects_oversize_strided_and_grad_tensors():
    arena = PinnedHostArena(256, pin_memory=False)
    with pytest.raises(ValueError, match="one arena slab"):
        arena.copy(torch.zeros(65, dtype=torch.float32))
    assert arena._closed is False
    with pytest.raises(ValueError, match="dense CPU"):
        arena.copy(torch.zeros(4, 4).to_sparse())
    with pytest.raises(ValueError, match="dense CPU"):
        arena.copy(torch.zeros(4, requires_grad=True))
    with pytest.raises(ValueError, match="dense CPU"):
        arena.copy([1, 2, 3])


def test_non_contiguous_sources_are_copied_densely():
    arena = PinnedHostArena(4096, pin_memory=False)
    src = torch.arange(64, dtype=torch.float32).reshape(8, 8).t()
    out = arena.copy(src)
    assert out.is_contiguous() and torch.equal(out, src)


def test_block_layout_pack_round_trip():
    layout = BlockLayout.for_shapes([(n, r, c) for n, r, c in SHAPES])
    assert layout.nbytes % ALIGN == 0
    for f in layout.fields:
        assert f.offset % ALIGN == 0
    block = random_block(1)
    buf = torch.zeros(layout.nbytes, dtype=torch.uint8)
    layout.pack(block, buf)
    views = layout.views(buf)
    for name, w in block.items():
        assert torch.equal(views[name].codes.view(torch.uint8), w.codes.view(torch.uint8))
        assert torch.equal(views[name].row_scale, w.row_scale)
        assert (views[name].codes.data_ptr() - buf.data_ptr()) % ALIGN == 0


def test_rank_ranges_concatenate_to_the_packed_block():
    world = 4
    layout = BlockLayout.for_shapes(SHAPES, multiple=ALIGN * world)
    blocks = [random_block(s) for s in range(3)]
    arena = PinnedHostArena(1 << 20, pin_memory=False)
    per_rank = [pin_blocks(layout, blocks, arena, rank=r, world=world) for r in range(world)]
    for i, block in enumerate(blocks):
        whole = torch.cat([per_rank[r][i] for r in range(world)])
        expect = torch.zeros(layout.nbytes, dtype=torch.uint8)
        layout.pack(block, expect)
        assert torch.equal(whole, expect)
        for r in range(world):
            assert per_rank[r][i].data_ptr() % ALIGN == 0


def test_uneven_rank_split_is_rejected():
    layout = BlockLayout.for_shapes(SHAPES)
    world = 7
    assert layout.nbytes % world
    with pytest.raises(ValueError, match="divide evenly"):
        pin_blocks(layout, [random_block(0)], PinnedHostArena(1 << 20, pin_memory=False), world=world)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _assemble_worker(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        layout = BlockLayout.for_shapes(SHAPES, multiple=ALIGN * world)
        arena = PinnedHostArena(1 << 20, pin_memory=False)
        blocks = [random_block(10 + s) for s in range(2)]
        host = pin_blocks(layout, blocks, arena, rank=rank, world=world)
        ok = True
        for i, block in enumerate(blocks):
            dest = torch.full((layout.nbytes,), 0xAB, dtype=torch.uint8)
            assemble_block(dest, host[i], rank=rank, world=world)
            views = layout.views(dest)
            for name, w in block.items():
                ok &= torch.equal(views[name].codes.view(torch.uint8), w.codes.view(torch.uint8))
                ok &= torch.equal(views[name].row_scale, w.row_scale)
        torch.save(bool(ok), f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_two_rank_assembly_rebuilds_every_block(tmp_path):
    world = 2
    mp.spawn(_assemble_worker, args=(world, _free_port(), str(tmp_path / "a")), nprocs=world)
    for r in range(world):
        assert torch.load(tmp_path / f"a.{r}"), f"rank {r} assembled a different block"
