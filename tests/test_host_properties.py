"""Property checks (hypothesis) of the host-side layouts and plans that the GPU paths rely on.

Each property is what a kernel or a copy assumes: 256-byte aligned, disjoint
fields inside a packed block that splits evenly between ranks; row
partitions that cover every token once; chunk plans that cover every row once
with aligned starts; weight shards that reassemble the matrix in branch order.
"""

from __future__ import annotations

import pytest
import torch

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from vflash_b200.native.h3_host_stream import plan_chunks  # noqa: E402
from vflash_b200.native.h3_parallel import partition_rows, split_matrix  # noqa: E402
from vflash_b200.native.h3_pinned_arena import ALIGN, BlockLayout  # noqa: E402

shapes = st.lists(st.tuples(st.sampled_from(["qkv", "attention_out", "ffn_in", "ffn_out"]),
                            st.integers(1, 300), st.integers(1, 300)), min_size=1, max_size=4,
                  unique_by=lambda t: t[0])


@settings(max_examples=200, deadline=None)
@given(shapes, st.sampled_from([1, 2, 4, 8]))
def test_block_layout_fields_are_aligned_disjoint_and_split_evenly(block, world):
    layout = BlockLayout.for_shapes(block, multiple=ALIGN * world)
    assert layout.nbytes % (ALIGN * world) == 0
    end = 0
    for field in layout.fields:
        assert field.offset % ALIGN == 0 and field.offset >= end
        end = field.offset + field.nbytes
    assert end <= layout.nbytes
    assert len(layout.fields) == 2 * len(block)


@settings(max_examples=200, deadline=None)
@given(st.integers(0, 2000), st.integers(1, 8))
def test_row_partitions_cover_every_token_once(total, world):
    states = torch.arange(total, dtype=torch.float32)[:, None]
    seen, lengths = [], set()
    for rank in range(world):
        shard, valid = partition_rows(states, rank, world)
        lengths.add(shard.shape[0])
        assert not shard[valid:].any()  # padding rows are zeros
        seen.extend(shard[:valid, 0].tolist())
    assert len(lengths) == 1  # equal shards for the collective
    assert seen == list(range(total))


@settings(max_examples=200, deadline=None)
@given(st.integers(0, 100000), st.integers(1, 9000), st.sampled_from([1, 8, 16, 128]))
def test_chunk_plans_cover_every_row_once_with_aligned_starts(rows, chunk, align):
    plan = plan_chunks(rows, chunk, align)
    assert [b for b, _ in plan] == sorted(b for b, _ in plan)
    covered = 0
    for begin, end in plan:
        assert begin == covered and begin % align == 0 and end > begin
        assert end - begin <= max(align, chunk // align * align)
        covered = end
    assert covered == rows


@settings(max_examples=100, deadline=None)
@given(st.sampled_from([1, 2, 4, 8]), st.sampled_from([1, 2, 3]), st.integers(1, 4), st.integers(1, 5),
       st.sampled_from([0, 1]))
def test_weight_shards_reassemble_in_branch_order(world, parts, piece, other, axis):
    size = world * parts * piece
    shape = (size, other) if axis == 0 else (other, size)
    matrix = torch.arange(size * other, dtype=torch.float32).reshape(shape)
    shards = [split_matrix(matrix, r, world, axis=axis, parts=parts) for r in range(world)]
    # branch b of the matrix = the ranks' b-th slices, in rank order
    width = size // parts
    for b in range(parts):
        pieces = [s.narrow(axis, b * piece, piece) for s in shards]
        assert torch.equal(torch.cat(pieces, dim=axis), matrix.narrow(axis, b * width, width))
