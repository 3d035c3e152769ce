"""Block stack with weights streamed from the pinned arena: streamed == resident == direct.

The ring must only change where the weights come from, never the result: the
streamed stack (two device slots reused across blocks and steps), the
resident stack and a direct loop over separately allocated device weights
run the same kernels and must agree bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import fp8_weight, outlier_activations
from vflash_b200.native.h3_block_stack import FP8BlockStack, block_linears, block_shapes
from vflash_b200.native.h3_fp8_linear import RowFP8Execution
from vflash_b200.native.h3_parallel import FP8Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"
H, F = 256, 1024


def make_blocks(count: int, seed: int = 0, device=DEV) -> list[dict[str, FP8Weight]]:
    blocks = []
    for b in range(count):
        block = {}
        for j, (name, n, k) in enumerate(block_shapes(H, F)):
            codes, scale = fp8_weight(n, k, seed + 10 * b + j)
            block[name] = FP8Weight(codes.to(device), scale.to(device))
        blocks.append(block)
    return blocks


def direct(blocks, hidden, gate):
    execution = RowFP8Execution("w8a8")
    for block in blocks:
        hidden = block_linears(execution, block, hidden, gate)
    return hidden


def inputs(rows: int):
    hidden = outlier_activations(rows, H, 5).to(DEV).reshape(rows, 1, H)
    gate = torch.full((1, H), 1 / 32, dtype=torch.bfloat16, device=DEV)
    return hidden, gate


@pytest.mark.parametrize("count", [1, 2, 5])
def test_streamed_and_resident_equal_direct(count):
    blocks = make_blocks(count)
    hidden, gate = inputs(300)
    want = direct(blocks, hidden, gate)
    assert torch.isfinite(want.float()).all()
    streamed = FP8BlockStack(blocks, H, F, DEV, chunk_bytes=1 << 20)
    resident = FP8BlockStack(blocks, H, F, DEV, resident=True, chunk_bytes=1 << 20)
    for step in range(2):  # the second step reuses slots filled during the first
        got = streamed.forward(hidden, gate)
        assert torch.equal(got, want), f"streamed step {step} differs"
        got = resident.forward(hidden, gate)
        assert torch.equal(got, want), f"resident step {step} differs"
    torch.cuda.synchronize()
    assert streamed.ring.h2d_bytes == 2 * count * streamed.weight_bytes_per_block
    assert resident.ring.h2d_bytes == count * resident.weight_bytes_per_block


def test_host_blocks_are_pinned_and_sources_may_be_freed():
    blocks = make_blocks(3, seed=100)
    hidden, gate = inputs(64)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack(blocks, H, F, DEV, chunk_bytes=1 << 20)
    for host in stack.host_blocks:
        assert host.is_pinned() and host.data_ptr() % 256 == 0
    del blocks
    torch.cuda.empty_cache()
    assert torch.equal(stack.forward(hidden, gate), want)


def test_stack_on_a_side_stream_waits_for_its_copies():
    # Compute on a non-default stream: the ring's events order it against the copy stream.
    blocks = make_blocks(4, seed=200)
    hidden, gate = inputs(4096)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack(blocks, H, F, DEV, chunk_bytes=1 << 20)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        got = stack.forward(hidden, gate)
    torch.cuda.current_stream().wait_stream(side)
    assert torch.equal(got, want)


def test_rejects_inputs_of_the_wrong_shape():
    stack = FP8BlockStack(make_blocks(1), H, F, DEV, chunk_bytes=1 << 20)
    hidden, gate = inputs(16)
    with pytest.raises(ValueError, match="rows, 1, hidden"):
        stack.forward(hidden.reshape(16, H), gate)


def test_stack_from_block_files_equals_in_memory(tmp_path):
    safetensors_torch = pytest.importorskip("safetensors.torch")
    from vflash_b200.native.h3_weight_files import FP8_BLOCK_KEYS

    blocks = make_blocks(3, seed=300)
    paths = []
    for i, block in enumerate(blocks):
        tensors = {}
        for name, w in block.items():
            tensors[FP8_BLOCK_KEYS[name]] = w.codes.cpu().contiguous()
            tensors[FP8_BLOCK_KEYS[name] + ".row_scale"] = w.row_scale.cpu().contiguous()
        paths.append(tmp_path / f"block_{i}.safetensors")
        safetensors_torch.save_file(tensors, str(paths[-1]))
    hidden, gate = inputs(256)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack.from_files(paths, H, F, DEV, chunk_bytes=1 << 20)
    for host in stack.host_blocks:
        assert host.is_pinned()
    assert torch.equal(stack.forward(hidden, gate), want)


def test_graph_replay_of_a_resident_stack_equals_eager():
    blocks = make_blocks(3, seed=400)
    hidden, gate = inputs(512)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack(blocks, H, F, DEV, resident=True, chunk_bytes=1 << 20)
    replay = stack.capture(hidden, gate)
    assert torch.equal(replay(), want)
    # a replay reads the current input: new values give the new eager result
    hidden.copy_(inputs(512)[0] * 0.5)
    want2 = direct(blocks, hidden, gate)
    assert torch.equal(replay(), want2)
    streamed = FP8BlockStack(blocks, H, F, DEV, chunk_bytes=1 << 20)
    with pytest.raises(ValueError, match="resident"):
        streamed.capture(hidden, gate)


@pytest.mark.parametrize("count,resident_blocks", [(5, 2), (4, 3), (3, 1), (2, 2)])
def test_partially_resident_stack_equals_direct(count, resident_blocks):
    blocks = make_blocks(count, seed=500)
    hidden, gate = inputs(300)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack(blocks, H, F, DEV, resident_blocks=resident_blocks, chunk_bytes=1 << 20)
    for _ in range(3):
        assert torch.equal(stack.forward(hidden, gate), want)
    torch.cuda.synchronize()
    streamed = count - resident_blocks
    assert stack.ring.h2d_bytes == (resident_blocks + 3 * streamed) * stack.weight_bytes_per_block


@pytest.mark.parametrize("count,slots,resident_blocks", [(6, 3, 0), (5, 4, 1), (3, 4, 0)])
def test_deeper_ring_equals_direct(count, slots, resident_blocks):
    blocks = make_blocks(count, seed=600)
    hidden, gate = inputs(200)
    want = direct(blocks, hidden, gate)
    stack = FP8BlockStack(blocks, H, F, DEV, slots=slots, resident_blocks=resident_blocks, chunk_bytes=1 << 20)
    for _ in range(3):
        assert torch.equal(stack.forward(hidden, gate), want)
    assert len(stack.ring.slots) == resident_blocks + min(slots, count - resident_blocks)
