"""The linear set of a stack of H3 DiT blocks, with weights streamed from pinned host memory.

One block's quantised linears are those of the reference's block forward
(``forward_prevalidated``, src/vflash/native/h3_native_denoiser.py:492-576):
the merged QKV projection ``[3H, H]`` (541), the attention output ``[H, H]``
with its gated residual ``residual + gate * projected`` (551-556, 366-367),
the FFN input ``[F, H]`` (568) and the FFN output ``[H, F]`` with its gated
residual (570-575).  The stack measured here uses the GELU-tanh FFN of the
fused-FFN benchmark (``F = 4H``); the packed SwiGLU input of 369-373 is the
``swiglu`` activation of ``RowFP8Execution.ffn``.  Attention and the
modulation/normalisation steps are not part of this path: ``block_linears``
feeds the V plane to the attention output projection in attention's place,
so the four GEMMs run at their real shapes on real data, and the gate is a
caller-supplied ``[1, H]`` row, fused into the GEMM epilogues.

Weights live in a ``PinnedHostArena`` and reach the GPU through an
``FP8BlockRing`` (two device slots, side copy stream), or stay resident.
Tokens are sharded across ranks by the caller (``h3_parallel.partition_rows``);
weights are replicated, so the linears need no collective.
"""

from __future__ import annotations

from collections.abc import Iterable

import torch

from .h3_fp8_linear import RowFP8Execution
from .h3_parallel import FP8Weight
from .h3_pinned_arena import ALIGN, BlockLayout, FP8BlockRing, PinnedHostArena, pin_blocks


def block_shapes(hidden: int, ffn: int) -> tuple[tuple[str, int, int], ...]:
    """(name, N, K) of one block's four linears, in execution order."""
    return (("qkv", 3 * hidden, hidden), ("attention_out", hidden, hidden),
            ("ffn_in", ffn, hidden), ("ffn_out", hidden, ffn))


def block_flops(rows: int, hidden: int, ffn: int) -> int:
    return sum(2 * rows * n * k for _, n, k in block_shapes(hidden, ffn))


def block_linears(execution: RowFP8Execution, weights: dict[str, FP8Weight], hidden: torch.Tensor,
                  gate: torch.Tensor) -> torch.Tensor:
    """One block's linears on ``hidden`` ``[rows, 1, H]`` (bf16) with gate ``[1, H]``.

    qkv -> (V as attention output) -> attention_out with gated residual ->
    FFN (GELU-tanh up, per-token requant, down with gated residual).
    """
    qkv = weights["qkv"]
    _q, _k, v = execution.qkv_linear(hidden, qkv.codes, qkv.row_scale)
    out = weights["attention_out"]
    hidden = execution.gate_residual_linear(v, out.codes, out.row_scale, hidden, gate)
    up, down = weights["ffn_in"], weights["ffn_out"]
    return execution.ffn(hidden, up.codes, up.row_scale, down.codes, down.row_scale,
                         activation="gelu_tanh", residual=hidden, gate=gate)


class FP8BlockStack:
    """A stack of FP8 block linear sets whose weights stream from a pinned host arena.

    ``blocks`` yields one ``{name: FP8Weight}`` dict per block (any device);
    each is packed, this rank's byte range is pinned, and the source may be
    freed afterwards.  ``forward(hidden, gate)`` runs every block on the
    current stream.
    """

    def __init__(self, blocks: Iterable[dict[str, FP8Weight]], hidden: int, ffn: int, device, *,
                 group=None, resident: bool = False, resident_blocks: int = 0, slots: int = 2,
                 chunk_bytes: int = 2 * 1024**3, execution: RowFP8Execution | None = None) -> None:
        import torch.distributed as dist

        world = dist.get_world_size(group) if group is not None else 1
        rank = dist.get_rank(group) if group is not None else 0
        self.hidden = hidden
        self.ffn = ffn
        self.layout = BlockLayout.for_shapes(block_shapes(hidden, ffn), multiple=ALIGN * world)
        chunk = self.layout.nbytes // world
        slab = max(chunk_bytes, 1 << (chunk - 1).bit_length())
        self.arena = PinnedHostArena(slab)
        self.host_blocks = pin_blocks(self.layout, blocks, self.arena, rank=rank, world=world)
        self.arena.close()  # the views keep their slabs; no further allocations
        self.ring = FP8BlockRing(self.layout, self.host_blocks, device, group=group, resident=resident,
                                 resident_blocks=resident_blocks, slots=slots)
        self.execution = execution or RowFP8Execution("w8a8")

    @classmethod
    def from_files(cls, paths, hidden: int, ffn: int, device, *, group=None, resident: bool = False,
                   chunk_bytes: int = 2 * 1024**3, execution: RowFP8Execution | None = None) -> FP8BlockStack:
        """A stack whose blocks are read from the reference's per-block safetensors files.

        Each rank reads only its share of every block, straight into pinned
        memory (``h3_weight_files.pin_fp8_block_files``).
        """
        import torch.distributed as dist

        from .h3_weight_files import pin_fp8_block_files

        self = cls.__new__(cls)
        world = dist.get_world_size(group) if group is not None else 1
        rank = dist.get_rank(group) if group is not None else 0
        self.hidden, self.ffn = hidden, ffn
        self.layout = BlockLayout.for_shapes(block_shapes(hidden, ffn), multiple=ALIGN * world)
        chunk = self.layout.nbytes // world
        self.arena = PinnedHostArena(max(chunk_bytes, 1 << (chunk - 1).bit_length()))
        self.host_blocks = pin_fp8_block_files(paths, self.layout, self.arena, rank=rank, world=world)
        self.arena.close()
        self.ring = FP8BlockRing(self.layout, self.host_blocks, device, group=group, resident=resident)
        self.execution = execution or RowFP8Execution("w8a8")
        return self

    @property
    def weight_bytes_per_block(self) -> int:
        return self.layout.nbytes

    def capture(self, hidden: torch.Tensor, gate: torch.Tensor):
        """CUDA graph of ``forward`` over a resident stack; returns ``replay() -> output``.

        The stack runs once eagerly first (loading every block and setting up
        the kernels), then the block loop is captured; a replay reads the
        current contents of ``hidden`` and ``gate`` and rewrites the returned
        output tensor.  One graph launch replaces the per-block host work of
        issuing 8 kernels per block.
        """
        if not self.ring.resident:
            raise ValueError("graph capture needs a resident stack")
        self.forward(hidden, gate)
        torch.cuda.synchronize(self.ring.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.ring.run(hidden, lambda w, h: block_linears(self.execution, w, h, gate), wait_ready=False)

        def replay() -> torch.Tensor:
            graph.replay()
            return out

        replay.graph = graph
        return replay

    def forward(self, hidden: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        if hidden.ndim != 3 or hidden.shape[1] != 1 or hidden.shape[2] != self.hidden:
            raise ValueError("block stack input must be bf16 [rows, 1, hidden]")
        return self.ring.run(hidden, lambda w, h: block_linears(self.execution, w, h, gate))
