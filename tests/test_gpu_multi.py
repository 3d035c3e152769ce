"""Two-GPU token sharding and tensor parallelism over NCCL with the native kernels.

Token-sharded rows must equal the single-GPU result bit for bit (each output
row depends only on its own input row); the row-parallel (reduce-scatter)
variant must agree with the unsharded linear within bf16 tolerance
(rel-L2 <= 1e-2); the block stack whose weights each rank pins half of and
all-gathers must equal a direct loop over device weights bit for bit.  Needs two SM100 GPUs; skipped otherwise.  The process
group uses a short timeout, and NVLS is off (NCCL_NVLS_ENABLE=0).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from oracle import fp8 as ofp8
    from vflash_b200.native import h3_parallel as par
    from vflash_b200.native.h3_fp8_linear import RowFP8Execution

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        def weight(n, k, seed):
            w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).numpy()
            codes, scales = ofp8.quantize_weight(w)
            return par.FP8Weight(torch.from_numpy(codes).view(torch.float8_e4m3fn).to(device),
                                 torch.from_numpy(scales).to(device))

        execution = RowFP8Execution("w8a8")

        def linear(x, w, bias):
            return execution.linear(x, w.codes, w.row_scale, bias)

        m, k, n = 1001, 1024, 768
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(device)
        w = weight(n, k, 2)
        bias = torch.randn(n, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(device)
        full = par.token_sharded_linear(x, w, linear, rank=rank, world=world, bias=bias, gather=True)
        single = linear(x, w, bias)
        token_exact = bool(torch.equal(full, single))

        w_out = weight(512, k, 4)
        x_cols = x.chunk(world, dim=1)[rank].contiguous()
        shard = par.shard_fp8_weight(w_out, rank, world, mode="row")
        local = par.row_parallel_fp8_linear(x_cols, shard)
        expected = linear(x, w_out, None).float()
        mine, valid = par.partition_rows(expected, rank, world)
        rel = ((local.float()[:valid] - mine[:valid]).norm() / mine[:valid].norm()).item()
        # the row-split quantisation with all-reduced row maxima equals the unsplit one
        from vflash_b200.kernels import quantize_fp8_rows, row_absmax

        amax = row_absmax(x_cols)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        codes, scales = quantize_fp8_rows(x_cols, amax=amax)
        full_codes, full_scales = quantize_fp8_rows(x)
        cols = k // world
        codes_exact = bool(torch.equal(codes.view(torch.uint8),
                                       full_codes.view(torch.uint8)[:, rank * cols:(rank + 1) * cols])
                           and torch.equal(scales, full_scales))
        # block stack: each rank pins half of every block, the all-gather over
        # NVLink rebuilds it, and the rank's token shard matches a direct loop
        from vflash_b200.native.h3_block_stack import FP8BlockStack, block_linears, block_shapes

        hid, ffn = 256, 1024
        blocks = [{name: weight(nn, kk, 50 + 10 * b + j)
                   for j, (name, nn, kk) in enumerate(block_shapes(hid, ffn))} for b in range(3)]
        tokens = torch.randn(333, hid, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(device)
        shard, _valid = par.partition_rows(tokens, rank, world)
        shard = shard.reshape(-1, 1, hid)
        gate = torch.full((1, hid), 1 / 32, dtype=torch.bfloat16, device=device)
        want = shard
        for block in blocks:
            want = block_linears(execution, block, want, gate)
        stack = FP8BlockStack(blocks, hid, ffn, device, group=dist.group.WORLD, chunk_bytes=1 << 20)
        stack_exact = all(bool(torch.equal(stack.forward(shard, gate), want)) for _ in range(2))
        torch.cuda.synchronize()
        torch.save({"token_exact": token_exact, "tp_rel": rel, "codes_exact": codes_exact,
                    "stack_exact": stack_exact}, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_token_sharding_and_tensor_parallel(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path / "g")), nprocs=world)
    for r in range(world):
        res = torch.load(tmp_path / f"g.{r}")
        assert res["token_exact"], f"rank {r}: token-sharded rows differ from the single-GPU result"
        assert res["codes_exact"], f"rank {r}: split-row codes differ from the unsplit quantisation"
        assert res["tp_rel"] <= 1e-2, res
        assert res["stack_exact"], f"rank {r}: the streamed block stack differs from a direct loop"
