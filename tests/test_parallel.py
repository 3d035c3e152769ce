"""Multi-rank host logic on CPU (gloo, world size 2): sharding identities
(ported from the reference's tests/test_native_parallel.py:54-89), token
sharding round trips, the tensor-parallel reduce-scatter and host-side failure
propagation.  The GEMM is the oracle's CPU restatement, injected; no GPU."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fp8 as ofp8
from vflash_b200.native import h3_parallel as par


def _fp8_weight(n, k, seed):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).numpy()
    codes, scales = ofp8.quantize_weight(w)
    return par.FP8Weight(torch.from_numpy(codes).view(torch.float8_e4m3fn), torch.from_numpy(scales))


def cpu_linear(x, weight: par.FP8Weight, bias):
    """The reference's weight-only CPU path (test-side GEMM stand-in)."""
    return ofp8.weight_only_linear(x, weight.codes, weight.row_scale, bias)


@pytest.mark.parametrize("world", [2, 4])
def test_column_shards_keep_branch_order(world):
    w = _fp8_weight(12 * world, 16, 1)
    for parts in (1, 2, 3):
        if (12 * world) % (world * parts):
            continue
        shards = [par.shard_fp8_weight(w, r, world, mode="column", parts=parts) for r in range(world)]
        codes = torch.cat([s.codes.view(torch.uint8).reshape(parts, -1, 16) for s in shards], dim=1)
        assert torch.equal(codes.reshape(-1, 16), w.codes.view(torch.uint8))
        scales = torch.cat([s.row_scale.reshape(parts, -1, 1) for s in shards], dim=1)
        assert torch.equal(scales.reshape(-1, 1), w.row_scale)


def test_row_shards_split_inputs_and_keep_row_scales():
    w = _fp8_weight(8, 32, 2)
    shards = [par.shard_fp8_weight(w, r, 4, mode="row") for r in range(4)]
    assert torch.equal(torch.cat([s.codes.view(torch.uint8) for s in shards], dim=1), w.codes.view(torch.uint8))
    assert all(s.row_scale is w.row_scale for s in shards)
    with pytest.raises(par.ParallelError):
        par.shard_fp8_weight(w, 0, 3, mode="row")  # 32 inputs do not split in three


def test_row_parallel_sum_equals_full_product():
    # partial products over input shards add up to the full product (fp64)
    w = _fp8_weight(12, 24, 3)
    x = torch.randn(5, 24, dtype=torch.float64)
    full = x @ (w.codes.to(torch.float64) * w.row_scale.double()).T
    parts = []
    for r in range(3):
        s = par.shard_fp8_weight(w, r, 3, mode="row")
        parts.append(x.chunk(3, dim=1)[r] @ (s.codes.to(torch.float64) * s.row_scale.double()).T)
    torch.testing.assert_close(sum(parts), full, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("total,world", [(7, 2), (8, 2), (10, 3), (1, 4)])
def test_partition_rows_pads_and_restores(total, world):
    x = torch.arange(total * 3, dtype=torch.float32).reshape(total, 3) + 1
    shards = [par.partition_rows(x, r, world) for r in range(world)]
    rows = par.shard_rows_count(total, world)
    assert all(s.shape == (rows, 3) for s, _ in shards)
    assert sum(valid for _, valid in shards) == total
    restored = torch.cat([s for s, _ in shards])[:total]
    assert torch.equal(restored, x)
    for s, valid in shards:
        assert (s[valid:] == 0).all()


# ---------------------------------------------------------------------------
# gloo ranks
# ---------------------------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _token_worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _fp8_weight(32, 64, 5)
        x = torch.randn(13, 64, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
        bias = torch.randn(32, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
        full = par.token_sharded_linear(x, w, cpu_linear, rank=rank, world=world, bias=bias, gather=True)
        assert torch.equal(full, cpu_linear(x, w, bias))
        # tensor parallel: column-parallel ffn_in-style pair then row-parallel projection
        w_out = _fp8_weight(16, 64, 8)
        x_cols = x.chunk(world, dim=1)[rank].contiguous()
        shard = par.shard_fp8_weight(w_out, rank, world, mode="row")
        local = par.row_parallel_linear(x_cols, shard, cpu_linear)
        expected = cpu_linear(x, w_out, None).float()
        mine, valid = par.partition_rows(expected, rank, world)
        err = ((local.float()[:valid] - mine[:valid]).norm() / mine[:valid].norm()).item()
        assert err < 1e-2, err
        torch.save({"ok": True}, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_token_sharding_and_row_parallel_reduce_scatter_on_gloo(tmp_path):
    world = 2
    mp.spawn(_token_worker, args=(world, _free_port(), str(tmp_path / "r")), nprocs=world)
    assert all(torch.load(tmp_path / f"r.{r}")["ok"] for r in range(world))


def _failure_worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    outcome = "none"
    if rank == 1:
        def failing_step():
            raise RuntimeError("injected host failure")
        try:
            par.run_guarded(failing_step, store=store, rank=rank)
        except RuntimeError:
            outcome = "raised"
    else:
        # wait for the peer's record, then refuse to launch another collective
        import time

        deadline = time.time() + 20
        while time.time() < deadline:
            try:
                par.check_peers(store)
            except par.RankFailure:
                outcome = "refused"
                break
            time.sleep(0.05)
    store.set(f"done{rank}", outcome)
    torch.save({"outcome": outcome}, f"{result_path}.{rank}")


def test_injected_failure_is_seen_by_the_peer_before_its_next_collective(tmp_path):
    world = 2
    mp.spawn(_failure_worker, args=(world, _free_port(), str(tmp_path / "f")), nprocs=world)
    assert torch.load(tmp_path / "f.1")["outcome"] == "raised"
    assert torch.load(tmp_path / "f.0")["outcome"] == "refused"


def test_host_pipeline_chunk_plan_covers_rows_in_aligned_chunks():
    from vflash_b200.native.h3_host_stream import plan_chunks

    assert plan_chunks(0, 4096) == []
    assert plan_chunks(100, 4096) == [(0, 100)]
    assert plan_chunks(32760, 4096) == [(i, min(32760, i + 4096)) for i in range(0, 32760, 4096)]
    chunks = plan_chunks(10001, 1000)  # rounded down to a multiple of 16
    assert chunks[0] == (0, 992) and chunks[-1][1] == 10001
    assert all(b - a == 992 for a, b in chunks[:-1])
    assert plan_chunks(40, 5) == [(0, 16), (16, 32), (32, 40)]
    with pytest.raises(ValueError):
        plan_chunks(10, 0)


# ---------------------------------------------------------------------------
# low-rank adapters under tensor parallelism
# (reference tests/test_native_parallel.py:54-89, float64, 2 and 4 ranks)
# ---------------------------------------------------------------------------
def _adapter(inputs, outputs, seed):
    gen = torch.Generator().manual_seed(seed)
    return par.LowRankAdapter(torch.randn(2, inputs, generator=gen, dtype=torch.float64),
                              torch.randn(outputs, 2, generator=gen, dtype=torch.float64), 0.0625)


@pytest.mark.parametrize("world", [2, 4])
def test_adapter_shards_preserve_branch_order(world):
    adapters = {"qkv": tuple(_adapter(8, 8, 10 + b) for b in range(3)),
                "attention_out": _adapter(8, 8, 20), "ffn_in": _adapter(8, 24, 21),
                "ffn_out": _adapter(12, 8, 22)}
    shards = [par.shard_block_adapters(adapters, r, world) for r in range(world)]
    for b in range(3):
        assert torch.equal(torch.cat([s["qkv"][b].up for s in shards]), adapters["qkv"][b].up)
        assert all(torch.equal(s["qkv"][b].down, adapters["qkv"][b].down) for s in shards)
    packed = torch.cat([s["ffn_in"].up.reshape(2, -1, 2) for s in shards], dim=1)
    assert torch.equal(packed.reshape(-1, 2), adapters["ffn_in"].up)
    for name in ("attention_out", "ffn_out"):
        assert torch.equal(torch.cat([s[name].down for s in shards], dim=1), adapters[name].down)
        assert all(torch.equal(s[name].up, adapters[name].up) for s in shards)
    assert par.shard_adapter(None, 0, world, mode="row") is None


def _adapter_worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inputs, outputs, total = 12, 8, 7
        gen = torch.Generator().manual_seed(18)
        weight = torch.randn(outputs, inputs, generator=gen, dtype=torch.float64)
        adapter = _adapter(inputs, outputs, 19)
        states = torch.arange(inputs * total, dtype=torch.float64).reshape(total, inputs) / 32
        x_cols = states.chunk(world, dim=1)[rank].contiguous()
        w_shard = par.split_matrix(weight, rank, world, axis=1)
        a_shard = par.shard_adapter(adapter, rank, world, mode="row")
        base, update = par.row_parallel_adapter_linear(
            x_cols, w_shard, lambda x, w, _b: x @ w.T, a_shard)
        actual = base + update * adapter.scaling
        expected = states @ weight.T + ((states @ adapter.down.T) @ adapter.up.T) * adapter.scaling
        mine, valid = par.partition_rows(expected, rank, world)
        torch.testing.assert_close(actual[:valid], mine[:valid], rtol=1e-12, atol=1e-12)
        torch.save({"ok": True}, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_row_parallel_adapter_reduces_down_before_up_on_gloo(tmp_path):
    world = 2
    mp.spawn(_adapter_worker, args=(world, _free_port(), str(tmp_path / "a")), nprocs=world)
    assert all(torch.load(tmp_path / f"a.{r}")["ok"] for r in range(world))


def test_cpu_set_for_bus_id_decodes_nvml_affinity_masks():
    from vflash_b200.native.h3_host_stream import cpu_set_for_bus_id

    calls = []

    class FakeNVML:
        def nvmlInit(self):
            calls.append("init")

        def nvmlShutdown(self):
            calls.append("shutdown")

        def nvmlDeviceGetHandleByPciBusId(self, bus_id):
            calls.append(bus_id)
            return "handle"

        def nvmlDeviceGetCpuAffinity(self, handle, words):
            assert handle == "handle" and words >= 1
            return [0b1011, 1 << 3]

    assert cpu_set_for_bus_id("00000000:1B:00.0", FakeNVML()) == {0, 1, 3, 67}
    assert calls == ["init", "00000000:1B:00.0", "shutdown"]

    class Failing(FakeNVML):
        def nvmlDeviceGetHandleByPciBusId(self, bus_id):
            raise RuntimeError("no such device")

    assert cpu_set_for_bus_id("x", Failing()) == set()
