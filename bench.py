"""Benchmark of the B200 FP8 linear hot path (one JSON line on rank 0).

Workload (N=1 and per rank at N>1): benchmark config 1, the merged QKV FP8
projection of one H3-style block — X bf16 [32760, 4096] (N(0,1) with 0.1 %
x20 outliers), W_qkv e4m3 [12288, 4096] (N(0,0.02), per-output-row scales),
bias bf16 [12288], output Q, K, V bf16 [32760, 32, 128].  One step = the
per-token e4m3 quantisation of X plus the tcgen05 GEMM whose epilogue applies
row x column scales and bias and writes the three planes.

Timing: W warm-up steps, then K steps, each bracketed by CUDA events on the
launching stream with a 256 MB buffer written between steps to flush L2
(outside the events); a barrier + synchronize brackets the whole timed
region; multi-GPU value uses the max over ranks.  Tokens are independent, so
at N GPUs every rank runs its own full workload with replicated weights
(weak scaling, no collective on the data path).

``e2e`` runs the same step through the public API with the input in pinned
host memory and Q, K, V copied back to pinned host memory inside the timed
region: ``HostRowPipeline`` around ``RowFP8Execution("w8a8").qkv_linear``
(row chunks whose copies in, compute and copies out overlap); the
``unpipelined`` entry is one whole-tensor copy in, the linear, one copy out.

``stack_c4`` is benchmark config 4 on every rank: 48 blocks of FP8 linears
over M=65520 tokens sharded across the ranks, weights streamed from the
pinned host arena through the two-slot ring (and, for comparison, resident),
milliseconds per denoising step as the max over ranks.

``other_configs`` (benchmark configs 0, 2 and 3, the fused variants and
the same-box library bars, with their own clock record) and the CPU
baseline run at N=1 only.

``--impl reference`` times the reference's own CPU path for this layer
(``RowFP8Execution("weight-only").linear``: dequantise to bf16, then
``F.linear`` on the host cores) through the oracle's restatement, over the
same rows (``--reference-rows`` to sample fewer).
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M, K, N_QKV, HEADS = 32760, 4096, 12288, 32
METRIC = "FP8/NVFP4 linear TFLOP/s/GPU & % of tcgen05 peak; DiT-block linear ms at 1-8 GPU"
WORKLOAD = "c1 merged QKV FP8: X bf16 [32760,4096] -> e4m3 per-token, W e4m3 [12288,4096], bias, Q/K/V [32760,32,128]"
NOMINAL_FP8_TFLOPS = 4500.0
L2_FLUSH_BYTES = 256 << 20


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


def profile_traffic() -> float | None:
    """Per-launch DRAM bytes of the GEMM from the committed ncu summary, if present."""
    path = ROOT / "profiles" / "fp8_gemm_qkv_c1.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi around the timed region.

    nvidia-smi needs about a second to start, so sampling starts before the
    warm-up; ``mark_start``/``mark_end`` bracket the timed region and only
    samples stamped inside it are summarised (the nearest sample when the
    region is shorter than the sampling period).
    """

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self) -> dict:
        import datetime

        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        samples = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                stamp = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((stamp, float(parts[2]), float(parts[3]), float(parts[4]),
                                [n for n, f in zip(names, parts[6:10]) if f.lower() == "active"]))
            except ValueError:
                continue
        if not samples or self.t0 is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        inside = [s for s in samples if self.t0 <= s[0] <= self.t1]
        if not inside:
            mid = 0.5 * (self.t0 + self.t1)
            inside = [min(samples, key=lambda s: abs(s[0] - mid))]
        reasons = sorted({r for s in inside for r in s[4]})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": inside[0][2],
                "power_w_max": max(s[3] for s in inside), "reasons": reasons,
                "samples": len(inside)}


def synthetic_workload(device: torch.device, rank: int, M: int):
    """Seeded inputs of benchmark config 1 (seeds X 1001, W 2010, bias 3001; offset by rank)."""
    gen = torch.Generator().manual_seed(1001 + 97 * rank)
    x = torch.randn(M, K, generator=gen)
    count = round(0.001 * M * K)
    idx = torch.randperm(M * K, generator=torch.Generator().manual_seed(1002 + 97 * rank))[:count]
    x.view(-1)[idx] *= 20
    x = x.to(torch.bfloat16)
    w = (torch.randn(N_QKV, K, generator=torch.Generator().manual_seed(2010)) * 0.02)
    w = w.to(torch.bfloat16).to(device)
    # per-output-row e4m3 weight quantisation on the device with the library's
    # own quantiser (pad_to=1): identical to the activation formula per row
    from vflash_b200.kernels import quantize_fp8_rows

    w_codes, w_scales = quantize_fp8_rows(w, pad_to=1)
    bias = (torch.randn(N_QKV, generator=torch.Generator().manual_seed(3001)) * 0.01).to(torch.bfloat16)
    return x, w_codes, w_scales, bias.to(device)


def verify_step(x, M, w_codes, w_scales, bias) -> dict:
    """Checks one more step of the timed workload against the reference's GPU composition.

    The reference's w8a8 linear (src/vflash/native/h3_fp8_linear.py:18-31,
    92-121) is its quantiser expression evaluated by torch, rowwise
    ``torch._scaled_mm`` and a bf16 bias add.  The activation codes and scales
    must equal that expression bit for bit (the divisor is a device tensor:
    torch turns a division by a Python scalar into a reciprocal multiply) and
    the Q/K/V planes must be within rel-L2 1e-2 of its output.
    """
    from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows

    codes, scales = quantize_fp8_rows(x)
    planes = fp8_gemm(codes, scales, M, w_codes, w_scales, Epilogue(bias=bias, planes=3))
    floats = x.float()
    maxima = floats.abs().amax(dim=1, keepdim=True)
    want_scales = torch.where(maxima > 0, (maxima / torch.full_like(maxima, 448.0)).clamp_min(
        torch.finfo(torch.float32).tiny), torch.ones_like(maxima))
    want_codes = (floats / want_scales).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    del floats
    codes_equal = bool(torch.equal(codes[:M].view(torch.uint8), want_codes.view(torch.uint8))
                       and torch.equal(scales[:M].reshape(-1), want_scales.reshape(-1)))
    ref = torch._scaled_mm(want_codes, w_codes.t(), scale_a=want_scales, scale_b=w_scales.reshape(1, -1),
                           out_dtype=torch.bfloat16)
    ref = (ref[0] if isinstance(ref, tuple) else ref) + bias
    got = torch.cat([p for p in planes], dim=1)
    rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
    del ref, got, planes
    return {"codes_and_scales_bit_exact": codes_equal, "rel_l2_vs_scaled_mm_chain": float(f"{rel:.3g}"),
            "bar": 1e-2, "ok": codes_equal and rel <= 1e-2}


def run_e2e(args, M, x_host, w_codes, w_scales, bias, device, stream, barrier):
    """Same step through the public API, pinned host buffers in and out.

    Returns (ms, steps) for the row-chunked pipeline (``HostRowPipeline``:
    host->device copy, compute and device->host copy of successive row chunks
    overlap on three streams) and for one whole-tensor copy -> qkv_linear ->
    copy back.
    """
    from vflash_b200.native.h3_fp8_linear import RowFP8Execution
    from vflash_b200.native.h3_host_stream import HostRowPipeline

    execution = RowFP8Execution("w8a8", activation_quantizer="triton")
    x_pinned = x_host.pin_memory()
    x_dev = torch.empty(x_host.shape, dtype=x_host.dtype, device=device)
    head_dim = K // HEADS
    outs_host = [torch.empty((M, HEADS, head_dim), dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    pipeline = HostRowPipeline(lambda xd: execution.qkv_linear(xd, w_codes, w_scales, bias), device,
                               chunk_rows=args.e2e_chunk_rows)

    def whole_step():
        x_dev.copy_(x_pinned, non_blocking=True)
        q, k, v = execution.qkv_linear(x_dev, w_codes, w_scales, bias)
        for host, plane in zip(outs_host, (q, k, v)):
            host.copy_(plane.view(M, HEADS, head_dim), non_blocking=True)

    def pipelined_step():
        pipeline(x_pinned, outs_host)

    steps = max(3, min(args.steps, 10))
    results = []
    for fn in (pipelined_step, whole_step):
        for _ in range(args.warmup):
            fn()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(steps):
            fn()
        s1.record(stream)
        barrier()
        results.append((s0.elapsed_time(s1), steps))
    return results


def run_gpu(args) -> None:
    from vflash_b200 import _lib
    from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    distributed = world > 1
    if distributed:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # host buffers (pinned inputs/outputs of e2e, the weight arena) on this GPU's own socket
    from vflash_b200.native.h3_host_stream import bind_host_to_device

    all_cpus = os.sched_getaffinity(0)
    host_cpus = set() if args.no_numa_bind else bind_host_to_device(device)

    def barrier():
        if distributed:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(value: float) -> float:
        if not distributed:
            return value
        t = torch.tensor([value], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.item()

    M = args.rows
    flop_per_step = 2.0 * M * N_QKV * K
    x_host, w_codes, w_scales, bias = synthetic_workload(device, rank, M)
    x = x_host.to(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def step(ev):
        ev[0].record(stream)
        codes, scales = quantize_fp8_rows(x)
        ev[1].record(stream)
        fp8_gemm(codes, scales, M, w_codes, w_scales, Epilogue(bias=bias, planes=3))
        ev[2].record(stream)

    clocks = ClockSampler(local_rank).start()
    for _ in range(args.warmup):
        step([torch.cuda.Event(enable_timing=True) for _ in range(3)])
    barrier()
    time.sleep(1.0)  # nvidia-smi is sampling by now
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier()
    clocks.mark_start()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(float(i))
        step(events[i])
    barrier()
    wall = time.perf_counter() - wall0
    clocks.mark_end()
    clocks.stop()
    step_ms = [e[0].elapsed_time(e[2]) for e in events]
    quant_ms = [e[0].elapsed_time(e[1]) for e in events]
    gemm_ms = [e[1].elapsed_time(e[2]) for e in events]
    total_ms = max_over_ranks(sum(step_ms))
    status = _lib.device_status(clear=True)
    verified = verify_step(x, M, w_codes, w_scales, bias)

    # The short per-config measurements and the library bars run next, while
    # the GPU is in the same state as for the headline (the config 4 stack
    # below runs dense GEMMs for tens of seconds, after which the same kernels
    # measure up to ~25 % slower under the power cap); they carry their own
    # clock record.
    # They are single-GPU measurements: with several ranks they are skipped, so
    # that no rank waits at a collective while rank 0 runs them alone.
    library = same_shape = None
    other = None
    if world == 1 and not (args.no_library_probe and args.no_other_configs):
        phase_clocks = ClockSampler(local_rank).start()
        time.sleep(0.5)
        phase_clocks.mark_start()
        if not args.no_other_configs:
            other = other_configs(device, flush, stream,
                                  0.0 if args.no_cpu_baseline else min(args.cpu_seconds, 10.0))
        if not args.no_library_probe:
            library = library_fp8_probe(device)
            same_shape = library_same_shape(device, flush, stream)
        phase_clocks.mark_end()
        phase_clocks.stop()
        if other is not None:
            other["clocks"] = phase_clocks.summary()
    barrier()

    e2e_ms, e2e_steps, whole_ms, whole_steps = float("nan"), 0, float("nan"), 0
    if not args.no_e2e:
        (e2e_ms, e2e_steps), (whole_ms, whole_steps) = run_e2e(args, M, x_host, w_codes, w_scales, bias,
                                                               device, stream, barrier)
        e2e_ms = max_over_ranks(e2e_ms)
        whole_ms = max_over_ranks(whole_ms)

    stack = None
    if not args.no_stack:
        stack = stack_config(args, device, rank, world, barrier, max_over_ranks)
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline may use every host thread
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(x_host, w_codes.cpu(), w_scales.cpu(), bias.cpu(), args.cpu_seconds)

    if distributed:
        barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    peaks = measured_peaks()
    if "bf16_tflops" in peaks:
        peak = 2.0 * float(peaks["bf16_tflops"])
        peak_src = "2 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops) = dense fp8 equivalent"
    else:
        peak = 2.0 * 1590.0
        peak_src = "2 x fallback bf16 1.59 PFLOP/s"
    gemm_mean = statistics.mean(gemm_ms)
    achieved = flop_per_step / (gemm_mean * 1e-3) / 1e12
    value = world * args.steps * flop_per_step / (total_ms * 1e-3) / 1e12
    quant_mean = statistics.mean(quant_ms)
    quant_bytes = M * K * 2 + M * K + (M + 15) // 16 * 16 * 4
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.mean(step_ms), 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 acc -> bf16",
        "data": "synthetic (seeded N(0,1) activations with 0.1% x20 outliers; N(0,0.02) weights, per-row e4m3)",
        "config": {"workload": WORKLOAD if M == 32760 else f"profiling case: c1 with M={M}",
                   "M": M, "N": N_QKV, "K": K, "bias": True,
                   "l2": "flushed between steps (256 MB buffer written outside the timed events)",
                   "parallelism": f"token-sharded dp{world} (weights replicated)",
                   "step": "fp8 quantiser + tcgen05 GEMM with QKV-plane epilogue"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": profile_traffic(),
                     "kernel": "fp8_gemm_kernel<STORE> (QKV planes)", "peak_source": peak_src,
                     "frac_of_nominal_4500": round(achieved / NOMINAL_FP8_TFLOPS, 4),
                     "gemm_ms": round(gemm_mean, 4)},
        "quantiser": {"ms": round(quant_mean, 4),
                      "gb_per_s": round(quant_bytes / (quant_mean * 1e-3) / 1e9, 1),
                      "frac_of_measured_hbm": round(quant_bytes / (quant_mean * 1e-3) / 1e9 / hbm, 4)},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
        "wall_s_timed_region": round(wall, 3),
        "device_status": status,
        "verified": verified,
        "host_cpus_bound": len(host_cpus),
    }
    if e2e_steps:
        line["e2e"] = {"value": round(world * e2e_steps * flop_per_step / (e2e_ms * 1e-3) / 1e12, 2),
                       "unit": "TFLOP/s", "h2d_bytes_per_step": M * K * 2,
                       "d2h_bytes_per_step": M * N_QKV * 2,
                       "api": "HostRowPipeline(RowFP8Execution('w8a8').qkv_linear), pinned host in/out, "
                              f"{args.e2e_chunk_rows}-row chunks overlapping H2D, compute and D2H",
                       "ms_per_step": round(e2e_ms / e2e_steps, 3),
                       "unpipelined": {
                           "value": round(world * whole_steps * flop_per_step / (whole_ms * 1e-3) / 1e12, 2),
                           "ms_per_step": round(whole_ms / whole_steps, 3),
                           "api": "one copy in, RowFP8Execution('w8a8').qkv_linear, one copy out"}}
    if stack is not None:
        line["stack_c4"] = stack
    if library is not None:
        line["library_fp8_tflops"] = library
    if same_shape is not None:
        line["library_same_shape"] = same_shape
    if other is not None:
        line["other_configs"] = other
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def _timed(fn, flush, stream, reps: int = 50, warmup: int = 10) -> list[float]:
    """Per-call milliseconds of ``fn`` (CUDA events, L2 flushed before each call)."""
    for _ in range(warmup):
        fn()
    times = []
    for i in range(reps):
        flush.fill_(float(i))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def _timed_split(first, second, flush, stream, reps: int = 50, warmup: int = 10):
    """Per-call milliseconds of ``second(first())`` and of its ``second`` part alone.

    One event pair brackets each call and a third sits between the two parts,
    so both lists come from the same calls (L2 flushed before each).
    """
    for _ in range(warmup):
        second(first())
    marks = []
    for i in range(reps):
        flush.fill_(float(i))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        result = first()
        ev[1].record(stream)
        second(result)
        ev[2].record(stream)
        marks.append(ev)
    torch.cuda.synchronize()
    return [e[0].elapsed_time(e[2]) for e in marks], [e[1].elapsed_time(e[2]) for e in marks]


def _chain_output(x, up, ups, down, downs, m):
    """Config 2's FFN as four separate launches (quantiser, up GEMM + GELU, requantiser, down GEMM + residual)."""
    from vflash_b200 import _lib
    from vflash_b200.kernels import Epilogue, fp8_gemm, quantize_fp8_rows

    c, s = quantize_fp8_rows(x)
    mid = fp8_gemm(c, s, m, up, ups, Epilogue(kind=_lib.EPI_GELU_TANH))
    mc, ms_ = quantize_fp8_rows(mid)
    return fp8_gemm(mc, ms_, m, down, downs, Epilogue(kind=_lib.EPI_RESIDUAL, residual=x))


def nvfp4_cpu_baseline(ac, asf, wp, wsc, alpha, seconds: float) -> dict:
    """NVFP4 has no reference CPU path: the oracle's dequantise-then-fp32-matmul on a row sample."""
    from oracle.nvfp4 import dequant_matmul_f32

    rows, k = 1024, ac.shape[1] * 2
    kt = -(-(k // 16) // 4)
    a = ac[:rows].cpu().numpy()
    a_sf = asf.reshape(-1)[: rows // 128 * kt * 512].cpu().numpy()
    w = wp.cpu().numpy()
    w_sf = wsc.reshape(-1).cpu().numpy()
    al = float(alpha)
    reps, elapsed = 0, 0.0
    while elapsed < seconds or reps < 1:
        t0 = time.perf_counter()
        dequant_matmul_f32(a, a_sf, w, w_sf, al)
        elapsed += time.perf_counter() - t0
        reps += 1
    flop = 2.0 * rows * w.shape[0] * k * reps
    return {"value": round(flop / elapsed / 1e12, 4), "unit": "TFLOP/s", "cores": cpu_threads(),
            "kind": "port", "sample": f"{reps} x oracle dequantise (e2m1 x e4m3 block scales) + fp32 "
                                      f"matmul on {rows} rows, N={w.shape[0]}, K={k}: {elapsed:.1f} s "
                                      "(the reference has no NVFP4 CPU path)"}


def other_configs(device, flush, stream, cpu_seconds: float = 0.0) -> dict:
    """benchmark configs 0, 2 and 3 on one GPU: seeded synthetic inputs, 10 warm-up calls, median of 50
    timed calls with L2 flushed before each."""
    from vflash_b200 import _lib
    from vflash_b200.kernels import Epilogue, fp8_gemm, nvfp4_gemm, nvfp4_quantize, quantize_fp8_rows

    peaks = measured_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    fp4_peak = 2.0 * fp8_peak
    out: dict = {}

    def seeded(rows, cols, seed, std=1.0, outliers=False):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(rows, cols, generator=gen) * std
        if outliers:
            count = round(0.001 * rows * cols)
            idx = torch.randperm(rows * cols, generator=torch.Generator().manual_seed(seed + 1))[:count]
            x.view(-1)[idx] *= 20
        return x.to(torch.bfloat16).to(device)

    def summary(ms, flop, peak, extra=None):
        med = statistics.median(ms)
        d = {"ms": round(med, 4), "tflops": round(flop / (med * 1e-3) / 1e12, 1),
             "frac_of_peak": round(flop / (med * 1e-3) / 1e12 / peak, 4)}
        d.update(extra or {})
        return d

    # c0: single FP8 linear 4096^3 with bias
    x = seeded(4096, 4096, 1000, outliers=True)
    wc, ws = quantize_fp8_rows(seeded(4096, 4096, 2000, std=0.02), pad_to=1)
    b = seeded(1, 4096, 3000, std=0.01).view(-1)

    def c0():
        c, s = quantize_fp8_rows(x)
        fp8_gemm(c, s, 4096, wc, ws, Epilogue(bias=b))

    out["c0_fp8_linear_4096"] = summary(_timed(c0, flush, stream), 2.0 * 4096**3, fp8_peak,
                                        {"step": "quantiser + GEMM + bias"})
    del x, wc, ws, b

    # c2: FFN, GELU-tanh, per-token requant of the intermediate, residual:
    # vfb_fp8_ffn (quantiser, up GEMM + GELU, requantiser, down GEMM + residual;
    # per-launch times from the same chain issued step by step) and, for
    # comparison, vfb_fp8_ffn_one_kernel (the three steps after the quantiser
    # in one persistent launch)
    from vflash_b200.kernels import fp8_ffn

    m, h, f = 32760, 4096, 16384
    x = seeded(m, h, 1002)
    up, ups = quantize_fp8_rows(seeded(f, h, 2020, std=0.02), pad_to=1)
    down, downs = quantize_fp8_rows(seeded(h, f, 2021, std=0.02), pad_to=1)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    ffn_flop = 2.0 * m * f * h * 2

    def c2_ffn():
        fp8_ffn(x, up, ups, down, downs, activation=_lib.EPI_GELU_TANH, residual=x)

    def c2_one_kernel():
        fp8_ffn(x, up, ups, down, downs, activation=_lib.EPI_GELU_TANH, residual=x, one_kernel=True)

    def c2_chain():
        ev[0].record(stream)
        c, s = quantize_fp8_rows(x)
        ev[1].record(stream)
        mid = fp8_gemm(c, s, m, up, ups, Epilogue(kind=_lib.EPI_GELU_TANH))
        ev[2].record(stream)
        mc, ms_ = quantize_fp8_rows(mid)
        ev[3].record(stream)
        fp8_gemm(mc, ms_, m, down, downs, Epilogue(kind=_lib.EPI_RESIDUAL, residual=x))
        ev[4].record(stream)

    ffn_ms = _timed(c2_ffn, flush, stream)
    one_kernel_ms = statistics.median(_timed(c2_one_kernel, flush, stream))
    _timed(c2_chain, flush, stream, reps=10, warmup=3)
    parts = [ev[i].elapsed_time(ev[i + 1]) for i in range(4)]
    chain = _chain_output(x, up, ups, down, downs, m)
    same = bool(torch.equal(fp8_ffn(x, up, ups, down, downs, activation=_lib.EPI_GELU_TANH, residual=x), chain)
                and torch.equal(fp8_ffn(x, up, ups, down, downs, activation=_lib.EPI_GELU_TANH, residual=x,
                                        one_kernel=True), chain))
    del chain
    out["c2_fp8_ffn_gelu"] = summary(
        ffn_ms, ffn_flop, fp8_peak,
        {"step": "vfb_fp8_ffn: quant X, up GEMM + GELU-tanh epilogue, per-token requant of the bf16 "
                 "intermediate, down GEMM + residual epilogue (one C call, four launches)",
         "last_step_ms": {"quant_x": round(parts[0], 4), "up_gemm_gelu": round(parts[1], 4),
                          "requant_mid": round(parts[2], 4), "down_gemm_residual": round(parts[3], 4)},
         "one_kernel_ms": round(one_kernel_ms, 4),
         "one_kernel_tflops": round(ffn_flop / (one_kernel_ms * 1e-3) / 1e12, 1),
         "equal_bits": same})
    del up, ups

    # c2 SwiGLU variant (the reference model's packed FFN input [2F, H]) through
    # the public fused entry point RowFP8Execution.ffn
    from vflash_b200.native.h3_fp8_linear import RowFP8Execution

    packed, packeds = quantize_fp8_rows(seeded(2 * f, h, 2022, std=0.02), pad_to=1)
    execution = RowFP8Execution("w8a8")

    def c2_swiglu():
        execution.ffn(x, packed, packeds, down, downs, activation="swiglu", residual=x)

    ms = _timed(c2_swiglu, flush, stream)
    out["c2_fp8_ffn_swiglu"] = summary(
        ms, 2.0 * m * (2 * f) * h + 2.0 * m * f * h, fp8_peak,
        {"step": "RowFP8Execution.ffn(activation='swiglu'): quant X, packed up GEMM [2F,H] with "
                 "value * bf16(silu(gate)), requant, down GEMM + residual"})
    del x, packed, packeds, down, downs

    # c3: NVFP4 linear, M = 32760, K = 4096, N in {4096, 16384}
    x = seeded(32760, 4096, 1003)
    gsf_x = (448.0 * 6.0 / x.float().abs().max()).reshape(())
    for n in (4096, 16384):
        w = seeded(n, 4096, 2030 + n, std=0.02)
        gsf_w = (448.0 * 6.0 / w.float().abs().max()).reshape(())
        wp, wsc = nvfp4_quantize(w, gsf_w)
        wsc = wsc.view(n, 4096 // 16)
        alpha = ((1.0 / gsf_w) / gsf_x).to(torch.float32)

        # the GEMM's share is read from the same timed calls (and clocks) as the step
        ms, gemm_part = _timed_split(lambda: nvfp4_quantize(x, gsf_x),
                                     lambda q: nvfp4_gemm(q[0], q[1], wp, wsc, alpha), flush, stream)
        gemm_ms = statistics.median(gemm_part)
        flop = 2.0 * 32760 * n * 4096
        out[f"c3_nvfp4_n{n}"] = summary(ms, flop, fp4_peak, {
            "step": "NVFP4 quantiser + block-scaled GEMM",
            "gemm_only_ms": round(gemm_ms, 4),
            "gemm_only_tflops": round(flop / (gemm_ms * 1e-3) / 1e12, 1),
            "gemm_frac_of_peak": round(flop / (gemm_ms * 1e-3) / 1e12 / fp4_peak, 4)})
        out[f"c3_nvfp4_n{n}"]["library_flashinfer"] = flashinfer_nvfp4(x, gsf_x, wp, wsc, alpha, flop, fp4_peak,
                                                                       flush, stream)
        if n == 4096 and cpu_seconds > 0:
            ac, asf = nvfp4_quantize(x, gsf_x)
            out["c3_nvfp4_n4096"]["cpu_baseline"] = nvfp4_cpu_baseline(ac, asf, wp, wsc, alpha, cpu_seconds)
    del x
    # QAD-style NVFP4 FFN at config 2's shape (H 4096, F 16384, GELU-tanh):
    # NVFP4Execution.ffn, whose up GEMM writes the intermediate as NVFP4 codes
    # for the down linear, against the unfused linear(gelu_linear(...)) chain
    from vflash_b200.native.h3_nvfp4_linear import NVFP4Execution, NVFP4Weight

    m, h, f = 32760, 4096, 16384
    x = seeded(m, h, 1004)

    def nv_weight(rows, cols, seed, input_scale):
        w = seeded(rows, cols, seed, std=0.02)
        gw = (448.0 * 6.0 / w.float().abs().max()).reshape(())
        packed, scales = nvfp4_quantize(w, gw)
        return NVFP4Weight(packed, scales.view(rows, cols // 16).contiguous(), (1.0 / gw).to(torch.float32),
                           input_scale.to(torch.float32))

    engine = NVFP4Execution()
    up = nv_weight(f, h, 2040, (448.0 * 6.0 / x.float().abs().max()).reshape(()))
    mid = engine.gelu_linear(x, up)
    down = nv_weight(h, f, 2041, (448.0 * 6.0 / mid.float().abs().max()).reshape(()))
    del mid
    fused_ms = statistics.median(_timed(lambda: engine.ffn(x, up, down), flush, stream))
    unfused_ms = statistics.median(_timed(lambda: engine.linear(engine.gelu_linear(x, up), down), flush, stream))
    same = bool(torch.equal(engine.ffn(x, up, down), engine.linear(engine.gelu_linear(x, up), down)))
    ffn_flop = 4.0 * m * h * f
    out["c2_shape_nvfp4_ffn_gelu"] = {
        "ms": round(fused_ms, 4), "tflops": round(ffn_flop / (fused_ms * 1e-3) / 1e12, 1),
        "frac_of_peak": round(ffn_flop / (fused_ms * 1e-3) / 1e12 / fp4_peak, 4),
        "unfused_ms": round(unfused_ms, 4), "equal_bits": same,
        "step": "NVFP4Execution.ffn (quantiser, up GEMM + GELU-tanh writing NVFP4 codes, down GEMM) vs "
                "linear(gelu_linear(x, up), down) (the bf16 intermediate round-trips and is quantised again)"}
    del x, up, down
    # --- the next-row fusions, after the benchmark configurations (which run
    # first, in the GPU state closest to the headline's) ---
    # next-row prologue at config 1's shape: RMSNorm + AdaLN modulate (per-token
    # scale / shift) + per-token e4m3 quantisation, fused vs the three launches
    from vflash_b200.kernels import quantize_fp8_norm_modulate
    from vflash_b200.native.h3_fused_ops import triton_strict_bf16_modulate

    m1 = 32760
    xp = seeded(m1, 4096, 1005)
    nw = (1 + seeded(1, 4096, 1006, std=0.1)).view(-1)
    sc = seeded(m1, 4096, 1007, std=0.3)
    sh = seeded(m1, 4096, 1008, std=0.3)

    def fused_prologue():
        quantize_fp8_norm_modulate(xp, nw, 1e-6, sc, sh)

    def unfused_prologue():
        normed = torch.nn.functional.rms_norm(xp, (4096,), nw, 1e-6)
        quantize_fp8_rows(triton_strict_bf16_modulate(normed.view(1, m1, 4096), sc, sh).view(m1, 4096))

    fused_ms = statistics.median(_timed(fused_prologue, flush, stream))
    unfused_ms = statistics.median(_timed(unfused_prologue, flush, stream))
    pbytes = m1 * 4096 * (2 + 2 + 2 + 1) + m1 * 4 + 4096 * 2
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    out["prologue_norm_modulate_quant"] = {
        "ms": round(fused_ms, 4), "gb_per_s": round(pbytes / (fused_ms * 1e-3) / 1e9, 1),
        "frac_of_measured_hbm": round(pbytes / (fused_ms * 1e-3) / 1e9 / hbm, 4),
        "unfused_ms": round(unfused_ms, 4),
        "step": "x [32760,4096] bf16, per-token scale/shift [32760,4096]: one pass (x, scale, shift "
                "read, codes written) vs torch rms_norm + vfb_modulate + vfb_fp8_quant_rows"}
    # the same prologue in front of an NVFP4 linear (codes 0.5 B and one
    # scale byte per 16 elements written instead of e4m3 codes)
    from vflash_b200.kernels import nvfp4_norm_modulate_quantize

    gsf_p = torch.full((), 448.0 * 6.0 / 8.0, device=device, dtype=torch.float32)

    def fused_prologue_nv():
        nvfp4_norm_modulate_quantize(xp, nw, 1e-6, sc, sh, gsf_p)

    def unfused_prologue_nv():
        normed = torch.nn.functional.rms_norm(xp, (4096,), nw, 1e-6)
        nvfp4_quantize(triton_strict_bf16_modulate(normed.view(1, m1, 4096), sc, sh).view(m1, 4096), gsf_p)

    fused_ms = statistics.median(_timed(fused_prologue_nv, flush, stream))
    unfused_ms = statistics.median(_timed(unfused_prologue_nv, flush, stream))
    pbytes = m1 * 4096 * (2 + 2 + 2) + m1 * 4096 // 2 + m1 * 4096 // 16 + 4096 * 2
    out["prologue_norm_modulate_nvfp4"] = {
        "ms": round(fused_ms, 4), "gb_per_s": round(pbytes / (fused_ms * 1e-3) / 1e9, 1),
        "frac_of_measured_hbm": round(pbytes / (fused_ms * 1e-3) / 1e9 / hbm, 4),
        "unfused_ms": round(unfused_ms, 4),
        "step": "as prologue_norm_modulate_quant, quantised to NVFP4 (vfb_nvfp4_norm_modulate_quant) vs torch "
                "rms_norm + vfb_modulate + vfb_nvfp4_quant_rows"}
    del xp, nw, sc, sh

    # next-row epilogue at config 1's shape: QKV projection + per-head QK-norm +
    # rotary, fused vs the GEMM followed by rms_norm and the strict rotary on Q and K
    from vflash_b200.native.h3_fp8_linear import QKNormRope, RowFP8Execution as _Exec
    from vflash_b200.native.h3_fused_ops import triton_strict_bf16_rotary

    xq = seeded(m1, 4096, 1009, outliers=True)
    wq, wqs = quantize_fp8_rows(seeded(12288, 4096, 2011, std=0.02), pad_to=1)
    qn = (1 + seeded(1, 128, 1010, std=0.1)).view(-1)
    kn = (1 + seeded(1, 128, 1011, std=0.1)).view(-1)
    pos = torch.arange(m1, device=device, dtype=torch.float32)[:, None]
    freq = 1.0 / (10000 ** (torch.arange(64, device=device, dtype=torch.float32) / 64))
    ang = torch.cat([pos * freq, pos * freq], dim=1)
    rc, rs = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    ex = _Exec("w8a8")
    rope = QKNormRope(qn, kn, rc, rs, 1e-5)
    x3 = xq.view(1, m1, 4096)

    def fused_qkv():
        ex.qkv_linear(x3, wq, wqs, qk_norm_rope=rope)

    def unfused_qkv():
        q, k, _v = ex.qkv_linear(x3, wq, wqs)
        for t, w in ((q, qn), (k, kn)):
            h = torch.nn.functional.rms_norm(t.view(1, m1, 32, 128), (128,), w, 1e-5)
            triton_strict_bf16_rotary(h, rc, rs)

    fq = statistics.median(_timed(fused_qkv, flush, stream))
    uq = statistics.median(_timed(unfused_qkv, flush, stream))
    qflop = 2.0 * m1 * 12288 * 4096
    out["qkv_qk_norm_rope"] = {
        "ms": round(fq, 4), "tflops": round(qflop / (fq * 1e-3) / 1e12, 1), "unfused_ms": round(uq, 4),
        "step": "quantiser + QKV GEMM with per-head QK-norm + rotary on Q and K in the epilogue, vs the "
                "same GEMM then torch rms_norm and vfb_rotary on Q and K"}

    # the same projection stored straight into pack_qkv's destination-major wire
    # layout (2 destinations x 2 chunks), vs planar Q/K/V then the permuting copy
    def wire_qkv():
        ex.qkv_linear(x3, wq, wqs, pack_chunks=2)

    def planar_then_pack():
        q, k, v = ex.qkv_linear(x3, wq, wqs)
        torch.stack([t.view(1, m1, 32, 128) for t in (q, k, v)]).reshape(
            3, 1, m1, 2, 2, 8, 128).permute(4, 3, 0, 1, 2, 5, 6).contiguous()

    fw = statistics.median(_timed(wire_qkv, flush, stream))
    uw = statistics.median(_timed(planar_then_pack, flush, stream))
    out["qkv_wire_pack"] = {
        "ms": round(fw, 4), "tflops": round(qflop / (fw * 1e-3) / 1e12, 1), "unfused_ms": round(uw, 4),
        "step": "quantiser + QKV GEMM storing (chunk, destination, qkv, rows, heads, dim) directly, vs "
                "planar Q/K/V then the pack_qkv permutation as a copy"}

    # the QKV projection with three rank-32 low-rank branches: native (one
    # concatenated down GEMM, three up GEMMs on tcgen05, merge in the QKV
    # epilogue) vs the reference's composition (cuBLAS bf16 linears, eager
    # scale and add after the projection)
    from dataclasses import dataclass as _dc

    @_dc(frozen=True)
    class _Residual:
        down: torch.Tensor
        up: torch.Tensor
        scaling: float

    lr_rank = 32
    residuals = tuple(_Residual(seeded(lr_rank, 4096, 1020 + i, std=0.02), seeded(4096, lr_rank, 1030 + i, std=0.02),
                                s) for i, s in enumerate((0.5, 1.0, 0.25)))

    def native_lora_qkv():
        ex.qkv_linear(x3, wq, wqs, residuals=residuals)

    def reference_lora_qkv():
        planes = ex.qkv_linear(x3, wq, wqs)
        torch.cat([p + torch.nn.functional.linear(torch.nn.functional.linear(x3, r.down), r.up) * r.scaling
                   for p, r in zip(planes, residuals)], dim=-1)

    def native_products():
        ex.qkv_low_rank(x3, residuals)

    def cublas_products():
        for r in residuals:
            torch.nn.functional.linear(torch.nn.functional.linear(x3, r.down), r.up)

    fl = statistics.median(_timed(native_lora_qkv, flush, stream))
    rl = statistics.median(_timed(reference_lora_qkv, flush, stream))
    fp_ = statistics.median(_timed(native_products, flush, stream))
    cp_ = statistics.median(_timed(cublas_products, flush, stream))
    lr_bytes = m1 * 4096 * 2 + 3 * m1 * 4096 * 2  # read the input once, write three [M, 4096] outputs
    out["qkv_low_rank_r32"] = {
        "ms": round(fl, 4), "reference_composition_ms": round(rl, 4),
        "products_ms": round(fp_, 4), "products_cublas_ms": round(cp_, 4),
        "products_gb_per_s": round(lr_bytes / (fp_ * 1e-3) / 1e9, 1),
        "step": "QKV projection + three rank-32 LoRA branches (down [32,4096], up [4096,32] each): one "
                "concatenated bf16 down GEMM, three bf16 up GEMMs (tcgen05 kind::f16), merge fused in the "
                "QKV epilogue; vs planar QKV then per branch cuBLAS linear(linear(x, down), up) * s + add"}
    del xq, wq, wqs, rc, rs, ang, residuals

    out["peak_note"] = ("fp8 peak = 2 x measured cuBLAS bf16 burst, fp4 peak = 4 x; nominal dense "
                        "fp8 4.5, fp4 9 PFLOP/s")
    return out


STACK_BLOCKS, STACK_TOKENS, STACK_HIDDEN, STACK_FFN = 48, 65520, 4096, 16384


def stack_blocks(count: int, device):
    """Seeded N(0,0.02) FP8 weights of ``count`` blocks, one block at a time (per-row e4m3)."""
    from vflash_b200.native.h3_block_stack import block_shapes
    from vflash_b200.native.h3_parallel import FP8Weight

    gen = torch.Generator(device=device)
    for b in range(count):
        block = {}
        for j, (name, n, k) in enumerate(block_shapes(STACK_HIDDEN, STACK_FFN)):
            gen.manual_seed(7000 + 10 * b + j)
            w = torch.randn(n, k, generator=gen, device=device) * 0.02
            scale = w.abs().amax(dim=1, keepdim=True) / 448.0
            block[name] = FP8Weight((w / scale).to(torch.float8_e4m3fn), scale)
            del w
        yield block


def stack_config(args, device, rank: int, world: int, barrier, max_over_ranks) -> dict:
    """Config 4: 48 blocks of FP8 linears, M = 65520 tokens sharded over the ranks.

    Weights stream from the pinned arena through the two-slot ring (each rank
    pins and copies 1/world of every block; NCCL all-gathers the rest) and,
    for comparison, from a resident copy of the stack.  Every rank runs the
    same collective steps; times are the max over ranks.
    """
    import torch.distributed as dist

    from vflash_b200.native.h3_block_stack import FP8BlockStack, block_flops, block_linears
    from vflash_b200.native.h3_parallel import partition_rows, shard_rows_count
    from vflash_b200.native.h3_pinned_arena import FP8BlockRing

    group = dist.group.WORLD if world > 1 else None
    blocks = args.stack_blocks
    t0 = time.perf_counter()
    stack = FP8BlockStack(stack_blocks(blocks, device), STACK_HIDDEN, STACK_FFN, device, group=group)
    setup_s = time.perf_counter() - t0
    gen = torch.Generator(device=device).manual_seed(4004)
    tokens = torch.randn(STACK_TOKENS, STACK_HIDDEN, generator=gen, device=device).to(torch.bfloat16)
    shard, valid = partition_rows(tokens, rank, world)
    del tokens
    shard = shard.reshape(-1, 1, STACK_HIDDEN)
    gate = torch.full((1, STACK_HIDDEN), 1 / 32, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    def timed(forward, steps: int) -> tuple[float, torch.Tensor]:
        out = forward(shard, gate)  # warm-up step
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            out = forward(shard, gate)
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps), out

    steps = args.stack_steps
    streamed_ms, out = timed(stack.forward, steps)
    finite = bool(torch.isfinite(out[:valid].float()).all())
    # one more streamed step with CUDA events around each block's host copy and
    # all-gather on the copy stream (the weight path's own cost per block)
    stack.ring.profile = True
    stack.forward(shard, gate)
    torch.cuda.synchronize(device)
    h2d_ms, gather_ms, profiled = stack.ring.copy_times()
    stack.ring.profile = False
    h2d_ms, gather_ms = max_over_ranks(h2d_ms), max_over_ranks(gather_ms)
    resident_ring = FP8BlockRing(stack.layout, stack.host_blocks, device, group=group, resident=True)
    resident_ms, out2 = timed(
        lambda h, g: resident_ring.run(h, lambda w, x: block_linears(stack.execution, w, x, g)), steps)
    same = bool(torch.equal(out, out2))
    # the same resident stack replayed from one CUDA graph (no per-block host work)
    import copy

    graphed = copy.copy(stack)
    graphed.ring = resident_ring
    replay = graphed.capture(shard, gate)
    graph_ms, out3 = timed(lambda h, g: replay(), steps)
    graph_same = bool(torch.equal(out3, out2))
    del resident_ring, out, out2, out3, replay, graphed
    torch.cuda.empty_cache()
    peaks = measured_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
    rows = shard_rows_count(STACK_TOKENS, world)
    flop_step = blocks * block_flops(STACK_TOKENS, STACK_HIDDEN, STACK_FFN)
    per_gpu_tflops = blocks * block_flops(rows, STACK_HIDDEN, STACK_FFN) / (streamed_ms * 1e-3) / 1e12
    return {
        "workload": f"c4: {blocks} blocks x FP8 linears (QKV [12288,4096], out [4096,4096], up [16384,4096] "
                    f"GELU-tanh, down [4096,16384]); M={STACK_TOKENS} tokens, {rows} per rank",
        "scaling": "strong (the M=65520 tokens are split over the ranks, weights replicated)",
        "streamed_ms_per_step": round(streamed_ms, 2),
        "resident_ms_per_step": round(resident_ms, 2),
        "resident_graph_ms_per_step": round(graph_ms, 2),
        "graph_equals_eager": graph_same,
        "streaming_overhead": round(streamed_ms / resident_ms - 1.0, 4),
        "tflops_whole_job": round(flop_step / (streamed_ms * 1e-3) / 1e12, 1),
        "tflops_per_gpu": round(per_gpu_tflops, 1),
        "frac_of_sustained_peak": round(per_gpu_tflops / fp8_peak, 4),
        "weight_bytes_per_block": stack.weight_bytes_per_block,
        "h2d_bytes_per_rank_per_step": blocks * stack.ring.chunk,
        "copy_stream_per_block_ms": {"host_copy": round(h2d_ms, 4), "all_gather": round(gather_ms, 4),
                                     "blocks_profiled": profiled,
                                     "note": "CUDA events on the copy stream, max over ranks; overlapped "
                                             "with the compute stream"},
        "weight_path": "pinned arena -> copy stream (two slots)" + (
            f", each rank copies 1/{world} of a block and NCCL all-gathers the rest" if world > 1 else ""),
        "output_finite": finite,
        "streamed_equals_resident": same,
        "setup_s": round(setup_s, 1),
        "steps": steps,
        "l2": "inputs larger than L2 (201 MB of weights per block)",
    }


def library_same_shape(device, flush, stream) -> dict:
    """The reference's W8A8 call at config 1's exact shape on this box: the per-token quantiser then
    rowwise ``torch._scaled_mm`` (cuBLASLt) + bias (src/vflash/native/h3_fp8_linear.py:109-121), with the
    quantiser's codes from this library (bit-identical to the reference's), median of 20 calls with L2
    flushed before each."""
    try:
        from vflash_b200.kernels import quantize_fp8_rows

        x_host, w_codes, w_scales, bias = synthetic_workload(device, 0, M)
        x = x_host.to(device)
        codes, scales = quantize_fp8_rows(x)

        def gemm():
            out = torch._scaled_mm(codes, w_codes.t(), scale_a=scales, scale_b=w_scales.t(),
                                   out_dtype=torch.bfloat16)
            out = out[0] if isinstance(out, tuple) else out
            return out[:M] + bias

        def step():
            c, s = quantize_fp8_rows(x)
            out = torch._scaled_mm(c, w_codes.t(), scale_a=s, scale_b=w_scales.t(), out_dtype=torch.bfloat16)
            out = out[0] if isinstance(out, tuple) else out
            return out[:M] + bias

        flop = 2.0 * M * N_QKV * K
        gemm_ms = statistics.median(_timed(gemm, flush, stream, reps=20, warmup=3))
        step_ms = statistics.median(_timed(step, flush, stream, reps=20, warmup=3))
        return {"gemm_plus_bias_ms": round(gemm_ms, 4),
                "gemm_plus_bias_tflops": round(flop / (gemm_ms * 1e-3) / 1e12, 1),
                "step_ms": round(step_ms, 4), "step_tflops": round(flop / (step_ms * 1e-3) / 1e12, 1),
                "call": "rowwise torch._scaled_mm(codes, W.t(), scale_a [M,1], scale_b [1,N], bf16)[:M] + bias"}
    except Exception as exc:  # pragma: no cover - diagnostic only
        return {"error": str(exc)[:200]}


FLASHINFER_MODULES = Path(__file__).resolve().parent / "tests" / ".flashinfer_ref"


def flashinfer_nvfp4(x, gsf_x, wp, wsc, alpha, flop, peak, flush, stream) -> dict:
    """The reference's NVFP4 backend at the same shape on this box (same-box library bar).

    src/vflash/native/h3_nvfp4_linear.py:102 and 118-130 call FlashInfer's
    ``nvfp4_quantize`` (128x4 scales, no shuffle) and ``mm_fp4(...,
    backend="cutlass")``.  FlashInfer compiles those modules just in time;
    they are used only when prebuilt in-tree (tests/golden/
    build_flashinfer_reference.py --gemm), so the bench never compiles on
    the box.  The weight codes are this library's (bit-identical to
    FlashInfer's quantiser); median of 20 calls with L2 flushed before each.
    """
    ops = FLASHINFER_MODULES.glob("**/cached_ops/*/*.so")
    names = {p.parent.name for p in ops}
    if not {"fp4_gemm_cutlass", "fp4_quantization_100"} <= names:
        return {"unavailable": "FlashInfer's NVFP4 modules are not prebuilt in tests/.flashinfer_ref"}
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(FLASHINFER_MODULES))
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    try:
        import flashinfer as fi

        layout = fi.SfLayout.layout_128x4

        def quantize():
            return fi.nvfp4_quantize(x, gsf_x, sfLayout=layout, do_shuffle=False)

        def gemm(q):
            return fi.mm_fp4(q[0], wp.T, q[1], wsc.T, alpha, torch.bfloat16, None, block_size=16,
                             use_8x4_sf_layout=False, backend="cutlass", use_nvfp4=True)

        step, gemm_part = _timed_split(quantize, gemm, flush, stream, reps=20, warmup=3)
        step_ms, gemm_ms = statistics.median(step), statistics.median(gemm_part)
        return {"ms": round(step_ms, 4), "tflops": round(flop / (step_ms * 1e-3) / 1e12, 1),
                "gemm_only_ms": round(gemm_ms, 4),
                "gemm_only_tflops": round(flop / (gemm_ms * 1e-3) / 1e12, 1),
                "gemm_frac_of_peak": round(flop / (gemm_ms * 1e-3) / 1e12 / peak, 4),
                "call": f"flashinfer {fi.__version__} nvfp4_quantize + mm_fp4(backend='cutlass')"}
    except Exception as exc:  # pragma: no cover - diagnostic only
        return {"error": str(exc)[:200]}


def library_fp8_probe(device) -> dict:
    """cuBLASLt FP8 GEMM throughput (torch._scaled_mm, tensorwise) on this box, for context."""
    try:
        n = 8192
        a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=device)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record()
        for _ in range(reps):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / reps
        return {"tflops": round(2 * n**3 / (ms * 1e-3) / 1e12, 1), "shape": "8192^3 tensorwise"}
    except Exception as exc:  # pragma: no cover - diagnostic only
        return {"error": str(exc)[:200]}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


def cpu_baseline(x_host, w_codes, w_scales, bias, seconds: float) -> dict:
    """The reference's weight-only CPU path, timed on a bounded row sample."""
    from oracle.fp8 import weight_only_linear

    threads = cpu_threads()
    torch.set_num_threads(threads)
    rows = 1024
    sample = x_host[:rows].contiguous()
    weight_only_linear(sample[:16], w_codes, w_scales, bias)  # warm-up
    reps, elapsed = 0, 0.0
    while elapsed < seconds or reps < 1:
        t0 = time.perf_counter()
        weight_only_linear(sample, w_codes, w_scales, bias)
        elapsed += time.perf_counter() - t0
        reps += 1
    flop = 2.0 * rows * N_QKV * K * reps
    return {"value": round(flop / elapsed / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "cpu": cpu_model(),
            "sample": f"{reps} x RowFP8Execution('weight-only').linear on {rows} of {M} rows "
                      f"(dequantise W to bf16 each call, then F.linear on bf16), {elapsed:.1f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.fp8 import weight_only_linear

    threads = cpu_threads()
    torch.set_num_threads(threads)
    rows = args.reference_rows
    gen = torch.Generator().manual_seed(1001)
    x = torch.randn(rows, K, generator=gen)
    count = round(0.001 * rows * K)
    idx = torch.randperm(rows * K, generator=torch.Generator().manual_seed(1002))[:count]
    x.view(-1)[idx] *= 20
    x = x.to(torch.bfloat16)
    w = (torch.randn(N_QKV, K, generator=torch.Generator().manual_seed(2010)) * 0.02)
    from oracle.fp8 import quantize_weight

    codes, scales = quantize_weight(w.numpy())
    w_codes = torch.from_numpy(codes).view(torch.float8_e4m3fn)
    w_scales = torch.from_numpy(scales)
    bias = (torch.randn(N_QKV, generator=torch.Generator().manual_seed(3001)) * 0.01).to(torch.bfloat16)
    for _ in range(args.warmup):
        weight_only_linear(x, w_codes, w_scales, bias)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        y = weight_only_linear(x, w_codes, w_scales, bias)
        q, k, v = y.chunk(3, dim=-1)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    flop = 2.0 * rows * N_QKV * K
    value = args.steps * flop / total / 1e12
    sample = (f"{rows} of {M} rows per step through RowFP8Execution('weight-only').linear "
              f"(reference CPU path: dequantise W to bf16, F.linear) + chunk(3)")
    line = {
        "impl": "reference",
        "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (dequantised e4m3 weights)",
        "data": "synthetic (seeded, same generators as the GPU arm)",
        "config": {"workload": WORKLOAD, "M": M, "N": N_QKV, "K": K, "bias": True,
                   "sample_rows": rows, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "cpu": cpu_model(), "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["vflash_b200", "reference"], default="vflash_b200")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--reference-rows", type=int, default=M,
                        help="rows of X per reference step (default: all of config 1's 32760)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-library-probe", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-stack", action="store_true", help="skip the config 4 block stack")
    parser.add_argument("--e2e-chunk-rows", type=int, default=4096)
    parser.add_argument("--no-numa-bind", action="store_true",
                        help="keep the process on all host CPUs (default: the GPU's local CPUs)")
    parser.add_argument("--stack-blocks", type=int, default=STACK_BLOCKS)
    parser.add_argument("--stack-steps", type=int, default=2)
    parser.add_argument("--no-other-configs", action="store_true",
                        help="skip the extra benchmark config 0/2/3 measurements")
    parser.add_argument("--rows", type=int, default=M,
                        help="token rows M (default 32760 = benchmark config 1; smaller only for profiling)")
    args = parser.parse_args()
    args.warmup = max(3, args.warmup)  # the timing rules require >= 3 warm-up steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
