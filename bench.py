#!/usr/bin/env python3
"""Benchmark of the fused W8A8 INT8 linear on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one pass of the hot path over one batch: fp16 activations
X[4096,3072] (1% outlier channels x20) -> block-128 Hadamard rotation +
per-token INT8 quantization (prologue kernel) -> tcgen05 kind::i8 GEMM
against the rotated, per-channel-quantized weight W[12288,3072] with the
fused scale/bias/fp16 epilogue.  Metric: TOPS = 2*M*N*K / step time.

Multi-GPU (torchrun, one rank per GPU): column-parallel N-sharding of the
same config-2 layer (strong scaling: each of P ranks owns 12288/P output
columns), with the output reassembled on every rank INSIDE the step: the
GEMM epilogue writes each output tile into every rank's full Y over NVLink
(b2_quant_linear_gather) and the step ends when every rank has all of Y
(b2_gather_wait).  Side figures: the same step with an NCCL all-gather
instead, the rank-local linear alone, and weak scaling (12288 columns per
rank, gather included).

The reference arm (--impl reference) times the CPU oracle -- the reference's
math restated in C (oracle/) -- on the host cores over a bounded sample of
the same workload.
"""
import argparse
import json
import re
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "rdna2-gfx1030-ai-handbook_b200"))

M, K, N = 4096, 3072, 12288
ROT = 128
METRIC = "INT8 fused-GEMM TOPS & % of tensor peak at 1/2/4/8 B200 vs host-CPU ref"
UNIT = "TOPS"
SEED = 20261106


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sustained", action="store_true", help="skip the >= 1 s sustained leg (profiling runs)")
    ap.add_argument("--sets", type=int, default=4, help="input sets cycled to defeat L2 reuse")
    ap.add_argument("--gather", choices=("fused", "ce"), default="fused",
                    help="N > 1 step: gather by SM peer stores in the GEMM epilogue (fused) or by copy engines "
                         "overlapped with a chunked GEMM (ce)")
    ap.add_argument("--gather-store", choices=("auto", "sm", "tma"), default="auto",
                    help="transport of the fused gather's peer copies: SM stores or TMA stores")
    ap.add_argument("--activations", choices=("fp16", "int8"), default="int8",
                    help="c5 column-parallel stack: gather every fp16 layer output, or exchange only the next "
                         "layer's INT8 input codes")
    ap.add_argument("--exchange-two-launch", action="store_true",
                    help="c5 INT8 exchange: the two phases as separate kernels instead of one cooperative launch")
    ap.add_argument("--column-parallel", action="store_true",
                    help="c5 on one GPU through the column-parallel stack (the N > 1 code path, eager calls)")
    ap.add_argument("--workload", default="c2",
                    help="c2 (headline, default), c1, c3m1/c3m16/c3m128/c3m2048 (W4A16), "
                         "c4m1/c4m2048 (FP8), w4a8m<M> (W4A8), c5 (28-block W8A8 DiT stack; also "
                         "column-parallel under torchrun), moss (the reference's four M=1061 shapes); "
                         "other workloads run on one GPU")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
            "source": "fallback"}


def synth_inputs(rng, m, k):
    x = rng.standard_normal((m, k), dtype=np.float32)
    idx = rng.choice(k, size=max(1, round(0.01 * k)), replace=False)
    x[:, idx] *= 20.0
    return x


# ------------------------------------------------------------- CPU oracle
def host_threads():
    """Host cores this process may run on.  torchrun sets OMP_NUM_THREADS=1
    for every rank; the CPU legs run on rank 0 alone and pass this count to
    the oracle explicitly, so they use every core either way."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def cpu_run(rows, threads=0):
    """Time the oracle's full W8A8 linear on `rows` tokens of the workload."""
    import oracle
    rng = np.random.default_rng(SEED)
    x = synth_inputs(rng, rows, K).astype(np.float16).view(np.uint16)
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    wq, sw = oracle.quant_rows_int8(oracle.rotate_rows(w, oracle.F32, ROT))
    bias = oracle.encode((rng.standard_normal(N) * 0.02).astype(np.float32), oracle.F16)
    t0 = time.perf_counter()
    oracle.w8a8_linear(x, oracle.F16, ROT, wq, sw, bias, oracle.F16, oracle.EPI_SEPARATE,
                       oracle.F16, threads=threads)
    return time.perf_counter() - t0


def cpu_baseline(budget_s):
    threads = host_threads()
    t1 = cpu_run(64, threads)
    rows = int(min(M, max(64, budget_s / max(t1 / 64, 1e-9))))
    rows = max(64, rows // 64 * 64)
    dt = cpu_run(rows, threads)
    return {"value": round(2.0 * rows * N * K / dt / 1e12, 4), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"oracle/qlinear_oracle.c w8a8 linear (rotate+quantize+exact GEMM+epilogue) "
                      f"on {rows} of {M} tokens x N={N} x K={K}, {dt:.2f} s, {threads} OpenMP threads"}


def _hadamard(b):
    """Orthonormal Sylvester Hadamard matrix of order b (fp32)."""
    import torch
    h = torch.ones((1, 1))
    while h.shape[0] < b:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / float(b) ** 0.5


def torch_cpu_linear(x16, h, wq, sw, bias16):
    """The reference's PyTorch math for the MOSS INT8 linear, on the CPU:
    block rotation by a matmul with the orthonormal Hadamard
    (production/MOSS_RDNA2_INT8/backend.py:112-118), per-row absmax/127
    round-half-even INT8 (the quantize_int8_rowwise call, :122), the exact
    INT8 GEMM (torch._int_mm in the role of the backend's
    _int8_matmul_accumulate), and the epilogue
    (acc.float() * (sx * sw)).to(out) + bias (:128-145)."""
    import torch
    m, k = x16.shape
    b = h.shape[0]
    xr = (x16.float().reshape(m, k // b, b) @ h).reshape(m, k)
    amax = xr.abs().amax(1, keepdim=True)
    sx = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.clamp(torch.round(xr / sx), -127, 127).to(torch.int8)
    acc = torch._int_mm(q, wq.T)
    return (acc.float() * (sx * sw[None, :])).to(torch.float16) + bias16


def torch_cpu_baseline(budget_s, threads):
    """The torch CPU leg on `threads` host threads over a bounded token
    sample of the config-2 workload (the same op count per token)."""
    import torch
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(SEED)
        w = torch.randn((N, K), generator=g) * 0.02
        h = _hadamard(ROT)
        wr = (w.reshape(N, K // ROT, ROT) @ h).reshape(N, K)
        sw = wr.abs().amax(1) / 127.0
        wq = torch.clamp(torch.round(wr / sw[:, None]), -127, 127).to(torch.int8)
        bias = (torch.randn(N, generator=g) * 0.02).half()

        def run(rows):
            x = torch.from_numpy(synth_inputs(np.random.default_rng(SEED), rows, K)).half()
            t0 = time.perf_counter()
            torch_cpu_linear(x, h, wq, sw, bias)
            return time.perf_counter() - t0

        run(64)
        t1 = run(64)
        rows = int(min(M, max(64, 0.5 * budget_s / max(t1 / 64, 1e-9)))) // 64 * 64
        dt = min(run(rows), run(rows))  # the first large call also pays page faults
    finally:
        torch.set_num_threads(prev)
    return {"value": round(2.0 * rows * N * K / dt / 1e12, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"torch CPU restatement of the reference's linear math (matmul rotation, rowwise INT8, "
                      f"torch._int_mm, backend.py epilogue) on {rows} of {M} tokens x N={N} x K={K}, {dt:.2f} s, "
                      f"{threads} torch threads"}


def c2_config(world, sets):
    """The config dict of the config-2 line at `world` GPUs (both arms print it)."""
    if world == 1:
        return {"workload": "config2: W8A8 INT8 linear with block-128 Hadamard rotation, "
                            "fp16 X[4096,3072] (1% outlier channels x20) -> fp16 Y[4096,12288]",
                "M": M, "N": N, "N_per_rank": N, "K": K, "rotation_block": ROT, "parallelism": "single GPU",
                "l2": f"inputs cycled over {sets} buffer sets "
                      f"({sets * (M * K * 2 + N * K) / 2**20:.0f} MiB > 126 MB L2)"}
    return {"workload": "config2 column-parallel: W8A8 INT8 linear with block-128 Hadamard rotation, "
                        "fp16 X[4096,3072] -> fp16 Y[4096,12288], N sharded over the ranks, Y reassembled "
                        "on every rank inside the step",
            "M": M, "N": N, "N_per_rank": N // world, "K": K, "rotation_block": ROT,
            "parallelism": f"column-parallel N-shard x{world}, output gather fused into the GEMM epilogue "
                           "(NVLink peer stores)",
            "l2": f"inputs cycled over {sets} buffer sets, output buffers alternate (> 126 MB L2)"}


def run_reference(args, rank):
    """--impl reference: the CPU oracle port on the host cores (rank 0 only)."""
    if rank != 0:
        return
    threads = host_threads()
    t1 = cpu_run(64, threads)
    per_row = t1 / 64
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(min(M, max(8, budget / per_row)))
    import oracle as o
    rng = np.random.default_rng(SEED)
    x = synth_inputs(rng, rows, K).astype(np.float16).view(np.uint16)
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    wq, sw = o.quant_rows_int8(o.rotate_rows(w, o.F32, ROT))
    bias = o.encode((rng.standard_normal(N) * 0.02).astype(np.float32), o.F16)

    def step():
        o.w8a8_linear(x, o.F16, ROT, wq, sw, bias, o.F16, o.EPI_SEPARATE, o.F16, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(1, args.steps)
    value = 2.0 * rows * N * K / dt / 1e12
    torch_leg = torch_cpu_baseline(min(10.0, args.cpu_budget_s), threads)
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "impl": "reference",
            "config": c2_config(args.gpus, args.sets),
            "torch_reference_math": torch_leg,
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "port",
                             "sample": f"{rows} of {M} tokens per step, the whole {N}-column layer on the host "
                                       f"(oracle port, C/OpenMP)"},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons with NVML every 5 ms
    while the timed region runs (same fields as the nvidia-smi clocks query)."""

    NAMES = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
             "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index):
        self.samples, self.power, self.reasons = [], [], set()
        self.stop_evt = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _loop(self):
        while not self.stop_evt.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                self.power.append(self.nvml.nvmlDeviceGetPowerUsage(self.h) / 1000.0)
                mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.NAMES.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                break
            time.sleep(0.005)

    def __enter__(self):
        if self.nvml:
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.nvml:
            self.stop_evt.set()
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_mhz_min": min(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "power_w_max": max(self.power) if self.power else None,
                "samples": len(self.samples)}


def e2e_pipeline(torch, dev, stream, xs, linear, out_shape, n_e, barrier):
    """End-to-end steps through a public call with host buffers: every step
    uploads its X from pinned host memory and reads its Y back into pinned
    host memory.  Uploads run on one copy stream, the linear on the compute
    stream and read-backs on another copy stream, double buffered, so step
    i's read-back overlaps step i+1's upload and linear (PCIe is full duplex)
    -- how a serving loop streams requests through the call.  Every step's
    copies stay inside the timed region.  The last output read back is
    checked against a direct call.  Returns ms per step on this rank."""
    m, k = xs[0].shape
    x_host = [xs[b].cpu().pin_memory() for b in range(2)]
    y_host = [torch.empty(out_shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    xd = [torch.empty((m, k), device=dev, dtype=torch.float16) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    up = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    down = [torch.cuda.Event() for _ in range(2)]
    started = [False, False]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_up):
            if started[b]:
                s_up.wait_event(done[b])        # the linear of step i-2 has read xd[b]
            xd[b].copy_(x_host[b], non_blocking=True)
            up[b].record(s_up)
        stream.wait_event(up[b])
        if started[b]:
            stream.wait_event(down[b])          # y_host[b] of step i-2 is home (the buffer is reused)
        y = linear(xd[b])
        done[b].record(stream)
        with torch.cuda.stream(s_down):
            s_down.wait_event(done[b])
            y_host[b].copy_(y, non_blocking=True)
            y.record_stream(s_down)
            down[b].record(s_down)
        started[b] = True

    def drain():
        for b in range(2):
            if started[b]:
                stream.wait_event(down[b])

    for i in range(4):
        e2e_step(i)
    drain()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n_e):
        e2e_step(i)
    drain()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n_e
    ref_y = linear(xd[(n_e - 1) % 2]).cpu()
    assert torch.equal(y_host[(n_e - 1) % 2].view(torch.int16), ref_y.view(torch.int16)), \
        "pipelined end-to-end output differs from a direct call"
    return ms


# ------------------------------------------------------------------ B200
def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import rdna2_ops
    from rdna2_ops import _native as nat
    from rdna2_ops import qlinear

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = nat.library()
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)

    w = torch.randn((N, K), generator=gen, device=dev) * 0.02
    wq, sw = qlinear.quantize_weight(w, rotation_block=ROT)
    del w
    bias = (torch.randn(N, generator=gen, device=dev) * 0.02).half()
    xs = []
    for s in range(args.sets):
        x = torch.randn((M, K), generator=gen, device=dev)
        idx = torch.randperm(K, generator=gen, device=dev)[: round(0.01 * K)]
        x[:, idx] *= 20.0
        xs.append(x.half())
    # Distinct weight copies per set so no operand stays L2-resident across steps.
    wqs = [wq] + [wq.clone() for _ in range(args.sets - 1)]
    out = torch.empty((M, N), device=dev, dtype=torch.float16)
    ws_bytes = lib.b2_quant_linear_workspace_bytes(M, K)
    workspace = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        s = i % args.sets
        st = lib.b2_quant_linear(nat.KIND_I8, xs[s].data_ptr(), nat.F16, M, K, K, ROT,
                                 wqs[s].data_ptr(), K, N, sw.data_ptr(), N, bias.data_ptr(),
                                 nat.F16, nat.EPI_SEPARATE, out.data_ptr(), nat.F16, N,
                                 workspace.data_ptr(), ws_bytes, stream.cuda_stream)
        if st:
            nat.check(st, "b2_quant_linear")

    def barrier():
        pass  # one rank

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    nat.device_status(reset=True)

    # ---- timed region: K fused-linear steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        t_wall = time.perf_counter()
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
    ms = e0.elapsed_time(e1) / args.steps
    value = 2.0 * M * N * K / (ms * 1e-3) / 1e12

    # ---- sustained: the same step back to back for >= 1 s (clock record beside it)
    n_sus = args.steps if args.no_sustained else max(args.steps, int(1.0 / (ms * 1e-3)) + 1)
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as sus_clocks:
        e0.record(stream)
        for i in range(n_sus):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    sus_ms = e0.elapsed_time(e1) / n_sus

    # ---- dominant kernel alone (GEMM on pre-quantized activations), same stream
    qa, sa = rdna2_ops.act_quant(xs[0], rotation_block=ROT)
    qas = [qa] + [rdna2_ops.act_quant(xs[s], rotation_block=ROT)[0] for s in range(1, args.sets)]

    def gemm(i):
        s = i % args.sets
        st = lib.b2_qgemm(nat.KIND_I8, qas[s].data_ptr(), K, wqs[s].data_ptr(), K, M, N, K,
                          sa.data_ptr(), sw.data_ptr(), N, bias.data_ptr(), nat.F16,
                          nat.EPI_SEPARATE, out.data_ptr(), nat.F16, N, stream.cuda_stream)
        if st:
            nat.check(st, "b2_qgemm")

    for i in range(5):
        gemm(i)
    n_g = max(20, args.steps // 2)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(n_g):
        gemm(i)
    e1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = e0.elapsed_time(e1) / n_g
    # prologue alone: a CUDA graph of the C-ABI calls the linear makes (the
    # kernel's own time, not the host's launch rate)
    def prologue(i):
        nat.check(lib.b2_act_quant(xs[i % args.sets].data_ptr(), nat.F16, M, K, K, ROT, 0, qa.data_ptr(), K,
                                   sa.data_ptr(), nat.stream_ptr(dev)), "b2_act_quant")

    for i in range(3):
        prologue(i)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(40):
            prologue(i)
    graph.replay()
    torch.cuda.synchronize()
    reps = max(1, n_g // 40)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    pro_ms = e0.elapsed_time(e1) / (reps * 40)
    del graph

    pk = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]
    achieved = 2.0 * M * N * K / (gemm_ms * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers
    e2e_ms = e2e_pipeline(torch, dev, stream, xs,
                          lambda xd: rdna2_ops.w8a8_linear(xd, wq, sw, bias, rotation_block=ROT,
                                                           out_dtype=torch.float16, workspace=workspace),
                          (M, N), max(10, min(100, args.steps // 5)), barrier)

    status = nat.device_status()
    if rank != 0:
        return
    cpu = cpu_torch = cpu_torch2 = None
    if not args.no_cpu_baseline:  # host baselines are N=1 figures
        cpu = cpu_baseline(args.cpu_budget_s)
        cpu_torch = torch_cpu_baseline(args.cpu_budget_s, host_threads())
        cpu_torch2 = torch_cpu_baseline(args.cpu_budget_s, 2)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": c2_config(1, args.sets),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
                     "unit": "TOPS", "frac": round(achieved / int8_peak, 4), "traffic": None,
                     "traffic_note": "not measured in this run (no profiler inside the bench); the ncu capture "
                                     "of this kernel on this workload is summarised in profiles/",
                     "kernel": "qgemm_pair_kernel<kind::i8,BN=256> (auto path on C2)",
                     "peak_source": f"2 x bf16_tflops ({pk['source']}): kind::i8 issues at twice "
                                    "the kind::f16 rate",
                     "frac_of_nominal_4500": round(achieved / 4500.0, 4),
                     "gemm_ms": round(gemm_ms, 5), "prologue_ms": round(pro_ms, 5),
                     "prologue_gbs": round((M * K * 2 + M * K + M * 4) / (pro_ms * 1e-3) / 1e9, 1)},
        "cpu_baseline": cpu,
        "cpu_baseline_torch": cpu_torch,
        "cpu_baseline_torch_2threads": cpu_torch2,
        "sustained": {"value": round(2.0 * M * N * K / (sus_ms * 1e-3) / 1e12, 2), "ms_per_step": round(sus_ms, 5),
                      "steps": n_sus, "seconds": round(sus_ms * n_sus * 1e-3, 3), "clocks": sus_clocks.summary()},
        "e2e": {"value": round(2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, 3), "unit": UNIT,
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                "api": "rdna2_ops.w8a8_linear (C ABI b2_quant_linear), pinned host X in, Y out, "
                       "uploads / linear / read-backs on three streams, double buffered",
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
        "device_status": status,
        "wall_s_timed": round(t_wall, 4),
    }
    print(json.dumps(line), flush=True)


def _max_over_ranks(torch, dist, dev, value):
    t = torch.tensor([value], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def run_b200_multi(args, rank, world, local_rank):
    """N > 1: config 2 column-parallel over the ranks with the output gather
    inside every step (strong scaling; weak scaling and the NCCL gather as
    side figures).  Every rank generates the same X and full weight from the
    same seed and keeps its shard."""
    import torch
    import torch.distributed as dist
    import rdna2_ops
    from rdna2_ops import _native as nat
    from rdna2_ops import qlinear
    from rdna2_ops.column_parallel import PeerGather, ce_chunks, set_gather_store

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = nat.library()
    set_gather_store(args.gather_store)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    w = torch.randn((N, K), generator=gen, device=dev) * 0.02
    wq_full, sw_full = qlinear.quantize_weight(w, rotation_block=ROT)
    del w
    bias_full = (torch.randn(N, generator=gen, device=dev) * 0.02).half()
    xs = []
    for _ in range(args.sets):
        x = torch.randn((M, K), generator=gen, device=dev)
        idx = torch.randperm(K, generator=gen, device=dev)[: round(0.01 * K)]
        x[:, idx] *= 20.0
        xs.append(x.half())
    ns = N // world
    c0 = rank * ns
    wq = wq_full[c0:c0 + ns].contiguous()
    sw = sw_full[c0:c0 + ns].contiguous()
    bias = bias_full[c0:c0 + ns].contiguous()
    wqs = [wq] + [wq.clone() for _ in range(args.sets - 1)]
    ws_bytes = lib.b2_quant_linear_workspace_bytes(M, K)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    # Every rank maps every peer's buffers; if that fails anywhere, all ranks
    # agree (one all-reduce) and time the NCCL-gather step instead, saying so.
    g, peer_error = None, ""
    try:
        g = PeerGather(M * N * world, torch.float16)   # also holds the weak-scaling output (N * world columns)
    except Exception as exc:                           # reported in the line, not swallowed
        peer_error = f"{type(exc).__name__}: {exc}"[:200]
    ok_t = torch.tensor([0.0 if g is None else 1.0], device=dev)
    dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
    if ok_t.item() < 1.0:
        if g is not None:
            g.close(barrier=False)
        dist.barrier(device_ids=[local_rank])          # every rank, mapped or not
        return run_b200_multi_nccl(args, rank, world, local_rank, xs, wq_full, sw_full, bias_full,
                                   peer_error or "a peer rank could not map the gather buffers")

    def barrier():
        dist.barrier(device_ids=[local_rank])

    def gather_step(i, w_rows, sw_rows, b_rows, n_total, col0):
        s = i % args.sets
        epoch, slot = g.next_slot()
        st = lib.b2_quant_linear_gather(nat.KIND_I8, xs[s].data_ptr(), nat.F16, M, K, K, ROT,
                                        w_rows[s].data_ptr(), K, w_rows[s].shape[0], sw_rows.data_ptr(),
                                        sw_rows.numel(), b_rows.data_ptr(), nat.F16, nat.EPI_SEPARATE, nat.F16,
                                        n_total, col0, world, rank, g.outs[slot], g.states, epoch,
                                        ws.data_ptr(), ws_bytes, sptr)
        if st:
            nat.check(st, "b2_quant_linear_gather")
        g.wait(epoch, sptr)
        return slot

    def gather_step_ce(i, w_rows, sw_rows, b_rows, n_total, col0, chunks):
        s = i % args.sets
        _, slot = g.next_slot()
        st = lib.b2_quant_linear_gather_ce(nat.KIND_I8, xs[s].data_ptr(), nat.F16, M, K, K, ROT,
                                           w_rows[s].data_ptr(), K, w_rows[s].shape[0], sw_rows.data_ptr(),
                                           sw_rows.numel(), b_rows.data_ptr(), nat.F16, nat.EPI_SEPARATE, nat.F16,
                                           n_total, col0, world, rank, g.outs[slot], g.states, chunks,
                                           ws.data_ptr(), ws_bytes, sptr)
        if st:
            nat.check(st, "b2_quant_linear_gather_ce")
        nat.check(lib.b2_gather_wait_ce(g.state.data_ptr(), world, rank, sptr), "b2_gather_wait_ce")
        return slot

    def strong(i):
        if args.gather == "ce":
            return gather_step_ce(i, wqs, sw, bias, N, c0, ce_chunks(world))
        return gather_step(i, wqs, sw, bias, N, c0)

    def timed(fn, steps, sample_clocks=False):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(local_rank) if sample_clocks else None
        if sampler:
            sampler.__enter__()
        t_wall = time.perf_counter()
        e0.record(stream)
        for i in range(steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
        if sampler:
            sampler.__exit__()
        barrier()
        return _max_over_ranks(torch, dist, dev, e0.elapsed_time(e1) / steps), t_wall, sampler

    # ---- correctness once: every rank holds the whole single-GPU result
    ref = rdna2_ops.w8a8_linear(xs[0], wq_full, sw_full, bias_full, rotation_block=ROT, out_dtype=torch.float16)
    for check in (lambda: gather_step(0, wqs, sw, bias, N, c0),
                  lambda: gather_step_ce(0, wqs, sw, bias, N, c0, ce_chunks(world))):
        slot = check()
        torch.cuda.synchronize()
        got = g.local[slot][: M * N].view(M, N)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), "gathered output differs from 1-GPU linear"
        g.local[slot].fill_(0)
        barrier()
    del ref, wq_full
    for i in range(max(3, args.warmup)):
        strong(i)
    torch.cuda.synchronize()
    nat.device_status(reset=True)

    # ---- timed region: K strong-scaling steps, gather inside
    ms, t_wall, clocks = timed(strong, args.steps, sample_clocks=True)
    value = 2.0 * M * N * K / (ms * 1e-3) / 1e12

    # ---- side figures (same discipline, fewer steps)
    n_side = max(20, min(args.steps, 200))
    out_local = torch.empty((M, ns), device=dev, dtype=torch.float16)

    def local(i):
        s = i % args.sets
        nat.check(lib.b2_quant_linear(nat.KIND_I8, xs[s].data_ptr(), nat.F16, M, K, K, ROT, wqs[s].data_ptr(), K, ns,
                                      sw.data_ptr(), ns, bias.data_ptr(), nat.F16, nat.EPI_SEPARATE,
                                      out_local.data_ptr(), nat.F16, ns, ws.data_ptr(), ws_bytes, sptr),
                  "b2_quant_linear")

    for i in range(3):
        local(i)
    local_ms, _, _ = timed(local, n_side)
    gathered = torch.empty((world * M, ns), device=dev, dtype=torch.float16)

    def nccl(i):
        local(i)
        dist.all_gather_into_tensor(gathered, out_local)

    for i in range(3):
        nccl(i)
    nccl_ms, _, _ = timed(nccl, n_side)
    del gathered
    # link bandwidth in this run: every rank copies its [M, N/P] block into the
    # same columns of every peer's full output with the copy engines (one 2-D
    # copy per peer, each on its own stream) -- the gather's traffic without
    # the GEMM
    slot = 0
    peer_streams = [torch.cuda.Stream(dev) for _ in range(world - 1)]
    src_ptr = g.outs[slot][rank] + c0 * 2

    def ce_gather(i):
        ev = torch.cuda.Event()
        ev.record(stream)
        j = 0
        for q in range(world):
            if q == rank:
                continue
            st_ = peer_streams[j]
            st_.wait_event(ev)
            nat.check(lib.b2_peer_copy_2d(g.outs[slot][q] + c0 * 2, N * 2, src_ptr, N * 2, ns * 2, M,
                                          st_.cuda_stream), "b2_peer_copy_2d")
            stream.wait_stream(st_)
            j += 1

    for i in range(3):
        ce_gather(i)
    ce_ms, _, _ = timed(ce_gather, max(10, n_side // 4))
    # the other gather variant's step, and the copy-engine step by chunk count
    other = {}
    for store in ("sm", "tma"):
        set_gather_store(store)
        for i in range(3):
            gather_step(i, wqs, sw, bias, N, c0)
        other[f"fused_gather_step_ms_{store}_stores"], _, _ = timed(lambda i: gather_step(i, wqs, sw, bias, N, c0),
                                                                   n_side)
    set_gather_store(args.gather_store)
    for ch in (1, 2, 4, 8):
        def step_ch(i, ch=ch):
            return gather_step_ce(i, wqs, sw, bias, N, c0, ch)
        for i in range(3):
            step_ch(i)
        other[f"ce_gather_step_ms_chunks{ch}"], _, _ = timed(step_ch, n_side)
    # end to end: X uploaded to every rank, the rank's columns computed by the
    # public call and read back over the rank's own PCIe link; the host holds
    # Y by column shards (no device gather: the consumer is the host)
    e2e_ms = e2e_pipeline(torch, dev, stream, xs,
                          lambda xd: rdna2_ops.w8a8_linear(xd, wq, sw, bias, rotation_block=ROT,
                                                           out_dtype=torch.float16, workspace=ws),
                          (M, ns), max(10, min(100, args.steps // 5)), barrier)
    e2e_ms = _max_over_ranks(torch, dist, dev, e2e_ms)
    # weak scaling: a 12288-column shard per rank of a (12288 * P)-column layer
    gen_w = torch.Generator(device=dev)
    gen_w.manual_seed(SEED + 1 + rank)
    w = torch.randn((N, K), generator=gen_w, device=dev) * 0.02
    wq_w, sw_w = qlinear.quantize_weight(w, rotation_block=ROT)
    del w
    b_w = (torch.randn(N, generator=gen_w, device=dev) * 0.02).half()
    wq_ws = [wq_w] + [wq_w.clone() for _ in range(args.sets - 1)]
    del wqs

    def weak(i):
        return gather_step(i, wq_ws, sw_w, b_w, N * world, rank * N)

    for i in range(3):
        weak(i)
    weak_ms, _, _ = timed(weak, n_side)
    del wq_ws
    status = nat.device_status()
    g.close()
    if rank != 0:
        return
    pk = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]
    nvlink_gbs = 770.0
    recv = (world - 1) * M * ns * 2                   # bytes every rank must receive per step
    if args.gather == "ce":
        rows = -(-(-(-M // ce_chunks(world))) // 256) * 256
        n_chunks = -(-M // rows)
        launches = 2 * n_chunks + (world - 1) + 1     # prologue + GEMM per chunk, a signal per peer, the wait
        gather_desc = (f"copy engines: the linear in {n_chunks} M-chunks, one 2-D copy per peer and chunk on "
                       "per-peer copy streams overlapping the next chunk's GEMM, counter signal + bounded wait")
    else:
        launches = 3                                  # prologue, GEMM with peer-store epilogue, wait
        gather_desc = ("fused: peer copies from the GEMM epilogue ("
                       + ("TMA stores" if args.gather_store == "tma" else "SM stores")
                       + ") + epoch flags + bounded wait")
    t_gemm = 2.0 * M * ns * K / (int8_peak * 1e12) * 1e3
    t_link = recv / (nvlink_gbs * 1e9) * 1e3
    target = max(t_gemm, t_link)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": c2_config(world, args.sets),
        "roofline": {"bound": "nvlink" if t_link >= t_gemm else "tensor", "achieved_ms": round(ms, 5),
                     "target_ms": round(target, 5), "frac": round(target / ms, 4),
                     "nvlink_bytes_received_per_rank": recv, "nvlink_gbs_ref": nvlink_gbs,
                     "gemm_floor_ms": round(t_gemm, 5), "link_floor_ms": round(t_link, 5),
                     "note": "fused compute+collective: target = max(ops / measured INT8 peak, bytes each rank "
                             "receives / 770 GB/s measured peer bandwidth)"},
        "cpu_baseline": None,
        "e2e": {"value": round(2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, 3), "unit": UNIT,
                "h2d_bytes_per_step": M * K * 2 * world, "d2h_bytes_per_step": M * N * 2,
                "api": "rdna2_ops.w8a8_linear on each rank's shard (C ABI b2_quant_linear); pinned host X to "
                       "every GPU, each rank's N/P columns back over its own PCIe link; uploads / linear / "
                       "read-backs on three streams, double buffered",
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": launches * args.steps,
        "gather": gather_desc,
        "clocks": clocks.summary(),
        "device_status": status,
        "wall_s_timed": round(t_wall, 4),
        "side": {
            "local_linear_only_ms": round(local_ms, 5),
            "local_linear_only_tops": round(world * 2.0 * M * ns * K / (local_ms * 1e-3) / 1e12, 2),
            "nccl_allgather_step_ms": round(nccl_ms, 5),
            "nccl_allgather_step_tops": round(2.0 * M * N * K / (nccl_ms * 1e-3) / 1e12, 2),
            "nccl_note": "local linear + all_gather_into_tensor into [P*M, N/P] (no permute), serial",
            "weak_ms": round(weak_ms, 5),
            "weak_tops": round(world * 2.0 * M * N * K / (weak_ms * 1e-3) / 1e12, 2),
            "weak_note": "12288 columns per rank of a 12288*P-column layer, fused gather inside the step",
            "copy_engine_gather_ms": round(ce_ms, 5),
            "copy_engine_gather_gbs_per_rank": round(recv / (ce_ms * 1e-3) / 1e9, 1),
            "copy_engine_note": "each rank's [M, N/P] block copied to every peer's Y by 2-D copy-engine "
                                "copies, one stream per peer, no GEMM: the link bandwidth measured in this run",
            "step_gather_gbs_per_rank": round(recv / (ms * 1e-3) / 1e9, 1),
            **{k_: round(v_, 5) for k_, v_ in other.items()},
            "ce_note": "b2_quant_linear_gather_ce: the linear in M-chunks, each chunk's block copied to every "
                       "peer by the copy engines while the next chunk is multiplied; counter completion",
        },
    }
    print(json.dumps(line), flush=True)


def run_b200_multi_nccl(args, rank, world, local_rank, xs, wq_full, sw_full, bias_full, why):
    """N > 1 when the fused peer gather is unavailable: the rank-local fused
    linear followed by one NCCL all-gather of the shard outputs inside every
    step (strong scaling), checked against the 1-GPU linear first."""
    import torch
    import torch.distributed as dist
    import rdna2_ops
    from rdna2_ops import _native as nat

    dev = torch.device("cuda", local_rank)
    lib = nat.library()
    stream = torch.cuda.current_stream(dev)
    ns = N // world
    c0 = rank * ns
    wq = wq_full[c0:c0 + ns].contiguous()
    sw = sw_full[c0:c0 + ns].contiguous()
    bias = bias_full[c0:c0 + ns].contiguous()
    wqs = [wq] + [wq.clone() for _ in range(args.sets - 1)]
    ws_bytes = lib.b2_quant_linear_workspace_bytes(M, K)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    out_local = torch.empty((M, ns), device=dev, dtype=torch.float16)
    gathered = torch.empty((world * M, ns), device=dev, dtype=torch.float16)

    def step(i):
        s = i % args.sets
        nat.check(lib.b2_quant_linear(nat.KIND_I8, xs[s].data_ptr(), nat.F16, M, K, K, ROT, wqs[s].data_ptr(), K, ns,
                                      sw.data_ptr(), ns, bias.data_ptr(), nat.F16, nat.EPI_SEPARATE,
                                      out_local.data_ptr(), nat.F16, ns, ws.data_ptr(), ws_bytes, stream.cuda_stream),
                  "b2_quant_linear")
        dist.all_gather_into_tensor(gathered, out_local)

    step(0)
    torch.cuda.synchronize()
    ref = rdna2_ops.w8a8_linear(xs[0], wq_full, sw_full, bias_full, rotation_block=ROT, out_dtype=torch.float16)
    full = gathered.view(world, M, ns).permute(1, 0, 2).reshape(M, N)
    assert torch.equal(full.view(torch.int16), ref.view(torch.int16)), "gathered output differs from 1-GPU linear"
    del ref, full
    for i in range(max(3, args.warmup)):
        step(i)
    dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    dist.barrier(device_ids=[local_rank])
    ms = _max_over_ranks(torch, dist, dev, e0.elapsed_time(e1) / args.steps)
    status = nat.device_status()
    if rank != 0:
        return
    recv = (world - 1) * M * ns * 2
    cfg = c2_config(world, args.sets)
    cfg["parallelism"] = f"column-parallel N-shard x{world}, NCCL all-gather of the shard outputs ([P, M, N/P])"
    line = {"metric": METRIC, "value": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": cfg,
            "roofline": {"bound": "nvlink", "achieved_ms": round(ms, 5),
                         "link_floor_ms": round(recv / 770e9 * 1e3, 5),
                         "frac": round(recv / 770e9 * 1e3 / ms, 4)},
            "cpu_baseline": None, "e2e": None, "gpu_launches": 2 * args.steps, "clocks": clocks.summary(),
            "device_status": status, "fused_gather_unavailable": why}
    print(json.dumps(line), flush=True)


def run_c5_multi(args, rank, world, local_rank):
    """Config 5 on P GPUs: the 28-block DiT linear stack column-parallel, every
    layer output reassembled on every rank inside the GEMM epilogue (fused
    gather) before the next linear reads it.  One step = the whole stack."""
    import torch
    import torch.distributed as dist
    from rdna2_ops import _native as nat
    from rdna2_ops import qlinear
    from rdna2_ops.column_parallel import (ActivationExchange, ColumnParallelStack, PeerGather, ce_chunks,
                                           set_gather_store)

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    set_gather_store(args.gather_store)
    stream = torch.cuda.current_stream(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    m, hid, nblocks = 8192, 3072, 28
    shapes = ((3 * hid, hid), (hid, hid), (4 * hid, hid), (hid, 4 * hid))
    blocks = []
    for _ in range(nblocks):
        blk = []
        for n_, k_ in shapes:
            w = torch.randn((n_, k_), generator=gen, device=dev) * (1.0 / k_ ** 0.5)
            blk.append(qlinear.quantize_weight(w, rotation_block=ROT))
            del w
        blocks.append(blk)
    x0 = torch.randn((m, hid), generator=gen, device=dev).half()
    g = PeerGather(m * 4 * hid, torch.float16)
    ex = None
    if args.activations == "int8":
        ex = ActivationExchange(m, 4 * hid, fused=not args.exchange_two_launch)
        stack = ColumnParallelStack(blocks, peers=g, activations="int8", codes=ex)
    else:
        stack = ColumnParallelStack(blocks, peers=g, gather="ce" if args.gather == "ce" else "peer")
    del blocks
    torch.cuda.empty_cache()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, args.warmup)):
        y = stack(x0)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y).all()), "stack output not finite"
    nat.device_status(reset=True)
    steps = max(3, min(args.steps, 30))
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for _ in range(steps):
            stack(x0)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        ms = _max_over_ranks(torch, dist, dev, ms)
    status = nat.device_status()
    if ex is not None:
        ex.close()
    g.close()
    if rank != 0:
        return
    flops = 2.0 * m * sum(n_ * k_ for n_, k_ in shapes) * nblocks
    recv = (world - 1) / world * m * sum(n_ for n_, _ in shapes) * 2 * nblocks
    if args.activations == "int8":
        # the next layer's input columns as int8 (Q third, h, 4h, h per block; the last layer's fp16 output)
        # plus the per-row absmax slots
        cols = (hid + hid + 4 * hid + hid) * nblocks - hid
        recv = (world - 1) / world * m * cols + (world - 1) / world * m * hid * 2 \
            + (world - 1) * m * 4 * (4 * nblocks - 1)
        stack_launches = 1 + (5 if args.exchange_two_launch else 3) * (4 * nblocks - 1) + 2
    elif args.gather == "ce":
        rows = -(-(-(-m // ce_chunks(world))) // 256) * 256
        stack_launches = 4 * nblocks * (2 * -(-m // rows) + (world - 1 if world > 1 else 0) + 1)
    else:
        stack_launches = 3 * 4 * nblocks
    line = {"workload": "c5", "metric": "W8A8 DiT stack TOPS (config 5, 28 blocks, rotated)",
            "value": round(flops / (ms * 1e-3) / 1e12, 2), "unit": "TOPS", "n_gpus": world, "steps": steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "dtype": "int8", "data": "synthetic",
            "config": {"M": m, "hidden": hid, "blocks": nblocks,
                       "linears": "QKV 9216x3072, out 3072x3072 (on the Q third), up 12288x3072, down 3072x12288, "
                                  "block-128 rotation, every weight N-sharded over the ranks",
                       "parallelism": f"column-parallel x{world}, " + (
                           "only the next layer's input exchanged, as INT8 codes (slice rotation + per-row absmax "
                           "exchange + quantize into every rank's code buffer); the last output gathered in fp16"
                           if args.activations == "int8" else
                           "every layer output gathered to every rank "
                           + ("by copy engines overlapping a chunked GEMM" if args.gather == "ce"
                              else "inside the GEMM epilogue (NVLink peer stores)"))},
            "roofline": {"bound": "nvlink", "nvlink_bytes_received_per_rank": int(recv),
                         "link_floor_ms": round(recv / 770e9 * 1e3, 3),
                         "gemm_floor_ms": round(flops / world / (2.0 * peaks()["bf16_tflops"] * 1e12) * 1e3, 3),
                         "frac": round(max(recv / 770e9 * 1e3,
                                           flops / world / (2.0 * peaks()["bf16_tflops"] * 1e12) * 1e3) / ms, 4)},
            "gpu_launches": stack_launches * steps, "gather": args.gather, "activations": args.activations,
            "exchange": None if args.activations != "int8" else (
                "two launches per layer" if args.exchange_two_launch else "one cooperative launch per layer"),
            "gather_store": args.gather_store if args.gather != "ce" else None, "clocks": clocks.summary(),
            "device_status": status,
            "timing": "eager public ColumnParallelStack calls"}
    print(json.dumps(line), flush=True)


def _raw_linear_step(nat, rdna2_ops, torch, dev, xs, wqs, sw, bias, m, n, k, block, kind, x_dtype, out_dtype,
                     public):
    """The C-ABI call the public linear makes (b2_quant_linear), checked bit
    for bit against the public call once, for graph-replayed timing."""
    lib = nat.library()
    sets = len(xs)
    ws_bytes = lib.b2_quant_linear_workspace_bytes(m, k)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    outs = [torch.empty((m, n), device=dev, dtype=out_dtype) for _ in range(sets)]

    def step(i):
        j = i % sets
        nat.check(lib.b2_quant_linear(kind, xs[j].data_ptr(), nat.DTYPE_CODE[x_dtype], m, k, k, block or 0,
                                      wqs[j].data_ptr(), k, n, sw.data_ptr(), sw.numel(),
                                      bias.data_ptr() if bias is not None else None,
                                      nat.DTYPE_CODE[bias.dtype] if bias is not None else 0, nat.EPI_SEPARATE,
                                      outs[j].data_ptr(), nat.DTYPE_CODE[out_dtype], n, ws.data_ptr(), ws_bytes,
                                      nat.stream_ptr(dev)), "b2_quant_linear")
    ref = public(xs[0], wqs[0])
    step(0)
    torch.cuda.synchronize()
    assert torch.equal(outs[0].view(torch.int16), ref.view(torch.int16)), "raw C-ABI call differs from public call"
    return step, True


def torch_cpu_int4_baseline(m, n, k, budget_s, threads):
    """The reference's PyTorch CPU path for W4A16 (int4_linear_a16 method
    "dequant": unpack_int4_cpu of the pack, then F.linear in bf16,
    rdna2_ops/int4_weight_gemm_v07.py:49-92, 540-564) on a bounded row sample."""
    import torch
    from rdna2_ops import int4_weight_gemm_v07 as i4
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(SEED)
        p = i4.pack_int4_cpu(torch.randn((n, k), generator=g) * 0.02, group_size=128, symmetric=False)
        rows = m

        def run(r):
            a = torch.randn((r, k), generator=g).to(torch.bfloat16)
            t0 = time.perf_counter()
            w = i4.unpack_int4_cpu(p).to(torch.bfloat16)
            torch.nn.functional.linear(a, w)
            return time.perf_counter() - t0

        run(1)
        t1 = run(min(m, 16))
        if m > 16 and t1 * m / 16 > budget_s:
            rows = max(16, int(budget_s / t1 * 16) // 16 * 16)
        dt = min(run(rows), run(rows))
    finally:
        torch.set_num_threads(prev)
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"unpack_int4_cpu + F.linear bf16 (method 'dequant') on {rows} of {m} rows, N={n} K={k}, "
                      f"{dt * 1e3:.1f} ms, {threads} torch threads"}


def torch_cpu_fp8_baseline(m, n, k, budget_s, threads):
    """The reference's PyTorch CPU math for the FP8 weight GEMM (the "upcast"
    method, F.linear on the decoded weight, rdna2_ops/fp8_weight_gemm_v06.py
    :166-167) with config 4's scales: per-token e4m3 activations and
    per-channel e4m3 weights, dequantized to bf16, then F.linear."""
    import torch
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(SEED)
        w = torch.randn((n, k), generator=g) * 0.02
        sw = w.abs().amax(1, keepdim=True) / 448.0
        wq = (w / sw).to(torch.float8_e4m3fn)
        rows = m

        def run(r):
            a = torch.randn((r, k), generator=g).to(torch.bfloat16)
            t0 = time.perf_counter()
            sa = a.float().abs().amax(1, keepdim=True) / 448.0
            aq = (a.float() / sa).to(torch.float8_e4m3fn)
            torch.nn.functional.linear((aq.to(torch.bfloat16) * sa.to(torch.bfloat16)),
                                       (wq.to(torch.bfloat16) * sw.to(torch.bfloat16)))
            return time.perf_counter() - t0

        run(1)
        t1 = run(min(m, 16))
        if m > 16 and t1 * m / 16 > budget_s:
            rows = max(16, int(budget_s / t1 * 16) // 16 * 16)
        dt = min(run(rows), run(rows))
    finally:
        torch.set_num_threads(prev)
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"e4m3 per-token / per-channel quantize, dequantize to bf16, F.linear on {rows} of {m} rows, "
                      f"N={n} K={k}, {dt * 1e3:.1f} ms, {threads} torch threads"}


# The reference's measured MOSS linear shapes (M = 1061 tokens) and its
# published RX 6900 XT times for "fused INT8 GEMM + FP32 dequant" and the
# row-quantizer + fused GEMM pipeline (rdna2-ops/RDNA2_OPTIMIZATION_GUIDE_KO.md
# :1135-1138; results/int8_gemm_moss_shapes_v05.json).
MOSS_SHAPES = ((1061, 3072, 3072, 0.698), (1061, 9216, 3072, 1.869), (1061, 16384, 3072, 3.302),
               (1061, 3072, 8192, 1.932))


def run_moss(args):
    """One line per MOSS shape: the INT8 GEMM with the fp32 dequant epilogue
    on pre-quantized operands (int8_gemm_dequant's C-ABI call, b2_qgemm) and
    the whole linear from fp32 activations (ConvRot 256 + row quantization +
    GEMM, b2_quant_linear), each a CUDA graph of C-ABI calls with operands
    cycled over copies larger than L2."""
    import torch
    import rdna2_ops
    from rdna2_ops import _native as nat
    from rdna2_ops import qlinear

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = nat.library()
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    for m, n, k, ref_ms in MOSS_SHAPES:
        sets = max(4, int(200e6 // (n * k + m * k * 4)) + 1)
        xs = [torch.randn((m, k), generator=gen, device=dev) for _ in range(sets)]
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        wq, sw = qlinear.quantize_weight(w, rotation_block=256)
        del w
        wqs = [wq.clone() for _ in range(sets)]
        qa = [rdna2_ops.act_quant(x, rotation_block=256) for x in xs]
        out = torch.empty((m, n), device=dev, dtype=torch.float32)
        ws_bytes = lib.b2_quant_linear_workspace_bytes(m, k)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        ref = rdna2_ops.int8_gemm_dequant(qa[0][0], wqs[0].T, qa[0][1], sw)

        def gemm(i):
            j = i % sets
            nat.check(lib.b2_qgemm(nat.KIND_I8, qa[j][0].data_ptr(), k, wqs[j].data_ptr(), k, m, n, k,
                                   qa[j][1].data_ptr(), sw.data_ptr(), n, None, 0, nat.EPI_SEPARATE,
                                   out.data_ptr(), nat.F32, n, nat.stream_ptr(dev)), "b2_qgemm")

        def linear(i):
            j = i % sets
            nat.check(lib.b2_quant_linear(nat.KIND_I8, xs[j].data_ptr(), nat.F32, m, k, k, 256, wqs[j].data_ptr(),
                                          k, n, sw.data_ptr(), n, None, 0, nat.EPI_SEPARATE, out.data_ptr(),
                                          nat.F32, n, ws.data_ptr(), ws_bytes, nat.stream_ptr(dev)),
                      "b2_quant_linear")

        gemm(0)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32)), "raw GEMM differs from int8_gemm_dequant"
        times = {}
        for name, fn in (("gemm", gemm), ("linear", linear)):
            for i in range(3):
                fn(i)
            per = 4 * sets
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(per):
                    fn(i)
            graph.replay()
            torch.cuda.synchronize()
            if name == "gemm":   # the replayed graph really computes the product
                assert torch.equal(out.view(torch.int32), rdna2_ops.int8_gemm_dequant(
                    qa[(per - 1) % sets][0], wqs[(per - 1) % sets].T, qa[(per - 1) % sets][1], sw).view(torch.int32))
            reps = max(1, args.steps // per)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(0) as clocks:
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                torch.cuda.synchronize()
            times[name] = (e0.elapsed_time(e1) / (reps * per), reps * per, clocks.summary())
            del graph
        g_ms, l_ms = times["gemm"][0], times["linear"][0]
        ops = 2.0 * m * n * k
        line = {"workload": f"moss m{m} n{n} k{k}", "metric": "INT8 GEMM + FP32 dequant TOPS (MOSS shape)",
                "value": round(ops / (g_ms * 1e-3) / 1e12, 2), "unit": "TOPS", "n_gpus": 1,
                "steps": times["gemm"][1], "warmup": 3, "ms_per_step": round(g_ms, 5), "higher_is_better": True,
                "dtype": "int8", "data": "synthetic",
                "config": {"M": m, "N": n, "K": k, "out": "fp32", "l2": f"operands cycled over {sets} copies"},
                "pipeline": {"ms_per_step": round(l_ms, 5), "tops": round(ops / (l_ms * 1e-3) / 1e12, 2),
                             "what": "fp32 x -> ConvRot 256 + per-token INT8 + GEMM + fp32 dequant (b2_quant_linear)"},
                "roofline": {"bound": "tensor", "achieved": round(ops / (g_ms * 1e-3) / 1e12, 1),
                             "peak": round(2.0 * pk["bf16_tflops"], 1), "unit": "TOPS",
                             "frac": round(ops / (g_ms * 1e-3) / 1e12 / (2.0 * pk["bf16_tflops"]), 4)},
                "reference_published_ms_rx6900xt": ref_ms,
                "gpu_launches": times["gemm"][1], "clocks": times["gemm"][2], "timing": "cuda graph of C-ABI calls",
                "device_status": nat.device_status()}
        print(json.dumps(line), flush=True)
        del xs, wqs, qa


def run_workload(args):
    """Configs 1, 3 and 4 of the benchmark plan on one GPU: one JSON line with
    the same timing discipline (warm-up, CUDA events on the launch stream,
    weights cycled over enough copies to exceed L2) and a roofline for the
    op's own kernel."""
    import torch
    import rdna2_ops
    from rdna2_ops import _native as nat
    from rdna2_ops import int4_weight_gemm_v07 as i4
    from rdna2_ops import qlinear

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    pk = peaks()
    name = args.workload
    sets = max(args.sets, 8)
    graph_ok = False
    per_graph_override = None
    if name == "c1":
        m, n, k = 1024, 3072, 3072
        xs = [(torch.randn((m, k), generator=gen, device=dev)).half() for _ in range(sets)]
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        wq, sw = qlinear.quantize_weight(w)
        wqs = [wq.clone() for _ in range(sets)]
        bias = (torch.randn(n, generator=gen, device=dev) * 0.02).half()
        step, graph_ok = _raw_linear_step(nat, rdna2_ops, torch, dev, xs, wqs, sw, bias, m, n, k, None,
                                          nat.KIND_I8, torch.float16, torch.float16,
                                          lambda x, w: rdna2_ops.w8a8_linear(x, w, sw, bias, out_dtype=torch.float16))
        metric, flops, launches = "W8A8 INT8 linear TOPS (config 1)", 2.0 * m * n * k, 2
        bound, peak, unit, traffic = "tensor", 2.0 * pk["bf16_tflops"], "TOPS", None
        dtype = "int8"
    elif name.startswith("c3m"):
        m, n, k = int(name[3:]), 14336, 4096
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        wt = i4.quantize_w4a16(w, group_size=128, dtype=torch.bfloat16)
        del w
        wts = [wt] + [wt.clone() for _ in range(sets - 1)]
        xs = [torch.randn((m, k), generator=gen, device=dev).to(torch.bfloat16) for _ in range(sets)]
        lib = nat.library()
        need = lib.b2_w4a16_workspace_bytes(m, n, k, 128)
        ws = torch.zeros(max(need, 16), device=dev, dtype=torch.uint8)  # zero once (arrival counters)
        outs = [torch.empty((m, n), device=dev, dtype=torch.bfloat16) for _ in range(sets)]
        # the public call once, checked against the raw C-ABI call timed below
        ref_out = i4.w4a16_gemm(xs[0], wts[0], workspace=ws)

        def raw_step(i):  # the C-ABI call i4.w4a16_gemm makes, without its host work
            j = i % sets
            nat.check(lib.b2_w4a16_gemm(xs[j].data_ptr(), nat.DTYPE_CODE[torch.bfloat16], k,
                                        wts[j].tiles.data_ptr(), wts[j].groups.data_ptr(), 128, m, n, k,
                                        None, 0, outs[j].data_ptr(), n, ws.data_ptr() if need else None,
                                        need, nat.stream_ptr(dev)), "b2_w4a16_gemm")
        raw_step(0)
        torch.cuda.synchronize()
        assert torch.equal(outs[0].view(torch.int16), ref_out.view(torch.int16))
        step = raw_step
        graph_ok = True
        metric, flops = f"W4A16 GEMM TFLOPS (config 3, M={m})", 2.0 * m * n * k
        launches = 2 if need else 1
        traffic = n * k // 2 + 2 * n * (k // 128) * 2 + m * k * 2 + m * n * 2
        # the bound follows the arithmetic intensity against the bf16 ridge
        # (peak FLOP/s over HBM bytes/s): M = 128 is ~480 FLOP/B, tensor-bound
        if flops / traffic < pk["bf16_tflops"] * 1e12 / (pk["hbm_gbs"] * 1e9):
            bound, peak, unit = "hbm", pk["hbm_gbs"], "GB/s"
        else:
            bound, peak, unit = "tensor", pk["bf16_tflops"], "TFLOP/s"
        dtype = "bf16"
    elif name.startswith("w4a8m"):
        # W4A8 (int4_linear_a8) at the config-3 weight shape: int8 A [M,4096]
        # with per-row scales, uint4 g128 affine W [14336,4096], fp32 out.
        m, n, k = int(name[5:]), 14336, 4096
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        wt = i4.prepare_w4a8(i4.pack_int4(w, group_size=128, symmetric=False))
        del w
        wts = [wt] + [i4.W4A8Weight(wt.tiles.clone(), wt.groups.clone(), n, k, 128) for _ in range(sets - 1)]
        xs = [torch.randint(-128, 128, (m, k), generator=gen, device=dev, dtype=torch.int8) for _ in range(sets)]
        sa = torch.rand(m, generator=gen, device=dev) * 0.02 + 0.001
        lib = nat.library()
        need = lib.b2_w4a8_workspace_bytes(m, k, 128)
        ws = torch.empty(max(need, 256), device=dev, dtype=torch.uint8)
        outs = [torch.empty((m, n), device=dev, dtype=torch.float32) for _ in range(sets)]
        ref_out = i4.int4_linear_a8(xs[0], None, sa, prepared=wts[0])

        def raw_step(i):  # the C-ABI call int4_linear_a8 makes, without its host work
            j = i % sets
            nat.check(lib.b2_w4a8_gemm(xs[j].data_ptr(), k, wts[j].tiles.data_ptr(), wts[j].groups.data_ptr(), 128,
                                       m, n, k, sa.data_ptr(), None, 0, 0, outs[j].data_ptr(), n, ws.data_ptr(),
                                       ws.numel(), nat.stream_ptr(dev)), "b2_w4a8_gemm")
        raw_step(0)
        torch.cuda.synchronize()
        assert torch.equal(outs[0].view(torch.int32), ref_out.view(torch.int32))
        step, graph_ok = raw_step, True
        metric, flops = f"W4A8 GEMM TOPS (config-3 shape, M={m})", 2.0 * m * n * k
        launches = 2
        traffic = n * k // 2 + n * (k // 128) * 8 + m * k + m * n * 4
        if flops / traffic < 2.0 * pk["bf16_tflops"] * 1e12 / (pk["hbm_gbs"] * 1e9):
            bound, peak, unit = "hbm", pk["hbm_gbs"], "GB/s"
        else:
            bound, peak, unit = "tensor", 2.0 * pk["bf16_tflops"], "TOPS"
        dtype = "int8"
    elif name.startswith("c4m"):
        m, n, k = int(name[3:]), 5120, 5120
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        wq, sw = qlinear.quantize_weight(w, quant="e4m3")
        wqs = [wq.clone() for _ in range(sets)]
        xs = [torch.randn((m, k), generator=gen, device=dev).to(torch.bfloat16) for _ in range(sets)]
        step, graph_ok = _raw_linear_step(nat, rdna2_ops, torch, dev, xs, wqs, sw, None, m, n, k, None,
                                          nat.KIND_E4M3, torch.bfloat16, torch.bfloat16,
                                          lambda x, w: rdna2_ops.fp8_linear(x, w, sw, out_dtype=torch.bfloat16))
        metric, flops, launches = f"FP8 e4m3 linear TFLOPS (config 4, M={m})", 2.0 * m * n * k, 2
        traffic = n * k + n * 4 + m * k * 2 + m * n * 2
        if m <= 32:  # decode sizes stream the weights: HBM-bound
            bound, peak, unit = "hbm", pk["hbm_gbs"], "GB/s"
        else:
            bound, peak, unit = "tensor", 2.0 * pk["bf16_tflops"], "TFLOP/s"
        dtype = "e4m3"
    elif name == "c5":
        # Config 5: 28 DiT blocks, hidden 3072, MLP ratio 4, every linear W8A8
        # with block-128 rotation; fp16 activations [8192, 3072] ~N(0,1).
        # Linears only (attention is not on the path): QKV, then the out
        # projection on the Q third (a strided view, row stride 9216), up,
        # down; the down output feeds the next block.  Weights ~N(0, 1/K)
        # keep the activations O(1) through the 28 blocks.  One step = the
        # whole stack, 112 fused linears; 3.2 GB of int8 weights (> L2).
        m, hid, blocks = 8192, 3072, 28
        shapes = ((3 * hid, hid), (hid, hid), (4 * hid, hid), (hid, 4 * hid))
        layers = []
        for _ in range(blocks):
            blk = []
            for n_, k_ in shapes:
                w = torch.randn((n_, k_), generator=gen, device=dev) * (1.0 / k_ ** 0.5)
                wq, sw = qlinear.quantize_weight(w, rotation_block=ROT)
                blk.append((wq, sw, n_, k_))
                del w
            layers.append(blk)
        x0 = torch.randn((m, hid), generator=gen, device=dev).half()
        bufs = {"qkv": torch.empty((m, 3 * hid), device=dev, dtype=torch.float16),
                "o": torch.empty((m, hid), device=dev, dtype=torch.float16),
                "h": torch.empty((m, 4 * hid), device=dev, dtype=torch.float16),
                "x": torch.empty((m, hid), device=dev, dtype=torch.float16)}
        lib = nat.library()
        ws_bytes = lib.b2_quant_linear_workspace_bytes(m, 4 * hid)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        # (input, its row stride, output) per linear of a block
        wiring = ((None, hid, "qkv"), ("qkv", 3 * hid, "o"), ("o", hid, "h"), ("h", 4 * hid, "x"))

        def raw_linear(x_ptr, ldx, wq, sw, n_, k_, out):
            nat.check(lib.b2_quant_linear(nat.KIND_I8, x_ptr, nat.F16, m, k_, ldx, ROT, wq.data_ptr(), k_, n_,
                                          sw.data_ptr(), sw.numel(), None, 0, nat.EPI_SEPARATE, out.data_ptr(),
                                          nat.F16, n_, ws.data_ptr(), ws_bytes, nat.stream_ptr(dev)),
                      "b2_quant_linear")

        def step(i):
            for b, blk in enumerate(layers):
                for (src, ldx, dst), (wq, sw, n_, k_) in zip(wiring, blk):
                    x = (x0 if b == 0 else bufs["x"]) if src is None else bufs[src]
                    raw_linear(x.data_ptr(), ldx, wq, sw, n_, k_, bufs[dst])

        # the public call on the first QKV and on the strided out-projection
        # input, against the raw calls the stack makes
        wq, sw, n_, k_ = layers[0][0]
        ref = rdna2_ops.w8a8_linear(x0, wq, sw, None, rotation_block=ROT, out_dtype=torch.float16)
        raw_linear(x0.data_ptr(), hid, wq, sw, n_, k_, bufs["qkv"])
        torch.cuda.synchronize()
        assert torch.equal(bufs["qkv"].view(torch.int16), ref.view(torch.int16)), "raw QKV differs from public call"
        wq, sw, n_, k_ = layers[0][1]
        ref = rdna2_ops.w8a8_linear(bufs["qkv"][:, :hid], wq, sw, None, rotation_block=ROT, out_dtype=torch.float16)
        raw_linear(bufs["qkv"].data_ptr(), 3 * hid, wq, sw, n_, k_, bufs["o"])
        torch.cuda.synchronize()
        assert torch.equal(bufs["o"].view(torch.int16), ref.view(torch.int16)), "raw out-proj differs from public call"
        step(0)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(bufs["x"]).all()), "stack output not finite"
        graph_ok, per_graph_override = True, 1
        metric = "W8A8 DiT stack TOPS (config 5, 28 blocks, rotated)"
        flops = 2.0 * m * sum(n_ * k_ for n_, k_ in shapes) * blocks  # 51.95 TOP
        launches = 2 * 4 * blocks
        bound, peak, unit, traffic = "tensor", 2.0 * pk["bf16_tflops"], "TOPS", None
        dtype = "int8"
        n, k = hid, hid
    else:
        raise SystemExit(f"unknown workload {name}")
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph_ok:
        # Launch-bound small shapes: the timed steps replay one CUDA graph of
        # `per_graph` back-to-back C-ABI calls (cycling the weight copies), so
        # the device time is the kernels' own, not the host's launch rate.
        per_graph = per_graph_override or sets * 4
        replays = max(1, -(-args.steps // per_graph))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(per_graph):
                step(i)
        graph.replay()
        torch.cuda.synchronize()
        steps_timed = replays * per_graph
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for _ in range(replays):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        del graph
    else:
        steps_timed = args.steps
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for i in range(args.steps):
                step(i)
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps_timed
    value = flops / (ms * 1e-3) / 1e12
    if bound == "hbm":
        achieved = traffic / (ms * 1e-3) / 1e9
    else:
        achieved = value
    line = {"workload": name, "metric": metric, "value": round(value, 2), "unit": "TOPS" if dtype == "int8" else "TFLOP/s",
            "n_gpus": 1, "steps": steps_timed, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
            "higher_is_better": True, "dtype": dtype, "data": "synthetic",
            "config": ({"M": m, "hidden": 3072, "blocks": 28, "linears": "QKV 9216x3072, out 3072x3072, "
                        "up 12288x3072, down 3072x12288, block-128 rotation", "l2": "3.2 GB of weights per step"}
                       if name == "c5" else {"M": m, "N": n, "K": k, "l2": f"weights cycled over {sets} copies"}),
            "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
                         "frac": round(achieved / peak, 4), "algorithmic_bytes": traffic,
                         "peak_source": pk["source"]},
            "gpu_launches": launches * steps_timed, "clocks": clocks.summary(),
            "timing": "cuda graph of C-ABI calls" if graph_ok else "eager public API calls",
            "device_status": nat.device_status()}
    if not args.no_cpu_baseline:
        if name.startswith("c3m"):
            line["cpu_baseline"] = torch_cpu_int4_baseline(m, n, k, 0.5 * args.cpu_budget_s, host_threads())
        elif name.startswith("c4m"):
            line["cpu_baseline"] = torch_cpu_fp8_baseline(m, n, k, 0.5 * args.cpu_budget_s, host_threads())
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "moss":
        if rank == 0:
            run_moss(args)
        return
    if args.workload not in ("c2", "c5") or (args.workload == "c5" and world == 1 and not args.column_parallel):
        if rank == 0:
            run_workload(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "c5":
            run_c5_multi(args, rank, world, local_rank)
        elif world > 1:
            run_b200_multi(args, rank, world, local_rank)
        else:
            run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
