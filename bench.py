#!/usr/bin/env python
"""Benchmark of the B200 quantized-linear path (one JSON line on rank 0).

Default workload ``decode``: every decode product the benchmark
configurations name, one step = all of them, each with its own weight copy:
  * Q8_0 4096x4096, M = 1 (the single-linear configuration);
  * Llama-3-8B FFN: Q4_0 and Q4_1 gate/up W 14336x4096 and down W 4096x14336,
    M = 1, 4 and 16 (the configuration the metric is quoted on);
  * 70B shapes: Q4_0 gate/up W 28672x8192 and down W 8192x28672, and the Q8_0
    lm_head W 128256x8192, M = 1 and 32 (the row-sharded configuration).
Weights ~N(0, 0.02) packed by the bit-exact device quantizer, activations
~N(0, 1) F32. A step streams 3.7 GB of distinct packed weights (inputs far
larger than the 126 MB L2), so no launch finds its weights in L2.

Metric: GB/s of algorithmic bytes, N*ceil(K/32)*block_bytes + 4*M*K + 4*M*N
per product (each product counted once, whatever the number of GPUs), over
the whole step.
  value : device time of a CUDA graph holding exactly K steps, weights and
          activations resident in HBM;
  e2e   : through the public API with host buffers: every step copies every
          product's activations from pinned host memory (one host-to-device
          copy of the step's input arena) and every product's outputs back
          (one device-to-host copy) inside the timed region; the copies run on
          copy streams with double-buffered device arenas, overlapping the
          next step's products, as a serving loop does.
At one GPU the line also carries ``prefill``: the ragged prefill GEMM (Q8_0
W 11008x4096 and 4096x11008, 8 requests of 1..512 rows packed to M = 1456)
in TFLOP/s of 2*M*N*K against the measured dense bf16 peak, with its own
roofline and CPU baseline, and ``forward``: a full LLaMA-style forward with
random Q8_0 weights (32 layers, dim 4096, 32 / 8 heads, hidden 14336, vocab
128256; 4 requests x 128 prompt tokens, then 128 greedy decode steps each) in
tokens/s, served by the C++ backend's batched forward
(mini_ai_b200/adapter/forward_bench.cc), with the reference CPU forward timed
on 2 of the 32 layers and extrapolated.

Multi-GPU (torchrun, N ranks): tensor-parallel row sharding with strong
scaling. The global matrices are fixed; rank r holds rows [r*N/G, (r+1)*N/G)
of every matrix and every product ends with the all-gather of the [M, N/G]
output slices over NVLink (mq_linear_sharded_allgather, inside the timed
graph), so every rank holds the full output. value = the products' bytes /
max-over-ranks time.

``--workload llama3_8b_ffn_decode`` (the 8B FFN products alone) and
``--workload prefill_ragged_q8_0`` run one configuration on its own.

``--impl reference`` times the reference's own CPU implementation
(LinearDispatch kThreadedSimd from the reference sources built in
oracle/_ref, else the C port of it) on the same workload, metric and unit:
the reference runs one activation row per call, so each product is timed on
one row and its time scaled by its row count M.
"""
from __future__ import annotations

import argparse
import ctypes as C
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

Q4_0, Q4_1, Q8_0 = 2, 3, 8
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20}
TNAME = {Q8_0: "q8_0", Q4_0: "q4_0", Q4_1: "q4_1"}
METRIC = "quantized linear GB/s & % HBM peak (decode), TFLOP/s (prefill); tokens/s at 1/2/4/8 GPU"

LLAMA8B_FFN = (("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336))
FFN70B = (("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672))


def _group(tag: str, qtypes, ms, mats):
    """(qtype, m, name, n, k, class) for a block of products; the class names the kernel class."""
    return [(q, m, f"{tag}_{name}", n, k, f"{tag}_{TNAME[q]}_m{m}") for q in qtypes for m in ms
            for (name, n, k) in mats]


WORKLOADS = {
    # decode GEMVs of every configuration (the default): GB/s of algorithmic bytes
    "decode": {
        "products": (_group("linear4096", (Q8_0,), (1,), (("linear", 4096, 4096),))
                     + _group("llama3_8b_ffn", (Q4_0, Q4_1), (1, 4, 16), LLAMA8B_FFN)
                     + _group("70b_ffn", (Q4_0,), (1, 32), FFN70B)
                     + _group("70b_lm_head", (Q8_0,), (1, 32), (("lm_head", 128256, 8192),))),
        "unit": "GB/s",
        "desc": ("Q8_0 4096x4096 M=1; Llama-3-8B FFN Q4_0/Q4_1 gate/up 14336x4096, down 4096x14336, M=1/4/16; "
                 "70B FFN Q4_0 gate/up 28672x8192, down 8192x28672 and lm_head Q8_0 128256x8192, M=1/32"),
        "l2": "inputs larger than L2: 3.7 GB of distinct weights per step",
        "cpu_rows": None,
    },
    # the Llama-3-8B FFN decode products alone (the configuration the metric is quoted on)
    "llama3_8b_ffn_decode": {
        "products": _group("llama3_8b_ffn", (Q4_0, Q4_1), (1, 4, 16), LLAMA8B_FFN),
        "unit": "GB/s",
        "desc": "gate/up 14336x4096, down 4096x14336; Q4_0, Q4_1; M = 1, 4, 16",
        "l2": "inputs larger than L2: 627 MB of distinct weights per step",
        "cpu_rows": None,
    },
    # ragged prefill GEMM: 8 requests of {1,7,33,64,128,200,511,512} rows (M = 1456) packed
    # contiguously, Q8_0 W 11008x4096 and 4096x11008: TFLOP/s of 2*M*N*K
    "prefill_ragged_q8_0": {
        "products": [(Q8_0, 1456, "w_up", 11008, 4096, "prefill_q8_0_m1456"),
                     (Q8_0, 1456, "w_down", 4096, 11008, "prefill_q8_0_m1456")],
        "unit": "TFLOP/s",
        "desc": "Q8_0 11008x4096 and 4096x11008; 8 ragged requests, M = 1456",
        "l2": "every product streams 47.9 MB of weights and a 23.9 MB (or 64 MB) activation block",
        "cpu_rows": 8,  # the CPU reference runs prefill row by row: a bounded sample of rows is timed
    },
}


def algo_bytes(q: int, n: int, k: int, m: int) -> int:
    return n * ((k + 31) // 32) * BLOCK_BYTES[q] + 4 * m * k + 4 * m * n


def algo_work(wl: dict, q: int, n: int, k: int, m: int) -> float:
    """The metric's unit of work for one product: bytes (GB/s) or flops (TFLOP/s)."""
    return 2.0 * m * n * k if wl["unit"] == "TFLOP/s" else algo_bytes(q, n, k, m)


def work_rate(wl: dict, work: float, seconds: float) -> float:
    return work / seconds / (1e12 if wl["unit"] == "TFLOP/s" else 1e9)


def products(wl: dict):
    """(qtype, m, name, n, k, class) for every product of one step, in launch order."""
    return list(wl["products"])


def select(prods, only: str | None):
    """Restrict to the products of one kernel class, e.g. ``llama3_8b_ffn_q4_0_m16`` (profiling one class)."""
    if not only:
        return prods
    sel = [p for p in prods if p[5] == only]
    if not sel:
        raise SystemExit(f"no products of class {only!r}; classes: {sorted({p[5] for p in prods})}")
    return sel


def peaks(unit: str = "GB/s") -> tuple[float, str]:
    """HBM GB/s or dense bf16 TFLOP/s (burst) measured on this pool, else the fallback figures."""
    p = ROOT / "MEASURED_PEAKS.json"
    key, fallback = ("bf16_tflops", 1590.0) if unit == "TFLOP/s" else ("hbm_gbs", 6650.0)
    try:
        return float(json.loads(p.read_text())[key]), "measured"
    except Exception:
        return fallback, "fallback"


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (NVML, fast polling in a thread).
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {  # NVML clocks-event-reason bits
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report that no clocks were seen
            self.nvml = None
            self.error = repr(exc)

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception:
                break
            time.sleep(0.002)

    def __enter__(self):
        if self.nvml:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        names = [n for b, n in self.REASONS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": int(statistics.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
class Arm:
    """The products of one workload on this rank: weights (row shard `rank` of
    every matrix when world > 1), activations, outputs and the calls."""

    def __init__(self, args, wl, prods, rank, world, local_rank, torch, mq, comm, keep_host):
        lib = mq.lib()
        dev = torch.device("cuda", local_rank)
        stream = torch.cuda.current_stream(dev)
        sh = C.c_void_p(stream.cuda_stream)
        self.wl, self.prods, self.world = wl, prods, world
        gen = torch.Generator(device=dev)
        self.handles, self.host_blocks = [], []
        for i, (q, m, name, n, k, _) in enumerate(prods):
            if n % world:
                raise SystemExit(f"{name}: {n} rows do not split into {world} equal shards")
            gen.manual_seed(1000 + i)  # the same seed on every rank: the shards form one global matrix
            w32 = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32).mul_(0.02)
            blocks = torch.empty(lib.mq_quantized_bytes(q, n, k), dtype=torch.uint8, device=dev)
            rc = lib.mq_quantize_device(local_rank, q, w32.data_ptr(), n, k, blocks.data_ptr(), blocks.numel(), sh)
            if rc:
                raise RuntimeError(mq._lib.last_error())
            del w32
            r0, r1 = rank * n // world, (rank + 1) * n // world
            self.handles.append(mq.CudaWeight.from_device_blocks(blocks, q, n, k, device=local_rank, stream=stream,
                                                                 row_range=(r0, r1)))
            if keep_host:
                self.host_blocks.append(blocks.cpu().numpy())
            del blocks
        gen.manual_seed(424242)
        self.xs = {(m, k): torch.randn((m, k), generator=gen, device=dev, dtype=torch.float32)
                   for (_, m, _, _, k, _) in prods}
        self.ys = {(m, n): torch.empty((m, n), dtype=torch.float32, device=dev) for (_, m, _, n, _, _) in prods}
        self.calls = [(self.handles[i].handle, self.xs[(m, k)].data_ptr(), m, k, self.ys[(m, n)].data_ptr(), n)
                      for i, (q, m, name, n, k, _) in enumerate(prods)]
        # whole-job algorithmic work: every product once (its full weights, activations and outputs)
        self.work_per_step = sum(algo_work(wl, q, n, k, m) for (q, m, _, n, k, _) in prods)
        if world > 1:
            gather = lib.mq_linear_sharded_allgather

            def linear(h, x, m, k, b, y, n, s):
                return gather(h, x, m, k, b, y, n, comm.handle, s)
        else:
            linear = lib.mq_linear
        self.linear = linear
        self.mq = mq

    def run(self, stream_handle, idx=None):
        for j in (range(len(self.calls)) if idx is None else idx):
            h, x, m, k, y, n = self.calls[j]
            rc = self.linear(h, x, m, k, None, y, n, stream_handle)
            if rc:
                raise RuntimeError(self.mq._lib.last_error())

    def close(self):
        for h in self.handles:
            h.close()


def _graph_ms(torch, cap, cap_h, fn, steps, barrier, max_over_ranks):
    """Device ms of one pass of fn, from a CUDA graph holding `steps` passes
    replayed once untimed and once between two events on the capture stream."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        for _ in range(steps):
            fn(cap_h)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cap):
        g.replay()
        barrier()
        c0.record(cap)
        g.replay()
        c1.record(cap)
        barrier()
    ms = max_over_ranks(c0.elapsed_time(c1) / steps)
    del g
    return ms


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    import mini_ai_b200 as mq
    from mini_ai_b200 import build as mq_build

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if not mq.LIB_PATH.exists():
        mq_build.build()
    lib = mq.lib()
    wl = WORKLOADS[args.workload]
    prods = select(products(wl), args.only)
    stream = torch.cuda.current_stream(dev)
    sh = C.c_void_p(stream.cuda_stream)
    keep_host = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.only
    comm = mq.CudaComm.from_process_group(local_rank) if world > 1 else None
    arm = Arm(args, wl, prods, rank, world, local_rank, torch, mq, comm, keep_host)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(ms):
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # The timed region replays a CUDA graph holding exactly K steps, captured on
    # a dedicated stream after eager warm-up on that stream (so per-stream
    # scratch already exists). Nothing sits between the products inside the
    # graph, so consecutive kernels overlap through programmatic dependent
    # launch as they do in an application's stream.
    cap = torch.cuda.Stream(dev)
    cap_h = C.c_void_p(cap.cuda_stream)
    with torch.cuda.stream(cap):
        for _ in range(args.warmup):
            arm.run(cap_h)
    barrier()
    graph = torch.cuda.CUDAGraph()
    launches0 = lib.mq_kernel_launches()
    with torch.cuda.graph(graph, stream=cap):
        for s in range(args.steps):
            arm.run(cap_h)
    launches = lib.mq_kernel_launches() - launches0  # kernels inside the timed graph
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cap):  # replay, and both timing events, on the capture stream
        graph.replay()  # upload + one untimed pass
        barrier()
        with ClockSampler(local_rank) as clocks:
            barrier()
            t0.record(cap)
            graph.replay()
            t1.record(cap)
            barrier()
    ms_per_step = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    del graph

    # Device time per kernel class: a graph per class holding the class's
    # products K times back to back (the same calls as in the step, so the
    # kernels overlap the same way); ms = one pass over the class's products.
    cls_idx: dict[str, list[int]] = {}
    cls_work: dict[str, float] = {}
    for j, (q, m, name, n, k, c) in enumerate(prods):
        cls_idx.setdefault(c, []).append(j)
        cls_work[c] = cls_work.get(c, 0.0) + algo_work(wl, q, n, k, m)
    class_ms = {c: _graph_ms(torch, cap, cap_h, lambda h, idx=idx: arm.run(h, idx), args.steps, barrier,
                             max_over_ranks) for c, idx in cls_idx.items()}
    # The roofline's kernel: the class with the largest share of the step.
    dominant = max(class_ms, key=class_ms.get)
    j = cls_idx[dominant][0]
    kernels_per_product = _launches_for(lib, arm.linear, arm.calls[j], sh, torch)
    dom_n = len(cls_idx[dominant])
    dom_work_per_launch = cls_work[dominant] / dom_n / world  # one rank's share of one product
    dom_ms_per_launch = class_ms[dominant] / dom_n
    peak, peak_kind = peaks(wl["unit"])
    achieved = work_rate(wl, dom_work_per_launch, dom_ms_per_launch * 1e-3)
    traffic, traffic_src = _traffic(dominant)
    value = work_rate(wl, arm.work_per_step, ms_per_step * 1e-3)

    e2e = None if args.no_e2e else _e2e(args, arm, torch, mq, comm, stream, dev, barrier, max_over_ranks)
    cpu = cpu_baseline(wl, prods, arm.host_blocks, {key: t.cpu().numpy() for key, t in arm.xs.items()},
                       max_seconds=args.cpu_seconds) if keep_host else None

    prefill = None
    if world == 1 and args.workload == "decode" and not args.only and not args.no_prefill:
        prefill = _prefill_line(args, torch, mq, local_rank, cap, cap_h, barrier, max_over_ranks, keep_host)
    forward = None
    if world == 1 and args.workload == "decode" and not args.only and not args.no_forward:
        forward = _forward_line(args, peak if wl["unit"] == "GB/s" else None)

    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": wl["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (GGUF " + "/".join(sorted({TNAME[p[0]].upper() for p in prods})) + " weights)",
            "data": "synthetic (seeded N(0,0.02) weights packed bit-exactly, N(0,1) activations)",
            "config": {"workload": args.workload + (f" (class {args.only})" if args.only else ""),
                       "products": wl["desc"],
                       ("flops_per_step" if wl["unit"] == "TFLOP/s" else "bytes_per_step"): arm.work_per_step,
                       "l2": wl["l2"],
                       "parallelism": (f"tp{world}: fixed global matrices, rank r holds rows [r*N/{world}, "
                                       f"(r+1)*N/{world}) of each; all-gather of the output slices per product")
                       if world > 1 else "single GPU"},
            "roofline": {"bound": "tensor" if wl["unit"] == "TFLOP/s" else "hbm", "kernel": dominant,
                         "achieved": round(achieved, 1), "peak": peak,
                         "unit": wl["unit"], "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "traffic_source": traffic_src,
                         ("algorithmic_flops_per_launch" if wl["unit"] == "TFLOP/s"
                          else "algorithmic_bytes_per_launch"): int(dom_work_per_launch),
                         "ms_per_launch": round(dom_ms_per_launch, 6),
                         "launch": f"one product on one rank ({kernels_per_product} kernel(s)"
                                   + (": the linear kernel and its activation split" if kernels_per_product > 1
                                      and world == 1 else "") + ")"},
            "per_class_ms": {c: round(v, 5) for c, v in sorted(class_ms.items())},
            "per_class_frac": {c: round(work_rate(wl, cls_work[c] / world, class_ms[c] * 1e-3) / peak, 4)
                               for c in sorted(class_ms)},
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            out["cpu_baseline"] = cpu
        if prefill is not None:
            out["prefill"] = prefill
        if forward is not None:
            out["forward"] = forward
        print(json.dumps(out), flush=True)
    torch.cuda.synchronize(dev)
    arm.close()
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()


def _e2e(args, arm, torch, mq, comm, stream, dev, barrier, max_over_ranks) -> dict:
    """The same step end to end through the public API with host buffers (pinned),
    as a serving loop runs it: every step copies all of its inputs from one
    pinned host arena into a device arena (one host-to-device copy), runs the
    products through the Python API on the caller's stream, and reads all of its
    results back into a pinned host arena (one device-to-host copy). The copies
    run on two copy streams and the device arenas are double-buffered, so step
    s + 1's inputs come in and step s's outputs go out while the next products
    compute; the timed region ends when the last step's results are on the
    host."""
    prods = arm.prods
    x_off, y_off = [0], [0]
    for (_, m, _, n, k, _) in prods:
        x_off.append(x_off[-1] + m * k)
        y_off.append(y_off[-1] + m * n)
    hx_all = torch.empty(x_off[-1], dtype=torch.float32).pin_memory()
    hy_all = torch.empty(y_off[-1], dtype=torch.float32).pin_memory()
    dx_all = [torch.empty(x_off[-1], dtype=torch.float32, device=dev) for _ in range(2)]
    dy_all = [torch.empty(y_off[-1], dtype=torch.float32, device=dev) for _ in range(2)]
    for i, (_, m, _, n, k, _) in enumerate(prods):
        hx_all[x_off[i]:x_off[i + 1]].copy_(arm.xs[(m, k)].reshape(-1).cpu())
    dxs = [[dx_all[b][x_off[i]:x_off[i + 1]].view(m, k) for i, (_, m, _, n, k, _) in enumerate(prods)]
           for b in range(2)]
    dys = [[dy_all[b][y_off[i]:y_off[i + 1]].view(m, n) for i, (_, m, _, n, k, _) in enumerate(prods)]
           for b in range(2)]
    apis = [mq.ShardedLinear.from_shard(h, comm) if arm.world > 1 else h for h in arm.handles]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(s):
        b = s % 2
        if s >= 2:
            h2d.wait_event(comp_done[b])  # arena b's inputs were read by step s - 2
        with torch.cuda.stream(h2d):
            dx_all[b].copy_(hx_all, non_blocking=True)
            in_ready[b].record(h2d)
        stream.wait_event(in_ready[b])
        if s >= 2:
            stream.wait_event(out_done[b])  # arena b's outputs of step s - 2 are on the host
        for i in range(len(prods)):
            apis[i].linear(dxs[b][i], out=dys[b][i], stream=stream)
        comp_done[b].record(stream)
        d2h.wait_event(comp_done[b])
        with torch.cuda.stream(d2h):
            hy_all.copy_(dy_all[b], non_blocking=True)
            out_done[b].record(d2h)

    def run(steps):
        start = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        h2d.wait_event(start)
        for s in range(steps):
            e2e_step(s)
        stream.wait_event(out_done[(steps - 1) % 2])
        end = torch.cuda.Event(enable_timing=True)
        end.record(stream)
        return start, end

    run(args.warmup)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = run(args.steps)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    return {"value": round(work_rate(arm.wl, arm.work_per_step, e2e_ms / args.steps * 1e-3), 2),
            "unit": arm.wl["unit"], "h2d_bytes_per_step": 4 * x_off[-1], "d2h_bytes_per_step": 4 * y_off[-1],
            "ms_per_step": round(e2e_ms / args.steps, 6),
            "copies": "double-buffered: step s + 1's inputs in and step s's outputs out on copy streams while "
                      "the products compute"}


FORWARD_EXE = ROOT / "mini_ai_b200" / "adapter" / "_ref" / "mini-ai-b200-forward"


def _forward_line(args, hbm_gbs) -> dict:
    """The full LLaMA-style forward (32 layers, dim 4096, Q8_0, 4 requests x 128
    prompt tokens + 128 greedy decode steps) through the C++ backend's batched
    forward, in tokens/s (mini_ai_b200/adapter/forward_bench.cc), with the
    reference CPU forward timed on 2 layers of the same weights and
    extrapolated. The binary is built where the reference sources exist."""
    if not FORWARD_EXE.exists():
        return {"unavailable": "mini_ai_b200/adapter/_ref/mini-ai-b200-forward is not built (it links the "
                               "reference's sources: make -C mini_ai_b200/adapter REF=...)"}
    cmd = [str(FORWARD_EXE)] + (["--hbm-gbs", str(hbm_gbs)] if hbm_gbs else [])
    if not args.no_cpu_baseline:
        cmd += ["--cpu-layers", "2"]
    res = subprocess.run(cmd, cwd=FORWARD_EXE.parent, capture_output=True, text=True, timeout=900)
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    if res.returncode != 0 or not lines:
        return {"error": f"exit {res.returncode}: " + (res.stdout + res.stderr)[-400:]}
    return json.loads(lines[-1])


def _prefill_line(args, torch, mq, local_rank, cap, cap_h, barrier, max_over_ranks, keep_host) -> dict:
    """The ragged prefill GEMM on one GPU: TFLOP/s over its two products, its own
    roofline against the dense bf16 peak, and the CPU reference on a row sample."""
    wl = WORKLOADS["prefill_ragged_q8_0"]
    prods = products(wl)
    arm = Arm(args, wl, prods, 0, 1, local_rank, torch, mq, None, keep_host)
    with torch.cuda.stream(cap):
        for _ in range(args.warmup):
            arm.run(cap_h)
    barrier()
    ms = _graph_ms(torch, cap, cap_h, arm.run, args.steps, barrier, max_over_ranks)
    value = work_rate(wl, arm.work_per_step, ms * 1e-3)
    peak, peak_kind = peaks(wl["unit"])
    traffic, traffic_src = _traffic(prods[0][5])
    out = {"workload": "prefill_ragged_q8_0", "products": wl["desc"], "value": round(value, 2), "unit": wl["unit"],
           "ms_per_step": round(ms, 6), "flops_per_step": arm.work_per_step,
           "offsets": [0, 1, 8, 41, 105, 233, 433, 944, 1456],
           "roofline": {"bound": "tensor", "kernel": prods[0][5], "achieved": round(value, 1), "peak": peak,
                        "unit": "TFLOP/s", "frac": round(value / peak, 4), "peak_kind": peak_kind,
                        "emulation": "three bf16 products per fp32 product (hi*hi + hi*lo + lo*hi): "
                                     f"ceiling {round(peak / 3, 1)} TFLOP/s",
                        "traffic": traffic, "traffic_source": traffic_src,
                        "algorithmic_flops_per_launch": int(arm.work_per_step / len(prods)),
                        "ms_per_launch": round(ms / len(prods), 6)}}
    if keep_host:
        out["cpu_baseline"] = cpu_baseline(wl, prods, arm.host_blocks,
                                           {key: t.cpu().numpy() for key, t in arm.xs.items()},
                                           max_seconds=min(args.cpu_seconds, 10.0))
    arm.close()
    return out


def _launches_for(lib, linear, call, sh, torch) -> int:
    """Kernel launches one product issues (read from the library's counter)."""
    h, x, m, k, y, n = call
    a = lib.mq_kernel_launches()
    rc = linear(h, x, m, k, None, y, n, sh)
    torch.cuda.synchronize()
    if rc:
        raise RuntimeError("mq_linear failed")
    return max(1, int(lib.mq_kernel_launches() - a))


def kernel_source_digest() -> str:
    """Short digest of the engine's CUDA sources: a DRAM-traffic figure measured
    on other sources no longer describes the kernels that run."""
    h = hashlib.sha256()
    for f in sorted((ROOT / "mini_ai_b200" / "csrc").glob("*.cu*")):
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()[:12]


def _traffic(kernel_class: str):
    """DRAM bytes per launch for the kernel class, from the committed ncu summary
    profiles/dram_traffic.txt, and where the figure comes from. The file records
    the source digest it was captured at; a figure from other sources is not used."""
    f = ROOT / "profiles" / "dram_traffic.txt"
    if not f.exists():
        return None, "no ncu capture"
    digest = None
    for line in f.read_text().splitlines():
        if line.startswith("# sources:"):
            digest = line.split(":", 1)[1].strip()
    now = kernel_source_digest()
    if digest != now:
        return None, f"profiles/dram_traffic.txt was captured on sources {digest}, not the current {now}"
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_class:
            try:
                return int(float(parts[1])), f"ncu capture (profiles/dram_traffic.txt, sources {digest})"
            except ValueError:
                break
    return None, f"no ncu capture of {kernel_class} in profiles/dram_traffic.txt"


# ---------------------------------------------------------------------------
# CPU: the reference's own implementation (oracle/_ref) or its C port.
# ---------------------------------------------------------------------------
def _cpu_engine():
    from oracle import Oracle, Reference, reference_available

    if reference_available():
        return "reference", Reference()
    return "port", Oracle()


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_time_rows(kind, eng, prod, blocks, x, threads) -> float:
    """Seconds for one product on the given activation rows (the reference: one
    LinearDispatch call per row)."""
    q, m, name, n, k, _ = prod
    if kind == "reference":
        w = eng.weight(q, blocks, n, k)
        t = time.perf_counter()
        w.linear(x, threads=threads)
        dt = time.perf_counter() - t
        w.close()
        return dt
    t = time.perf_counter()
    eng.linear(q, blocks, n, k, x, threads=threads)
    return time.perf_counter() - t


def cpu_pass(wl, kind, eng, prods, blocks, xs, threads) -> tuple[float, float]:
    """One pass over the workload on the CPU: every product timed on a bounded
    number of its activation rows (one for decode, `cpu_rows` for prefill) and
    its time scaled to all M rows (the reference runs rows one call at a time,
    src/forward.cc:189-193). Returns (work, seconds)."""
    rows = wl["cpu_rows"] or 1
    work, secs = 0.0, 0.0
    for i, p in enumerate(prods):
        q, m, name, n, k, _ = p
        r = min(rows, m)
        dt = cpu_time_rows(kind, eng, p, blocks[i], xs[(m, k)][:r], threads)
        work += algo_work(wl, q, n, k, m)
        secs += dt * m / r
    return work, secs


def cpu_baseline(wl, prods, blocks, xs, max_seconds: float = 20.0) -> dict:
    kind, eng = _cpu_engine()
    threads = cpu_threads()
    rows = wl["cpu_rows"] or 1
    work, secs, reps, wall = 0.0, 0.0, 0, time.perf_counter()
    while reps < 1 or (time.perf_counter() - wall < max_seconds * 0.5 and reps < 5):
        w, t = cpu_pass(wl, kind, eng, prods, blocks, xs, threads)
        work, secs, reps = work + w, secs + t, reps + 1
    return {"value": round(work_rate(wl, work, secs), 6), "unit": wl["unit"], "cores": threads, "kind": kind,
            "sample": (f"{reps} pass(es) over the workload's {len(prods)} products, each timed on its first "
                       f"{rows} activation row(s) and scaled to its M rows (the reference runs one row per call); "
                       + (f"LinearDispatch kThreadedSimd with SetMatmulThreads({threads})" if kind == "reference"
                          else f"C port of QuantizedDotRow, {threads} threads"))}


def host_workload(prods, seed: int = 0):
    """Seeded host weights (packed by the reference's own QuantizeTensor in row
    chunks on threads; packing is row-independent), one per distinct matrix
    shape and type, and activations."""
    from concurrent.futures import ThreadPoolExecutor

    kind, eng = _cpu_engine()
    rng = np.random.default_rng(seed)
    cache, blocks = {}, []
    for (q, m, name, n, k, _) in prods:
        if (q, n, k) not in cache:
            w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
            chunks = np.array_split(np.arange(n), min(64, n))
            with ThreadPoolExecutor(max_workers=cpu_threads()) as ex:
                parts = list(ex.map(lambda r: eng.quantize(q, w[r[0]:r[-1] + 1]), chunks))
            cache[(q, n, k)] = np.concatenate(parts)
            del w
        blocks.append(cache[(q, n, k)])
    xs = {}
    for (q, m, name, n, k, _) in prods:
        if (m, k) not in xs:
            xs[(m, k)] = rng.standard_normal((m, k), dtype=np.float32)
    return kind, eng, blocks, xs


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    wl = WORKLOADS[args.workload]
    prods = select(products(wl), args.only)
    kind, eng, blocks, xs = host_workload(prods)
    threads = cpu_threads()
    cpu_time_rows(kind, eng, prods[0], blocks[0], xs[(prods[0][1], prods[0][4])][:1], threads)  # warm the pool
    for _ in range(max(0, args.warmup)):
        pass  # the CPU path keeps no state between calls: warm-up passes would only repeat the first step
    # Each step = one pass over every product of the workload (each product sampled once).
    total_w, total_t = 0.0, 0.0
    for _ in range(args.steps):
        w, t = cpu_pass(wl, kind, eng, prods, blocks, xs, threads)
        total_w, total_t = total_w + w, total_t + t
    value = work_rate(wl, total_w, total_t)
    rows = wl["cpu_rows"] or 1
    sample = (f"each step = one pass over the workload's {len(prods)} products, each timed on its first {rows} "
              f"activation row(s) and scaled to its M rows (the reference runs one row per call); "
              f"{'reference LinearDispatch kThreadedSimd' if kind == 'reference' else 'C port'}, {threads} threads")
    unit = wl["unit"]
    out = {"metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(total_t / args.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None,
           "dtype": "f32 (GGUF " + "/".join(sorted({TNAME[p[0]].upper() for p in prods})) + " weights)",
           "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)", "impl": "reference",
           "config": {"workload": args.workload + (f" (class {args.only})" if args.only else ""),
                      "products": wl["desc"], "parallelism": f"{threads} host threads"},
           "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads, "kind": kind,
                            "sample": sample},
           "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-forward", action="store_true")
    ap.add_argument("--only", default=None, help="one kernel class, e.g. llama3_8b_ffn_q4_0_m16 (profiling)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
