#!/usr/bin/env python
"""Benchmark of the B200 quantized-linear path (one JSON line on rank 0).

Workload (default, ``llama3_8b_ffn_decode``): Llama-3-8B FFN decode GEMVs over
GGUF Q4_0 and Q4_1 weights — gate/up W 14336x4096 and down W 4096x14336,
weights ~N(0, 0.02) quantized with the bit-exact packer, activations ~N(0, 1)
F32 with M = 1, 4 and 16 rows. One step = all 18 products (2 types x 3 M x
3 matrices). Every (type, M, matrix) has its own weight copy, so a step
streams 627 MB of distinct packed weights (> the 126 MB L2) and no launch
finds its weights in L2.

Metric: GB/s of algorithmic bytes, N*ceil(K/32)*block_bytes + 4*M*K + 4*M*N
per product, over the whole step.

``--workload prefill_ragged_q8_0``: the ragged prefill GEMM (Q8_0 W 11008x4096
and 4096x11008, 8 requests of 1..512 rows packed to M = 1456) in TFLOP/s of
2*M*N*K, against the measured dense bf16 peak.
  value : device time, weights and activations resident in HBM;
  e2e   : through the public API with host buffers: every step copies every
          product's activations from pinned host memory (one host-to-device
          copy of the step's input arena) and every product's outputs back
          (one device-to-host copy) inside the timed region.

Multi-GPU (torchrun, N ranks): tensor-parallel row sharding with weak
scaling. Every matrix grows to N x its rows (an N-times wider FFN); rank r
holds the equal row shard r, which is exactly the 1-GPU matrix size, so every
GPU streams the same bytes as the 1-GPU run, and every product ends with the
NCCL all-gather of the output slices over NVLink (mq_linear_sharded_allgather,
inside the timed graph). value = all ranks' algorithmic bytes / max-over-ranks
time.

``--impl reference`` times the reference's own CPU implementation
(LinearDispatch kThreadedSimd from the reference sources built in
oracle/_ref, else the C port of it) on the same workload, metric and unit.
"""
from __future__ import annotations

import argparse
import ctypes as C
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

WORKLOADS = {
    # decode GEMVs (the default, the configuration the metric is quoted on): GB/s of algorithmic bytes
    "llama3_8b_ffn_decode": {
        "qtypes": (Q4_0, Q4_1),
        "ms": (1, 4, 16),
        "mats": (("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)),
        "unit": "GB/s",
        "desc": "gate/up 14336x4096, down 4096x14336; Q4_0, Q4_1; M = 1, 4, 16",
        "l2": "inputs larger than L2: 627 MB of distinct weights per GPU per step",
        "cpu_rows": None,
    },
    # ragged prefill GEMM: 8 requests of {1,7,33,64,128,200,511,512} rows (M = 1456) packed
    # contiguously, Q8_0 W 11008x4096 and 4096x11008: TFLOP/s of 2*M*N*K
    "prefill_ragged_q8_0": {
        "qtypes": (Q8_0,),
        "ms": (1456,),
        "mats": (("w_up", 11008, 4096), ("w_down", 4096, 11008)),
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
    """(qtype, m, name, n, k) for every product of one step, in launch order."""
    return [(q, m, name, n, k) for q in wl["qtypes"] for m in wl["ms"] for (name, n, k) in wl["mats"]]


def select(prods, only: str | None):
    """Restrict to products of one type and M, e.g. ``q4_0:16`` (profiling a single kernel class)."""
    if not only:
        return prods
    t, m = only.split(":")
    q = {v: k for k, v in TNAME.items()}[t]
    return [p for p in prods if p[0] == q and p[1] == int(m)]


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

    # Weights: generated on the device, packed by the bit-exact device quantizer.
    # With N ranks each matrix has N x rows and this rank keeps row shard `rank`
    # (the same seed on every rank, so the shards form one global matrix).
    gen = torch.Generator(device=dev)
    handles, host_blocks = [], []
    keep_host = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.only
    for i, (q, m, name, n, k) in enumerate(prods):
        gen.manual_seed(1000 + i)
        w32 = torch.randn((n * world, k), generator=gen, device=dev, dtype=torch.float32).mul_(0.02)
        blocks = torch.empty(lib.mq_quantized_bytes(q, n * world, k), dtype=torch.uint8, device=dev)
        rc = lib.mq_quantize_device(local_rank, q, w32.data_ptr(), n * world, k, blocks.data_ptr(), blocks.numel(), sh)
        if rc:
            raise RuntimeError(mq._lib.last_error())
        del w32
        handles.append(mq.CudaWeight.from_device_blocks(blocks, q, n * world, k, device=local_rank, stream=stream,
                                                        row_range=(rank * n, (rank + 1) * n)))
        if keep_host:
            host_blocks.append(blocks.cpu().numpy())
        del blocks
    comm = mq.CudaComm.from_process_group(local_rank) if world > 1 else None
    gen.manual_seed(424242)
    xs = {(m, k): torch.randn((m, k), generator=gen, device=dev, dtype=torch.float32)
          for (_, m, _, _, k) in prods}
    ys = {(m, n): torch.empty((m, n * world), dtype=torch.float32, device=dev) for (_, m, _, n, _) in prods}
    calls = [(handles[i].handle, xs[(m, k)].data_ptr(), m, k, ys[(m, n)].data_ptr(), n * world)
             for i, (q, m, name, n, k) in enumerate(prods)]
    # whole-job algorithmic bytes: every rank's shard product (its weights, x, its output slice)
    work_per_step = sum(world * algo_work(wl, q, n, k, m) for (q, m, _, n, k) in prods)
    if world > 1:
        gather = lib.mq_linear_sharded_allgather

        def linear(h, x, m, k, b, y, n, s):
            return gather(h, x, m, k, b, y, n, comm.handle, s)
    else:
        linear = lib.mq_linear

    def run_calls(stream_handle, idx):
        for j in idx:
            h, x, m, k, y, n = calls[j]
            rc = linear(h, x, m, k, None, y, n, stream_handle)
            if rc:
                raise RuntimeError(mq._lib.last_error())

    def step(stream_handle):
        run_calls(stream_handle, range(len(calls)))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # The timed region replays a CUDA graph holding exactly K steps, captured on
    # a dedicated stream after eager warm-up on that stream (so per-stream
    # scratch already exists). Nothing sits between the products inside the
    # graph, so consecutive kernels overlap through programmatic dependent
    # launch as they do in an application's stream.
    cap = torch.cuda.Stream(dev)
    cap_h = C.c_void_p(cap.cuda_stream)
    with torch.cuda.stream(cap):
        for _ in range(args.warmup):
            step(cap_h)
    barrier()
    graph = torch.cuda.CUDAGraph()
    launches0 = lib.mq_kernel_launches()
    with torch.cuda.graph(graph, stream=cap):
        for s in range(args.steps):
            step(cap_h)
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
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps

    # Device time per kernel class (type, M): a graph per class holding the
    # class's products (gate, up, down) K times back to back, timed with CUDA
    # events on the capture stream; the same calls as in the step, so the
    # kernels overlap the same way. ms = one pass over the class's products.
    cls_idx: dict[str, list[int]] = {}
    cls_bytes: dict[str, int] = {}
    for j, (q, m, name, n, k) in enumerate(prods):
        c = f"linear_{TNAME[q]}_m{m}"
        cls_idx.setdefault(c, []).append(j)
        cls_bytes[c] = cls_bytes.get(c, 0) + algo_work(wl, q, n, k, m)
    cls_first = {c: idx[0] for c, idx in cls_idx.items()}
    cls_count = {c: len(idx) for c, idx in cls_idx.items()}
    class_ms: dict[str, float] = {}
    for c, idx in cls_idx.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for _ in range(args.steps):
                run_calls(cap_h, idx)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cap):
            g.replay()
            barrier()
            c0.record(cap)
            g.replay()
            c1.record(cap)
            barrier()
        cms = c0.elapsed_time(c1) / args.steps
        if world > 1:
            t = torch.tensor([cms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            cms = float(t.item())
        class_ms[c] = cms
        del g
    dominant = max(class_ms, key=class_ms.get)
    j = cls_first[dominant]
    q, m, _, n, k = prods[j]
    # One "launch" of the dominant kernel = one product: its linear kernel (plus,
    # on the fp16 tensor-core paths, the small activation split before it).
    kernels_per_product = _launches_for(lib, linear, calls[j], sh, torch)
    dom_launches = cls_count[dominant]
    dom_bytes_per_launch = cls_bytes[dominant] / dom_launches
    dom_ms_per_launch = class_ms[dominant] / dom_launches
    peak, peak_kind = peaks(wl["unit"])
    achieved = work_rate(wl, dom_bytes_per_launch, dom_ms_per_launch * 1e-3)
    traffic = _traffic(dominant)

    value = work_rate(wl, work_per_step, ms_per_step * 1e-3)  # work_per_step is already the whole job's

    # End to end through the public API with host buffers (pinned), same stream.
    # Every product has its own input and output slice in one pinned host arena
    # and one device arena: a step copies all of its inputs in with one
    # host-to-device copy, runs the products through the Python API, and reads
    # all of its results back with one device-to-host copy.
    e2e_value, e2e_ms = None, None
    x_off, y_off = [0], [0]
    for (_, m, _, n, k) in prods:
        x_off.append(x_off[-1] + m * k)
        y_off.append(y_off[-1] + m * n * world)
    hx_all = torch.empty(x_off[-1], dtype=torch.float32).pin_memory()
    hy_all = torch.empty(y_off[-1], dtype=torch.float32).pin_memory()
    dx_all = torch.empty(x_off[-1], dtype=torch.float32, device=dev)
    dy_all = torch.empty(y_off[-1], dtype=torch.float32, device=dev)
    for i, (_, m, _, n, k) in enumerate(prods):
        hx_all[x_off[i]:x_off[i + 1]].copy_(xs[(m, k)].reshape(-1).cpu())
    dxs = [dx_all[x_off[i]:x_off[i + 1]].view(m, k) for i, (_, m, _, n, k) in enumerate(prods)]
    dys = [dy_all[y_off[i]:y_off[i + 1]].view(m, n * world) for i, (_, m, _, n, k) in enumerate(prods)]
    h2d = 4 * x_off[-1]
    d2h = 4 * y_off[-1]

    apis = [mq.ShardedLinear.from_shard(h, comm) if world > 1 else h for h in handles]

    def e2e_step():
        dx_all.copy_(hx_all, non_blocking=True)
        for i in range(len(prods)):
            apis[i].linear(dxs[i], out=dys[i], stream=stream)
        hy_all.copy_(dy_all, non_blocking=True)

    if not args.no_e2e:
        for _ in range(args.warmup):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_value = work_rate(wl, work_per_step, e2e_ms / args.steps * 1e-3)

    cpu = None
    if keep_host:
        cpu = cpu_baseline(wl, prods, host_blocks, {key: t.cpu().numpy() for key, t in xs.items()},
                           max_seconds=args.cpu_seconds)

    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": wl["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (GGUF " + "/".join(TNAME[q].upper() for q in wl["qtypes"]) + " weights)",
            "data": "synthetic (seeded N(0,0.02) weights packed bit-exactly, N(0,1) activations)",
            "config": {"workload": args.workload,
                       "products": wl["desc"] + (f"; rows x{world}, row-sharded" if world > 1 else ""),
                       ("flops_per_step" if wl["unit"] == "TFLOP/s" else "bytes_per_step"): work_per_step,
                       "l2": wl["l2"],
                       "parallelism": f"tp{world}: row shards + NCCL all-gather per product" if world > 1
                       else "single GPU"},
            "roofline": {"bound": "tensor" if wl["unit"] == "TFLOP/s" else "hbm", "kernel": dominant,
                         "achieved": round(achieved, 1), "peak": peak,
                         "unit": wl["unit"], "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, ("algorithmic_flops_per_launch" if wl["unit"] == "TFLOP/s"
                                              else "algorithmic_bytes_per_launch"): int(dom_bytes_per_launch),
                         "ms_per_launch": round(dom_ms_per_launch, 6),
                         "launch": f"one product ({kernels_per_product} kernel(s)"
                                   + (": the linear kernel + its activation split)" if kernels_per_product > 1
                                      else ")")},
            "per_class_ms": {c: round(v, 5) for c, v in sorted(class_ms.items())},
            "e2e": None if e2e_value is None else {
                "value": round(e2e_value, 2), "unit": wl["unit"], "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 6)},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            out["cpu_baseline"] = cpu
        print(json.dumps(out), flush=True)
    del graph  # a graph holding NCCL calls is released before the communicators
    torch.cuda.synchronize(dev)
    for h in handles:
        h.close()
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()


def _launches_for(lib, linear, call, sh, torch) -> int:
    """Kernel launches one product issues (read from the library's counter)."""
    h, x, m, k, y, n = call
    a = lib.mq_kernel_launches()
    rc = linear(h, x, m, k, None, y, n, sh)
    torch.cuda.synchronize()
    if rc:
        raise RuntimeError("mq_linear failed")
    return max(1, int(lib.mq_kernel_launches() - a))


def _traffic(kernel_class: str):
    """DRAM bytes per launch for the kernel class, from the committed ncu summary."""
    f = ROOT / "profiles" / "dram_traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_class:
            try:
                return int(float(parts[1]))
            except ValueError:
                return None
    return None


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


def cpu_run(kind, eng, prods, blocks, xs, threads):
    """One pass over `prods` on the CPU (each product over the rows of xs[(m, k)]); returns seconds."""
    if kind == "reference":
        ws = [eng.weight(q, blocks[i], n, k) for i, (q, m, name, n, k) in enumerate(prods)]
        t = time.perf_counter()
        for i, (q, m, name, n, k) in enumerate(prods):
            ws[i].linear(xs[(m, k)], threads=threads)
        dt = time.perf_counter() - t
        for w in ws:
            w.close()
        return dt
    t = time.perf_counter()
    for i, (q, m, name, n, k) in enumerate(prods):
        eng.linear(q, blocks[i], n, k, xs[(m, k)], threads=threads)
    return time.perf_counter() - t


def cpu_baseline(wl, prods, blocks, xs, max_seconds: float = 20.0) -> dict:
    kind, eng = _cpu_engine()
    threads = cpu_threads()
    rows = wl["cpu_rows"]
    if rows:  # a bounded sample: the first `rows` activation rows of every product
        xs = {key: x[:rows] for key, x in xs.items()}
        prods = [(q, min(m, rows), name, n, k) for (q, m, name, n, k) in prods]
        xs = {(min(m, rows), k): x for (m, k), x in xs.items()}
    work_step = sum(algo_work(wl, q, n, k, m) for (q, m, _, n, k) in prods)
    reps, total = 0, 0.0
    while reps < 1 or (total < max_seconds * 0.5 and reps < 5):
        total += cpu_run(kind, eng, prods, blocks, xs, threads)
        reps += 1
    return {"value": round(work_rate(wl, work_step * reps, total), 6), "unit": wl["unit"], "cores": threads,
            "kind": kind,
            "sample": (f"{reps} pass(es) over the workload's {len(prods)} products"
                       + (f" restricted to their first {rows} activation rows" if rows else "")
                       + f" ({work_step:.4g} units of work each), "
                       + (f"LinearDispatch kThreadedSimd per activation row with SetMatmulThreads({threads})"
                          if kind == "reference" else f"C port of QuantizedDotRow, {threads} threads"))}


def host_workload(prods, seed: int = 0):
    """Seeded host weights (packed by the reference's own QuantizeTensor in row
    chunks on threads; packing is row-independent) and activations."""
    from concurrent.futures import ThreadPoolExecutor

    kind, eng = _cpu_engine()
    rng = np.random.default_rng(seed)
    blocks = []
    for (q, m, name, n, k) in prods:
        w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
        chunks = np.array_split(np.arange(n), min(32, n))
        with ThreadPoolExecutor(max_workers=cpu_threads()) as ex:
            parts = list(ex.map(lambda r: eng.quantize(q, w[r[0]:r[-1] + 1]), chunks))
        blocks.append(np.concatenate(parts))
    xs = {}
    for (q, m, name, n, k) in prods:
        if (m, k) not in xs:
            xs[(m, k)] = rng.standard_normal((m, k), dtype=np.float32)
    return kind, eng, blocks, xs


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    wl = WORKLOADS[args.workload]
    prods = products(wl)
    rows = wl["cpu_rows"]
    if rows:  # the reference runs prefill row by row: each product is sampled on its first rows
        prods = [(q, min(m, rows), name, n, k) for (q, m, name, n, k) in prods]
    kind, eng, blocks, xs = host_workload(prods)
    threads = cpu_threads()
    cpu_run(kind, eng, prods[:1], blocks[:1], xs, threads)  # warm the thread pool and caches
    # Each step is a bounded sample of the workload: one of its products, in launch order.
    work_all = [algo_work(wl, q, n, k, m) for (q, m, _, n, k) in prods]
    total_w, total_t = 0.0, 0.0
    for s in range(args.steps):
        i = s % len(prods)
        total_t += cpu_run(kind, eng, [prods[i]], [blocks[i]], xs, threads)
        total_w += work_all[i]
    value = work_rate(wl, total_w, total_t)
    sample = (f"each step = one of the workload's {len(prods)} products, in launch order"
              + (f", on its first {rows} activation rows" if rows else "") + "; "
              f"{'reference LinearDispatch kThreadedSimd' if kind == 'reference' else 'C port'}, {threads} threads")
    unit = wl["unit"]
    out = {"metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(total_t / args.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "dtype": "f32 (GGUF " + "/".join(TNAME[q].upper() for q in wl["qtypes"]) + " weights)",
           "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)", "impl": "reference",
           "config": {"workload": args.workload, "products": wl["desc"], "parallelism": f"{threads} host threads"},
           "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads, "kind": kind,
                            "sample": sample},
           "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3_8b_ffn_decode")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--only", default=None, help="one kernel class, e.g. q4_0:16 (profiling)")
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
