"""One rank of the two-GPU sharded-linear check (launched by tests/test_sharded.py
through torchrun): the gathered output must equal this GPU's unsharded product
bit for bit (at 1024 x 4096 neither launch has more (tile, K step) chunks than
SMs, so both give every chunk its own CTA and sum in the same order), and the
oracle within the parity tolerance."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main() -> int:
    import torch
    import torch.distributed as dist

    import mini_ai_b200 as mq
    from conftest import abs_dot_bound, assert_linear_close
    from oracle import Oracle, QTYPES

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    orc = Oracle()
    try:
        comm = mq.CudaComm.from_process_group(dev)
        for q in QTYPES:
            rng = np.random.default_rng(99 + q)  # same weights and inputs on every rank
            rows, cols = 1024, 4096
            w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
            s = mq.QuantizeTensor(w, q)
            sl = mq.ShardedLinear(s, comm)
            full = mq.CudaWeight(s, device=dev)
            deq = orc.dequantize(q, s.bytes, rows, cols)
            for m in (1, 4, 17):
                xn = rng.standard_normal((m, cols)).astype(np.float32)
                x = torch.from_numpy(xn).cuda(dev)
                a = sl.linear(x).cpu().numpy()
                b = full.linear(x).cpu().numpy()
                if not np.array_equal(a.view(np.uint32), b.view(np.uint32)):
                    print(f"rank {rank}: sharded != unsharded (type {q}, m {m})", flush=True)
                    return 1
                assert_linear_close(a, orc.linear(q, s.bytes, rows, cols, xn), abs_dot_bound(deq, xn))
            # Consecutive calls into one output (the gather alternates its two
            # staging halves), then the same calls captured in a CUDA graph and
            # replayed with new inputs (the gather's epoch lives on the device).
            for m in (1, 16):
                xs = torch.from_numpy(rng.standard_normal((3, m, cols)).astype(np.float32)).cuda(dev)
                out = torch.empty((m, rows), dtype=torch.float32, device=f"cuda:{dev}")
                for i in range(3):
                    sl.linear(xs[i], out=out)
                    if not torch.equal(out, full.linear(xs[i])):
                        print(f"rank {rank}: consecutive call {i} differs (type {q}, m {m})", flush=True)
                        return 1
                st = torch.cuda.Stream(dev)
                xin = torch.empty((m, cols), dtype=torch.float32, device=f"cuda:{dev}")
                with torch.cuda.stream(st):
                    sl.linear(xin.copy_(xs[0]), out=out, stream=st)  # eager call on the capture stream first
                torch.cuda.synchronize(dev)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=st):
                    sl.linear(xin, out=out, stream=st)
                    sl.linear(xin, out=out, stream=st)
                for i in (1, 2):
                    xin.copy_(xs[i])
                    torch.cuda.synchronize(dev)
                    graph.replay()
                    torch.cuda.synchronize(dev)
                    if not torch.equal(out, full.linear(xs[i])):
                        print(f"rank {rank}: graph replay {i} differs (type {q}, m {m})", flush=True)
                        return 1
                del graph
            sl.close()
            full.close()
        comm.close()
        print(f"rank {rank}: sharded ok", flush=True)
        return 0
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
