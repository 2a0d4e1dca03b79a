"""One rank of the two-GPU bounded-wait check of the peer-memory gather
(launched by tests/test_sharded.py through torchrun with MQ_P2P_GATHER=1,
MQ_P2P_WAIT_NS=200000000 and NCCL_NVLS_ENABLE=0).

Both ranks make one ordinary sharded call; then rank 1 leaves out the next
call (between calls, with nothing of its own in flight) while rank 0 makes
it. Rank 0's pull kernel waits for rank 1's arrival flag for 0.2 s, gives up,
writes NaN into rank 1's output columns and poisons the communicator: its
next call and every later one fail with MQ_ERR_TIMEOUT before launching
anything. No GPU is faulted or hung: the wait is bounded in the kernel."""
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
    from oracle import Q4_0

    rank = int(os.environ["RANK"])
    dev = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    status = 0
    try:
        comm = mq.CudaComm.from_process_group(dev)
        peer = comm.uses_peer_gather
        agree = [None, None]
        dist.all_gather_object(agree, peer)
        if not all(agree):
            # Without the peer-memory gather a skipped call would leave NCCL
            # waiting without a bound: the check does not run.
            print(f"rank {rank}: peer gather not available, timeout check skipped", flush=True)
            comm.close()
            return 0
        rng = np.random.default_rng(7)
        rows, cols, m = 512, 1024, 2
        s = mq.QuantizeTensor((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32), Q4_0)
        sl = mq.ShardedLinear(s, comm)
        full = mq.CudaWeight(s, device=dev)
        x = torch.from_numpy(rng.standard_normal((m, cols)).astype(np.float32)).cuda(dev)
        ref = full.linear(x)
        out = sl.linear(x)
        torch.cuda.synchronize(dev)
        ok = torch.equal(out, ref)
        dist.barrier()
        half = rows // 2
        if rank == 0:
            out2 = sl.linear(x)  # rank 1 never arrives: the bounded wait runs out
            torch.cuda.synchronize(dev)
            mine = torch.equal(out2[:, :half], ref[:, :half])
            nan_peer = bool(torch.isnan(out2[:, half:]).all())
            codes = []
            for _ in range(2):  # poisoned: every later call fails at once
                try:
                    sl.linear(x)
                    codes.append(0)
                except mq.MQError as e:
                    codes.append(e.code)
            torch.cuda.synchronize(dev)
            ok = ok and mine and nan_peer and codes == [mq._lib.MQ_ERR_TIMEOUT] * 2
            print(f"rank 0: own columns {mine}, peer columns NaN {nan_peer}, later calls {codes}", flush=True)
        dist.barrier()
        sl.close()
        full.close()
        comm.close()
        if ok:
            print(f"rank {rank}: timeout ok", flush=True)
        else:
            status = 1
    finally:
        dist.barrier()
        dist.destroy_process_group()
    return status


if __name__ == "__main__":
    sys.exit(main())
