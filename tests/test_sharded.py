"""Row-sharded linear with an all-gather of the output slices (the multi-GPU
row of the hot path): partition math, the ABI's argument checks, and the
gather semantics on world-size-2 gloo ranks on the CPU; the NCCL path itself
on GPUs (one rank on any B200 box, two ranks where two GPUs exist).

Oracle: concatenating the per-shard outputs must equal the unsharded output
bit for bit (rows are independent), and the unsharded output is checked
against the CPU oracle like every other product."""
from __future__ import annotations

import ctypes as C
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, abs_dot_bound, assert_linear_close
from oracle import NAMES, Q4_0, Q4_1, Q8_0, QTYPES


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_partition(mq):
    for rows, world in [(14336, 8), (4096, 2), (128256, 8), (16, 4), (7, 1)]:
        spans = [mq.shard_rows(rows, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert len({e - b for b, e in spans}) == 1
    with pytest.raises(ValueError):
        mq.shard_rows(10, 4, 0)  # unequal slices
    with pytest.raises(ValueError):
        mq.shard_rows(16, 4, 4)


def test_sharded_abi_validation(mq):
    lib = mq.lib()
    out = C.c_void_p()
    buf = C.create_string_buffer(128)
    assert lib.mq_comm_create(0, 2, 2, buf, 128, C.byref(out)) == mq._lib.MQ_ERR_INVALID and not out.value
    assert lib.mq_comm_create(0, 2, 0, buf, 64, C.byref(out)) == mq._lib.MQ_ERR_INVALID
    assert lib.mq_comm_unique_id(buf, 16) == mq._lib.MQ_ERR_INVALID
    rc = lib.mq_linear_sharded_allgather(None, None, 1, 32, None, None, 32, None, None)
    assert rc == mq._lib.MQ_ERR_INVALID and "null" in mq._lib.last_error()
    lib.mq_comm_destroy(None)


def _gloo_rank(rank: int, world: int, port: int, q: int, conn) -> None:
    """One CPU rank: its shard's rows through the oracle, then a gloo all-gather."""
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle import Oracle

    import mini_ai_b200 as mq

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(77 + q)
        rows, cols, m = 96, 200, 3
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, cols)).astype(np.float32)
        orc = Oracle()
        blocks = orc.quantize(q, w)
        bb = ((cols + 31) // 32) * {Q8_0: 34, Q4_0: 18, Q4_1: 20}[q]
        r0, r1 = mq.shard_rows(rows, world, rank)
        mine = orc.linear(q, blocks[r0 * bb:r1 * bb], r1 - r0, cols, x)
        parts = [torch.zeros((m, r1 - r0), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
        full = mq.assemble([p.numpy() for p in parts])
        ref = orc.linear(q, blocks, rows, cols, x)
        conn.send(bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_gloo_two_ranks_gather_is_bit_identical(q):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    pipes = [ctx.Pipe(duplex=False) for _ in range(2)]
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q, pipes[r][1])) for r in range(2)]
    for p in procs:
        p.start()
    results = [pipes[r][0].recv() if pipes[r][0].poll(120) else None for r in range(2)]
    for p in procs:
        p.join(60)
    assert results == [True, True], results
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.gpu
@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_single_rank_nccl_path_matches_linear(mq, oracle, cuda_device, q):
    """World of one: the full C-ABI path (communicator, shard checks, in-place
    gather for m = 1, gather buffer + interleave for m > 1) on one GPU."""
    import torch

    rng = np.random.default_rng(5 + q)
    rows, cols = 512, 4097
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(w, q)
    comm = mq.CudaComm(cuda_device, 1, 0, mq.CudaComm.new_id())
    sl = mq.ShardedLinear(s, comm)
    full = mq.CudaWeight(s, device=cuda_device)
    deq = oracle.dequantize(q, s.bytes, rows, cols)
    for m in (1, 3, 16):
        x = torch.from_numpy(rng.standard_normal((m, cols)).astype(np.float32)).to(f"cuda:{cuda_device}")
        y_sh = sl.linear(x)
        y_1 = full.linear(x)
        torch.cuda.synchronize(cuda_device)
        a, b = y_sh.cpu().numpy(), y_1.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), m
        assert_linear_close(a, oracle.linear(q, s.bytes, rows, cols, x.cpu().numpy()), abs_dot_bound(deq, x.cpu().numpy()))
    sl.close()
    full.close()
    comm.close()


@pytest.mark.gpu
@pytest.mark.parametrize("gather", ["peer", "nccl"])
def test_two_ranks_allgather(gather):
    """Two processes on two GPUs through torchrun (skipped on one-GPU boxes): the
    peer-memory gather (MQ_P2P_GATHER=1) and NCCL's all-gather."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MQ_P2P_GATHER="1" if gather == "peer" else "0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(ROOT / "tests" / "sharded_worker.py")]
    res = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("sharded ok") == 2


@pytest.mark.gpu
def test_two_ranks_peer_gather_timeout():
    """A rank that leaves out a call: the other rank's peer-memory gather gives up
    after its wait limit (0.2 s here), writes NaN into the missing columns and
    reports MQ_ERR_TIMEOUT from then on (tests/timeout_worker.py). Two GPUs."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MQ_P2P_GATHER="1", MQ_P2P_WAIT_NS="200000000")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(ROOT / "tests" / "timeout_worker.py")]
    res = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    out = res.stdout
    assert out.count("timeout ok") == 2 or out.count("timeout check skipped") == 2, out[-3000:]
