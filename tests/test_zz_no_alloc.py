"""mq_linear_noalloc: the decode product for callers that cannot allocate device
memory (their own pool owns every byte, a fixed memory budget, or a hot loop
that cannot afford cudaMalloc's synchronisation). Its scratch is a fixed
device array, so the call itself must allocate nothing.

Checked through the C ABI against mq_linear on the same inputs, on two calls
in a row (the array keeps the previous call's contents), with the parity
tolerance the other GPU tests use. Collected last so that a run stopping at
the first failure has already run every other test; it also passes alone.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import abs_dot_bound, assert_linear_close
from oracle import NAMES, Q4_0, Q4_1, Q8_0

pytestmark = pytest.mark.gpu

CASES = [  # (type, rows, cols, m): tails, split-K fixup, both tile widths of activations
    (Q4_0, 14336, 4096, 4),
    (Q8_0, 4096, 14336, 16),
    (Q4_1, 300, 4097, 1),
    (Q4_0, 136, 320, 7),
    (Q4_1, 4096, 14336, 16),
]


def _case(mq, oracle, q, rows, cols, m, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    s = mq.QuantizeTensor(w, q)
    xs = [rng.standard_normal((m, cols), dtype=np.float32) for _ in range(2)]
    deq = oracle.dequantize(q, s.bytes, rows, cols)
    return s, xs, deq


@pytest.mark.parametrize("q,rows,cols,m", CASES, ids=[f"{NAMES[c[0]]}-{c[1]}x{c[2]}-m{c[3]}" for c in CASES])
def test_noalloc_matches_linear(mq, oracle, cuda_device, q, rows, cols, m):
    import torch

    lib = mq.lib()
    s, xs, deq = _case(mq, oracle, q, rows, cols, m, seed=rows + cols + m)
    wt = mq.CudaWeight(s, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device)
    sh = C.c_void_p(stream.cuda_stream)
    bias = torch.linspace(-0.5, 0.5, rows, device=f"cuda:{cuda_device}")
    for call, x in enumerate(xs):  # two calls in a row, different activations
        xd = torch.from_numpy(x).to(f"cuda:{cuda_device}")
        y_ref = torch.empty((m, rows), device=f"cuda:{cuda_device}")
        y_na = torch.full((m, rows), 123.0, device=f"cuda:{cuda_device}")
        assert lib.mq_linear(wt.handle, xd.data_ptr(), m, cols, bias.data_ptr(), y_ref.data_ptr(), rows, sh) == 0
        rc = lib.mq_linear_noalloc(wt.handle, xd.data_ptr(), m, cols, bias.data_ptr(), y_na.data_ptr(), rows, sh)
        assert rc == 0, mq._lib.last_error()
        torch.cuda.synchronize(cuda_device)
        b = bias.cpu().numpy()
        bound = abs_dot_bound(deq, x) + np.abs(b)[None, :]
        assert_linear_close(y_na.cpu().numpy(), y_ref.cpu().numpy(), bound)
        assert np.all(np.isfinite(y_na.cpu().numpy())), f"call {call}"


def test_noalloc_allocates_nothing_and_rejects_oversize(mq, oracle, cuda_device):
    import torch

    lib = mq.lib()
    s, xs, _ = _case(mq, oracle, Q4_0, 2048, 1024, 8, seed=3)
    wt = mq.CudaWeight(s, device=cuda_device)
    sh = C.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    xd = torch.from_numpy(xs[0]).to(f"cuda:{cuda_device}")
    y = torch.empty((8, 2048), device=f"cuda:{cuda_device}")
    assert lib.mq_linear_noalloc(wt.handle, xd.data_ptr(), 8, 1024, None, y.data_ptr(), 2048, sh) == 0  # set-up
    torch.cuda.synchronize(cuda_device)
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(5):
        assert lib.mq_linear_noalloc(wt.handle, xd.data_ptr(), 8, 1024, None, y.data_ptr(), 2048, sh) == 0
    torch.cuda.synchronize(cuda_device)
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0, "device memory changed across allocation-free calls"
    rc = lib.mq_linear_noalloc(wt.handle, xd.data_ptr(), 17, 1024, None, y.data_ptr(), 2048, sh)
    assert rc == mq._lib.MQ_ERR_INVALID and "at most 16" in mq._lib.last_error()
    big = mq.CudaWeight(mq.QuantizeTensor(np.zeros((16, 16416), np.float32), Q8_0), device=cuda_device)
    xb = torch.zeros((1, 16416), device=f"cuda:{cuda_device}")
    yb = torch.zeros((1, 16), device=f"cuda:{cuda_device}")
    rc = lib.mq_linear_noalloc(big.handle, xb.data_ptr(), 1, 16416, None, yb.data_ptr(), 16, sh)
    assert rc == mq._lib.MQ_ERR_INVALID and "16384" in mq._lib.last_error()
    assert lib.mq_linear_noalloc(wt.handle, xd.data_ptr(), 0, 1024, None, y.data_ptr(), 2048, sh) == 0
