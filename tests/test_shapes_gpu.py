"""GPU parity at the shapes the benchmark configurations name but the per-type
tests do not reach, and on activations with outliers.

* 70B-shape FFN and lm_head (the row-sharded configuration's matrices: Q4_0
  28672x8192 and 8192x28672, Q8_0 128256x8192) at M = 1 and 32, and the
  Llama-3-8B projections not covered elsewhere (k/v 1024x4096 for every type,
  lm_head Q8_0 128256x4096): weights are generated and packed on the device
  (the device quantizer is bit-exact with the reference's QuantizeTensor,
  tests/test_linear_gpu.py), and a spread of output rows is checked against
  the oracle (rows are independent, so a row sample checks those rows
  exactly).
* Activation outliers: real hidden states carry a few features 10^3..10^4
  times the median. Every 256-wide K step gets one such entry and half of the
  weight rows are zero at those columns, so the condition-aware bound is set
  by the small activations alone; every decode kernel (automatic and forced)
  must stay within it.

Tolerance (tests/conftest.py): max|dy|/max|y| <= 1e-4 and
|dy_i| <= 1e-4 * sum_k |w_ik x_k| + 1e-6 for every element.
Reference: QuantizedDotRow, src/quantized_tensor.cc:161-191; the callers'
shapes, src/forward.cc:56-63, 106-110, 148-153.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from conftest import abs_dot_bound, assert_linear_close
from oracle import BLOCK_BYTES, NAMES, Q4_0, Q4_1, Q8_0, QTYPES

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


def _torch():
    import torch

    return torch


def _dev(a, device):
    return _torch().from_numpy(np.ascontiguousarray(a)).to(f"cuda:{device}")


def _device_weight(mq, q, rows, cols, seed, device):
    """N(0, 0.02) weights generated on the device and packed by the device quantizer.
    Returns the uploaded handle and the GGUF block stream (device tensor [rows, row_bytes])."""
    torch = _torch()
    d = f"cuda:{device}"
    g = torch.Generator(device=d)
    g.manual_seed(seed)
    w32 = torch.randn((rows, cols), generator=g, device=d, dtype=torch.float32).mul_(0.02)
    row_bytes = ((cols + 31) // 32) * BLOCK_BYTES[q]
    blocks = torch.empty((rows, row_bytes), dtype=torch.uint8, device=d)
    rc = mq.lib().mq_quantize_device(device, q, w32.data_ptr(), rows, cols, blocks.data_ptr(), blocks.numel(),
                                     C.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    assert rc == 0, mq._lib.last_error()
    del w32
    w = mq.CudaWeight.from_device_blocks(blocks.view(-1), q, rows, cols, device=device)
    return w, blocks


def _check_sampled_rows(mq, oracle, q, w, blocks, x, device, n_pick=192, seed=0, path=0):
    torch = _torch()
    rows, cols = blocks.shape[0], x.shape[1]
    prev = mq.set_path(path)
    try:
        y = w.linear(_dev(x, device))
        torch.cuda.synchronize(device)
    finally:
        mq.set_path(prev)
    y = y.cpu().numpy()
    rng = np.random.default_rng(seed)
    pick = np.sort(np.concatenate([[0, rows - 1], rng.choice(np.arange(1, rows - 1), n_pick - 2, replace=False)]))
    sub = blocks[torch.from_numpy(pick).to(blocks.device)].cpu().numpy().reshape(-1)
    y_ref = oracle.linear(q, sub, len(pick), cols, x, threads=THREADS)
    bound = abs_dot_bound(oracle.dequantize(q, sub, len(pick), cols), x)
    assert np.all(np.isfinite(y)), "non-finite output outside the checked rows"
    return assert_linear_close(y[:, pick], y_ref, bound)


@pytest.mark.parametrize("q,rows,cols", [(Q4_0, 28672, 8192), (Q4_0, 8192, 28672), (Q8_0, 128256, 8192)],
                         ids=["ffn_up_q4_0", "ffn_down_q4_0", "lm_head_q8_0"])
@pytest.mark.parametrize("m", [1, 32])
def test_70b_shapes_rows_checked(mq, oracle, cuda_device, q, rows, cols, m):
    w, blocks = _device_weight(mq, q, rows, cols, seed=rows + cols + q, device=cuda_device)
    x = np.random.default_rng(rows * 3 + m).standard_normal((m, cols), dtype=np.float32)
    _check_sampled_rows(mq, oracle, q, w, blocks, x, cuda_device, seed=m)
    w.close()


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
@pytest.mark.parametrize("m", [1, 4, 16])
def test_llama3_8b_kv_projection(mq, oracle, cuda_device, q, m):
    """k/v projections, 1024x4096 (8 KV heads x head_dim 128), checked on every row."""
    rng = np.random.default_rng(1024 + m + q)
    wf = (rng.standard_normal((1024, 4096)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(wf, q)
    x = rng.standard_normal((m, 4096)).astype(np.float32)
    w = mq.CudaWeight(s, device=cuda_device)
    y = w.linear(_dev(x, cuda_device)).cpu().numpy()
    y_ref = oracle.linear(q, s.bytes, 1024, 4096, x, threads=THREADS)
    assert_linear_close(y, y_ref, abs_dot_bound(oracle.dequantize(q, s.bytes, 1024, 4096), x))
    w.close()


@pytest.mark.parametrize("m", [1, 16])
def test_llama3_8b_lm_head_rows_checked(mq, oracle, cuda_device, m):
    w, blocks = _device_weight(mq, Q8_0, 128256, 4096, seed=128256, device=cuda_device)
    x = np.random.default_rng(77 + m).standard_normal((m, 4096), dtype=np.float32)
    _check_sampled_rows(mq, oracle, Q8_0, w, blocks, x, cuda_device, seed=m)
    w.close()


def _outlier_case(q, rows, cols, m, seed):
    """W ~ N(0, 0.02) with half of its rows zero at one column per 256-wide K
    step; x ~ N(0, 1) with that column set to +-10^U(3, 4)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    steps = (cols + 255) // 256
    cols_out = np.array([min(cols - 1, 256 * s + int(rng.integers(256))) for s in range(steps)])
    w[::2][:, cols_out] = 0.0
    x = rng.standard_normal((m, cols)).astype(np.float32)
    mag = np.power(10.0, rng.uniform(3.0, 4.0, size=(m, steps))).astype(np.float32)
    sign = np.where(rng.random((m, steps)) < 0.5, -1.0, 1.0).astype(np.float32)
    x[:, cols_out] = mag * sign
    return w, x


# Paths (mq_set_path): 0 automatic, 1 stream-K SIMT GEMV, 3 tcgen05 int8 decode, 4 tcgen05 fp16 decode,
# 5 SIMT dp4a GEMV, 6 tcgen05 scale-folded decode, 7 the same on CTA pairs.
OUTLIER_PATHS = {0: [1, 2, 4, 16, 32], 1: [1, 2, 4], 3: [1, 2, 3, 4], 4: [1, 5, 16, 32], 5: [1, 2, 3], 6: [5, 16, 32],
                 7: [5, 16, 32]}


@pytest.mark.parametrize("path", sorted(OUTLIER_PATHS), ids=lambda p: {0: "automatic", 1: "streamk_simt_gemv",
                                                                      3: "tcgen05_i8_decode", 4: "tcgen05_decode",
                                                                      5: "simt_dp4a_gemv", 6: "tcgen05_folded_decode",
                                                                      7: "tcgen05_folded_decode_cta_pairs"}[p])
@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_activation_outliers(mq, oracle, cuda_device, path, q):
    torch = _torch()
    for rows, cols in [(512, 4096), (256, 14336)]:
        for m in OUTLIER_PATHS[path]:
            wf, x = _outlier_case(q, rows, cols, m, seed=rows + m * 13 + q + path * 101)
            s = mq.QuantizeTensor(wf, q)
            w = mq.CudaWeight(s, device=cuda_device)
            prev = mq.set_path(path)
            try:
                y = w.linear(_dev(x, cuda_device))
                torch.cuda.synchronize(cuda_device)
            finally:
                mq.set_path(prev)
            y_ref = oracle.linear(q, s.bytes, rows, cols, x, threads=THREADS)
            bound = abs_dot_bound(oracle.dequantize(q, s.bytes, rows, cols), x)
            assert_linear_close(y.cpu().numpy(), y_ref, bound)
            w.close()
