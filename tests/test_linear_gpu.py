"""GPU parity of the quantized linear against the oracle, through the C ABI.

Every case runs the device path (libmq_b200.so) and compares it with the CPU
oracle on the same seeded inputs, using the tolerance defined in conftest:
max|dy|/max|y| <= 1e-4 and |dy_i| <= 1e-4 * sum_k |w_ik x_k| + 1e-6.
Byte-level results (device layout round trip, device quantizer) must be
bit-identical.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import abs_dot_bound, assert_linear_close, case_names
from oracle import NAMES, Q4_0, Q4_1, Q8_0, QTYPES

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


def _torch():
    import torch

    return torch


def dev(a, device=0):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{device}")


def gpu_linear(mq, storage, x, device=0, bias=None, path=0):
    torch = _torch()
    w = mq.CudaWeight(storage, device=device)
    prev = mq.set_path(path)
    try:
        y = w.linear(dev(x, device), bias=None if bias is None else dev(bias, device))
        torch.cuda.synchronize(device)
    finally:
        mq.set_path(prev)
    return y.cpu().numpy()


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_golden_cases(mq, golden, cuda_device, q):
    g = golden[q]
    for name in case_names(g):
        w, blocks, x, y_ref = g[f"{name}/w"], g[f"{name}/blocks"], g[f"{name}/x"], g[f"{name}/y"]
        rows, cols = w.shape
        s = mq.TensorFromQuantized(blocks, rows, cols, q)
        y = gpu_linear(mq, s, x, cuda_device)
        assert_linear_close(y, y_ref, abs_dot_bound(g[f"{name}/dequant"], x))


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_device_layout_round_trip(mq, golden, cuda_device, q):
    g = golden[q]
    for name in case_names(g) + ["edge"]:
        rows, cols = g[f"{name}/w"].shape
        blocks = g[f"{name}/blocks"]
        w = mq.CudaWeight(mq.TensorFromQuantized(blocks, rows, cols, q), device=cuda_device)
        assert np.array_equal(w.export().bytes, blocks), name
    rng = np.random.default_rng(3)
    big = (rng.standard_normal((1024, 4096)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(big, q)
    assert np.array_equal(mq.CudaWeight(s, device=cuda_device).export().bytes, s.bytes)


def _device_quantize(mq, q, w, device):
    import ctypes as C

    torch = _torch()
    src = dev(w, device)
    out = torch.zeros(mq.lib().mq_quantized_bytes(q, *w.shape), dtype=torch.uint8, device=f"cuda:{device}")
    rc = mq.lib().mq_quantize_device(device, q, src.data_ptr(), w.shape[0], w.shape[1], out.data_ptr(), out.numel(),
                                     C.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    return rc, out.cpu().numpy()


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_device_quantizer_bit_exact(mq, golden, oracle, cuda_device, q):
    g = golden[q]
    for name in case_names(g) + ["edge"]:
        rc, got = _device_quantize(mq, q, g[f"{name}/w"], cuda_device)
        assert rc == 0, mq._lib.last_error()
        assert np.array_equal(got, g[f"{name}/blocks"]), name
    rng = np.random.default_rng(21 + q)
    for rows, cols, scale in [(333, 4096, 0.02), (64, 4097, 1e-6), (7, 95, 40.0)]:
        w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
        w[0, :6] = [0.5, -0.5, 2.5, -0.0, 0.0, -3.5]
        rc, got = _device_quantize(mq, q, w, cuda_device)
        assert rc == 0
        assert np.array_equal(got, mq.QuantizeTensor(w, q).bytes)
        assert np.array_equal(got, oracle.quantize(q, w))


def test_device_quantizer_errors(mq, cuda_device):
    w = np.zeros((8, 64), np.float32)
    w[1, 40] = -1.0e5
    w[6, 3] = np.inf
    rc, _ = _device_quantize(mq, Q4_1, w, cuda_device)
    assert rc == mq._lib.MQ_ERR_RANGE and "offset" in mq._lib.last_error()
    rc, _ = _device_quantize(mq, Q8_0, w, cuda_device)
    assert rc == mq._lib.MQ_ERR_NONFINITE


def _llama_case(mq, oracle, q, rows, cols, m, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(w, q)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    y_ref = oracle.linear(q, s.bytes, rows, cols, x, threads=THREADS)
    bound = abs_dot_bound(oracle.dequantize(q, s.bytes, rows, cols), x)
    return s, x, y_ref, bound


@pytest.mark.parametrize("q,rows,cols", [(Q8_0, 4096, 4096), (Q4_0, 14336, 4096), (Q4_1, 14336, 4096),
                                         (Q4_0, 4096, 14336), (Q4_1, 4096, 14336), (Q8_0, 4096, 14336)])
@pytest.mark.parametrize("m", [1, 4, 16])
def test_llama_shapes(mq, oracle, cuda_device, q, rows, cols, m):
    s, x, y_ref, bound = _llama_case(mq, oracle, q, rows, cols, m, seed=rows + cols + m + q)
    stats = assert_linear_close(gpu_linear(mq, s, x, cuda_device), y_ref, bound)
    assert stats["max_rel"] < 1e-4


@pytest.mark.parametrize("m", [2, 3, 5, 7, 8, 9, 33])
def test_odd_activation_counts(mq, oracle, cuda_device, m):
    for q in QTYPES:
        s, x, y_ref, bound = _llama_case(mq, oracle, q, 300, 4097, m, seed=m * 7 + q)
        assert_linear_close(gpu_linear(mq, s, x, cuda_device), y_ref, bound)


def test_bias_strides_and_alignment(mq, oracle, cuda_device):
    torch = _torch()
    q, rows, cols, m = Q4_1, 257, 130, 3
    s, x, y_ref, bound = _llama_case(mq, oracle, q, rows, cols, m, seed=5)
    bias = np.linspace(-1, 1, rows).astype(np.float32)
    w = mq.CudaWeight(s, device=cuda_device)
    # strided, unaligned activations: x lives at column offset 1 of a wider buffer
    xbuf = torch.zeros((m, cols + 7), dtype=torch.float32, device=f"cuda:{cuda_device}")
    xbuf[:, 1:cols + 1] = dev(x, cuda_device)
    xv = xbuf[:, 1:cols + 1]
    ybuf = torch.full((m, rows + 5), 7.0, dtype=torch.float32, device=f"cuda:{cuda_device}")
    w.linear(xv, bias=dev(bias, cuda_device), out=ybuf[:, :rows])
    torch.cuda.synchronize()
    got = ybuf.cpu().numpy()
    assert_linear_close(got[:, :rows], y_ref + bias[None, :], bound + np.abs(bias)[None, :])
    assert np.all(got[:, rows:] == 7.0)  # nothing written past the output rows


def test_sharded_rows_are_slices_of_full(mq, oracle, cuda_device):
    """A row shard computes exactly the rows of the full matrix (bit-identical:
    at 1024 x 512 both launches give every (tile, K step) chunk its own CTA, so
    the sums run in the same order)."""
    torch = _torch()
    for q in QTYPES:
        s, x, y_ref, bound = _llama_case(mq, oracle, q, 1024, 512, 2, seed=9 + q)
        full = mq.CudaWeight(s, device=cuda_device).linear(dev(x, cuda_device)).cpu().numpy()
        parts = []
        for g in range(4):
            sh = mq.CudaWeight(s, device=cuda_device, row_range=(256 * g, 256 * (g + 1)))
            parts.append(sh.linear(dev(x, cuda_device)).cpu().numpy())
        torch.cuda.synchronize()
        assert np.array_equal(np.concatenate(parts, axis=1).view(np.uint32), full.view(np.uint32))
        assert_linear_close(full, y_ref, bound)


@pytest.mark.parametrize("m", [1, 16, 300], ids=["int8_decode", "folded_decode", "prefill_gemm"])
def test_large_shards_match_full_to_rounding(mq, oracle, cuda_device, m):
    """At Llama-3-8B FFN size the shards' launches split K differently from the
    whole weight's (more (tile, K step) chunks than SMs), so the sums run in a
    different order: every shard's rows must still match the full product
    within the parity tolerance (relative to sum_k |w_nk x_mk|)."""
    torch = _torch()
    rng = np.random.default_rng(4242 + m)
    rows, cols, q = 14336, 4096, Q4_0
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(w, q)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    xd = dev(x, cuda_device)
    full_w = mq.CudaWeight(s, device=cuda_device)
    full = full_w.linear(xd).cpu().numpy()
    full_w.close()
    bound = abs_dot_bound(oracle.dequantize(q, s.bytes, rows, cols), x)
    for G in (2, 8):
        R = rows // G
        parts = []
        for g in range(G):
            sh = mq.CudaWeight(s, device=cuda_device, row_range=(R * g, R * (g + 1)))
            parts.append(sh.linear(xd).cpu().numpy())
            sh.close()
        torch.cuda.synchronize()
        assert_linear_close(np.concatenate(parts, axis=1), full, bound)


def test_ragged_offsets(mq, oracle, cuda_device):
    import ctypes as C

    torch = _torch()
    lengths = [1, 7, 33, 64, 2, 5]
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    q = Q8_0
    s, x, y_ref, bound = _llama_case(mq, oracle, q, 96, 256, int(offsets[-1]), seed=17)
    w = mq.CudaWeight(s, device=cuda_device)
    xd = dev(x, cuda_device)
    y = torch.empty((int(offsets[-1]), 96), dtype=torch.float32, device=f"cuda:{cuda_device}")
    offs = (C.c_int * len(offsets))(*offsets.tolist())
    rc = mq.lib().mq_linear_ragged(w.handle, xd.data_ptr(), offs, len(lengths), 256, None, y.data_ptr(), 96,
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, mq._lib.last_error()
    torch.cuda.synchronize()
    assert_linear_close(y.cpu().numpy(), y_ref, bound)
    bad = (C.c_int * 3)(0, 5, 4)
    assert mq.lib().mq_linear_ragged(w.handle, xd.data_ptr(), bad, 2, 256, None, y.data_ptr(), 96, None) == -1


def test_deterministic_and_m_zero(mq, oracle, cuda_device):
    torch = _torch()
    s, x, _, _ = _llama_case(mq, oracle, Q4_0, 2048, 1024, 4, seed=1)
    w = mq.CudaWeight(s, device=cuda_device)
    xd = dev(x, cuda_device)
    a = w.linear(xd).cpu().numpy()
    b = w.linear(xd).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    y = torch.full((1, 2048), 3.0, device=f"cuda:{cuda_device}")
    assert mq.lib().mq_linear(w.handle, xd.data_ptr(), 0, 1024, None, y.data_ptr(), 2048, None) == 0
    assert float(y[0, 0]) == 3.0


def test_dimension_mismatch_raises(mq, cuda_device):
    s = mq.QuantizeTensor(np.ones((8, 64), np.float32), Q8_0)
    w = mq.CudaWeight(s, device=cuda_device)
    torch = _torch()
    with pytest.raises(RuntimeError, match="dimension mismatch"):
        w.linear(torch.zeros(63, device=f"cuda:{cuda_device}"))
    assert "CUDA devices=" in mq.CudaDeviceInfo()


PATHS = {1: "streamk_simt_gemv", 3: "tcgen05_i8_decode", 4: "tcgen05_decode", 2: "tcgen05_gemm", 5: "simt_dp4a_gemv",
         6: "tcgen05_folded_decode", 7: "tcgen05_folded_decode_cta_pairs"}


def _rows(path, rows):
    """The CTA-pair kernel (path 7) takes weights with an even number of 128-row
    tiles: 300 rows (3 tiles) become 200 (2 tiles, still a row tail)."""
    return 200 if path == 7 and rows == 300 else rows


@pytest.mark.parametrize("path", sorted(PATHS), ids=lambda p: PATHS[p])
@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_every_path_against_oracle(mq, oracle, cuda_device, path, q):
    """Each kernel, forced, on odd shapes: tail blocks (K % 32), row tails
    (N % 16, N % 128), activation counts around every tile edge."""
    ms = {1: [1, 2, 3, 4, 5, 9], 3: [1, 2, 3, 4, 5, 9], 4: [1, 2, 4, 5, 8, 9, 16, 17, 32, 33],
          2: [1, 7, 128, 129, 300], 5: [1, 2, 3, 5], 6: [1, 5, 8, 9, 16, 17, 32, 33],
          7: [1, 5, 8, 9, 16, 17, 32, 33]}[path]
    for rows, cols in [(_rows(path, 300), 4097), (136, 320), (1000, 96)]:
        for m in ms:
            s, x, y_ref, bound = _llama_case(mq, oracle, q, rows, cols, m, seed=rows * 7 + m + path)
            assert_linear_close(gpu_linear(mq, s, x, cuda_device, path=path), y_ref, bound)


def test_prefill_ragged_q8_0_rows_checked(mq, oracle, cuda_device):
    """The prefill configuration (W 11008x4096 and 4096x11008, 8 requests of
    lengths 1..512, M = 1456) through the tcgen05 GEMM; 192 output rows spread
    over the matrix are checked against the oracle (rows are independent)."""
    torch = _torch()
    lengths = [1, 7, 33, 64, 128, 200, 511, 512]
    m = sum(lengths)
    rng = np.random.default_rng(1456)
    for rows, cols in [(11008, 4096), (4096, 11008)]:
        w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
        s = mq.QuantizeTensor(w, Q8_0)
        x = rng.standard_normal((m, cols), dtype=np.float32)
        y = gpu_linear(mq, s, x, cuda_device, path=0)
        pick = np.sort(rng.choice(rows, 192, replace=False))
        bb = ((cols + 31) // 32) * 34
        sub = np.concatenate([s.bytes[r * bb:(r + 1) * bb] for r in pick])
        y_ref = oracle.linear(Q8_0, sub, len(pick), cols, x, threads=THREADS)
        bound = abs_dot_bound(oracle.dequantize(Q8_0, sub, len(pick), cols), x)
        assert_linear_close(y[:, pick], y_ref, bound)
        torch.cuda.synchronize()


def _silu(v):
    return v / (1.0 + np.exp(-v))


@pytest.mark.parametrize("path", [0] + sorted(PATHS), ids=lambda p: PATHS.get(p, "automatic"))
@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_swiglu_gate_up_against_oracle(mq, oracle, cuda_device, path, q):
    """mq_linear_swiglu = SwiGlu(Linear(x, w_gate), Linear(x, w_up)) (src/forward.cc:105-110,
    SwiGluKernel src/cuda_backend.cu:241-245) through every kernel's output epilogue, on odd
    shapes (tail blocks, row tails) and activation counts across the automatic path's regimes.
    Tolerance: the linear parity bound carried through silu (|silu'| < 1.1)."""
    torch = _torch()
    ms = {0: [1, 3, 16, 40], 1: [1, 3, 5], 3: [1, 2, 4, 5], 4: [1, 5, 16, 33], 2: [1, 129], 5: [1, 2, 3],
          6: [5, 16, 32], 7: [5, 16, 32]}[path]
    for rows, cols in [(_rows(path, 300), 4097), (1024, 4096)]:
        for m in ms:
            sg, x, g_ref, bg = _llama_case(mq, oracle, q, rows, cols, m, seed=rows * 3 + m + path * 11)
            su, _, _, _ = _llama_case(mq, oracle, q, rows, cols, m, seed=rows * 5 + m + path * 13)
            u_ref = oracle.linear(q, su.bytes, rows, cols, x, threads=THREADS)
            bu = abs_dot_bound(oracle.dequantize(q, su.bytes, rows, cols), x)
            g64, u64 = g_ref.astype(np.float64), u_ref.astype(np.float64)
            ref = _silu(g64) * u64
            bound = 1.1 * bg * np.abs(u64) + np.abs(_silu(g64)) * bu
            wg, wu = mq.CudaWeight(sg, device=cuda_device), mq.CudaWeight(su, device=cuda_device)
            prev = mq.set_path(path)
            try:
                y = mq.LinearSwiGlu(dev(x, cuda_device), wg, wu)
                # the same two products, unfused, with the reference's elementwise SwiGLU
                g = wg.linear(dev(x, cuda_device))
                u = wu.linear(dev(x, cuda_device))
                torch.cuda.synchronize(cuda_device)
            finally:
                mq.set_path(prev)
            assert_linear_close(y.cpu().numpy(), ref, bound)
            unfused = (g / (1.0 + torch.exp(-g)) * u).cpu().numpy()
            np.testing.assert_allclose(y.cpu().numpy(), unfused, rtol=2e-6, atol=1e-7)
            wg.close()
            wu.close()


def test_swiglu_validation(mq, cuda_device):
    """Shape and device mismatches are rejected before any launch."""
    rng = np.random.default_rng(5)
    a = mq.QuantizeTensor((rng.standard_normal((256, 128)) * 0.02).astype(np.float32), Q4_0)
    b = mq.QuantizeTensor((rng.standard_normal((128, 128)) * 0.02).astype(np.float32), Q4_0)
    wa, wb = mq.CudaWeight(a, device=cuda_device), mq.CudaWeight(b, device=cuda_device)
    with pytest.raises(mq.MQError, match="shape mismatch"):
        mq.LinearSwiGlu(dev(np.zeros((1, 128), np.float32), cuda_device), wa, wb)
    with pytest.raises(RuntimeError, match="dimension mismatch"):
        mq.LinearSwiGlu(dev(np.zeros((1, 64), np.float32), cuda_device), wa, wa)
    wa.close()
    wb.close()


@pytest.mark.parametrize("path", [0] + sorted(PATHS), ids=lambda p: PATHS.get(p, "automatic"))
@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_residual_add_against_oracle(mq, oracle, cuda_device, path, q):
    """mq_linear_residual = residual + (x · Wᵀ + bias) (the wo / w_down linear and ForwardCuda's
    AddKernel, src/cuda_backend.cu:236-240), in place and out of place, through every kernel:
    within the parity bound of the oracle, and bit-identical to the unfused product plus the add."""
    torch = _torch()
    ms = {0: [1, 3, 16, 40], 1: [1, 3, 5], 3: [1, 2, 4, 5], 4: [1, 5, 16, 33], 2: [1, 129], 5: [1, 2, 3],
          6: [5, 16, 32], 7: [5, 16, 32]}[path]
    for rows, cols in [(_rows(path, 300), 4097), (1024, 4096)]:
        for m in ms:
            s, x, y_ref, bound = _llama_case(mq, oracle, q, rows, cols, m, seed=rows * 17 + m + path * 7)
            rng = np.random.default_rng(rows + m)
            r = rng.standard_normal((m, rows)).astype(np.float32)
            b = (rng.standard_normal(rows) * 0.1).astype(np.float32)
            ref = r.astype(np.float64) + (y_ref.astype(np.float64) + b.astype(np.float64))
            w = mq.CudaWeight(s, device=cuda_device)
            prev = mq.set_path(path)
            try:
                xd, rd, bd = dev(x, cuda_device), dev(r, cuda_device), dev(b, cuda_device)
                y = w.linear_residual(xd, rd, bias=bd)
                unfused = rd + w.linear(xd, bias=bd)
                inplace = rd.clone()
                w.linear_residual(xd, inplace, bias=bd, out=inplace)
                torch.cuda.synchronize(cuda_device)
            finally:
                mq.set_path(prev)
            assert_linear_close(y.cpu().numpy(), ref, bound)
            assert torch.equal(y, unfused) and torch.equal(inplace, y)
            w.close()


def test_large_scales_fall_back_from_the_folded_kernel(mq, oracle, cuda_device):
    """Weights whose block scales would overflow fp16 once folded into the codes
    (|d * c| >= 65504: here Q8_0 blocks of magnitude ~1e5, d ~ 790) run on the
    unfolded fp16 decode kernel in automatic mode, and the folded kernel refuses
    them when forced; results stay within the parity bound."""
    torch = _torch()
    rng = np.random.default_rng(65504)
    rows, cols, m = 256, 512, 16
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[7, 40] = 1.0e5
    w[200, 300] = -0.9e5
    s = mq.QuantizeTensor(w, Q8_0)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    y_ref = oracle.linear(Q8_0, s.bytes, rows, cols, x, threads=THREADS)
    bound = abs_dot_bound(oracle.dequantize(Q8_0, s.bytes, rows, cols), x)
    assert_linear_close(gpu_linear(mq, s, x, cuda_device, path=0), y_ref, bound)
    # Prefill rows: the GEMM keeps such a weight on its bf16 form.
    xg = rng.standard_normal((64, cols)).astype(np.float32)
    bound_g = abs_dot_bound(oracle.dequantize(Q8_0, s.bytes, rows, cols), xg)
    assert_linear_close(gpu_linear(mq, s, xg, cuda_device, path=0),
                        oracle.linear(Q8_0, s.bytes, rows, cols, xg, threads=THREADS), bound_g)
    dw = mq.CudaWeight(s, device=cuda_device)
    prev = mq.set_path(6)
    try:
        with pytest.raises(mq.MQError, match="too large for the scale-folded"):
            dw.linear(dev(x, cuda_device))
    finally:
        mq.set_path(prev)
    torch.cuda.synchronize(cuda_device)
    dw.close()


@pytest.mark.parametrize("q", [Q8_0, Q4_0, Q4_1], ids=["q8_0", "q4_0", "q4_1"])
def test_gemm_rows_of_any_magnitude(mq, oracle, cuda_device, q):
    """Prefill GEMM (m > 32) with activation rows from 1e-30 to 1e30 in one
    launch, an all-zero row and a row with one large outlier: the scale-folded
    form (Q8_0, Q4_0) scales each row by its own power of two, the bf16 form
    (Q4_1) needs none; both stay within the parity bound."""
    rng = np.random.default_rng(1000 + q)
    rows, cols, m = 384, 1024, 70
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    s = mq.QuantizeTensor(w, q)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    x *= (10.0 ** np.linspace(-30, 30, m)).astype(np.float32)[:, None]
    x[5] = 0.0
    x[9, 100] = 3.0e4 * np.abs(x[9]).max()
    y_ref = oracle.linear(q, s.bytes, rows, cols, x, threads=THREADS)
    bound = abs_dot_bound(oracle.dequantize(q, s.bytes, rows, cols), x)
    got = gpu_linear(mq, s, x, cuda_device, path=0)
    assert np.all(got[5] == 0.0)
    assert_linear_close(got, y_ref, bound)


def test_cta_pair_kernel_rejects_odd_tile_counts(mq, cuda_device):
    """The CTA-pair kernel processes two 128-row tiles per pair: a weight with
    an odd number of tiles is refused when that kernel is forced, and the
    automatic path serves it."""
    torch = _torch()
    rng = np.random.default_rng(7)
    s = mq.QuantizeTensor((rng.standard_normal((300, 256)) * 0.02).astype(np.float32), Q4_0)  # 3 tiles
    dw = mq.CudaWeight(s, device=cuda_device)
    x = dev(rng.standard_normal((8, 256)).astype(np.float32), cuda_device)
    prev = mq.set_path(7)
    try:
        with pytest.raises(mq.MQError, match="even number of 128-row tiles"):
            dw.linear(x)
    finally:
        mq.set_path(prev)
    assert torch.isfinite(dw.linear(x)).all()
    dw.close()


def test_two_devices_one_process(mq, oracle):
    """One process drives two GPUs: every kernel class's first launch on the
    second device raises its shared-memory limit there (the attribute is per
    device), and both devices give bit-identical results within the oracle's
    bound."""
    torch = _torch()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rows, cols = 1024, 4096
    for q in QTYPES:
        for m in (1, 4, 16, 32, 64):  # int8 decode, folded decode, prefill GEMM
            s, x, y_ref, bound = _llama_case(mq, oracle, q, rows, cols, m, seed=q * 101 + m)
            ys = []
            for d in (1, 0):  # device 1 first: its first launches set that device's limits
                w = mq.CudaWeight(s, device=d)
                with torch.cuda.device(d):
                    ys.append(w.linear(dev(x, d)).cpu().numpy())
                w.close()
            assert np.array_equal(ys[0], ys[1])
            assert_linear_close(ys[0], y_ref, bound)
