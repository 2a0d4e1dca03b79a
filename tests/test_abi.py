"""CPU tests of the product library: it loads, exports every symbol the C
header declares, and its host codec (mq_quantize / mq_dequantize) is
byte-identical to the oracle, with the reference's error behaviour.
No compute is sent to a GPU here."""
from __future__ import annotations

import ctypes as C
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, case_names
from oracle import NAMES, Q4_0, Q4_1, Q8_0, QTYPES

HEADER = ROOT / "include" / "mq_b200.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(mq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(mq):
    import subprocess

    syms = declared_symbols()
    assert len(syms) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", str(mq.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (\w+)$", out, flags=re.M))
    missing = [s for s in syms if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    from mini_ai_b200._lib import SIGNATURES

    assert set(SIGNATURES) == set(syms), "ctypes signature table out of sync with the header"


def test_version_and_sizes(mq):
    lib = mq.lib()
    assert b"sm_100a" in lib.mq_version()
    assert lib.mq_quantized_bytes(Q8_0, 4096, 4096) == 4096 * 128 * 34
    assert lib.mq_quantized_bytes(Q4_0, 14336, 4096) == 33030144
    assert lib.mq_quantized_bytes(Q4_1, 3, 37) == 3 * 2 * 20
    assert lib.mq_quantized_bytes(7, 3, 37) == 0
    assert lib.mq_quantized_bytes(Q8_0, 0, 37) == 0


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_host_quantize_matches_golden(mq, golden, q):
    g = golden[q]
    for name in case_names(g) + ["edge"]:
        w = g[f"{name}/w"]
        for threads in (1, 3, 0):
            s = mq.QuantizeTensor(w, q, threads=threads)
            assert np.array_equal(s.bytes, g[f"{name}/blocks"]), (name, threads)
        if name != "edge":
            d = mq.DequantizeTensor(s)
            assert np.array_equal(d.view(np.uint32), g[f"{name}/dequant"].view(np.uint32)), name


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_host_quantize_matches_oracle_random(mq, oracle, q):
    rng = np.random.default_rng(100 + q)
    for rows, cols, scale in [(1, 1, 1.0), (3, 31, 1e-7), (17, 33, 0.02), (64, 4096, 0.02), (5, 4097, 50.0),
                              (8, 200, 1e-3)]:
        w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
        if cols > 8:
            w[0, :8] = [0.5, -0.5, 1.5, -2.5, 0.0, -0.0, 3.5, -3.5]  # exact ties and signed zeros
        assert np.array_equal(mq.QuantizeTensor(w, q, threads=4).bytes, oracle.quantize(q, w)), (rows, cols)


def test_quantize_errors_like_reference(mq):
    g = np.load(GOLDEN / "golden_errors.npz")
    inv = {v: k for k, v in NAMES.items()}
    for key in g.files:
        if key.endswith("/w"):
            continue
        case, tname = key.split("/")
        expected = str(g[key])
        w = g[f"{case}/w"]
        if expected == "ok":
            mq.QuantizeTensor(w, inv[tname])
            continue
        with pytest.raises(RuntimeError) as exc:
            mq.QuantizeTensor(w, inv[tname])
        assert expected.split(": ", 1)[1] in str(exc.value), (key, str(exc.value))
    with pytest.raises(ValueError):
        mq.QuantizeTensor(np.zeros(32, np.float32), Q8_0)  # not a matrix
    with pytest.raises(ValueError):
        mq.QuantizeTensor(np.zeros((2, 32), np.float32), 7)  # unknown type


def test_first_error_in_row_major_order(mq):
    """With an offset overflow in an early block and a NaN later, the reference
    throws for the earlier block; so must every thread split."""
    w = np.zeros((8, 64), np.float32)
    w[1, 40] = -1.0e5  # Q4_1 offset overflow in row 1, block 1
    w[6, 3] = np.nan
    for threads in (1, 2, 8):
        with pytest.raises(RuntimeError, match="offset exceeds"):
            mq.QuantizeTensor(w, Q4_1, threads=threads)
    w[1, 40] = 0.0
    with pytest.raises(RuntimeError, match="non-finite"):
        mq.QuantizeTensor(w, Q4_1, threads=3)


def test_tensor_from_quantized_checks(mq):
    with pytest.raises(RuntimeError, match="size mismatch"):
        mq.TensorFromQuantized(np.zeros(33, np.uint8), 1, 32, Q8_0)
    with pytest.raises(ValueError):
        mq.TensorFromQuantized(np.zeros(34, np.uint8), 0, 32, Q8_0)
    s = mq.TensorFromQuantized(np.zeros(34, np.uint8), 1, 32, Q8_0)
    assert s.rows == 1 and s.cols == 32


def test_known_answer_block_through_product(mq):
    """tests/test_compute.cc:54-68 through the product's decoder."""
    blk = np.zeros(18, np.uint8)
    blk[1] = 0x3C
    blk[2:] = 0xF0
    d = mq.DequantizeTensor(mq.TensorFromQuantized(blk, 1, 32, Q4_0))[0]
    assert d[0] == -8.0 and d[16] == 7.0


def test_abi_validation_without_device(mq):
    lib = mq.lib()
    assert lib.mq_linear(None, None, 1, 32, None, None, 32, None) == mq._lib.MQ_ERR_INVALID
    assert b"null weight" in lib.mq_last_error()
    out = C.c_void_p()
    blocks = np.zeros(34, np.uint8)
    rc = lib.mq_weight_create(0, Q8_0, 1, 32, blocks.ctypes.data, 33, 0, None, C.byref(out))
    assert rc == mq._lib.MQ_ERR_SIZE and not out.value
    rc = lib.mq_weight_create(0, 5, 1, 32, blocks.ctypes.data, 34, 0, None, C.byref(out))
    assert rc == mq._lib.MQ_ERR_INVALID
    rc = lib.mq_weight_shard_create(0, Q8_0, 2, 32, 1, 1, blocks.ctypes.data, 68, 0, None, C.byref(out))
    assert rc == mq._lib.MQ_ERR_INVALID
    offs = (C.c_int * 3)(0, 5, 3)
    assert lib.mq_linear_ragged(None, None, offs, 2, 32, None, None, 32, None) == mq._lib.MQ_ERR_INVALID
    buf = C.create_string_buffer(256)
    lib.mq_device_info(buf, 256)
    assert buf.value.startswith(b"CUDA devices=")
    assert lib.mq_set_path(1) == 0 and lib.mq_set_path(0) == 1
