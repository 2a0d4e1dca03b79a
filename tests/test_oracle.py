"""Pins the CPU oracle (oracle/mq_oracle.c) before anything is checked against it.

* golden fixtures produced by the reference's own sources (tests/golden);
* the reference test-suite's known answers (tests/test_compute.cc:54-68);
* an independent NumPy packer of the GGUF block layout (the format the
  reference's CLI regression writes, scripts/test_cli.py:62-80), decoded by the oracle;
* the reference build itself, exhaustively over fp16/fp32, where it is present.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import case_names
from oracle import NAMES, Q4_0, Q4_1, Q8_0, QTYPES


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_oracle_matches_golden(oracle, golden, q):
    g = golden[q]
    for name in case_names(g):
        w, blocks, x = g[f"{name}/w"], g[f"{name}/blocks"], g[f"{name}/x"]
        rows, cols = w.shape
        assert np.array_equal(oracle.quantize(q, w), blocks), name
        assert np.array_equal(oracle.dequantize(q, blocks, rows, cols).view(np.uint32),
                              g[f"{name}/dequant"].view(np.uint32)), name
        y = oracle.linear(q, blocks, rows, cols, x, threads=2)
        assert np.array_equal(y.view(np.uint32), g[f"{name}/y"].view(np.uint32)), name
    assert np.array_equal(oracle.quantize(q, g["edge/w"]), g["edge/blocks"])


def test_oracle_errors_match_golden(oracle):
    from conftest import GOLDEN
    from oracle import OracleError

    g = np.load(GOLDEN / "golden_errors.npz")
    for key in g.files:
        if key.endswith("/w"):
            continue
        case, tname = key.split("/")
        q = {v: k for k, v in NAMES.items()}[tname]
        expected = str(g[key])
        if expected == "ok":
            oracle.quantize(q, g[f"{case}/w"])
        else:
            with pytest.raises(OracleError):
                oracle.quantize(q, g[f"{case}/w"])


def test_known_answer_q4_0_block(oracle):
    """tests/test_compute.cc:54-68: scale 0x3c00 (1.0), every byte 0xF0."""
    blk = np.zeros(18, np.uint8)
    blk[1] = 0x3C
    blk[2:] = 0xF0
    d = oracle.dequantize(Q4_0, blk, 1, 32)[0]
    assert d[0] == -8.0 and d[16] == 7.0
    assert np.all(d[:16] == -8.0) and np.all(d[16:] == 7.0)
    assert oracle.lib.oracle_half_to_float(1) == np.ldexp(np.float32(1), -24)
    assert oracle.lib.oracle_float_to_half(float(np.ldexp(np.float32(1), -24))) == 1


def test_fp16_tables_match_golden(oracle):
    from conftest import GOLDEN

    g = np.load(GOLDEN / "golden_fp16.npz")
    assert np.array_equal(oracle.half_to_float_all().view(np.uint32), g["h2f"].view(np.uint32))
    got = np.array([oracle.float_to_half_range(int(b), 1)[0] for b in g["f2h_in"]], dtype=np.uint16)
    assert np.array_equal(got, g["f2h_out"])


def test_fp16_against_numpy(oracle):
    """Independent RNE conversion: NumPy's float16 cast, on every non-NaN value of a
    large stride through the fp32 bit space plus the whole subnormal-half range."""
    starts = list(range(0, 1 << 32, 1 << 26)) + [0x33000000, 0x38000000, 0xB3000000, 0xB8000000]
    for s in starts:
        n = 1 << 16
        bits = (np.arange(n, dtype=np.uint64) + s).astype(np.uint32)
        f = bits.view(np.float32)
        got = oracle.float_to_half_range(s, n)
        with np.errstate(over="ignore"):
            want = f.astype(np.float16).view(np.uint16)
        ok = ~np.isnan(f)
        assert np.array_equal(got[ok], want[ok]), hex(s)
        assert np.all((got[~ok] & 0x7FFF) == 0x7E00)
    h = np.arange(65536, dtype=np.uint16)
    hf = h.view(np.float16).astype(np.float32)
    got = oracle.half_to_float_all()
    ok = ~np.isnan(hf)
    assert np.array_equal(got[ok].view(np.uint32), hf[ok].view(np.uint32))
    assert np.all(got[~ok].view(np.uint32) == 0x7FC00000)


def _numpy_pack(q: int, w: np.ndarray):
    """Independent block packer for the GGUF layout (rint rounding, plain block
    min for Q4_1), returning (bytes, values those bytes decode to)."""
    blocks, dec = [], []
    for blk in w.reshape(-1, 32).astype(np.float32):
        if q == Q8_0:
            d = np.float16(np.max(np.abs(blk)) / 127)
            qv = np.clip(np.rint(blk / np.float32(d)), -127, 127).astype(np.int8) if d else np.zeros(32, np.int8)
            blocks.append(d.tobytes() + qv.tobytes())
            dec.append(qv.astype(np.float32) * np.float32(d))
        else:
            m = np.float16(np.min(blk)) if q == Q4_1 else np.float16(0)
            d = np.float16((np.max(blk) - np.min(blk)) / 15) if q == Q4_1 else np.float16(
                blk[np.argmax(np.abs(blk))] / -8)
            qv = np.rint((blk - np.float32(m)) / np.float32(d)) if d else np.zeros(32)
            qv = np.clip(qv + (8 if q == Q4_0 else 0), 0, 15).astype(np.uint8)
            blocks.append(d.tobytes() + (m.tobytes() if q == Q4_1 else b"") + (qv[:16] | qv[16:] << 4).tobytes())
            dec.append((qv.astype(np.float32) - (8 if q == Q4_0 else 0)) * np.float32(d) + np.float32(m))
    return np.frombuffer(b"".join(blocks), np.uint8), np.concatenate(dec).reshape(w.shape)


@pytest.mark.parametrize("q", QTYPES, ids=lambda q: NAMES[q])
def test_layout_against_independent_packer(oracle, q):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((9, 96)) * 0.3).astype(np.float32)
    blocks, decoded = _numpy_pack(q, w)
    assert np.array_equal(oracle.dequantize(q, blocks, 9, 96), decoded)


def test_thread_count_invariance(oracle, golden):
    g = golden[Q4_1]
    w, blocks, x = g["r16c86/w"], g["r16c86/blocks"], g["r16c86/x"]
    a = oracle.linear(Q4_1, blocks, 16, 86, x, threads=1)
    b = oracle.linear(Q4_1, blocks, 16, 86, x, threads=3)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_against_reference_build(oracle, reference):
    """Exhaustive fp32 -> fp16 over all 2^32 inputs, and random matrices."""
    assert np.array_equal(oracle.half_to_float_all().view(np.uint32), reference.half_to_float_all().view(np.uint32))
    chunk = 1 << 24
    for s in range(0, 1 << 32, chunk):
        assert np.array_equal(oracle.float_to_half_range(s, chunk), reference.float_to_half_range(s, chunk)), hex(s)
    rng = np.random.default_rng(5)
    for q in QTYPES:
        for rows, cols in [(3, 1), (7, 31), (5, 33), (19, 250)]:
            w = (rng.standard_normal((rows, cols)) * rng.choice([1e-6, 0.02, 3.0])).astype(np.float32)
            a, b = oracle.quantize(q, w), reference.quantize(q, w)
            assert np.array_equal(a, b), (q, rows, cols)
            x = rng.standard_normal((2, cols)).astype(np.float32)
            assert np.array_equal(oracle.linear(q, a, rows, cols, x).view(np.uint32),
                                  reference.linear(q, b, rows, cols, x, threads=2).view(np.uint32))
