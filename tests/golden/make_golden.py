"""Generate the golden fixtures of the quantized-linear path from the reference itself.

Runs the reference's own C++ sources (oracle/_ref/libmini_ai_ref.so, built by
oracle/Makefile from the mini_ai tree) on seeded inputs and stores inputs and
outputs as small .npz files next to this script:

* ``golden_<type>.npz`` — for several shapes (tail blocks included): the F32
  weight, the bytes QuantizeTensor packs, DequantizeTensor's output, the
  activations and LinearDispatch(kThreadedSimd)'s output per activation row.
* ``golden_edge.npz`` — quantizer edge blocks (zeros, signed zeros, exact
  ties, fp16-boundary and subnormal scales, first-of-equal-magnitude peaks)
  with the packed bytes, and the inputs on which QuantizeTensor throws.
* ``golden_fp16.npz`` — HalfToFloat over all 65536 inputs and FloatToHalf
  over a seeded sample of fp32 bit patterns plus every boundary class.

Usage (where the reference tree exists): python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import NAMES, QTYPES, Reference, build  # noqa: E402

# (rows, cols, activation rows, seed). cols 37 and 86 come from the reference's
# own tests (tests/test_compute.cc:30-52, models/tiny hidden_dim 86).
SHAPES = [(41, 37, 1, 0), (16, 86, 3, 1), (5, 4097, 2, 2), (33, 64, 4, 3), (12, 320, 16, 4)]


def sincos_case():
    """The reference test's inputs: x[i] = sin(i), W[i] = cos(i) * 0.1, 41 x 37."""
    x = np.sin(np.arange(37, dtype=np.float32)).astype(np.float32)[None, :]
    w = (np.cos(np.arange(41 * 37, dtype=np.float32)) * np.float32(0.1)).astype(np.float32).reshape(41, 37)
    return w, x


def edge_blocks(q: int):
    """Rows of 32 values that stress the packing rules (the fp16-boundary row
    is sized so that the type's scale lands exactly on the largest fp16)."""
    rows = []
    z = np.zeros(32, np.float32)
    rows.append(z.copy())                                   # all zero
    rows.append(-z)                                         # all negative zero
    t = np.arange(32, dtype=np.float32) - 15.5              # exact .5 ties after scaling
    rows.append(t)
    rows.append(t * np.float32(127.0 / 16.0))
    a = np.zeros(32, np.float32); a[3] = -2.0; a[9] = 2.0   # equal magnitude: first wins
    rows.append(a)
    b = np.zeros(32, np.float32); b[5] = 2.0; b[20] = -2.0
    rows.append(b)
    top = {8: 127.0, 2: 8.0, 3: 15.0}[q]
    rows.append(np.full(32, 65504.0 * top, np.float32))    # scale at the fp16 maximum
    rows.append(np.linspace(-1e-6, 1e-6, 32).astype(np.float32))   # subnormal fp16 scales
    rows.append(np.linspace(-3e-8, 2e-8, 32).astype(np.float32))   # scales round to 0
    rows.append(np.full(32, -1.0, np.float32))                     # Q4_1: min < 0 = max
    rows.append(np.full(32, 3.0, np.float32))                      # Q4_1: min clamped to 0
    rows.append(np.float32(7.0) * np.sign(np.sin(np.arange(32, dtype=np.float32))).astype(np.float32))
    return np.stack(rows).astype(np.float32)


def error_inputs():
    """(name, matrix) pairs on which QuantizeTensor throws for every type."""
    inf = np.zeros((1, 32), np.float32); inf[0, 7] = np.inf
    nan = np.zeros((2, 40), np.float32); nan[1, 33] = np.nan
    big = np.zeros((1, 32), np.float32); big[0, 0] = 3.0e38; big[0, 1] = -3.0e38  # overflows every scale
    low = np.zeros((1, 32), np.float32); low[0, 2] = -1.0e5   # Q4_1 min overflows fp16, scales do not
    return [("inf", inf), ("nan", nan), ("overflow", big), ("offset", low)]


def main() -> None:
    build()
    ref = Reference()
    for q in QTYPES:
        out = {}
        w, x = sincos_case()
        cases = [("sincos", w, x)]
        for rows, cols, m, seed in SHAPES:
            rng = np.random.default_rng(1000 * q + seed)
            cases.append((f"r{rows}c{cols}", (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32),
                          rng.standard_normal((m, cols)).astype(np.float32)))
        for name, w, x in cases:
            rows, cols = w.shape
            blocks = ref.quantize(q, w)
            out[f"{name}/w"] = w
            out[f"{name}/blocks"] = blocks
            out[f"{name}/dequant"] = ref.dequantize(q, blocks, rows, cols)
            out[f"{name}/x"] = x
            out[f"{name}/y"] = ref.linear(q, blocks, rows, cols, x, threads=3)
        e = edge_blocks(q)
        out["edge/w"] = e
        out["edge/blocks"] = ref.quantize(q, e)
        np.savez_compressed(HERE / f"golden_{NAMES[q]}.npz", **out)

    errs = {}
    for name, w in error_inputs():
        errs[f"{name}/w"] = w
        for q in QTYPES:
            try:
                ref.quantize(q, w)
                errs[f"{name}/{NAMES[q]}"] = np.array("ok")
            except RuntimeError as exc:
                errs[f"{name}/{NAMES[q]}"] = np.array(str(exc))
    np.savez_compressed(HERE / "golden_errors.npz", **errs)

    rng = np.random.default_rng(7)
    specials = [0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00001, 0x7F7FFFFF,
                0x477FEFFF, 0x477FF000, 0x477FF001, 0x38800000, 0x387FFFFF, 0x33800000, 0x33000000,
                0x33000001, 0x32FFFFFF, 0x337FFFFF, 0x3F800000, 0x3F801000, 0x3F803000, 0x3F801001]
    sample = np.concatenate([np.array(specials, np.uint32),
                             rng.integers(0, 2 ** 32, size=1 << 16, dtype=np.uint64).astype(np.uint32),
                             np.arange(0x33000000, 0x33000000 + 4096, dtype=np.uint32),
                             np.arange(0x38000000, 0x38000000 + 4096, dtype=np.uint32),
                             np.arange(0x477FE000, 0x477FE000 + 8192, dtype=np.uint32)])
    f2h = np.concatenate([ref.float_to_half_range(int(v), 1) for v in sample])
    np.savez_compressed(HERE / "golden_fp16.npz", h2f=ref.half_to_float_all(), f2h_in=sample, f2h_out=f2h)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
