"""ORACLE — CPU checkers for the quantized-linear path (test infrastructure only).

Two independent CPU implementations, loaded with ctypes:

* ``Oracle``    — ``oracle/mq_oracle.c``, a plain-C restatement of the
  reference algorithm (src/quantized_tensor.cc:13-206).
* ``Reference`` — ``oracle/_ref/libmini_ai_ref.so``, the reference's own C++
  sources (src/quantized_tensor.cc, src/matmul_optimized.cc,
  src/thread_pool.cc, src/tensor.cc) compiled unmodified by oracle/Makefile.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
use this package, and only as the checker or the timed CPU baseline; the
product path (``mini_ai_b200``) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libmq_oracle.so"
REF_SO = HERE / "_ref" / "libmini_ai_ref.so"

Q8_0, Q4_0, Q4_1 = 8, 2, 3
QTYPES = (Q8_0, Q4_0, Q4_1)
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20}
NAMES = {Q8_0: "q8_0", Q4_0: "q4_0", Q4_1: "q4_1"}


def quantized_bytes(qtype: int, rows: int, cols: int) -> int:
    return rows * ((cols + 31) // 32) * BLOCK_BYTES[qtype]


# Where the read-only mini_ai checkout lives when the checker is built
# (MINI_AI_REF overrides it); the GPU hosts only use the prebuilt files.
DEFAULT_REFERENCE = "/root/reference"


def reference_root() -> str | None:
    root = os.environ.get("MINI_AI_REF") or DEFAULT_REFERENCE
    return root if (Path(root) / "src" / "quantized_tensor.cc").exists() else None


def build(reference_root_dir: str | None = None) -> None:
    """Compile the C restatement (and the reference build when its sources exist)."""
    env = dict(os.environ)
    root = reference_root_dir or reference_root()
    if root:
        env["REF"] = root
    else:
        env.pop("REF", None)
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


class OracleError(RuntimeError):
    pass


class Oracle:
    """ctypes view of oracle/mq_oracle.c."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            build()
        lib = C.CDLL(str(path))
        lib.oracle_half_to_float.restype = C.c_float
        lib.oracle_half_to_float.argtypes = [C.c_uint16]
        lib.oracle_float_to_half.restype = C.c_uint16
        lib.oracle_float_to_half.argtypes = [C.c_float]
        lib.oracle_quantize.restype = C.c_int
        lib.oracle_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]
        lib.oracle_dequantize.restype = C.c_int
        lib.oracle_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p]
        lib.oracle_dot_row.restype = C.c_float
        lib.oracle_dot_row.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.oracle_linear.restype = C.c_int
        lib.oracle_linear.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                      C.c_int, C.c_void_p, C.c_int, C.c_int]
        lib.oracle_float_to_half_range.restype = None
        lib.oracle_float_to_half_range.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t]
        lib.oracle_half_to_float_batch.restype = None
        lib.oracle_half_to_float_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        self.lib = lib

    def quantize(self, qtype: int, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(quantized_bytes(qtype, rows, cols), dtype=np.uint8)
        rc = self.lib.oracle_quantize(qtype, _ptr(w), rows, cols, _ptr(out), out.nbytes)
        if rc:
            raise OracleError(f"oracle_quantize failed ({rc})")
        return out

    def dequantize(self, qtype: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty((rows, cols), dtype=np.float32)
        rc = self.lib.oracle_dequantize(qtype, _ptr(blocks), blocks.nbytes, rows, cols, _ptr(out))
        if rc:
            raise OracleError(f"oracle_dequantize failed ({rc})")
        return out

    def linear(self, qtype: int, blocks: np.ndarray, rows: int, cols: int, x: np.ndarray,
               threads: int = 1) -> np.ndarray:
        """y[m, n] = dot(row n, x[m]) with the reference's sequential fp32 order."""
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        m = x.shape[0]
        y = np.empty((m, rows), dtype=np.float32)
        rc = self.lib.oracle_linear(qtype, _ptr(blocks), blocks.nbytes, rows, cols, _ptr(x), m, cols, _ptr(y),
                                    rows, threads)
        if rc:
            raise OracleError(f"oracle_linear failed ({rc})")
        return y

    def float_to_half_range(self, start: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint16)
        self.lib.oracle_float_to_half_range(start, _ptr(out), n)
        return out

    def half_to_float_all(self) -> np.ndarray:
        src = np.arange(65536, dtype=np.uint16)
        out = np.empty(65536, dtype=np.float32)
        self.lib.oracle_half_to_float_batch(_ptr(src), _ptr(out), 65536)
        return out


class Reference:
    """ctypes view of the reference's own sources (oracle/_ref/libmini_ai_ref.so)."""

    def __init__(self, path: Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (needs the reference sources; run make -C oracle)")
        lib = C.CDLL(str(path))
        lib.ref_last_error.restype = C.c_char_p
        lib.ref_half_to_float.restype = C.c_float
        lib.ref_half_to_float.argtypes = [C.c_uint16]
        lib.ref_float_to_half.restype = C.c_uint16
        lib.ref_float_to_half.argtypes = [C.c_float]
        lib.ref_float_to_half_range.restype = None
        lib.ref_float_to_half_range.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t]
        lib.ref_half_to_float_batch.restype = None
        lib.ref_half_to_float_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        lib.ref_quantize.restype = C.c_int
        lib.ref_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]
        lib.ref_dequantize.restype = C.c_int
        lib.ref_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p]
        lib.ref_weight_create.restype = C.c_void_p
        lib.ref_weight_create.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_int, C.c_int]
        lib.ref_weight_destroy.restype = None
        lib.ref_weight_destroy.argtypes = [C.c_void_p]
        lib.ref_set_threads.restype = C.c_int
        lib.ref_set_threads.argtypes = [C.c_uint]
        lib.ref_linear.restype = C.c_int
        lib.ref_linear.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
        self.lib = lib

    def error(self) -> str:
        return self.lib.ref_last_error().decode()

    def quantize(self, qtype: int, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(quantized_bytes(qtype, rows, cols), dtype=np.uint8)
        rc = self.lib.ref_quantize(qtype, _ptr(w), rows, cols, _ptr(out), out.nbytes)
        if rc:
            raise OracleError(f"QuantizeTensor threw: {self.error()}")
        return out

    def dequantize(self, qtype: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty((rows, cols), dtype=np.float32)
        rc = self.lib.ref_dequantize(qtype, _ptr(blocks), blocks.nbytes, rows, cols, _ptr(out))
        if rc:
            raise OracleError(f"DequantizeTensor threw: {self.error()}")
        return out

    def weight(self, qtype: int, blocks: np.ndarray, rows: int, cols: int) -> "RefWeight":
        return RefWeight(self, qtype, blocks, rows, cols)

    def linear(self, qtype: int, blocks: np.ndarray, rows: int, cols: int, x: np.ndarray,
               threads: int = 0) -> np.ndarray:
        with self.weight(qtype, blocks, rows, cols) as w:
            return w.linear(x, threads)

    def float_to_half_range(self, start: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint16)
        self.lib.ref_float_to_half_range(start, _ptr(out), n)
        return out

    def half_to_float_all(self) -> np.ndarray:
        src = np.arange(65536, dtype=np.uint16)
        out = np.empty(65536, dtype=np.float32)
        self.lib.ref_half_to_float_batch(_ptr(src), _ptr(out), 65536)
        return out


class RefWeight:
    """A packed weight wrapped once as a reference Tensor (TensorFromQuantized)."""

    def __init__(self, ref: Reference, qtype: int, blocks: np.ndarray, rows: int, cols: int):
        self.ref, self.rows, self.cols = ref, rows, cols
        self._blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        self.handle = ref.lib.ref_weight_create(qtype, _ptr(self._blocks), self._blocks.nbytes, rows, cols)
        if not self.handle:
            raise OracleError(f"TensorFromQuantized threw: {ref.error()}")

    def linear(self, x: np.ndarray, threads: int = 0) -> np.ndarray:
        """LinearDispatch(x[m], W, kThreadedSimd) for each activation row m."""
        x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        y = np.empty((x.shape[0], self.rows), dtype=np.float32)
        if self.ref.lib.ref_set_threads(threads):
            raise OracleError(self.ref.error())
        rc = self.ref.lib.ref_linear(C.c_void_p(self.handle), _ptr(x), x.shape[0], x.shape[1], _ptr(y), self.rows)
        if rc:
            raise OracleError(f"LinearDispatch threw: {self.ref.error()}")
        return y

    def close(self) -> None:
        if self.handle:
            self.ref.lib.ref_weight_destroy(C.c_void_p(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def reference_available() -> bool:
    return REF_SO.exists()
