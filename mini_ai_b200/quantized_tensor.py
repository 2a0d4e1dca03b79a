"""Host mirror of mini_ai's quantized-tensor and linear operator surface.

Same names, argument meaning and error behaviour as the reference
(include/mini_llama/quantized_tensor.h:10-26, include/mini_llama/matmul_dispatch.h:28,
include/mini_llama/backend.h:9-14), implemented over the mq_b200 C ABI:

* ``QuantizeTensor`` / ``DequantizeTensor`` / ``TensorFromQuantized`` run the
  engine's bit-exact host codec (``mq_quantize`` / ``mq_dequantize``).
* ``CudaWeight`` is ``CudaModelState::UploadWeight`` (src/cuda_backend.cu:275-283):
  a packed weight resident on one B200.
* ``LinearDispatch`` / ``Linear`` compute ``y = x · Wᵀ`` on the device through
  ``mq_linear``; unlike the reference (``[K]`` or ``[1, K]`` only,
  src/matmul_optimized.cc:153-161) any number of activation rows is accepted.

Errors follow the reference: ``ValueError`` where it throws
``std::invalid_argument``, ``RuntimeError`` where it throws ``std::runtime_error``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from enum import IntEnum

import numpy as np

from . import _lib
from ._lib import MQError, check, lib


class QuantType(IntEnum):
    """GGML type ids (include/mini_llama/quantized_tensor.h:10)."""

    kQ80 = _lib.MQ_Q8_0
    kQ40 = _lib.MQ_Q4_0
    kQ41 = _lib.MQ_Q4_1


_BLOCK_BYTES = {QuantType.kQ80: 34, QuantType.kQ40: 18, QuantType.kQ41: 20}


def BlockBytes(qtype: QuantType) -> int:
    """Bytes per 32-weight block (src/quantized_tensor.cc:13-23)."""
    try:
        return _BLOCK_BYTES[QuantType(qtype)]
    except ValueError as exc:
        raise ValueError("unknown quantization type") from exc


@dataclass
class QuantizedStorage:
    """``QuantizedStorage{type, rows, cols, bytes}`` (quantized_tensor.h:12-17)."""

    type: QuantType
    rows: int
    cols: int
    bytes: np.ndarray  # uint8 GGUF block stream, row-major

    @property
    def blocks_per_row(self) -> int:
        return (self.cols + 31) // 32


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(a, dtype=np.uint8) if isinstance(a, (bytes, bytearray)) else a,
                                dtype=np.uint8)


def TensorFromQuantized(data, rows: int, cols: int, qtype: QuantType) -> QuantizedStorage:
    """Wrap a GGUF block stream after the reference's size check (quantized_tensor.cc:88-102)."""
    qtype = QuantType(qtype)
    if rows <= 0 or cols <= 0:
        raise ValueError("invalid quantized shape")
    data = _u8(data)
    if data.size != lib().mq_quantized_bytes(int(qtype), rows, cols):
        raise RuntimeError("quantized storage size mismatch")
    return QuantizedStorage(qtype, rows, cols, data)


def QuantizeTensor(tensor: np.ndarray, qtype: QuantType, threads: int = 0) -> QuantizedStorage:
    """Pack an F32 matrix into GGUF blocks, byte-identical to the reference's
    QuantizeTensor (src/quantized_tensor.cc:104-159). A QuantizedStorage input
    is decoded first and re-packed, as the reference does for quantized tensors."""
    qtype = QuantType(qtype)
    if isinstance(tensor, QuantizedStorage):
        tensor = DequantizeTensor(tensor)
    src = np.asarray(tensor)
    if src.ndim != 2:
        raise ValueError("quantization requires a matrix")
    src = np.ascontiguousarray(src, dtype=np.float32)
    rows, cols = src.shape
    out = np.zeros(lib().mq_quantized_bytes(int(qtype), rows, cols), dtype=np.uint8)
    rc = lib().mq_quantize(int(qtype), src.ctypes.data, rows, cols, out.ctypes.data, out.nbytes, threads)
    if rc == _lib.MQ_ERR_INVALID:
        raise ValueError(_lib.last_error())
    check(rc)
    return QuantizedStorage(qtype, rows, cols, out)


def DequantizeTensor(storage: QuantizedStorage) -> np.ndarray:
    """Decode to F32 with the reference's element formula (quantized_tensor.cc:32-43, 193-206)."""
    out = np.empty((storage.rows, storage.cols), dtype=np.float32)
    check(lib().mq_dequantize(int(storage.type), storage.bytes.ctypes.data, storage.bytes.nbytes, storage.rows,
                              storage.cols, out.ctypes.data))
    return out


def _torch():
    import torch  # plumbing only: device memory and streams

    return torch


def _stream_handle(stream) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


class CudaWeight:
    """A packed weight resident on one GPU (CudaModelState::UploadWeight).

    ``rows``/``row_range`` select an output-row shard: the device holds rows
    ``[row_begin, row_end)`` of the full matrix.
    """

    def __init__(self, storage: QuantizedStorage, device: int = 0, row_range: tuple[int, int] | None = None,
                 stream=None):
        torch = _torch()
        self.storage_type = storage.type
        self.full_rows, self.cols = storage.rows, storage.cols
        self.device = device
        r0, r1 = row_range if row_range is not None else (0, storage.rows)
        self.row_begin, self.row_end = r0, r1
        handle = C.c_void_p()
        with torch.cuda.device(device):
            sh = _stream_handle(stream)
            rc = lib().mq_weight_shard_create(device, int(storage.type), storage.rows, storage.cols, r0, r1,
                                              storage.bytes.ctypes.data, storage.bytes.nbytes, 0, sh,
                                              C.byref(handle))
        if rc == _lib.MQ_ERR_INVALID:
            raise ValueError(_lib.last_error())
        check(rc, "UploadWeight")
        self.handle = handle

    @classmethod
    def from_device_blocks(cls, blocks, qtype: QuantType, rows: int, cols: int, device: int = 0,
                           row_range: tuple[int, int] | None = None, stream=None) -> "CudaWeight":
        """Upload from a device-resident GGUF block stream (a uint8 CUDA tensor)."""
        torch = _torch()
        self = cls.__new__(cls)
        self.storage_type = QuantType(qtype)
        self.full_rows, self.cols, self.device = rows, cols, device
        r0, r1 = row_range if row_range is not None else (0, rows)
        self.row_begin, self.row_end = r0, r1
        handle = C.c_void_p()
        with torch.cuda.device(device):
            rc = lib().mq_weight_shard_create(device, int(qtype), rows, cols, r0, r1, blocks.data_ptr(),
                                              blocks.numel(), 1, _stream_handle(stream), C.byref(handle))
        check(rc, "UploadWeight")
        self.handle = handle
        return self

    @property
    def rows(self) -> int:
        return self.row_end - self.row_begin

    @property
    def device_bytes(self) -> int:
        n = C.c_size_t()
        check(lib().mq_weight_info(self.handle, None, None, None, None, C.byref(n)))
        return n.value

    def export(self) -> QuantizedStorage:
        """Read the device weight back as a GGUF block stream (round-trip check)."""
        out = np.zeros(lib().mq_quantized_bytes(int(self.storage_type), self.rows, self.cols), dtype=np.uint8)
        check(lib().mq_weight_export(self.handle, out.ctypes.data, out.nbytes), "export")
        return QuantizedStorage(self.storage_type, self.rows, self.cols, out)

    def linear(self, x, bias=None, out=None, stream=None):
        """y = x · Wᵀ (+ bias) on the device; x is a float32 CUDA tensor [K] or [M, K]."""
        torch = _torch()
        if x.dtype != torch.float32 or not x.is_cuda:
            raise RuntimeError("Linear requires F32 activations on the weight's device")
        squeeze = x.dim() == 1
        x2 = x.unsqueeze(0) if squeeze else x
        if x2.dim() != 2 or x2.shape[1] != self.cols:
            raise RuntimeError("LinearDispatch: dimension mismatch")
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        m = x2.shape[0]
        if out is None:
            out = torch.empty((m, self.rows), dtype=torch.float32, device=x.device)
        elif out.shape[-1] != self.rows or out.dtype != torch.float32:
            raise RuntimeError("output shape mismatch")
        out2 = out.view(m, self.rows) if out.dim() == 1 else out
        if bias is not None and (bias.numel() != self.rows or bias.dtype != torch.float32):
            raise RuntimeError("bias shape mismatch")
        check(lib().mq_linear(self.handle, x2.data_ptr(), m, x2.stride(0), bias.data_ptr() if bias is not None else None,
                              out2.data_ptr(), out2.stride(0), _stream_handle(stream)), "LinearDispatch")
        return out2.view(self.rows) if squeeze and out.dim() != 1 else out

    def linear_residual(self, x, residual, bias=None, out=None, stream=None):
        """residual + (x · Wᵀ + bias), the linear and ForwardCuda's residual AddKernel
        (src/cuda_backend.cu:236-240) in one launch; ``out`` may be ``residual`` (in place)."""
        torch = _torch()
        if x.dtype != torch.float32 or not x.is_cuda:
            raise RuntimeError("Linear requires F32 activations on the weight's device")
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        if x2.dim() != 2 or x2.shape[1] != self.cols:
            raise RuntimeError("LinearDispatch: dimension mismatch")
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        m = x2.shape[0]
        r2 = residual.view(1, -1) if residual.dim() == 1 else residual
        if tuple(r2.shape) != (m, self.rows) or r2.dtype != torch.float32 or r2.stride(1) != 1:
            raise RuntimeError("ElementwiseAdd: shape mismatch")
        if out is None:
            out = torch.empty_like(r2)
        o2 = out.view(1, -1) if out.dim() == 1 else out
        if o2.shape != r2.shape or o2.stride(0) != r2.stride(0):
            raise RuntimeError("output shape mismatch (the output must have the residual's layout)")
        if bias is not None and (bias.numel() != self.rows or bias.dtype != torch.float32):
            raise RuntimeError("bias shape mismatch")
        check(lib().mq_linear_residual(self.handle, x2.data_ptr(), m, x2.stride(0),
                                       bias.data_ptr() if bias is not None else None, r2.data_ptr(), o2.data_ptr(),
                                       o2.stride(0), _stream_handle(stream)), "LinearDispatch")
        return out

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().mq_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def LinearSwiGlu(x, w_gate: CudaWeight, w_up: CudaWeight, out=None, stream=None):
    """SwiGlu(Linear(x, w_gate), Linear(x, w_up)) in one call (FfnForward's gate/up half,
    src/forward.cc:105-110, with SwiGluKernel, src/cuda_backend.cu:241-245)."""
    torch = _torch()
    if x.dtype != torch.float32 or not x.is_cuda:
        raise RuntimeError("Linear requires F32 activations on the weight's device")
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dim() != 2 or x2.shape[1] != w_up.cols:
        raise RuntimeError("LinearDispatch: dimension mismatch")
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    m, n = x2.shape[0], w_up.rows
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    elif out.shape[-1] != n or out.dtype != torch.float32:
        raise RuntimeError("output shape mismatch")
    out2 = out.view(m, n) if out.dim() == 1 else out
    check(lib().mq_linear_swiglu(w_gate.handle, w_up.handle, x2.data_ptr(), m, x2.stride(0), out2.data_ptr(),
                                 out2.stride(0), _stream_handle(stream)), "SwiGlu")
    return out2.view(n) if squeeze and out.dim() != 1 else out


def LinearDispatch(x, weight: CudaWeight, bias=None):
    """Quantized branch of LinearDispatch (src/matmul_optimized.cc:146-182) on the GPU."""
    return weight.linear(x, bias=bias)


def Linear(x, weight: CudaWeight):
    """``Linear`` (src/ops.cc:12-14)."""
    return LinearDispatch(x, weight)


def CudaDeviceInfo() -> str:
    """Device list, as CudaDeviceInfo (src/cuda_backend.cu:355-369)."""
    buf = C.create_string_buffer(4096)
    check(lib().mq_device_info(buf, len(buf)))
    return buf.value.decode()


def set_path(mode: int) -> int:
    """Kernel selection for this thread (mq_set_path): 0 automatic, 1 stream-K SIMT GEMV,
    2 tcgen05 prefill GEMM, 3 tcgen05 int8 decode GEMV, 4 tcgen05 fp16 decode GEMM,
    5 SIMT dp4a decode GEMV, 6 tcgen05 scale-folded decode GEMM, 7 the same on CTA pairs (cta_group::2)."""
    return lib().mq_set_path(mode)


__all__ = [
    "QuantType", "QuantizedStorage", "BlockBytes", "TensorFromQuantized", "QuantizeTensor", "DequantizeTensor",
    "CudaWeight", "LinearDispatch", "Linear", "CudaDeviceInfo", "set_path", "MQError",
]
