"""mini_ai_b200 — B200-native (sm_100a) quantized linear path of mini_ai.

The engine is the shared library ``libmq_b200.so`` (C ABI, include/mq_b200.h);
this package is the host-side mirror of the reference operator surface over it.
"""
from ._lib import LIB_PATH, MQError, lib
from .quantized_tensor import (BlockBytes, CudaDeviceInfo, CudaWeight, DequantizeTensor, Linear, LinearDispatch,
                               LinearSwiGlu, QuantizedStorage, QuantizeTensor, QuantType, TensorFromQuantized,
                               set_path)
from .sharded import CudaComm, ShardedLinear, assemble, shard_rows

__all__ = [
    "LIB_PATH", "MQError", "lib", "BlockBytes", "CudaDeviceInfo", "CudaWeight", "DequantizeTensor", "Linear",
    "LinearDispatch", "LinearSwiGlu", "QuantizedStorage", "QuantizeTensor", "QuantType", "TensorFromQuantized", "set_path",
    "CudaComm", "ShardedLinear", "assemble", "shard_rows",
]
