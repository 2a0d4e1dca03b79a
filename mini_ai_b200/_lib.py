"""ctypes binding of libmq_b200.so (the C ABI declared in include/mq_b200.h).

The library is built in-tree by ``python -m mini_ai_b200.build``. There is no
fallback: if the shared object is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmq_b200.so"

MQ_Q4_0, MQ_Q4_1, MQ_Q8_0 = 2, 3, 8
MQ_OK = 0
MQ_ERR_INVALID = -1
MQ_ERR_CUDA = -2
MQ_ERR_SIZE = -3
MQ_ERR_NONFINITE = -4
MQ_ERR_RANGE = -5
MQ_ERR_TIMEOUT = -6
MQ_ERR_UNSUPPORTED = -7

# Every symbol include/mq_b200.h declares, with (restype, argtypes).
_vp, _i, _sz, _f = C.c_void_p, C.c_int, C.c_size_t, C.c_float
SIGNATURES = {
    "mq_last_error": (C.c_char_p, []),
    "mq_version": (C.c_char_p, []),
    "mq_quantized_bytes": (_sz, [_i, _i, _i]),
    "mq_quantize": (_i, [_i, _vp, _i, _i, _vp, _sz, _i]),
    "mq_dequantize": (_i, [_i, _vp, _sz, _i, _i, _vp]),
    "mq_quantize_device": (_i, [_i, _i, _vp, _i, _i, _vp, _sz, _vp]),
    "mq_weight_create": (_i, [_i, _i, _i, _i, _vp, _sz, _i, _vp, C.POINTER(_vp)]),
    "mq_weight_shard_create": (_i, [_i, _i, _i, _i, _i, _i, _vp, _sz, _i, _vp, C.POINTER(_vp)]),
    "mq_weight_destroy": (None, [_vp]),
    "mq_weight_info": (_i, [_vp, C.POINTER(_i), C.POINTER(_i), C.POINTER(_i), C.POINTER(_i), C.POINTER(_sz)]),
    "mq_weight_export": (_i, [_vp, _vp, _sz]),
    "mq_linear": (_i, [_vp, _vp, _i, _i, _vp, _vp, _i, _vp]),
    "mq_linear_ragged": (_i, [_vp, _vp, C.POINTER(_i), _i, _i, _vp, _vp, _i, _vp]),
    "mq_linear_noalloc": (_i, [_vp, _vp, _i, _i, _vp, _vp, _i, _vp]),
    "mq_linear_swiglu": (_i, [_vp, _vp, _vp, _i, _i, _vp, _i, _vp]),
    "mq_linear_residual": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "mq_comm_unique_id": (_i, [_vp, _sz]),
    "mq_comm_create": (_i, [_i, _i, _i, _vp, _sz, C.POINTER(_vp)]),
    "mq_comm_destroy": (None, [_vp]),
    "mq_comm_uses_peer_gather": (_i, [_vp]),
    "mq_linear_sharded_allgather": (_i, [_vp, _vp, _i, _i, _vp, _vp, _i, _vp, _vp]),
    "mq_set_path": (_i, [_i]),
    "mq_kernel_launches": (C.c_uint64, []),
    "mq_device_info": (_i, [C.c_char_p, _sz]),
    "mq_device_error_flag": (_i, [_i, C.POINTER(_vp)]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


class MQError(RuntimeError):
    """A failing mq_* call: ``code`` is the MQ_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def lib() -> C.CDLL:
    """Load libmq_b200.so once; raises if it is absent (no CPU fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m mini_ai_b200.build`")
            handle = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def last_error() -> str:
    return lib().mq_last_error().decode()


def check(rc: int, what: str = "") -> None:
    if rc != MQ_OK:
        raise MQError(rc, f"{what}: {last_error()}" if what else last_error())
