"""The bounded-wait error flag reaches the caller (1 GPU, no fault, no hang).

Every wait of the tensor-core kernels is bounded; a wait that runs out stores
1 into the device's error flag (mapped host memory), and the next tensor-core
call on that device must return MQ_ERR_TIMEOUT once and clear the flag. Here
the flag is raised from the device with cudaMemset, as a kernel would, and the
automatic path is called for every kernel class (int8 decode, scale-folded
decode, prefill GEMM). The call after the reported one must succeed with the
same result as before.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import Q4_0

pytestmark = pytest.mark.gpu


def _raise_flag(mq, device):
    from cuda.bindings import runtime as rt

    flag = C.c_void_p()
    assert mq.lib().mq_device_error_flag(device, C.byref(flag)) == 0, mq._lib.last_error()
    assert flag.value
    (err,) = rt.cudaMemset(flag.value, 1, 4)
    assert int(err) == 0
    (err,) = rt.cudaDeviceSynchronize()
    assert int(err) == 0


@pytest.mark.parametrize("m", [1, 8, 64], ids=["int8_decode", "folded_decode", "prefill_gemm"])
def test_raised_error_flag_is_reported_once(mq, cuda_device, m):
    import torch

    rng = np.random.default_rng(m)
    w = mq.CudaWeight(mq.QuantizeTensor((rng.standard_normal((256, 1024)) * 0.02).astype(np.float32), Q4_0),
                      device=cuda_device)
    x = torch.from_numpy(rng.standard_normal((m, 1024)).astype(np.float32)).to(f"cuda:{cuda_device}")
    y0 = w.linear(x)
    torch.cuda.synchronize(cuda_device)
    _raise_flag(mq, cuda_device)
    with pytest.raises(mq.MQError) as info:
        w.linear(x)
    assert info.value.code == mq._lib.MQ_ERR_TIMEOUT
    assert "bounded wait" in str(info.value)
    y1 = w.linear(x)  # the flag was cleared by the reported call
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(y0, y1)
    w.close()


def test_error_flag_argument_checks(mq):
    flag = C.c_void_p()
    assert mq.lib().mq_device_error_flag(-1, C.byref(flag)) == mq._lib.MQ_ERR_INVALID
    assert mq.lib().mq_device_error_flag(0, None) == mq._lib.MQ_ERR_INVALID
