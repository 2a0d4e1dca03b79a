"""The product's own fp16 conversions against the reference build, over every input.

mini_ai_b200/csrc/mq_common.cuh implements fp32 -> fp16 (round to nearest
even) and fp16 -> fp32 from the IEEE bit layout; the quantizer stores every
scale (and Q4_1 min) through the first and every decode path reads them back
through the second. They must equal the reference's FloatToHalf / HalfToFloat
(src/quantized_tensor.cc:46-86) bit for bit: here on all 2^32 fp32 bit
patterns and all 65536 fp16 values, with the product's host build of the same
inline functions (tests/probes/fp16_probe.cu, compiled with nvcc into a
temporary directory). CPU only.
"""
from __future__ import annotations

import ctypes as C
import subprocess

import numpy as np
import pytest

from conftest import ROOT

NVCC = "/usr/local/cuda/bin/nvcc"


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    out = tmp_path_factory.mktemp("fp16probe") / "libfp16probe.so"
    cmd = [NVCC, "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-I", str(ROOT / "include"), "-I",
           str(ROOT / "mini_ai_b200" / "csrc"), "-o", str(out), str(ROOT / "tests" / "probes" / "fp16_probe.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    lib = C.CDLL(str(out))
    lib.probe_f32_to_f16_range.restype = None
    lib.probe_f32_to_f16_range.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t]
    lib.probe_f16_to_f32_all.restype = None
    lib.probe_f16_to_f32_all.argtypes = [C.c_void_p]
    return lib


def test_product_half_to_float_all_inputs(probe, reference):
    got = np.empty(65536, np.float32)
    probe.probe_f16_to_f32_all(got.ctypes.data)
    assert np.array_equal(got.view(np.uint32), reference.half_to_float_all().view(np.uint32))


def test_product_float_to_half_all_inputs(probe, reference):
    chunk = 1 << 26
    got = np.empty(chunk, np.uint16)
    for start in range(0, 1 << 32, chunk):
        probe.probe_f32_to_f16_range(start, got.ctypes.data, chunk)
        ref = reference.float_to_half_range(start, chunk)
        if not np.array_equal(got, ref):
            bad = int(np.flatnonzero(got != ref)[0])
            pytest.fail(f"fp32 bits {start + bad:#010x}: product {got[bad]:#06x}, reference {ref[bad]:#06x}")
