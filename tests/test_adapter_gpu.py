"""mini_ai's own test suite run against the B200 backend (the drop-in boundary).

mini_ai_b200/adapter/b200_backend.cu implements the reference's backend
surface (EnableCuda, CudaDeviceInfo, CudaStats, ForwardCuda;
include/mini_llama/backend.h) over include/mq_b200.h, and
mini_ai_b200/adapter/Makefile links it with the reference's unmodified
sources and its minimal-framework test suite (tests/*.cc) in place of
src/cuda_backend.cu. The binary is built where the reference checkout exists
(build() of __graft_entry__) and carries the tiny model data it loads.

The suite's CUDA test (tests/test_cuda.cc:9-49) is the parity check of the
boundary: the tiny model (hidden 86: tail blocks) with normal and NeoX RoPE,
q/k/v biases, and F32, Q8_0, Q4_0 and Q4_1 weights (QuantizeModel), five
tokens through ForwardToken on the CPU and through the B200 backend, every
logit within 1e-4. The other 152 tests of the reference's suite check that
linking the backend leaves the rest of mini_ai unchanged.

Four more tests in the same runner (mini_ai_b200/adapter/test_b200_backend.cc)
cover the backend's surface beyond backend.h: the batched forward of several
ragged requests against the CPU ForwardBatch (decode kernels and the prefill
GEMM), its input checks, QuantizeModelB200 against QuantizeModel, and a GGUF
file with Q8_0 / Q4_0 / Q4_1 linears loaded by the reference's loader and run
on the device.
"""
from __future__ import annotations

import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SUITE = ROOT / "mini_ai_b200" / "adapter" / "_ref" / "mini-ai-b200-tests"


def test_reference_suite_with_b200_backend():
    if not SUITE.exists():
        pytest.skip("the suite is built where the reference checkout exists (make -C mini_ai_b200/adapter REF=...)")
    res = subprocess.run([str(SUITE)], cwd=SUITE.parent, capture_output=True, text=True, timeout=600)
    out = res.stdout + res.stderr
    assert "[PASS] cuda_backend_availability_and_forward" in out, out[-4000:]
    assert res.returncode == 0, out[-4000:]
    for name in ("b200_batched_forward_matches_cpu", "b200_batched_forward_rejects_bad_input",
                 "b200_quantize_model_matches_reference", "b200_gguf_quantized_model_forward"):
        assert f"[PASS] {name}" in out, out[-4000:]
    assert "Results: 157 passed, 0 failed" in out, out[-2000:]
    # CudaStats after each (layout, type) case: weights went through the backend.
    stats = [line for line in out.splitlines() if line.startswith("uploaded_weights=")]
    assert len(stats) == 8 and all("cuda_linear_calls=" in s for s in stats), stats
