// Tensor-core GEMM for large activation counts (prefill): placeholder until
// the tcgen05 kernel lands; every m is served by the streaming GEMV.
#pragma once

#include <climits>

#include "mq_common.cuh"

namespace mq {
inline int gemm_min_m(int) { return INT_MAX; }
inline bool gemm_supported(int) { return false; }
int run_gemv(const mq_weight *, const float *, int, int64_t, const float *, float *, int64_t, cudaStream_t);
inline int run_gemm(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
                    cudaStream_t s) {
  return run_gemv(w, x, m, ldx, bias, y, ldy, s);
}
}  // namespace mq
