// Host interface of the tcgen05 decode GEMM, shared by mq_linear (scratch from
// the per-stream workspace) and mq_linear_noalloc (scratch in a static device
// array). Definitions live in mq_gemm_host.cuh.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "mq_common.cuh"
#include "mq_peer.cuh"

namespace mq {

// Packed K steps per tile, padded K, 128-row tiles and the persistent grid
// (one CTA per SM, at most one per step of work).
struct DecPlan {
  int steps, kpad, tiles, grid;
};

// Scratch one launch pair needs.
struct DecBuffers {
  __half *x2;         // [2 bn][kpad]: activation rows split into fp16 hi rows, then lo rows
  float *xsum;        // [kpad / 32][bn]: scaled block sums of x (Q4_1)
  float *xinv;        // [steps][bn]: 2^-e per (256-K step, activation row); folded kernel: [bn], per row
  float *partial;     // [grid][2][128][bn]: head / tail partial tile of every CTA
  int *tickets;       // [tiles], zero between launches
  int *err;           // device-visible timeout flag
};

// max_grid caps the persistent grid (0: one CTA per SM).
DecPlan tcdec_plan(const WeightView &w, int device, int max_grid = 0);

inline int dec_tile_rows(int m) { return m <= 8 ? 8 : (m <= 16 ? 16 : 32); }
// Activation tile height of the scale-folded decode kernel (mq_fdec.cuh): 16 or 32.
inline int fdec_tile_rows(int m) { return m <= 16 ? 16 : 32; }

// One launch pair (activation split + decode GEMM) for m <= 32 rows; bn (the
// activation tile height, dec_tile_rows) is 8 for m <= 8, 16 for m <= 16, else
// 32. nan_on_abort: a timed-out bounded wait writes NaN to the outputs instead
// of leaving them unwritten. folded: the scale-folded kernel (mq_fdec.cuh; bn
// from fdec_tile_rows), for weights whose scales allow the fold.
int tcdec_launch(const WeightView &w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
                 cudaStream_t s, const DecPlan &plan, const DecBuffers &buf, int nan_on_abort,
                 const float *gate = nullptr, const float *resid = nullptr, bool folded = false,
                 const PeerOut *peer = nullptr, bool pairs = false);

// The automatic decode kernel of mq_linear with the row-sharded gather fused
// into its output stores (PeerOut, mq_peer.cuh): one launch that also stores
// the slice into every peer's staging and raises the arrival flags. Returns
// MQ_ERR_UNSUPPORTED (message unset) when the automatic choice for this
// weight and m is not a single int8 or scale-folded decode launch, or a kernel
// path is forced (mq_set_path); the caller then gathers separately.
int run_linear_peer(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
                    cudaStream_t s, const PeerOut &peer);

bool gemm_supported(int device);

}  // namespace mq
