// Shared definitions for the mq_b200 engine: error state, the device weight
// layout, fp16 bit conversions, and small PTX helpers for sm_100a.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "mq_b200.h"

namespace mq {

// ---------------------------------------------------------------------------
// Errors: every entry point returns a code and leaves the message here.
// ---------------------------------------------------------------------------
std::string &last_error();
int fail(int code, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
// Counts every kernel launch issued by the library (mq_kernel_launches).
void count_launch(int n = 1);

#define MQ_CUDA(call)                                  \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return mq::cuda_fail(e_, #call); \
  } while (0)

// ---------------------------------------------------------------------------
// GGUF block geometry (src/quantized_tensor.cc:13-23 of the reference).
// ---------------------------------------------------------------------------
__host__ __device__ inline int block_bytes(int qtype) {
  return qtype == MQ_Q8_0 ? 34 : qtype == MQ_Q4_0 ? 18 : qtype == MQ_Q4_1 ? 20 : 0;
}
// Quant bytes per 32-weight block in the device layout (scales live apart).
__host__ __device__ inline int block_qbytes(int qtype) { return qtype == MQ_Q8_0 ? 32 : 16; }

// ---------------------------------------------------------------------------
// Device-resident weight ("step chunks").
//
// The kernels stream a weight as a sequence of (tile, step) units: a tile is
// 128 rows, a step 8 quant blocks (256 K). Each unit is one contiguous chunk,
// tile-major, so that a persistent CTA walking consecutive units reads one
// contiguous address range with a single bulk copy per unit:
//   chunk(t, k) = base + (t * steps + k) * chunk_bytes
//   [ packed quant bytes | fp16 scales d [128][8] | fp16 Q4_1 mins [128][8] ]
// Packed bytes: Q4_x 128 rows x 128 B; Q8_0 two halves of 128 rows x 128 B
// (half = quad). A quad is 4 blocks; inside a row's quad the bytes follow
//   Q4_x: byte 16*t + 4*j + p = quant byte 2t + {0, 8, 1, 9}[p] of block j;
//   Q8_0: byte 32*t + 8*j + p = quant byte 2t + {0,1,8,9,16,17,24,25}[p],
// i.e. the K positions {2t, 2t+1, 2t+8, 2t+9} (+16) that one 16-byte chunk
// (Q4_x) or 32-byte pair of chunks (Q8_0) hands each consumer, and every
// 128-byte row is stored with the 16-byte chunk c at position c ^ (row & 7)
// (the 128-byte swizzle of a TMA tile, pre-applied, so that the threads that
// read one chunk position of 32 consecutive rows hit distinct banks).
// Rows are padded to a multiple of 128 and blocks to a multiple of 8 with
// zero bytes (a zero scale decodes to 0), so no kernel needs bounds checks on
// weight loads. Apart from that padding the bytes per weight are the GGUF ones.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 128;
constexpr int kStepBlocks = 8;

struct WeightView {
  int qtype, rows, cols, nb;   // nb = ceil(cols / 32)
  int steps, tiles, rows_pad;  // ceil(nb / 8), rows_pad / 128, rows rounded up to 128
  const uint8_t *base;         // chunk(0, 0)
  int64_t chunk_bytes;         // bytes of one (tile, step) chunk
  int pk_bytes;                // packed quant bytes at the start of a chunk
};

__host__ __device__ constexpr int group_bytes(int qtype) { return qtype == MQ_Q8_0 ? 128 : 64; }
__host__ __device__ constexpr int step_pk_bytes(int qtype) { return kTileRows * (qtype == MQ_Q8_0 ? 256 : 128); }
__host__ __device__ constexpr int step_sc_bytes(int qtype) { return kTileRows * 16 * (qtype == MQ_Q4_1 ? 2 : 1); }
__host__ __device__ constexpr int64_t step_chunk_bytes(int qtype) { return step_pk_bytes(qtype) + step_sc_bytes(qtype); }

// Position, inside its 4-block group (quad), of quant byte i of block j.
__host__ __device__ inline int permuted_pos(int qtype, int i, int j) {
  const int t = (i & 7) >> 1;
  if (qtype == MQ_Q8_0) return 32 * t + 8 * j + 2 * (i >> 3) + (i & 1);
  return 16 * t + 4 * j + ((i >> 3) | ((i & 1) << 1));
}

// Byte offset, inside a chunk, of 16-byte chunk c (0..7) of tile row r in
// half h (Q8_0; 0 for Q4_x).
__host__ __device__ inline int chunk16_off(int r, int c, int h) { return h * (kTileRows * 128) + r * 128 + ((c ^ (r & 7)) << 4); }

// Byte offset, inside a chunk, of quant byte i of step block jb (0..7) of tile row r.
__host__ __device__ inline int pk_byte_off(int qtype, int r, int jb, int i) {
  const int pos = permuted_pos(qtype, i, jb & 3);
  if (qtype == MQ_Q8_0) return chunk16_off(r, pos >> 4, jb >> 2) + (pos & 15);
  return chunk16_off(r, 4 * (jb >> 2) + (pos >> 4), 0) + (pos & 15);
}

// Chunk of (tile t, step k); scales of row r at + pk_bytes + 16 r, mins at + pk_bytes + 2048 + 16 r.
// Output epilogues, both on buffers laid out like y ([m, ldy]): the fused
// gate/up product (the reference's SwiGluKernel, src/cuda_backend.cu:241-245,
// applied to the up product's output): y = g / (1 + exp(-g)) * v; and the
// residual add (AddKernel, src/cuda_backend.cu:236-240): y = r + v, r may be
// y itself (each element is read and written by the same thread once).
__device__ __forceinline__ float epilogue_out(float v, const float *gate, const float *resid, int64_t idx) {
  if (gate) {
    const float g = gate[idx];
    v = g / (1.0f + expf(-g)) * v;
  }
  if (resid) v = resid[idx] + v;
  return v;
}

// Largest |d| for which every weight d * c (c = q - zp, |c| <= 8, 15, 128)
// stays inside the fp16 range, so that the folded decode kernel
// (mq_fdec.cuh) can hold it exactly as an fp16 hi + lo pair.
__host__ __device__ constexpr float fold_max_scale(int qtype) {
  return qtype == MQ_Q8_0 ? 65504.0f / 128.0f : qtype == MQ_Q4_1 ? 65504.0f / 16.0f : 65504.0f / 9.0f;
}

__host__ __device__ inline const uint8_t *chunk_ptr(const WeightView &w, int t, int k) {
  return w.base + ((int64_t)t * w.steps + k) * w.chunk_bytes;
}

// ---------------------------------------------------------------------------
// fp16 <-> fp32 by bit manipulation (IEEE binary16, round to nearest even),
// identical on host and device. Matches the reference's FloatToHalf /
// HalfToFloat (src/quantized_tensor.cc:46-86) for every non-NaN input and
// produces the same NaN encodings.
// ---------------------------------------------------------------------------
__host__ __device__ inline float bits_f32(uint32_t b) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
#endif
}
__host__ __device__ inline uint32_t f32_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t b;
  __builtin_memcpy(&b, &f, 4);
  return b;
#endif
}

__host__ __device__ inline uint16_t f32_to_f16_rne(float f) {
  const uint32_t b = f32_bits(f);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const uint32_t e8 = (b >> 23) & 255u, man = b & 0x7fffffu;
  if (e8 == 255u) return sign | (man ? 0x7e00u : 0x7c00u);
  const int e = (int)e8 - 112;
  if (e >= 31) return sign | 0x7c00u;
  if (e <= 0) {
    if (e < -10) return sign;
    const uint32_t sig = man | 0x800000u;
    const int sh = 14 - e;
    const uint32_t keep = sig >> sh, rest = sig & ((1u << sh) - 1u), tie = 1u << (sh - 1);
    return sign | (uint16_t)(keep + ((rest > tie) | ((rest == tie) & (keep & 1u))));
  }
  uint32_t keep = man >> 13;
  const uint32_t rest = man & 0x1fffu;
  keep += (rest > 0x1000u) | ((rest == 0x1000u) & (keep & 1u));
  uint32_t ee = (uint32_t)e + (keep >> 10);
  keep &= 1023u;
  if (ee >= 31u) return sign | 0x7c00u;
  return sign | (uint16_t)(ee << 10) | (uint16_t)keep;
}

__host__ __device__ inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, f = h & 1023u;
  if (e == 31u) return f ? bits_f32(0x7fc00000u) : bits_f32(sign | 0x7f800000u);
  if (e == 0u) return bits_f32(f32_bits((float)f * 5.9604644775390625e-8f) | sign);
  return bits_f32(sign | ((e + 112u) << 23) | (f << 13));
}

// ---------------------------------------------------------------------------
// PTX helpers (sm_100a).
// ---------------------------------------------------------------------------
// Streaming 16-byte load that bypasses L1 allocation: weights are read once.
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void *p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_nc_f4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }

}  // namespace mq

// Opaque handle behind mq_weight*.
struct mq_weight {
  int device = 0;
  mq::WeightView v{};
  void *base = nullptr;       // single device allocation holding all planes
  size_t bytes = 0;
  int row_begin = 0;          // first row of the full matrix (shards)
  int full_rows = 0;
  bool foldable = false;      // every |d| < fold_max_scale: the folded decode kernel applies
};
