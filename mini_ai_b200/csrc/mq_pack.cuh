// Weight layout kernels and the bit-exact block quantizer.
//
// * repack / unpack: GGUF block stream <-> the step chunks of WeightView.
// * quantize_block : one 32-slot block packed exactly as the reference's
//   QuantizeTensor (src/quantized_tensor.cc:104-159) packs it. Shared by the
//   host quantizer (threads over rows) and the device quantizer (one thread
//   per block), so both produce identical bytes.
#pragma once

#include <math.h>

#include "mq_common.cuh"

namespace mq {

// GGUF block stream (rows x nb blocks, starting at `src`) -> step chunks.
// `unfoldable` (optional) is raised when a block scale is not finite or so
// large that d * c leaves the fp16 range (the folded decode kernel, mq_fdec.cuh).
__global__ void repack_kernel(const uint8_t *__restrict__ src, WeightView w, int *unfoldable = nullptr) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)w.rows * w.nb) return;
  const int r = (int)(i / w.nb), b = (int)(i % w.nb);
  const int bb = block_bytes(w.qtype), qb = block_qbytes(w.qtype), hdr = bb - qb;
  const uint8_t *blk = src + i * bb;
  if (unfoldable) {
    const float d = fabsf(f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8))));
    if (!(d < fold_max_scale(w.qtype))) atomicOr(unfoldable, 1);
  }
  const int rr = r % kTileRows, jb = b % kStepBlocks;
  uint8_t *c = const_cast<uint8_t *>(chunk_ptr(w, r / kTileRows, b / kStepBlocks));
  uint8_t *sc = c + w.pk_bytes + rr * 16 + 2 * jb;
  sc[0] = blk[0];
  sc[1] = blk[1];
  if (w.qtype == MQ_Q4_1) sc[2048] = blk[2], sc[2049] = blk[3];
  for (int q = 0; q < qb; ++q) c[pk_byte_off(w.qtype, rr, jb, q)] = blk[hdr + q];
}

// Step chunks -> GGUF block stream (the inverse of repack_kernel).
__global__ void unpack_kernel(uint8_t *__restrict__ dst, const WeightView w) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)w.rows * w.nb) return;
  const int r = (int)(i / w.nb), b = (int)(i % w.nb);
  const int bb = block_bytes(w.qtype), qb = block_qbytes(w.qtype), hdr = bb - qb;
  uint8_t *blk = dst + i * bb;
  const int rr = r % kTileRows, jb = b % kStepBlocks;
  const uint8_t *c = chunk_ptr(w, r / kTileRows, b / kStepBlocks);
  const uint8_t *sc = c + w.pk_bytes + rr * 16 + 2 * jb;
  blk[0] = sc[0];
  blk[1] = sc[1];
  if (w.qtype == MQ_Q4_1) blk[2] = sc[2048], blk[3] = sc[2049];
  for (int q = 0; q < qb; ++q) blk[hdr + q] = c[pk_byte_off(w.qtype, rr, jb, q)];
}

// Failure kinds of quantize_block (mapped to MQ_ERR_* and the reference's
// messages by the callers).
enum QuantFail { kQuantOk = 0, kQuantNonFinite = 1, kQuantScaleRange = 2, kQuantOffsetRange = 3 };

// Pack one block of `n` (1..32) source values into `blk` (block_bytes(qtype)
// bytes). Returns a QuantFail.
//  - statistics start at 0 and cover only the n real values; slots past n
//    quantize the value 0, like the zero-initialised values[32] the
//    reference packs (src/quantized_tensor.cc:115-117);
//  - the signed maximum keeps the first value of largest magnitude;
//  - scale and Q4_1 min are rounded to fp16 and the rounded values are used;
//  - q = round-half-away((v - min) / scale) with an IEEE fp32 divide.
__host__ __device__ inline int quantize_block(int qtype, const float *src, int n, uint8_t *blk) {
  float v[32];
  float lo = 0.0f, hi = 0.0f, peak = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float x = j < n ? src[j] : 0.0f;
    if (!isfinite(x)) return kQuantNonFinite;
    v[j] = x;
    lo = x < lo ? x : lo;
    hi = hi < x ? x : hi;
    peak = fabsf(x) > fabsf(peak) ? x : peak;
  }
  // The reference's min/max start at +0 and only a strictly smaller/larger
  // value replaces them, so a zero result is always +0. A compiler may lower
  // the selects above to a hardware min/max that returns -0 for (-0, +0);
  // adding +0 canonicalises the sign (x + 0 == x for every non-zero x).
  lo += 0.0f;
  hi += 0.0f;
  float scale = qtype == MQ_Q8_0 ? fabsf(peak) / 127.0f : qtype == MQ_Q4_0 ? peak / -8.0f : (hi - lo) / 15.0f;
  const uint16_t sh = f32_to_f16_rne(scale);
  scale = f16_to_f32(sh);
  if (!isfinite(scale)) return kQuantScaleRange;
  blk[0] = (uint8_t)(sh & 255);
  blk[1] = (uint8_t)(sh >> 8);
  float zero = 0.0f;
  if (qtype == MQ_Q4_1) {
    const uint16_t mh = f32_to_f16_rne(lo);
    zero = f16_to_f32(mh);
    if (!isfinite(zero)) return kQuantOffsetRange;
    blk[2] = (uint8_t)(mh & 255);
    blk[3] = (uint8_t)(mh >> 8);
  }
  int q[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) q[j] = scale == 0.0f ? 0 : (int)roundf((v[j] - zero) / scale);
  if (qtype == MQ_Q8_0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(int8_t)(q[j] < -127 ? -127 : q[j] > 127 ? 127 : q[j]);
  } else {
    const int base = qtype == MQ_Q4_1 ? 4 : 2, zp = qtype == MQ_Q4_0 ? 8 : 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      int a = q[j] + zp, c = q[j + 16] + zp;
      a = a < 0 ? 0 : a > 15 ? 15 : a;
      c = c < 0 ? 0 : c > 15 ? 15 : c;
      blk[base + j] = (uint8_t)(a | (c << 4));
    }
  }
  return kQuantOk;
}

// One thread per block. *first_bad (initialised to ~0) receives the smallest
// (block index << 2 | QuantFail) over failing blocks: the failure of the
// first bad block in row-major order, where the reference's loop throws.
__global__ void quantize_kernel(const float *__restrict__ src, int qtype, int rows, int cols, uint8_t *__restrict__ dst,
                                unsigned long long *first_bad) {
  const int nb = (cols + 31) >> 5;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * nb) return;
  const int64_t r = i / nb, b = i % nb;
  const int c0 = (int)b * 32, n = min(32, cols - c0);
  uint8_t blk[34];
  const int rc = quantize_block(qtype, src + r * cols + c0, n, blk);
  if (rc != kQuantOk) {
    atomicMin(first_bad, ((unsigned long long)i << 2) | (unsigned long long)rc);
    return;
  }
  const int bb = block_bytes(qtype);
  uint8_t *out = dst + i * bb;
  for (int j = 0; j < bb; ++j) out[j] = blk[j];
}

}  // namespace mq
