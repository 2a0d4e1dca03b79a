// Streaming quantized GEMV for small activation counts (decode).
//
// y[i, n] = sum_b d[n,b] * sum_{j<32} q[n,b,j] * x[i, 32b + j]   (+ m[n,b] * sum_j x)
//
// HBM-bound: each weight byte is read exactly once with a 16-byte
// L1-bypassing load. A CTA owns RPW consecutive output rows and its warps
// split the K blocks between them (lane l of warp w takes blocks
// l + 32*(w + W*j)), so even a 4096-row matrix launches ~1000 CTAs.
// Each lane decodes whole 32-weight blocks in registers: a nibble or byte is
// turned into an exact fp32 by splicing it under the exponent of 2^23
// (byte_perm) and subtracting 2^23 + zero point, then fused-multiply-added
// into a per-block partial; the fp16 scale (and the Q4_1 min times the block
// sum of x) is applied once per block. x is read through the read-only path
// and reused across the RPW rows held in registers. Warps reduce with
// shuffles, then the CTA combines the warp partials in a fixed order, so the
// result is deterministic.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191
// (and LinearKernel, src/cuda_backend.cu:94-110, with its fused bias).
#pragma once

#include "mq_common.cuh"

namespace mq {

struct GemvArgs {
  WeightView w;
  const float *x;
  int64_t ldx;
  const float *bias;
  float *y;
  int64_t ldy;
};

// 2^23 + zero point: subtracting it from the spliced float yields q - zp.
template <int QT> struct Zp;
template <> struct Zp<MQ_Q4_0> { static constexpr float kMagic = 8388616.0f; };  // 2^23 + 8
template <> struct Zp<MQ_Q4_1> { static constexpr float kMagic = 8388608.0f; };  // 2^23
template <> struct Zp<MQ_Q8_0> { static constexpr float kMagic = 8388736.0f; };  // 2^23 + 128 (after ^0x80)

// Byte k of `v` spliced under 2^23: the float 2^23 + byte.
__device__ __forceinline__ float splice(uint32_t v, int k) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)k));
}

// x values a lane needs for one 32-element block, loaded per 4-element group.
template <bool VECX>
__device__ __forceinline__ float4 load_x4(const float *xr, int k0, int K, bool full) {
  if (VECX && full) return ld_nc_f4(xr + k0);
  float4 v;
  v.x = k0 + 0 < K ? __ldg(xr + k0 + 0) : 0.0f;
  v.y = k0 + 1 < K ? __ldg(xr + k0 + 1) : 0.0f;
  v.z = k0 + 2 < K ? __ldg(xr + k0 + 2) : 0.0f;
  v.w = k0 + 3 < K ? __ldg(xr + k0 + 3) : 0.0f;
  return v;
}

__device__ __forceinline__ float dot4(float a0, float a1, float a2, float a3, float4 x, float acc) {
  acc = fmaf(a0, x.x, acc);
  acc = fmaf(a1, x.y, acc);
  acc = fmaf(a2, x.z, acc);
  acc = fmaf(a3, x.w, acc);
  return acc;
}

template <int QT, int M, int RPW, bool VECX>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a) {
  constexpr int QW = QT == MQ_Q8_0 ? 8 : 4;  // 32-bit words of quants per block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int row0 = blockIdx.x * RPW;
  const WeightView &w = a.w;
  const int K = w.cols, nb = w.nb, nb_full = w.cols >> 5;
  const int nrow = min(RPW, w.rows - row0);

  float acc[RPW][M];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) acc[r][i] = 0.0f;

  for (int b = lane + 32 * warp; b < nb; b += 32 * nwarps) {
    uint32_t q[RPW][QW];
    float dsc[RPW], msc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      if (r < nrow) {
        const uint8_t *p = w.qs + (int64_t)(row0 + r) * w.ld_qs + (int64_t)b * (QW * 4);
#pragma unroll
        for (int h = 0; h < QW / 4; ++h) {
          const uint4 v = ld_stream_v4(p + 16 * h);
          q[r][4 * h + 0] = v.x;
          q[r][4 * h + 1] = v.y;
          q[r][4 * h + 2] = v.z;
          q[r][4 * h + 3] = v.w;
        }
        dsc[r] = __half2float(w.d[(int64_t)(row0 + r) * w.ld_s + b]);
        msc[r] = QT == MQ_Q4_1 ? __half2float(w.mn[(int64_t)(row0 + r) * w.ld_s + b]) : 0.0f;
      } else {
#pragma unroll
        for (int h = 0; h < QW; ++h) q[r][h] = 0u;
        dsc[r] = 0.0f;
        msc[r] = 0.0f;
      }
    }
    const bool full = b < nb_full;
    float part[RPW][M], xs[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      xs[i] = 0.0f;
#pragma unroll
      for (int r = 0; r < RPW; ++r) part[r][i] = 0.0f;
    }
    const int kb = b * 32;
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
      if constexpr (QT == MQ_Q8_0) {
        // words 2*wd and 2*wd+1 hold elements 8wd .. 8wd+7
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int widx = 2 * wd + half;
          float4 xv[M];
#pragma unroll
          for (int i = 0; i < M; ++i) xv[i] = load_x4<VECX>(a.x + (int64_t)i * a.ldx, kb + 4 * widx, K, full);
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            const uint32_t u = q[r][widx] ^ 0x80808080u;
            const float v0 = splice(u, 0) - Zp<QT>::kMagic, v1 = splice(u, 1) - Zp<QT>::kMagic;
            const float v2 = splice(u, 2) - Zp<QT>::kMagic, v3 = splice(u, 3) - Zp<QT>::kMagic;
#pragma unroll
            for (int i = 0; i < M; ++i) part[r][i] = dot4(v0, v1, v2, v3, xv[i], part[r][i]);
          }
        }
      } else {
        // word wd: low nibbles = elements 4wd..4wd+3, high = 16+4wd..16+4wd+3
        float4 xl[M], xh[M];
#pragma unroll
        for (int i = 0; i < M; ++i) {
          xl[i] = load_x4<VECX>(a.x + (int64_t)i * a.ldx, kb + 4 * wd, K, full);
          xh[i] = load_x4<VECX>(a.x + (int64_t)i * a.ldx, kb + 16 + 4 * wd, K, full);
          if constexpr (QT == MQ_Q4_1) xs[i] += ((xl[i].x + xl[i].y) + (xl[i].z + xl[i].w)) +
                                               ((xh[i].x + xh[i].y) + (xh[i].z + xh[i].w));
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const uint32_t lo = q[r][wd] & 0x0F0F0F0Fu, hi = (q[r][wd] >> 4) & 0x0F0F0F0Fu;
          const float l0 = splice(lo, 0) - Zp<QT>::kMagic, l1 = splice(lo, 1) - Zp<QT>::kMagic;
          const float l2 = splice(lo, 2) - Zp<QT>::kMagic, l3 = splice(lo, 3) - Zp<QT>::kMagic;
          const float h0 = splice(hi, 0) - Zp<QT>::kMagic, h1 = splice(hi, 1) - Zp<QT>::kMagic;
          const float h2 = splice(hi, 2) - Zp<QT>::kMagic, h3 = splice(hi, 3) - Zp<QT>::kMagic;
#pragma unroll
          for (int i = 0; i < M; ++i) {
            part[r][i] = dot4(l0, l1, l2, l3, xl[i], part[r][i]);
            part[r][i] = dot4(h0, h1, h2, h3, xh[i], part[r][i]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int i = 0; i < M; ++i) {
        acc[r][i] = fmaf(dsc[r], part[r][i], acc[r][i]);
        if constexpr (QT == MQ_Q4_1) acc[r][i] = fmaf(msc[r], xs[i], acc[r][i]);
      }
  }

  // Warp reduction, then a fixed-order combine of the warps' partials.
  __shared__ float red[8][RPW * M];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) {
      float v = acc[r][i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][r * M + i] = v;
    }
  __syncthreads();
  for (int t = threadIdx.x; t < RPW * M; t += blockDim.x) {
    const int r = t / M, i = t % M;
    if (r >= nrow) continue;
    float v = red[0][t];
    for (int ww = 1; ww < nwarps; ++ww) v += red[ww][t];
    const int n = row0 + r;
    if (a.bias) v += a.bias[n];
    a.y[(int64_t)i * a.ldy + n] = v;
  }
}

}  // namespace mq
