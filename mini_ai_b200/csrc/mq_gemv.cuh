// Streaming SIMT GEMV for one or two activation rows (decode).
//
// y[i, n] = sum_b d[n,b] * sum_{k<32} q[n,b,k] * x[i, 32b + k]   (+ m[n,b] * sum_k x[i, 32b + k])
//
// HBM-bound: every weight byte is read once, 16 bytes per load, bypassing L1.
// A lane owns whole 4-block groups of a row (64 bytes Q4_x / 128 bytes Q8_0
// of the lane-permuted layout), so a warp streams 2-4 KB contiguous per row.
// Each CTA holds RPW rows per warp (x reused from registers across them);
// the CTA's warps split the groups of K between them when K is long.
// Decoding stays in registers: a nibble or byte is spliced under the
// exponent of 2^23 (byte_perm) and 2^23 + zero point is subtracted with a
// packed fp32 add, then packed fp32 FMAs accumulate a per-block partial; the
// fp16 scale (and the Q4_1 min times the block sum of x) is applied once per
// block. Lanes reduce with warp shuffles, warps through shared memory in a
// fixed order, so results are deterministic.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
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

// Bytes a and b of v, each spliced under 2^23, minus the magic: two exact floats.
template <int QT>
__device__ __forceinline__ float2 decode_pair(uint32_t v, int a, int b) {
  const float2 f = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)a)),
                               __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)b)));
  return __fadd2_rn(f, make_float2(-Zp<QT>::kMagic, -Zp<QT>::kMagic));
}

template <int QT, int M, int RPW>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a, int warps_k) {
  constexpr int GW = QT == MQ_Q8_0 ? 32 : 16;  // 32-bit words per row per group
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wk = warp % warps_k, wr = warp / warps_k, warps_r = (blockDim.x >> 5) / warps_k;
  const WeightView &w = a.w;
  const int row0 = (blockIdx.x * warps_r + wr) * RPW;
  const int nrow = min(RPW, w.rows - row0);
  const int K = w.cols;

  float2 acc[RPW][M];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) acc[r][i] = make_float2(0.0f, 0.0f);

  if (nrow > 0) {
    for (int G = lane + 32 * wk; G < w.nb4; G += 32 * warps_k) {
      uint32_t q[RPW][GW];
      float dsc[RPW][4], msc[RPW][4];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int row = row0 + (r < nrow ? r : 0);
        const uint8_t *p = w.qs + (int64_t)row * w.ld_qs + (int64_t)G * (GW * 4);
#pragma unroll
        for (int h = 0; h < GW / 4; ++h) {
          const uint4 v = ld_stream_v4(p + 16 * h);
          q[r][4 * h + 0] = v.x;
          q[r][4 * h + 1] = v.y;
          q[r][4 * h + 2] = v.z;
          q[r][4 * h + 3] = v.w;
        }
        const uint2 s = *reinterpret_cast<const uint2 *>(w.d + (int64_t)row * w.ld_s + 4 * G);
        const float2 s01 = __half22float2(*reinterpret_cast<const __half2 *>(&s.x));
        const float2 s23 = __half22float2(*reinterpret_cast<const __half2 *>(&s.y));
        const bool live = r < nrow;
        dsc[r][0] = live ? s01.x : 0.0f;
        dsc[r][1] = live ? s01.y : 0.0f;
        dsc[r][2] = live ? s23.x : 0.0f;
        dsc[r][3] = live ? s23.y : 0.0f;
        if constexpr (QT == MQ_Q4_1) {
          const uint2 mm = *reinterpret_cast<const uint2 *>(w.mn + (int64_t)row * w.ld_s + 4 * G);
          const float2 m01 = __half22float2(*reinterpret_cast<const __half2 *>(&mm.x));
          const float2 m23 = __half22float2(*reinterpret_cast<const __half2 *>(&mm.y));
          msc[r][0] = live ? m01.x : 0.0f;
          msc[r][1] = live ? m01.y : 0.0f;
          msc[r][2] = live ? m23.x : 0.0f;
          msc[r][3] = live ? m23.y : 0.0f;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kb = 32 * (4 * G + j);
        // x[i, kb .. kb+31] as 8 float4; zero past K (tail and padded blocks)
        float4 xv[M][8];
#pragma unroll
        for (int i = 0; i < M; ++i) {
          const float *xr = a.x + (int64_t)i * a.ldx + kb;
          if (kb + 32 <= K && (((uintptr_t)xr) & 15) == 0) {
#pragma unroll
            for (int c = 0; c < 8; ++c) xv[i][c] = ld_nc_f4(xr + 4 * c);
          } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int k = kb + 4 * c;
              xv[i][c] = make_float4(k < K ? __ldg(xr + 4 * c) : 0.0f, k + 1 < K ? __ldg(xr + 4 * c + 1) : 0.0f,
                                     k + 2 < K ? __ldg(xr + 4 * c + 2) : 0.0f, k + 3 < K ? __ldg(xr + 4 * c + 3) : 0.0f);
            }
          }
        }
        float xs[M];
        if constexpr (QT == MQ_Q4_1) {
#pragma unroll
          for (int i = 0; i < M; ++i) {
            float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              s2 = __fadd2_rn(s2, make_float2(xv[i][c].x, xv[i][c].y));
              s2 = __fadd2_rn(s2, make_float2(xv[i][c].z, xv[i][c].w));
            }
            xs[i] = s2.x + s2.y;
          }
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          float2 part[M];
#pragma unroll
          for (int i = 0; i < M; ++i) part[i] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            // x pairs (2t,2t+1), (2t+8,2t+9), (2t+16,2t+17), (2t+24,2t+25) sit in float4 t/2, 2+t/2, ...
            float2 v0, v1, v2, v3;
            if constexpr (QT == MQ_Q8_0) {
              const uint32_t u0 = q[r][8 * t + 2 * j] ^ 0x80808080u, u1 = q[r][8 * t + 2 * j + 1] ^ 0x80808080u;
              v0 = decode_pair<QT>(u0, 0, 1);  // k 2t, 2t+1
              v1 = decode_pair<QT>(u0, 2, 3);  // k 2t+8, 2t+9
              v2 = decode_pair<QT>(u1, 0, 1);  // k 2t+16, 2t+17
              v3 = decode_pair<QT>(u1, 2, 3);  // k 2t+24, 2t+25
            } else {
              const uint32_t wd = q[r][4 * t + j];
              const uint32_t lo = wd & 0x0F0F0F0Fu, hi = (wd >> 4) & 0x0F0F0F0Fu;
              v0 = decode_pair<QT>(lo, 0, 2);  // k 2t, 2t+1
              v1 = decode_pair<QT>(lo, 1, 3);  // k 2t+8, 2t+9
              v2 = decode_pair<QT>(hi, 0, 2);  // k 2t+16, 2t+17
              v3 = decode_pair<QT>(hi, 1, 3);  // k 2t+24, 2t+25
            }
#pragma unroll
            for (int i = 0; i < M; ++i) {
              const float4 xa = xv[i][t >> 1], xb = xv[i][2 + (t >> 1)], xc = xv[i][4 + (t >> 1)],
                           xd = xv[i][6 + (t >> 1)];
              const bool odd = t & 1;
              part[i] = __ffma2_rn(v0, odd ? make_float2(xa.z, xa.w) : make_float2(xa.x, xa.y), part[i]);
              part[i] = __ffma2_rn(v1, odd ? make_float2(xb.z, xb.w) : make_float2(xb.x, xb.y), part[i]);
              part[i] = __ffma2_rn(v2, odd ? make_float2(xc.z, xc.w) : make_float2(xc.x, xc.y), part[i]);
              part[i] = __ffma2_rn(v3, odd ? make_float2(xd.z, xd.w) : make_float2(xd.x, xd.y), part[i]);
            }
          }
#pragma unroll
          for (int i = 0; i < M; ++i) {
            acc[r][i] = __ffma2_rn(make_float2(dsc[r][j], dsc[r][j]), part[i], acc[r][i]);
            if constexpr (QT == MQ_Q4_1) acc[r][i].x = fmaf(msc[r][j], xs[i], acc[r][i].x);
          }
        }
      }
    }
  }

  // Warp reduction, then a fixed-order combine of the K-split warps.
  __shared__ float red[8][RPW * M];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) {
      float v = acc[r][i].x + acc[r][i].y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][r * M + i] = v;
    }
  __syncthreads();
  const int nout = warps_r * RPW * M;
  for (int o = threadIdx.x; o < nout; o += blockDim.x) {
    const int wr2 = o / (RPW * M), e = o % (RPW * M), r = e / M, i = e % M;
    const int n = (blockIdx.x * warps_r + wr2) * RPW + r;
    if (n >= w.rows) continue;
    float v = red[wr2 * warps_k][e];
    for (int k2 = 1; k2 < warps_k; ++k2) v += red[wr2 * warps_k + k2][e];
    if (a.bias) v += a.bias[n];
    a.y[(int64_t)i * a.ldy + n] = v;
  }
}

}  // namespace mq
