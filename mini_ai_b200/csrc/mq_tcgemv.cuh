// Tensor-core decode GEMV for a few activation rows (M <= 8 * NT).
//
// HBM-bound like the SIMT GEMV, but the multiply-accumulate runs on the
// tensor pipe, so the SIMT issue budget only pays for decoding: at M = 4..16
// the fp32 FMA count of a SIMT dot would exceed the time HBM needs to
// stream the weights.
//
// Each warp owns RG groups of 16 weight rows (the MMA M dimension) and the
// activations are the MMA N dimension, 8 rows per tile (NT tiles). Because
// the device layout is lane-permuted, one 16-byte load per fragment row
// hands every lane exactly the 4 bytes per block that an m16n8k16 A
// fragment needs. Decode is three integer ops per pair of weights: shift,
// mask the two nibbles into the mantissa of 1024.0 (fp16), subtract
// 1024 + zero point with one packed half subtract -> exact small integers
// (bytes: byte_perm under 0x64 instead of the mask). Per 32-element block a
// fresh fp32 fragment accumulates 4 MMAs (two K steps, activation high and
// low parts) and is scaled into the running fp32 accumulator by the block's
// fp16 scale (plus the Q4_1 min times the block sum of x), so the block scale
// is applied exactly as in the reference dot, once per block.
//
// Activations are pre-split by tcx_prep_kernel: each row is scaled by a power
// of two (its largest magnitude lands in [2^13, 2^14)), split into fp16
// hi + lo (22 significant bits, error <= 2^-22 relative or 2^-38 of the row
// maximum), and written in B-fragment order so one 16-byte load gives a lane
// both parts of a K step. Products of exact integers and fp16 values are exact
// in the fp32 accumulator; the result matches the fp32 reference dot to
// accumulation-order rounding.
//
// The CTA's warps split K; their fragments are combined in shared memory in a
// fixed order (deterministic), then scaled back by 2^-e per activation row.
#pragma once

#include <cuda_fp16.h>

#include "mq_common.cuh"

namespace mq {

struct TcArgs {
  WeightView w;
  const uint4 *xf;      // [NT][nbp][2][32] fragments {hi b01, hi b23, lo b01, lo b23}
  const float *xsum;    // [NT][nbp][8] scaled block sums (Q4_1)
  const float *xinv;    // [8*NT] 2^-e per activation row
  int m;
  const float *bias;
  float *y;
  int64_t ldy;
};

// Activation split: one CTA per activation row (rows >= m are written as zeros).
__global__ void tcx_prep_kernel(const float *__restrict__ x, int64_t ldx, int m, int K, int nbp, uint4 *__restrict__ xf,
                                float *__restrict__ xsum, float *__restrict__ xinv, int want_sums) {
  const int row = blockIdx.x;
  const bool live = row < m;
  const float *xr = x + (int64_t)(live ? row : 0) * ldx;
  __shared__ float red[32];
  __shared__ float s_scale;
  float mx = 0.0f;
  if (live)
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(xr[k]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, red[i]);
    int e = 0;
    if (v > 0.0f && isfinite(v)) {
      int E;
      frexpf(v, &E);  // v < 2^E
      e = min(100, max(-100, 14 - E));
    }
    s_scale = ldexpf(1.0f, e);
    xinv[row] = ldexpf(1.0f, -e);
  }
  __syncthreads();
  const float sc = s_scale;
  const int nt = row >> 3, g = row & 7;
  // fragments: item = (block b, step s, lane quad t)
  for (int it = threadIdx.x; it < nbp * 8; it += blockDim.x) {
    const int b = it >> 3, s = (it >> 2) & 1, t = it & 3;
    const int k0 = 32 * b + 16 * s + 2 * t;
    float v[4];
    const int ks[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = (live && ks[u] < K) ? xr[ks[u]] * sc : 0.0f;
    const __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v[0] - f01.x, v[1] - f01.y), l23 = __floats2half2_rn(v[2] - f23.x, v[3] - f23.y);
    uint4 out;
    out.x = *reinterpret_cast<const uint32_t *>(&h01);
    out.y = *reinterpret_cast<const uint32_t *>(&h23);
    out.z = *reinterpret_cast<const uint32_t *>(&l01);
    out.w = *reinterpret_cast<const uint32_t *>(&l23);
    xf[(((int64_t)nt * nbp + b) * 2 + s) * 32 + g * 4 + t] = out;
  }
  if (want_sums)
    for (int b = threadIdx.x; b < nbp; b += blockDim.x) {
      float s = 0.0f;
      if (live)
        for (int k = 32 * b; k < min(K, 32 * b + 32); ++k) s += xr[k] * sc;
      xsum[((int64_t)nt * nbp + b) * 8 + g] = s;
    }
}

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two exact fp16 values (q - zp) from the nibbles at bits sh..sh+3 and 16+sh..19+sh.
template <int QT>
__device__ __forceinline__ uint32_t dec_q4(uint32_t w, int sh) {
  const uint32_t v = ((w >> sh) & 0x000F000Fu) | 0x64006400u;  // 1024 + q, two halves
  const __half2 z = QT == MQ_Q4_0 ? __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408))   // 1032
                                  : __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));  // 1024
  const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&v), z);
  return *reinterpret_cast<const uint32_t *>(&r);
}
// Two exact fp16 int8 values from bytes (sel) of u (already ^0x80 per byte).
__device__ __forceinline__ uint32_t dec_q8(uint32_t u, unsigned sel) {
  const uint32_t v = __byte_perm(u, 0x64646464u, sel);  // 1024 + (b + 128)
  const __half2 z = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&v), z);
  return *reinterpret_cast<const uint32_t *>(&r);
}

template <int QT, int NT, int RG>
__global__ void __launch_bounds__(256) tcgemv_kernel(const TcArgs a) {
  constexpr int LW = QT == MQ_Q8_0 ? 8 : 4;  // words per lane per fragment row per group
  static_assert(LW * 16 == (QT == MQ_Q8_0 ? 128 : 64), "group bytes");
  extern __shared__ float tc_red[];           // [nwarps][RG*NT*4][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const WeightView &w = a.w;
  const int r0 = blockIdx.x * 16 * RG;
  const int nbp = 4 * w.nb4;

  float acc[RG][NT][4];
#pragma unroll
  for (int rg = 0; rg < RG; ++rg)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[rg][n][c] = 0.0f;

  for (int G = warp; G < w.nb4; G += nwarps) {
    uint32_t qa[RG][LW], qb[RG][LW];
    float2 da[RG][2], db[RG][2], ma[RG][2], mb[RG][2];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) {
      const int ra = min(r0 + 16 * rg + g, w.rows_pad - 1), rb = min(ra + 8, w.rows_pad - 1);
      const uint8_t *pa = w.qs + (int64_t)ra * w.ld_qs + (int64_t)G * (LW * 16) + t * (LW * 4);
      const uint8_t *pb = w.qs + (int64_t)rb * w.ld_qs + (int64_t)G * (LW * 16) + t * (LW * 4);
#pragma unroll
      for (int h = 0; h < LW / 4; ++h) {
        const uint4 va = ld_stream_v4(pa + 16 * h), vb = ld_stream_v4(pb + 16 * h);
        qa[rg][4 * h] = va.x, qa[rg][4 * h + 1] = va.y, qa[rg][4 * h + 2] = va.z, qa[rg][4 * h + 3] = va.w;
        qb[rg][4 * h] = vb.x, qb[rg][4 * h + 1] = vb.y, qb[rg][4 * h + 2] = vb.z, qb[rg][4 * h + 3] = vb.w;
      }
      const uint2 sa = *reinterpret_cast<const uint2 *>(w.d + (int64_t)ra * w.ld_s + 4 * G);
      const uint2 sb = *reinterpret_cast<const uint2 *>(w.d + (int64_t)rb * w.ld_s + 4 * G);
      da[rg][0] = __half22float2(*reinterpret_cast<const __half2 *>(&sa.x));
      da[rg][1] = __half22float2(*reinterpret_cast<const __half2 *>(&sa.y));
      db[rg][0] = __half22float2(*reinterpret_cast<const __half2 *>(&sb.x));
      db[rg][1] = __half22float2(*reinterpret_cast<const __half2 *>(&sb.y));
      if constexpr (QT == MQ_Q4_1) {
        const uint2 na = *reinterpret_cast<const uint2 *>(w.mn + (int64_t)ra * w.ld_s + 4 * G);
        const uint2 nb = *reinterpret_cast<const uint2 *>(w.mn + (int64_t)rb * w.ld_s + 4 * G);
        ma[rg][0] = __half22float2(*reinterpret_cast<const __half2 *>(&na.x));
        ma[rg][1] = __half22float2(*reinterpret_cast<const __half2 *>(&na.y));
        mb[rg][0] = __half22float2(*reinterpret_cast<const __half2 *>(&nb.x));
        mb[rg][1] = __half22float2(*reinterpret_cast<const __half2 *>(&nb.y));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = 4 * G + j;
      uint4 f0[NT], f1[NT];
      float2 xs[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4 *p = a.xf + (((int64_t)n * nbp + b) * 2) * 32 + lane;
        f0[n] = __ldg(p);
        f1[n] = __ldg(p + 32);
        if constexpr (QT == MQ_Q4_1) xs[n] = __ldg(reinterpret_cast<const float2 *>(a.xsum + ((int64_t)n * nbp + b) * 8) + t);
      }
#pragma unroll
      for (int rg = 0; rg < RG; ++rg) {
        uint32_t A0[4], A1[4];  // K steps 0 and 1: {row g k 2t.., row g+8 k 2t.., row g k 2t+8.., row g+8 k 2t+8..}
        if constexpr (QT == MQ_Q8_0) {
          const uint32_t ua0 = qa[rg][2 * j] ^ 0x80808080u, ua1 = qa[rg][2 * j + 1] ^ 0x80808080u;
          const uint32_t ub0 = qb[rg][2 * j] ^ 0x80808080u, ub1 = qb[rg][2 * j + 1] ^ 0x80808080u;
          A0[0] = dec_q8(ua0, 0x4140u), A0[1] = dec_q8(ub0, 0x4140u);
          A0[2] = dec_q8(ua0, 0x4342u), A0[3] = dec_q8(ub0, 0x4342u);
          A1[0] = dec_q8(ua1, 0x4140u), A1[1] = dec_q8(ub1, 0x4140u);
          A1[2] = dec_q8(ua1, 0x4342u), A1[3] = dec_q8(ub1, 0x4342u);
        } else {
          const uint32_t wa = qa[rg][j], wb = qb[rg][j];
          A0[0] = dec_q4<QT>(wa, 0), A0[1] = dec_q4<QT>(wb, 0), A0[2] = dec_q4<QT>(wa, 8), A0[3] = dec_q4<QT>(wb, 8);
          A1[0] = dec_q4<QT>(wa, 4), A1[1] = dec_q4<QT>(wb, 4), A1[2] = dec_q4<QT>(wa, 12), A1[3] = dec_q4<QT>(wb, 12);
        }
        const float sa = (j & 1) ? da[rg][j >> 1].y : da[rg][j >> 1].x;
        const float sb = (j & 1) ? db[rg][j >> 1].y : db[rg][j >> 1].x;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma_f16(d, A0, f0[n].x, f0[n].y);
          mma_f16(d, A0, f0[n].z, f0[n].w);
          mma_f16(d, A1, f1[n].x, f1[n].y);
          mma_f16(d, A1, f1[n].z, f1[n].w);
          float2 lo = __ffma2_rn(make_float2(sa, sa), make_float2(d[0], d[1]), make_float2(acc[rg][n][0], acc[rg][n][1]));
          float2 hi = __ffma2_rn(make_float2(sb, sb), make_float2(d[2], d[3]), make_float2(acc[rg][n][2], acc[rg][n][3]));
          if constexpr (QT == MQ_Q4_1) {
            const float na = (j & 1) ? ma[rg][j >> 1].y : ma[rg][j >> 1].x;
            const float nb = (j & 1) ? mb[rg][j >> 1].y : mb[rg][j >> 1].x;
            lo = __ffma2_rn(make_float2(na, na), xs[n], lo);
            hi = __ffma2_rn(make_float2(nb, nb), xs[n], hi);
          }
          acc[rg][n][0] = lo.x, acc[rg][n][1] = lo.y, acc[rg][n][2] = hi.x, acc[rg][n][3] = hi.y;
        }
      }
    }
  }

  // Fixed-order combine of the K-split warps.
  constexpr int E = RG * NT * 4;
#pragma unroll
  for (int rg = 0; rg < RG; ++rg)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) tc_red[((warp * E) + (rg * NT + n) * 4 + c) * 32 + lane] = acc[rg][n][c];
  __syncthreads();
  for (int o = threadIdx.x; o < E * 32; o += blockDim.x) {
    const int e = o >> 5, l = o & 31;
    const int rg = e / (NT * 4), n = (e / 4) % NT, c = e & 3;
    const int row = r0 + 16 * rg + (l >> 2) + 8 * (c >> 1);
    const int xrow = 8 * n + 2 * (l & 3) + (c & 1);
    if (row >= w.rows || xrow >= a.m) continue;
    float v = 0.0f;
    for (int ww = 0; ww < nwarps; ++ww) v += tc_red[(ww * E + e) * 32 + l];
    v *= a.xinv[xrow];
    if (a.bias) v += a.bias[row];
    a.y[(int64_t)xrow * a.ldy + row] = v;
  }
}

}  // namespace mq
