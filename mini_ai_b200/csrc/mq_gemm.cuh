// Tensor-core GEMM for many activation rows (prefill): y = x · Wᵀ on tcgen05.
//
// Precision scheme (the reference accumulates in fp32, tolerance 1e-4
// relative): both operands are split into two bf16 terms with round-to-
// nearest, x = xh + xl and w = wh + wl (each pair carries ~16 significant
// bits), and the tile accumulates xh·wh + xl·wh + xh·wl in fp32 in TMEM.
// The dropped xl·wl term and the split residues bound the relative error of
// every product by ~2^-15.4 (2.3e-5) of |w x|.
//
// Tile: 128 weight rows (MMA M, TMEM lanes) x BN activation rows (MMA N,
// TMEM columns), K in steps of 64 (two quant blocks, one 128-byte swizzle
// row of bf16). One CTA per tile, grid (activation tiles, weight tiles),
// warp-specialised:
//   warp 0      TMA loads of the x-split tiles (xh, xl) for each K step;
//   warp 1      TMEM allocation and the single MMA-issuing thread;
//   warps 2..5  load the packed weights, decode and scale each block in
//               registers, split into bf16 hi/lo and store them into the
//               swizzled smem stage; afterwards they drain TMEM to y.
// Stages are recycled through mbarriers: full_x (TMA bytes), full_w (128
// producer arrivals), empty (tcgen05.commit). Every wait is bounded in time;
// an exhausted wait raises a flag the host reports as MQ_ERR_TIMEOUT.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <climits>

#include "mq_common.cuh"
#include "mq_peer.cuh"
#include "mq_sm100.cuh"

namespace mq {

constexpr int kGemmRows = 128;       // weight rows per tile (MMA M)
constexpr int kGemmK = 64;           // K elements per stage
constexpr int kGemmThreads = 192;    // 6 warps
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait (a K step takes microseconds)
constexpr uint64_t kDrainLimitNs = 20000000ull;  // 20 ms for copies already in flight

struct GemmArgs {
  WeightView w;
  float *y;
  int64_t ldy;
  const float *bias;
  int m;         // activation rows
  int ktiles;    // ceil(nb / 2) K steps of 64
  int *err;      // device-visible error flag
  const float *gate = nullptr;   // fused gate/up product: y = silu(gate) * (product + bias); gate [m, ldy]
  const float *resid = nullptr;  // residual add: y = resid + (product + bias); resid [m, ldy], may be y
};

// x (fp32, [m, ldx]) -> xh, xl (bf16, [m, kpad]); columns >= K are zero.
__global__ void split_x_kernel(const float *__restrict__ x, int64_t ldx, int m, int K, int kpad,
                               __nv_bfloat16 *__restrict__ xh, __nv_bfloat16 *__restrict__ xl) {
  const int pairs = kpad >> 1;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)m * pairs) return;
  const int64_t r = i / pairs;
  const int k = (int)(i % pairs) * 2;
  const float v0 = k < K ? x[r * ldx + k] : 0.0f;
  const float v1 = k + 1 < K ? x[r * ldx + k + 1] : 0.0f;
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
  reinterpret_cast<__nv_bfloat162 *>(xh + r * kpad)[k >> 1] = h;
  reinterpret_cast<__nv_bfloat162 *>(xl + r * kpad)[k >> 1] = l;
}

// bf16 hi/lo split of a decoded pair, packed as two 32-bit words.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Byte k of v spliced under 2^23 (exact small-integer-to-float).
__device__ __forceinline__ float gsplice(uint32_t v, int k) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)k));
}

template <int QT> struct GemmQ;
template <> struct GemmQ<MQ_Q4_0> { static constexpr float kMagic = 8388616.0f; };
template <> struct GemmQ<MQ_Q4_1> { static constexpr float kMagic = 8388608.0f; };
template <> struct GemmQ<MQ_Q8_0> { static constexpr float kMagic = 8388736.0f; };

// Quant words of one weight row for one 64-wide K step (blocks j0, j0 + 1 of
// a 4-block group of the lane-permuted layout): for each lane quad t,
// Q4_x: word (t, j) = bytes {2t, 2t+8, 2t+1, 2t+9} of block j;
// Q8_0: words (t, j, 0..1) = bytes {2t, 2t+1, 2t+8, 2t+9 | 2t+16, 2t+17, 2t+24, 2t+25}.
template <int QT> struct StepWords { uint32_t w[4][2][QT == MQ_Q8_0 ? 2 : 1]; };

// Decoded values of chunk u (elements 8u..8u+7) of block jj of the K step:
// element 2t and 2t+1 of the chunk come from lane quad t's word.
template <int QT>
__device__ __forceinline__ void decode_chunk(const StepWords<QT> &q, int jj, int u, float d, float mn, float (&v)[8]) {
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float qa, qb;
    if constexpr (QT == MQ_Q8_0) {
      const uint32_t x = q.w[t][jj][u >> 1] ^ 0x80808080u;
      qa = gsplice(x, (u & 1) ? 2 : 0) - GemmQ<QT>::kMagic;
      qb = gsplice(x, (u & 1) ? 3 : 1) - GemmQ<QT>::kMagic;
    } else {
      const uint32_t wd = q.w[t][jj][0];
      const uint32_t x = (u >= 2) ? (wd >> 4) & 0x0F0F0F0Fu : wd & 0x0F0F0F0Fu;
      qa = gsplice(x, (u & 1) ? 1 : 0) - GemmQ<QT>::kMagic;
      qb = gsplice(x, (u & 1) ? 3 : 2) - GemmQ<QT>::kMagic;
    }
    if constexpr (QT == MQ_Q4_1) {
      v[2 * t] = fmaf(d, qa, mn);
      v[2 * t + 1] = fmaf(d, qb, mn);
    } else {
      v[2 * t] = d * qa;
      v[2 * t + 1] = d * qb;
    }
  }
}

template <int QT, int BN, int STAGES>
struct GemmSmem {
  static constexpr int kW = kGemmRows * kGemmK * 2;  // bytes of one bf16 weight tile (hi or lo)
  static constexpr int kX = BN * kGemmK * 2;         // bytes of one bf16 activation tile
  static constexpr int kStage = 2 * kW + 2 * kX;
  static constexpr int kBarOff = STAGES * kStage;
  static constexpr int kBytes = kBarOff + 8 * (3 * STAGES + 1) + 16;  // barriers, TMEM slot, abort flag
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

template <int QT, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl, const GemmArgs a) {
  using L = GemmSmem<QT, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_x = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full_w = full_x + STAGES;
  uint64_t *empty = full_w + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Raster: the activation tile varies fastest, so the CTAs that share a
  // weight tile run at the same time and its bytes come from HBM once.
  const int n0 = blockIdx.y * kGemmRows, m0 = blockIdx.x * BN;
  const int KT = a.ktiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full_x[s], 1);
      sm100::mbar_init(&full_w[s], 128);
      sm100::mbar_init(&empty[s], 1);
    }
    sm100::mbar_init(acc_full, 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    sm100::prefetch_tmap(&tm_xh);
    sm100::prefetch_tmap(&tm_xl);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s) { return smem + s * L::kStage; };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer: activation split tiles
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!sm100::mbar_wait(&empty[s], ph ^ 1u, a.err, abort, kWaitLimitNs)) break;
        uint8_t *st = stage_ptr(s);
        sm100::mbar_arrive_expect_tx(&full_x[s], 2 * L::kX);
        sm100::tma_load_2d(st + 2 * L::kW, &tm_xh, kt * kGemmK, m0, &full_x[s]);
        sm100::tma_load_2d(st + 2 * L::kW + L::kX, &tm_xl, kt * kGemmK, m0, &full_x[s]);
        issued = kt + 1;
      }
      // Let the last copies land before the CTA can exit (immediate on the normal path).
      for (int kt = issued - STAGES < 0 ? 0 : issued - STAGES; kt < issued; ++kt)
        sm100::mbar_wait(&full_x[kt % STAGES], (uint32_t)(kt / STAGES) & 1u, nullptr, nullptr, kDrainLimitNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(kGemmRows, BN);
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!sm100::mbar_wait(&full_x[s], ph, a.err, abort, kWaitLimitNs)) break;
        if (!sm100::mbar_wait(&full_w[s], ph, a.err, abort, kWaitLimitNs)) break;
        sm100::tc_fence_after();
        const uint32_t base = sm100::smem_u32(stage_ptr(s));
        const uint64_t dwh = sm100::umma_desc_sw128(base), dwl = sm100::umma_desc_sw128(base + L::kW);
        const uint64_t dxh = sm100::umma_desc_sw128(base + 2 * L::kW);
        const uint64_t dxl = sm100::umma_desc_sw128(base + 2 * L::kW + L::kX);
#pragma unroll
        for (int kk = 0; kk < kGemmK / 16; ++kk) {
          const uint64_t off = (uint64_t)(2 * kk);  // 32 bytes per 16-element K step, in 16-byte units
          sm100::umma_bf16(tmem, dwh + off, dxh + off, idesc, (kt | kk) != 0);
          sm100::umma_bf16(tmem, dwh + off, dxl + off, idesc, 1u);
          sm100::umma_bf16(tmem, dwl + off, dxh + off, idesc, 1u);
        }
        sm100::umma_commit(&empty[s]);
      }
      sm100::umma_commit(acc_full);
    }
  } else {
    // ---------------- weight producers (128 threads), then the epilogue
    const int r = 32 * (warp & 3) + lane;  // tile row == TMEM lane this warp may access
    const int n = n0 + r;
    const bool row_ok = n < a.w.rows;
    const WeightView &w = a.w;
    const int rn = row_ok ? n : 0, tn = rn / kTileRows, rr = rn % kTileRows;

    StepWords<QT> qn;
    float2 dn = make_float2(0.0f, 0.0f), mnn = make_float2(0.0f, 0.0f);
    auto fetch = [&](int kt) {  // blocks 2kt, 2kt+1 (zero-padded past nb in the layout)
      const uint8_t *chunk = chunk_ptr(w, tn, kt >> 2);  // 8 blocks per chunk step
      const int qd = (kt & 3) >> 1, jb = 2 * (kt & 3);    // quad of the step, first block of the pair
      if (row_ok) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if constexpr (QT == MQ_Q8_0) {
            const uint4 v = ld_stream_v4(chunk + chunk16_off(rr, 2 * t + (kt & 1), qd));
            qn.w[t][0][0] = v.x, qn.w[t][0][1] = v.y, qn.w[t][1][0] = v.z, qn.w[t][1][1] = v.w;
          } else {
            const uint2 v = ld_stream_v2(chunk + chunk16_off(rr, 4 * qd + t, 0) + 8 * (kt & 1));
            qn.w[t][0][0] = v.x, qn.w[t][1][0] = v.y;
          }
        }
        const uint8_t *sc = chunk + w.pk_bytes + rr * 16 + 2 * jb;
        dn = __half22float2(*reinterpret_cast<const __half2 *>(sc));
        if constexpr (QT == MQ_Q4_1) mnn = __half22float2(*reinterpret_cast<const __half2 *>(sc + 2048));
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
#pragma unroll
            for (int h = 0; h < (QT == MQ_Q8_0 ? 2 : 1); ++h) qn.w[t][jj][h] = 0u;
        dn = make_float2(0.0f, 0.0f);
        mnn = make_float2(0.0f, 0.0f);
      }
    };
    fetch(0);
    for (int kt = 0; kt < KT; ++kt) {
      const StepWords<QT> q = qn;
      const float2 d = dn, mn = mnn;
      if (kt + 1 < KT) fetch(kt + 1);  // next K step's weights in flight while this one is decoded
      const int s = kt % STAGES;
      const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
      if (!sm100::mbar_wait(&empty[s], ph ^ 1u, a.err, abort, kWaitLimitNs)) break;
      uint8_t *wh = stage_ptr(s) + r * 128, *wl = wh + L::kW;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = elements 8c..8c+7 of the 64-wide K step
        float v[8];
        decode_chunk<QT>(q, c >> 2, c & 3, (c >> 2) ? d.y : d.x, (c >> 2) ? mn.y : mn.x, v);
        uint4 hv, lv;
        split_pair(v[0], v[1], hv.x, lv.x);
        split_pair(v[2], v[3], hv.y, lv.y);
        split_pair(v[4], v[5], hv.z, lv.z);
        split_pair(v[6], v[7], hv.w, lv.w);
        const int off = (c ^ (r & 7)) * 16;  // 128-byte swizzle
        *reinterpret_cast<uint4 *>(wh + off) = hv;
        *reinterpret_cast<uint4 *>(wl + off) = lv;
      }
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(&full_w[s]);
    }

    // ---------------- epilogue: TMEM -> registers -> y (+ bias)
    // acc_full is committed on every path (after the MMAs issued so far), so
    // this wait also guarantees no MMA still writes TMEM when it is freed.
    const bool acc_ok = sm100::mbar_wait(acc_full, 0u, a.err, nullptr, kWaitLimitNs) && !*abort;
    sm100::tc_fence_after();
    const float bias = (row_ok && a.bias) ? a.bias[n] : 0.0f;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
#pragma unroll 1
    for (int c0 = 0; acc_ok && c0 < BN; c0 += 32) {
      uint32_t v[32];
      sm100::tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)c0, v);
      sm100::tmem_ld_wait();
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int mm = m0 + c0 + j;
          if (mm < a.m) a.y[(int64_t)mm * a.ldy + n] = epilogue_out(__uint_as_float(v[j]) + bias, a.gate, a.resid, (int64_t)mm * a.ldy + n);
        }
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, BN);
  }
}

// Host side (mq_gemm_host.cuh).
int decode_max_m();
int sdec_max_m();
bool gemm_supported(int device);
// gate, resid: optional [m, ldy] buffers of the output epilogues (fused
// gate/up product: y = silu(gate) * product; residual add: y = resid + product).
int run_sdec(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
             cudaStream_t s, const float *gate = nullptr, const float *resid = nullptr);
// folded: the scale-folded kernel (mq_fdec.cuh), for weights with mq_weight::foldable.
int run_tcdec(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
              cudaStream_t s, const float *gate = nullptr, const float *resid = nullptr, bool folded = false,
              const PeerOut *peer = nullptr, bool pairs = false);
int run_gemm(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
             cudaStream_t s, const float *gate = nullptr, const float *resid = nullptr);

}  // namespace mq
