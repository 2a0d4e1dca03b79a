// Tensor-core GEMM for many activation rows (prefill): y = x · Wᵀ on tcgen05.
//
// Precision scheme (the reference accumulates in fp32, tolerance 1e-4
// relative): both operands are split into two terms, x = xh + xl and
// w = wh + wl, and the tile accumulates xh·wh + xl·wh + xh·wl in fp32 in TMEM.
//   Scale-folded form (Q8_0 and Q4_0 weights whose d * code fits fp16, i.e.
//   mq_weight::foldable): every weight d * code is split EXACTLY into fp16
//   wh + wl (hmul2 / hfma2 of the exact fp16 code and the fp16 scale), and x
//   into fp16 xh + xl in units of a power of two per activation row
//   (split_x_f16_kernel; the epilogue multiplies by 2^-e). fp16 products are
//   exact in fp32; the dropped xl·wl term is below 2^-22 of |w x|.
//   bf16 form (Q4_1, and weights outside the fp16 range): round-to-nearest
//   bf16 splits (~16 significant bits each); the dropped xl·wl term and the
//   split residues bound every product's error by ~2^-15.4 (2.3e-5) of |w x|.
//
// Tile: 128 weight rows (MMA M, TMEM lanes) x BN activation rows (MMA N,
// TMEM columns), K in steps of 64 (two quant blocks, one 128-byte swizzle
// row of bf16). Persistent: one CTA per SM walks the tiles (activation tile
// fastest, so the CTAs working at the same time share weight tiles) with two
// TMEM accumulators, so a tile's epilogue runs while the next accumulates.
// Warp-specialised:
//   warp 0      TMA loads of the x-split tiles (xh, xl) for each K step;
//   warp 1      TMEM allocation and the single MMA-issuing thread;
//   warps 2..5  load the packed weights, decode and scale each block in
//               registers, split into bf16 hi/lo and store them into the
//               swizzled smem stage;
//   warps 6..9  drain an accumulator from TMEM to y (bias, epilogues).
// Stages are recycled through mbarriers: full_x (TMA bytes), full_w (128
// producer arrivals), empty (tcgen05.commit); accumulators through acc_full
// (commit) and acc_empty (epilogue warps). Every wait is bounded in time;
// an exhausted wait raises a flag the host reports as MQ_ERR_TIMEOUT.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <climits>

#include "mq_common.cuh"
#include "mq_fdec.cuh"
#include "mq_peer.cuh"
#include "mq_sm100.cuh"

namespace mq {

constexpr int kGemmRows = 128;       // weight rows per tile (MMA M)
constexpr int kGemmK = 64;           // K elements per stage
constexpr int kGemmEpiWarps = 4;     // epilogue warps (one per TMEM lane quarter)
constexpr int kGemmThreads = 320;    // 10 warps: TMA, MMA, 4 weight producers, 4 epilogue
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
  int *tickets = nullptr;  // one per tile, zero between launches (split tiles' arrival counts)
  float *part = nullptr;   // split segments' partial tiles: [gridDim.x][BN columns][128 rows]
  int waves = 0;           // whole-tile waves: CTA c takes tiles c, c + G, ..., c + (waves-1) G
  int tail = 0;            // tiles left after the waves (< G)
  int split = 1;           // K pieces of every tail tile (tail * split <= G)
  const float *xinv = nullptr;  // scale-folded form: 2^-e of every activation row
};

// Schedule (G CTAs, one per SM): the tiles run in whole waves, CTA c taking
// tile c + w G in wave w, so the CTAs of a wave work on neighbouring tiles at
// the same K position and share their operands in L2. The last tail < G tiles
// are split into `split` K pieces each, piece j of tail tile r going to CTA
// r + j * tail: the CTAs again work on neighbouring tiles at the same K range.
// A piece writes its partial tile to its CTA's slot; the piece that arrives
// last sums the slots in K order (deterministic) and writes y.
struct GemmSeg {
  int t, k0, k1;
};
__device__ __forceinline__ GemmSeg gemm_seg(const GemmArgs &a, int u) {
  const int G = gridDim.x, c = blockIdx.x, KT = a.ktiles;
  if (u < a.waves) return {c + u * G, 0, KT};
  const int r = c % a.tail, j = c / a.tail;
  return {a.waves * G + r, (int)((int64_t)j * KT / a.split), (int)((int64_t)(j + 1) * KT / a.split)};
}
__device__ __forceinline__ int gemm_segments(const GemmArgs &a) {
  return a.waves + ((int)blockIdx.x < a.tail * a.split ? 1 : 0);
}

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

// Scale-folded form: x (fp32, [m, ldx]) -> xh, xl (fp16, [m, kpad]) in units
// of 2^e of its row, e putting the row's max |x| in [2^13, 2^14) (hi stays in
// the fp16 range; lo misses x by at most 2^-25 of those units, 2^-38 of the
// row's max); xinv[row] = 2^-e. One CTA per row; columns >= K are zero.
constexpr int kSplitThreads = 256;
__global__ void __launch_bounds__(kSplitThreads)
    split_x_f16_kernel(const float *__restrict__ x, int64_t ldx, int K, int kpad, __half *__restrict__ xh,
                       __half *__restrict__ xl, float *__restrict__ xinv) {
  __shared__ float s_max[kSplitThreads / 32];
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float *xr = x + (int64_t)row * ldx;
  float mx = 0.0f;
  for (int k = threadIdx.x; k < K; k += kSplitThreads) mx = fmaxf(mx, fabsf(xr[k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_max[warp] = mx;
  __syncthreads();
  mx = s_max[0];
#pragma unroll
  for (int w = 1; w < kSplitThreads / 32; ++w) mx = fmaxf(mx, s_max[w]);
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int E;
    frexpf(mx, &E);
    e = min(100, max(-100, 14 - E));
  }
  const float sc = ldexpf(1.0f, e);
  if (threadIdx.x == 0) xinv[row] = ldexpf(1.0f, -e);
  __half2 *h2 = reinterpret_cast<__half2 *>(xh + (int64_t)row * kpad);
  __half2 *l2 = reinterpret_cast<__half2 *>(xl + (int64_t)row * kpad);
  for (int p = threadIdx.x; p < (kpad >> 1); p += kSplitThreads) {
    const int k = 2 * p;
    const float v0 = k < K ? xr[k] * sc : 0.0f, v1 = k + 1 < K ? xr[k + 1] * sc : 0.0f;
    const __half2 hh = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(hh);
    h2[p] = hh;
    l2[p] = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
  }
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
  // full_x, full_w, empty per stage; acc_full, acc_empty per accumulator; fin
  static constexpr int kBytes = kBarOff + 8 * (3 * STAGES + 5) + 16;  // + TMEM slot, abort flag
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static_assert(2 * BN <= 512, "two accumulators in TMEM");
};

template <int QT, int BN, int STAGES, bool FOLD>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl, const GemmArgs a) {
  using L = GemmSmem<QT, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_x = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full_w = full_x + STAGES;
  uint64_t *empty = full_w + STAGES;
  uint64_t *acc_full = empty + STAGES;  // [2]
  uint64_t *acc_empty = acc_full + 2;   // [2]
  uint64_t *fin = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = a.ktiles;
  // Tile t = (weight tile t / ntm, activation tile t % ntm): the activation
  // tile varies fastest, so neighbouring tiles share their weight tile.
  const int ntm = (a.m + BN - 1) / BN;
  const int NU = gemm_segments(a);  // this CTA's segments (tile, K range)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full_x[s], 1);
      sm100::mbar_init(&full_w[s], 128);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) sm100::mbar_init(&acc_full[i], 1), sm100::mbar_init(&acc_empty[i], kGemmEpiWarps);
    sm100::mbar_init(fin, 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    sm100::prefetch_tmap(&tm_xh);
    sm100::prefetch_tmap(&tm_xl);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 2 * BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s) { return smem + s * L::kStage; };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer: activation split tiles
      int it = 0, issued = 0;
      bool ok = true;
      for (int u = 0; ok && u < NU; ++u) {
        const GemmSeg sg = gemm_seg(a, u);
        const int k0 = sg.k0, k1 = sg.k1;
        const int m0 = (sg.t % ntm) * BN;
        for (int kt = k0; kt < k1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!(ok = sm100::mbar_wait(&empty[s], ph ^ 1u, a.err, abort, kWaitLimitNs))) break;
          uint8_t *st = stage_ptr(s);
          sm100::mbar_arrive_expect_tx(&full_x[s], 2 * L::kX);
          sm100::tma_load_2d(st + 2 * L::kW, &tm_xh, kt * kGemmK, m0, &full_x[s]);
          sm100::tma_load_2d(st + 2 * L::kW + L::kX, &tm_xl, kt * kGemmK, m0, &full_x[s]);
          issued = it + 1;
        }
      }
      // Let the last copies land before the CTA can exit (immediate on the normal path).
      for (int i = issued - STAGES < 0 ? 0 : issued - STAGES; i < issued; ++i)
        sm100::mbar_wait(&full_x[i % STAGES], (uint32_t)(i / STAGES) & 1u, nullptr, nullptr, kDrainLimitNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer: segment lt into accumulator lt & 1
      constexpr uint32_t idesc = FOLD ? idesc_f16_f32(kGemmRows, BN) : sm100::idesc_bf16_f32(kGemmRows, BN);
      int it = 0, lt = 0;
      bool ok = true;
      for (int u = 0; ok && u < NU; ++u, ++lt) {
        const GemmSeg sg = gemm_seg(a, u);
        const int k0 = sg.k0, k1 = sg.k1;
        const int acc = lt & 1;
        // the epilogue has read this accumulator's previous segment
        ok = sm100::mbar_wait(&acc_empty[acc], ((uint32_t)(lt >> 1) & 1u) ^ 1u, a.err, abort, kWaitLimitNs);
        sm100::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kt = k0; ok && kt < k1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!(ok = sm100::mbar_wait(&full_x[s], ph, a.err, abort, kWaitLimitNs))) break;
          if (!(ok = sm100::mbar_wait(&full_w[s], ph, a.err, abort, kWaitLimitNs))) break;
          sm100::tc_fence_after();
          const uint32_t base = sm100::smem_u32(stage_ptr(s));
          const uint64_t dwh = sm100::umma_desc_sw128(base), dwl = sm100::umma_desc_sw128(base + L::kW);
          const uint64_t dxh = sm100::umma_desc_sw128(base + 2 * L::kW);
          const uint64_t dxl = sm100::umma_desc_sw128(base + 2 * L::kW + L::kX);
#pragma unroll
          for (int kk = 0; kk < kGemmK / 16; ++kk) {
            const uint64_t off = (uint64_t)(2 * kk);  // 32 bytes per 16-element K step, in 16-byte units
            sm100::umma_bf16(d, dwh + off, dxh + off, idesc, (kt != k0 || kk != 0) ? 1u : 0u);
            sm100::umma_bf16(d, dwh + off, dxl + off, idesc, 1u);
            sm100::umma_bf16(d, dwl + off, dxh + off, idesc, 1u);
          }
          sm100::umma_commit(&empty[s]);
        }
        if (ok) sm100::umma_commit(&acc_full[acc]);
      }
      // Every MMA issued has completed before the TMEM is released.
      sm100::umma_commit(fin);
      sm100::mbar_wait(fin, 0u, nullptr, nullptr, kDrainLimitNs);
    }
  } else if (warp < 2 + 4) {
    // ---------------- weight producers (128 threads): decode, scale, split into bf16 hi/lo stages
    const int r = 32 * (warp & 3) + lane;  // tile row
    const WeightView &w = a.w;
    int it = 0;
    bool ok = true;
    for (int u = 0; ok && u < NU; ++u) {
      const GemmSeg sg = gemm_seg(a, u);
      const int t = sg.t, k0 = sg.k0, k1 = sg.k1;
      const int n = (t / ntm) * kGemmRows + r;
      const bool row_ok = n < w.rows;
      const int rn = row_ok ? n : 0, tn = rn / kTileRows, rr = rn % kTileRows;
      // Weights of the next two K steps in flight (a ring of two register sets).
      StepWords<QT> qa, qb;
      float2 da = make_float2(0.0f, 0.0f), db = da, ma = da, mb = da;
      auto fetch = [&](int kt, StepWords<QT> &qn, float2 &dn, float2 &mnn) {  // blocks 2kt, 2kt+1 (zero-padded past nb)
        const uint8_t *chunk = chunk_ptr(w, tn, kt >> 2);  // 8 blocks per chunk step
        const int qd = (kt & 3) >> 1, jb = 2 * (kt & 3);    // quad of the step, first block of the pair
        if (row_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            if constexpr (QT == MQ_Q8_0) {
              // cached in L1: the rest of each 32-byte sector is the next K step's
              const uint4 v = __ldg(reinterpret_cast<const uint4 *>(chunk + chunk16_off(rr, 2 * q4 + (kt & 1), qd)));
              qn.w[q4][0][0] = v.x, qn.w[q4][0][1] = v.y, qn.w[q4][1][0] = v.z, qn.w[q4][1][1] = v.w;
            } else {
              const uint2 v =
                  __ldg(reinterpret_cast<const uint2 *>(chunk + chunk16_off(rr, 4 * qd + q4, 0) + 8 * (kt & 1)));
              qn.w[q4][0][0] = v.x, qn.w[q4][1][0] = v.y;
            }
          }
          const uint8_t *sc = chunk + w.pk_bytes + rr * 16 + 2 * jb;
          dn = __half22float2(*reinterpret_cast<const __half2 *>(sc));
          if constexpr (QT == MQ_Q4_1) mnn = __half22float2(*reinterpret_cast<const __half2 *>(sc + 2048));
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj)
#pragma unroll
              for (int h = 0; h < (QT == MQ_Q8_0 ? 2 : 1); ++h) qn.w[q4][jj][h] = 0u;
          dn = make_float2(0.0f, 0.0f);
          mnn = make_float2(0.0f, 0.0f);
        }
      };
      fetch(k0, qa, da, ma);
      if (k0 + 1 < k1) fetch(k0 + 1, qb, db, mb);
      for (int kt = k0; kt < k1; ++kt, ++it) {
        const StepWords<QT> q = qa;
        const float2 d = da, mn = ma;
        qa = qb, da = db, ma = mb;
        if (kt + 2 < k1) fetch(kt + 2, qb, db, mb);
        const int s = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!(ok = sm100::mbar_wait(&empty[s], ph ^ 1u, a.err, abort, kWaitLimitNs))) break;
        uint8_t *wh = stage_ptr(s) + r * 128, *wl = wh + L::kW;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = elements 8c..8c+7 of the 64-wide K step
          uint4 hv, lv;
          if constexpr (FOLD) {  // exact fp16 codes, d * code split exactly into fp16 hi + lo
            const int jj = c >> 2, u = c & 3;
            const __half2 d2 = __float2half2_rn(jj ? d.y : d.x);  // the fp16 scale itself
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {  // elements 2t, 2t+1 of the chunk
              uint32_t code;
              if constexpr (QT == MQ_Q8_0)
                code = dcode_q8(q.w[t][jj][u >> 1] ^ 0x80808080u, (u & 1) ? 0x4342u : 0x4140u);
              else
                code = dcode_q4<QT>(q.w[t][jj][0], ((u & 1) ? 8 : 0) + ((u >= 2) ? 4 : 0));
              fold_pair(code, d2, hw[t], lw[t]);
            }
            hv = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            lv = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          } else {
            float v[8];
            decode_chunk<QT>(q, c >> 2, c & 3, (c >> 2) ? d.y : d.x, (c >> 2) ? mn.y : mn.x, v);
            split_pair(v[0], v[1], hv.x, lv.x);
            split_pair(v[2], v[3], hv.y, lv.y);
            split_pair(v[4], v[5], hv.z, lv.z);
            split_pair(v[6], v[7], hv.w, lv.w);
          }
          const int off = (c ^ (r & 7)) * 16;  // 128-byte swizzle
          *reinterpret_cast<uint4 *>(wh + off) = hv;
          *reinterpret_cast<uint4 *>(wl + off) = lv;
        }
        sm100::fence_proxy_async_smem();
        sm100::mbar_arrive(&full_w[s]);
      }
    }
  } else {
    // ---------------- epilogue (4 warps): accumulator lt & 1 -> y, or -> a partial slot
    // Failed waits do not leave the loop: the four warps take the same
    // named-barrier sequence, and every split segment counts its arrival so
    // the tickets return to zero.
    const int r = 32 * (warp & 3) + lane;  // tile row == TMEM lane this warp may access
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const bool leader = threadIdx.x == (2 + 4) * 32;
    int lt = 0;
    for (int u = 0; u < NU; ++u, ++lt) {
      const GemmSeg sg = gemm_seg(a, u);
      const int t = sg.t, k0 = sg.k0, k1 = sg.k1;
      const int acc = lt & 1;
      const int m0 = (t % ntm) * BN, n = (t / ntm) * kGemmRows + r;
      const bool row_ok = n < a.w.rows;
      const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait(&acc_full[acc], (uint32_t)(lt >> 1) & 1u, a.err, abort,
                                                               kWaitLimitNs)) &&
                      !*abort;
      sm100::tc_fence_after();
      const float bias = (row_ok && a.bias) ? a.bias[n] : 0.0f;
      if (k0 == 0 && k1 == KT) {  // the whole tile in this segment: straight to y
#pragma unroll 1
        for (int c0 = 0; ok && c0 < BN; c0 += 32) {
          uint32_t v[32];
          sm100::tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(acc * BN + c0), v);
          sm100::tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int mm = m0 + c0 + j;
              if (mm < a.m) {
                const float acc_v = FOLD ? __uint_as_float(v[j]) * __ldg(a.xinv + mm) : __uint_as_float(v[j]);
                a.y[(int64_t)mm * a.ldy + n] = epilogue_out(acc_v + bias, a.gate, a.resid, (int64_t)mm * a.ldy + n);
              }
            }
          }
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&acc_empty[acc]);
        continue;
      }
      // A split tile: the partial goes to this CTA's slot (column-major, rows contiguous).
      float *ps = a.part + (size_t)blockIdx.x * (BN * kGemmRows);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        if (ok) {
          sm100::tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(acc * BN + c0), v);
          sm100::tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0x7fc00000u;  // NaN: the launch failed
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) ps[(c0 + j) * kGemmRows + r] = __uint_as_float(v[j]);
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&acc_empty[acc]);
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (leader) s_last = atomicAdd(&a.tickets[t], 1) == a.split - 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!s_last) continue;
      __threadfence();
      // Every segment of the tile has arrived: sum the slots in K order, 32
      // columns at a time (32 loads in flight per thread).
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float sum[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[j] = 0.0f;
#pragma unroll 1
        for (int j = 0; j < a.split; ++j) {  // piece j of tail tile t was CTA (t - waves G) + j tail
          const int slot = (t - a.waves * (int)gridDim.x) + j * a.tail;
          const float *src = a.part + (size_t)slot * (BN * kGemmRows) + c0 * kGemmRows + r;
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[j] += __ldcg(src + j * kGemmRows);
        }
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int mm = m0 + c0 + j;
            if (mm < a.m) {
              const float acc_v = FOLD ? sum[j] * __ldg(a.xinv + mm) : sum[j];
              a.y[(int64_t)mm * a.ldy + n] = epilogue_out(acc_v + bias, a.gate, a.resid, (int64_t)mm * a.ldy + n);
            }
          }
        }
      }
      if (leader) a.tickets[t] = 0;  // ready for the next launch
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 2 * BN);
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
