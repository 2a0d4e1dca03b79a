// tcgen05 decode GEMM for a few activation rows (M <= 32).
//
// Decode is HBM-bound: every packed weight byte is streamed once. With M in
// the tens, an fp32 SIMT dot would need M FMAs per weight and fall behind
// HBM, so the products run on the 5th-generation tensor cores while the SIMT
// lanes only decode.
//
// Exactness scheme. The A operand holds the exact integers q - zp (fp16), not
// the scaled weights, so no rounding or range issue is introduced by the
// per-block fp16 scale; the activation rows are scaled by a power of two and
// split into fp16 hi + lo (22 significant bits). Each 32-weight block's MMAs
// (two K=16 steps x hi/lo) accumulate into their own TMEM slot, and drainer
// warps apply the block scale in fp32:  acc += d_b * D_b (+ m_b * sum_b x).
// Products of small integers and fp16 values are exact in the fp32
// accumulator, so the result equals the fp32 reference dot up to
// accumulation-order rounding.
//
// Persistent stream-K: one CTA per SM walks a contiguous range of the
// tile-major (128-row tile, packed K step) space, so the weight stream never
// restarts; a tile whose K loop is split across CTAs is completed by the last
// contributor from at most two partial slots per CTA (deterministic order).
// The tile is 128 weight rows (MMA M, TMEM lanes) x BN activation rows (MMA
// N); a packed step is 8 quant blocks (256 K). Warp roles (16 warps; every
// role that blocks on an mbarrier has a warp of its own, since a lane
// suspended in try_wait holds up the diverged lanes of its warp):
//   warp 0         TMA: packed quant rows (128-byte swizzle), PS stages;
//   warp 1         TMEM allocation, single-thread MMA issue into the slot ring;
//   warp 2         TMA: fp16 block scales (+ Q4_1 mins) of each step, SS stages;
//   warp 3         TMA: fp16 activation hi/lo tiles, 64 K per MMA stage;
//   warps 4..11    decoders: swizzled packed bytes -> exact fp16 codes in the
//                  K-major 128-byte-swizzle layout of the A stage;
//   warps 12..15   drainers: NB slots per batch, TMEM -> registers, one
//                  tcgen05.wait::ld, free the slots, scale in fp32; flush per
//                  tile (x row scale 2^-e, bias, store or partial + ticket).
// Every wait is bounded in time; a timeout raises the CTA abort flag and the
// host-visible error flag, and all roles leave their loops (the drainers keep
// their loop shape so that their named barriers still match).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec_api.h"

namespace mq {

constexpr int kDecRows = 128;
constexpr int kDecWarps = 16;
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecBlocksPerStep = 8;  // quant blocks per packed step (Q4_x: 128 B per row, Q8_0: 256 B)
constexpr uint64_t kDecWaitNs = 1000000000ull;
constexpr uint64_t kDecDrainNs = 20000000ull;

struct DecArgs {
  WeightView w;
  int m;                 // activation rows (<= NC)
  const float *xinv;     // [BN] 2^-e per activation row
  const float *xsum;     // [kpad / 32][BN] scaled block sums of x (Q4_1)
  const float *bias;
  float *y;
  int64_t ldy;
  float *partial;        // [gridDim.x][2][128][BN]: head / tail partial tile of every CTA
  int *tickets;          // [tiles], zero between launches
  int steps;             // packed steps per tile (the K loop)
  int tiles;
  int *err;
  int nan_on_abort;      // on a timed-out wait, write NaN outputs instead of skipping them
};

template <int QT, int BN>
struct DecCfg {
  static constexpr int kPkBytes = kDecRows * (QT == MQ_Q8_0 ? 256 : 128);  // packed step
  static constexpr int kScBytes = kDecRows * 16 * (QT == MQ_Q4_1 ? 2 : 1);  // scales (+ mins) of a step
  static constexpr int PS = QT == MQ_Q8_0 ? 3 : 4;  // packed stages
  static constexpr int SS = 12;                     // scale stages
  static constexpr int AS = 4;                      // A / activation stages (64 K each)
  static constexpr int R = 512 / BN;                // TMEM slots (one per block in flight)
  static constexpr int NB = BN == 16 ? 4 : 1;       // blocks per drain batch
  static constexpr int kA = kDecRows * 64 * 2;      // fp16 codes, 64 K
  static constexpr int kX = BN * 64 * 2;            // fp16 activation tile (hi or lo)
  static constexpr int kPkOff = 0;
  static constexpr int kScOff = kPkOff + PS * kPkBytes;
  static constexpr int kAOff = kScOff + SS * kScBytes;
  static constexpr int kXOff = kAOff + AS * kA;
  static constexpr int kBarOff = kXOff + AS * 2 * kX;
  static constexpr int kNumBars = 2 * PS + 2 * SS + 3 * AS + 2 * R;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

// Stream-K ownership: CTA c of G walks global steps [c*T/G, (c+1)*T/G) of the
// tile-major step space (T = tiles * steps).
__device__ __forceinline__ int dec_first_step(int c, int G, int T) { return (int)((int64_t)c * T / G); }
__device__ __forceinline__ int dec_cta_of_step(int g, int G, int T) {
  return (int)(((int64_t)(g + 1) * G - 1) / T);
}

// Two exact fp16 codes (q - zp) from the nibbles at bits sh..sh+3 and 16+sh..19+sh.
template <int QT>
__device__ __forceinline__ uint32_t dcode_q4(uint32_t w, int sh) {
  const uint32_t v = ((w >> sh) & 0x000F000Fu) | 0x64006400u;
  const uint32_t z = QT == MQ_Q4_0 ? 0x64086408u : 0x64006400u;  // 1032 / 1024
  const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&v), *reinterpret_cast<const __half2 *>(&z));
  return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t dcode_q8(uint32_t u, unsigned sel) {  // u already ^ 0x80 per byte
  const uint32_t v = __byte_perm(u, 0x64646464u, sel);
  const uint32_t z = 0x64806480u;  // 1152
  const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&v), *reinterpret_cast<const __half2 *>(&z));
  return *reinterpret_cast<const uint32_t *>(&r);
}

// Instruction descriptor, kind::f16: F16 x F16 -> F32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  sm100::umma_bf16(tmem_d, adesc, bdesc, idesc, accumulate);  // same instruction; formats live in idesc
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[NC]) {
  if constexpr (NC == 4) tmem_ld_x4(taddr, r);
  else if constexpr (NC == 16) tmem_ld_x16(taddr, r);
  else sm100::tmem_ld_32x32b_x32(taddr, r);
}

template <int QT, int BN, int NC>
__global__ void __launch_bounds__(kDecThreads, 1)
    tcdec_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_d,
                 const __grid_constant__ CUtensorMap tm_m, const __grid_constant__ CUtensorMap tm_xh,
                 const __grid_constant__ CUtensorMap tm_xl, const DecArgs a) {
  using L = DecCfg<QT, BN>;
  constexpr int PS = L::PS, SS = L::SS, AS = L::AS, R = L::R, NB = L::NB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = pk_full + PS;
  uint64_t *sc_full = pk_empty + PS, *sc_empty = sc_full + SS;
  uint64_t *a_full = sc_empty + SS, *x_full = a_full + AS, *a_empty = x_full + AS;
  uint64_t *s_full = a_empty + AS, *s_empty = s_full + R;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.steps, T = a.tiles * a.steps, G = gridDim.x, cta = blockIdx.x;
  const int g0 = dec_first_step(cta, G, T), g1 = dec_first_step(cta + 1, G, T);
  const int nsteps = g1 - g0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&pk_full[i], 1), sm100::mbar_init(&pk_empty[i], 256);
    for (int i = 0; i < SS; ++i) sm100::mbar_init(&sc_full[i], 1), sm100::mbar_init(&sc_empty[i], 128);
    for (int i = 0; i < AS; ++i) {
      sm100::mbar_init(&a_full[i], 256);
      sm100::mbar_init(&x_full[i], 1);
      sm100::mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < R; ++i) sm100::mbar_init(&s_full[i], 1), sm100::mbar_init(&s_empty[i], 128);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------- TMA: packed quant rows
      sm100::prefetch_tmap(&tm_q);
      int issued = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int i = ls % PS;
        if (!sm100::mbar_wait(&pk_empty[i], ((uint32_t)(ls / PS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) break;
        const int g = g0 + ls, t = g / S, k = g % S;
        uint8_t *dst = smem + L::kPkOff + i * L::kPkBytes;
        sm100::mbar_arrive_expect_tx(&pk_full[i], L::kPkBytes);
        if constexpr (QT == MQ_Q8_0) {
          sm100::tma_load_2d(dst, &tm_q, k * 256, t * kDecRows, &pk_full[i]);
          sm100::tma_load_2d(dst + kDecRows * 128, &tm_q, k * 256 + 128, t * kDecRows, &pk_full[i]);
        } else {
          sm100::tma_load_2d(dst, &tm_q, k * 128, t * kDecRows, &pk_full[i]);
        }
        issued = ls + 1;
      }
      for (int p = issued - PS < 0 ? 0 : issued - PS; p < issued; ++p)
        sm100::mbar_wait(&pk_full[p % PS], (uint32_t)(p / PS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 2) {
    if (lane == 0) {  // ------------------------------------- TMA: block scales (+ Q4_1 mins)
      sm100::prefetch_tmap(&tm_d);
      if (QT == MQ_Q4_1) sm100::prefetch_tmap(&tm_m);
      int issued = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int i = ls % SS;
        if (!sm100::mbar_wait(&sc_empty[i], ((uint32_t)(ls / SS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) break;
        const int g = g0 + ls, t = g / S, k = g % S;
        uint8_t *dst = smem + L::kScOff + i * L::kScBytes;
        sm100::mbar_arrive_expect_tx(&sc_full[i], L::kScBytes);
        sm100::tma_load_2d(dst, &tm_d, k * kDecBlocksPerStep, t * kDecRows, &sc_full[i]);
        if constexpr (QT == MQ_Q4_1)
          sm100::tma_load_2d(dst + kDecRows * 16, &tm_m, k * kDecBlocksPerStep, t * kDecRows, &sc_full[i]);
        issued = ls + 1;
      }
      for (int p = issued - SS < 0 ? 0 : issued - SS; p < issued; ++p)
        sm100::mbar_wait(&sc_full[p % SS], (uint32_t)(p / SS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 3) {
    if (lane == 0) {  // ------------------------------------- TMA: activation hi/lo tiles
      sm100::prefetch_tmap(&tm_xh);
      sm100::prefetch_tmap(&tm_xl);
      int issued = 0;
      const int nst = 4 * nsteps;
      for (int s = 0; s < nst; ++s) {
        const int i = s % AS;
        if (!sm100::mbar_wait(&a_empty[i], ((uint32_t)(s / AS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) break;
        const int k = (g0 + s / 4) % S;
        const int kx = (k * kDecBlocksPerStep + 2 * (s % 4)) * 32;
        uint8_t *dst = smem + L::kXOff + i * 2 * L::kX;
        sm100::mbar_arrive_expect_tx(&x_full[i], 2 * L::kX);
        sm100::tma_load_2d(dst, &tm_xh, kx, 0, &x_full[i]);
        sm100::tma_load_2d(dst + L::kX, &tm_xl, kx, 0, &x_full[i]);
        issued = s + 1;
      }
      for (int s = issued - AS < 0 ? 0 : issued - AS; s < issued; ++s)
        sm100::mbar_wait(&x_full[s % AS], (uint32_t)(s / AS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------- MMA issue into the TMEM slot ring
      constexpr uint32_t idesc = idesc_f16_f32(kDecRows, BN);
      const int nst = 4 * nsteps;
      for (int s = 0; s < nst; ++s) {
        const int i = s % AS;
        const uint32_t ph = (uint32_t)(s / AS) & 1u;
        if (!sm100::mbar_wait(&a_full[i], ph, a.err, abort, kDecWaitNs)) break;
        if (!sm100::mbar_wait(&x_full[i], ph, a.err, abort, kDecWaitNs)) break;
        sm100::tc_fence_after();
        const uint32_t abase = sm100::smem_u32(smem + L::kAOff + i * L::kA);
        const uint32_t xbase = sm100::smem_u32(smem + L::kXOff + i * 2 * L::kX);
        const uint64_t da = sm100::umma_desc_sw128(abase);
        const uint64_t dh = sm100::umma_desc_sw128(xbase), dl = sm100::umma_desc_sw128(xbase + L::kX);
        bool ok = true;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          const int b = 2 * s + blk;
          const int slot = b % R;
          if (!sm100::mbar_wait(&s_empty[slot], ((uint32_t)(b / R) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(slot * BN);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const uint64_t off = (uint64_t)(2 * (2 * blk + k));  // 32-byte K steps, in 16-byte units
            umma_f16(d, da + off, dh + off, idesc, k);
            umma_f16(d, da + off, dl + off, idesc, 1u);
          }
          sm100::umma_commit(&s_full[slot]);
        }
        sm100::umma_commit(&a_empty[i]);
        if (!ok) break;
      }
    }
  } else if (warp < 12) {  // -------------------------------- decoders: packed bytes -> exact fp16 codes
    const int t256 = threadIdx.x - 128;
    const int r = t256 & 127;  // tile row
    const int h = t256 >> 7;   // group h of the step: MMA stages 2h, 2h+1
    const int sw = r & 7;
    for (int ls = 0; ls < nsteps; ++ls) {
      const int pi = ls % PS;
      if (!sm100::mbar_wait(&pk_full[pi], (uint32_t)(ls / PS) & 1u, a.err, abort, kDecWaitNs)) break;
      bool ok = true;
      for (int q = 0; q < 4; ++q) {
        const int s = 4 * ls + q;
        const int i = s % AS;
        if (!sm100::mbar_wait(&a_empty[i], ((uint32_t)(s / AS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) {
          ok = false;
          break;
        }
        if ((q >> 1) == h) {
          const int sub = q & 1;  // blocks 2*sub, 2*sub+1 of group h
          uint8_t *arow = smem + L::kAOff + i * L::kA + r * 128;
          if constexpr (QT == MQ_Q8_0) {
            const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + h * (kDecRows * 128) + r * 128;
            uint32_t *o = reinterpret_cast<uint32_t *>(arow);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint4 c = *reinterpret_cast<const uint4 *>(prow + (((2 * t + sub) ^ sw) << 4));
              const uint32_t u[2][2] = {{c.x ^ 0x80808080u, c.y ^ 0x80808080u}, {c.z ^ 0x80808080u, c.w ^ 0x80808080u}};
#pragma unroll
              for (int bl = 0; bl < 2; ++bl) {
                o[(((4 * bl + 0) ^ sw) << 2) + t] = dcode_q8(u[bl][0], 0x4140u);
                o[(((4 * bl + 1) ^ sw) << 2) + t] = dcode_q8(u[bl][0], 0x4342u);
                o[(((4 * bl + 2) ^ sw) << 2) + t] = dcode_q8(u[bl][1], 0x4140u);
                o[(((4 * bl + 3) ^ sw) << 2) + t] = dcode_q8(u[bl][1], 0x4342u);
              }
            }
          } else {
            const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + r * 128;
            uint4 c[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) c[t] = *reinterpret_cast<const uint4 *>(prow + (((4 * h + t) ^ sw) << 4));
#pragma unroll
            for (int bl = 0; bl < 2; ++bl) {
              const int j = 2 * sub + bl;
              uint4 oc[4];
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const uint32_t wd = j == 0 ? c[t].x : j == 1 ? c[t].y : j == 2 ? c[t].z : c[t].w;
                const uint32_t v0 = dcode_q4<QT>(wd, 0), v1 = dcode_q4<QT>(wd, 8);
                const uint32_t v2 = dcode_q4<QT>(wd, 4), v3 = dcode_q4<QT>(wd, 12);
                (t == 0 ? oc[0].x : t == 1 ? oc[0].y : t == 2 ? oc[0].z : oc[0].w) = v0;
                (t == 0 ? oc[1].x : t == 1 ? oc[1].y : t == 2 ? oc[1].z : oc[1].w) = v1;
                (t == 0 ? oc[2].x : t == 1 ? oc[2].y : t == 2 ? oc[2].z : oc[2].w) = v2;
                (t == 0 ? oc[3].x : t == 1 ? oc[3].y : t == 2 ? oc[3].z : oc[3].w) = v3;
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4 *>(arow + (((4 * bl + u) ^ sw) << 4)) = oc[u];
            }
          }
          sm100::fence_proxy_async_smem();
        }
        sm100::mbar_arrive(&a_full[i]);
      }
      if (!ok) break;
      sm100::mbar_arrive(&pk_empty[pi]);
    }
  } else {  // ------------------------------------------------ drainers (TMEM lane = tile row)
    const int r = 32 * (warp & 3) + lane;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    float acc[NC];
    int cur = -1;
    // Completes the tile's output: directly when this CTA owns the whole K loop
    // of the tile, else through the head/tail partial slots and the tile's
    // ticket (the last contributor sums the slots in CTA order).
    auto flush = [&](int tile) {
      const bool aborted = *abort;
      if (aborted && a.nan_on_abort) {
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[c] = __int_as_float(0x7fc00000);
      }
      const bool write = !aborted || a.nan_on_abort;
      const int n = tile * kDecRows + r;
      const bool row_ok = n < a.w.rows;
      const int tg0 = tile * S, tg1 = tg0 + S;
      if (tg0 >= g0 && tg1 <= g1) {
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < NC; ++c)
            if (c < a.m) a.y[(int64_t)c * a.ldy + n] = acc[c] * a.xinv[c] + bias;
        }
        return;
      }
      const int kind = (tile == g0 / S) ? 0 : 1;
      float *slot = a.partial + (((int64_t)cta * 2 + kind) * kDecRows + r) * BN;
#pragma unroll
      for (int c = 0; c < NC; c += 4)
        *reinterpret_cast<float4 *>(slot + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int cf = dec_cta_of_step(tg0, G, T), cl = dec_cta_of_step(tg1 - 1, G, T);
      if (warp == 12 && lane == 0) s_last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        float tot[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) tot[c] = 0.0f;
        for (int cc = cf; cc <= cl; ++cc) {  // fixed CTA order: deterministic
          const int kk = (tile == dec_first_step(cc, G, T) / S) ? 0 : 1;
          const float *ps = a.partial + (((int64_t)cc * 2 + kk) * kDecRows + r) * BN;
#pragma unroll
          for (int c = 0; c < NC; c += 4) {
            const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(ps + c));
            tot[c] += v4.x, tot[c + 1] += v4.y, tot[c + 2] += v4.z, tot[c + 3] += v4.w;
          }
        }
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < NC; ++c)
            if (c < a.m) a.y[(int64_t)c * a.ldy + n] = tot[c] * a.xinv[c] + bias;
        }
        if (warp == 12 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      // the next tile's slot may reuse this CTA's slot only after s_last is read
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    for (int ls = 0; ls < nsteps; ++ls) {
      const int g = g0 + ls, tile = g / S, kstep = g % S;
      if (tile != cur) {
        if (cur >= 0) flush(cur);
        cur = tile;
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
      }
      const int si = ls % SS;
      // Failed waits do not leave the loop: every drainer must run the same
      // sequence of flushes (they synchronise on a named barrier).
      bool ok = sm100::mbar_wait(&sc_full[si], (uint32_t)(ls / SS) & 1u, a.err, abort, kDecWaitNs);
      const uint8_t *sc = smem + L::kScOff + si * L::kScBytes;
      const uint4 dq = *reinterpret_cast<const uint4 *>(sc + r * 16);
      uint4 mq = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (QT == MQ_Q4_1) mq = *reinterpret_cast<const uint4 *>(sc + kDecRows * 16 + r * 16);
#pragma unroll
      for (int bb = 0; bb < kDecBlocksPerStep; bb += NB) {
        int slots[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const int b = kDecBlocksPerStep * ls + bb + j;
          slots[j] = b % R;
          ok = sm100::mbar_wait(&s_full[slots[j]], (uint32_t)(b / R) & 1u, a.err, abort, kDecWaitNs) && ok;
        }
        ok = __all_sync(0xffffffffu, ok);
        uint32_t v[NB][NC];
        if (ok) {
          sm100::tc_fence_after();
#pragma unroll
          for (int j = 0; j < NB; ++j) tmem_ld_cols<NC>(tmem + lane_base + (uint32_t)(slots[j] * BN), v[j]);
          sm100::tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < NB; ++j)
#pragma unroll
            for (int c = 0; c < NC; ++c) v[j][c] = 0u;
        }
        sm100::tc_fence_before();
#pragma unroll
        for (int j = 0; j < NB; ++j) sm100::mbar_arrive(&s_empty[slots[j]]);
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const int jb = bb + j;
          const uint32_t dw = jb < 4 ? (jb < 2 ? dq.x : dq.y) : (jb < 6 ? dq.z : dq.w);
          const __half2 d2 = *reinterpret_cast<const __half2 *>(&dw);
          const float d = (jb & 1) ? __high2float(d2) : __low2float(d2);
#pragma unroll
          for (int c = 0; c < NC; c += 2) {
            const float2 r2 = __ffma2_rn(make_float2(d, d),
                                         make_float2(__uint_as_float(v[j][c]), __uint_as_float(v[j][c + 1])),
                                         make_float2(acc[c], acc[c + 1]));
            acc[c] = r2.x, acc[c + 1] = r2.y;
          }
          if constexpr (QT == MQ_Q4_1) {
            const uint32_t mw = jb < 4 ? (jb < 2 ? mq.x : mq.y) : (jb < 6 ? mq.z : mq.w);
            const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw);
            const float mm = (jb & 1) ? __high2float(m2) : __low2float(m2);
            const float4 *xs = reinterpret_cast<const float4 *>(a.xsum + (int64_t)(kstep * kDecBlocksPerStep + jb) * BN);
#pragma unroll
            for (int c = 0; c < NC; c += 4) {
              const float4 s4 = __ldg(xs + c / 4);
              acc[c] = fmaf(mm, s4.x, acc[c]);
              acc[c + 1] = fmaf(mm, s4.y, acc[c + 1]);
              acc[c + 2] = fmaf(mm, s4.z, acc[c + 2]);
              acc[c + 3] = fmaf(mm, s4.w, acc[c + 3]);
            }
          }
        }
      }
      sm100::mbar_arrive(&sc_empty[si]);
    }
    if (cur >= 0) flush(cur);
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// Activation split for the decode GEMM: one CTA per activation row (rows >= m
// become zeros). Row i is scaled by 2^e_i (largest magnitude in [2^13, 2^14)),
// split into fp16 hi + lo, K-major [BN][kpad] for TMA; block sums (Q4_1) and
// 2^-e_i are written alongside.
__global__ void dec_prep_kernel(const float *__restrict__ x, int64_t ldx, int m, int K, int kpad, int bn,
                                __half *__restrict__ xh, __half *__restrict__ xl, float *__restrict__ xsum,
                                float *__restrict__ xinv, int want_sums) {
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
      frexpf(v, &E);
      e = min(100, max(-100, 14 - E));
    }
    s_scale = ldexpf(1.0f, e);
    xinv[row] = ldexpf(1.0f, -e);
  }
  __syncthreads();
  const float sc = s_scale;
  __half2 *h2 = reinterpret_cast<__half2 *>(xh + (int64_t)row * kpad);
  __half2 *l2 = reinterpret_cast<__half2 *>(xl + (int64_t)row * kpad);
  for (int k = 2 * threadIdx.x; k < kpad; k += 2 * blockDim.x) {
    const float v0 = (live && k < K) ? xr[k] * sc : 0.0f, v1 = (live && k + 1 < K) ? xr[k + 1] * sc : 0.0f;
    const __half2 hh = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(hh);
    h2[k >> 1] = hh;
    l2[k >> 1] = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
  }
  if (want_sums) {
    const int nb = kpad >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += blockDim.x >> 5) {
      const int k = 32 * b + lane;
      float s = (live && k < K) ? xr[k] * sc : 0.0f;
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) xsum[(int64_t)b * bn + row] = s;
    }
  }
}

}  // namespace mq
