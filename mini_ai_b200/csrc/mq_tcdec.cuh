// tcgen05 decode GEMM for a few activation rows (2 <= M <= 32).
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
// CTA = one tile of 128 weight rows (MMA M, TMEM lanes) x BN activation rows
// (MMA N) over a K range (split-K over CTAs, deterministic fixup by the last
// CTA of a tile). Warp roles (14 warps):
//   warp 0       TMA: packed quant rows (128 B per row per packed step, 128-byte
//                swizzle) and the fp16 activation hi/lo tiles (64 K per MMA stage);
//   warp 1       TMEM allocation, single-thread MMA issue into the slot ring;
//   warps 2..9   decoders: swizzled packed bytes -> exact fp16 codes in the
//                K-major 128-byte-swizzle layout of the A stage;
//   warps 10..13 drainers: per block, TMEM slot -> registers, scale, free slot;
//                at the end the epilogue (x row scale 2^-e, bias, store / fixup).
// Every wait is bounded in time; a timeout raises the CTA abort flag and the
// host-visible error flag, and all roles leave their loops.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec_api.h"

namespace mq {

constexpr int kDecRows = 128;
constexpr int kDecWarps = 14;
constexpr int kDecThreads = kDecWarps * 32;
constexpr uint64_t kDecWaitNs = 1000000000ull;
constexpr uint64_t kDecDrainNs = 20000000ull;

struct DecArgs {
  WeightView w;
  int m;                 // activation rows (<= BN)
  const float *xinv;     // [BN] 2^-e per activation row
  const float *xsum;     // [nbp][BN] scaled block sums of x (Q4_1)
  const float *bias;
  float *y;
  int64_t ldy;
  float *partial;        // [ksplit][tiles * 128][BN] (ksplit > 1)
  int *counters;         // [tiles], zero between launches
  int ksplit;
  int steps_total;       // packed steps over the whole K
  int *err;
  int nan_on_abort;      // on a timed-out wait, write NaN outputs instead of skipping them
};

template <int QT> struct DecQ {
  static constexpr int kBlocksPerStep = QT == MQ_Q8_0 ? 4 : 8;  // 128 packed bytes per row per step
  static constexpr int kStagesPerStep = kBlocksPerStep / 2;       // MMA stages (64 K) per packed step
};

template <int QT, int BN, int PS, int AS>
struct DecSmem {
  static constexpr int kPk = kDecRows * 128;             // packed stage
  static constexpr int kA = kDecRows * 64 * 2;           // fp16 codes, 64 K
  static constexpr int kX = BN * 64 * 2;                 // fp16 activation tile (hi or lo)
  static constexpr int kPkOff = 0;
  static constexpr int kAOff = PS * kPk;
  static constexpr int kXOff = kAOff + AS * kA;
  static constexpr int kBarOff = kXOff + AS * 2 * kX;
  static constexpr int kSlots = (BN == 16 ? 32 : 16);
  static constexpr int kNumBars = 2 * PS + 3 * AS + 2 * kSlots;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

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

template <int QT, int BN, int PS, int AS>
__global__ void __launch_bounds__(kDecThreads, 1)
    tcdec_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_xh,
                 const __grid_constant__ CUtensorMap tm_xl, const DecArgs a) {
  using L = DecSmem<QT, BN, PS, AS>;
  using Q = DecQ<QT>;
  constexpr int R = L::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = bars + PS;
  uint64_t *a_full = bars + 2 * PS, *x_full = a_full + AS, *a_empty = x_full + AS;
  uint64_t *s_full = a_empty + AS, *s_empty = s_full + R;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kDecRows;
  // This CTA's packed steps [p0, p1) of the K loop.
  const int p0 = (int)((int64_t)a.steps_total * split / a.ksplit);
  const int p1 = (int)((int64_t)a.steps_total * (split + 1) / a.ksplit);
  const int nsteps = p1 - p0;
  const int nstages = nsteps * Q::kStagesPerStep;  // MMA stages of 64 K
  const int nblocks = 2 * nstages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) {
      sm100::mbar_init(&pk_full[i], 1);
      sm100::mbar_init(&pk_empty[i], 256);
    }
    for (int i = 0; i < AS; ++i) {
      sm100::mbar_init(&a_full[i], 256);
      sm100::mbar_init(&x_full[i], 1);
      sm100::mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < R; ++i) {
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_empty[i], 128);
    }
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    sm100::prefetch_tmap(&tm_q);
    sm100::prefetch_tmap(&tm_xh);
    sm100::prefetch_tmap(&tm_xl);
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
    if (lane == 0) {  // ---------------------------------------------- TMA
      // Interleave packed steps (weights) and MMA stages (activations) so the
      // weight stream runs PS steps ahead of the consumer.
      int issued_pk = 0, issued_x = 0;
      bool ok = true;
      for (int s = 0; ok && s < nstages; ++s) {
        while (ok && issued_pk < nsteps && issued_pk * Q::kStagesPerStep <= s + (PS - 1) * Q::kStagesPerStep) {
          const int i = issued_pk % PS;
          const uint32_t ph = (uint32_t)(issued_pk / PS) & 1u;
          if (!sm100::mbar_wait(&pk_empty[i], ph ^ 1u, a.err, abort, kDecWaitNs)) { ok = false; break; }
          sm100::mbar_arrive_expect_tx(&pk_full[i], L::kPk);
          sm100::tma_load_2d(smem + L::kPkOff + i * L::kPk, &tm_q, (p0 + issued_pk) * 128, n0, &pk_full[i]);
          ++issued_pk;
        }
        if (!ok) break;
        const int i = s % AS;
        const uint32_t ph = (uint32_t)(s / AS) & 1u;
        if (!sm100::mbar_wait(&a_empty[i], ph ^ 1u, a.err, abort, kDecWaitNs)) break;
        const int kx = (p0 * Q::kBlocksPerStep + 2 * s) * 32;  // activation column of this stage
        sm100::mbar_arrive_expect_tx(&x_full[i], 2 * L::kX);
        sm100::tma_load_2d(smem + L::kXOff + i * 2 * L::kX, &tm_xh, kx, 0, &x_full[i]);
        sm100::tma_load_2d(smem + L::kXOff + i * 2 * L::kX + L::kX, &tm_xl, kx, 0, &x_full[i]);
        issued_x = s + 1;
      }
      // Let copies already in flight land before the CTA can exit.
      for (int p = issued_pk - PS < 0 ? 0 : issued_pk - PS; p < issued_pk; ++p)
        sm100::mbar_wait(&pk_full[p % PS], (uint32_t)(p / PS) & 1u, nullptr, nullptr, kDecDrainNs);
      for (int s = issued_x - AS < 0 ? 0 : issued_x - AS; s < issued_x; ++s)
        sm100::mbar_wait(&x_full[s % AS], (uint32_t)(s / AS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------- MMA
      constexpr uint32_t idesc = idesc_f16_f32(kDecRows, BN);
      for (int s = 0; s < nstages; ++s) {
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
  } else if (warp < 10) {  // ---------------------------------------------- decoders
    const int t256 = threadIdx.x - 64;
    const int r = t256 & 127;   // tile row
    const int h = t256 >> 7;    // which half of the packed step this thread decodes
    for (int s = 0; s < nstages; ++s) {
      const int p = s / Q::kStagesPerStep, q = s % Q::kStagesPerStep;
      // Q4_x: thread half h decodes group h (MMA stages 2h, 2h+1 of the step);
      // Q8_0: thread half h decodes MMA stage 2*(q/2) + h... one stage each: stage q == h + 2*(q>>1).
      const bool mine = QT == MQ_Q8_0 ? ((q & 1) == h) : ((q >> 1) == h);
      const int pi = p % PS;
      if (q == 0 && !sm100::mbar_wait(&pk_full[pi], (uint32_t)(p / PS) & 1u, a.err, abort, kDecWaitNs)) break;
      const int i = s % AS;
      const uint32_t ph = (uint32_t)(s / AS) & 1u;
      if (!sm100::mbar_wait(&a_empty[i], ph ^ 1u, a.err, abort, kDecWaitNs)) break;
      if (mine) {
        const uint8_t *prow = smem + L::kPkOff + pi * L::kPk + r * 128;
        uint8_t *arow = smem + L::kAOff + i * L::kA + r * 128;
        const int sw = r & 7;
        if constexpr (QT == MQ_Q8_0) {
          // stage q covers blocks 2(q&1)... within the group: blocks jj = 2*(q&1) + {0,1}
          const int jb = 2 * (q & 1);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            // quad t: 32 bytes at 32t; blocks jb, jb+1 -> 16 bytes at 32t + 8*jb = chunk 2t + (jb >> 1)
            const uint4 c = *reinterpret_cast<const uint4 *>(prow + (((2 * t + (jb >> 1)) ^ sw) << 4));
            const uint32_t u[2][2] = {{c.x ^ 0x80808080u, c.y ^ 0x80808080u}, {c.z ^ 0x80808080u, c.w ^ 0x80808080u}};
#pragma unroll
            for (int bl = 0; bl < 2; ++bl) {
              // element pair (2t, 2t+1) of chunks u = 0..3 of block bl: u0 bytes 0,1 | u0 2,3 | u1 0,1 | u1 2,3
              const uint32_t v0 = dcode_q8(u[bl][0], 0x4140u), v1 = dcode_q8(u[bl][0], 0x4342u);
              const uint32_t v2 = dcode_q8(u[bl][1], 0x4140u), v3 = dcode_q8(u[bl][1], 0x4342u);
              // write word t of output chunks 4*bl + {0,1,2,3}
              uint32_t *o = reinterpret_cast<uint32_t *>(arow);
              o[(((4 * bl + 0) ^ sw) << 2) + t] = v0;
              o[(((4 * bl + 1) ^ sw) << 2) + t] = v1;
              o[(((4 * bl + 2) ^ sw) << 2) + t] = v2;
              o[(((4 * bl + 3) ^ sw) << 2) + t] = v3;
            }
          }
        } else {
          // group h of the packed step: quad t chunk (4h + t) holds words for blocks j = 0..3
          uint4 c[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) c[t] = *reinterpret_cast<const uint4 *>(prow + (((4 * h + t) ^ sw) << 4));
          // this MMA stage holds blocks 2(q&1), 2(q&1)+1 of the group
          const int jb = 2 * (q & 1);
#pragma unroll
          for (int bl = 0; bl < 2; ++bl) {
            uint4 oc[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint32_t wd = (jb + bl) == 0 ? c[t].x : (jb + bl) == 1 ? c[t].y : (jb + bl) == 2 ? c[t].z : c[t].w;
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
      if (q == Q::kStagesPerStep - 1) sm100::mbar_arrive(&pk_empty[pi]);
    }
  } else {  // -------------------------------------------------------------- drainers
    const int r = 32 * (warp & 3) + lane;  // TMEM lane = tile row
    const int n = n0 + r;
    const bool row_ok = n < a.w.rows;
    const int nrow = row_ok ? n : 0;
    const __half *drow = a.w.d + (int64_t)nrow * a.w.ld_s;
    const __half *mrow = QT == MQ_Q4_1 ? a.w.mn + (int64_t)nrow * a.w.ld_s : nullptr;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int b0 = p0 * Q::kBlocksPerStep;  // first block of this CTA
    float acc[BN];
#pragma unroll
    for (int c = 0; c < BN; ++c) acc[c] = 0.0f;
    // scales for 4 blocks at a time, one group ahead
    uint2 dq = *reinterpret_cast<const uint2 *>(drow + b0), dqn = dq;
    uint2 mq = QT == MQ_Q4_1 ? *reinterpret_cast<const uint2 *>(mrow + b0) : make_uint2(0u, 0u), mqn = mq;
    for (int bb = 0; bb < nblocks; ++bb) {
      if ((bb & 3) == 0) {
        dq = dqn;
        mq = mqn;
        if (bb + 4 < nblocks) {
          dqn = *reinterpret_cast<const uint2 *>(drow + b0 + bb + 4);
          if constexpr (QT == MQ_Q4_1) mqn = *reinterpret_cast<const uint2 *>(mrow + b0 + bb + 4);
        }
      }
      const int slot = bb % R;
      if (!sm100::mbar_wait(&s_full[slot], (uint32_t)(bb / R) & 1u, a.err, abort, kDecWaitNs)) break;
      sm100::tc_fence_after();
      uint32_t v[BN];
      if constexpr (BN == 16) {
        uint32_t (&vv)[16] = *reinterpret_cast<uint32_t(*)[16]>(v);
        tmem_ld_x16(tmem + lane_base + (uint32_t)(slot * BN), vv);
      } else {
        uint32_t (&vv)[32] = *reinterpret_cast<uint32_t(*)[32]>(v);
        sm100::tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(slot * BN), vv);
      }
      sm100::tmem_ld_wait();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&s_empty[slot]);
      const uint32_t dw = (bb & 2) ? dq.y : dq.x;
      const __half2 d2 = *reinterpret_cast<const __half2 *>(&dw);
      const float d = (bb & 1) ? __high2float(d2) : __low2float(d2);
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float2 r2 = __ffma2_rn(make_float2(d, d), make_float2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])),
                                     make_float2(acc[c], acc[c + 1]));
        acc[c] = r2.x, acc[c + 1] = r2.y;
      }
      if constexpr (QT == MQ_Q4_1) {
        const uint32_t mw = (bb & 2) ? mq.y : mq.x;
        const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw);
        const float mm = (bb & 1) ? __high2float(m2) : __low2float(m2);
        const float4 *xs = reinterpret_cast<const float4 *>(a.xsum + (int64_t)(b0 + bb) * BN);
#pragma unroll
        for (int c = 0; c < BN; c += 4) {
          const float4 s4 = __ldg(xs + c / 4);
          acc[c] = fmaf(mm, s4.x, acc[c]);
          acc[c + 1] = fmaf(mm, s4.y, acc[c + 1]);
          acc[c + 2] = fmaf(mm, s4.z, acc[c + 2]);
          acc[c + 3] = fmaf(mm, s4.w, acc[c + 3]);
        }
      }
    }
    // ------------------------------------------------ epilogue
    const bool aborted = *abort;
    if (aborted && a.nan_on_abort) {
#pragma unroll
      for (int c = 0; c < BN; ++c) acc[c] = __int_as_float(0x7fc00000);
    }
    const bool ok = !aborted || a.nan_on_abort;
    if (a.ksplit == 1) {
      if (ok && row_ok) {
        const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c < a.m) a.y[(int64_t)c * a.ldy + n] = acc[c] * a.xinv[c] + bias;
      }
    } else {
      float *part = a.partial + ((int64_t)split * gridDim.x * kDecRows + (int64_t)tile * kDecRows + r) * BN;
#pragma unroll
      for (int c = 0; c < BN; c += 4)
        *reinterpret_cast<float4 *>(part + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      __threadfence();
      // named barrier over the 4 drainer warps, then one thread takes a ticket
      asm volatile("bar.sync 1, 128;" ::: "memory");
      __shared__ int s_last;
      if (warp == 10 && lane == 0) s_last = (atomicAdd(&a.counters[tile], 1) == a.ksplit - 1);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        float tot[BN];
#pragma unroll
        for (int c = 0; c < BN; ++c) tot[c] = 0.0f;
        for (int sp = 0; sp < a.ksplit; ++sp) {  // fixed split order: deterministic
          const float *pp = a.partial + ((int64_t)sp * gridDim.x * kDecRows + (int64_t)tile * kDecRows + r) * BN;
#pragma unroll
          for (int c = 0; c < BN; c += 4) {
            const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(pp + c));
            tot[c] += v4.x, tot[c + 1] += v4.y, tot[c + 2] += v4.z, tot[c + 3] += v4.w;
          }
        }
        if (ok && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c < a.m) a.y[(int64_t)c * a.ldy + n] = tot[c] * a.xinv[c] + bias;
        }
        if (warp == 10 && lane == 0) a.counters[tile] = 0;  // ready for the next launch
      }
    }
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
