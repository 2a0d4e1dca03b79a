// SIMT decode GEMV for one or two activation rows: the HBM-streaming path.
//
// One activation row makes decode a pure weight stream: every packed byte is
// read once and used for one multiply-add per weight. Here the weights stay
// in their packed integer form all the way into the dot product:
//
//   y[i, n] = sum_b d[n,b] * 2^-e[i,b] * sum_k q[n,b,k] * X[i,b,k]  (Q8_0)
//           = sum_b d[n,b] * 2^-e[i,b] * (sum_k q X - 8 sum_k X)     (Q4_0)
//           = sum_b (d[n,b] * 2^-e[i,b] * sum_k q X + m[n,b] * sum_k x) (Q4_1)
//
// Exactness scheme. Every 32-element block of an activation row is scaled by
// a power of two 2^e so that its largest magnitude lies in [2^21, 2^22) and
// rounded to integers X (the rounding error is below 2^-22 of the block's
// largest |x|, one block at a time, so an outlier only coarsens its own 32
// elements). X is split into its bytes, X = b0 + 2^8 b1 + 2^16 b2 (b0, b1
// unsigned, b2 signed: |X| <= 2^22), and `dp4a` (four 8-bit products and a
// 32-bit add per instruction, each operand signed or unsigned) forms the
// exact integer sums sum_k q * b. For Q4_x the limb sums combine in
// int32 (|sum q X| < 2^31, so the wrapping combination is exact), for Q8_0 in
// fp32; the fp16 block scale and 2^-e are then applied once per block in fp32,
// so the result equals the reference's fp32 dot up to accumulation-order
// rounding. Q4_x nibbles are used in place: the low nibbles are masked out
// of the packed word (values q), the high ones too (values 16 q, divided out
// of their sum exactly).
//
// Data flow per (128-row tile, 8-block step) of the tile-major device layout:
//   warp 0 (one thread): one bulk copy of the weight chunk (codes, fp16
//     scales, Q4_1 mins) into a ring of PS chunks;
//   warp 1: the step's activation limbs and per-block header (2^-e, sum X,
//     sum x) into a ring of LS slots, in the word order of the weight
//     layout (one 32-bit limb word per four K positions of a weight word):
//     lane l loads exactly the eight elements behind its block's two word
//     slots 2t, 2t+1 (block l / 4, t = l % 4), so a limb word is three byte
//     permutes of its four X values;
//   warps 2..9: eight consumer warps; warp w handles 32 tile rows and one of
//     the step's two quads (4 blocks), so a row's step is split over two
//     threads whose sums meet in shared memory at the end of the tile. Their
//     limb loads are warp-wide broadcasts; their weight loads follow the
//     pre-applied 128-byte swizzle and are bank-conflict free.
//
// Residency. The kernel holds at most 113 KB of shared memory and no tensor
// memory, so two CTAs fit on an SM: launched with programmatic dependent
// launch, the next product's CTA starts while this one still computes and
// streams its own weights early (the weights never depend on the previous
// kernel); only its prep and consumer warps wait for the previous kernel
// (griddepcontrol.wait), because its activations may be that kernel's output.
//
// Persistent stream-K over the tile-major step space, as the other decode
// kernels (dec_first_step): a tile whose K loop is split across CTAs is
// completed by the last contributor from at most two partial slots per CTA,
// in CTA order (deterministic).
//
// Every wait is bounded in time; a timeout raises the CTA abort flag and the
// host-visible error flag and every role leaves its work (consumers keep
// their loop shape so that their named barriers still match); copies in
// flight are waited for (bounded) before the CTA exits. The producer's first
// wait on a consumer release comes after the prep warp has passed the
// dependency wait (a `go` barrier), so a long-running previous kernel does
// not count against the limit.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
#pragma once

#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec.cuh"

namespace mq {

constexpr int kGvRows = 128;
constexpr int kGvGroups = 2;                        // consumer groups, taking the steps in turn
constexpr int kGvGroupWarps = 8;                    // consumer warps per group (128 rows x 2 quads)
constexpr int kGvConsumers = kGvGroups * kGvGroupWarps;
constexpr int kGvWarps = 2 + kGvConsumers;
constexpr int kGvThreads = 32 * kGvWarps;
constexpr int kGvMinBlocks = kGvGroups == 1 ? 2 : 1;
constexpr uint64_t kGvWaitNs = 1000000000ull;       // 1 s per wait once the dependency is resolved
constexpr uint64_t kGvDepNs = 120000000000ull;      // 120 s: the previous kernel's run time
constexpr uint64_t kGvDrainNs = 20000000ull;        // copies already in flight
// One group: two CTAs per SM (228 KB, 1 KB reserved per CTA); two groups: one CTA per SM.
constexpr int kGvSmemCap = kGvGroups == 1 ? 113 * 1024 : 220 * 1024;

struct GvArgs {
  WeightView w;
  int m;                 // activation rows (<= MC)
  const float *x;        // [m][ldx]
  int64_t ldx;
  const float *bias;
  float *y;
  int64_t ldy;
  float *partial;        // [gridDim.x][2][128][MC]: head / tail partial tile of every CTA
  int *tickets;          // [tiles], zero between launches
  int steps;             // packed steps per tile
  int tiles;
  int *err;
  int nan_on_abort;
  const float *gate = nullptr;   // fused gate/up product: y = silu(gate) * (product + bias)
  const float *resid = nullptr;  // residual add: y = resid + (product + bias); may be y
};

template <int QT, int MC>
struct GvCfg {
  static constexpr int kChunk = (int)step_chunk_bytes(QT);
  static constexpr int kPk = step_pk_bytes(QT);
  static constexpr int kLimbRow = 8 * 8 * 3 * 4;        // [8 blocks][8 word slots][3 limbs] u32
  static constexpr int kHdrRow = 8 * 16;                // [8 blocks] {sum X, 2^-e, sum x, 0}
  static constexpr int kLimbSlot = MC * (kLimbRow + kHdrRow);
  static constexpr int LS = 4;                          // limb slots
  static constexpr int kXch = 2 * (2 * kGvGroups) * kGvRows * MC * 4;   // tile sums of the other (group, quad) pairs
  static constexpr int kFixed = LS * kLimbSlot + kXch + 8 * (2 * 12 + 2 * LS + 1) + 64;
  // Weight chunks in flight: as many as fit beside the rest in the residency
  // budget (at most 12), a multiple of the groups so that every slot belongs
  // to one group.
  static constexpr int PS0 = (kGvSmemCap - kFixed) / kChunk;
  static constexpr int PS = (PS0 > 12 ? 12 : PS0) / kGvGroups * kGvGroups;
  static constexpr int kRingOff = 0;
  static constexpr int kLimbOff = kRingOff + PS * kChunk;
  static constexpr int kXchOff = kLimbOff + LS * kLimbSlot;     // [2 halves][group * 2 + quad][128][MC] float
  static constexpr int kBarOff = kXchOff + kXch;
  static constexpr int kNumBars = 2 * PS + 2 * LS + 1;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  static_assert(PS >= 2 && PS % kGvGroups == 0 && LS % kGvGroups == 0, "rings owned by one group a slot");
  static_assert(kBytes <= kGvSmemCap, "two CTAs per SM");
  static_assert(kChunk % 16 == 0 && kLimbSlot % 16 == 0 && kBarOff % 8 == 0, "alignment");
};

// d = a . b + c over four byte lanes: a unsigned, b signed.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// d = a . b + c over four byte lanes: both signed.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// d = a . b + c over four byte lanes: both unsigned (sums stay below 2^31 here).
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// d = a . b + c over four byte lanes: a signed, b unsigned.
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Byte l of each of four words, in order: one limb word.
__device__ __forceinline__ uint32_t gather_byte(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, int l) {
  const uint32_t sel = (uint32_t)l | ((uint32_t)(4 + l) << 4);
  return __byte_perm(__byte_perm(x0, x1, sel), __byte_perm(x2, x3, sel), 0x5410);
}

template <int QT, int MC, bool EPI>
__global__ void __launch_bounds__(kGvThreads, kGvMinBlocks) gemv_kernel(const GvArgs a) {
  using L = GvCfg<QT, MC>;
  constexpr int PS = L::PS, LS = L::LS;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full = bars, *empty = bars + PS, *lfull = bars + 2 * PS, *lempty = bars + 2 * PS + LS;
  uint64_t *go = bars + 2 * PS + 2 * LS;
  volatile int *abort = reinterpret_cast<volatile int *>(bars + L::kNumBars);
  volatile int *s_last = abort + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, GR = gridDim.x;
  const int S = a.steps, T = a.tiles * S;
  const int g0 = dec_first_step(cta, GR, T), g1 = dec_first_step(cta + 1, GR, T);
  const int nsteps = g1 - g0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&full[i], 1), sm100::mbar_init(&empty[i], kGvGroupWarps);
    for (int i = 0; i < LS; ++i) sm100::mbar_init(&lfull[i], 1), sm100::mbar_init(&lempty[i], kGvGroupWarps);
    sm100::mbar_init(go, 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) sm100::griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------------ weight chunks, one bulk copy a step
      int issued = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int i = ls % PS;
        if (ls == PS && !sm100::mbar_wait_sleep(go, 0u, a.err, abort, kGvDepNs)) break;
        if (ls >= PS && !sm100::mbar_wait(&empty[i], ((uint32_t)(ls / PS) & 1u) ^ 1u, a.err, abort, kGvWaitNs))
          break;
        sm100::mbar_arrive_expect_tx(&full[i], L::kChunk);
        const int g = g0 + ls;
        sm100::bulk_load(smem + L::kRingOff + i * L::kChunk, chunk_ptr(a.w, g / S, g % S), L::kChunk, &full[i]);
        issued = ls + 1;
      }
      // No copy may still be landing when the CTA exits.
      for (int p = issued - PS < 0 ? 0 : issued - PS; p < issued; ++p)
        sm100::mbar_wait(&full[p % PS], (uint32_t)(p / PS) & 1u, nullptr, nullptr, kGvDrainNs);
    }
  } else if (warp == 1) {  // -------------------------------------------- activation limbs, one step a slot
    sm100::griddep_wait();  // the activations may be the previous kernel's output
    if (lane == 0) sm100::mbar_arrive(go);
    // Lane l: block jb = l / 4 of the step, word slots 2t and 2t + 1 (t = l % 4),
    // i.e. the elements 2t + {0, 1, 8, 9, 16, 17, 24, 25} of the block, read as
    // four pairs. The activations sit in L2 (possibly on the other die, most
    // of a microsecond away), so the loads run PD steps ahead of the step
    // being built (a register ring).
    constexpr int PD = MC == 1 ? 4 : 2;
    const int jb = lane >> 2, t = lane & 3;
    const bool vec = ((reinterpret_cast<uintptr_t>(a.x) | (uintptr_t)(a.ldx * 4)) & 7) == 0;
    float nv[PD][MC][8];
    auto load = [&](float (&dst)[MC][8], int ls) {
      const int k0 = ((g0 + ls) % S) * 256 + 32 * jb + 2 * t;
#pragma unroll
      for (int c = 0; c < MC; ++c) {
        const float *xr = a.x + (int64_t)(c < a.m ? c : 0) * a.ldx + k0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // pair u: elements 8u, 8u + 1 (+ 2t)
          const int k = k0 + 8 * u;
          if (c < a.m && vec && k + 2 <= a.w.cols) {
            const float2 f = __ldg(reinterpret_cast<const float2 *>(xr + 8 * u));
            dst[c][2 * u] = f.x, dst[c][2 * u + 1] = f.y;
          } else {
            dst[c][2 * u] = (c < a.m && k < a.w.cols) ? __ldg(xr + 8 * u) : 0.0f;
            dst[c][2 * u + 1] = (c < a.m && k + 1 < a.w.cols) ? __ldg(xr + 8 * u + 1) : 0.0f;
          }
        }
      }
    };
#pragma unroll
    for (int d = 0; d < PD; ++d)
      if (d < nsteps) load(nv[d], d);
    // Builds step ls from its activations v; false once a wait has failed.
    auto build = [&](const float (&v)[MC][8], int ls) -> bool {
      const int j = ls % LS;
      bool ok = true;
      if (ls >= LS) ok = sm100::mbar_wait(&lempty[j], ((uint32_t)(ls / LS) & 1u) ^ 1u, a.err, abort, kGvWaitNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return false;
      uint8_t *slot = smem + L::kLimbOff + j * L::kLimbSlot;
#pragma unroll
      for (int c = 0; c < MC; ++c) {
        // Block scale: 2^e puts the block's largest |x| in [2^21, 2^22).
        float amax = 0.0f;
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          amax = fmaxf(amax, fabsf(v[c][i]));
          bad |= !isfinite(v[c][i]);
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        bad = ((__ballot_sync(0xffffffffu, bad) >> (lane & ~3)) & 0xFu) != 0u;  // any of the block's four lanes
        // Blocks whose largest |x| is below 2^-100 contribute below 2^-95 |w|
        // to any output and are taken as zero.
        const int ex = (int)((__float_as_uint(amax) >> 23) & 255u);
        const bool zero = bad || amax < 7.8886091e-31f;  // 2^-100
        const int e = zero ? 0 : 148 - ex;
        const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
        const float inv = bad ? __int_as_float(0x7fc00000) : __uint_as_float((uint32_t)(127 - e) << 23);
        uint32_t X[8];
        int sx = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int xi = zero ? 0 : __float2int_rn(v[c][i] * sc);
          X[i] = (uint32_t)xi;
          sx += xi;
        }
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);
        // X[] holds elements 2t + {0, 1, 8, 9, 16, 17, 24, 25}. Word slot 2t
        // takes the first four, 2t + 1 the last four, in the byte order of the
        // weight words: Q4_x {0, 8, 1, 9}, Q8_0 {0, 1, 8, 9}.
        uint32_t wd[6];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int l = 0; l < 3; ++l) {
            const uint32_t *q4 = X + 4 * hh;
            wd[3 * hh + l] = QT == MQ_Q8_0 ? gather_byte(q4[0], q4[1], q4[2], q4[3], l)
                                           : gather_byte(q4[0], q4[2], q4[1], q4[3], l);
          }
        uint2 *dst = reinterpret_cast<uint2 *>(slot + ((c * 8 + jb) * 8 + 2 * t) * 12);
        dst[0] = make_uint2(wd[0], wd[1]);
        dst[1] = make_uint2(wd[2], wd[3]);
        dst[2] = make_uint2(wd[4], wd[5]);
        if (t == 0) {
          const float sxf = (float)sx * inv;
          *reinterpret_cast<int4 *>(slot + MC * L::kLimbRow + (c * 8 + jb) * 16) =
              make_int4(sx, __float_as_int(inv), __float_as_int(sxf), 0);
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&lfull[j]);
      return true;
    };
    // Each ring slot is consumed in place and reloaded for the step PD ahead
    // (moving a register whose load is still in flight would wait for it).
    bool alive = true;
    for (int ls0 = 0; ls0 < nsteps && alive; ls0 += PD) {
#pragma unroll
      for (int d = 0; d < PD; ++d) {
        const int ls = ls0 + d;
        if (alive && ls < nsteps) {
          alive = build(nv[d], ls);
          if (ls + PD < nsteps) load(nv[d], ls + PD);
        }
      }
    }
  } else {  // ------------------------------------------------------------- consumers
    sm100::griddep_wait();  // outputs, partial slots and tickets may still be in use by the previous kernel
    const int cw = warp - 2, grp = cw / kGvGroupWarps, h = (cw % kGvGroupWarps) >> 2;
    const int r = 32 * (cw & 3) + lane;
    const bool owner = grp == 0 && h == 0;  // completes the tile: warps 2..5
    float acc[MC];
    float *xch = reinterpret_cast<float *>(smem + L::kXchOff);
    auto flush = [&](int tile) {
      const bool aborted = *abort;
      if (aborted && a.nan_on_abort) {
#pragma unroll
        for (int c = 0; c < MC; ++c) acc[c] = __int_as_float(0x7fc00000);
      }
      const bool write = !aborted || a.nan_on_abort;
      const int n = tile * kGvRows + r;
      const bool row_ok = n < a.w.rows;
      const int tg0 = tile * S, tg1 = tg0 + S;
      if (tg0 >= g0 && tg1 <= g1) {
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < MC; ++c)
            if (c < a.m)
              a.y[(int64_t)c * a.ldy + n] =
                  EPI ? epilogue_out(acc[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : acc[c] + bias;
        }
        return;
      }
      const int kind = (tile == g0 / S) ? 0 : 1;
      float *slot = a.partial + (((int64_t)cta * 2 + kind) * kGvRows + r) * MC;
#pragma unroll
      for (int c = 0; c < MC; ++c) slot[c] = acc[c];
      // Release: the barrier orders the 128 threads' slot writes before one
      // thread's device-scope fence and ticket; acquire mirrors it for the
      // last contributor (one fence per CTA instead of one per thread).
      asm volatile("bar.sync 2, 128;" ::: "memory");
      const int cf = dec_cta_of_step(tg0, GR, T), cl = dec_cta_of_step(tg1 - 1, GR, T);
      if (cw == 0 && lane == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
        if (last) __threadfence();
        *s_last = last;
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (*s_last) {
        float tot[MC];
#pragma unroll
        for (int c = 0; c < MC; ++c) tot[c] = 0.0f;
        for (int cc = cf; cc <= cl; ++cc) {  // fixed CTA order: deterministic
          const int kk = (tile == dec_first_step(cc, GR, T) / S) ? 0 : 1;
          const float *ps = a.partial + (((int64_t)cc * 2 + kk) * kGvRows + r) * MC;
#pragma unroll
          for (int c = 0; c < MC; ++c) tot[c] += __ldcg(ps + c);
        }
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < MC; ++c)
            if (c < a.m)
              a.y[(int64_t)c * a.ldy + n] =
                  EPI ? epilogue_out(tot[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : tot[c] + bias;
        }
        if (cw == 0 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      // the next tile's slot may reuse this CTA's slot only after s_last is read
      asm volatile("bar.sync 2, 128;" ::: "memory");
    };

    const int tfirst = g0 / S, tlast = nsteps > 0 ? (g1 - 1) / S : tfirst - 1;
    for (int tile = tfirst; tile <= tlast; ++tile) {
      const int lo = max(g0, tile * S) - g0, hi = min(g1, (tile + 1) * S) - g0;
#pragma unroll
      for (int c = 0; c < MC; ++c) acc[c] = 0.0f;
      for (int ls = lo + (((grp - lo) % kGvGroups) + kGvGroups) % kGvGroups; ls < hi; ls += kGvGroups) {
        const int i = ls % PS, j = ls % LS;
        // Failed waits do not leave the loop: every consumer must run the
        // same sequence of flushes (they meet on named barriers).
        bool ok = !*abort;
        ok = ok && sm100::mbar_wait(&full[i], (uint32_t)(ls / PS) & 1u, a.err, abort, kGvWaitNs);
        ok = ok && sm100::mbar_wait(&lfull[j], (uint32_t)(ls / LS) & 1u, a.err, abort, kGvWaitNs);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          const uint8_t *ck = smem + L::kRingOff + i * L::kChunk;
          const uint8_t *lslot = smem + L::kLimbOff + j * L::kLimbSlot;
          // Block scales (and Q4_1 mins) of this row's quad.
          const uint2 d2 = *reinterpret_cast<const uint2 *>(ck + L::kPk + 16 * r + 8 * h);
          uint2 m2 = make_uint2(0u, 0u);
          if constexpr (QT == MQ_Q4_1) m2 = *reinterpret_cast<const uint2 *>(ck + L::kPk + 2048 + 16 * r + 8 * h);
          const uint32_t dw[2] = {d2.x, d2.y}, mw[2] = {m2.x, m2.y};
          uint4 W[QT == MQ_Q8_0 ? 8 : 4];
          if constexpr (QT == MQ_Q8_0) {
#pragma unroll
            for (int c16 = 0; c16 < 8; ++c16) W[c16] = *reinterpret_cast<const uint4 *>(ck + chunk16_off(r, c16, h));
          } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) W[t] = *reinterpret_cast<const uint4 *>(ck + chunk16_off(r, 4 * h + t, 0));
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int jb = 4 * h + jj;
            const __half2 dh = *reinterpret_cast<const __half2 *>(&dw[jj >> 1]);
            const float d = (jj & 1) ? __high2float(dh) : __low2float(dh);
            float mn = 0.0f;
            if constexpr (QT == MQ_Q4_1) {
              const __half2 mh = *reinterpret_cast<const __half2 *>(&mw[jj >> 1]);
              mn = (jj & 1) ? __high2float(mh) : __low2float(mh);
            }
#pragma unroll
            for (int c = 0; c < MC; ++c) {
              const uint4 *lw = reinterpret_cast<const uint4 *>(lslot + ((c * 8 + jb) * 8) * 12);
              const int4 hdr = *reinterpret_cast<const int4 *>(lslot + MC * L::kLimbRow + (c * 8 + jb) * 16);
              uint32_t lmb[24];
#pragma unroll
              for (int q = 0; q < 6; ++q) {
                const uint4 u4 = lw[q];
                lmb[4 * q] = u4.x, lmb[4 * q + 1] = u4.y, lmb[4 * q + 2] = u4.z, lmb[4 * q + 3] = u4.w;
              }
              const float dinv = d * __int_as_float(hdr.y);
              if constexpr (QT == MQ_Q8_0) {
                int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const uint4 wc = W[2 * t + (jj >> 1)];
                  const uint32_t w0 = (jj & 1) ? wc.z : wc.x, w1 = (jj & 1) ? wc.w : wc.y;
                  s0 = dp4a_su(w0, lmb[6 * t + 0], s0);
                  s1 = dp4a_su(w0, lmb[6 * t + 1], s1);
                  s2 = dp4a_ss(w0, lmb[6 * t + 2], s2);
                  s0 = dp4a_su(w1, lmb[6 * t + 3], s0);
                  s1 = dp4a_su(w1, lmb[6 * t + 4], s1);
                  s2 = dp4a_ss(w1, lmb[6 * t + 5], s2);
                }
                const int s01 = s0 + (int)((uint32_t)s1 << 8);  // |.| < 2^29
                acc[c] = fmaf(fmaf((float)s2, 65536.0f, (float)s01), dinv, acc[c]);
              } else {
                int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const uint4 wc = W[t];
                  const uint32_t w = jj == 0 ? wc.x : jj == 1 ? wc.y : jj == 2 ? wc.z : wc.w;
                  const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
                  a0 = dp4a_uu(lo, lmb[6 * t + 0], a0);
                  a1 = dp4a_uu(lo, lmb[6 * t + 1], a1);
                  a2 = dp4a_us(lo, lmb[6 * t + 2], a2);
                  b0 = dp4a_uu(hi, lmb[6 * t + 3], b0);
                  b1 = dp4a_uu(hi, lmb[6 * t + 4], b1);
                  b2 = dp4a_us(hi, lmb[6 * t + 5], b2);
                }
                // sum q X = sum_l 2^(8 l) (a_l + b_l / 16): exact in wrapping int32.
                uint32_t tq = (uint32_t)(a0 + (b0 >> 4)) + ((uint32_t)(a1 + (b1 >> 4)) << 8) +
                              ((uint32_t)(a2 + (b2 >> 4)) << 16);
                if constexpr (QT == MQ_Q4_0) tq -= (uint32_t)hdr.x << 3;
                acc[c] = fmaf((float)(int)tq, dinv, acc[c]);
                if constexpr (QT == MQ_Q4_1) acc[c] = fmaf(mn, __int_as_float(hdr.z), acc[c]);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          sm100::mbar_arrive(&empty[i]);
          sm100::mbar_arrive(&lempty[j]);
        }
      }
      // The row's (group, quad) sums meet: the other warps hand theirs over,
      // the group-0 quad-0 warps add them in a fixed order and complete the tile.
      float *xb = xch + (int64_t)((tile - tfirst) & 1) * (2 * kGvGroups) * kGvRows * MC;
      if (!owner) {
#pragma unroll
        for (int c = 0; c < MC; ++c) xb[((grp * 2 + h) * kGvRows + r) * MC + c] = acc[c];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kGvConsumers) : "memory");
      if (owner) {
#pragma unroll
        for (int q = 1; q < 2 * kGvGroups; ++q)
#pragma unroll
          for (int c = 0; c < MC; ++c) acc[c] += xb[(q * kGvRows + r) * MC + c];
        flush(tile);
      }
    }
  }
}

}  // namespace mq
