// tcgen05 decode GEMM with the block scales folded into the A operand, for
// 5..32 activation rows.
//
// The other tensor-core decode kernel (mq_tcdec.cuh) multiplies the weights'
// integer codes and applies each 32-weight block's fp16 scale afterwards, so
// every block's partial sums make a round trip through their own TMEM slot
// (MMA, commit, tcgen05.ld, release). With 16-32 activation rows a block's
// partial sums fill 32-64 TMEM columns, few blocks fit in flight, and that
// round trip sets the pace. Here the scale is folded into the weights
// exactly, and a tile's accumulators stay in TMEM over the CTA's whole K
// range of the tile: they are read once per tile.
//
// Exactness scheme. A weight is w = d * c with c = q - zp (Q4_0: q - 8, Q4_1:
// q, Q8_0: q) and d the block's fp16 scale. d has at most 11 significant bits
// and c at most 4 (Q4_x) or 7 (Q8_0), so d * c has at most 15 / 18 and splits
// exactly into an fp16 pair, w = A_hi + A_lo with A_hi = fp16(d * c) (round to
// nearest) and A_lo = d * c - A_hi (one fused multiply-add, exact: its lowest
// bit is that of d, at least 2^-24). Each activation row is scaled by one
// power of two (max |x| in [2^13, 2^14)) and split into fp16 hi + lo rows
// (fold_prep_kernel), the B operand [x_hi | x_lo] (N = 2 bn). Per K16 two MMAs
// accumulate into the same D: A_hi x [x_hi | x_lo] and A_lo x [x_hi | x_lo],
// so D[:, c] + D[:, bn + c] = sum_k w_k (x_hi + x_lo)_k: every product of
// fp16 values is exact in the fp32 accumulator. x_hi + x_lo carries 22
// significant bits of every activation whose lo part is an fp16 normal, and
// misses any activation by at most 2^-25 in the scaled units (2^-38 of the
// row's max |x|); the result equals the reference fp32 dot up to that and to
// accumulation-order rounding. The Q4_1 block minimum is applied in the drain
// (m * sum_k x, from the split's block sums). The fold needs |d * c| < 65504
// (the fp16 range): mq_weight_create checks the scales once and weights
// outside it stay on mq_tcdec.cuh.
//
// Two independent pipelines, one per K half h of every quant block (K
// positions 16h..16h+15 of each 32): decoder group h writes the A columns of
// half h, issuer h issues that half's 8 MMAs of a quad (4 blocks x {A_hi,
// A_lo}) into its own accumulator D_h and commits; D_0 + D_1 is the tile's
// result. Each accumulator is written by one thread's in-order MMA stream, so
// the sums are deterministic.
//
// TMEM: three A slots of one quad each (128 K: A_hi in columns 0..63, A_lo in
// 64..127, each [K half][block][8 columns] as the activation tile), then NT
// tile accumulator pairs (D_0, D_1) of 2 bn columns each.
//
// Warp roles (16 warps):
//   warp 0         bulk copies of each step's packed codes (PS stages) and
//                  fp16 scales / Q4_1 mins (SS stages);
//   warps 1, 3     MMA issue for K half 0 / 1, one thread each; warp 1 also
//                  allocates the TMEM;
//   warp 2         TMA: the activation tile of every quad (hi rows, lo rows);
//   warps 4..11    decoders: warps 4..7 K half 0, 8..11 K half 1, one TMEM
//                  lane quarter each; packed bytes -> exact codes -> d * c
//                  split into A_hi / A_lo (fp16 pairs) -> tcgen05.st;
//   warps 12..15   drainers (TMEM lane = tile row): per step, the Q4_1 minima;
//                  per tile, tcgen05.ld of both accumulators, 2^-e of the row
//                  scale, bias, store or stream-K partial.
// Persistent stream-K over the tile-major (128-row tile, 8-block step) space
// as the other decode kernels; a split tile is completed by its last
// contributor from the partial slots in CTA order (deterministic).
// Launched with programmatic dependent launch after the activation split:
// TMEM allocation, the weight stream and the decoding of the first quads
// start while the split still runs.
// Every wait is bounded in time; a timeout raises the CTA abort flag and the
// host-visible error flag and every role leaves its loop (drainers keep their
// loop shape so that their named barriers still match); in-flight copies and
// MMAs are waited for (bounded) before the TMEM is released.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec.cuh"

namespace mq {

constexpr int kFdWarps = 16;
constexpr int kFdThreads = 32 * kFdWarps;
constexpr int kFdQuadBars = 16;  // quad-completion barriers per K half (ring)

template <int QT, int BN>
struct FdCfg {
  static constexpr int N = 2 * BN;     // MMA N: hi rows, then lo rows
  static constexpr int NA = 3;         // A slots (one quad each, hi + lo: 128 columns)
  static constexpr int kACols = 128;
  static constexpr int kDOff = NA * kACols;
  static constexpr int NT = (512 - kDOff) / (2 * N);  // tile accumulator pairs (D_0, D_1)
  static_assert(NT >= 1, "TMEM budget");
  // Parity waits on a quad ring must not alias: a decoder waits for quad
  // q - NA and the TMA warp for q - XS while quads up to q - 1 may commit.
  static_assert(kFdQuadBars >= NA && kFdQuadBars >= 4, "quad ring too short");
  static constexpr int kPkBytes = kDecRows * (QT == MQ_Q8_0 ? 256 : 128);
  static constexpr int kScBytes = kDecRows * 16 * (QT == MQ_Q4_1 ? 2 : 1);
  static_assert(kPkBytes == step_pk_bytes(QT) && kScBytes == step_sc_bytes(QT), "stages hold one weight chunk");
  static constexpr int kXBytes = N * 128 * 2;   // activation tile of a quad (128 K)
  static constexpr int PS = QT == MQ_Q8_0 ? 3 : 4;
  static constexpr int SS = 4;
  static constexpr int XS = 4;
  static constexpr int kPkOff = 0;
  static constexpr int kScOff = kPkOff + PS * kPkBytes;
  static constexpr int kXOff = kScOff + SS * kScBytes;   // 1 KB aligned (128-byte swizzle atoms)
  static_assert(kXOff % 1024 == 0, "activation tiles on 1 KB boundaries");
  static constexpr int kBarOff = kXOff + XS * kXBytes;
  static constexpr int kNumBars = 2 * PS + 2 * SS + XS + 2 * NA + NT + 2 * NT + 2 * kFdQuadBars + 2;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  // Large enough that a second CTA (and its 512-column TMEM request) never
  // lands on an SM this kernel already occupies.
  static constexpr int kAlloc = (kBytes + 1024) > 118784 ? (kBytes + 1024) : 118784;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

// d * c split into fp16 hi + lo: hi = fp16(d c), lo = d c - hi (exact).
__device__ __forceinline__ void fold_pair(uint32_t code2, __half2 d2, uint32_t &hi, uint32_t &lo) {
  const __half2 c = *reinterpret_cast<const __half2 *>(&code2);
  const __half2 h = __hmul2(c, d2);
  const __half2 l = __hfma2(c, d2, __hneg2(h));
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Activation split of the scale-folded kernel: ONE power-of-two scale per
// activation row (the kernel's accumulators run along K, so the scale must not
// change along K). Grid (bn, ceil(steps / kFpSteps)): CTA (row, g) reduces
// max |x| over the whole row (every CTA of the row; x is L2-resident) and
// splits the steps [kFpSteps g, kFpSteps (g + 1)) into fp16 hi / lo pairs in
// the layout of dec_prep_kernel (one warp per step). Rows >= m are zeros.
// Outputs: x2 [2 bn][kpad], xsum [kpad / 32][bn] (scaled block sums, Q4_1),
// xinv [bn] (2^-e of each row).
constexpr int kFpThreads = 512;
constexpr int kFpSteps = 32;

__global__ void __launch_bounds__(kFpThreads)
    fold_prep_kernel(const float *x, int64_t ldx, int m, int K, int kpad, int bn, __half *__restrict__ x2,
                     float *__restrict__ xsum, float *__restrict__ xinv, int want_sums) {
  // x may come from the previous kernel, and the split buffers may still be
  // read by the previous decode launch; the decode GEMM itself may start now.
  sm100::griddep_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) sm100::griddep_launch_dependents();
  __shared__ float s_max[kFpThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = blockIdx.x;
  const bool live = row < m;
  const float *xr = x + (int64_t)(live ? row : 0) * ldx;
  float mx = 0.0f;
  if (live) {
    if ((reinterpret_cast<uintptr_t>(xr) & 15u) == 0) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xr);
      const int k4 = K >> 2;
#pragma unroll 4
      for (int i = threadIdx.x; i < k4; i += kFpThreads) {
        const float4 v = x4[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
      for (int k = 4 * k4 + threadIdx.x; k < K; k += kFpThreads) mx = fmaxf(mx, fabsf(xr[k]));
    } else {
#pragma unroll 8
      for (int k = threadIdx.x; k < K; k += kFpThreads) mx = fmaxf(mx, fabsf(xr[k]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_max[warp] = mx;
  __syncthreads();
  mx = s_max[0];
#pragma unroll
  for (int w = 1; w < kFpThreads / 32; ++w) mx = fmaxf(mx, s_max[w]);  // same order in every thread
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int E;
    frexpf(mx, &E);
    e = min(100, max(-100, 14 - E));
  }
  const float sc = ldexpf(1.0f, e);
  if (blockIdx.y == 0 && threadIdx.x == 0) xinv[row] = ldexpf(1.0f, -e);
  const int steps = kpad / 256;
  const int s1 = min(steps, (int)(blockIdx.y + 1) * kFpSteps);
  for (int step = blockIdx.y * kFpSteps + warp; step < s1; step += kFpThreads / 32) {
    const int k0 = step * 256;
    if (want_sums) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // block j of the step, element `lane`
        const int k = k0 + 32 * j + lane;
        float s = (live && k < K) ? xr[k] * sc : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) xsum[(int64_t)(step * 8 + j) * bn + row] = s;
      }
    }
    __half2 *h2 = reinterpret_cast<__half2 *>(x2 + (int64_t)row * kpad + k0);
    __half2 *l2 = reinterpret_cast<__half2 *>(x2 + (int64_t)(bn + row) * kpad + k0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // fp16 pair p = TMEM column c of block p / 16
      const int p = lane + 32 * j, c = p & 15;
      const int k = k0 + (p >> 4) * 32 + 8 * (c & 3) + 2 * (c >> 2);
      const float v0 = (live && k < K) ? xr[k] * sc : 0.0f, v1 = (live && k + 1 < K) ? xr[k + 1] * sc : 0.0f;
      const __half2 hh = __floats2half2_rn(v0, v1);
      const float2 hf = __half22float2(hh);
      h2[p] = hh;
      l2[p] = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
    }
  }
}

template <int QT, int BN, int NC, bool EPI, bool PEER>
__global__ void __launch_bounds__(kFdThreads, 1)
    fdec_kernel(const __grid_constant__ CUtensorMap tm_x, const DecArgs a) {
  using L = FdCfg<QT, BN>;
  constexpr int PS = L::PS, SS = L::SS, XS = L::XS, NA = L::NA, NT = L::NT, N = L::N;
  constexpr int NQB = kFdQuadBars;
  static_assert(NC <= BN && NC % 16 == 0, "live activation columns, 16 at a time");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = pk_full + PS;
  uint64_t *sc_full = pk_empty + PS, *sc_empty = sc_full + SS;
  uint64_t *x_full = sc_empty + SS;
  uint64_t *a_full = x_full + XS;            // [K half][A slot]
  uint64_t *d_empty = a_full + 2 * NA;       // [tile accumulator pair]
  uint64_t *tile_done = d_empty + NT;        // [K half][tile accumulator pair]
  uint64_t *quad_done = tile_done + 2 * NT;  // [K half][quad ring]
  uint64_t *fin = quad_done + 2 * NQB;       // one per issuer
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;
  __shared__ uint32_t s_peer_e;  // the gather's epoch, when the outputs also go to the peers

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.steps, T = a.tiles * a.steps, GR = gridDim.x, cta = blockIdx.x;
  const int g0 = dec_first_step(cta, GR, T), g1 = dec_first_step(cta + 1, GR, T);
  const int nsteps = g1 - g0;
  const int nquads = 2 * nsteps;
  const int tfirst = g0 / S, tlast = nsteps > 0 ? (g1 - 1) / S : tfirst - 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&pk_full[i], 1), sm100::mbar_init(&pk_empty[i], 8);
    for (int i = 0; i < SS; ++i)
      sm100::mbar_init(&sc_full[i], 1), sm100::mbar_init(&sc_empty[i], QT == MQ_Q4_1 ? 12 : 8);
    for (int i = 0; i < XS; ++i) sm100::mbar_init(&x_full[i], 1);
    for (int i = 0; i < 2 * NA; ++i) sm100::mbar_init(&a_full[i], 4);
    for (int i = 0; i < NT; ++i) sm100::mbar_init(&d_empty[i], 4);
    for (int i = 0; i < 2 * NT; ++i) sm100::mbar_init(&tile_done[i], 1);
    for (int i = 0; i < 2 * NQB; ++i) sm100::mbar_init(&quad_done[i], 1);
    for (int i = 0; i < 2; ++i) sm100::mbar_init(&fin[i], 1);
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
  if (threadIdx.x == 0) sm100::griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------- bulk copies: packed codes and their scales
      int issued_pk = 0, issued_sc = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int g = g0 + ls;
        const uint8_t *chunk = chunk_ptr(a.w, g / S, g % S);
        const int i = ls % PS;
        if (!sm100::mbar_wait_sleep(&pk_empty[i], ((uint32_t)(ls / PS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) break;
        sm100::mbar_arrive_expect_tx(&pk_full[i], L::kPkBytes);
        sm100::bulk_load(smem + L::kPkOff + i * L::kPkBytes, chunk, L::kPkBytes, &pk_full[i]);
        issued_pk = ls + 1;
        const int j = ls % SS;
        if (!sm100::mbar_wait_sleep(&sc_empty[j], ((uint32_t)(ls / SS) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) break;
        sm100::mbar_arrive_expect_tx(&sc_full[j], L::kScBytes);
        sm100::bulk_load(smem + L::kScOff + j * L::kScBytes, chunk + L::kPkBytes, L::kScBytes, &sc_full[j]);
        issued_sc = ls + 1;
      }
      for (int p = issued_pk - PS < 0 ? 0 : issued_pk - PS; p < issued_pk; ++p)
        sm100::mbar_wait(&pk_full[p % PS], (uint32_t)(p / PS) & 1u, nullptr, nullptr, kDecDrainNs);
      for (int p = issued_sc - SS < 0 ? 0 : issued_sc - SS; p < issued_sc; ++p)
        sm100::mbar_wait(&sc_full[p % SS], (uint32_t)(p / SS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 2) {
    if (lane == 0) {  // ------------------------------------- TMA: activation tiles, one per quad
      sm100::prefetch_tmap(&tm_x);
      sm100::griddep_wait();  // the activation split is the previous kernel
      int issued = 0;
      for (int q = 0; q < nquads; ++q) {
        const int i = q % XS;
        if (q >= XS) {  // the stage is free once both halves' MMAs of quad q - XS completed
          const int qb = q - XS;
          const uint32_t par = (uint32_t)(qb / NQB) & 1u;
          if (!sm100::mbar_wait_sleep(&quad_done[qb % NQB], par, a.err, abort, kDecWaitNs) ||
              !sm100::mbar_wait_sleep(&quad_done[NQB + qb % NQB], par, a.err, abort, kDecWaitNs))
            break;
        }
        const int k = (g0 + q / 2) % S;
        const int kx = (k * kDecBlocksPerStep + 4 * (q & 1)) * 32;
        uint8_t *dst = smem + L::kXOff + i * L::kXBytes;
        sm100::mbar_arrive_expect_tx(&x_full[i], L::kXBytes);
        sm100::tma_load_2d(dst, &tm_x, kx, 0, &x_full[i]);
        sm100::tma_load_2d(dst + N * 128, &tm_x, kx + 64, 0, &x_full[i]);
        issued = q + 1;
      }
      for (int q = issued - XS < 0 ? 0 : issued - XS; q < issued; ++q)
        sm100::mbar_wait(&x_full[q % XS], (uint32_t)(q / XS) & 1u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp == 1 || warp == 3) {
    const int h = warp >> 1;  // K half: warp 1 issues half 0, warp 3 half 1
    if (lane == 0) {  // ------------------------------------- MMA issue: 8 MMAs and one commit per quad
      constexpr uint32_t idesc = idesc_f16_f32(kDecRows, N);
      uint64_t *afull = a_full + h * NA, *qdone = quad_done + h * NQB;
      bool ok = true;
      int lt = 0;
      for (int tile = tfirst; ok && tile <= tlast; ++tile, ++lt) {
        const int q0 = 2 * (max(g0, tile * S) - g0), q1 = 2 * (min(g1, (tile + 1) * S) - g0);
        // the accumulator pair is free once the drainers read the tile NT before
        ok = sm100::mbar_wait(&d_empty[lt % NT], ((uint32_t)(lt / NT) & 1u) ^ 1u, a.err, abort, kDecWaitNs);
        const uint32_t dbase = tmem + (uint32_t)(L::kDOff + (lt % NT) * 2 * N + h * N);
        for (int q = q0; ok && q < q1; ++q) {
          ok = sm100::mbar_wait(&afull[q % NA], (uint32_t)(q / NA) & 1u, a.err, abort, kDecWaitNs);
          ok = ok && sm100::mbar_wait(&x_full[q % XS], (uint32_t)(q / XS) & 1u, a.err, abort, kDecWaitNs);
          if (!ok) break;
          sm100::tc_fence_after();
          const uint32_t abase = tmem + (uint32_t)((q % NA) * L::kACols);
          const uint64_t xdesc = sm100::umma_desc_sw128(sm100::smem_u32(smem + L::kXOff + (q % XS) * L::kXBytes));
#pragma unroll
          for (int jq = 0; jq < 4; ++jq) {
            constexpr int kRow = N * 128;  // bytes of one 64-K atom column of the activation tile
            const int kk = 32 * jq + 16 * h;
            const uint32_t off = (uint32_t)((kk >> 6) * kRow + (kk & 63) * 2);
            const uint32_t acol = (uint32_t)(32 * h + 8 * jq);
            umma_f16_tmem_a(dbase, abase + acol, xdesc + (off >> 4), idesc, (q == q0 && jq == 0) ? 0u : 1u);
            umma_f16_tmem_a(dbase, abase + 64u + acol, xdesc + (off >> 4), idesc, 1u);
          }
          sm100::umma_commit(&qdone[q % NQB]);
        }
        if (ok) sm100::umma_commit(&tile_done[h * NT + lt % NT]);
      }
      // Everything issued has completed before the TMEM is released.
      sm100::umma_commit(&fin[h]);
      sm100::mbar_wait(&fin[h], 0u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp < 12) {  // ------------------------------- decoders: packed bytes -> d * c as fp16 hi + lo in TMEM
    const int qq = warp & 3;          // TMEM lane quarter
    const int hh = (warp - 4) >> 2;   // K half of every block: A columns 32hh..32hh+31 of a slot half
    const int r = 32 * qq + lane;     // tile row
    const int sw = r & 7;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    uint64_t *afull = a_full + hh * NA, *qdone = quad_done + hh * NQB;
    for (int ls = 0; ls < nsteps; ++ls) {
      const int pi = ls % PS, si = ls % SS;
      // tcgen05.st is warp-collective: every wait result is made warp-uniform.
      bool ok = sm100::mbar_wait_sleep(&pk_full[pi], (uint32_t)(ls / PS) & 1u, a.err, abort, kDecWaitNs);
      ok = ok && sm100::mbar_wait_sleep(&sc_full[si], (uint32_t)(ls / SS) & 1u, a.err, abort, kDecWaitNs);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint4 dq = *reinterpret_cast<const uint4 *>(smem + L::kScOff + si * L::kScBytes + r * 16);
      const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll 1
      for (int qi = 0; qi < 2; ++qi) {
        const int q = 2 * ls + qi;
        if (q >= NA) {  // this half of the A slot is free once its MMAs of quad q - NA completed
          const int qb = q - NA;
          if (!__all_sync(0xffffffffu, sm100::mbar_wait_sleep(&qdone[qb % NQB], (uint32_t)(qb / NQB) & 1u, a.err,
                                                              abort, kDecWaitNs))) {
            ok = false;
            break;
          }
        }
        uint32_t hi[32], lo[32];  // [block j][8 columns]: K pairs 16hh..16hh+15 of every block
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t dbits = dw[(4 * qi + j) >> 1];
          const uint16_t d16 = (uint16_t)(((4 * qi + j) & 1) ? (dbits >> 16) : (dbits & 0xFFFFu));
          const __half2 d2 = __halves2half2(__ushort_as_half(d16), __ushort_as_half(d16));
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int t = 2 * hh + tt;
            uint32_t code[4];
            if constexpr (QT == MQ_Q8_0) {
              const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + qi * (kDecRows * 128) + r * 128;
              const uint4 c4 = *reinterpret_cast<const uint4 *>(prow + (((2 * t + (j >> 1)) ^ sw) << 4));
              const uint32_t u0 = ((j & 1) ? c4.z : c4.x) ^ 0x80808080u, u1 = ((j & 1) ? c4.w : c4.y) ^ 0x80808080u;
              code[0] = dcode_q8(u0, 0x4140u);
              code[1] = dcode_q8(u0, 0x4342u);
              code[2] = dcode_q8(u1, 0x4140u);
              code[3] = dcode_q8(u1, 0x4342u);
            } else {
              const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + r * 128;
              const uint4 c4 = *reinterpret_cast<const uint4 *>(prow + (((4 * qi + t) ^ sw) << 4));
              const uint32_t wv = j == 0 ? c4.x : j == 1 ? c4.y : j == 2 ? c4.z : c4.w;
              code[0] = dcode_q4<QT>(wv, 0);
              code[1] = dcode_q4<QT>(wv, 8);
              code[2] = dcode_q4<QT>(wv, 4);
              code[3] = dcode_q4<QT>(wv, 12);
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) fold_pair(code[s], d2, hi[8 * j + 4 * tt + s], lo[8 * j + 4 * tt + s]);
          }
        }
        const uint32_t aslot = tmem + lane_base + (uint32_t)((q % NA) * L::kACols + 32 * hh);
        tmem_st_x32(aslot, hi);
        tmem_st_x32(aslot + 64u, lo);
        tmem_st_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&afull[q % NA]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) {
        sm100::mbar_arrive(&pk_empty[pi]);
        sm100::mbar_arrive(&sc_empty[si]);
      }
    }
  } else {  // ------------------------------------------------ drainers (TMEM lane = tile row)
    sm100::griddep_wait();  // block sums, row scales, outputs and workspace
    const uint32_t pe = PEER ? peer_epoch(a.peer) : 0u;
    if (warp == 12 && lane == 0) s_peer_e = pe;
    const int qq = warp & 3;
    const int r = 32 * qq + lane;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    float acc[NC];
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
            if (c < a.m) {
              const float v =
                  EPI ? epilogue_out(acc[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : acc[c] + bias;
              a.y[(int64_t)c * a.ldy + n] = v;
              if constexpr (PEER) peer_store(a.peer, pe, c, n, v);
            }
        }
        return;
      }
      const int kind = (tile == g0 / S) ? 0 : 1;
      float *slot = a.partial + (((int64_t)cta * 2 + kind) * kDecRows + r) * BN;
#pragma unroll
      for (int c = 0; c < NC; c += 4)
        *reinterpret_cast<float4 *>(slot + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      // Release: the barrier orders the 128 threads' slot writes before one
      // thread's device-scope fence and ticket; the last contributor mirrors it.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int cf = dec_cta_of_step(tg0, GR, T), cl = dec_cta_of_step(tg1 - 1, GR, T);
      if (warp == 12 && lane == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
        if (last) __threadfence();
        s_last = last;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        float tot[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) tot[c] = 0.0f;
        for (int cc = cf; cc <= cl; ++cc) {  // fixed CTA order: deterministic
          const int kk = (tile == dec_first_step(cc, GR, T) / S) ? 0 : 1;
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
            if (c < a.m) {
              const float v =
                  EPI ? epilogue_out(tot[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : tot[c] + bias;
              a.y[(int64_t)c * a.ldy + n] = v;
              if constexpr (PEER) peer_store(a.peer, pe, c, n, v);
            }
        }
        if (warp == 12 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      // the next tile's slot may reuse this CTA's slot only after s_last is read
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    int lt = 0;
    for (int tile = tfirst; tile <= tlast; ++tile, ++lt) {
      const int lo = max(g0, tile * S) - g0, hi = min(g1, (tile + 1) * S) - g0;
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
      if constexpr (QT == MQ_Q4_1) {  // sum_b m_b * sum_k x over the tile's blocks (x in the row scale)
        // Failed waits do not leave the loop: every drainer must run the same
        // sequence of flushes (they synchronise on a named barrier).
        for (int ls = lo; ls < hi; ++ls) {
          const int kstep = (g0 + ls) % S;
          const int si = ls % SS;
          const bool sc_ok = sm100::mbar_wait_sleep(&sc_full[si], (uint32_t)(ls / SS) & 1u, a.err, abort, kDecWaitNs);
          if (sc_ok) {
            const uint4 mq4 =
                *reinterpret_cast<const uint4 *>(smem + L::kScOff + si * L::kScBytes + kDecRows * 16 + r * 16);
            const uint32_t mw[4] = {mq4.x, mq4.y, mq4.z, mq4.w};
#pragma unroll
            for (int jb = 0; jb < kDecBlocksPerStep; ++jb) {
              const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw[jb >> 1]);
              const float mm = (jb & 1) ? __high2float(m2) : __low2float(m2);
              const float4 *xs =
                  reinterpret_cast<const float4 *>(a.xsum + (int64_t)(kstep * kDecBlocksPerStep + jb) * BN);
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
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&sc_empty[si]);
        }
      }
      // Both halves' accumulators of the tile: D_0 (hi, lo columns) + D_1 (hi, lo).
      const uint32_t par = (uint32_t)(lt / NT) & 1u;
      bool ok = sm100::mbar_wait_sleep(&tile_done[lt % NT], par, a.err, abort, kDecWaitNs);
      ok = ok && sm100::mbar_wait_sleep(&tile_done[NT + lt % NT], par, a.err, abort, kDecWaitNs);
      ok = __all_sync(0xffffffffu, ok);
      sm100::tc_fence_after();
      const uint32_t dbase = tmem + lane_base + (uint32_t)(L::kDOff + (lt % NT) * 2 * N);
#pragma unroll
      for (int c0 = 0; c0 < NC; c0 += 16) {
        float sum[16];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t vh[16], vl[16];
          if (ok) {
            tmem_ld_x16(dbase + (uint32_t)(hf * N + c0), vh);
            tmem_ld_x16(dbase + (uint32_t)(hf * N + BN + c0), vl);
            sm100::tmem_ld_wait();
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) vh[c] = vl[c] = 0u;
          }
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float v = __uint_as_float(vh[c]) + __uint_as_float(vl[c]);
            sum[c] = hf ? sum[c] + v : v;
          }
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c0 + c] += sum[c];
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&d_empty[lt % NT]);
      {  // back to x's own scale: 2^-e of each activation row
        const float4 *inv = reinterpret_cast<const float4 *>(a.xinv);
#pragma unroll
        for (int c = 0; c < NC; c += 4) {
          const float4 v4 = __ldg(inv + c / 4);
          acc[c] *= v4.x, acc[c + 1] *= v4.y, acc[c + 2] *= v4.z, acc[c + 3] *= v4.w;
        }
      }
      flush(tile);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if constexpr (PEER) peer_finish(a.peer, s_peer_e);  // every CTA's outputs are in the peers' staging
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

}  // namespace mq
