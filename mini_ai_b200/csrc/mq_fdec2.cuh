// The scale-folded decode kernel (mq_fdec.cuh) on CTA pairs: tcgen05
// cta_group::2, for 5..32 activation rows and weights with an even number of
// 128-row tiles.
//
// Why pairs. In the one-CTA kernel the SM's tensor pipe accepts the 16 MMAs
// of a quad (M 128, N 32-64, K 16, A from TMEM) at a fixed rate that more
// issuing threads do not raise, and that rate, not the bytes, sets the pace.
// A pair of CTAs on the two SMs of a TPC processes two tiles together: the
// leader issues MMAs of M = 256 whose A rows 0..127 are the leader's tile
// (its TMEM) and 128..255 the peer's tile (the peer's TMEM, same columns),
// so each SM's quad needs half the MMA issues.
//
// Layout of the work: pair p of P (= gridDim.x / 2) owns a contiguous range
// of the (pair tile, 8-block step) space, pair tile t covering weight tiles
// 2t (leader) and 2t + 1 (peer); both CTAs of a pair walk the same steps.
// The B operand [x_hi | x_lo] (N = 2 bn) is split by columns across the
// pair: the leader's stage holds the x_hi rows, the peer's the x_lo rows,
// each CTA loading its half by TMA with the completion bytes counted on the
// leader's barrier. D (128 lanes x N columns) lands in each CTA's own TMEM.
//
// Roles as in mq_fdec.cuh, with the MMA issue (warps 1, 3) in the leader
// only. Hand-offs across the pair:
//   decoders -> leader's A-slot barrier (remote arrive, release.cluster);
//   TMA loads of both CTAs -> leader's activation barrier (transaction bytes);
//   MMA completion -> commit multicast to both CTAs (quad, tile, final);
//   drainers -> leader's accumulator-free barrier (remote arrive).
// The leader waits on barriers that the peer arrives on with cluster-scope
// acquire. Both CTAs allocate and free the TMEM together (cta_group::2) and
// synchronise the cluster after the barrier set-up and before the free.
// Every wait on a barrier is bounded as in the other kernels.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_fdec.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec.cuh"

namespace mq {

template <int QT, int BN>
struct Fd2Cfg {
  static constexpr int N = 2 * BN;     // MMA N: hi rows (leader's stage), then lo rows (peer's stage)
  static constexpr int NA = 3;         // A slots (one quad each, hi + lo: 128 columns)
  static constexpr int kACols = 128;
  static constexpr int kDOff = NA * kACols;
  static constexpr int NT = (512 - kDOff) / (2 * N);  // tile accumulator pairs (D_0, D_1)
  static_assert(NT >= 1, "TMEM budget");
  static constexpr int kPkBytes = kDecRows * (QT == MQ_Q8_0 ? 256 : 128);
  static constexpr int kScBytes = kDecRows * 16 * (QT == MQ_Q4_1 ? 2 : 1);
  static_assert(kPkBytes == step_pk_bytes(QT) && kScBytes == step_sc_bytes(QT), "stages hold one weight chunk");
  static constexpr int kXBytes = BN * 128 * 2;  // this CTA's half of a quad's activation tile (128 K)
  static constexpr int PS = QT == MQ_Q8_0 ? 3 : 4;
  static constexpr int SS = 4;
  static constexpr int XS = 4;
  static_assert(kFdQuadBars >= NA && kFdQuadBars >= XS, "quad ring too short");
  static constexpr int kPkOff = 0;
  static constexpr int kScOff = kPkOff + PS * kPkBytes;
  static constexpr int kXOff = kScOff + SS * kScBytes;   // 1 KB aligned (128-byte swizzle atoms)
  static_assert(kXOff % 1024 == 0 && kXBytes % 1024 == 0, "activation tiles on 1 KB boundaries");
  static constexpr int kBarOff = kXOff + XS * kXBytes;
  static constexpr int kNumBars = 2 * PS + 2 * SS + XS + 2 * NA + NT + 2 * NT + 2 * kFdQuadBars + 2;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  // One CTA per SM (and its 512-column TMEM request alone there).
  static constexpr int kAlloc = (kBytes + 1024) > 118784 ? (kBytes + 1024) : 118784;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void umma2_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int QT, int BN, int NC, bool EPI>
__global__ void __launch_bounds__(kFdThreads, 1)
    fdec2_kernel(const __grid_constant__ CUtensorMap tm_x, const DecArgs a) {
  using L = Fd2Cfg<QT, BN>;
  constexpr int PS = L::PS, SS = L::SS, XS = L::XS, NA = L::NA, NT = L::NT, N = L::N;
  constexpr int NQB = kFdQuadBars;
  static_assert(NC <= BN && NC % 16 == 0, "live activation columns, 16 at a time");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = pk_full + PS;
  uint64_t *sc_full = pk_empty + PS, *sc_empty = sc_full + SS;
  uint64_t *x_full = sc_empty + SS;            // leader: both halves' bytes
  uint64_t *a_full = x_full + XS;              // leader: [K half][A slot], both CTAs' decoders
  uint64_t *d_empty = a_full + 2 * NA;         // leader: [tile accumulator pair], both CTAs' drainers
  uint64_t *tile_done = d_empty + NT;          // both: [K half][tile accumulator pair] (commit multicast)
  uint64_t *quad_done = tile_done + 2 * NT;    // both: [K half][quad ring] (commit multicast)
  uint64_t *fin = quad_done + 2 * NQB;         // both: one per issuer (commit multicast)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_rank();  // 0: leader (issues the MMAs), 1: peer
  const int pair = blockIdx.x >> 1, NP = gridDim.x >> 1;
  const int S = a.steps, T = (a.tiles >> 1) * a.steps, cta = blockIdx.x;
  const int g0 = dec_first_step(pair, NP, T), g1 = dec_first_step(pair + 1, NP, T);
  const int nsteps = g1 - g0;
  const int nquads = 2 * nsteps;
  const int tfirst = g0 / S, tlast = nsteps > 0 ? (g1 - 1) / S : tfirst - 1;  // pair tiles
  // a barrier of the leader, addressed from either CTA
  auto leader = [](uint64_t *bar) { return sm100::mapa_shared(sm100::smem_u32(bar), 0u); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&pk_full[i], 1), sm100::mbar_init(&pk_empty[i], 8);
    for (int i = 0; i < SS; ++i)
      sm100::mbar_init(&sc_full[i], 1), sm100::mbar_init(&sc_empty[i], QT == MQ_Q4_1 ? 12 : 8);
    for (int i = 0; i < XS; ++i) sm100::mbar_init(&x_full[i], 1);
    for (int i = 0; i < 2 * NA; ++i) sm100::mbar_init(&a_full[i], 8);  // 4 decoder warps x 2 CTAs
    for (int i = 0; i < NT; ++i) sm100::mbar_init(&d_empty[i], 8);     // 4 drainer warps x 2 CTAs
    for (int i = 0; i < 2 * NT; ++i) sm100::mbar_init(&tile_done[i], 1);
    for (int i = 0; i < 2 * NQB; ++i) sm100::mbar_init(&quad_done[i], 1);
    for (int i = 0; i < 2; ++i) sm100::mbar_init(&fin[i], 1);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc_pair(tmem_slot, 512);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  sm100::cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) sm100::griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------- bulk copies: this CTA's tile of each pair tile
      int issued_pk = 0, issued_sc = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int g = g0 + ls;
        const uint8_t *chunk = chunk_ptr(a.w, 2 * (g / S) + (int)rank, g % S);
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
    if (lane == 0) {  // ------------------------------------- TMA: this CTA's half of every quad's activation tile
      sm100::prefetch_tmap(&tm_x);
      sm100::griddep_wait();  // the activation split is the previous kernel
      for (int q = 0; q < nquads; ++q) {
        const int i = q % XS;
        if (q >= XS) {  // the stage is free once both halves' MMAs of quad q - XS completed (multicast commits)
          const int qb = q - XS;
          const uint32_t par = (uint32_t)(qb / NQB) & 1u;
          if (!sm100::mbar_wait_sleep(&quad_done[qb % NQB], par, a.err, abort, kDecWaitNs) ||
              !sm100::mbar_wait_sleep(&quad_done[NQB + qb % NQB], par, a.err, abort, kDecWaitNs))
            break;
        }
        const int k = (g0 + q / 2) % S;
        const int kx = (k * kDecBlocksPerStep + 4 * (q & 1)) * 32;
        uint8_t *dst = smem + L::kXOff + i * L::kXBytes;
        if (rank == 0) sm100::mbar_arrive_expect_tx(&x_full[i], 2 * L::kXBytes);  // both halves
        const uint32_t bar = leader(&x_full[i]);
        sm100::tma_load_2d_pair(dst, &tm_x, kx, (int)rank * BN, bar);
        sm100::tma_load_2d_pair(dst + BN * 128, &tm_x, kx + 64, (int)rank * BN, bar);
      }
      // No copy may still be landing when the CTA exits: every issued stage is
      // consumed by an MMA whose commit the other roles wait for, and the final
      // cluster barrier follows the issuers' wait for their last commit.
    }
  } else if (warp == 1 || warp == 3) {
    const int h = warp >> 1;  // K half: warp 1 issues half 0, warp 3 half 1
    if (lane == 0 && rank == 0) {  // ------------------------ MMA issue (leader): 8 MMAs of M 256 per quad
      constexpr uint32_t idesc = idesc_f16_f32(2 * kDecRows, N);
      uint64_t *afull = a_full + h * NA, *qdone = quad_done + h * NQB;
      bool ok = true;
      int lt = 0;
      for (int tile = tfirst; ok && tile <= tlast; ++tile, ++lt) {
        const int q0 = 2 * (max(g0, tile * S) - g0), q1 = 2 * (min(g1, (tile + 1) * S) - g0);
        ok = sm100::mbar_wait_cluster(&d_empty[lt % NT], ((uint32_t)(lt / NT) & 1u) ^ 1u, a.err, abort, kDecWaitNs);
        const uint32_t dbase = tmem + (uint32_t)(L::kDOff + (lt % NT) * 2 * N + h * N);
        for (int q = q0; ok && q < q1; ++q) {
          ok = sm100::mbar_wait_cluster(&afull[q % NA], (uint32_t)(q / NA) & 1u, a.err, abort, kDecWaitNs);
          ok = ok && sm100::mbar_wait(&x_full[q % XS], (uint32_t)(q / XS) & 1u, a.err, abort, kDecWaitNs);
          if (!ok) break;
          sm100::tc_fence_after();
          const uint32_t abase = tmem + (uint32_t)((q % NA) * L::kACols);
          const uint64_t xdesc = sm100::umma_desc_sw128(sm100::smem_u32(smem + L::kXOff + (q % XS) * L::kXBytes));
#pragma unroll
          for (int jq = 0; jq < 4; ++jq) {
            constexpr int kRow = BN * 128;  // bytes of one 64-K atom column of this CTA's half tile
            const int kk = 32 * jq + 16 * h;
            const uint32_t off = (uint32_t)((kk >> 6) * kRow + (kk & 63) * 2);
            const uint32_t acol = (uint32_t)(32 * h + 8 * jq);
            umma2_f16_tmem_a(dbase, abase + acol, xdesc + (off >> 4), idesc, (q == q0 && jq == 0) ? 0u : 1u);
            umma2_f16_tmem_a(dbase, abase + 64u + acol, xdesc + (off >> 4), idesc, 1u);
          }
          sm100::umma_commit_pair(&qdone[q % NQB]);
        }
        if (ok) sm100::umma_commit_pair(&tile_done[h * NT + lt % NT]);
      }
      // Everything issued has completed before either CTA releases its TMEM.
      sm100::umma_commit_pair(&fin[h]);
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
        if (lane == 0) sm100::mbar_arrive_cluster(leader(&afull[q % NA]));
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
    const int qq = warp & 3;
    const int r = 32 * qq + lane;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    float acc[NC];
    // The output rows of pair tile pt in this CTA: weight tile 2 pt + rank.
    // A pair tile split across pairs is completed by the last contributing
    // pair's CTA of the same rank, from the partial slots in pair order.
    auto flush = [&](int pt) {
      const bool aborted = *abort;
      if (aborted && a.nan_on_abort) {
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[c] = __int_as_float(0x7fc00000);
      }
      const bool write = !aborted || a.nan_on_abort;
      const int tile = 2 * pt + (int)rank;
      const int n = tile * kDecRows + r;
      const bool row_ok = n < a.w.rows;
      const int tg0 = pt * S, tg1 = tg0 + S;
      if (tg0 >= g0 && tg1 <= g1) {
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < NC; ++c)
            if (c < a.m)
              a.y[(int64_t)c * a.ldy + n] =
                  EPI ? epilogue_out(acc[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : acc[c] + bias;
        }
        return;
      }
      const int kind = (pt == g0 / S) ? 0 : 1;
      float *slot = a.partial + (((int64_t)cta * 2 + kind) * kDecRows + r) * BN;
#pragma unroll
      for (int c = 0; c < NC; c += 4)
        *reinterpret_cast<float4 *>(slot + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int pf = dec_cta_of_step(tg0, NP, T), pl = dec_cta_of_step(tg1 - 1, NP, T);  // contributing pairs
      if (warp == 12 && lane == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.tickets[tile], 1) == pl - pf;
        if (last) __threadfence();
        s_last = last;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        float tot[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) tot[c] = 0.0f;
        for (int pp = pf; pp <= pl; ++pp) {  // fixed pair order: deterministic
          const int kk = (pt == dec_first_step(pp, NP, T) / S) ? 0 : 1;
          const float *ps = a.partial + (((int64_t)(2 * pp + (int)rank) * 2 + kk) * kDecRows + r) * BN;
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
            if (c < a.m)
              a.y[(int64_t)c * a.ldy + n] =
                  EPI ? epilogue_out(tot[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : tot[c] + bias;
        }
        if (warp == 12 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    int lt = 0;
    for (int pt = tfirst; pt <= tlast; ++pt, ++lt) {
      const int lo = max(g0, pt * S) - g0, hi = min(g1, (pt + 1) * S) - g0;
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
      if constexpr (QT == MQ_Q4_1) {  // sum_b m_b * sum_k x over the tile's blocks (x in the row scale)
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
      if (lane == 0) sm100::mbar_arrive_cluster(leader(&d_empty[lt % NT]));
      {  // back to x's own scale: 2^-e of each activation row
        const float4 *inv = reinterpret_cast<const float4 *>(a.xinv);
#pragma unroll
        for (int c = 0; c < NC; c += 4) {
          const float4 v4 = __ldg(inv + c / 4);
          acc[c] *= v4.x, acc[c + 1] *= v4.y, acc[c + 2] *= v4.z, acc[c + 3] *= v4.w;
        }
      }
      flush(pt);
    }
  }

  // The peer's TMEM is written by the leader's MMAs: it waits for their
  // completion (the final commits reach both CTAs) before the free.
  if (warp == 1 && lane == 0 && rank == 1) {
    sm100::mbar_wait(&fin[0], 0u, nullptr, nullptr, kDecDrainNs);
    sm100::mbar_wait(&fin[1], 0u, nullptr, nullptr, kDecDrainNs);
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // neither CTA frees its TMEM or leaves while the pair still works on it
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace mq
