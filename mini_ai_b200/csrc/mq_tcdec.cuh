// tcgen05 decode GEMM for a few activation rows (M <= 32).
//
// Decode is HBM-bound: every packed weight byte is streamed once. With M in
// the tens, an fp32 SIMT dot would need M FMAs per weight and fall behind
// HBM, so the products run on the 5th-generation tensor cores while the SIMT
// lanes only decode.
//
// Exactness scheme. The A operand holds the exact integers q - zp (fp16), not
// the scaled weights, so no rounding or range issue is introduced by the
// per-block fp16 scale; each activation row is scaled, per 256-K step, by a
// power of two and split into fp16 hi + lo (22 significant bits), stacked as
// the two halves of the MMA's N dimension. Each 32-weight block accumulates into its own TMEM
// slot, and drainer warps apply the block scale in fp32:
//   acc += d_b * (D_b,hi + D_b,lo) (+ m_b * sum_b x).
// Products of small integers and fp16 values are exact in the fp32
// accumulator, so the result equals the fp32 reference dot up to
// accumulation-order rounding.
//
// Cost model (measured on B200): one tcgen05.mma with N <= 64 occupies the
// SM's tensor pipe for ~44 cycles whatever its operands' source, and so does
// a commit. A block of 128 rows x 32 weights therefore takes two MMAs
// (K = 16 each, hi and lo in one instruction through N) and commits are
// batched per group of G blocks. The tensor pipe queues only about two MMAs,
// so the issuing thread must not stall: its loop is fully unrolled over a
// quad with precomputed addresses, and a second issuer on another warp
// scheduler covers the first one's barrier waits. Roles that wait off the
// issue path sleep in the barrier (try_wait with a time hint) instead of
// spinning, leaving the issue slots to the decoders and the issuers. The A operand is written by the decoders
// straight into TMEM (tcgen05.st), which keeps the 2 B/weight of fp16 codes
// off the shared-memory port entirely; shared memory only carries the packed
// bytes and the activation tiles.
//
// K order inside a block. Decoder warp h (of the two per TMEM lane quarter)
// writes the K pairs 8h..8h+7 of every block (the A operand of the block's
// MMA h), taken from its own two 16-byte chunks of the lane-permuted weight
// layout; an A slot is [h][block][8 columns]. The activation tile uses
// the same order: column c = 4t + s of a block holds the original K pair
// (8s + 2t, 8s + 2t + 1), for both the Q4 and the Q8 layouts.
//
// Persistent stream-K: one CTA per SM walks a contiguous range of the
// tile-major (128-row tile, packed K step) space, so the weight stream never
// restarts; a tile whose K loop is split across CTAs is completed by the last
// contributor from at most two partial slots per CTA (deterministic order).
// A packed step is 8 quant blocks (256 K) = two quads of 4 blocks.
// Warp roles (20 warps, 16 for 32 activation rows; every role that blocks on
// an mbarrier has a warp of its own, since a lane suspended in try_wait holds
// up the diverged lanes of its warp):
//   warp 0         bulk copies of each step's weight chunk: packed quant rows
//                  (pre-swizzled, PS stages) and fp16 block scales (+ Q4_1
//                  mins, SS stages);
//   warps 1, 3     TMEM allocation (warp 1); MMA issue from one thread each,
//                  alternate quads, one commit per group;
//   warp 2         TMA: fp16 activation tiles (hi rows, lo rows), one per quad;
//   warps 4..11    decoders: two per TMEM lane quarter, one per K half of
//                  every block; packed bytes -> exact fp16 codes -> one
//                  tcgen05.st per quad into the A ring (one quad a slot);
//   warps 12..19   drainers, two sets of one warp per lane quarter taking
//                  the D groups in turn (one set for 32 rows): per group,
//                  TMEM -> registers, scale in fp32; flush per tile (x row
//                  scale 2^-e, bias, store or partial + ticket) by set 0 after
//                  adding set 1's sums. A group's drain is a chain of barrier
//                  wait, TMEM loads and dependent arithmetic that one set
//                  alone ran at well under the MMA rate (measured on B200).
// Launched with programmatic stream serialization after the activation split:
// TMEM allocation and the weight stream start while the split still runs; the
// activation TMA and the drainers wait for it (griddepcontrol.wait).
// Every wait is bounded in time; a timeout raises the CTA abort flag and the
// host-visible error flag, and all roles leave their loops (the drainers keep
// their loop shape so that their named barriers still match). Before the TMEM
// is released the MMA thread waits for its last commit and the TMA threads
// for their copies in flight.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_peer.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec_api.h"

namespace mq {

constexpr int kDecRows = 128;
constexpr int kDecWarps = 16;  // without the second drainer set
constexpr int kDecBlocksPerStep = 8;  // quant blocks per packed step (Q4_x: 128 B per row, Q8_0: 256 B)
constexpr int kDecGroupBars = 16;     // commit barriers, one per group in a ring
constexpr uint64_t kDecWaitNs = 1000000000ull;
constexpr uint64_t kDecDrainNs = 20000000ull;

struct DecArgs {
  WeightView w;
  int m;                 // activation rows (<= NC)
  const float *xinv;     // [steps][BN] 2^-e per (step, activation row); folded kernel: [BN] per row
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
  const float *gate = nullptr;   // fused gate/up product: y = silu(gate) * (product + bias); gate [m, ldy]
  const float *resid = nullptr;  // residual add: y = resid + (product + bias); resid [m, ldy], may be y
  PeerOut peer;                  // row-sharded linear: also store the outputs into the peers' staging (G > 1)
};

template <int QT, int BN>
struct DecCfg {
  static constexpr int N = 2 * BN;    // MMA N: hi rows, then lo rows
  static constexpr int G = 64 / N;     // blocks per commit group: a group's D is 64 TMEM columns
  static constexpr int NA = 4;         // A quads in TMEM (64 columns each)
  static constexpr int ND = 4;         // D groups in TMEM
  static constexpr int kACols = 64;
  static constexpr int kDCols = G * N;
  static constexpr int kDOff = NA * kACols;
  static_assert(kDCols == 64 && kDOff + ND * kDCols <= 512, "TMEM budget");
  // Parity waits on the commit ring must not alias: a decoder waits for the
  // last group of quad q - NA while quads up to q - 1 may have committed.
  static_assert(kDecGroupBars > (4 / G) * (NA - 1), "commit ring too short");
  static constexpr int kPkBytes = kDecRows * (QT == MQ_Q8_0 ? 256 : 128);  // packed step
  static constexpr int kScBytes = kDecRows * 16 * (QT == MQ_Q4_1 ? 2 : 1);  // scales (+ mins) of a step
  static_assert(kDecRows == kTileRows && kPkBytes == step_pk_bytes(QT) && kScBytes == step_sc_bytes(QT),
                "stages hold the parts of one weight chunk");
  static constexpr int kXBytes = N * 128 * 2;                               // activation tile of a quad (128 K)
  static constexpr int PS = QT == MQ_Q8_0 ? 3 : 4;  // packed stages
  static constexpr int SS = 6;                      // scale stages
  static constexpr int XS = 4;                      // activation stages (one quad each)
  static constexpr int kPkOff = 0;
  static constexpr int kScOff = kPkOff + PS * kPkBytes;
  static constexpr int kXOff = kScOff + SS * kScBytes;
  static constexpr int kBarOff = kXOff + XS * kXBytes;
  static constexpr int kQuadsPerUnit = 1;            // an MMA issuer's unit: one quad (whole groups)
  // Two issuers take alternate quads. With G = 1 a quad's four groups use
  // every D slot, so both issuers would wait on the same slots: one issuer.
  static constexpr int kIssuers = G == 1 ? 1 : 2;
  // Drainer sets (warps 12..15, and 16..19 when there are two): set s drains
  // the D groups gi with gi % DSETS == s, so each D slot (ND is a multiple of
  // DSETS) and each commit barrier is released / awaited by one set in order.
  // The 32-row configuration keeps one set: its drain needs the registers.
  static constexpr int DSETS = N == 64 ? 1 : 2;
  static constexpr int kThreads = (kDecWarps + 4 * (DSETS - 1)) * 32;
  static_assert(ND % DSETS == 0 && kDecGroupBars % DSETS == 0 && (kDecBlocksPerStep / G) % DSETS == 0,
                "drainer set ownership of the D slots and commit barriers");
  static constexpr int kNumBars = 2 * PS + 2 * SS + XS + NA + ND + kDecGroupBars + 2;
  static constexpr int kXchOff = (kBarOff + 8 * kNumBars + 16 + 15) / 16 * 16;  // set 1's tile sums: float[2][128][BN]
  static constexpr int kBytes = kXchOff + (DSETS > 1 ? 2 * kDecRows * BN * 4 : 0);
  // At least 116 KB, so that a second CTA (and its 512-column TMEM request)
  // never lands on an SM this kernel already occupies.
  static constexpr int kAlloc = (kBytes + 1024) > 118784 ? (kBytes + 1024) : 118784;
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

// D[tmem] (+)= A[tmem] x B[smem]^T, kind::f16, A read from tensor memory.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// N consecutive 32-bit columns of this warp's 32 lanes.
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 16) {
    tmem_ld_x16(taddr, r);
  } else if constexpr (N == 32) {
    sm100::tmem_ld_32x32b_x32(taddr, r);
  } else {
    static_assert(N == 64, "activation tile width");
    sm100::tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    sm100::tmem_ld_32x32b_x32(taddr + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
  }
}

// EPI: the output write applies the epilogues of DecArgs::gate / resid (a
// separate instantiation: the plain product is compiled without them).
template <int QT, int BN, int NC, bool EPI>
__global__ void __launch_bounds__(DecCfg<QT, BN>::kThreads, 1)
    tcdec_kernel(const __grid_constant__ CUtensorMap tm_x, const DecArgs a) {
  using L = DecCfg<QT, BN>;
  constexpr int PS = L::PS, SS = L::SS, XS = L::XS, NA = L::NA, ND = L::ND, G = L::G, N = L::N;
  constexpr int NGB = kDecGroupBars;
  constexpr int kGroupsPerStep = kDecBlocksPerStep / G;
  constexpr int kQPU = L::kQuadsPerUnit, NI = L::kIssuers;
  static_assert(NC <= BN && NC % 4 == 0, "live activation columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = pk_full + PS;
  uint64_t *sc_full = pk_empty + PS, *sc_empty = sc_full + SS;
  uint64_t *x_full = sc_empty + SS, *a_full = x_full + XS, *d_empty = a_full + NA;
  uint64_t *grp_done = d_empty + ND, *fin = grp_done + NGB;  // fin: one per issuer
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.steps, T = a.tiles * a.steps, GR = gridDim.x, cta = blockIdx.x;
  const int g0 = dec_first_step(cta, GR, T), g1 = dec_first_step(cta + 1, GR, T);
  const int nsteps = g1 - g0;
  const int nquads = 2 * nsteps;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&pk_full[i], 1), sm100::mbar_init(&pk_empty[i], 8);
    for (int i = 0; i < SS; ++i) sm100::mbar_init(&sc_full[i], 1), sm100::mbar_init(&sc_empty[i], 4 * L::DSETS);
    for (int i = 0; i < XS; ++i) sm100::mbar_init(&x_full[i], 1);
    for (int i = 0; i < NA; ++i) sm100::mbar_init(&a_full[i], 8);
    for (int i = 0; i < ND; ++i) sm100::mbar_init(&d_empty[i], 4);
    for (int i = 0; i < NGB; ++i) sm100::mbar_init(&grp_done[i], 1);
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

  // Commit group of the last block of quad q: its completion frees the quad's
  // A slot and activation stage.
  auto quad_group = [&](int q) { return (4 * q + 3) / G; };

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------- bulk copies: packed quant rows and their scales
      // A CTA's steps are consecutive chunks of the weight: one linear stream.
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
        if (q >= XS) {  // the stage is free once the MMAs of quad q - XS completed
          const int gq = quad_group(q - XS);
          if (!sm100::mbar_wait_sleep(&grp_done[gq % NGB], (uint32_t)(gq / NGB) & 1u, a.err, abort, kDecWaitNs))
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
    const int issuer = warp >> 1;  // warp 1: units 0, 2, 4, ...; warp 3: units 1, 3, 5, ...
    if (lane == 0 && issuer < NI) {  // ------------------------- MMA issue, one commit per group
      // A unit is one quad (two when a commit group spans two quads). The two
      // issuers sit on different warp schedulers and take alternate units, so
      // that one issues while the other waits. Every barrier slot an issuer
      // waits on was last waited on by the same issuer, or completes in order
      // with one it has waited on, so parity waits never alias.
      constexpr uint32_t idesc = idesc_f16_f32(kDecRows, N);
      const int nunits = nquads / kQPU;
      for (int u = issuer; u < nunits; u += NI) {
        bool ok = true;
        uint32_t abase[kQPU];
        uint64_t xdesc[kQPU];
#pragma unroll
        for (int qi = 0; qi < kQPU; ++qi) {
          const int q = u * kQPU + qi;
          ok = ok && sm100::mbar_wait(&a_full[q % NA], (uint32_t)(q / NA) & 1u, a.err, abort, kDecWaitNs);
          ok = ok && sm100::mbar_wait(&x_full[q % XS], (uint32_t)(q / XS) & 1u, a.err, abort, kDecWaitNs);
          abase[qi] = tmem + (uint32_t)((q % NA) * L::kACols);
          xdesc[qi] = sm100::umma_desc_sw128(sm100::smem_u32(smem + L::kXOff + (q % XS) * L::kXBytes));
        }
        if (!ok) break;
        uint32_t dbase = 0;
#pragma unroll
        for (int bl = 0; bl < 4 * kQPU; ++bl) {
          const int qi = bl >> 2, jq = bl & 3;
          const int b = u * 4 * kQPU + bl;
          const int jg = bl % G;  // units start on group boundaries
          if (jg == 0) {
            const int gi = b / G;
            if (!sm100::mbar_wait(&d_empty[gi % ND], ((uint32_t)(gi / ND) & 1u) ^ 1u, a.err, abort, kDecWaitNs)) {
              ok = false;
              break;
            }
            sm100::tc_fence_after();
            dbase = tmem + (uint32_t)(L::kDOff + (gi % ND) * L::kDCols);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            constexpr int kRow = N * 128;  // bytes of one 64-K atom column of the activation tile
            const int kk = 32 * jq + 16 * h;
            const uint32_t off = (uint32_t)((kk >> 6) * kRow + (kk & 63) * 2);
            umma_f16_tmem_a(dbase + (uint32_t)(jg * N), abase[qi] + (uint32_t)(32 * h + 8 * jq),
                            xdesc[qi] + (off >> 4), idesc, (uint32_t)h);
          }
          if (jg == G - 1) sm100::umma_commit(&grp_done[(b / G) % NGB]);
        }
        if (!ok) break;
      }
      // Everything issued has completed before the TMEM is released.
      sm100::umma_commit(&fin[issuer]);
      sm100::mbar_wait(&fin[issuer], 0u, nullptr, nullptr, kDecDrainNs);
    }
  } else if (warp < 12) {  // -------------------------------- decoders: packed bytes -> exact fp16 codes in TMEM
    const int qq = warp & 3;          // TMEM lane quarter
    const int hh = (warp - 4) >> 2;   // K half of every block: A columns 32hh..32hh+31 of a slot
    const int r = 32 * qq + lane;     // tile row
    const int sw = r & 7;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    for (int ls = 0; ls < nsteps; ++ls) {
      const int pi = ls % PS;
      // tcgen05.st is warp-collective: every wait result is made warp-uniform.
      if (!__all_sync(0xffffffffu,
                      sm100::mbar_wait_sleep(&pk_full[pi], (uint32_t)(ls / PS) & 1u, a.err, abort, kDecWaitNs)))
        break;
      bool ok = true;
#pragma unroll 1
      for (int qi = 0; qi < 2; ++qi) {
        const int q = 2 * ls + qi;
        if (q >= NA) {  // the A slot is free once the MMAs of quad q - NA completed
          const int gq = quad_group(q - NA);
          if (!__all_sync(0xffffffffu, sm100::mbar_wait_sleep(&grp_done[gq % NGB], (uint32_t)(gq / NGB) & 1u, a.err,
                                                              abort, kDecWaitNs))) {
            ok = false;
            break;
          }
        }
        uint32_t col[32];  // [block j][8 columns]: K pairs 16hh..16hh+15 of every block
        if constexpr (QT == MQ_Q8_0) {
          const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + qi * (kDecRows * 128) + r * 128;
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int t = 2 * hh + tt;
            const uint4 c0 = *reinterpret_cast<const uint4 *>(prow + (((2 * t) ^ sw) << 4));      // blocks 0, 1
            const uint4 c1 = *reinterpret_cast<const uint4 *>(prow + (((2 * t + 1) ^ sw) << 4));  // blocks 2, 3
            const uint32_t wv[4][2] = {{c0.x, c0.y}, {c0.z, c0.w}, {c1.x, c1.y}, {c1.z, c1.w}};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t u0 = wv[j][0] ^ 0x80808080u, u1 = wv[j][1] ^ 0x80808080u;
              col[8 * j + 4 * tt + 0] = dcode_q8(u0, 0x4140u);
              col[8 * j + 4 * tt + 1] = dcode_q8(u0, 0x4342u);
              col[8 * j + 4 * tt + 2] = dcode_q8(u1, 0x4140u);
              col[8 * j + 4 * tt + 3] = dcode_q8(u1, 0x4342u);
            }
          }
        } else {
          const uint8_t *prow = smem + L::kPkOff + pi * L::kPkBytes + r * 128;
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int t = 2 * hh + tt;
            const uint4 c = *reinterpret_cast<const uint4 *>(prow + (((4 * qi + t) ^ sw) << 4));
            const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              col[8 * j + 4 * tt + 0] = dcode_q4<QT>(wv[j], 0);
              col[8 * j + 4 * tt + 1] = dcode_q4<QT>(wv[j], 8);
              col[8 * j + 4 * tt + 2] = dcode_q4<QT>(wv[j], 4);
              col[8 * j + 4 * tt + 3] = dcode_q4<QT>(wv[j], 12);
            }
          }
        }
        tmem_st_x32(tmem + lane_base + (uint32_t)((q % NA) * L::kACols + 32 * hh), col);
        tmem_st_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&a_full[q % NA]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&pk_empty[pi]);
    }
  } else {  // ------------------------------------------------ drainers (TMEM lane = tile row)
    // DSETS sets of four warps (one per TMEM lane quarter); set ds drains the
    // D groups gi = ds, ds + DSETS, ... of every step. Set 1 hands its tile
    // sums to set 0 through shared memory, and set 0 adds them to its own
    // (fixed order) and completes the tile.
    constexpr int DSETS = L::DSETS;
    const int ds = (warp - 12) >> 2;
    sm100::griddep_wait();  // block sums, row scales, outputs and workspace
    const int qq = warp & 3;
    const int r = 32 * qq + lane;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    float acc[NC];
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
            if (c < a.m) a.y[(int64_t)c * a.ldy + n] = EPI ? epilogue_out(acc[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : acc[c] + bias;
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
      const int cf = dec_cta_of_step(tg0, GR, T), cl = dec_cta_of_step(tg1 - 1, GR, T);
      if (warp == 12 && lane == 0) s_last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
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
            if (c < a.m) a.y[(int64_t)c * a.ldy + n] = EPI ? epilogue_out(tot[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : tot[c] + bias;
        }
        if (warp == 12 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      // the next tile's slot may reuse this CTA's slot only after s_last is read
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    // Every tile that the CTA's step range touches, in order; the sets meet on
    // named barrier 2 at its end (the exchange buffer alternates between two
    // halves, so a set-1 write for the next tile cannot meet a set-0 read).
    const int tfirst = g0 / S, tlast = nsteps > 0 ? (g1 - 1) / S : tfirst - 1;
    for (int tile = tfirst; tile <= tlast; ++tile) {
      const int lo = max(g0, tile * S) - g0, hi = min(g1, (tile + 1) * S) - g0;
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
      for (int ls = lo; ls < hi; ++ls) {
        const int kstep = (g0 + ls) % S;
        const int si = ls % SS;
        // Failed waits do not leave the loop: every drainer must run the same
        // sequence of flushes (they synchronise on a named barrier).
        const bool sc_ok = sm100::mbar_wait_sleep(&sc_full[si], (uint32_t)(ls / SS) & 1u, a.err, abort, kDecWaitNs);
        const uint8_t *sc = smem + L::kScOff + si * L::kScBytes;
        const uint4 dq = *reinterpret_cast<const uint4 *>(sc + r * 16);
        uint4 mq = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (QT == MQ_Q4_1) mq = *reinterpret_cast<const uint4 *>(sc + kDecRows * 16 + r * 16);
        const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
        const uint32_t mw[4] = {mq.x, mq.y, mq.z, mq.w};
        float st[NC];  // this step's sum, in the step's activation scale
#pragma unroll
        for (int c = 0; c < NC; ++c) st[c] = 0.0f;
#pragma unroll
        for (int gl = ds; gl < kGroupsPerStep; gl += DSETS) {
          const int gi = ls * kGroupsPerStep + gl;
          bool ok = sm100::mbar_wait_sleep(&grp_done[gi % NGB], (uint32_t)(gi / NGB) & 1u, a.err, abort, kDecWaitNs);
          ok = __all_sync(0xffffffffu, ok && sc_ok);
          sm100::tc_fence_after();
          const uint32_t dbase = tmem + lane_base + (uint32_t)(L::kDOff + (gi % ND) * L::kDCols);
          if constexpr (N == 64) {
            // 32 activation rows (G = 1): the hi and lo halves one after the other,
            // so that a half, the step sum and the accumulator fit the registers.
            const int jb = gl;
            const __half2 d2 = *reinterpret_cast<const __half2 *>(&dw[jb >> 1]);
            const float d = (jb & 1) ? __high2float(d2) : __low2float(d2);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              uint32_t vh[32];
              if (ok) {
                sm100::tmem_ld_32x32b_x32(dbase + (uint32_t)(32 * half), vh);
                sm100::tmem_ld_wait();
              } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) vh[c] = 0u;
              }
#pragma unroll
              for (int c = 0; c < NC; c += 2) {
                const float2 r2 = __ffma2_rn(make_float2(d, d), make_float2(__uint_as_float(vh[c]), __uint_as_float(vh[c + 1])),
                                             make_float2(st[c], st[c + 1]));
                st[c] = r2.x, st[c + 1] = r2.y;
              }
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&d_empty[gi % ND]);
            if constexpr (QT == MQ_Q4_1) {
              const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw[jb >> 1]);
              const float mm = (jb & 1) ? __high2float(m2) : __low2float(m2);
              const float4 *xs =
                  reinterpret_cast<const float4 *>(a.xsum + (int64_t)(kstep * kDecBlocksPerStep + jb) * BN);
#pragma unroll
              for (int c = 0; c < NC; c += 4) {
                const float4 s4 = __ldg(xs + c / 4);
                st[c] = fmaf(mm, s4.x, st[c]);
                st[c + 1] = fmaf(mm, s4.y, st[c + 1]);
                st[c + 2] = fmaf(mm, s4.z, st[c + 2]);
                st[c + 3] = fmaf(mm, s4.w, st[c + 3]);
              }
            }
            continue;
          }
          // One block at a time (N columns: the hi rows, then the lo rows); the
          // D slot is released once the group's last block is in registers.
#pragma unroll
          for (int jg = 0; jg < G; ++jg) {
            const int jb = gl * G + jg;  // block of the step
            uint32_t vb[N];
            if (ok) {
              tmem_ld_n<N>(dbase + (uint32_t)(jg * N), vb);
              sm100::tmem_ld_wait();
            } else {
#pragma unroll
              for (int c = 0; c < N; ++c) vb[c] = 0u;
            }
            if (jg == G - 1) {
              sm100::tc_fence_before();
              __syncwarp();
              if (lane == 0) sm100::mbar_arrive(&d_empty[gi % ND]);
            }
            const __half2 d2 = *reinterpret_cast<const __half2 *>(&dw[jb >> 1]);
            const float d = (jb & 1) ? __high2float(d2) : __low2float(d2);
#pragma unroll
            for (int c = 0; c < NC; c += 2) {
              float2 r2 = __ffma2_rn(make_float2(d, d), make_float2(__uint_as_float(vb[c]), __uint_as_float(vb[c + 1])),
                                     make_float2(st[c], st[c + 1]));
              r2 = __ffma2_rn(make_float2(d, d),
                              make_float2(__uint_as_float(vb[BN + c]), __uint_as_float(vb[BN + c + 1])), r2);
              st[c] = r2.x, st[c + 1] = r2.y;
            }
            if constexpr (QT == MQ_Q4_1) {
              const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw[jb >> 1]);
              const float mm = (jb & 1) ? __high2float(m2) : __low2float(m2);
              const float4 *xs =
                  reinterpret_cast<const float4 *>(a.xsum + (int64_t)(kstep * kDecBlocksPerStep + jb) * BN);
#pragma unroll
              for (int c = 0; c < NC; c += 4) {
                const float4 s4 = __ldg(xs + c / 4);
                st[c] = fmaf(mm, s4.x, st[c]);
                st[c + 1] = fmaf(mm, s4.y, st[c + 1]);
                st[c + 2] = fmaf(mm, s4.z, st[c + 2]);
                st[c + 3] = fmaf(mm, s4.w, st[c + 3]);
              }
            }
          }
        }
        {  // back to x's own scale: 2^-e of this step
          const float4 *inv = reinterpret_cast<const float4 *>(a.xinv + (int64_t)kstep * BN);
#pragma unroll
          for (int c = 0; c < NC; c += 4) {
            const float4 v4 = __ldg(inv + c / 4);
            acc[c] = fmaf(st[c], v4.x, acc[c]);
            acc[c + 1] = fmaf(st[c + 1], v4.y, acc[c + 1]);
            acc[c + 2] = fmaf(st[c + 2], v4.z, acc[c + 2]);
            acc[c + 3] = fmaf(st[c + 3], v4.w, acc[c + 3]);
          }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&sc_empty[si]);
      }
      if constexpr (DSETS > 1) {
        float *xb = reinterpret_cast<float *>(smem + L::kXchOff) + ((int64_t)((tile - tfirst) & 1) * kDecRows + r) * BN;
        if (ds == 1) {
#pragma unroll
          for (int c = 0; c < NC; ++c) xb[c] = acc[c];
        }
        asm volatile("bar.sync 2, 256;" ::: "memory");
        if (ds == 0) {
#pragma unroll
          for (int c = 0; c < NC; ++c) acc[c] += xb[c];
        }
      }
      if (ds == 0) flush(tile);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// Activation split for the decode GEMM: one warp per (256-K step, activation
// row), so the whole split is a single parallel pass (rows >= m become
// zeros). The step's slice of row i is scaled by 2^e (largest magnitude in
// [2^13, 2^14)), split into fp16 hi + lo and written K-major into x2
// ([2 bn][kpad]: hi rows, then lo rows) in the decode kernel's K order
// (column c = 4t + s of a block holds the original pair 8s + 2t, 8s + 2t + 1);
// the scaled block sums (Q4_1, natural order) and 2^-e ([steps][bn]) are
// written alongside. Grid: (steps, ceil(bn / 8)), 256 threads.
__global__ void dec_prep_kernel(const float *__restrict__ x, int64_t ldx, int m, int K, int kpad, int bn,
                                __half *__restrict__ x2, float *__restrict__ xsum, float *__restrict__ xinv,
                                int want_sums) {
  // x may come from the previous kernel, and the split buffers may still be
  // read by the previous decode launch; the decode GEMM itself may start now.
  sm100::griddep_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) sm100::griddep_launch_dependents();
  const int lane = threadIdx.x & 31, row = blockIdx.y * 8 + (threadIdx.x >> 5), step = blockIdx.x;
  if (row >= bn) return;
  const bool live = row < m;
  const float *xr = x + (int64_t)(live ? row : 0) * ldx;
  const int k0 = step * 256;
  float v[8];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // block j of the step, element `lane`
    const int k = k0 + 32 * j + lane;
    v[j] = (live && k < K) ? xr[k] : 0.0f;
    mx = fmaxf(mx, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int E;
    frexpf(mx, &E);
    e = min(100, max(-100, 14 - E));
  }
  const float sc = ldexpf(1.0f, e);
  if (lane == 0) xinv[(int64_t)step * bn + row] = ldexpf(1.0f, -e);
  if (want_sums) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = v[j] * sc;
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

}  // namespace mq
