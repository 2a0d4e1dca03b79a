// tcgen05 int8 decode GEMV/GEMM for one to five activation rows.
//
// Decode streams every packed weight byte once, so the kernel must keep up
// with HBM while doing as little SIMT work per weight as possible. Here the
// tensor cores do all the multiplications on the weights' own integer codes:
//
//   y[i, n] = sum_b d[n,b] * sum_k q[n,b,k] * x[i, 32b + k]   (Q8_0: q signed)
//           = sum_b d[n,b] * sum_k (q - 8) * x                (Q4_0: q unsigned)
//           = sum_b (d[n,b] * sum_k q * x + m[n,b] * sum_k x) (Q4_1)
//
// Exactness scheme. Each activation row is scaled, per 32-element quant
// block, by a power of two 2^e so that the block's largest magnitude lies in
// [2^21, 2^22), and rounded to an integer X (22 significant bits: the
// rounding error of an element is at most 2^-22 of the largest |x| of its
// block, so an outlier costs precision only inside its own block). X is split into three signed 8-bit limbs,
// X = l2 * 2^16 + l1 * 2^8 + l0, and the limbs are the rows of the MMA's B
// operand (row 3t + l for activation row t, limb l). One tcgen05.mma of
// kind::i8 (M = 128 weight rows, N = 16, K = 32 = one quant block) gives, per
// weight row and block, the exact int32 sums L_l = sum_k q * l_l. The drainer
// warps combine the limbs (in int32 for Q4_x, where |sum q X| < 2^31, so the
// wrapping sum is exact; in fp32 for Q8_0) and apply the fp16 block scale and
// the block's 2^-e in fp32, so the result equals the reference's fp32 dot up
// to that rounding and accumulation order.
//
// Data flow per (128-row tile, 8-block step):
//   weight chunk (packed codes, fp16 scales, Q4_1 mins; consecutive in
//   memory): one bulk copy into the chunk ring;
//   prep warps: the step's activations (plain loads: they stay in L2, and
//   keeping them off the TMA engine keeps them from queueing behind the
//   weight copies) -> limb tile (B operand, 128-byte-swizzled K-major) in
//   the tile ring and a header (2^-e and the integer block sums of X per
//   activation row) in the step's drain slot;
//   unpacker warps: packed bytes -> int8/uint8 codes in TMEM (tcgen05.st),
//   one 64-column A slot per step (no conversion for Q8_0: the codes are
//   moved as they are; Q4_x: two logic ops per 8 nibbles); they also copy
//   the row's scales into the drain slot and release the chunk at once;
//   issuer threads, taking the steps in turn: 8 MMAs per step (A from TMEM,
//   B from shared memory) into the step's D slot, one commit per step;
//   drainer warps: tcgen05.ld of the step's D slots, limb combine, block
//   scales, accumulate; at the end of a tile: bias, store or stream-K partial.
// Every ring is released as soon as its data has moved on, so the weight
// stream is throttled only by the chunk ring and the A slots.
//
// K order inside a block. The A columns of a block follow the device weight
// layout: column 2t + h holds, in its four bytes p = 0..3,
//   Q4_x: the codes of elements 2t + {0, 8, 1, 9}[p] + 16h,
//   Q8_0: the codes of elements 2t + {0, 1, 8, 9}[p] + 16h,
// and the B image's K slot 4c + p holds the limb of the same element.
//
// Persistent stream-K over the tile-major step space, as the other decode
// kernels: a tile whose K loop is split across CTAs is completed by the last
// contributor from at most two partial slots per CTA (deterministic order).
// Warp roles (25 warps): warp 0 bulk copies of the weight chunks; warps 1, 2, 3
// and 20 MMA issue, one thread each, taking the steps in turn (issuing a
// tcgen05.mma occupies its thread for about 80 ns, measured on B200, so one
// issuer could not keep up with HBM); warp 1 also
// allocates the TMEM; warps 4..7 prep (limb tiles from the L2-resident
// activations, one step ahead), taking the steps in turn;
// warps 8..15 unpackers (one or two activation rows: two groups of one warp
// per TMEM lane quarter taking the steps in turn, a warp converting both quads
// of its row; three to five rows: all eight on every step, two per lane
// quarter, one quad of 4 blocks each); warps 16..19 and 21..24 drainers, two
// groups of one warp per lane quarter taking the steps in turn (an unpack or a
// drain step is a chain of barrier waits, shared-memory and TMEM accesses
// and dependent arithmetic: a drain step took about 0.55 us, measured on
// B200, and one group alone held every product to that step rate). Every wait is
// bounded in time; a timeout raises the CTA abort flag and the host-visible
// error flag and every role leaves its loop (drainers keep their loop shape so
// that their named barriers still match); in-flight bulk copies and MMAs are
// waited for (bounded) before the TMEM is released.
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "mq_common.cuh"
#include "mq_peer.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec.cuh"

namespace mq {

constexpr int kI8Rows = 128;
constexpr int kI8Warps = 25;
constexpr int kI8Issuers = 4;       // MMA issue threads at most (warps 1, 2, 3, 20), taking the steps in turn
constexpr int kI8Preps = 4;         // prep warps (4..7): step s is built by warp 4 + s % 4
constexpr int kI8DrainGroups = 2;   // drainer groups (warps 16..19 and 21..24): step s is drained by group s % 2
constexpr int kI8Threads = kI8Warps * 32;
constexpr int kI8MaxM = 5;          // activation rows per launch: 3 limbs x 5 rows <= N = 16
constexpr int kI8N = 16;            // MMA N (B rows)
constexpr int kI8BTile = 4096;      // B tile of a step: 2 slabs x 16 rows x 128 B (128-byte swizzle)
constexpr int kI8HdrInv = 0;        // header: 2^-e per (block, activation row), float[8 blocks][8 rows]
constexpr int kI8HdrSx = 256;       // header: integer block sums of X, int32[8 blocks][8 rows]
constexpr int kI8Done = 8;          // commit barriers (ring)
constexpr uint64_t kI8WaitNs = 1000000000ull;
constexpr uint64_t kI8DrainNs = 20000000ull;

struct I8Args {
  WeightView w;
  int m;                 // activation rows (<= MC)
  const float *x;        // [m][ldx] activations
  int64_t ldx;
  const float *bias;
  float *y;
  int64_t ldy;
  float *partial;        // [gridDim.x][2][128][MC]: head / tail partial tile of every CTA
  int *tickets;          // [tiles], zero between launches
  int steps;             // packed steps per tile (the K loop)
  int tiles;
  int *err;
  int nan_on_abort;
  const float *gate = nullptr;   // fused gate/up product: y = silu(gate) * (product + bias); gate [m, ldy]
  const float *resid = nullptr;  // residual add: y = resid + (product + bias); resid [m, ldy], may be y
  PeerOut peer;                  // row-sharded linear: also store the outputs into the peers' staging (G > 1)
};

template <int QT, int MC>
struct I8Cfg {
  static constexpr int kPkBytes = step_pk_bytes(QT);   // packed codes of a step
  static constexpr int kScBytes = step_sc_bytes(QT);   // fp16 scales (+ Q4_1 mins) of a step
  static constexpr int kChunk = kPkBytes + kScBytes;   // one weight chunk: one bulk copy per step
  static constexpr int kDrBytes = kScBytes + 512;      // drain slot: scales (+ mins) | header
  static constexpr int kDrHdr = kScBytes;
  static constexpr int NB = kI8Preps;                  // limb tiles (4 KB each)
  static constexpr int DS = 8;                         // drain slots
  // Blocks per D region: with 3 MC limb rows <= 8, block 2i + 1's limbs sit in
  // B rows 8.. and block 2i's in rows 0.. (each with zeros in the other
  // half), so the pair's two MMAs accumulate into one 16-column region and a
  // step needs half the D columns.
  static constexpr int G = 3 * MC <= 8 ? 2 : 1;
  static constexpr int kRowOff = 16 / G;               // B row offset between the blocks of a pair
  // TMEM: the unpack -> MMA -> completion round trip (~1.1 us measured) gates
  // the A slots, the MMA -> drain round trip (~1 us) the D slots.
  static constexpr int NA = 4;                         // A slots in TMEM (64 columns each)
  static constexpr int kACols = 64, kDCols = 8 * kI8N / G, kDOff = NA * kACols;
  // D slots in TMEM: a multiple of the drainer groups, so that every phase of
  // a slot's barrier is released by the same group (in step order).
  static constexpr int ND = (512 - kDOff) / kDCols / kI8DrainGroups * kI8DrainGroups;
  // Issuers take the steps in turn (each issues a whole step: tcgen05.mma
  // costs its thread ~80 ns, so several steps must be in issue at once). A
  // parity wait is sound only while the awaited phase is the barrier's
  // current or immediately preceding one; with I issuers that holds when every
  // per-step ring (A slots, tiles, commits) is a multiple of I, so that one
  // issuer owns all phases of a barrier, and ND >= I with ND - I a multiple
  // of the drainer groups (before it waits for the drain of s - ND, the issuer
  // of step s waited for the drain of s - I - ND, which the group that drains
  // s - 2 ND drains no earlier).
  static constexpr int I = ND >= 4 ? 4 : (ND >= 2 ? 2 : 1);
  static_assert(NA % I == 0 && NB % I == 0 && kI8Done % I == 0 && ND >= I && (ND - I) % kI8DrainGroups == 0,
                "issuer ownership of the rings");
  static_assert(kDOff + ND * kDCols <= 512, "TMEM budget");
  static_assert(kI8Preps <= DS && kI8Preps <= kI8Done && DS % kI8Preps == 0, "ring depths (see the waits)");
  static_assert(DS % kI8DrainGroups == 0 && kI8Done % kI8DrainGroups == 0, "drainer group ownership of the rings");
  static constexpr int kBOff = 0;                               // 1 KB aligned (128-byte swizzle atoms)
  static constexpr int kDrOff = kBOff + NB * kI8BTile;
  static constexpr int kXchOff = kDrOff + DS * kDrBytes;        // drainer groups' tile sums: float[2][128][MC]
  static constexpr int kPkOff = kXchOff + ((2 * kI8Rows * MC * 4 + 15) / 16) * 16;  // 16-byte aligned bulk destinations
  static constexpr int kPsFit = (222 * 1024 - kPkOff) / kChunk;
  // Unpacker groups taking the steps in turn (see the unpackers): two for the
  // paired-block configurations (G == 2), one for the others, the faster
  // choice for each, measured on B200.
  static constexpr int UG = G == 2 ? 2 : 1;
  // Weight chunks in flight: a multiple of UG, so that each chunk slot belongs to one unpacker group.
  static constexpr int PS = (kPsFit < 12 ? kPsFit : 12) / UG * UG;
  static constexpr int kBarOff = kPkOff + PS * kChunk;
  static constexpr int kNumBars = 2 * PS + NB + 2 * DS + NA + ND + kI8Done + kI8Issuers;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(PS >= 4 && kAlloc <= 227 * 1024, "shared memory budget");
  static_assert(PS % UG == 0 && NA % UG == 0 && DS % UG == 0 && kI8Done % UG == 0,
                "unpacker group ownership of the rings");
  static_assert(kChunk % 16 == 0 && kDrBytes % 16 == 0, "copy alignment");
  // D columns the drainers read per region and regions per batch of TMEM
  // loads (32 registers a batch).
  static constexpr int NCOL = G == 2 ? 16 : (MC <= 1 ? 4 : (MC <= 2 ? 8 : 16));
  static constexpr int BB = 32 / NCOL;
  static_assert(3 * MC <= NCOL, "limb columns");
  static_assert(MC <= kI8MaxM, "activation rows");
};

// Instruction descriptor, kind::i8: A unsigned (Q4_x) or signed (Q8_0) 8-bit,
// B signed 8-bit, D int32, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8_s32(int M, int N, bool a_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] x B[smem]^T, kind::i8.
__device__ __forceinline__ void umma_i8_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <int NCOL>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t *r) {
  if constexpr (NCOL == 4) {
    tmem_ld_x4(taddr, r);
  } else if constexpr (NCOL == 8) {
    tmem_ld_x8(taddr, r);
  } else {
    tmem_ld_x16(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
  }
}

// Element (0..31) of a quant block whose code sits in byte p of A column c
// (see "K order inside a block").
__host__ __device__ inline int i8_slot_elem(int qtype, int c, int p) {
  const int t = c >> 1, h = c & 1;
  const int q4[4] = {0, 8, 1, 9}, q8[4] = {0, 1, 8, 9};
  return 2 * t + (qtype == MQ_Q8_0 ? q8[p] : q4[p]) + 16 * h;
}

// EPI: the output write applies the epilogues of I8Args::gate / resid (a separate
// instantiation: the plain product is compiled without them).
template <int QT, int MC, bool EPI, bool PEER>
__global__ void __launch_bounds__(kI8Threads, 1) i8dec_kernel(const I8Args a) {
  using L = I8Cfg<QT, MC>;
  constexpr int PS = L::PS, NB = L::NB, DS = L::DS, NA = L::NA, ND = L::ND, NCOL = L::NCOL, BB = L::BB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *pk_full = bars, *pk_empty = pk_full + PS;   // weight chunks: bulk copy / unpackers
  uint64_t *b_full = pk_empty + PS;                     // limb tiles built (prep); reuse after the MMAs (done)
  uint64_t *dr_full = b_full + NB, *dr_empty = dr_full + DS;  // drain slots: unpackers + prep / drainers
  uint64_t *a_full = dr_empty + DS, *d_empty = a_full + NA;   // TMEM A slots (unpackers), D slots (drainers)
  uint64_t *done = d_empty + ND, *fin = done + kI8Done;       // MMA commits (4 a step), per-issuer final commit
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  __shared__ int s_last;
  __shared__ uint32_t s_peer_e;  // the gather's epoch, when the outputs also go to the peers

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.steps, T = a.tiles * a.steps, GR = gridDim.x, cta = blockIdx.x;
  const int g0 = dec_first_step(cta, GR, T), g1 = dec_first_step(cta + 1, GR, T);
  const int nsteps = g1 - g0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PS; ++i) sm100::mbar_init(&pk_full[i], 1), sm100::mbar_init(&pk_empty[i], 8 / L::UG);
    for (int i = 0; i < NB; ++i) sm100::mbar_init(&b_full[i], 1);
    for (int i = 0; i < DS; ++i) sm100::mbar_init(&dr_full[i], 5), sm100::mbar_init(&dr_empty[i], 4);
    for (int i = 0; i < NA; ++i) sm100::mbar_init(&a_full[i], 8 / L::UG);
    for (int i = 0; i < ND; ++i) sm100::mbar_init(&d_empty[i], 4);
    for (int i = 0; i < kI8Done; ++i) sm100::mbar_init(&done[i], 1);
    for (int i = 0; i < kI8Issuers; ++i) sm100::mbar_init(&fin[i], 1);
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

  // Parity waits are sound only while the awaited phase is the barrier's
  // current or immediately preceding one. Every ring below is filled and
  // drained in step order, except that the prep warps take steps in turn:
  // the tile ring has one stage per prep warp, and a prep warp's waits on the
  // shared rings (done, dr_empty) for step s come after its own waits for
  // step s - kI8Preps, which covered the previous phase (kI8Preps <= DS, kDone).
  if (warp == 0) {
    if (lane == 0) {  // --------------------------------------- weight chunks: codes + scales, one bulk copy a step
      int issued = 0;
      for (int ls = 0; ls < nsteps; ++ls) {
        const int g = g0 + ls, i = ls % PS;
        if (ls >= PS &&
            !sm100::mbar_wait_sleep(&pk_empty[i], ((uint32_t)(ls / PS) & 1u) ^ 1u, a.err, abort, kI8WaitNs))
          break;
        sm100::mbar_arrive_expect_tx(&pk_full[i], L::kChunk);
        sm100::bulk_load(smem + L::kPkOff + i * L::kChunk, chunk_ptr(a.w, g / S, g % S), L::kChunk, &pk_full[i]);
        issued = ls + 1;
      }
      // No copy may still be landing when the CTA exits.
      for (int p = issued - PS < 0 ? 0 : issued - PS; p < issued; ++p)
        sm100::mbar_wait(&pk_full[p % PS], (uint32_t)(p / PS) & 1u, nullptr, nullptr, kI8DrainNs);
    }
  } else if (warp >= 4 && warp < 4 + kI8Preps) {  // ---------- prep: activation slice -> limb tile + header
    // Lane l builds the 4-slot words w = l and l + 32 of each limb row (word
    // w: block w / 8, A column w % 8), so lanes 8i..8i+7 hold block i (u = 0)
    // and block 4 + i (u = 1). Each block of a row is scaled by its own 2^e
    // (largest magnitude in [2^21, 2^22)) and rounded to integers X (round to
    // nearest even through the fp32 magic 1.5 * 2^23), split into balanced
    // limbs X = l0 + 2^8 l1 + 2^16 l2; the header holds 2^-e and the integer
    // sum of X of every (block, row). A non-finite value in a block makes its
    // 2^-e NaN, so that row's outputs become NaN.
    const int pw = warp - 4;
    auto word_off = [](int n, int w) {  // byte offset of word w of B row n inside a limb tile
      const int j = w >> 3, c8 = w & 7;
      const int pos = 32 * (j & 3) + 4 * c8;  // byte inside the slab's 128-byte row
      return (j >> 2) * 2048 + (n >> 3) * 1024 + (n & 7) * 128 + (((pos >> 4) ^ (n & 7)) << 4) + (pos & 15);
    };
    // A lane's 8 values of row t: the slots 4c + p of column c = 2 tt + h hold
    // the elements 2 tt + {0, 8, 1, 9} + 16 h (Q4_x) or 2 tt + {0, 1, 8, 9} +
    // 16 h (Q8_0); rows >= m and K past the end read as zeros. The
    // activations are L2-resident: each prep warp loads its next step's values
    // while it builds the current one.
    auto load = [&](int ls, float (&v)[MC][8]) {
      const int k0 = ((g0 + ls) % S) * 256;
#pragma unroll
      for (int t = 0; t < MC; ++t) {
        const bool live = t < a.m;
        const float *xr = a.x + (int64_t)(live ? t : 0) * a.ldx;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int w = lane + 32 * u, j = w >> 3, c8 = w & 7;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int k = k0 + 32 * j + i8_slot_elem(QT, c8, p);
            v[t][4 * u + p] = (live && k < a.w.cols) ? __ldg(xr + k) : 0.0f;
          }
        }
      }
    };
    sm100::griddep_wait();  // the activations may come from the previous kernel
    constexpr bool kPf = MC <= 2;  // prefetch the next step's values (register budget: not for 4 rows)
    float v[MC][8], nv[kPf ? MC : 1][8];
    if (kPf && pw < nsteps) load(pw, *reinterpret_cast<float(*)[MC][8]>(&nv[0][0]));
    for (int ls = pw; ls < nsteps; ls += kI8Preps) {
      const int bi = ls % NB, di = ls % DS;
      if constexpr (kPf) {
#pragma unroll
        for (int t = 0; t < MC; ++t)
#pragma unroll
          for (int q = 0; q < 8; ++q) v[t][q] = nv[t][q];
        if (ls + kI8Preps < nsteps) load(ls + kI8Preps, *reinterpret_cast<float(*)[MC][8]>(&nv[0][0]));
      } else {
        load(ls, v);
      }
      bool ok = true;
      if (ls >= NB) {  // the limb tile is free once the MMAs of step ls - NB completed
        const int pd = ls - NB;
        ok = ok && sm100::mbar_wait_sleep(&done[pd % kI8Done], (uint32_t)(pd / kI8Done) & 1u, a.err, abort, kI8WaitNs);
      }
      if (ls >= DS)
        ok = ok && sm100::mbar_wait_sleep(&dr_empty[di], ((uint32_t)(ls / DS) & 1u) ^ 1u, a.err, abort, kI8WaitNs);
      if (!__all_sync(0xffffffffu, ok)) break;
      uint8_t *tile = smem + L::kBOff + bi * kI8BTile;
      uint8_t *hdr = smem + L::kDrOff + di * L::kDrBytes + L::kDrHdr;
      float *inv = reinterpret_cast<float *>(hdr + kI8HdrInv);
      int *sx = reinterpret_cast<int *>(hdr + kI8HdrSx);
#pragma unroll
      for (int t = 0; t < MC; ++t) {
        // The lane's two blocks one at a time (u = 0: block lane / 8, u = 1: block
        // 4 + lane / 8), so that only one block's values are live.
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          uint32_t mb = 0u;  // largest |x| bits (integer order = magnitude order, NaN above Inf)
#pragma unroll
          for (int p = 0; p < 4; ++p) mb = max(mb, __float_as_uint(v[t][4 * u + p]) & 0x7fffffffu);
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));  // the block's 8 lanes
          const bool finite = mb < 0x7f800000u;
          // mx = f * 2^E with f in [0.5, 1): E = biased exponent - 126 (subnormal blocks use E = -125)
          const int be = (int)(mb >> 23);
          const int e = (mb == 0u || !finite) ? 0 : min(126, max(-126, 22 - ((be > 0 ? be : 1) - 126)));
          const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
          const int w = lane + 32 * u;
          uint32_t b0 = 0u, b1 = 0u, b2 = 0u;
          int sum = 0;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int xv = finite ? (int)(__float_as_uint(fmaf(v[t][4 * u + p], sc, 12582912.0f)) - 0x4B400000u) : 0;
            const int x1 = (xv - (int)(int8_t)xv) >> 8;  // balanced: l0 = sext(low byte)
            const int l2 = (x1 - (int)(int8_t)x1) >> 8;
            b0 |= ((uint32_t)xv & 255u) << (8 * p);
            b1 |= ((uint32_t)x1 & 255u) << (8 * p);
            b2 |= ((uint32_t)l2 & 255u) << (8 * p);
            sum += xv;
          }
          // rows of this word's block; with block pairs, zeros in the partner block's rows
          const int rb = ((w >> 3) % L::G) * L::kRowOff + 3 * t;
          *reinterpret_cast<uint32_t *>(tile + word_off(rb + 0, w)) = b0;
          *reinterpret_cast<uint32_t *>(tile + word_off(rb + 1, w)) = b1;
          *reinterpret_cast<uint32_t *>(tile + word_off(rb + 2, w)) = b2;
          if constexpr (L::G == 2) {
            const int rz = (1 - ((w >> 3) & 1)) * L::kRowOff + 3 * t;
#pragma unroll
            for (int l = 0; l < 3; ++l) *reinterpret_cast<uint32_t *>(tile + word_off(rz + l, w)) = 0u;
          }
          // integer block sum over the block's 8 lanes, and the block's 2^-e
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          if ((lane & 7) == 0) {
            const int j = 4 * u + (lane >> 3);
            sx[j * 8 + t] = sum;
            inv[j * 8 + t] = finite ? __uint_as_float((uint32_t)(127 - e) << 23) : __int_as_float(0x7fc00000);
          }
        }
      }
      sm100::fence_proxy_async_smem();  // the MMAs read the tile through the async proxy
      __syncwarp();
      if (lane == 0) {
        sm100::mbar_arrive(&b_full[bi]);
        sm100::mbar_arrive(&dr_full[di]);
      }
    }
  } else if ((warp >= 1 && warp <= 3) || warp == 20) {
    const int issuer = warp == 20 ? 3 : warp - 1;
    if (lane == 0 && issuer < L::I) {  // ------------------------- MMA issue: steps issuer, issuer + I, ...
      constexpr uint32_t idesc = idesc_i8_s32(kI8Rows, kI8N, QT == MQ_Q8_0);
      for (int ls = issuer; ls < nsteps; ls += L::I) {
        bool ok = sm100::mbar_wait(&a_full[ls % NA], (uint32_t)(ls / NA) & 1u, a.err, abort, kI8WaitNs);
        ok = ok && sm100::mbar_wait(&b_full[ls % NB], (uint32_t)(ls / NB) & 1u, a.err, abort, kI8WaitNs);
        ok = ok && sm100::mbar_wait(&d_empty[ls % ND], ((uint32_t)(ls / ND) & 1u) ^ 1u, a.err, abort, kI8WaitNs);
        if (!ok) break;
        sm100::tc_fence_after();
        const uint32_t abase = tmem + (uint32_t)((ls % NA) * L::kACols);
        const uint32_t dbase = tmem + (uint32_t)(L::kDOff + (ls % ND) * L::kDCols);
        const uint64_t bdesc = sm100::umma_desc_sw128(sm100::smem_u32(smem + L::kBOff + (ls % NB) * kI8BTile));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // block j: slab j / 4 (2 KB), K offset 32 * (j % 4) bytes inside the 128-byte row; a
          // block pair of one D region accumulates in issue order
          const uint32_t off = (uint32_t)((j >> 2) * 2048 + (j & 3) * 32);
          umma_i8_tmem_a(dbase + (uint32_t)((j / L::G) * kI8N), abase + (uint32_t)(8 * j), bdesc + (off >> 4), idesc,
                         (uint32_t)(j % L::G));
        }
        sm100::umma_commit(&done[ls % kI8Done]);
      }
      // Everything issued has completed before the TMEM is released.
      sm100::umma_commit(&fin[issuer]);
      sm100::mbar_wait(&fin[issuer], 0u, nullptr, nullptr, kI8DrainNs);
    }
  } else if (warp >= 8 && warp < 16) {  // ----------------------- unpackers: packed bytes -> codes in TMEM
    // UG == 2: two groups of four warps (one per TMEM lane quarter) take the
    // steps in turn, and a warp converts both quads of its row's step (A
    // columns 0..31 and 32..63 of the slot). UG == 1: every step by all eight
    // warps, two per lane quarter, one quad each. The warps of the first quad
    // (all of them with UG == 2) also move the row's scales into the drain slot.
    constexpr int UG = L::UG, NQ = UG;  // quads per warp and step
    const int qq = warp & 3;                // TMEM lane quarter
    const int hq = UG == 2 ? 0 : (warp - 8) >> 2;
    const bool scales = hq == 0;
    const int r = 32 * qq + lane;           // tile row
    const int sw = r & 7;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    for (int ls = UG == 2 ? (warp - 8) >> 2 : 0; ls < nsteps; ls += UG) {
      const int pi = ls % PS, di = ls % DS;
      // tcgen05.st is warp-collective: every wait result is made warp-uniform.
      bool ok = sm100::mbar_wait_sleep(&pk_full[pi], (uint32_t)(ls / PS) & 1u, a.err, abort, kI8WaitNs);
      if (ls >= NA) {  // the A slot is free once the MMAs of step ls - NA completed
        const int pd = ls - NA;
        ok = ok && sm100::mbar_wait_sleep(&done[pd % kI8Done], (uint32_t)(pd / kI8Done) & 1u, a.err, abort, kI8WaitNs);
      }
      if (scales && ls >= DS)  // the drain slot is free once step ls - DS was drained
        ok = ok && sm100::mbar_wait_sleep(&dr_empty[di], ((uint32_t)(ls / DS) & 1u) ^ 1u, a.err, abort, kI8WaitNs);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t *chunk = smem + L::kPkOff + pi * L::kChunk;
      if (scales) {  // the row's scales (and Q4_1 mins) go to the drain slot first
        uint8_t *dr = smem + L::kDrOff + di * L::kDrBytes;
        *reinterpret_cast<uint4 *>(dr + r * 16) = *reinterpret_cast<const uint4 *>(chunk + L::kPkBytes + r * 16);
        if constexpr (QT == MQ_Q4_1)
          *reinterpret_cast<uint4 *>(dr + kI8Rows * 16 + r * 16) =
              *reinterpret_cast<const uint4 *>(chunk + L::kPkBytes + kI8Rows * 16 + r * 16);
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&dr_full[di]);
      }
      const uint32_t acol = tmem + lane_base + (uint32_t)((ls % NA) * L::kACols);
      uint32_t col[32];  // [block j of the quad][8 columns]
      if constexpr (QT == MQ_Q8_0) {
        // 128 code bytes per row and quad: a warp's quads are loaded, converted
        // and stored one after the other; the chunk is released after the last load.
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
          const int h = hq + qi;
          const uint8_t *prow = chunk + h * (kI8Rows * 128) + r * 128;
          uint32_t cw[8][4];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = *reinterpret_cast<const uint4 *>(prow + ((c ^ sw) << 4));
            cw[c][0] = v.x, cw[c][1] = v.y, cw[c][2] = v.z, cw[c][3] = v.w;
          }
          if (qi == NQ - 1) {
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&pk_empty[pi]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              col[8 * j + 2 * t] = cw[2 * t + (j >> 1)][2 * (j & 1)];
              col[8 * j + 2 * t + 1] = cw[2 * t + (j >> 1)][2 * (j & 1) + 1];
            }
          tmem_st_x32(acol + (uint32_t)(32 * h), col);
        }
      } else {
        // 64 packed bytes per row and quad: a warp's quads go to registers and
        // the chunk is released before they are converted and stored.
        const uint8_t *prow = chunk + r * 128;
        uint4 v4[4 * NQ];
#pragma unroll
        for (int t = 0; t < 4 * NQ; ++t) v4[t] = *reinterpret_cast<const uint4 *>(prow + (((4 * hq + t) ^ sw) << 4));
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&pk_empty[pi]);
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint4 q = v4[4 * qi + t];
            const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              col[8 * j + 2 * t] = wv[j] & 0x0F0F0F0Fu;
              col[8 * j + 2 * t + 1] = (wv[j] >> 4) & 0x0F0F0F0Fu;
            }
          }
          tmem_st_x32(acol + (uint32_t)(32 * (hq + qi)), col);
        }
      }
      tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&a_full[ls % NA]);
    }
  } else if (warp >= 16 && warp != 20) {  // ------------------------- drainers (TMEM lane = tile row)
    // Two groups of four warps (one per TMEM lane quarter) take the steps in
    // turn: group 1 hands its tile sums to group 0 through shared memory, and
    // group 0 adds them to its own (fixed order) and completes the tile.
    const int grp = warp > 20 ? 1 : 0;
    if (grp == 0) sm100::griddep_wait();  // outputs, partial slots and tickets may still be in use by the previous kernel
    const uint32_t pe = (PEER && grp == 0) ? peer_epoch(a.peer) : 0u;  // group 0 writes the outputs
    if (warp == 16 && lane == 0) s_peer_e = pe;
    const int qq = warp & 3;
    const int r = 32 * qq + lane;
    const uint32_t lane_base = (uint32_t)(32 * qq) << 16;
    float acc[MC];
    float *xch = reinterpret_cast<float *>(smem + L::kXchOff);
    // Completes the tile's output: directly when this CTA owns the whole K loop
    // of the tile, else through the head/tail partial slots and the tile's
    // ticket (the last contributor sums the slots in CTA order).
    auto flush = [&](int tile) {
      const bool aborted = *abort;
      if (aborted && a.nan_on_abort) {
#pragma unroll
        for (int c = 0; c < MC; ++c) acc[c] = __int_as_float(0x7fc00000);
      }
      const bool write = !aborted || a.nan_on_abort;
      const int n = tile * kI8Rows + r;
      const bool row_ok = n < a.w.rows;
      const int tg0 = tile * S, tg1 = tg0 + S;
      if (tg0 >= g0 && tg1 <= g1) {
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < MC; ++c)
            if (c < a.m) {
              const float v = EPI ? epilogue_out(acc[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : acc[c] + bias;
              a.y[(int64_t)c * a.ldy + n] = v;
              if constexpr (PEER) peer_store(a.peer, pe, c, n, v);
            }
        }
        return;
      }
      const int kind = (tile == g0 / S) ? 0 : 1;
      float *slot = a.partial + (((int64_t)cta * 2 + kind) * kI8Rows + r) * MC;
#pragma unroll
      for (int c = 0; c < MC; ++c) slot[c] = acc[c];
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int cf = dec_cta_of_step(tg0, GR, T), cl = dec_cta_of_step(tg1 - 1, GR, T);
      if (warp == 16 && lane == 0) s_last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        float tot[MC];
#pragma unroll
        for (int c = 0; c < MC; ++c) tot[c] = 0.0f;
        for (int cc = cf; cc <= cl; ++cc) {  // fixed CTA order: deterministic
          const int kk = (tile == dec_first_step(cc, GR, T) / S) ? 0 : 1;
          const float *ps = a.partial + (((int64_t)cc * 2 + kk) * kI8Rows + r) * MC;
#pragma unroll
          for (int c = 0; c < MC; ++c) tot[c] += __ldcg(ps + c);
        }
        if (write && row_ok) {
          const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
          for (int c = 0; c < MC; ++c)
            if (c < a.m) {
              const float v = EPI ? epilogue_out(tot[c] + bias, a.gate, a.resid, (int64_t)c * a.ldy + n) : tot[c] + bias;
              a.y[(int64_t)c * a.ldy + n] = v;
              if constexpr (PEER) peer_store(a.peer, pe, c, n, v);
            }
        }
        if (warp == 16 && lane == 0) a.tickets[tile] = 0;  // ready for the next launch
      }
      // the next tile's slot may reuse this CTA's slot only after s_last is read
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    // Every tile that the CTA's step range touches, in order; both groups visit
    // each one (a group may own no step of a short tile piece) and meet on
    // named barrier 2 at its end. The exchange buffer alternates between two
    // halves, so a group-1 write for the next tile cannot meet a group-0 read.
    const int tfirst = g0 / S, tlast = nsteps > 0 ? (g1 - 1) / S : tfirst - 1;
    for (int tile = tfirst; tile <= tlast; ++tile) {
      const int lo = max(g0, tile * S) - g0, hi = min(g1, (tile + 1) * S) - g0;
#pragma unroll
      for (int c = 0; c < MC; ++c) acc[c] = 0.0f;
      for (int ls = lo + ((lo & 1) != grp); ls < hi; ls += kI8DrainGroups) {
        const int di = ls % DS;
        // Failed waits do not leave the loop: every drainer must run the same
        // sequence of flushes (they synchronise on a named barrier).
        bool ok = sm100::mbar_wait_sleep(&dr_full[di], (uint32_t)(ls / DS) & 1u, a.err, abort, kI8WaitNs);
        ok = ok && sm100::mbar_wait_sleep(&done[ls % kI8Done], (uint32_t)(ls / kI8Done) & 1u, a.err, abort, kI8WaitNs);
        ok = __all_sync(0xffffffffu, ok);
        sm100::tc_fence_after();
        const uint8_t *dr = smem + L::kDrOff + di * L::kDrBytes;
        const uint4 dq = *reinterpret_cast<const uint4 *>(dr + r * 16);
        uint4 mq4 = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (QT == MQ_Q4_1) mq4 = *reinterpret_cast<const uint4 *>(dr + kI8Rows * 16 + r * 16);
        const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
        const uint32_t mw[4] = {mq4.x, mq4.y, mq4.z, mq4.w};
        const float *inv = reinterpret_cast<const float *>(dr + L::kDrHdr + kI8HdrInv);
        const int *sx = reinterpret_cast<const int *>(dr + L::kDrHdr + kI8HdrSx);
        const uint32_t dbase = tmem + lane_base + (uint32_t)(L::kDOff + (ls % ND) * L::kDCols);
        float st[MC];  // this step's sum
#pragma unroll
        for (int c = 0; c < MC; ++c) st[c] = 0.0f;
        constexpr int kRegions = 8 / L::G;
#pragma unroll
        for (int r0 = 0; r0 < kRegions; r0 += BB) {
          uint32_t v[BB * NCOL];
          if (ok) {
#pragma unroll
            for (int rb = 0; rb < BB; ++rb) tmem_ld_cols<NCOL>(dbase + (uint32_t)((r0 + rb) * kI8N), &v[rb * NCOL]);
            sm100::tmem_ld_wait();
          } else {
#pragma unroll
            for (int c = 0; c < BB * NCOL; ++c) v[c] = 0u;
          }
          if (r0 + BB == kRegions) {  // the D slot is released before the last batch's arithmetic
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&d_empty[ls % ND]);
          }
#pragma unroll
          for (int jb = 0; jb < BB * L::G; ++jb) {
            const int j = r0 * L::G + jb;
            const __half2 d2 = *reinterpret_cast<const __half2 *>(&dw[j >> 1]);
            const float d = (j & 1) ? __high2float(d2) : __low2float(d2);
            float mn = 0.0f;
            if constexpr (QT == MQ_Q4_1) {
              const __half2 m2 = *reinterpret_cast<const __half2 *>(&mw[j >> 1]);
              mn = (j & 1) ? __high2float(m2) : __low2float(m2);
            }
            const uint32_t *vb = &v[(jb / L::G) * NCOL + (jb % L::G) * L::kRowOff];
            float bis[MC];  // the block's 2^-e of every activation row: exact scaling
            if constexpr (MC >= 4) {
#pragma unroll
              for (int c = 0; c < MC; c += 4) {
                const float4 b4 = *reinterpret_cast<const float4 *>(inv + j * 8 + c);
                bis[c] = b4.x, bis[c + 1] = b4.y, bis[c + 2] = b4.z, bis[c + 3] = b4.w;
              }
            } else {
#pragma unroll
              for (int c = 0; c < MC; ++c) bis[c] = inv[j * 8 + c];
            }
#pragma unroll
            for (int c = 0; c < MC; ++c) {
              const int l0 = (int)vb[3 * c], l1 = (int)vb[3 * c + 1], l2 = (int)vb[3 * c + 2];
              const float bi = bis[c];
              if constexpr (QT == MQ_Q8_0) {
                const int v01 = l0 + (int)((uint32_t)l1 << 8);  // |.| < 2^27: exact
                st[c] = fmaf(d * fmaf((float)l2, 65536.0f, (float)v01), bi, st[c]);
              } else {
                // sum q * X fits int32, so the wrapping combination is exact.
                int vv = (int)((uint32_t)l0 + ((uint32_t)l1 << 8) + ((uint32_t)l2 << 16));
                if constexpr (QT == MQ_Q4_0) {
                  vv = (int)((uint32_t)vv - ((uint32_t)sx[j * 8 + c] << 3));
                  st[c] = fmaf(d * (float)vv, bi, st[c]);
                } else {
                  st[c] = fmaf(fmaf(d, (float)vv, mn * (float)sx[j * 8 + c]), bi, st[c]);
                }
              }
            }
          }
        }
#pragma unroll
        for (int c = 0; c < MC; ++c) acc[c] += st[c];
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&dr_empty[di]);
      }
      float *xb = xch + ((int64_t)((tile - tfirst) & 1) * kI8Rows + r) * MC;
      if (grp == 1) {
#pragma unroll
        for (int c = 0; c < MC; ++c) xb[c] = acc[c];
      }
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (grp == 0) {
#pragma unroll
        for (int c = 0; c < MC; ++c) acc[c] += xb[c];
        flush(tile);
      }
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
