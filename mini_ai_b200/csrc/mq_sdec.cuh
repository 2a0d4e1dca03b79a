// Stream-K SIMT decode GEMV for one to four activation rows.
//
// y[i, n] = sum_b d[n,b] * sum_{k<32} (q[n,b,k] - zp) * x[i, 32b + k]  (+ m[n,b] * sum_k x[i, 32b + k]) + bias[n]
//
// With M <= 4 the arithmetic per weight is small enough for the SIMT lanes
// (decode about 2 instructions per weight, M/2 packed fp32 FMAs), so the
// kernel is a pure HBM stream: a persistent CTA per SM walks a contiguous
// range of the tile-major (128-row tile, 8-block step) space, exactly like the
// tcgen05 decode GEMM, with one producer thread keeping a deep ring of steps
// in flight. A stage holds the step's weight chunk (packed quant rows, 128-byte
// swizzle pre-applied, fp16 scales, Q4_1 mins: one linear bulk copy of
// consecutive memory) and the fp32 activations of the step's 256 K, loaded by
// TMA straight from x (no split kernel, no extra launch). Launched with
// programmatic stream serialization: the weight stream starts while the
// previous kernel finishes; activations, outputs and workspace are touched
// only after griddepcontrol.wait.
//
// Compute: thread = weight row of the tile. The 16 compute warps are 4 row
// quarters x 4 block pairs: warp w owns rows 32(w%4).. and blocks
// 2(w/4), 2(w/4)+1 of every step. All 32 lanes of a warp read the same
// activations, so every activation load is a shared-memory broadcast; packed
// bytes come from the swizzled rows without bank conflicts beyond 2-way.
// Decoding splices a nibble or byte under the exponent of 2^23 and subtracts
// 2^23 + zp with a packed fp32 add; packed fp32 FMAs accumulate per block and
// the block scale is applied once per block. At the end of a tile the four
// block-pair partials of a row are summed in a fixed order and completed like
// the decode GEMM: directly, or through per-CTA partial slots and the tile's
// ticket (deterministic CTA order).
//
// Reference semantics: QuantizedDotRow, src/quantized_tensor.cc:161-191, and
// LinearKernel's fused bias, src/cuda_backend.cu:94-110.
#pragma once

#include <cuda.h>

#include "mq_common.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec.cuh"

namespace mq {

// 2^23 + zero point: subtracting it from a code spliced under the exponent of
// 2^23 (byte_perm) yields q - zp exactly.
template <int QT> struct Zp;
template <> struct Zp<MQ_Q4_0> { static constexpr float kMagic = 8388616.0f; };  // 2^23 + 8
template <> struct Zp<MQ_Q4_1> { static constexpr float kMagic = 8388608.0f; };  // 2^23
template <> struct Zp<MQ_Q8_0> { static constexpr float kMagic = 8388736.0f; };  // 2^23 + 128 (after ^0x80)

// Bytes a and b of v, each spliced under 2^23, minus the magic: two exact floats.
template <int QT>
__device__ __forceinline__ float2 decode_pair(uint32_t v, int a, int b) {
  const float2 f = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)a)),
                               __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (unsigned)b)));
  return __fadd2_rn(f, make_float2(-Zp<QT>::kMagic, -Zp<QT>::kMagic));
}

constexpr int kSdRows = 128;
constexpr int kSdComputeWarps = 16;
constexpr int kSdThreads = (kSdComputeWarps + 1) * 32;  // + warp 16: TMA producer
constexpr int kSdBlocksPerStep = 8;
constexpr uint64_t kSdWaitNs = 1000000000ull;
constexpr uint64_t kSdDrainNs = 20000000ull;

struct SdecArgs {
  WeightView w;
  int m;              // activation rows (<= MC)
  const float *bias;
  float *y;
  int64_t ldy;
  float *partial;     // [gridDim.x][2][128][MC]: head / tail partial tile of every CTA
  int *tickets;       // [tiles], zero between launches
  int steps;          // 8-block steps per tile (the K loop)
  int tiles;
  int *err;
  int nan_on_abort;
  const float *gate = nullptr;   // fused gate/up product: y = silu(gate) * (product + bias); gate [m, ldy]
  const float *resid = nullptr;  // residual add: y = resid + (product + bias); resid [m, ldy], may be y
};

template <int QT, int MC>
struct SdCfg {
  // Two CTAs per SM (more warps, half the ring each) measured slower than
  // one CTA with the deeper ring: one per SM.
  static constexpr int kCtasPerSm = 1;
  static constexpr int kPkBytes = step_pk_bytes(QT);
  static constexpr int kScBytes = step_sc_bytes(QT);
  static constexpr int kXBytes = MC * 256 * 4;
  static constexpr int kStage = kPkBytes + kScBytes + kXBytes;
  static constexpr int kBudget = (kCtasPerSm == 2 ? 104 : 200) * 1024;
  static constexpr int ST = (kBudget / kStage) < 8 ? (kBudget / kStage) : 8;  // ring depth
  static constexpr int kRedOff = ST * kStage;                                       // [4][128][MC] floats
  static constexpr int kBarOff = kRedOff + 4 * kSdRows * MC * 4;
  static constexpr int kBytes = kBarOff + 16 * ST + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(ST >= 3 && kAlloc <= 227 * 1024, "shared memory budget");
  static_assert(kPkBytes % 1024 == 0 && kScBytes % 1024 == 0 && kXBytes % 1024 == 0, "1 KB aligned stage parts");
};

template <int QT, int MC>
__global__ void __launch_bounds__(kSdThreads, SdCfg<QT, MC>::kCtasPerSm)
    sdec_kernel(const __grid_constant__ CUtensorMap tm_x, const SdecArgs a) {
  using L = SdCfg<QT, MC>;
  constexpr int ST = L::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOff), *empty = full + ST;
  volatile int *abort = reinterpret_cast<volatile int *>(empty + ST);
  float *red = reinterpret_cast<float *>(smem + L::kRedOff);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.steps, T = a.tiles * a.steps, GR = gridDim.x, cta = blockIdx.x;
  const int g0 = dec_first_step(cta, GR, T), g1 = dec_first_step(cta + 1, GR, T);
  const int nsteps = g1 - g0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) sm100::mbar_init(&full[i], 1), sm100::mbar_init(&empty[i], kSdComputeWarps);
    *abort = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();

  if (threadIdx.x == 0) sm100::griddep_launch_dependents();
  if (warp == kSdComputeWarps) {  // ------------------------- producer: one stage per step
    if (lane == 0) {
      sm100::prefetch_tmap(&tm_x);
      // The weights are read-only: the first ring's worth streams in while
      // the previous kernel of the stream (which may produce x) finishes.
      const int pre = nsteps < ST ? nsteps : ST;
      for (int ls = 0; ls < pre; ++ls) {
        const int g = g0 + ls;
        sm100::mbar_arrive_expect_tx(&full[ls], L::kStage);
        sm100::bulk_load(smem + ls * L::kStage, chunk_ptr(a.w, g / S, g % S), L::kPkBytes + L::kScBytes, &full[ls]);
      }
      sm100::griddep_wait();
      for (int ls = 0; ls < pre; ++ls)
        sm100::tma_load_2d(smem + ls * L::kStage + L::kPkBytes + L::kScBytes, &tm_x, ((g0 + ls) % S) * 256, 0,
                           &full[ls]);
      int issued = pre;
      for (int ls = pre; ls < nsteps; ++ls) {
        const int i = ls % ST;
        if (!sm100::mbar_wait_sleep(&empty[i], ((uint32_t)(ls / ST) & 1u) ^ 1u, a.err, abort, kSdWaitNs)) break;
        const int g = g0 + ls, k = g % S;
        uint8_t *st = smem + i * L::kStage;
        sm100::mbar_arrive_expect_tx(&full[i], L::kStage);
        // the step's weight chunk (packed rows + scales + mins) in one linear copy
        sm100::bulk_load(st, chunk_ptr(a.w, g / S, k), L::kPkBytes + L::kScBytes, &full[i]);
        sm100::tma_load_2d(st + L::kPkBytes + L::kScBytes, &tm_x, k * 256, 0, &full[i]);
        issued = ls + 1;
      }
      for (int p = issued - ST < 0 ? 0 : issued - ST; p < issued; ++p)
        sm100::mbar_wait(&full[p % ST], (uint32_t)(p / ST) & 1u, nullptr, nullptr, kSdDrainNs);
    }
  } else {  // ------------------------------------------------ compute: thread = row, warp = (quarter, block pair)
    sm100::griddep_wait();  // y, partial slots and tickets may still be in use by the previous kernel
    const int rq = warp & 3, bp = warp >> 2;
    const int r = 32 * rq + lane, sw = r & 7;
    const int qd = bp >> 1, j0 = 2 * (bp & 1);  // quad of the step, first block of the pair inside it
    float acc[MC];
#pragma unroll
    for (int i = 0; i < MC; ++i) acc[i] = 0.0f;
    int cur = -1;

    // Sums the four block-pair partials of each row (fixed order) and
    // completes the tile: directly, or through the partial slots + ticket.
    auto flush = [&](int tile) {
#pragma unroll
      for (int i = 0; i < MC; ++i) red[(bp * kSdRows + r) * MC + i] = acc[i];
      asm volatile("bar.sync 1, 512;" ::: "memory");
      if (bp == 0) {
        float tot[MC];
#pragma unroll
        for (int i = 0; i < MC; ++i)
          tot[i] = ((red[(0 * kSdRows + r) * MC + i] + red[(1 * kSdRows + r) * MC + i]) +
                    red[(2 * kSdRows + r) * MC + i]) + red[(3 * kSdRows + r) * MC + i];
        const bool aborted = *abort;
        if (aborted && a.nan_on_abort) {
#pragma unroll
          for (int i = 0; i < MC; ++i) tot[i] = __int_as_float(0x7fc00000);
        }
        const bool write = !aborted || a.nan_on_abort;
        const int n = tile * kSdRows + r;
        const bool row_ok = n < a.w.rows;
        const int tg0 = tile * S, tg1 = tg0 + S;
        if (tg0 >= g0 && tg1 <= g1) {
          if (write && row_ok) {
            const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
            for (int i = 0; i < MC; ++i)
              if (i < a.m) a.y[(int64_t)i * a.ldy + n] = epilogue_out(tot[i] + bias, a.gate, a.resid, (int64_t)i * a.ldy + n);
          }
        } else {
          const int kind = (tile == g0 / S) ? 0 : 1;
          float *slot = a.partial + (((int64_t)cta * 2 + kind) * kSdRows + r) * MC;
#pragma unroll
          for (int i = 0; i < MC; ++i) slot[i] = tot[i];
          __threadfence();
          asm volatile("bar.sync 2, 128;" ::: "memory");
          const int cf = dec_cta_of_step(tg0, GR, T), cl = dec_cta_of_step(tg1 - 1, GR, T);
          if (r == 0) s_last = atomicAdd(&a.tickets[tile], 1) == cl - cf;
          asm volatile("bar.sync 2, 128;" ::: "memory");
          if (s_last) {
            __threadfence();
            float sum[MC];
#pragma unroll
            for (int i = 0; i < MC; ++i) sum[i] = 0.0f;
            for (int cc = cf; cc <= cl; ++cc) {  // fixed CTA order: deterministic
              const int kk = (tile == dec_first_step(cc, GR, T) / S) ? 0 : 1;
              const float *ps = a.partial + (((int64_t)cc * 2 + kk) * kSdRows + r) * MC;
#pragma unroll
              for (int i = 0; i < MC; ++i) sum[i] += __ldcg(ps + i);
            }
            if (write && row_ok) {
              const float bias = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
              for (int i = 0; i < MC; ++i)
                if (i < a.m) a.y[(int64_t)i * a.ldy + n] = epilogue_out(sum[i] + bias, a.gate, a.resid, (int64_t)i * a.ldy + n);
            }
            if (r == 0) a.tickets[tile] = 0;  // ready for the next launch
          }
          asm volatile("bar.sync 2, 128;" ::: "memory");
        }
      }
      // red and the partial slots are reused by the next tile only after this
      asm volatile("bar.sync 1, 512;" ::: "memory");
    };

    for (int ls = 0; ls < nsteps; ++ls) {
      const int g = g0 + ls, tile = g / S;
      if (tile != cur) {
        if (cur >= 0) flush(cur);
        cur = tile;
#pragma unroll
        for (int i = 0; i < MC; ++i) acc[i] = 0.0f;
      }
      const int si = ls % ST;
      // A failed wait keeps the loop shape (the flushes synchronise on named
      // barriers) and contributes nothing.
      const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait_sleep(&full[si], (uint32_t)(ls / ST) & 1u, a.err,
                                                                      abort, kSdWaitNs));
      if (ok) {
        const uint8_t *st = smem + si * L::kStage;
        const uint8_t *sc = st + L::kPkBytes + r * 16;
        const float *xs = reinterpret_cast<const float *>(st + L::kPkBytes + L::kScBytes);
        const uint32_t dword = *reinterpret_cast<const uint32_t *>(sc + 4 * bp);  // d of blocks 2bp, 2bp+1
        const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&dword));
        float2 mm = make_float2(0.0f, 0.0f);
        if constexpr (QT == MQ_Q4_1) {
          const uint32_t mword = *reinterpret_cast<const uint32_t *>(sc + kSdRows * 16 + 4 * bp);
          mm = __half22float2(*reinterpret_cast<const __half2 *>(&mword));
        }
        // Packed words of the two blocks: wq[t][e] = word of block j0 + e in 16-byte chunk t of the quad.
        uint32_t wq[4][2];
        if constexpr (QT == MQ_Q8_0) {
          const uint8_t *prow = st + qd * (kSdRows * 128) + r * 128;
          uint32_t w8[4][4];  // [t][block e: words 0,1]
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint4 c = *reinterpret_cast<const uint4 *>(prow + (((2 * t + (j0 >> 1)) ^ sw) << 4));
            w8[t][0] = c.x, w8[t][1] = c.y, w8[t][2] = c.z, w8[t][3] = c.w;
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float2 part[MC];
#pragma unroll
            for (int i = 0; i < MC; ++i) part[i] = make_float2(0.0f, 0.0f);
            const int jb = 2 * bp + e;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint32_t u0 = w8[t][2 * e] ^ 0x80808080u, u1 = w8[t][2 * e + 1] ^ 0x80808080u;
              const float2 v0 = decode_pair<QT>(u0, 0, 1), v1 = decode_pair<QT>(u0, 2, 3);
              const float2 v2 = decode_pair<QT>(u1, 0, 1), v3 = decode_pair<QT>(u1, 2, 3);
#pragma unroll
              for (int i = 0; i < MC; ++i) {
                const float *xb = xs + i * 256 + 32 * jb + 2 * t;
                part[i] = __ffma2_rn(v0, *reinterpret_cast<const float2 *>(xb), part[i]);
                part[i] = __ffma2_rn(v1, *reinterpret_cast<const float2 *>(xb + 8), part[i]);
                part[i] = __ffma2_rn(v2, *reinterpret_cast<const float2 *>(xb + 16), part[i]);
                part[i] = __ffma2_rn(v3, *reinterpret_cast<const float2 *>(xb + 24), part[i]);
              }
            }
            const float d = e ? dd.y : dd.x;
#pragma unroll
            for (int i = 0; i < MC; ++i) acc[i] = fmaf(d, part[i].x + part[i].y, acc[i]);
          }
          (void)wq;
        } else {
          const uint8_t *prow = st + r * 128;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint2 c = *reinterpret_cast<const uint2 *>(prow + (((4 * qd + t) ^ sw) << 4) + 4 * j0);
            wq[t][0] = c.x, wq[t][1] = c.y;
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jb = 2 * bp + e;
            float2 part[MC];
#pragma unroll
            for (int i = 0; i < MC; ++i) part[i] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int th = 0; th < 2; ++th) {  // t pairs (0,1), (2,3): x float4 c = th, th+2, th+4, th+6
              float4 x4[MC][4];
#pragma unroll
              for (int i = 0; i < MC; ++i)
#pragma unroll
                for (int u = 0; u < 4; ++u)
                  x4[i][u] = *reinterpret_cast<const float4 *>(xs + i * 256 + 32 * jb + 4 * (th + 2 * u));
#pragma unroll
              for (int tt = 0; tt < 2; ++tt) {
                const int t = 2 * th + tt;
                const uint32_t wd = wq[t][e];
                const uint32_t lo = wd & 0x0F0F0F0Fu, hi = (wd >> 4) & 0x0F0F0F0Fu;
                const float2 v0 = decode_pair<QT>(lo, 0, 2);  // k 2t, 2t+1
                const float2 v1 = decode_pair<QT>(lo, 1, 3);  // k 2t+8, 2t+9
                const float2 v2 = decode_pair<QT>(hi, 0, 2);  // k 2t+16, 2t+17
                const float2 v3 = decode_pair<QT>(hi, 1, 3);  // k 2t+24, 2t+25
#pragma unroll
                for (int i = 0; i < MC; ++i) {
                  const float2 xa = tt ? make_float2(x4[i][0].z, x4[i][0].w) : make_float2(x4[i][0].x, x4[i][0].y);
                  const float2 xb = tt ? make_float2(x4[i][1].z, x4[i][1].w) : make_float2(x4[i][1].x, x4[i][1].y);
                  const float2 xc = tt ? make_float2(x4[i][2].z, x4[i][2].w) : make_float2(x4[i][2].x, x4[i][2].y);
                  const float2 xd = tt ? make_float2(x4[i][3].z, x4[i][3].w) : make_float2(x4[i][3].x, x4[i][3].y);
                  part[i] = __ffma2_rn(v0, xa, part[i]);
                  part[i] = __ffma2_rn(v1, xb, part[i]);
                  part[i] = __ffma2_rn(v2, xc, part[i]);
                  part[i] = __ffma2_rn(v3, xd, part[i]);
                }
              }
            }
            const float d = e ? dd.y : dd.x;
#pragma unroll
            for (int i = 0; i < MC; ++i) acc[i] = fmaf(d, part[i].x + part[i].y, acc[i]);
          }
        }
        if constexpr (QT == MQ_Q4_1) {  // + m_b * sum_k x: block sums shared by the warp (all lanes, same blocks)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jb = 2 * bp + e;
#pragma unroll
            for (int i = 0; i < MC; ++i) {
              float s = xs[i * 256 + 32 * jb + lane];
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
              acc[i] = fmaf(e ? mm.y : mm.x, s, acc[i]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[si]);
    }
    if (cur >= 0) flush(cur);
  }
}

}  // namespace mq
