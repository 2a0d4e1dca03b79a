// Peer-memory staging of the row-sharded linear's all-gather (mq_comm.cu),
// shared by the gather kernels and by the decode kernels that store their
// slice into the peers' staging themselves.
//
// Every rank owns a staging region, mapped by every peer through CUDA IPC:
//   data  [2 halves][G source ranks][kP2PSlotFloats] floats,
//   flags [2 halves][G] u32 (source rank p raised epoch e in half e & 1),
//   ctl   {epoch, push arrivals, pull arrivals, poisoned} u32.
// A call of epoch e (= ctl[0] + 1 when it starts) uses half e & 1. The source
// rank stores its [m, R] slice (row-major, row stride R) into slot (half,
// rank) of every peer, fences at system scope, and raises its flag in every
// peer with a release store; the pull kernel at each rank waits for the
// flags (acquire, bounded), copies the slots into its output and advances
// the epoch.
#pragma once

#include <cstdint>

namespace mq {

constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PSlotFloats = size_t(1) << 20;  // 4 MiB per slot: m * rows_per_rank <= 1,048,576

__host__ __device__ inline size_t p2p_data_bytes(int G) { return 2 * (size_t)G * kP2PSlotFloats * sizeof(float); }
__host__ __device__ inline size_t p2p_region_bytes(int G) { return p2p_data_bytes(G) + (2 * (size_t)G + 4) * 4; }

__device__ __forceinline__ uint32_t *p2p_flags(char *base, int G) {
  return reinterpret_cast<uint32_t *>(base + p2p_data_bytes(G));
}
__device__ __forceinline__ float *p2p_slot(char *base, int G, int half, int src) {
  return reinterpret_cast<float *>(base) + ((size_t)half * G + src) * kP2PSlotFloats;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The gather fused into a decode kernel (G <= 1: off): every output element
// (c, n) the kernel writes is also stored at [c * R + n] of slot (half, rank)
// of every peer; after the kernel's last CTA has seen every CTA's stores
// fenced at system scope, it raises this rank's flag in every peer.
struct PeerOut {
  int G = 0, rank = 0, R = 0;
  char *base[kP2PMaxRanks] = {};  // every rank's staging region as mapped here
};

// The call's epoch. Read after griddepcontrol.wait: the previous call's pull
// kernel, which advanced it, has completed.
__device__ __forceinline__ uint32_t peer_epoch(const PeerOut &p) {
  const uint32_t *ctl = p2p_flags(p.base[p.rank], p.G) + 2 * p.G;
  return *reinterpret_cast<const volatile uint32_t *>(&ctl[0]) + 1u;
}

__device__ __forceinline__ void peer_store(const PeerOut &p, uint32_t e, int c, int n, float v) {
  const int half = (int)(e & 1u);
  for (int q = 0; q < p.G; ++q)
    if (q != p.rank) p2p_slot(p.base[q], p.G, half, p.rank)[(size_t)c * p.R + n] = v;
}

// Called by every thread of every CTA after its last output store (the
// caller synchronises the CTA first).
__device__ __forceinline__ void peer_finish(const PeerOut &p, uint32_t e) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t *ctl = p2p_flags(p.base[p.rank], p.G) + 2 * p.G;
    if (atomicAdd(&ctl[1], 1u) == gridDim.x - 1) {  // every CTA's stores are fenced
      __threadfence_system();
      for (int q = 0; q < p.G; ++q)
        if (q != p.rank) st_release_sys(p2p_flags(p.base[q], p.G) + (e & 1u) * p.G + p.rank, e);
      ctl[1] = 0u;
    }
  }
}

}  // namespace mq
