// Row-sharded linear with an all-gather of the output slices over NVLink.
//
// A projection too large for one GPU (or worth splitting for bandwidth) is
// split by output rows: rank r of G holds rows [r*R, (r+1)*R) as its own
// mq_weight (mq_weight_shard_create). Rows are independent (y_n = <W_n, x>),
// so each rank computes its R outputs with the ordinary decode/prefill
// kernels and one all-gather over NVLink assembles y [m, G*R] on every rank.
// Each rank runs the kernels of mq_linear on its rows. The decode and prefill
// kernels split every tile's K range across CTAs according to the launch's
// total work, so a shard's split, and with it the fp32 summation order, can
// differ from the whole weight's: the gathered result then matches mq_linear
// on the whole weight to fp32 rounding (both within the oracle's bound), and
// is bit-identical where the two launches split K alike (for instance when
// neither has more (tile, K step) chunks than CTAs, as in the tests).
//
// The gather runs over peer memory: at communicator creation every rank
// allocates a staging region ([2 halves][nranks slots][kP2PSlotFloats] floats,
// then [2][nranks] arrival flags and three local counters), and the ranks
// exchange CUDA IPC handles for it (through NCCL) and map each other's
// regions. Per call, after the rank's decode kernel has written its slice into
// its own output, a push kernel stores the slice into every peer's slot of the
// current half and, once all its CTAs' stores are fenced at system scope,
// raises this rank's flag in every peer's region (release store); a pull
// kernel waits (bounded, 1 s) for every peer's flag (acquire load) and copies
// the peers' slices from the local staging into the output. The epoch (and
// with it the half) lives in device memory and is advanced by the pull
// kernel, so a CUDA graph that captured these launches replays correctly.
// A rank can be at most one call ahead of a peer (its next push waits for the
// peer's flags of the current call), so two halves are enough. A peer that
// does not arrive within the wait limit (MQ_P2P_WAIT_NS, default 1 s) poisons
// the communicator: the pull writes NaN into the missing columns, raises the
// communicator's error flag, and from then on every peer-memory gather of
// this communicator fails with MQ_ERR_TIMEOUT at once (replays of a captured
// graph write NaN without waiting); the epoch no longer matters. Outputs larger
// than a slot, communicators whose ranks could not all map each other's
// regions, and processes without MQ_P2P_GATHER=1 use NCCL's all-gather.
//
// NCCL is loaded at the first mq_comm call with dlopen("libnccl.so.2"), so
// the library has no link-time dependency on it and, inside a PyTorch
// process, shares the NCCL that torch already loaded.
#include <dlfcn.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "mq_common.cuh"
#include "mq_peer.cuh"
#include "mq_sm100.cuh"
#include "mq_tcdec_api.h"

#include "nccl.h"

namespace mq {
int gather_workspace_for(int device, cudaStream_t s, size_t bytes, void **out);
void count_launch(int n);

constexpr uint64_t kP2PWaitNs = 1000000000ull;  // default wait limit for a peer's arrival flag
}  // namespace mq

struct mq_comm {
  int device = 0, nranks = 1, rank = 0;
  ncclComm_t comm = nullptr;
  bool p2p = false;                           // peer-memory gather set up on every rank
  char *stage = nullptr;                      // this rank's staging region
  char *peer[mq::kP2PMaxRanks] = {nullptr};   // every rank's region as mapped here (own at [rank])
  uint64_t wait_ns = mq::kP2PWaitNs;           // bound of the pull kernel's wait for a peer
  int *err_host = nullptr, *err_dev = nullptr;  // mapped flag: a peer gather of this communicator timed out
  bool poisoned = false;                       // a timeout was reported: peer gathers fail from then on
};

namespace mq {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = {0};
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "libnccl.so.2 not loadable: %s", dlerror());
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.error_string;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks a required symbol");
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char *what) {
  return fail(MQ_ERR_CUDA, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// y[i, r*R + j] = g[r][i][j]: the rank-major gather buffer into row-major outputs.
__global__ void interleave_kernel(const float *__restrict__ g, int nranks, int m, int R, float *__restrict__ y,
                                  int64_t ldy) {
  const int64_t n = (int64_t)nranks * m * R;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % R);
    const int64_t t = e / R;
    const int i = (int)(t % m), r = (int)(t / m);
    y[(int64_t)i * ldy + (int64_t)r * R + j] = g[e];
  }
}

// Byte layout of a staging region: mq_peer.cuh.

struct P2PArgs {
  float *y;          // the output [m, ldy]; this rank's slice at column rank * R
  int64_t ldy;
  int m, R, G, rank;
  char *base[kP2PMaxRanks];
  int *err;          // the communicator's host-mapped timeout flag
  uint64_t wait_ns;  // bound of the wait for a peer's flag
};


// This rank's slice [m, R] (row stride ldy) -> slot (half, rank) of every peer.
template <bool VEC>
__global__ void __launch_bounds__(256) p2p_push_kernel(const P2PArgs a) {
  sm100::griddep_wait();  // the slice is the previous kernel's output
  uint32_t *ctl = p2p_flags(a.base[a.rank], a.G) + 2 * a.G;
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(&ctl[0]) + 1u;
  const int half = (int)(e & 1u);
  const float *src = a.y + (int64_t)a.rank * a.R;
  const int64_t n = (int64_t)a.m * a.R;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int pp = 1; pp < a.G; ++pp) {
    const int p = (a.rank + pp) % a.G;  // spread the peers' links over the CTAs' start order
    float *dst = p2p_slot(a.base[p], a.G, half, a.rank);
    if constexpr (VEC) {
      const int rq = a.R / 4;
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += stride) {
        const int64_t c = i / rq, j = i % rq;
        reinterpret_cast<float4 *>(dst)[i] = __ldcg(reinterpret_cast<const float4 *>(src + c * a.ldy + 4 * j));
      }
    } else {
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __ldcg(src + (i / a.R) * a.ldy + i % a.R);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&ctl[1], 1u) == gridDim.x - 1) {  // every CTA's stores are fenced
    __threadfence_system();
    for (int p = 0; p < a.G; ++p)
      if (p != a.rank) st_release_sys(p2p_flags(a.base[p], a.G) + half * a.G + a.rank, e);
    ctl[1] = 0u;
  }
}

// Waits for every peer's slice of this epoch, then copies the peers' slots
// into their columns of the output; the last CTA advances the epoch. A wait
// that runs out (or a communicator poisoned by an earlier one) writes NaN
// into the peers' columns instead and raises the error flag.
template <bool VEC>
__global__ void __launch_bounds__(256) p2p_pull_kernel(const P2PArgs a) {
  __shared__ int s_ok;
  // The previous kernel (push, or the decode kernel that pushed its slice
  // itself) reads the epoch this kernel advances: it must have completed.
  sm100::griddep_wait();
  char *mine = a.base[a.rank];
  uint32_t *flags = p2p_flags(mine, a.G);
  uint32_t *ctl = flags + 2 * a.G;
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(&ctl[0]) + 1u;
  const int half = (int)(e & 1u);
  if (threadIdx.x == 0) {
    int ok = *reinterpret_cast<volatile uint32_t *>(&ctl[3]) == 0u;
    const uint64_t t0 = sm100::globaltimer_ns();
    for (int p = 0; p < a.G && ok; ++p) {
      if (p == a.rank) continue;
      for (uint32_t it = 0; ld_acquire_sys(flags + half * a.G + p) != e; ++it) {
        if ((it & 63u) == 63u && (sm100::globaltimer_ns() - t0 > a.wait_ns ||
                                  *reinterpret_cast<volatile uint32_t *>(&ctl[3]) != 0u)) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) {
      atomicExch(reinterpret_cast<unsigned int *>(&ctl[3]), 1u);
      atomicExch(a.err, 1);
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) {
    const int64_t n = (int64_t)a.m * a.R;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int p = 0; p < a.G; ++p) {
      if (p == a.rank) continue;
      float *dst = a.y + (int64_t)p * a.R;
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[(i / a.R) * a.ldy + i % a.R] = __int_as_float(0x7fc00000);
    }
  } else {
    const int64_t n = (int64_t)a.m * a.R;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int p = 0; p < a.G; ++p) {
      if (p == a.rank) continue;
      const float *slot = p2p_slot(mine, a.G, half, p);
      float *dst = a.y + (int64_t)p * a.R;
      if constexpr (VEC) {
        const int rq = a.R / 4;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += stride) {
          const int64_t c = i / rq, j = i % rq;
          *reinterpret_cast<float4 *>(dst + c * a.ldy + 4 * j) = __ldcg(reinterpret_cast<const float4 *>(slot) + i);
        }
      } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
          dst[(i / a.R) * a.ldy + i % a.R] = __ldcg(slot + i);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&ctl[2], 1u) == gridDim.x - 1) {
      ctl[2] = 0u;
      ctl[0] = e;  // the next call's epoch; the next kernels on the stream see it
      __threadfence();
    }
  }
}

// Device buffers and stream of the set-up exchanges, allocated before the
// rank joins the NCCL communicator, so that every rank that reaches an
// exchange has valid buffers (a rank that could not allocate them fails
// mq_comm_create before joining instead of leaving its peers waiting in a
// collective it cannot take part in).
struct P2PExchange {
  void *buf = nullptr;  // [G] records, then [G] agreement flags
  cudaStream_t s = nullptr;
  void release() {
    if (s) cudaStreamDestroy(s);
    if (buf) cudaFree(buf);
    s = nullptr;
    buf = nullptr;
  }
};

struct P2PRec {
  int ok;
  int pad[3];
  cudaIpcMemHandle_t h;
};

bool p2p_wanted(int G) {
  if (G < 2 || G > kP2PMaxRanks) return false;
  const char *env = std::getenv("MQ_P2P_GATHER");  // opt-in: MQ_P2P_GATHER=1
  return env && env[0] == '1';
}

cudaError_t p2p_exchange_alloc(int G, P2PExchange *x) {
  cudaError_t e = cudaMalloc(&x->buf, (sizeof(P2PRec) + sizeof(int)) * G);
  if (e == cudaSuccess) e = cudaStreamCreate(&x->s);
  if (e != cudaSuccess) x->release();
  return e;
}

// Maps every rank's staging region on every rank; false (and nothing held)
// unless all ranks succeeded. `x` holds the exchange buffers (allocated before
// the communicator was joined).
bool p2p_setup(mq_comm *c, P2PExchange &x) {
  const int G = c->nranks;
  const size_t bytes = p2p_region_bytes(G);
  bool ok = cudaMalloc(&c->stage, bytes) == cudaSuccess;
  ok = ok && cudaMemset(c->stage, 0, bytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  ok = ok && cudaHostAlloc(&c->err_host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess;
  if (ok) {
    *c->err_host = 0;
    ok = cudaHostGetDevicePointer(&c->err_dev, c->err_host, 0) == cudaSuccess;
  }
  // Exchange {ok, handle} records over NCCL (in place: every rank sends its own record).
  P2PRec mine{};
  mine.ok = ok && cudaIpcGetMemHandle(&mine.h, c->stage) == cudaSuccess;
  P2PRec *d_recs = static_cast<P2PRec *>(x.buf);
  P2PRec recs[kP2PMaxRanks];
  bool ex = cudaMemcpy(d_recs + c->rank, &mine, sizeof(P2PRec), cudaMemcpyHostToDevice) == cudaSuccess;
  // Every rank takes part in the exchange, whatever its own state, so that no rank waits alone.
  const ncclResult_t nr = nccl().all_gather(d_recs + c->rank, d_recs, sizeof(P2PRec), ncclUint8, c->comm, x.s);
  ex = ex && nr == ncclSuccess && cudaStreamSynchronize(x.s) == cudaSuccess &&
       cudaMemcpy(recs, d_recs, sizeof(P2PRec) * G, cudaMemcpyDeviceToHost) == cudaSuccess;
  bool all = ex;
  for (int p = 0; all && p < G; ++p) all = recs[p].ok != 0;
  if (all) {
    for (int p = 0; p < G; ++p) {
      if (p == c->rank) {
        c->peer[p] = c->stage;
        continue;
      }
      void *q = nullptr;
      if (cudaIpcOpenMemHandle(&q, recs[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        all = false;
        break;
      }
      c->peer[p] = static_cast<char *>(q);
    }
  }
  // Agree that every rank mapped every peer (a second exchange of one flag each).
  int *d_ok = reinterpret_cast<int *>(static_cast<char *>(x.buf) + sizeof(P2PRec) * G);
  int oks[kP2PMaxRanks] = {0};
  const int my_ok = all ? 1 : 0;
  bool ex2 = cudaMemcpy(d_ok + c->rank, &my_ok, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess;
  const ncclResult_t nr2 = nccl().all_gather(d_ok + c->rank, d_ok, 1, ncclInt32, c->comm, x.s);
  ex2 = ex2 && nr2 == ncclSuccess && cudaStreamSynchronize(x.s) == cudaSuccess &&
        cudaMemcpy(oks, d_ok, sizeof(int) * G, cudaMemcpyDeviceToHost) == cudaSuccess;
  bool agreed = ex2;
  for (int p = 0; agreed && p < G; ++p) agreed = oks[p] != 0;
  if (!agreed) {
    for (int p = 0; p < G; ++p)
      if (p != c->rank && c->peer[p]) cudaIpcCloseMemHandle(c->peer[p]);
    for (int p = 0; p < G; ++p) c->peer[p] = nullptr;
    if (c->stage) cudaFree(c->stage);
    c->stage = nullptr;
    if (c->err_host) cudaFreeHost(c->err_host);
    c->err_host = c->err_dev = nullptr;
    cudaGetLastError();  // the fallback is NCCL: clear a failed call's error state
    return false;
  }
  const char *w = std::getenv("MQ_P2P_WAIT_NS");
  if (w && *w) {
    const long long v = std::atoll(w);
    if (v > 0) c->wait_ns = (uint64_t)v;
  }
  return true;
}

void p2p_release(mq_comm *c) {
  if (!c->p2p) return;
  for (int p = 0; p < c->nranks; ++p)
    if (p != c->rank && c->peer[p]) cudaIpcCloseMemHandle(c->peer[p]);
  if (c->stage) cudaFree(c->stage);
  if (c->err_host) cudaFreeHost(c->err_host);
  c->err_host = c->err_dev = nullptr;
  c->p2p = false;
}

// Launches the push kernel with programmatic stream serialization (it starts
// while the decode kernel runs and waits for it with griddepcontrol.wait).
template <bool VEC>
cudaError_t p2p_launch(const P2PArgs &a, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, p2p_push_kernel<VEC>, a);
  if (e != cudaSuccess) return e;
  p2p_pull_kernel<VEC><<<grid, 256, 0, s>>>(a);
  count_launch(2);
  return cudaGetLastError();
}

// The pull alone: the decode kernel already stored this rank's slice into
// the peers' staging and raised the flags.
template <bool VEC>
cudaError_t p2p_pull_launch(const P2PArgs &a, int grid, cudaStream_t s) {
  p2p_pull_kernel<VEC><<<grid, 256, 0, s>>>(a);
  count_launch(1);
  return cudaGetLastError();
}

// MQ_P2P_FUSED=0 keeps the separate push kernel after the decode kernel.
bool p2p_fused() {
  static const bool on = [] {
    const char *v = std::getenv("MQ_P2P_FUSED");
    return !(v && *v && std::atoi(v) == 0);
  }();
  return on;
}

}  // namespace
}  // namespace mq

extern "C" {

int mq_comm_unique_id(void *id, size_t len) {
  using namespace mq;
  if (!id || len < NCCL_UNIQUE_ID_BYTES) return fail(MQ_ERR_INVALID, "unique id buffer must hold %d bytes", NCCL_UNIQUE_ID_BYTES);
  if (!nccl().ok) return fail(MQ_ERR_UNSUPPORTED, "%s", nccl().why);
  ncclUniqueId u;
  const ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return MQ_OK;
}

int mq_comm_create(int device, int nranks, int rank, const void *id, size_t len, mq_comm **out) {
  using namespace mq;
  if (!out || !id) return fail(MQ_ERR_INVALID, "null pointer");
  *out = nullptr;
  if (len != NCCL_UNIQUE_ID_BYTES) return fail(MQ_ERR_INVALID, "unique id must be %d bytes", NCCL_UNIQUE_ID_BYTES);
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MQ_ERR_INVALID, "rank %d of %d", rank, nranks);
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= count) return fail(MQ_ERR_INVALID, "CUDA device id %d out of range", device);
  if (!nccl().ok) return fail(MQ_ERR_UNSUPPORTED, "%s", nccl().why);
  int prev = -1;
  if ((e = cudaGetDevice(&prev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  P2PExchange xch;
  const bool want_p2p = p2p_wanted(nranks);
  if (want_p2p && (e = p2p_exchange_alloc(nranks, &xch)) != cudaSuccess) {
    cudaSetDevice(prev);
    return cuda_fail(e, "peer-gather exchange buffers (before joining the communicator)");
  }
  ncclUniqueId u;
  memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nccl().comm_init_rank(&comm, nranks, u, rank);
  if (r != ncclSuccess) {
    xch.release();
    cudaSetDevice(prev);
    return nccl_fail(r, "ncclCommInitRank");
  }
  auto *c = new (std::nothrow) mq_comm;
  if (!c) {
    xch.release();
    nccl().comm_destroy(comm);
    cudaSetDevice(prev);
    return fail(MQ_ERR_INVALID, "out of host memory");
  }
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  c->comm = comm;
  if (want_p2p) c->p2p = p2p_setup(c, xch);
  xch.release();
  cudaSetDevice(prev);
  *out = c;
  return MQ_OK;
}

int mq_comm_uses_peer_gather(const mq_comm *c) {
  if (!c) return mq::fail(MQ_ERR_INVALID, "null comm handle");
  return c->p2p ? 1 : 0;
}

void mq_comm_destroy(mq_comm *c) {
  if (!c) return;
  int prev = -1;
  if (c->p2p && cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(c->device) == cudaSuccess) {
    cudaDeviceSynchronize();
    mq::p2p_release(c);
    cudaSetDevice(prev);
  }
  if (c->comm && mq::nccl().ok) mq::nccl().comm_destroy(c->comm);
  delete c;
}

int mq_linear_sharded_allgather(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y,
                                int ldy, mq_comm *comm, void *stream) {
  using namespace mq;
  if (!w || !comm) return fail(MQ_ERR_INVALID, "null weight or comm handle");
  if (m < 0) return fail(MQ_ERR_INVALID, "negative activation count %d", m);
  if (m == 0) return MQ_OK;
  if (!x || !y) return fail(MQ_ERR_INVALID, "null activation or output pointer");
  const int R = w->v.rows, G = comm->nranks, r = comm->rank;
  if (w->device != comm->device)
    return fail(MQ_ERR_INVALID, "shard on device %d, communicator on device %d", w->device, comm->device);
  if (w->full_rows != G * R || w->row_begin != r * R)
    return fail(MQ_ERR_INVALID, "shard rows [%d, %d) of %d are not slice %d of %d equal slices", w->row_begin,
                w->row_begin + R, w->full_rows, r, G);
  if ((int64_t)ldy < (int64_t)G * R) return fail(MQ_ERR_INVALID, "output stride %d < rows %d", ldy, G * R);
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != w->device && (e = cudaSetDevice(w->device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  struct Restore {
    int dev;
    ~Restore() {
      if (dev >= 0) cudaSetDevice(dev);
    }
  } restore{prev != w->device ? prev : -1};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float *bias_slice = bias ? bias + (int64_t)r * R : nullptr;
  if (comm->p2p && (size_t)m * R <= kP2PSlotFloats) {  // peer-memory gather
    if (*(volatile int *)comm->err_host) comm->poisoned = true;
    if (comm->poisoned)
      return fail(MQ_ERR_TIMEOUT,
                  "peer-memory gather: a peer did not arrive within %llu ns in an earlier call on rank %d; this "
                  "communicator's gathers are disabled (destroy it and create a new one)",
                  (unsigned long long)comm->wait_ns, r);
    P2PArgs a{y, (int64_t)ldy, m, R, G, r, {}, comm->err_dev, comm->wait_ns};
    for (int p = 0; p < G; ++p) a.base[p] = comm->peer[p];
    const bool vec = R % 4 == 0 && ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const int64_t n = (int64_t)m * R / (vec ? 4 : 1);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148));
    int rc = MQ_ERR_UNSUPPORTED;
    if (p2p_fused()) {  // the decode kernel stores the slice into the peers itself: no push launch
      PeerOut peer;
      peer.G = G, peer.rank = r, peer.R = R;
      for (int p = 0; p < G; ++p) peer.base[p] = comm->peer[p];
      rc = run_linear_peer(w, x, m, ldx, bias_slice, y + (int64_t)r * R, ldy, s, peer);
      if (rc == MQ_OK) {
        e = vec ? p2p_pull_launch<true>(a, grid, s) : p2p_pull_launch<false>(a, grid, s);
        return e == cudaSuccess ? MQ_OK : cuda_fail(e, "peer gather launch");
      }
      if (rc != MQ_ERR_UNSUPPORTED) return rc;
    }
    rc = mq_linear(w, x, m, ldx, bias_slice, y + (int64_t)r * R, ldy, stream);
    if (rc) return rc;
    e = vec ? p2p_launch<true>(a, grid, s) : p2p_launch<false>(a, grid, s);
    return e == cudaSuccess ? MQ_OK : cuda_fail(e, "peer gather launch");
  }
  if (m == 1) {  // y is [G*R] contiguous: in-place gather straight into it
    float *mine = y + (int64_t)r * R;
    int rc = mq_linear(w, x, 1, ldx, bias_slice, mine, R, stream);
    if (rc) return rc;
    const ncclResult_t nr = nccl().all_gather(mine, y, (size_t)R, ncclFloat32, comm->comm, s);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclAllGather");
    return MQ_OK;
  }
  void *ws = nullptr;
  int rc = gather_workspace_for(w->device, s, (size_t)G * m * R * sizeof(float), &ws);
  if (rc) return rc;
  float *g = static_cast<float *>(ws);
  float *mine = g + (int64_t)r * m * R;  // this rank's [m, R] slice of the rank-major buffer
  if ((rc = mq_linear(w, x, m, ldx, bias_slice, mine, R, stream))) return rc;
  const ncclResult_t nr = nccl().all_gather(mine, g, (size_t)m * R, ncclFloat32, comm->comm, s);
  if (nr != ncclSuccess) return nccl_fail(nr, "ncclAllGather");
  const int64_t n = (int64_t)G * m * R;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  interleave_kernel<<<blocks, 256, 0, s>>>(g, G, m, R, y, ldy);
  count_launch(1);
  e = cudaGetLastError();
  return e == cudaSuccess ? MQ_OK : cuda_fail(e, "interleave launch");
}

}  // extern "C"
