// Row-sharded linear with an NCCL all-gather of the output slices.
//
// A projection too large for one GPU (or worth splitting for bandwidth) is
// split by output rows: rank r of G holds rows [r*R, (r+1)*R) as its own
// mq_weight (mq_weight_shard_create). Rows are independent (y_n = <W_n, x>),
// so each rank computes its R outputs with the ordinary decode/prefill
// kernels and one all-gather over NVLink assembles y [m, G*R] on every rank.
// The result is bit-identical to the unsharded product: the same kernels see
// the same rows.
//
// NCCL is loaded at the first mq_comm call with dlopen("libnccl.so.2"), so
// the library has no link-time dependency on it and, inside a PyTorch
// process, shares the NCCL that torch already loaded.
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "mq_common.cuh"
#include "mq_tcdec_api.h"

#include "nccl.h"

namespace mq {
int gather_workspace_for(int device, cudaStream_t s, size_t bytes, void **out);
void count_launch(int n);
}  // namespace mq

struct mq_comm {
  int device = 0, nranks = 1, rank = 0;
  ncclComm_t comm = nullptr;
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
  ncclUniqueId u;
  memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nccl().comm_init_rank(&comm, nranks, u, rank);
  cudaSetDevice(prev);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  auto *c = new (std::nothrow) mq_comm;
  if (!c) {
    nccl().comm_destroy(comm);
    return fail(MQ_ERR_INVALID, "out of host memory");
  }
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  c->comm = comm;
  *out = c;
  return MQ_OK;
}

void mq_comm_destroy(mq_comm *c) {
  if (!c) return;
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
