// mq_linear_noalloc: the decode product for callers that cannot allocate
// device memory. Such callers own every device byte through their own pool,
// run under a fixed memory budget, or sit in a hot loop where cudaMalloc's
// device-wide synchronisation and unbounded latency are not acceptable.
//
// The scratch the tcgen05 decode GEMM needs (the fp16 split of the
// activations, split-K partial sums, fixup tickets and the timeout flag)
// lives in one file-scope device array of fixed size. It is reserved when the
// library's device code is loaded on a GPU and held until the process exits;
// every call on that GPU shares it.
#include <algorithm>
#include <mutex>

#include "mq_common.cuh"
#include "mq_tcdec_api.h"

namespace mq {
namespace {

constexpr int kNaMaxM = 16;           // activation rows per call
constexpr int kNaMaxKpad = 16384;     // padded K: weights with cols <= 16384
constexpr int kNaMaxTiles = 1024;     // 128-row tiles: weights with rows <= 131072
constexpr int kNaMaxGrid = 160;       // persistent CTAs (two partial tiles each)
constexpr int kNaMaxDevices = 64;

constexpr size_t kNaX = (size_t)2 * kNaMaxM * kNaMaxKpad * sizeof(__half);    // 1 MiB: hi rows, lo rows
constexpr size_t kNaSum = (size_t)(kNaMaxKpad / 32) * kNaMaxM * sizeof(float);  // 32 KiB
constexpr size_t kNaInv = (size_t)(kNaMaxKpad / 256) * kNaMaxM * sizeof(float);  // 4 KiB: per (step, row)
constexpr size_t kNaPart = (size_t)kNaMaxGrid * 2 * 128 * kNaMaxM * sizeof(float);  // 2.5 MiB
constexpr size_t kNaTickets = (size_t)kNaMaxTiles * sizeof(int);
constexpr size_t kNaErr = 256;

constexpr size_t kOffX = 0;
constexpr size_t kOffSum = kOffX + kNaX;
constexpr size_t kOffInv = kOffSum + kNaSum;
constexpr size_t kOffPart = kOffInv + kNaInv;
constexpr size_t kOffTickets = kOffPart + kNaPart;
constexpr size_t kOffErr = kOffTickets + kNaTickets;
constexpr size_t kNaBytes = kOffErr + kNaErr;  // 3.6 MiB

}  // namespace

// In host code this name is only a host-side stand-in for the device array;
// its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

namespace {

std::mutex g_na_mu;
uint8_t *g_na_base[kNaMaxDevices] = {};

// Device address of the scratch array on `device`, which must be current.
// The first call per device resolves it (and may load the module there).
int na_scratch(int device, uint8_t **out) {
  std::lock_guard<std::mutex> lock(g_na_mu);
  if (!g_na_base[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_na_base[device] = static_cast<uint8_t *>(p);
  }
  *out = g_na_base[device];
  return MQ_OK;
}

struct CurrentDevice {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit CurrentDevice(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
    else if (err == cudaSuccess) prev = -1;
  }
  ~CurrentDevice() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace mq

using namespace mq;

extern "C" int mq_linear_noalloc(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y,
                                 int ldy, void *stream) {
  last_error().clear();
  if (!w) return fail(MQ_ERR_INVALID, "null weight handle");
  if (m < 0) return fail(MQ_ERR_INVALID, "negative activation count %d", m);
  if (m == 0) return MQ_OK;
  if (!x || !y) return fail(MQ_ERR_INVALID, "null activation or output pointer");
  if (ldx < w->v.cols) return fail(MQ_ERR_INVALID, "LinearDispatch: dimension mismatch (ldx %d < cols %d)", ldx, w->v.cols);
  if (ldy < w->v.rows) return fail(MQ_ERR_INVALID, "output stride %d < rows %d", ldy, w->v.rows);
  if (m > kNaMaxM)
    return fail(MQ_ERR_INVALID, "mq_linear_noalloc: at most %d activation rows per call (got %d)", kNaMaxM, m);
  if (w->device < 0 || w->device >= kNaMaxDevices)
    return fail(MQ_ERR_UNSUPPORTED, "mq_linear_noalloc: device %d beyond %d", w->device, kNaMaxDevices);
  CurrentDevice g(w->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  if (!gemm_supported(w->device))
    return fail(MQ_ERR_UNSUPPORTED, "mq_linear_noalloc needs an sm_100 device (device %d)", w->device);
  const DecPlan plan = tcdec_plan(w->v, w->device, kNaMaxGrid);
  if (plan.kpad > kNaMaxKpad)
    return fail(MQ_ERR_INVALID, "mq_linear_noalloc: weight has %d columns; the static scratch holds at most %d",
                w->v.cols, kNaMaxKpad);
  if (plan.tiles > kNaMaxTiles)
    return fail(MQ_ERR_INVALID, "mq_linear_noalloc: weight has %d rows; the static scratch holds at most %d",
                w->v.rows, kNaMaxTiles * 128);
  uint8_t *base = nullptr;
  int rc = na_scratch(w->device, &base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DecBuffers buf;
  buf.x2 = reinterpret_cast<__half *>(base + kOffX);
  buf.xsum = reinterpret_cast<float *>(base + kOffSum);
  buf.xinv = reinterpret_cast<float *>(base + kOffInv);
  buf.partial = reinterpret_cast<float *>(base + kOffPart);
  buf.tickets = reinterpret_cast<int *>(base + kOffTickets);
  buf.err = reinterpret_cast<int *>(base + kOffErr);
  // The array keeps the previous call's contents: the fixup tickets and the
  // timeout flag must start at zero (everything else is written before read).
  cudaError_t e = cudaMemsetAsync(buf.tickets, 0, (size_t)plan.tiles * sizeof(int), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(buf.err, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "clear no-alloc scratch");
  return tcdec_launch(w->v, x, m, ldx, bias, y, ldy, s, plan, buf, /*nan_on_abort=*/1);
}
