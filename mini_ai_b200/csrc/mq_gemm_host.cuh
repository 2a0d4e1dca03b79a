// Host side of the tcgen05 GEMM: activation-split workspace, TMA tensor
// maps, launch configuration and the device error flag.
#pragma once

#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "mq_fdec.cuh"
#include "mq_fdec2.cuh"
#include "mq_gemm.cuh"
#include "mq_gemv.cuh"
#include "mq_i8dec.cuh"
#include "mq_sdec.cuh"
#include "mq_tcdec.cuh"

namespace mq {

int env_threshold(const char *name, int dflt);  // integer from the environment, or dflt

namespace {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) acts on the calling
// thread's current device only, so each launcher keeps one bit per device
// (set once the attribute is in place there). Two host threads may both set
// it on first use; that is harmless, and the mask itself is atomic.
// `max_carveout` also asks for the largest shared-memory share of the unified
// L1 / shared storage, for kernels sized to keep two CTAs on an SM.
template <typename Kernel>
cudaError_t raise_smem_limit(std::atomic<uint64_t> &done, Kernel *kernel, int bytes, bool max_carveout = false) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  if (max_carveout) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}


// Activation-split workspace, one per (device, stream): calls on one stream
// are ordered, so they can share it; calls on different streams cannot.
struct Workspace {
  void *ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;

int workspace_for(int device, cudaStream_t s, size_t bytes, void **out) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  Workspace &w = g_ws[{device, s}];
  if (w.bytes < bytes) {
    if (w.ptr) {
      // The old buffer may still be read by work queued on this stream.
      MQ_CUDA(cudaStreamSynchronize(s));
      MQ_CUDA(cudaFree(w.ptr));
      w.ptr = nullptr;
      w.bytes = 0;
    }
    const size_t grow = bytes + bytes / 4;
    MQ_CUDA(cudaMalloc(&w.ptr, grow));
    w.bytes = grow;
  }
  *out = w.ptr;
  return MQ_OK;
}

// Gather buffer of the row-sharded linear (mq_comm.cu), one per (device,
// stream) and separate from the workspace the linear itself uses.
std::map<std::pair<int, cudaStream_t>, Workspace> g_gather;

}  // namespace

int gather_workspace_for(int device, cudaStream_t s, size_t bytes, void **out) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  Workspace &w = g_gather[{device, s}];
  if (w.bytes < bytes) {
    if (w.ptr) {
      MQ_CUDA(cudaStreamSynchronize(s));
      MQ_CUDA(cudaFree(w.ptr));
      w.ptr = nullptr;
      w.bytes = 0;
    }
    MQ_CUDA(cudaMalloc(&w.ptr, bytes));
    w.bytes = bytes;
  }
  *out = w.ptr;
  return MQ_OK;
}

// Gate-product buffer of mq_linear_swiglu, one per (device, stream).
std::map<std::pair<int, cudaStream_t>, Workspace> g_gate;

int gate_workspace_for(int device, cudaStream_t s, size_t bytes, void **out) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  Workspace &w = g_gate[{device, s}];
  if (w.bytes < bytes) {
    if (w.ptr) {
      MQ_CUDA(cudaStreamSynchronize(s));
      MQ_CUDA(cudaFree(w.ptr));
      w.ptr = nullptr;
      w.bytes = 0;
    }
    MQ_CUDA(cudaMalloc(&w.ptr, bytes));
    w.bytes = bytes;
  }
  *out = w.ptr;
  return MQ_OK;
}

namespace {

// Split-K fixup tickets, one zeroed array per (device, stream); each launch
// leaves them at zero again.
std::map<std::pair<int, cudaStream_t>, Workspace> g_tickets;

int tickets_for(int device, cudaStream_t s, size_t count, int **out) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  Workspace &w = g_tickets[{device, s}];
  const size_t bytes = count * sizeof(int);
  if (w.bytes < bytes) {
    if (w.ptr) {
      MQ_CUDA(cudaStreamSynchronize(s));
      MQ_CUDA(cudaFree(w.ptr));
      w.ptr = nullptr;
      w.bytes = 0;
    }
    MQ_CUDA(cudaMalloc(&w.ptr, bytes));
    MQ_CUDA(cudaMemsetAsync(w.ptr, 0, bytes, s));
    w.bytes = bytes;
  }
  *out = static_cast<int *>(w.ptr);
  return MQ_OK;
}

// Device-visible error flag in mapped pinned host memory, one per device:
// kernels raise it when a bounded wait runs out; the host reads it without
// synchronising.
struct ErrFlag {
  int *host = nullptr;
  int *dev = nullptr;
};
std::mutex g_err_mu;
std::map<int, ErrFlag> g_err;

int err_flag(int device, int **dev_ptr, int **host_ptr) {
  std::lock_guard<std::mutex> lock(g_err_mu);
  ErrFlag &f = g_err[device];
  if (!f.host) {
    MQ_CUDA(cudaHostAlloc(&f.host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    *f.host = 0;
    MQ_CUDA(cudaHostGetDevicePointer(&f.dev, f.host, 0));
  }
  *dev_ptr = f.dev;
  *host_ptr = f.host;
  return MQ_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000 *fn) {
  std::call_once(g_encode_once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!g_encode) return fail(MQ_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
  *fn = g_encode;
  return MQ_OK;
}

// 2-D bf16 tensor map over a [rows, cols] row-major matrix, box [box_rows, 64]
// with the 128-byte swizzle the UMMA descriptors expect; out-of-range reads
// return zeros.
int make_tmap_bf16(CUtensorMap *map, const void *base, int rows, int cols, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int rc = encode_fn(&enc);
  if (rc) return rc;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MQ_OK;
}

// 2-D tensor map with a 128-byte swizzle over a row-major matrix of `elem`-byte
// elements: dims {cols, rows}, box {box_cols, box_rows}; out-of-range reads
// return zeros.
int make_tmap(CUtensorMap *map, CUtensorMapDataType dtype, int elem, const void *base, int64_t rows, int64_t cols,
              int64_t row_stride_elems, int box_cols, int box_rows,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int rc = encode_fn(&enc);
  if (rc) return rc;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * elem)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MQ_OK;
}

template <int QT, int BN, int NC, bool EPI>
cudaError_t launch_tcdec_t(const CUtensorMap &tx, const DecArgs &a, int grid, cudaStream_t s) {
  using L = DecCfg<QT, BN>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, tcdec_kernel<QT, BN, NC, EPI>, L::kAlloc)) return e0;
  const cudaError_t e = launch_pdl(tcdec_kernel<QT, BN, NC, EPI>, dim3(grid), dim3(L::kThreads), L::kAlloc, s, tx, a);
  count_launch();
  return e;
}

template <int QT>
cudaError_t launch_tcdec_q(const CUtensorMap &tx, const DecArgs &a, int grid, int m, cudaStream_t s) {
  if (a.gate || a.resid) {
    if (m <= 4) return launch_tcdec_t<QT, 8, 4, true>(tx, a, grid, s);
    if (m <= 8) return launch_tcdec_t<QT, 8, 8, true>(tx, a, grid, s);
    if (m <= 16) return launch_tcdec_t<QT, 16, 16, true>(tx, a, grid, s);
    return launch_tcdec_t<QT, 32, 32, true>(tx, a, grid, s);
  }
  if (m <= 4) return launch_tcdec_t<QT, 8, 4, false>(tx, a, grid, s);
  if (m <= 8) return launch_tcdec_t<QT, 8, 8, false>(tx, a, grid, s);
  if (m <= 16) return launch_tcdec_t<QT, 16, 16, false>(tx, a, grid, s);
  return launch_tcdec_t<QT, 32, 32, false>(tx, a, grid, s);
}

template <int QT, int BN, bool EPI, bool PEER = false>
cudaError_t launch_fdec_t(const CUtensorMap &tx, const DecArgs &a, int grid, cudaStream_t s) {
  using L = FdCfg<QT, BN>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, fdec_kernel<QT, BN, BN, EPI, PEER>, L::kAlloc)) return e0;
  const cudaError_t e =
      launch_pdl(fdec_kernel<QT, BN, BN, EPI, PEER>, dim3(grid), dim3(kFdThreads), L::kAlloc, s, tx, a);
  count_launch();
  return e;
}

// The CTA-pair form: clusters of 2 CTAs, launched with programmatic stream
// serialization like the others (grid even).
template <int QT, int BN, bool EPI>
cudaError_t launch_fdec2_t(const CUtensorMap &tx, const DecArgs &a, int grid, cudaStream_t s) {
  using L = Fd2Cfg<QT, BN>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, fdec2_kernel<QT, BN, BN, EPI>, L::kAlloc)) return e0;
  static const bool pdl = env_threshold("MQ_PDL", 1) != 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFdThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fdec2_kernel<QT, BN, BN, EPI>, tx, a);
  count_launch();
  return e;
}

template <int QT>
cudaError_t launch_fdec2_q(const CUtensorMap &tx, const DecArgs &a, int grid, int bn, cudaStream_t s) {
  const bool epi = a.gate || a.resid;
  if (bn == 16) return epi ? launch_fdec2_t<QT, 16, true>(tx, a, grid, s) : launch_fdec2_t<QT, 16, false>(tx, a, grid, s);
  return epi ? launch_fdec2_t<QT, 32, true>(tx, a, grid, s) : launch_fdec2_t<QT, 32, false>(tx, a, grid, s);
}

template <int QT>
cudaError_t launch_fdec_q(const CUtensorMap &tx, const DecArgs &a, int grid, int bn, cudaStream_t s) {
  const bool epi = a.gate || a.resid;
  if (a.peer.G > 1)  // the row-sharded gather fused into the output stores (no epilogue there)
    return bn == 16 ? launch_fdec_t<QT, 16, false, true>(tx, a, grid, s) : launch_fdec_t<QT, 32, false, true>(tx, a, grid, s);
  if (bn == 16) return epi ? launch_fdec_t<QT, 16, true>(tx, a, grid, s) : launch_fdec_t<QT, 16, false>(tx, a, grid, s);
  return epi ? launch_fdec_t<QT, 32, true>(tx, a, grid, s) : launch_fdec_t<QT, 32, false>(tx, a, grid, s);
}

// Schedule of the persistent GEMM (one CTA per SM): whole waves of tiles,
// then the tail tiles split into K pieces of at least kGemmMinSteps steps so
// that the tail takes about one piece's time.
constexpr int kGemmMinSteps = 8;
template <int BN>
void gemm_schedule(GemmArgs &a, int sms, int *grid) {
  const int tiles = ((a.m + BN - 1) / BN) * ((a.w.rows + kGemmRows - 1) / kGemmRows);
  a.waves = tiles / sms;
  a.tail = tiles % sms;
  a.split = a.tail ? std::max(1, std::min(sms / a.tail, a.ktiles / kGemmMinSteps)) : 1;
  *grid = a.waves ? sms : a.tail * a.split;
}

template <int QT, int BN, int STAGES, bool FOLD>
cudaError_t launch_gemm_t(const CUtensorMap &th, const CUtensorMap &tl, const GemmArgs &a, int sms, cudaStream_t s) {
  using L = GemmSmem<QT, BN, STAGES>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, gemm_kernel<QT, BN, STAGES, FOLD>, L::kAlloc)) return e0;
  GemmArgs b = a;
  int grid = 1;
  gemm_schedule<BN>(b, sms, &grid);
  gemm_kernel<QT, BN, STAGES, FOLD><<<grid, kGemmThreads, L::kAlloc, s>>>(th, tl, b);
  count_launch();
  return cudaGetLastError();
}

}  // namespace

// The device's bounded-wait error flag, for kernels launched from other files
// (the peer-memory gather of the row-sharded linear).
int device_err_flag(int device, int **dev_ptr, int **host_ptr) { return err_flag(device, dev_ptr, host_ptr); }

int env_threshold(const char *name, int dflt) {
  const char *e = std::getenv(name);
  return e && *e ? std::atoi(e) : dflt;
}

// Launch with programmatic stream serialization (the kernel may start while
// the previous kernel of the stream finishes; it synchronises with
// griddepcontrol.wait where it depends on it). MQ_PDL=0 launches normally.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args &&...args) {
  static const bool on = env_threshold("MQ_PDL", 1) != 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = on ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Largest activation count served by the decode kernels in automatic mode;
// above it the tcgen05 prefill GEMM takes over.
int decode_max_m() {
  static const int v = std::min(32, env_threshold("MQ_DECODE_MAX_M", 32));
  return v;
}

bool gemm_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return false;
  return major == 10 && minor == 0;
}

DecPlan tcdec_plan(const WeightView &w, int device, int max_grid) {
  DecPlan p;
  p.steps = w.steps;
  p.kpad = w.steps * kDecBlocksPerStep * 32;
  p.tiles = w.tiles;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int grid = env_threshold("MQ_TCDEC_GRID", 0);
  if (grid <= 0) grid = sms;
  if (max_grid > 0) grid = std::min(grid, max_grid);
  p.grid = std::max(1, std::min(grid, p.tiles * p.steps));
  return p;
}

int tcdec_launch(const WeightView &w, const float *x, int mm, int64_t ldx, const float *bias, float *y, int64_t ldy,
                 cudaStream_t s, const DecPlan &plan, const DecBuffers &buf, int nan_on_abort, const float *gate,
                 const float *resid, bool folded, const PeerOut *peer, bool pairs_wanted) {
  const int bn = folded ? fdec_tile_rows(mm) : dec_tile_rows(mm);
  if (folded)  // one scale per activation row: the folded kernel accumulates along K
    MQ_CUDA(launch_pdl(fold_prep_kernel, dim3(bn, (plan.steps + kFpSteps - 1) / kFpSteps), dim3(kFpThreads), 0, s,
                       x, ldx, mm, w.cols, plan.kpad, bn, buf.x2, buf.xsum, buf.xinv, (int)(w.qtype == MQ_Q4_1)));
  else
    MQ_CUDA(launch_pdl(dec_prep_kernel, dim3(plan.steps, (bn + 7) / 8), dim3(256), 0, s, x, ldx, mm, w.cols,
                       plan.kpad, bn, buf.x2, buf.xsum, buf.xinv, (int)(w.qtype == MQ_Q4_1)));
  count_launch();
  // The scale-folded kernel on CTA pairs (mq_fdec2.cuh), when asked for and
  // the weight has an even number of tiles; each CTA of a pair loads bn
  // activation rows.
  const bool pairs = folded && pairs_wanted && !peer && w.tiles % 2 == 0 && plan.grid >= 2;
  CUtensorMap tx;
  int rc;
  if ((rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, buf.x2, 2 * bn, plan.kpad, plan.kpad, 64,
                      pairs ? bn : 2 * bn)))
    return rc;
  DecArgs a{w, mm, buf.xinv, buf.xsum, bias, y, ldy, buf.partial, buf.tickets, plan.steps, plan.tiles, buf.err,
            nan_on_abort, gate, resid};
  if (peer) a.peer = *peer;
  cudaError_t e;
  if (pairs) {
    const int grid = std::min(plan.grid, (w.tiles / 2) * plan.steps * 2) & ~1;
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_fdec2_q<MQ_Q8_0>(tx, a, grid, bn, s); break;
    case MQ_Q4_0: e = launch_fdec2_q<MQ_Q4_0>(tx, a, grid, bn, s); break;
    default: e = launch_fdec2_q<MQ_Q4_1>(tx, a, grid, bn, s); break;
    }
  } else if (folded) {
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_fdec_q<MQ_Q8_0>(tx, a, plan.grid, bn, s); break;
    case MQ_Q4_0: e = launch_fdec_q<MQ_Q4_0>(tx, a, plan.grid, bn, s); break;
    default: e = launch_fdec_q<MQ_Q4_1>(tx, a, plan.grid, bn, s); break;
    }
  } else {
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_tcdec_q<MQ_Q8_0>(tx, a, plan.grid, mm, s); break;
    case MQ_Q4_0: e = launch_tcdec_q<MQ_Q4_0>(tx, a, plan.grid, mm, s); break;
    default: e = launch_tcdec_q<MQ_Q4_1>(tx, a, plan.grid, mm, s); break;
    }
  }
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 decode launch");
  return MQ_OK;
}

// tcgen05 decode GEMM: up to 32 activation rows per launch (split + kernel);
// `folded` runs the scale-folded kernel (mq_fdec.cuh), which needs a foldable weight.
int run_tcdec(const mq_weight *wt, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
              cudaStream_t s, const float *gate, const float *resid, bool folded, const PeerOut *peer,
              bool pairs) {
  if (peer && m > 32) return fail(MQ_ERR_INVALID, "a fused gather needs one launch (m <= 32)");
  int *err_dev = nullptr, *err_host = nullptr;
  int rc = err_flag(wt->device, &err_dev, &err_host);
  if (rc) return rc;
  if (*(volatile int *)err_host) {
    *(volatile int *)err_host = 0;
    return fail(MQ_ERR_TIMEOUT, "an earlier tensor-core launch on device %d ran out of a bounded wait", wt->device);
  }
  const WeightView &w = wt->v;
  const DecPlan plan = tcdec_plan(w, wt->device);
  int *tickets = nullptr;
  if ((rc = tickets_for(wt->device, s, (size_t)plan.tiles, &tickets))) return rc;
  for (int i0 = 0; i0 < m; i0 += 32) {
    const int mm = std::min(32, m - i0);
    const int bn = folded ? fdec_tile_rows(mm) : dec_tile_rows(mm);
    const size_t xbytes = (size_t)2 * bn * plan.kpad * 2;
    const size_t sbytes = (size_t)(plan.kpad / 32) * bn * 4;
    const size_t ibytes = ((size_t)plan.steps * bn * 4 + 255) & ~size_t(255);
    const size_t pbytes = (size_t)plan.grid * 2 * kDecRows * bn * 4;
    void *ws = nullptr;
    if ((rc = workspace_for(wt->device, s, xbytes + sbytes + ibytes + pbytes + 1024, &ws))) return rc;
    uint8_t *base = static_cast<uint8_t *>(ws);
    DecBuffers buf;
    buf.x2 = reinterpret_cast<__half *>(base);
    buf.xsum = reinterpret_cast<float *>(base + xbytes);
    buf.xinv = reinterpret_cast<float *>(base + xbytes + sbytes);
    buf.partial = reinterpret_cast<float *>(base + ((xbytes + sbytes + ibytes + 1023) & ~size_t(1023)));
    buf.tickets = tickets;
    buf.err = err_dev;
    if ((rc = tcdec_launch(w, x + (int64_t)i0 * ldx, mm, ldx, bias, y + (int64_t)i0 * ldy, ldy, s, plan, buf, 0,
                           gate ? gate + (int64_t)i0 * ldy : nullptr, resid ? resid + (int64_t)i0 * ldy : nullptr,
                           folded, peer, pairs)))
      return rc;
  }
  return MQ_OK;
}

namespace {

template <int QT, int MC>
cudaError_t launch_sdec_t(const CUtensorMap &tx, const SdecArgs &a, int grid, cudaStream_t s) {
  using L = SdCfg<QT, MC>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, sdec_kernel<QT, MC>, L::kAlloc)) return e0;
  const cudaError_t e = launch_pdl(sdec_kernel<QT, MC>, dim3(grid), dim3(kSdThreads), L::kAlloc, s, tx, a);
  count_launch();
  return e;
}

template <int QT>
cudaError_t launch_sdec_q(const CUtensorMap &tx, const SdecArgs &a, int grid, int mc, cudaStream_t s) {
  if (mc == 1) return launch_sdec_t<QT, 1>(tx, a, grid, s);
  if (mc == 2) return launch_sdec_t<QT, 2>(tx, a, grid, s);
  return launch_sdec_t<QT, 4>(tx, a, grid, s);
}

}  // namespace

// Largest activation count served by the stream-K SIMT GEMV (mq_sdec.cuh).
int sdec_max_m() {
  static const int v = env_threshold("MQ_SDEC_MAX_M", 2);
  return v;
}

// Stream-K SIMT GEMV: up to 4 activation rows per launch. The activations
// are read by TMA straight from x when its base and row stride are 16-byte
// aligned; otherwise they are first copied to an aligned scratch.
int run_sdec(const mq_weight *wt, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
             cudaStream_t s, const float *gate, const float *resid) {
  int *err_dev = nullptr, *err_host = nullptr;
  int rc = err_flag(wt->device, &err_dev, &err_host);
  if (rc) return rc;
  if (*(volatile int *)err_host) {
    *(volatile int *)err_host = 0;
    return fail(MQ_ERR_TIMEOUT, "an earlier stream-K launch on device %d ran out of a bounded wait", wt->device);
  }
  const WeightView &w = wt->v;
  DecPlan plan = tcdec_plan(w, wt->device);
  int *tickets = nullptr;
  if ((rc = tickets_for(wt->device, s, (size_t)plan.tiles, &tickets))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, wt->device);
  for (int i0 = 0; i0 < m; i0 += 4) {
    const int mm = std::min(4, m - i0);
    const int mc = mm == 1 ? 1 : (mm == 2 ? 2 : 4);
    const int ctas_per_sm = 1;  // SdCfg<QT, mc>::kCtasPerSm
    plan.grid = std::max(1, std::min(ctas_per_sm * sms, plan.tiles * plan.steps));
    const float *xs = x + (int64_t)i0 * ldx;
    int64_t ldxs = ldx;
    const bool copy = (reinterpret_cast<uintptr_t>(xs) & 15) != 0 || (ldx & 3) != 0;
    const int64_t ldc = ((int64_t)w.cols + 3) & ~int64_t(3);
    const size_t pbytes = (size_t)plan.grid * 2 * kSdRows * mc * 4;
    const size_t cbytes = copy ? (size_t)mm * ldc * 4 : 0;
    void *ws = nullptr;
    if ((rc = workspace_for(wt->device, s, pbytes + cbytes + 1024, &ws))) return rc;
    uint8_t *base = static_cast<uint8_t *>(ws);
    if (copy) {
      float *xc = reinterpret_cast<float *>(base + ((pbytes + 255) & ~size_t(255)));
      MQ_CUDA(cudaMemcpy2DAsync(xc, (size_t)ldc * 4, xs, (size_t)ldx * 4, (size_t)w.cols * 4, (size_t)mm,
                                cudaMemcpyDeviceToDevice, s));
      xs = xc;
      ldxs = ldc;
    }
    CUtensorMap tx;
    if ((rc = make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xs, mm, w.cols, ldxs, 256, mc,
                        CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    SdecArgs a{w, mm, bias, y + (int64_t)i0 * ldy, ldy, reinterpret_cast<float *>(base), tickets, plan.steps,
               plan.tiles, err_dev, 0, gate ? gate + (int64_t)i0 * ldy : nullptr,
               resid ? resid + (int64_t)i0 * ldy : nullptr};
    cudaError_t e;
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_sdec_q<MQ_Q8_0>(tx, a, plan.grid, mc, s); break;
    case MQ_Q4_0: e = launch_sdec_q<MQ_Q4_0>(tx, a, plan.grid, mc, s); break;
    default: e = launch_sdec_q<MQ_Q4_1>(tx, a, plan.grid, mc, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "stream-K GEMV launch");
  }
  return MQ_OK;
}

namespace {

template <int QT, int MC, bool EPI, bool PEER = false>
cudaError_t launch_i8dec_t(const I8Args &a, int grid, cudaStream_t s) {
  using L = I8Cfg<QT, MC>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, i8dec_kernel<QT, MC, EPI, PEER>, L::kAlloc)) return e0;
  const cudaError_t e = launch_pdl(i8dec_kernel<QT, MC, EPI, PEER>, dim3(grid), dim3(kI8Threads), L::kAlloc, s, a);
  count_launch();
  return e;
}

template <int QT>
cudaError_t launch_i8dec_q(const I8Args &a, int grid, int mc, cudaStream_t s) {
  if (a.peer.G > 1) {  // the row-sharded gather fused into the output stores (no epilogue there)
    if (mc == 1) return launch_i8dec_t<QT, 1, false, true>(a, grid, s);
    if (mc == 2) return launch_i8dec_t<QT, 2, false, true>(a, grid, s);
    return launch_i8dec_t<QT, 4, false, true>(a, grid, s);
  }
  if (a.gate || a.resid) {
    if (mc == 1) return launch_i8dec_t<QT, 1, true>(a, grid, s);
    if (mc == 2) return launch_i8dec_t<QT, 2, true>(a, grid, s);
    return launch_i8dec_t<QT, 4, true>(a, grid, s);
  }
  if (mc == 1) return launch_i8dec_t<QT, 1, false>(a, grid, s);
  if (mc == 2) return launch_i8dec_t<QT, 2, false>(a, grid, s);
  return launch_i8dec_t<QT, 4, false>(a, grid, s);
}

}  // namespace

// Largest activation count served by the int8 tensor-core decode kernel in
// automatic mode (mq_i8dec.cuh); it takes up to 4 rows per launch.
int i8dec_max_m() {
  static const int v = env_threshold("MQ_I8DEC_MAX_M", 4);
  return v;
}

// int8 tensor-core decode: up to 4 activation rows per launch.
int run_i8dec(const mq_weight *wt, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
              cudaStream_t s, const float *gate = nullptr, const float *resid = nullptr,
              const PeerOut *peer = nullptr) {
  if (peer && m > 4) return fail(MQ_ERR_INVALID, "a fused gather needs one launch (m <= 4)");
  int *err_dev = nullptr, *err_host = nullptr;
  int rc = err_flag(wt->device, &err_dev, &err_host);
  if (rc) return rc;
  if (*(volatile int *)err_host) {
    *(volatile int *)err_host = 0;
    return fail(MQ_ERR_TIMEOUT, "an earlier int8 decode launch on device %d ran out of a bounded wait", wt->device);
  }
  const WeightView &w = wt->v;
  const DecPlan plan = tcdec_plan(w, wt->device);
  int *tickets = nullptr;
  if ((rc = tickets_for(wt->device, s, (size_t)plan.tiles, &tickets))) return rc;
  for (int i0 = 0; i0 < m; i0 += 4) {
    const int mm = std::min(4, m - i0);
    const int mc = mm == 1 ? 1 : (mm == 2 ? 2 : 4);
    const size_t pbytes = (size_t)plan.grid * 2 * kI8Rows * mc * 4;
    void *ws = nullptr;
    if ((rc = workspace_for(wt->device, s, pbytes + 1024, &ws))) return rc;
    I8Args a{w, mm, x + (int64_t)i0 * ldx, ldx, bias, y + (int64_t)i0 * ldy, ldy, static_cast<float *>(ws), tickets,
             plan.steps, plan.tiles, err_dev, 0, gate ? gate + (int64_t)i0 * ldy : nullptr,
             resid ? resid + (int64_t)i0 * ldy : nullptr};
    if (peer) a.peer = *peer;
    cudaError_t e;
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_i8dec_q<MQ_Q8_0>(a, plan.grid, mc, s); break;
    case MQ_Q4_0: e = launch_i8dec_q<MQ_Q4_0>(a, plan.grid, mc, s); break;
    default: e = launch_i8dec_q<MQ_Q4_1>(a, plan.grid, mc, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "int8 decode launch");
  }
  return MQ_OK;
}

namespace {

template <int QT, int MC, bool EPI>
cudaError_t launch_gemv_t(const GvArgs &a, int grid, cudaStream_t s) {
  using L = GvCfg<QT, MC>;
  static std::atomic<uint64_t> smem_set{0};
  if (const cudaError_t e0 = raise_smem_limit(smem_set, gemv_kernel<QT, MC, EPI>, L::kBytes, true)) return e0;
  const cudaError_t e = launch_pdl(gemv_kernel<QT, MC, EPI>, dim3(grid), dim3(kGvThreads), L::kBytes, s, a);
  count_launch();
  return e;
}

template <int QT>
cudaError_t launch_gemv_q(const GvArgs &a, int grid, int mc, cudaStream_t s) {
  if (a.gate || a.resid) return mc == 1 ? launch_gemv_t<QT, 1, true>(a, grid, s) : launch_gemv_t<QT, 2, true>(a, grid, s);
  return mc == 1 ? launch_gemv_t<QT, 1, false>(a, grid, s) : launch_gemv_t<QT, 2, false>(a, grid, s);
}

}  // namespace

// Largest activation count served by the SIMT dp4a GEMV in automatic mode
// (mq_gemv.cuh); it takes up to 2 rows per launch.
int gemv_max_m() {
  static const int v = env_threshold("MQ_GEMV_MAX_M", 0);
  return v;
}

// SIMT dp4a decode GEMV: up to 2 activation rows per launch.
int run_gemv(const mq_weight *wt, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
             cudaStream_t s, const float *gate = nullptr, const float *resid = nullptr) {
  int *err_dev = nullptr, *err_host = nullptr;
  int rc = err_flag(wt->device, &err_dev, &err_host);
  if (rc) return rc;
  if (*(volatile int *)err_host) {
    *(volatile int *)err_host = 0;
    return fail(MQ_ERR_TIMEOUT, "an earlier decode launch on device %d ran out of a bounded wait", wt->device);
  }
  const WeightView &w = wt->v;
  const DecPlan plan = tcdec_plan(w, wt->device);
  int *tickets = nullptr;
  if ((rc = tickets_for(wt->device, s, (size_t)plan.tiles, &tickets))) return rc;
  for (int i0 = 0; i0 < m; i0 += 2) {
    const int mm = std::min(2, m - i0);
    const size_t pbytes = (size_t)plan.grid * 2 * kGvRows * mm * 4;
    void *ws = nullptr;
    if ((rc = workspace_for(wt->device, s, pbytes + 1024, &ws))) return rc;
    GvArgs a{w, mm, x + (int64_t)i0 * ldx, ldx, bias, y + (int64_t)i0 * ldy, ldy, static_cast<float *>(ws), tickets,
             plan.steps, plan.tiles, err_dev, 0, gate ? gate + (int64_t)i0 * ldy : nullptr,
             resid ? resid + (int64_t)i0 * ldy : nullptr};
    cudaError_t e;
    switch (w.qtype) {
    case MQ_Q8_0: e = launch_gemv_q<MQ_Q8_0>(a, plan.grid, mm, s); break;
    case MQ_Q4_0: e = launch_gemv_q<MQ_Q4_0>(a, plan.grid, mm, s); break;
    default: e = launch_gemv_q<MQ_Q4_1>(a, plan.grid, mm, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "dp4a decode launch");
  }
  return MQ_OK;
}

int run_gemm(const mq_weight *wt, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
             cudaStream_t s, const float *gate, const float *resid) {
  int *err_dev = nullptr, *err_host = nullptr;
  int rc = err_flag(wt->device, &err_dev, &err_host);
  if (rc) return rc;
  if (*(volatile int *)err_host) {
    *(volatile int *)err_host = 0;
    return fail(MQ_ERR_TIMEOUT, "an earlier tensor-core GEMM on device %d ran out of a bounded wait", wt->device);
  }
  const WeightView &w = wt->v;
  const int kpad = w.nb * 32;
  constexpr int BN = 256, STAGES = 2;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, wt->device);
  const int ktiles = (w.nb + 1) / 2;
  const int tiles = ((m + BN - 1) / BN) * ((w.rows + kGemmRows - 1) / kGemmRows);
  int *tickets = nullptr;
  if ((rc = tickets_for(wt->device, s, (size_t)tiles, &tickets))) return rc;
  // The scale-folded form for weights whose every d * code fits fp16 (Q4_1's
  // block minimum has no exact fold); MQ_GEMM_FOLD=0 keeps the bf16 form.
  static const bool fold_on = env_threshold("MQ_GEMM_FOLD", 1) != 0;
  const bool fold = fold_on && wt->foldable && w.qtype != MQ_Q4_1;
  const size_t half = ((size_t)m * kpad * 2 + 255) & ~size_t(255);  // bf16 or fp16 [m, kpad]
  const size_t pbytes = (size_t)sms * BN * kGemmRows * sizeof(float);  // split pieces' partial tiles, one per CTA
  const size_t ibytes = ((size_t)m * sizeof(float) + 255) & ~size_t(255);
  void *ws = nullptr;
  rc = workspace_for(wt->device, s, 2 * half + pbytes + ibytes, &ws);
  if (rc) return rc;
  uint8_t *xh = static_cast<uint8_t *>(ws), *xl = xh + half;
  float *part = reinterpret_cast<float *>(xh + 2 * half);
  float *xinv = reinterpret_cast<float *>(xh + 2 * half + pbytes);
  if (fold) {
    split_x_f16_kernel<<<(unsigned)m, kSplitThreads, 0, s>>>(x, ldx, w.cols, kpad, reinterpret_cast<__half *>(xh),
                                                             reinterpret_cast<__half *>(xl), xinv);
  } else {
    const int64_t pairs = (int64_t)m * (kpad / 2);
    split_x_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, s>>>(x, ldx, m, w.cols, kpad,
                                                                   reinterpret_cast<__nv_bfloat16 *>(xh),
                                                                   reinterpret_cast<__nv_bfloat16 *>(xl));
  }
  count_launch();
  MQ_CUDA(cudaGetLastError());

  CUtensorMap th, tl;  // 2-byte elements, bf16 or fp16 alike (the copies are bitwise; out of range reads zero)
  if ((rc = make_tmap_bf16(&th, xh, m, kpad, BN))) return rc;
  if ((rc = make_tmap_bf16(&tl, xl, m, kpad, BN))) return rc;
  GemmArgs a{w, y, ldy, bias, m, ktiles, err_dev, gate, resid, tickets, part};
  a.xinv = xinv;
  cudaError_t e;
  switch (w.qtype) {
  case MQ_Q8_0:
    e = fold ? launch_gemm_t<MQ_Q8_0, BN, STAGES, true>(th, tl, a, sms, s)
             : launch_gemm_t<MQ_Q8_0, BN, STAGES, false>(th, tl, a, sms, s);
    break;
  case MQ_Q4_0:
    e = fold ? launch_gemm_t<MQ_Q4_0, BN, STAGES, true>(th, tl, a, sms, s)
             : launch_gemm_t<MQ_Q4_0, BN, STAGES, false>(th, tl, a, sms, s);
    break;
  default: e = launch_gemm_t<MQ_Q4_1, BN, STAGES, false>(th, tl, a, sms, s); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return MQ_OK;
}

}  // namespace mq
