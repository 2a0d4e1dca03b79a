// C-ABI entry points of the mq_b200 engine (declared in include/mq_b200.h).
//
// Host-side responsibilities: argument validation with the reference's error
// meanings, the device weight layout, kernel selection by activation count,
// and the bit-exact host quantizer. No exception crosses the ABI.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "mq_common.cuh"
#include "mq_gemm.cuh"
#include "mq_pack.cuh"

namespace mq {

std::string &last_error() {
  static thread_local std::string msg;
  return msg;
}

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error() = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(MQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

namespace {

thread_local int g_path_mode = 0;  // see mq_set_path in mq_b200.h

bool valid_qtype(int q) { return q == MQ_Q8_0 || q == MQ_Q4_0 || q == MQ_Q4_1; }

// Switches the calling thread to `device` for the scope and restores it.
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
    else if (err == cudaSuccess) prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Maps a QuantFail to the ABI code and the reference's exception message
// (src/quantized_tensor.cc:119-120, 134-135, 140-141).
int quant_status(int kind) {
  switch (kind) {
  case kQuantOk: return MQ_OK;
  case kQuantNonFinite: return fail(MQ_ERR_NONFINITE, "non-finite quantization input");
  case kQuantScaleRange: return fail(MQ_ERR_RANGE, "quantization scale exceeds F16 range");
  default: return fail(MQ_ERR_RANGE, "quantization offset exceeds F16 range");
  }
}

// Host quantizer: rows split into contiguous chunks over threads; the error
// reported is the one of the first failing block in row-major order, which is
// the block at which the reference's sequential loop throws.
int quantize_host(int qtype, const float *src, int rows, int cols, uint8_t *dst, int threads) {
  const int nb = (cols + 31) / 32, bb = block_bytes(qtype);
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  threads = std::min(threads, rows);
  std::vector<int64_t> first_bad(threads, INT64_MAX);
  std::vector<int> code(threads, kQuantOk);
  auto work = [&](int t) {
    const int r0 = (int)((int64_t)rows * t / threads), r1 = (int)((int64_t)rows * (t + 1) / threads);
    for (int r = r0; r < r1; ++r)
      for (int b = 0; b < nb; ++b) {
        const int c0 = b * 32, n = std::min(32, cols - c0);
        const int rc = quantize_block(qtype, src + (int64_t)r * cols + c0, n, dst + ((int64_t)r * nb + b) * bb);
        if (rc != kQuantOk) {
          first_bad[t] = (int64_t)r * nb + b;
          code[t] = rc;
          return;
        }
      }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto &th : pool) th.join();
  int64_t best = INT64_MAX;
  int rc = kQuantOk;
  for (int t = 0; t < threads; ++t)
    if (first_bad[t] < best) best = first_bad[t], rc = code[t];
  return quant_status(rc);
}

}  // namespace
}  // namespace mq

#include "mq_gemm_host.cuh"

using namespace mq;

namespace mq {
namespace {

// The kernel choice of mq_linear; `gate` and `resid` ([m, ldy], optional) turn
// the output write into the SwiGLU epilogue of the fused gate/up product and
// the residual add.
int linear_dispatch(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y, int ldy,
                    cudaStream_t s, const float *gate, const float *resid) {
  const int mode = g_path_mode;
  if (!gemm_supported(w->device))
    return fail(MQ_ERR_UNSUPPORTED, "the kernels need an sm_100 device (device %d)", w->device);
  if (mode == 1) return run_sdec(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (mode == 3) return run_i8dec(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (mode == 4) return run_tcdec(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (mode == 5) return run_gemv(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (mode == 7) {
    if (!w->foldable)
      return fail(MQ_ERR_UNSUPPORTED, "a block scale of this weight is too large for the scale-folded decode kernel");
    if (w->v.tiles % 2 != 0)
      return fail(MQ_ERR_UNSUPPORTED, "the CTA-pair decode kernel needs an even number of 128-row tiles");
    return run_tcdec(w, x, m, ldx, bias, y, ldy, s, gate, resid, true, nullptr, true);
  }
  if (mode == 6) {
    if (!w->foldable)
      return fail(MQ_ERR_UNSUPPORTED, "a block scale of this weight is too large for the scale-folded decode kernel");
    return run_tcdec(w, x, m, ldx, bias, y, ldy, s, gate, resid, true);
  }
  if (mode == 2 || (mode == 0 && m > decode_max_m())) return run_gemm(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (m <= gemv_max_m()) return run_gemv(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  if (m <= i8dec_max_m()) return run_i8dec(w, x, m, ldx, bias, y, ldy, s, gate, resid);
  return run_tcdec(w, x, m, ldx, bias, y, ldy, s, gate, resid, w->foldable);
}

}  // namespace

int run_linear_peer(const mq_weight *w, const float *x, int m, int64_t ldx, const float *bias, float *y, int64_t ldy,
                    cudaStream_t s, const PeerOut &peer) {
  if (g_path_mode != 0 || !gemm_supported(w->device) || m < 1 || m > decode_max_m() || m <= gemv_max_m())
    return MQ_ERR_UNSUPPORTED;
  if (m <= i8dec_max_m() && m <= 4) return run_i8dec(w, x, m, ldx, bias, y, ldy, s, nullptr, nullptr, &peer);
  if (m > i8dec_max_m() && m <= 32 && w->foldable)
    return run_tcdec(w, x, m, ldx, bias, y, ldy, s, nullptr, nullptr, true, &peer);
  return MQ_ERR_UNSUPPORTED;
}

}  // namespace mq

extern "C" {

const char *mq_last_error(void) { return last_error().c_str(); }

const char *mq_version(void) { return "mq_b200 0.1 (sm_100a)"; }

size_t mq_quantized_bytes(int qtype, int rows, int cols) {
  if (!valid_qtype(qtype) || rows <= 0 || cols <= 0) return 0;
  return (size_t)rows * (((size_t)cols + 31) / 32) * block_bytes(qtype);
}

int mq_quantize(int qtype, const float *src, int rows, int cols, void *dst, size_t dst_bytes, int threads) {
  last_error().clear();
  if (!valid_qtype(qtype)) return fail(MQ_ERR_INVALID, "unknown quantization type %d", qtype);
  if (rows <= 0 || cols <= 0) return fail(MQ_ERR_INVALID, "invalid quantized shape %dx%d", rows, cols);
  if (!src || !dst) return fail(MQ_ERR_INVALID, "null pointer");
  if (dst_bytes != mq_quantized_bytes(qtype, rows, cols))
    return fail(MQ_ERR_SIZE, "quantized storage size mismatch: %zu != %zu", dst_bytes,
                mq_quantized_bytes(qtype, rows, cols));
  return quantize_host(qtype, src, rows, cols, static_cast<uint8_t *>(dst), threads);
}

int mq_dequantize(int qtype, const void *blocks, size_t nbytes, int rows, int cols, float *dst) {
  last_error().clear();
  if (!valid_qtype(qtype)) return fail(MQ_ERR_INVALID, "unknown quantization type %d", qtype);
  if (rows <= 0 || cols <= 0) return fail(MQ_ERR_INVALID, "invalid quantized shape %dx%d", rows, cols);
  if (!blocks || !dst) return fail(MQ_ERR_INVALID, "null pointer");
  if (nbytes != mq_quantized_bytes(qtype, rows, cols)) return fail(MQ_ERR_SIZE, "quantized storage size mismatch");
  const int nb = (cols + 31) / 32, bb = block_bytes(qtype);
  const uint8_t *src = static_cast<const uint8_t *>(blocks);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) {
      const uint8_t *blk = src + ((int64_t)r * nb + c / 32) * bb;
      const int j = c % 32;
      const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      float v;
      if (qtype == MQ_Q8_0) {
        v = d * (float)(int8_t)blk[2 + j];
      } else {
        const int byte = blk[(qtype == MQ_Q4_1 ? 4 : 2) + (j & 15)];
        const int q = j < 16 ? (byte & 15) : (byte >> 4);
        v = qtype == MQ_Q4_1 ? d * (float)q + f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8))) : d * (float)(q - 8);
      }
      dst[(int64_t)r * cols + c] = v;
    }
  return MQ_OK;
}

int mq_quantize_device(int device, int qtype, const float *d_src, int rows, int cols, void *d_dst, size_t dst_bytes,
                       void *stream) {
  last_error().clear();
  if (!valid_qtype(qtype)) return fail(MQ_ERR_INVALID, "unknown quantization type %d", qtype);
  if (rows <= 0 || cols <= 0) return fail(MQ_ERR_INVALID, "invalid quantized shape %dx%d", rows, cols);
  if (!d_src || !d_dst) return fail(MQ_ERR_INVALID, "null pointer");
  if (dst_bytes != mq_quantized_bytes(qtype, rows, cols)) return fail(MQ_ERR_SIZE, "quantized storage size mismatch");
  DeviceGuard g(device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long *bad = nullptr, host_bad = ~0ull;
  MQ_CUDA(cudaMalloc(&bad, sizeof(*bad)));
  cudaError_t e = cudaMemsetAsync(bad, 0xff, sizeof(*bad), s);
  const int64_t blocks = (int64_t)rows * ((cols + 31) / 32);
  if (e == cudaSuccess) {
    quantize_kernel<<<(unsigned)((blocks + 255) / 256), 256, 0, s>>>(d_src, qtype, rows, cols,
                                                                      static_cast<uint8_t *>(d_dst), bad);
    count_launch();
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_bad, bad, sizeof(host_bad), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(bad);
  if (e != cudaSuccess) return cuda_fail(e, "device quantize");
  const int host_err = host_bad == ~0ull ? kQuantOk : (int)(host_bad & 3ull);
  return quant_status(host_err);
}

int mq_weight_shard_create(int device, int qtype, int rows, int cols, int row_begin, int row_end, const void *blocks,
                           size_t nbytes, int blocks_on_device, void *stream, mq_weight **out) {
  last_error().clear();
  if (!out) return fail(MQ_ERR_INVALID, "null output handle");
  *out = nullptr;
  if (!valid_qtype(qtype)) return fail(MQ_ERR_INVALID, "unknown quantization type %d", qtype);
  if (rows <= 0 || cols <= 0) return fail(MQ_ERR_INVALID, "invalid quantized shape %dx%d", rows, cols);
  if (row_begin < 0 || row_end > rows || row_begin >= row_end)
    return fail(MQ_ERR_INVALID, "invalid row range [%d, %d) of %d rows", row_begin, row_end, rows);
  if (!blocks) return fail(MQ_ERR_INVALID, "null block pointer");
  if (nbytes != mq_quantized_bytes(qtype, rows, cols))
    return fail(MQ_ERR_SIZE, "quantized storage size mismatch: %zu != %zu", nbytes, mq_quantized_bytes(qtype, rows, cols));
  int count = 0;
  MQ_CUDA(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) return fail(MQ_ERR_INVALID, "CUDA device id %d out of range", device);
  DeviceGuard g(device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const int nrows = row_end - row_begin, nb = (cols + 31) / 32, bb = block_bytes(qtype);
  const int steps = (nb + kStepBlocks - 1) / kStepBlocks, tiles = (nrows + kTileRows - 1) / kTileRows;
  const size_t total = (size_t)tiles * steps * (size_t)step_chunk_bytes(qtype);

  auto *w = new (std::nothrow) mq_weight;
  if (!w) return fail(MQ_ERR_INVALID, "out of host memory");
  w->device = device;
  w->row_begin = row_begin;
  w->full_rows = rows;
  cudaError_t e = cudaMalloc(&w->base, total);
  if (e != cudaSuccess) {
    delete w;
    return cuda_fail(e, "cudaMalloc weight");
  }
  w->bytes = total;
  uint8_t *base = static_cast<uint8_t *>(w->base);
  w->v = WeightView{qtype, nrows, cols, nb, steps, tiles, tiles * kTileRows, base, step_chunk_bytes(qtype),
                    step_pk_bytes(qtype)};
  const size_t shard_src_bytes = (size_t)nrows * nb * bb;
  const uint8_t *src = static_cast<const uint8_t *>(blocks) + (size_t)row_begin * nb * bb;
  void *staging = nullptr;
  int *unfoldable = nullptr, host_unfoldable = 1;
  e = cudaMemsetAsync(w->base, 0, total, s);
  if (e == cudaSuccess) e = cudaMalloc(&unfoldable, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(unfoldable, 0, sizeof(int), s);
  if (e == cudaSuccess && !blocks_on_device) {
    e = cudaMalloc(&staging, shard_src_bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(staging, src, shard_src_bytes, cudaMemcpyHostToDevice, s);
    src = static_cast<const uint8_t *>(staging);
  }
  if (e == cudaSuccess) {
    const int64_t n = (int64_t)nrows * nb;
    repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, w->v, unfoldable);
    count_launch();
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_unfoldable, unfoldable, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (unfoldable) cudaFree(unfoldable);
  w->foldable = host_unfoldable == 0;
  if (e != cudaSuccess) {
    cudaFree(w->base);
    delete w;
    return cuda_fail(e, "upload weight");
  }
  *out = w;
  return MQ_OK;
}

int mq_weight_create(int device, int qtype, int rows, int cols, const void *blocks, size_t nbytes,
                     int blocks_on_device, void *stream, mq_weight **out) {
  return mq_weight_shard_create(device, qtype, rows, cols, 0, rows, blocks, nbytes, blocks_on_device, stream, out);
}

void mq_weight_destroy(mq_weight *w) {
  if (!w) return;
  DeviceGuard g(w->device);
  cudaFree(w->base);
  delete w;
}

int mq_weight_info(const mq_weight *w, int *qtype, int *rows, int *cols, int *device, size_t *device_bytes) {
  last_error().clear();
  if (!w) return fail(MQ_ERR_INVALID, "null weight handle");
  if (qtype) *qtype = w->v.qtype;
  if (rows) *rows = w->v.rows;
  if (cols) *cols = w->v.cols;
  if (device) *device = w->device;
  if (device_bytes) *device_bytes = w->bytes;
  return MQ_OK;
}

int mq_weight_export(const mq_weight *w, void *dst, size_t dst_bytes) {
  last_error().clear();
  if (!w || !dst) return fail(MQ_ERR_INVALID, "null pointer");
  const size_t need = mq_quantized_bytes(w->v.qtype, w->v.rows, w->v.cols);
  if (dst_bytes != need) return fail(MQ_ERR_SIZE, "export size mismatch: %zu != %zu", dst_bytes, need);
  DeviceGuard g(w->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  void *tmp = nullptr;
  MQ_CUDA(cudaMalloc(&tmp, need));
  const int64_t n = (int64_t)w->v.rows * w->v.nb;
  unpack_kernel<<<(unsigned)((n + 255) / 256), 256>>>(static_cast<uint8_t *>(tmp), w->v);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpy(dst, tmp, need, cudaMemcpyDeviceToHost);
  cudaFree(tmp);
  if (e != cudaSuccess) return cuda_fail(e, "export weight");
  return MQ_OK;
}

int mq_set_path(int mode) {
  const int prev = g_path_mode;
  if (mode >= 0 && mode <= 7) g_path_mode = mode;
  return prev;
}

int mq_linear(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y, int ldy,
              void *stream) {
  last_error().clear();
  if (!w) return fail(MQ_ERR_INVALID, "null weight handle");
  if (m < 0) return fail(MQ_ERR_INVALID, "negative activation count %d", m);
  if (m == 0) return MQ_OK;
  if (!x || !y) return fail(MQ_ERR_INVALID, "null activation or output pointer");
  if (ldx < w->v.cols) return fail(MQ_ERR_INVALID, "LinearDispatch: dimension mismatch (ldx %d < cols %d)", ldx, w->v.cols);
  if (ldy < w->v.rows) return fail(MQ_ERR_INVALID, "output stride %d < rows %d", ldy, w->v.rows);
  DeviceGuard g(w->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  return linear_dispatch(w, x, m, ldx, bias, y, ldy, static_cast<cudaStream_t>(stream), nullptr, nullptr);
}

int mq_linear_residual(const mq_weight *w, const float *x, int m, int ldx, const float *bias, const float *residual,
                       float *y, int ldy, void *stream) {
  last_error().clear();
  if (!w) return fail(MQ_ERR_INVALID, "null weight handle");
  if (m < 0) return fail(MQ_ERR_INVALID, "negative activation count %d", m);
  if (m == 0) return MQ_OK;
  if (!x || !y || !residual) return fail(MQ_ERR_INVALID, "null activation, residual or output pointer");
  if (ldx < w->v.cols) return fail(MQ_ERR_INVALID, "LinearDispatch: dimension mismatch (ldx %d < cols %d)", ldx, w->v.cols);
  if (ldy < w->v.rows) return fail(MQ_ERR_INVALID, "output stride %d < rows %d", ldy, w->v.rows);
  DeviceGuard g(w->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  return linear_dispatch(w, x, m, ldx, bias, y, ldy, static_cast<cudaStream_t>(stream), nullptr, residual);
}

int mq_linear_swiglu(const mq_weight *w_gate, const mq_weight *w_up, const float *x, int m, int ldx, float *y,
                     int ldy, void *stream) {
  last_error().clear();
  if (!w_gate || !w_up) return fail(MQ_ERR_INVALID, "null weight handle");
  if (w_gate->device != w_up->device)
    return fail(MQ_ERR_INVALID, "gate on device %d, up on device %d", w_gate->device, w_up->device);
  if (w_gate->v.rows != w_up->v.rows || w_gate->v.cols != w_up->v.cols)
    return fail(MQ_ERR_INVALID, "SwiGlu: shape mismatch (gate %dx%d, up %dx%d)", w_gate->v.rows, w_gate->v.cols,
                w_up->v.rows, w_up->v.cols);
  if (m < 0) return fail(MQ_ERR_INVALID, "negative activation count %d", m);
  if (m == 0) return MQ_OK;
  if (!x || !y) return fail(MQ_ERR_INVALID, "null activation or output pointer");
  if (ldx < w_up->v.cols)
    return fail(MQ_ERR_INVALID, "LinearDispatch: dimension mismatch (ldx %d < cols %d)", ldx, w_up->v.cols);
  if (ldy < w_up->v.rows) return fail(MQ_ERR_INVALID, "output stride %d < rows %d", ldy, w_up->v.rows);
  DeviceGuard g(w_up->device);
  if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void *ws = nullptr;  // the gate product, laid out like y ([m, ldy])
  int rc = gate_workspace_for(w_up->device, s, (size_t)m * ldy * sizeof(float), &ws);
  if (rc) return rc;
  float *gate = static_cast<float *>(ws);
  if ((rc = linear_dispatch(w_gate, x, m, ldx, nullptr, gate, ldy, s, nullptr, nullptr))) return rc;
  return linear_dispatch(w_up, x, m, ldx, nullptr, y, ldy, s, gate, nullptr);
}

int mq_linear_ragged(const mq_weight *w, const float *x, const int *offsets, int n_seqs, int ldx, const float *bias,
                     float *y, int ldy, void *stream) {
  last_error().clear();
  if (!offsets || n_seqs < 0) return fail(MQ_ERR_INVALID, "invalid ragged offsets");
  if (offsets[0] != 0) return fail(MQ_ERR_INVALID, "ragged offsets must start at 0");
  for (int i = 0; i < n_seqs; ++i)
    if (offsets[i + 1] < offsets[i]) return fail(MQ_ERR_INVALID, "ragged offsets decrease at %d", i);
  return mq_linear(w, x, offsets[n_seqs], ldx, bias, y, ldy, stream);
}

uint64_t mq_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int mq_device_error_flag(int device, int **flag) {
  last_error().clear();
  if (!flag) return fail(MQ_ERR_INVALID, "null output pointer");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
    return fail(MQ_ERR_INVALID, "device %d is not a CUDA device of this process", device);
  DeviceGuard guard(device);
  int *host = nullptr;
  return device_err_flag(device, flag, &host);
}

int mq_device_info(char *buf, size_t len) {
  last_error().clear();
  if (!buf || !len) return fail(MQ_ERR_INVALID, "null buffer");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  std::string out;
  if (e != cudaSuccess) {
    out = std::string("CUDA devices=0 (") + cudaGetErrorString(e) + ")";
    count = 0;
  } else {
    out = "CUDA devices=" + std::to_string(count);
  }
  for (int i = 0; i < count; ++i) {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, i) != cudaSuccess) continue;
    out += "\n" + std::to_string(i) + ": " + p.name + " memory_bytes=" + std::to_string(p.totalGlobalMem) +
           " compute=" + std::to_string(p.major) + "." + std::to_string(p.minor) + " sms=" +
           std::to_string(p.multiProcessorCount);
  }
  std::snprintf(buf, len, "%s", out.c_str());
  return e == cudaSuccess ? MQ_OK : cuda_fail(e, "cudaGetDeviceCount");
}

}  // extern "C"
