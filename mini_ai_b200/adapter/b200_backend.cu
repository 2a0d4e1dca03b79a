// mini_ai's CUDA backend (include/mini_llama/backend.h: EnableCuda,
// CudaDeviceInfo, CudaStats, ForwardCuda) rebuilt over the mq_b200 C ABI, and
// the batched forward of several requests (b200_backend.h).
//
// This file takes the place of the reference's src/cuda_backend.cu in a
// mini_ai build: forward.cc calls ForwardCuda for a model that EnableCuda
// uploaded (src/forward.cc:160), and every projection of the forward
// (q, k, v, o, gate, up, down and lm_head) goes through include/mq_b200.h:
//   - quantized weights (QuantizeModel / GGUF Q8_0, Q4_0, Q4_1) are uploaded
//     with mq_weight_create from their packed blocks (UploadWeight,
//     src/cuda_backend.cu:275-283) and multiplied by mq_linear_ragged (q/k/v
//     with their biases, the rows of every request of a batch in one call),
//     mq_linear_residual (wo and w_down, the residual adds of
//     src/cuda_backend.cu:426-434 in the same kernel) and mq_linear_swiglu
//     (gate/up with SwiGluKernel, src/cuda_backend.cu:241-245);
//   - F32 weights, the embedding, RMSNorm, RoPE, the KV cache and attention
//     run on the small kernels below (the reference's EmbedKernel, NormKernel,
//     RopeKernel, StoreKvKernel, Scores/Softmax/AttentionKernel,
//     src/cuda_backend.cu:112-234), following the CPU forward's formulas
//     (src/forward.cc, src/ops.cc). Each kernel takes a block of token rows:
//     row t has its own token, position and request (KV cache).
// ForwardCuda is the one-token case of the same row-block forward.
// Errors are C++ exceptions as in the reference: a failing CUDA call or ABI
// call throws std::runtime_error("<operation>: <message>") (Check,
// src/cuda_backend.cu:17-21). CudaStats reports the same counters as the
// reference (src/cuda_backend.cu:446-460).
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "b200_backend.h"
#include "mini_llama/backend.h"
#include "mini_llama/context.h"
#include "mini_llama/model.h"
#include "mini_llama/quantized_tensor.h"
#include "mq_b200.h"

namespace mini_llama {
namespace {

void Check(cudaError_t status, const char *operation) {
  if (status != cudaSuccess) throw std::runtime_error(std::string(operation) + ": " + cudaGetErrorString(status));
}
void CheckMq(int rc, const char *operation) {
  if (rc != MQ_OK) throw std::runtime_error(std::string(operation) + ": " + mq_last_error());
}

// Owning device allocation on one device.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  DeviceBuffer(size_t bytes, int device) : device_(device) {
    Check(cudaSetDevice(device), "cudaSetDevice");
    Check(cudaMalloc(&ptr_, bytes == 0 ? 4 : bytes), "cudaMalloc");
  }
  ~DeviceBuffer() { reset(); }
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;
  DeviceBuffer(DeviceBuffer &&o) noexcept : ptr_(o.ptr_), device_(o.device_) { o.ptr_ = nullptr; }
  DeviceBuffer &operator=(DeviceBuffer &&o) noexcept {
    if (this != &o) {
      reset();
      ptr_ = o.ptr_;
      device_ = o.device_;
      o.ptr_ = nullptr;
    }
    return *this;
  }
  float *floats() const { return static_cast<float *>(ptr_); }
  void *get() const { return ptr_; }

 private:
  void reset() {
    if (ptr_) {
      cudaSetDevice(device_);
      cudaFree(ptr_);
      ptr_ = nullptr;
    }
  }
  void *ptr_ = nullptr;
  int device_ = 0;
};

// A projection weight on the device: a packed mq_weight, or F32 rows.
struct DeviceWeight {
  mq_weight *packed = nullptr;
  const float *dense = nullptr;
  int rows = 0, cols = 0;
};

constexpr int kThreads = 256;

// Kernels over a block of token rows: blockIdx.y (blockIdx.x for the norm) is
// the row t; tokens[t], positions[t] and request[t] (whose KV cache) describe it.

__global__ void EmbedKernel(const float *embedding, const int *tokens, int dim, float *out) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dim) out[(size_t)t * dim + i] = embedding[(size_t)tokens[t] * dim + i];
}

// RmsNorm (src/ops.cc): x * 1 / sqrt(mean(x^2) + eps) * w, one CTA per row.
__global__ void NormKernel(const float *x, const float *w, int dim, float eps, float *out) {
  __shared__ float part[kThreads / 32];
  x += (size_t)blockIdx.x * dim;
  out += (size_t)blockIdx.x * dim;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += x[i] * x[i];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) total += part[i];
  const float inv = 1.0f / sqrtf(total / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = x[i] * inv * w[i];
}

// Rope (src/ops.cc ApplyRopeNormalToHeads): pair i of a head rotates by
// pos / theta^(2i / head_dim); NeoX pairs (i, i + hd/2), normal (2i, 2i + 1).
__global__ void RopeKernel(float *x, int heads, int hd, const int *positions, float theta, bool neox) {
  const int t = blockIdx.y, pair = blockIdx.x * blockDim.x + threadIdx.x;
  if (pair >= heads * (hd / 2)) return;
  x += (size_t)t * heads * hd;
  const int head = pair / (hd / 2), i = 2 * (pair % (hd / 2));
  const float freq = 1.0f / powf(theta, (float)i / (float)hd);
  const float angle = (float)positions[t] * freq;
  const float c = cosf(angle), s = sinf(angle);
  const int a = head * hd + (neox ? i / 2 : i);
  const int b = neox ? a + hd / 2 : a + 1;
  const float x0 = x[a], x1 = x[b];
  x[a] = x0 * c - x1 * s;
  x[b] = x0 * s + x1 * c;
}

// K/V of row t into its request's cache at (layer, positions[t]).
__global__ void StoreKvKernel(const float *k, const float *v, int kv_dim, float *const *keys, float *const *values,
                              const int *request, const int *positions, int layer, int max_seq) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kv_dim) return;
  const size_t offset = ((size_t)layer * max_seq + positions[t]) * kv_dim + i;
  keys[request[t]][offset] = k[(size_t)t * kv_dim + i];
  values[request[t]][offset] = v[(size_t)t * kv_dim + i];
}

// Attention of one query head of row t over its request's positions
// 0..positions[t] (AttentionForward, src/forward.cc): scores = q . k_s /
// sqrt(hd), softmax, weighted sum of v_s. Grid (heads, rows); the scores live
// in dynamic shared memory.
__global__ void AttentionKernel(const float *q, float *const *keys, float *const *values, const int *request,
                                const int *positions, float *out, int hd, int heads, int kv_heads, int max_seq,
                                int layer) {
  extern __shared__ float scores[];
  __shared__ float red[kThreads / 32];
  const int h = blockIdx.x, t = blockIdx.y, kh = h / (heads / kv_heads), pos = positions[t];
  const float *kc = keys[request[t]], *vc = values[request[t]];
  q += (size_t)t * heads * hd;
  out += (size_t)t * heads * hd;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const float scale = 1.0f / sqrtf((float)hd);
  for (int s = warp; s <= pos; s += nwarps) {
    const float *kp = kc + (((size_t)layer * max_seq + s) * kv_heads + kh) * hd;
    float dot = 0.0f;
    for (int d = lane; d < hd; d += 32) dot += q[h * hd + d] * kp[d];
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) scores[s] = dot * scale;
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int s = threadIdx.x; s <= pos; s += blockDim.x) mx = fmaxf(mx, scores[s]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < nwarps; ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.0f;
  for (int s = threadIdx.x; s <= pos; s += blockDim.x) {
    const float e = expf(scores[s] - mx);
    scores[s] = e;
    sum += e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.0f;
  for (int i = 0; i < nwarps; ++i) sum += red[i];
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s <= pos; ++s) acc += (scores[s] / sum) * vc[(((size_t)layer * max_seq + s) * kv_heads + kh) * hd + d];
    out[h * hd + d] = acc;
  }
}

// F32 projection of row t: y[t][n] = W[n] . x[t] (+ bias[n]) (+ residual[t][n]),
// one warp per output.
__global__ void LinearF32Kernel(const float *x, const float *w, int rows, int cols, const float *bias,
                                const float *residual, float *y) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31, t = blockIdx.y;
  if (row >= rows) return;
  const float *wr = w + (size_t)row * cols, *xr = x + (size_t)t * cols;
  float dot = 0.0f;
  for (int c = lane; c < cols; c += 32) dot += wr[c] * xr[c];
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) {
    float v = dot + (bias ? bias[row] : 0.0f);
    if (residual) v += residual[(size_t)t * rows + row];
    y[(size_t)t * rows + row] = v;
  }
}

// SwiGlu (src/ops.cc): g * sigmoid(g) * u, in place on the gate.
__global__ void SwiGluKernel(float *gate, const float *up, size_t count) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) {
    const float g = gate[i];
    gate[i] = g * (1.0f / (1.0f + expf(-g))) * up[i];
  }
}

// out[r] = x[rows[r]]: the last token row of every request, for the logits.
__global__ void GatherRowsKernel(const float *x, const int *rows, int dim, float *out) {
  const int r = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dim) out[(size_t)r * dim + i] = x[(size_t)rows[r] * dim + i];
}

// Random model weights: element i of stream `id` is a normal deviate from a
// counter-based generator (splitmix64 of (seed, id, i) -> two uniforms ->
// Box-Muller), times `scale`.
__device__ __forceinline__ uint64_t Mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__global__ void NormalKernel(float *out, size_t count, float scale, uint64_t seed, uint64_t id) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t r = Mix64(seed ^ Mix64(id * 0x100000001b3ull + i));
    const float u1 = ((float)(r >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    out[i] = scale * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

__global__ void FillKernel(float *out, size_t count, float value) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
    out[i] = value;
}

int Grid(size_t count) { return (int)((count + kThreads - 1) / kThreads); }

}  // namespace

struct CudaModelState {
  int device;
  std::vector<DeviceBuffer> allocations;
  std::vector<mq_weight *> handles;
  struct Layer {
    const float *norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    DeviceWeight q, k, v, o, gate, up, down;
  };
  std::vector<Layer> layers;
  const float *embedding = nullptr;
  const float *final_norm = nullptr;
  DeviceWeight output;
  size_t uploaded_bytes = 0;
  int uploaded_weights = 0;

  // Row-block scratch shared by the contexts of this model (grown on demand).
  struct Scratch {
    int rows = 0, requests = 0;
    DeviceBuffer x, norm, q, k, v, attention, gate, up, last, logits, meta;
  } scratch;

  explicit CudaModelState(int id) : device(id) {}
  ~CudaModelState() {
    for (mq_weight *w : handles) mq_weight_destroy(w);
  }
  CudaModelState(const CudaModelState &) = delete;
  CudaModelState &operator=(const CudaModelState &) = delete;

  const float *UploadFloat(const Tensor &t) {
    if (t.data.empty()) return nullptr;
    const size_t bytes = t.data.size() * sizeof(float);
    allocations.emplace_back(bytes, device);
    Check(cudaMemcpy(allocations.back().get(), t.data.data(), bytes, cudaMemcpyHostToDevice), "upload weight");
    uploaded_bytes += bytes;
    return allocations.back().floats();
  }
  DeviceWeight UploadWeight(const Tensor &t) {
    ++uploaded_weights;
    DeviceWeight w;
    if (t.quantized) {
      const QuantizedStorage &s = *t.quantized;
      mq_weight *h = nullptr;
      CheckMq(mq_weight_create(device, static_cast<int>(s.type), s.rows, s.cols, s.bytes.data(), s.bytes.size(), 0,
                               nullptr, &h),
              "upload weight");
      handles.push_back(h);
      uploaded_bytes += s.bytes.size();
      w.packed = h;
      w.rows = s.rows;
      w.cols = s.cols;
      return w;
    }
    if (t.num_dims() != 2) throw std::runtime_error("upload weight: expected a 2D weight " + t.ShapeStringShort());
    w.dense = UploadFloat(t);
    w.rows = t.shape[0];
    w.cols = t.shape[1];
    return w;
  }

  // Scratch for `rows` token rows of `requests` requests; meta holds
  // tokens[rows], positions[rows], request[rows], last_row[requests], then
  // the requests' key and value cache pointers.
  void Reserve(const ModelConfig &c, int rows, int requests) {
    if (rows <= scratch.rows && requests <= scratch.requests) return;
    rows = std::max(rows, scratch.rows);
    requests = std::max(requests, scratch.requests);
    const size_t kv_dim = static_cast<size_t>(c.n_kv_heads) * c.head_dim;
    auto alloc = [&](size_t n) { return DeviceBuffer(n * sizeof(float), device); };
    scratch.x = alloc(rows * (size_t)c.dim);
    scratch.norm = alloc(rows * (size_t)c.dim);
    scratch.q = alloc(rows * (size_t)c.dim);
    scratch.k = alloc(rows * kv_dim);
    scratch.v = alloc(rows * kv_dim);
    scratch.attention = alloc(rows * (size_t)c.dim);
    scratch.gate = alloc(rows * (size_t)c.hidden_dim);
    scratch.up = alloc(rows * (size_t)c.hidden_dim);
    scratch.last = alloc(requests * (size_t)c.dim);
    scratch.logits = alloc(requests * (size_t)c.vocab_size);
    scratch.meta = DeviceBuffer((3 * (size_t)rows + requests) * sizeof(int) + 16 + 2 * requests * sizeof(float *),
                                device);
    scratch.rows = rows;
    scratch.requests = requests;
  }
};

struct CudaContextState {
  std::shared_ptr<CudaModelState> owner;
  DeviceBuffer keys, values;
  unsigned long long linear_calls = 0, activation_calls = 0, attention_calls = 0, d2h_bytes = 0;

  CudaContextState(const std::shared_ptr<CudaModelState> &model, const ModelConfig &c) : owner(model) {
    const size_t kv_dim = static_cast<size_t>(c.n_kv_heads) * c.head_dim;
    if (kv_dim > std::numeric_limits<size_t>::max() / c.n_layers / c.max_seq_len)
      throw std::runtime_error("CUDA KV cache size overflow");
    const size_t elements = kv_dim * c.n_layers * c.max_seq_len;
    if (elements > std::numeric_limits<size_t>::max() / sizeof(float))
      throw std::runtime_error("CUDA KV cache size overflow");
    keys = DeviceBuffer(elements * sizeof(float), model->device);
    values = DeviceBuffer(elements * sizeof(float), model->device);
    Check(cudaMemset(keys.get(), 0, elements * sizeof(float)), "clear keys");
    Check(cudaMemset(values.get(), 0, elements * sizeof(float)), "clear values");
  }
};

namespace {

// One forward over a row block: request r owns rows [offsets[r], offsets[r + 1])
// with tokens / positions; states[r] holds its KV cache. Writes the logits of
// the last row of every request to logits ([requests][vocab], host).
void ForwardRows(const MiniLlamaModel &model, const std::vector<CudaContextState *> &states,
                 const std::vector<int> &offsets, const std::vector<int> &tokens, const std::vector<int> &positions,
                 float *logits) {
  const auto &c = model.config;
  auto &gpu = *model.cuda;
  Check(cudaSetDevice(gpu.device), "cudaSetDevice");
  const int R = static_cast<int>(states.size()), M = static_cast<int>(tokens.size());
  const int kv_dim = c.n_kv_heads * c.head_dim;
  gpu.Reserve(c, M, R);
  auto &sc = gpu.scratch;
  // Row metadata and the requests' cache pointers: one host-to-device copy.
  std::vector<int> request(M), last(R);
  int max_pos = 0;
  for (int r = 0; r < R; ++r) {
    for (int t = offsets[r]; t < offsets[r + 1]; ++t) request[t] = r;
    last[r] = offsets[r + 1] - 1;
  }
  for (int p : positions) max_pos = std::max(max_pos, p);
  const size_t ints = 3 * (size_t)sc.rows + sc.requests;
  const size_t ptr_off = (ints * sizeof(int) + 15) & ~size_t(15);
  std::vector<uint8_t> meta(ptr_off + 2 * R * sizeof(float *));
  int *im = reinterpret_cast<int *>(meta.data());
  std::memcpy(im, tokens.data(), M * sizeof(int));
  std::memcpy(im + sc.rows, positions.data(), M * sizeof(int));
  std::memcpy(im + 2 * sc.rows, request.data(), M * sizeof(int));
  std::memcpy(im + 3 * sc.rows, last.data(), R * sizeof(int));
  float **ptrs = reinterpret_cast<float **>(meta.data() + ptr_off);
  for (int r = 0; r < R; ++r) {
    ptrs[r] = states[r]->keys.floats();
    ptrs[R + r] = states[r]->values.floats();
  }
  Check(cudaMemcpy(sc.meta.get(), meta.data(), meta.size(), cudaMemcpyHostToDevice), "upload batch rows");
  const int *d_tokens = static_cast<const int *>(sc.meta.get());
  const int *d_pos = d_tokens + sc.rows, *d_req = d_tokens + 2 * sc.rows, *d_last = d_tokens + 3 * sc.rows;
  float *const *d_keys = reinterpret_cast<float *const *>(static_cast<uint8_t *>(sc.meta.get()) + ptr_off);
  float *const *d_values = d_keys + R;
  unsigned long long linear_calls = 0, activation_calls = 0, attention_calls = 0;

  // y = W x (+ bias) (+ residual; y may be the residual), `rows` rows.
  auto linear = [&](const DeviceWeight &w, const float *x, int rows, float *y, const float *bias,
                    const float *residual) {
    if (w.packed) {
      if (residual)
        CheckMq(mq_linear_residual(w.packed, x, rows, w.cols, bias, residual, y, w.rows, nullptr), "CUDA linear");
      else
        CheckMq(mq_linear(w.packed, x, rows, w.cols, bias, y, w.rows, nullptr), "CUDA linear");
    } else {
      LinearF32Kernel<<<dim3((w.rows + 7) / 8, rows), kThreads>>>(x, w.dense, w.rows, w.cols, bias, residual, y);
    }
    ++linear_calls;
  };
  // q / k / v: the ragged rows of all requests in one call.
  auto project = [&](const DeviceWeight &w, const float *x, float *y, const float *bias) {
    if (w.packed)
      CheckMq(mq_linear_ragged(w.packed, x, offsets.data(), R, w.cols, bias, y, w.rows, nullptr), "CUDA linear");
    else
      LinearF32Kernel<<<dim3((w.rows + 7) / 8, M), kThreads>>>(x, w.dense, w.rows, w.cols, bias, nullptr, y);
    ++linear_calls;
  };
  auto norm = [&](const float *input, const float *weight, int rows, float *output) {
    NormKernel<<<rows, kThreads>>>(input, weight, c.dim, c.rms_norm_eps, output);
    ++activation_calls;
  };
  const size_t score_bytes = (size_t)(max_pos + 1) * sizeof(float);
  if (score_bytes > 48 * 1024)
    Check(cudaFuncSetAttribute(AttentionKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_bytes),
          "attention shared memory");

  EmbedKernel<<<dim3(Grid(c.dim), M), kThreads>>>(gpu.embedding, d_tokens, c.dim, sc.x.floats());
  const bool neox = c.rope_type == RopeType::kNeoX;
  for (int i = 0; i < c.n_layers; ++i) {
    const auto &layer = gpu.layers[i];
    norm(sc.x.floats(), layer.norm, M, sc.norm.floats());
    project(layer.q, sc.norm.floats(), sc.q.floats(), layer.bq);
    project(layer.k, sc.norm.floats(), sc.k.floats(), layer.bk);
    project(layer.v, sc.norm.floats(), sc.v.floats(), layer.bv);
    RopeKernel<<<dim3(Grid(c.dim / 2), M), kThreads>>>(sc.q.floats(), c.n_heads, c.head_dim, d_pos, c.rope_theta,
                                                        neox);
    RopeKernel<<<dim3(Grid(kv_dim / 2), M), kThreads>>>(sc.k.floats(), c.n_kv_heads, c.head_dim, d_pos,
                                                         c.rope_theta, neox);
    StoreKvKernel<<<dim3(Grid(kv_dim), M), kThreads>>>(sc.k.floats(), sc.v.floats(), kv_dim, d_keys, d_values, d_req,
                                                        d_pos, i, c.max_seq_len);
    AttentionKernel<<<dim3(c.n_heads, M), kThreads, score_bytes>>>(sc.q.floats(), d_keys, d_values, d_req, d_pos,
                                                                   sc.attention.floats(), c.head_dim, c.n_heads,
                                                                   c.n_kv_heads, c.max_seq_len, i);
    ++attention_calls;
    linear(layer.o, sc.attention.floats(), M, sc.x.floats(), nullptr, sc.x.floats());  // x += wo . attn
    norm(sc.x.floats(), layer.ffn_norm, M, sc.norm.floats());
    if (layer.gate.packed && layer.up.packed) {  // SwiGlu(gate, up) fused into the up product's output
      CheckMq(mq_linear_swiglu(layer.gate.packed, layer.up.packed, sc.norm.floats(), M, c.dim, sc.gate.floats(),
                               layer.up.rows, nullptr),
              "CUDA linear");
      linear_calls += 2;
    } else {
      linear(layer.gate, sc.norm.floats(), M, sc.gate.floats(), nullptr, nullptr);
      linear(layer.up, sc.norm.floats(), M, sc.up.floats(), nullptr, nullptr);
      SwiGluKernel<<<Grid((size_t)M * c.hidden_dim), kThreads>>>(sc.gate.floats(), sc.up.floats(),
                                                                (size_t)M * c.hidden_dim);
    }
    linear(layer.down, sc.gate.floats(), M, sc.x.floats(), nullptr, sc.x.floats());  // x += w_down . h
    activation_calls += 5;
  }
  GatherRowsKernel<<<dim3(Grid(c.dim), R), kThreads>>>(sc.x.floats(), d_last, c.dim, sc.last.floats());
  norm(sc.last.floats(), gpu.final_norm, R, sc.norm.floats());
  linear(gpu.output, sc.norm.floats(), R, sc.logits.floats(), nullptr, nullptr);
  Check(cudaGetLastError(), "CUDA forward kernel launch");
  // Sampling stays on the CPU: only the final logits come back, as in the reference.
  const size_t bytes = (size_t)R * c.vocab_size * sizeof(float);
  Check(cudaMemcpy(logits, sc.logits.get(), bytes, cudaMemcpyDeviceToHost), "download logits");
  for (CudaContextState *st : states) {  // every request of the block took part in every call
    st->linear_calls += linear_calls;
    st->activation_calls += activation_calls;
    st->attention_calls += attention_calls;
  }
  for (int r = 0; r < R; ++r) states[r]->d2h_bytes += (size_t)c.vocab_size * sizeof(float);
}

CudaContextState &StateOf(MiniLlamaContext &context, const MiniLlamaModel &model) {
  if (!model.cuda) throw std::runtime_error("model is not uploaded to CUDA");
  Check(cudaSetDevice(model.cuda->device), "cudaSetDevice");
  if (!context.cuda) context.cuda = std::make_shared<CudaContextState>(model.cuda, model.config);
  if (context.cuda->owner != model.cuda) throw std::runtime_error("CUDA context belongs to another model");
  return *context.cuda;
}

// ValidateForwardInputs (src/forward.cc:14-39) for one token at `pos`, minus
// the host-embedding size check (the embedding may live on the device only).
void ValidateToken(const MiniLlamaModel &model, int token, int pos) {
  const ModelConfig &c = model.config;
  if (!model.loaded) throw std::runtime_error("ForwardToken called with an unloaded model");
  if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.n_heads % c.n_kv_heads != 0 ||
      c.head_dim % 2 != 0 || c.dim != c.n_heads * c.head_dim)
    throw std::runtime_error("ForwardToken invalid attention dimensions");
  if (token < 0 || token >= c.vocab_size) throw std::out_of_range("ForwardToken token id out of range");
  if (pos < 0 || pos >= c.max_seq_len) throw std::out_of_range("ForwardToken position out of range");
  if (model.cuda && model.cuda->layers.size() != static_cast<size_t>(c.n_layers))
    throw std::runtime_error("ForwardToken layer count mismatch");
}

}  // namespace

void EnableCuda(MiniLlamaModel &model, int device) {
  if (!model.loaded) throw std::runtime_error("cannot upload an unloaded model");
  int count = 0;
  Check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) throw std::runtime_error("CUDA device id out of range");
  auto gpu = std::make_shared<CudaModelState>(device);
  gpu->embedding = gpu->UploadFloat(model.token_embedding);
  gpu->final_norm = gpu->UploadFloat(model.final_norm);
  gpu->output = gpu->UploadWeight(model.lm_head);
  for (const auto &layer : model.layers) {
    CudaModelState::Layer up;
    up.norm = gpu->UploadFloat(layer.attention_norm);
    up.ffn_norm = gpu->UploadFloat(layer.ffn_norm);
    up.bq = gpu->UploadFloat(layer.bq);
    up.bk = gpu->UploadFloat(layer.bk);
    up.bv = gpu->UploadFloat(layer.bv);
    up.q = gpu->UploadWeight(layer.wq);
    up.k = gpu->UploadWeight(layer.wk);
    up.v = gpu->UploadWeight(layer.wv);
    up.o = gpu->UploadWeight(layer.wo);
    up.gate = gpu->UploadWeight(layer.w_gate);
    up.up = gpu->UploadWeight(layer.w_up);
    up.down = gpu->UploadWeight(layer.w_down);
    gpu->layers.push_back(up);
  }
  model.cuda = std::move(gpu);
}

std::string CudaDeviceInfo() {
  int count = 0;
  Check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  std::ostringstream out;
  out << "CUDA devices=" << count;
  for (int device = 0; device < count; ++device) {
    cudaDeviceProp prop{};
    Check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    out << '\n'
        << device << ": " << prop.name << " memory_bytes=" << prop.totalGlobalMem << " compute=" << prop.major << '.'
        << prop.minor;
  }
  return out.str();
}

Tensor ForwardCuda(MiniLlamaContext &context, const MiniLlamaModel &model, int token) {
  CudaContextState &st = StateOf(context, model);
  Tensor output({model.config.vocab_size});
  ForwardRows(model, {&st}, {0, 1}, {token}, {context.pos}, output.data.data());
  return output;
}

std::vector<Tensor> ForwardBatchCuda(const std::vector<MiniLlamaContext *> &contexts, const MiniLlamaModel &model,
                                     const std::vector<MiniBatch> &batches) {
  if (contexts.size() != batches.size())
    throw std::runtime_error("ForwardBatchCuda: one batch per context is required");
  if (contexts.empty()) throw std::runtime_error("ForwardBatchCuda: no requests");
  std::vector<int> offsets{0}, tokens, positions;
  for (size_t r = 0; r < batches.size(); ++r) {
    const MiniBatch &b = batches[r];
    if (!contexts[r]) throw std::runtime_error("ForwardBatchCuda: null context");
    for (size_t s = 0; s < r; ++s)
      if (contexts[s] == contexts[r]) throw std::runtime_error("ForwardBatchCuda: a context appears twice");
    if (b.num_tokens() == 0) throw std::runtime_error("ForwardBatch: empty batch");
    if (b.tokens.size() != b.positions.size())
      throw std::runtime_error("ForwardBatch: tokens and positions size mismatch");
    for (int i = 0; i < b.num_tokens(); ++i) {
      ValidateToken(model, b.tokens[i], b.positions[i]);
      if (i > 0 && b.positions[i] <= b.positions[i - 1])
        throw std::runtime_error("ForwardBatchCuda: positions of a batch must increase");
    }
    tokens.insert(tokens.end(), b.tokens.begin(), b.tokens.end());
    positions.insert(positions.end(), b.positions.begin(), b.positions.end());
    offsets.push_back(static_cast<int>(tokens.size()));
  }
  if (!model.cuda) throw std::runtime_error("model is not uploaded to CUDA");
  std::vector<CudaContextState *> states;
  for (MiniLlamaContext *ctx : contexts) states.push_back(&StateOf(*ctx, model));
  const int V = model.config.vocab_size;
  std::vector<float> logits((size_t)batches.size() * V);
  ForwardRows(model, states, offsets, tokens, positions, logits.data());
  std::vector<Tensor> out;
  for (size_t r = 0; r < batches.size(); ++r) {
    Tensor t({V});
    std::memcpy(t.data.data(), logits.data() + r * V, V * sizeof(float));
    out.push_back(std::move(t));
    // ForwardBatch's bookkeeping (src/forward.cc:184-200).
    MiniLlamaContext &ctx = *contexts[r];
    const MiniBatch &b = batches[r];
    const bool prefill = ctx.token_history.empty() || b.num_tokens() > 1;
    ctx.pos = b.positions.back();
    for (int tok : b.tokens) ctx.token_history.push_back(tok);
    (prefill ? ctx.n_prefill_tokens : ctx.n_decode_tokens) += b.num_tokens();
  }
  return out;
}

void QuantizeModelB200(MiniLlamaModel &model, QuantType type) {
  if (model.cuda) throw std::runtime_error("quantize weights before uploading the model to CUDA");
  auto pack = [type](const Tensor &t) {
    if (t.num_dims() != 2) throw std::invalid_argument("quantization requires a matrix");
    const int rows = t.shape[0], cols = t.shape[1];
    std::vector<float> dense;
    const float *src = t.data.data();
    if (t.quantized) {  // as QuantizeTensor: decode, then pack again
      dense.resize((size_t)rows * cols);
      const QuantizedStorage &s = *t.quantized;
      CheckMq(mq_dequantize(static_cast<int>(s.type), s.bytes.data(), s.bytes.size(), rows, cols, dense.data()),
              "dequantize");
      src = dense.data();
    }
    std::vector<uint8_t> bytes(mq_quantized_bytes(static_cast<int>(type), rows, cols));
    const int rc = mq_quantize(static_cast<int>(type), src, rows, cols, bytes.data(), bytes.size(), 0);
    if (rc == MQ_ERR_INVALID) throw std::invalid_argument(mq_last_error());
    if (rc != MQ_OK) throw std::runtime_error(mq_last_error());
    return TensorFromQuantized(std::move(bytes), rows, cols, type);
  };
  for (auto &layer : model.layers)
    for (Tensor *weight : {&layer.wq, &layer.wk, &layer.wv, &layer.wo, &layer.w_gate, &layer.w_up, &layer.w_down})
      *weight = pack(*weight);
  model.lm_head = pack(model.lm_head);
}

MiniLlamaModel RandomCudaModel(const ModelConfig &config, int type, uint64_t seed, int device) {
  int count = 0;
  Check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) throw std::runtime_error("CUDA device id out of range");
  if (type != 0 && type != static_cast<int>(QuantType::kQ80) && type != static_cast<int>(QuantType::kQ40) &&
      type != static_cast<int>(QuantType::kQ41))
    throw std::invalid_argument("unsupported weight type");
  Check(cudaSetDevice(device), "cudaSetDevice");
  MiniLlamaModel model;
  model.config = config;
  model.loaded = true;
  auto gpu = std::make_shared<CudaModelState>(device);
  const ModelConfig &c = config;
  const size_t kv_dim = (size_t)c.n_kv_heads * c.head_dim;
  const size_t largest = std::max({(size_t)c.vocab_size * c.dim, (size_t)c.hidden_dim * c.dim,
                                   (size_t)c.dim * c.dim, kv_dim * c.dim});
  DeviceBuffer tmp(largest * sizeof(float), device);
  uint64_t stream_id = 0;
  auto dense = [&](size_t n, float scale, bool fill) {
    gpu->allocations.emplace_back(n * sizeof(float), device);
    float *p = gpu->allocations.back().floats();
    if (fill)
      FillKernel<<<592, kThreads>>>(p, n, scale);
    else
      NormalKernel<<<1184, kThreads>>>(p, n, scale, seed, stream_id++);
    Check(cudaGetLastError(), "random weights");
    gpu->uploaded_bytes += n * sizeof(float);
    return p;
  };
  auto weight = [&](int rows, int cols) {
    DeviceWeight w;
    w.rows = rows;
    w.cols = cols;
    ++gpu->uploaded_weights;
    if (type == 0) {
      w.dense = dense((size_t)rows * cols, 0.02f, false);
      return w;
    }
    NormalKernel<<<1184, kThreads>>>(tmp.floats(), (size_t)rows * cols, 0.02f, seed, stream_id++);
    Check(cudaGetLastError(), "random weights");
    const size_t nbytes = mq_quantized_bytes(type, rows, cols);
    DeviceBuffer blocks(nbytes, device);
    CheckMq(mq_quantize_device(device, type, tmp.floats(), rows, cols, blocks.get(), nbytes, nullptr), "quantize");
    mq_weight *h = nullptr;
    CheckMq(mq_weight_create(device, type, rows, cols, blocks.get(), nbytes, 1, nullptr, &h), "upload weight");
    Check(cudaDeviceSynchronize(), "upload weight");
    gpu->handles.push_back(h);
    gpu->uploaded_bytes += nbytes;
    w.packed = h;
    return w;
  };
  gpu->embedding = dense((size_t)c.vocab_size * c.dim, 1.0f, false);
  gpu->final_norm = dense(c.dim, 1.0f, true);
  for (int i = 0; i < c.n_layers; ++i) {
    CudaModelState::Layer l;
    l.norm = dense(c.dim, 1.0f, true);
    l.ffn_norm = dense(c.dim, 1.0f, true);
    l.q = weight(c.dim, c.dim);
    l.k = weight((int)kv_dim, c.dim);
    l.v = weight((int)kv_dim, c.dim);
    l.o = weight(c.dim, c.dim);
    l.gate = weight(c.hidden_dim, c.dim);
    l.up = weight(c.hidden_dim, c.dim);
    l.down = weight(c.dim, c.hidden_dim);
    gpu->layers.push_back(l);
  }
  gpu->output = weight(c.vocab_size, c.dim);
  Check(cudaDeviceSynchronize(), "random model");
  model.cuda = std::move(gpu);
  return model;
}

MiniLlamaModel HostCopyOfCudaModel(const MiniLlamaModel &model, int layers) {
  if (!model.cuda) throw std::runtime_error("model is not uploaded to CUDA");
  const CudaModelState &gpu = *model.cuda;
  if (layers < 0 || layers > static_cast<int>(gpu.layers.size())) throw std::out_of_range("layer count out of range");
  Check(cudaSetDevice(gpu.device), "cudaSetDevice");
  const ModelConfig &c = model.config;
  auto floats = [](const float *p, std::vector<int> shape) {
    Tensor t(shape);
    if (p) Check(cudaMemcpy(t.data.data(), p, t.data.size() * sizeof(float), cudaMemcpyDeviceToHost), "download");
    return t;
  };
  auto matrix = [&](const DeviceWeight &w) {
    if (!w.packed) return floats(w.dense, {w.rows, w.cols});
    int type = 0;
    size_t nbytes = 0;
    CheckMq(mq_weight_info(w.packed, &type, nullptr, nullptr, nullptr, &nbytes), "weight info");
    std::vector<uint8_t> bytes(nbytes);
    CheckMq(mq_weight_export(w.packed, bytes.data(), bytes.size()), "export weight");
    return TensorFromQuantized(std::move(bytes), w.rows, w.cols, static_cast<QuantType>(type));
  };
  MiniLlamaModel host;
  host.config = c;
  host.config.n_layers = layers;
  host.loaded = true;
  host.token_embedding = floats(gpu.embedding, {c.vocab_size, c.dim});
  host.final_norm = floats(gpu.final_norm, {c.dim});
  host.lm_head = matrix(gpu.output);
  for (int i = 0; i < layers; ++i) {
    const auto &g = gpu.layers[i];
    LayerWeights l;
    l.attention_norm = floats(g.norm, {c.dim});
    l.ffn_norm = floats(g.ffn_norm, {c.dim});
    l.wq = matrix(g.q);
    l.wk = matrix(g.k);
    l.wv = matrix(g.v);
    l.wo = matrix(g.o);
    l.w_gate = matrix(g.gate);
    l.w_up = matrix(g.up);
    l.w_down = matrix(g.down);
    host.layers.push_back(std::move(l));
  }
  return host;
}

std::string CudaStats(const MiniLlamaModel &model, const MiniLlamaContext &context) {
  if (!model.cuda) return "";
  std::ostringstream out;
  out << "uploaded_weights=" << model.cuda->uploaded_weights << " uploaded_bytes=" << model.cuda->uploaded_bytes;
  if (context.cuda)
    out << " cuda_linear_calls=" << context.cuda->linear_calls
        << " cuda_activation_calls=" << context.cuda->activation_calls
        << " cuda_attention_calls=" << context.cuda->attention_calls
        << " device_to_host_bytes=" << context.cuda->d2h_bytes << " cpu_attention_fallback_calls=0";
  return out.str();
}

}  // namespace mini_llama
