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
#include <map>
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

// RmsNorm (src/ops.cc): x * 1 / sqrt(mean(x^2) + eps) * w, one CTA per row;
// float4 loads, unrolled so that a thread's loads are in flight together.
__global__ void NormKernel(const float *x, const float *w, int dim, float eps, float *out) {
  __shared__ float part[kThreads / 32];
  x += (size_t)blockIdx.x * dim;
  out += (size_t)blockIdx.x * dim;
  float ss = 0.0f;
  const bool vec = (dim & 3) == 0;
  if (vec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
#pragma unroll 8
    for (int i = threadIdx.x; i < (dim >> 2); i += blockDim.x) {
      const float4 v = x4[i];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += x[i] * x[i];
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) total += part[i];
  const float inv = 1.0f / sqrtf(total / (float)dim + eps);
  if (vec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x), *w4 = reinterpret_cast<const float4 *>(w);
    float4 *o4 = reinterpret_cast<float4 *>(out);
#pragma unroll 8
    for (int i = threadIdx.x; i < (dim >> 2); i += blockDim.x) {
      const float4 v = x4[i], g = w4[i];
      o4[i] = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = x[i] * inv * w[i];
  }
}

// Rope (src/ops.cc ApplyRopeNormalToHeads) of q and k of row t, then the K/V
// store into the row's request cache at (layer, positions[t]) (the reference's
// RopeKernel + StoreKvKernel). qkv rows: [q (heads x hd) | k (kv x hd) | v], row
// stride `ld`. Pair i of a head rotates by pos / theta^(2i / head_dim); NeoX
// pairs (i, i + hd/2), normal (2i, 2i + 1). Thread p: q pair p, k pair p (and
// the two v elements at the same places).
__global__ void RopeStoreKernel(float *qkv, int ld, int heads, int kv_heads, int hd, const int *positions,
                                float theta, bool neox, float *const *keys, float *const *values, const int *request,
                                int layer, int max_seq) {
  const int t = blockIdx.y, p = blockIdx.x * blockDim.x + threadIdx.x, half = hd / 2;
  float *row = qkv + (size_t)t * ld;
  const int pos = positions[t];
  auto rotate = [&](float *x, int pair, int &a, int &b) {
    const int head = pair / half, i = 2 * (pair % half);
    const float freq = 1.0f / powf(theta, (float)i / (float)hd);
    const float angle = (float)pos * freq;
    const float c = cosf(angle), s = sinf(angle);
    a = head * hd + (neox ? i / 2 : i);
    b = neox ? a + half : a + 1;
    const float x0 = x[a], x1 = x[b];
    x[a] = x0 * c - x1 * s;
    x[b] = x0 * s + x1 * c;
  };
  int a, b;
  if (p < heads * half) rotate(row, p, a, b);
  if (p < kv_heads * half) {
    float *k = row + (size_t)heads * hd, *v = k + (size_t)kv_heads * hd;
    rotate(k, p, a, b);
    const size_t base = ((size_t)layer * max_seq + pos) * kv_heads * hd;
    float *kc = keys[request[t]] + base, *vc = values[request[t]] + base;
    kc[a] = k[a];
    kc[b] = k[b];
    vc[a] = v[a];
    vc[b] = v[b];
  }
}

// Attention of query head h of row t over its request's positions
// 0..positions[t] (AttentionForward, src/forward.cc): scores = q . k_s /
// sqrt(hd), softmax (exp(x - max) / sum, src/ops.cc Softmax), weighted sum of
// v_s; KV head h / (heads / kv_heads). Grid (heads, rows). Scores: one thread
// per position, its K row read as float4 (unrolled: the loads of a row are in
// flight together); values: each warp sums a stride of positions for its
// float4 columns, and the warps' partial sums are added in a fixed order.
// q rows have stride ld_q. Needs hd % 4 == 0. Shared memory (dynamic): q [hd],
// scores [max_seq rounded up to 4], partial sums [warps][hd] (16-byte aligned).
__device__ __forceinline__ float BlockReduce(float v, float *red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int i = 1; i < nwarps; ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
  return v;
}

__global__ void AttentionKernel(const float *q, int ld_q, float *const *keys, float *const *values,
                                const int *request, const int *positions, float *out, int hd, int heads, int kv_heads,
                                int max_seq, int layer) {
  extern __shared__ float4 sm4[];  // 16-byte aligned
  float *sm = reinterpret_cast<float *>(sm4);
  __shared__ float red[32];
  const int h = blockIdx.x, t = blockIdx.y, kh = h / (heads / kv_heads), pos = positions[t];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5, hd4 = hd >> 2;
  const size_t stride = (size_t)kv_heads * hd;  // floats between positions
  const float *kc = keys[request[t]] + (size_t)layer * max_seq * stride + (size_t)kh * hd;
  const float *vc = values[request[t]] + (size_t)layer * max_seq * stride + (size_t)kh * hd;
  // part is read and written as float4: its offset is rounded up to 4 floats
  float *qs = sm, *scores = sm + hd, *part = scores + ((max_seq + 3) & ~3);
  const float *qt = q + (size_t)t * ld_q + (size_t)h * hd;
  for (int i = tid; i < hd; i += blockDim.x) qs[i] = qt[i];
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)hd);
  const float4 *q4 = reinterpret_cast<const float4 *>(qs);
  for (int s = tid; s <= pos; s += blockDim.x) {
    const float4 *kp = reinterpret_cast<const float4 *>(kc + (size_t)s * stride);
    float dot = 0.0f;
#pragma unroll 8
    for (int c = 0; c < hd4; ++c) {
      const float4 k4 = kp[c], qq = q4[c];
      dot += qq.x * k4.x + qq.y * k4.y + qq.z * k4.z + qq.w * k4.w;
    }
    scores[s] = dot * scale;
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int s = tid; s <= pos; s += blockDim.x) mx = fmaxf(mx, scores[s]);
  mx = BlockReduce(mx, red, true);
  float sum = 0.0f;
  for (int s = tid; s <= pos; s += blockDim.x) {
    const float e = expf(scores[s] - mx);
    scores[s] = e;
    sum += e;
  }
  sum = BlockReduce(sum, red, false);
  for (int s = tid; s <= pos; s += blockDim.x) scores[s] = scores[s] / sum;
  __syncthreads();
  for (int c = lane; c < hd4; c += 32) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int s = warp; s <= pos; s += nwarps) {
      const float4 v4 = reinterpret_cast<const float4 *>(vc + (size_t)s * stride)[c];
      const float pr = scores[s];
      acc.x += pr * v4.x, acc.y += pr * v4.y, acc.z += pr * v4.z, acc.w += pr * v4.w;
    }
    reinterpret_cast<float4 *>(part + (size_t)warp * hd)[c] = acc;
  }
  __syncthreads();
  float *ot = out + (size_t)t * heads * hd + (size_t)h * hd;
  for (int e = tid; e < hd; e += blockDim.x) {
    float v = 0.0f;
    for (int w = 0; w < nwarps; ++w) v += part[(size_t)w * hd + e];
    ot[e] = v;
  }
}

size_t AttentionSmem(const ModelConfig &c) {
  return ((size_t)c.head_dim + (((size_t)c.max_seq_len + 3) & ~size_t(3)) + (size_t)(kThreads / 32) * c.head_dim) *
         sizeof(float);
}

// F32 projection of row t: y[t][n] = W[n] . x[t] (+ bias[n]) (+ residual[t][n]),
// one warp per output; y and residual rows have stride ldy.
__global__ void LinearF32Kernel(const float *x, const float *w, int rows, int cols, const float *bias,
                                const float *residual, float *y, int ldy) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31, t = blockIdx.y;
  if (row >= rows) return;
  const float *wr = w + (size_t)row * cols, *xr = x + (size_t)t * cols;
  float dot = 0.0f;
  for (int c = lane; c < cols; c += 32) dot += wr[c] * xr[c];
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) {
    float v = dot + (bias ? bias[row] : 0.0f);
    if (residual) v += residual[(size_t)t * ldy + row];
    y[(size_t)t * ldy + row] = v;
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
    // q, k and v of one packed type as one weight (rows [q | k | v]) and bias:
    // one product per layer instead of three. q, k, v are then unset.
    DeviceWeight qkv;
    const float *bqkv = nullptr;
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
    DeviceBuffer x, norm, qkv, attention, gate, up, last, logits, meta;
    void *host_meta = nullptr;    // pinned staging of the row metadata
    float *host_logits = nullptr;  // pinned staging of the logits
  } scratch;
  // The forward's launches run on `stream`. A row-block shape (rows,
  // requests) that recurs gets a stream of its own: its second call runs
  // there (the engine sizes that stream's scratch for exactly this shape, so
  // it never moves afterwards), its third is captured into a CUDA graph, and
  // every later call replays the graph. Tokens, positions, requests and cache
  // pointers are read from the metadata buffer, so one graph serves every
  // decode step of that shape.
  cudaStream_t stream = nullptr;
  struct Captured {
    cudaStream_t stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    unsigned long long linear_calls = 0, activation_calls = 0, attention_calls = 0;
  };
  static constexpr int kMaxGraphs = 64;
  std::map<std::pair<int, int>, Captured> graphs;  // by shape; exec null until captured
  std::map<std::pair<int, int>, int> seen;

  explicit CudaModelState(int id) : device(id) {}
  ~CudaModelState() {
    cudaSetDevice(device);
    DropGraphs();
    if (stream) cudaStreamDestroy(stream);
    if (scratch.host_meta) cudaFreeHost(scratch.host_meta);
    if (scratch.host_logits) cudaFreeHost(scratch.host_logits);
    for (mq_weight *w : handles) mq_weight_destroy(w);
  }
  void DropGraphs() {
    for (auto &g : graphs) {
      if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
      if (g.second.stream) cudaStreamDestroy(g.second.stream);
    }
    graphs.clear();
    seen.clear();
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
  DeviceWeight UploadPacked(int type, int rows, int cols, const std::vector<uint8_t> &bytes) {
    ++uploaded_weights;
    DeviceWeight w;
    mq_weight *h = nullptr;
    CheckMq(mq_weight_create(device, type, rows, cols, bytes.data(), bytes.size(), 0, nullptr, &h), "upload weight");
    handles.push_back(h);
    uploaded_bytes += bytes.size();
    w.packed = h;
    w.rows = rows;
    w.cols = cols;
    return w;
  }
  DeviceWeight UploadWeight(const Tensor &t) {
    if (t.quantized) {
      const QuantizedStorage &s = *t.quantized;
      return UploadPacked(static_cast<int>(s.type), s.rows, s.cols, s.bytes);
    }
    ++uploaded_weights;
    DeviceWeight w;
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
    if (!stream) Check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    if (rows <= scratch.rows && requests <= scratch.requests) return;
    DropGraphs();  // the graphs hold the old scratch addresses
    rows = std::max(rows, scratch.rows);
    requests = std::max(requests, scratch.requests);
    const size_t kv_dim = static_cast<size_t>(c.n_kv_heads) * c.head_dim;
    auto alloc = [&](size_t n) { return DeviceBuffer(n * sizeof(float), device); };
    scratch.x = alloc(rows * (size_t)c.dim);
    scratch.norm = alloc(rows * (size_t)c.dim);
    scratch.qkv = alloc(rows * ((size_t)c.dim + 2 * kv_dim));
    scratch.attention = alloc(rows * (size_t)c.dim);
    scratch.gate = alloc(rows * (size_t)c.hidden_dim);
    scratch.up = alloc(rows * (size_t)c.hidden_dim);
    scratch.last = alloc(requests * (size_t)c.dim);
    scratch.logits = alloc(requests * (size_t)c.vocab_size);
    const size_t meta_bytes = (3 * (size_t)rows + requests) * sizeof(int) + 16 + 2 * requests * sizeof(float *);
    scratch.meta = DeviceBuffer(meta_bytes, device);
    if (scratch.host_meta) cudaFreeHost(scratch.host_meta);
    if (scratch.host_logits) cudaFreeHost(scratch.host_logits);
    scratch.host_meta = scratch.host_logits = nullptr;
    Check(cudaMallocHost(&scratch.host_meta, meta_bytes), "cudaMallocHost");
    Check(cudaMallocHost(reinterpret_cast<void **>(&scratch.host_logits),
                         (size_t)requests * c.vocab_size * sizeof(float)),
          "cudaMallocHost");
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
  const int kv_dim = c.n_kv_heads * c.head_dim, QS = c.dim + 2 * kv_dim;  // qkv row: [q | k | v]
  gpu.Reserve(c, M, R);
  auto &sc = gpu.scratch;
  const auto key = std::make_pair(M, R);
  const int uses = ++gpu.seen[key];
  auto shape = gpu.graphs.find(key);
  if (shape == gpu.graphs.end() && uses >= 2 && (int)gpu.graphs.size() < CudaModelState::kMaxGraphs) {
    CudaModelState::Captured fresh;
    Check(cudaStreamCreateWithFlags(&fresh.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    shape = gpu.graphs.emplace(key, fresh).first;
  }
  cudaStream_t st = shape == gpu.graphs.end() ? gpu.stream : shape->second.stream;
  // Row metadata and the requests' cache pointers: one host-to-device copy
  // from pinned staging (the previous call's copies completed before it returned).
  const size_t ints = 3 * (size_t)sc.rows + sc.requests;
  const size_t ptr_off = (ints * sizeof(int) + 15) & ~size_t(15);
  int *im = static_cast<int *>(sc.host_meta);
  std::memcpy(im, tokens.data(), M * sizeof(int));
  std::memcpy(im + sc.rows, positions.data(), M * sizeof(int));
  for (int r = 0; r < R; ++r) {
    for (int t = offsets[r]; t < offsets[r + 1]; ++t) im[2 * sc.rows + t] = r;
    im[3 * sc.rows + r] = offsets[r + 1] - 1;
  }
  float **ptrs = reinterpret_cast<float **>(static_cast<uint8_t *>(sc.host_meta) + ptr_off);
  for (int r = 0; r < R; ++r) {
    ptrs[r] = states[r]->keys.floats();
    ptrs[R + r] = states[r]->values.floats();
  }
  Check(cudaMemcpyAsync(sc.meta.get(), sc.host_meta, ptr_off + 2 * R * sizeof(float *), cudaMemcpyHostToDevice, st),
        "upload batch rows");
  const int *d_tokens = static_cast<const int *>(sc.meta.get());
  const int *d_pos = d_tokens + sc.rows, *d_req = d_tokens + 2 * sc.rows, *d_last = d_tokens + 3 * sc.rows;
  float *const *d_keys = reinterpret_cast<float *const *>(static_cast<uint8_t *>(sc.meta.get()) + ptr_off);
  float *const *d_values = d_keys + R;
  // The scores of a row cover positions 0..pos <= max_seq_len - 1: one size for every step.
  if (c.head_dim % 4 != 0) throw std::runtime_error("CUDA attention needs head_dim % 4 == 0");
  const size_t score_bytes = AttentionSmem(c);
  if (score_bytes > 227 * 1024) throw std::runtime_error("CUDA attention: max_seq_len too large for shared memory");
  if (score_bytes > 48 * 1024)
    Check(cudaFuncSetAttribute(AttentionKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_bytes),
          "attention shared memory");

  CudaModelState::Captured counts;
  auto launch_all = [&]() {
    // y = W x (+ bias) (+ residual; y may be the residual), `rows` rows.
    auto linear = [&](const DeviceWeight &w, const float *x, int rows, float *y, const float *bias,
                      const float *residual) {
      if (w.packed) {
        if (residual)
          CheckMq(mq_linear_residual(w.packed, x, rows, w.cols, bias, residual, y, w.rows, st), "CUDA linear");
        else
          CheckMq(mq_linear(w.packed, x, rows, w.cols, bias, y, w.rows, st), "CUDA linear");
      } else {
        LinearF32Kernel<<<dim3((w.rows + 7) / 8, rows), kThreads, 0, st>>>(x, w.dense, w.rows, w.cols, bias,
                                                                           residual, y, w.rows);
      }
      ++counts.linear_calls;
    };
    // q / k / v: the ragged rows of all requests in one call, into the qkv rows (stride QS).
    auto project = [&](const DeviceWeight &w, const float *x, float *y, const float *bias) {
      if (w.packed)
        CheckMq(mq_linear_ragged(w.packed, x, offsets.data(), R, w.cols, bias, y, QS, st), "CUDA linear");
      else
        LinearF32Kernel<<<dim3((w.rows + 7) / 8, M), kThreads, 0, st>>>(x, w.dense, w.rows, w.cols, bias, nullptr,
                                                                        y, QS);
      ++counts.linear_calls;
    };
    auto norm = [&](const float *input, const float *weight, int rows, float *output) {
      NormKernel<<<rows, kThreads, 0, st>>>(input, weight, c.dim, c.rms_norm_eps, output);
      ++counts.activation_calls;
    };
    EmbedKernel<<<dim3(Grid(c.dim), M), kThreads, 0, st>>>(gpu.embedding, d_tokens, c.dim, sc.x.floats());
    const bool neox = c.rope_type == RopeType::kNeoX;
    float *qkv = sc.qkv.floats();
    for (int i = 0; i < c.n_layers; ++i) {
      const auto &layer = gpu.layers[i];
      norm(sc.x.floats(), layer.norm, M, sc.norm.floats());
      if (layer.qkv.packed || layer.qkv.dense) {
        project(layer.qkv, sc.norm.floats(), qkv, layer.bqkv);
        counts.linear_calls += 2;  // q, k and v
      } else {
        project(layer.q, sc.norm.floats(), qkv, layer.bq);
        project(layer.k, sc.norm.floats(), qkv + c.dim, layer.bk);
        project(layer.v, sc.norm.floats(), qkv + c.dim + kv_dim, layer.bv);
      }
      RopeStoreKernel<<<dim3(Grid(std::max(c.dim, kv_dim) / 2), M), kThreads, 0, st>>>(
          qkv, QS, c.n_heads, c.n_kv_heads, c.head_dim, d_pos, c.rope_theta, neox, d_keys, d_values, d_req, i,
          c.max_seq_len);
      AttentionKernel<<<dim3(c.n_heads, M), kThreads, score_bytes, st>>>(qkv, QS, d_keys, d_values, d_req, d_pos,
                                                                         sc.attention.floats(), c.head_dim,
                                                                         c.n_heads, c.n_kv_heads, c.max_seq_len, i);
      ++counts.attention_calls;
      linear(layer.o, sc.attention.floats(), M, sc.x.floats(), nullptr, sc.x.floats());  // x += wo . attn
      norm(sc.x.floats(), layer.ffn_norm, M, sc.norm.floats());
      if (layer.gate.packed && layer.up.packed) {  // SwiGlu(gate, up) fused into the up product's output
        CheckMq(mq_linear_swiglu(layer.gate.packed, layer.up.packed, sc.norm.floats(), M, c.dim, sc.gate.floats(),
                                 layer.up.rows, st),
                "CUDA linear");
        counts.linear_calls += 2;
      } else {
        linear(layer.gate, sc.norm.floats(), M, sc.gate.floats(), nullptr, nullptr);
        linear(layer.up, sc.norm.floats(), M, sc.up.floats(), nullptr, nullptr);
        SwiGluKernel<<<Grid((size_t)M * c.hidden_dim), kThreads, 0, st>>>(sc.gate.floats(), sc.up.floats(),
                                                                         (size_t)M * c.hidden_dim);
      }
      linear(layer.down, sc.gate.floats(), M, sc.x.floats(), nullptr, sc.x.floats());  // x += w_down . h
      counts.activation_calls += 5;
    }
    GatherRowsKernel<<<dim3(Grid(c.dim), R), kThreads, 0, st>>>(sc.x.floats(), d_last, c.dim, sc.last.floats());
    norm(sc.last.floats(), gpu.final_norm, R, sc.norm.floats());
    linear(gpu.output, sc.norm.floats(), R, sc.logits.floats(), nullptr, nullptr);
  };

  if (shape != gpu.graphs.end() && shape->second.exec) {
    Check(cudaGraphLaunch(shape->second.exec, st), "forward graph launch");
    counts.linear_calls = shape->second.linear_calls;
    counts.activation_calls = shape->second.activation_calls;
    counts.attention_calls = shape->second.attention_calls;
  } else if (shape == gpu.graphs.end() || uses == 2) {
    launch_all();  // plain launches (on a shape's own stream: sizes the engine's scratch of that stream)
    Check(cudaGetLastError(), "CUDA forward kernel launch");
  } else {  // third call of a shape: capture on its stream, then replay from now on
    cudaGraph_t graph = nullptr;
    Check(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin forward capture");
    try {
      launch_all();
    } catch (...) {
      cudaStreamEndCapture(st, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    Check(cudaStreamEndCapture(st, &graph), "end forward capture");
    CudaModelState::Captured &cap = shape->second;
    const cudaError_t e = cudaGraphInstantiate(&cap.exec, graph, 0);
    cudaGraphDestroy(graph);
    Check(e, "forward graph instantiate");
    cap.linear_calls = counts.linear_calls;
    cap.activation_calls = counts.activation_calls;
    cap.attention_calls = counts.attention_calls;
    Check(cudaGraphLaunch(cap.exec, st), "forward graph launch");
  }
  // Sampling stays on the CPU: only the final logits come back, as in the reference.
  const size_t bytes = (size_t)R * c.vocab_size * sizeof(float);
  Check(cudaMemcpyAsync(sc.host_logits, sc.logits.get(), bytes, cudaMemcpyDeviceToHost, st), "download logits");
  Check(cudaStreamSynchronize(st), "CUDA forward");
  std::memcpy(logits, sc.host_logits, bytes);
  for (CudaContextState *cs : states) {  // every request of the block took part in every call
    cs->linear_calls += counts.linear_calls;
    cs->activation_calls += counts.activation_calls;
    cs->attention_calls += counts.attention_calls;
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
    const QuantizedStorage *sq = layer.wq.quantized.get(), *sk = layer.wk.quantized.get(),
                           *sv = layer.wv.quantized.get();
    if (sq && sk && sv && sq->type == sk->type && sq->type == sv->type && sq->cols == sk->cols &&
        sq->cols == sv->cols) {  // one packed weight [q | k | v]: the GGUF rows concatenate
      std::vector<uint8_t> bytes(sq->bytes);
      bytes.insert(bytes.end(), sk->bytes.begin(), sk->bytes.end());
      bytes.insert(bytes.end(), sv->bytes.begin(), sv->bytes.end());
      up.qkv = gpu->UploadPacked(static_cast<int>(sq->type), sq->rows + sk->rows + sv->rows, sq->cols, bytes);
      gpu->uploaded_weights += 2;  // three projections
      if (!layer.bq.data.empty() || !layer.bk.data.empty() || !layer.bv.data.empty()) {
        Tensor b({sq->rows + sk->rows + sv->rows}, 0.0f);
        auto put = [&](const Tensor &t, int at) {
          std::copy(t.data.begin(), t.data.end(), b.data.begin() + at);
        };
        put(layer.bq, 0);
        put(layer.bk, sq->rows);
        put(layer.bv, sq->rows + sk->rows);
        up.bqkv = gpu->UploadFloat(b);
      }
    } else {
      up.q = gpu->UploadWeight(layer.wq);
      up.k = gpu->UploadWeight(layer.wk);
      up.v = gpu->UploadWeight(layer.wv);
    }
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

void PrepareCudaContext(MiniLlamaContext &context, const MiniLlamaModel &model) { StateOf(context, model); }

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
  // One weight whose rows are the given parts stacked (each part its own
  // random stream): q, k, v become one [q | k | v] weight.
  auto stacked = [&](std::vector<int> parts, int cols) {
    DeviceWeight w;
    int rows = 0;
    for (int p : parts) rows += p;
    w.rows = rows;
    w.cols = cols;
    gpu->uploaded_weights += static_cast<int>(parts.size());
    if (type == 0) {
      gpu->allocations.emplace_back((size_t)rows * cols * sizeof(float), device);
      float *dst = gpu->allocations.back().floats();
      for (int p : parts) {
        NormalKernel<<<1184, kThreads>>>(dst, (size_t)p * cols, 0.02f, seed, stream_id++);
        dst += (size_t)p * cols;
      }
      Check(cudaGetLastError(), "random weights");
      gpu->uploaded_bytes += (size_t)rows * cols * sizeof(float);
      w.dense = gpu->allocations.back().floats();
      return w;
    }
    const size_t nbytes = mq_quantized_bytes(type, rows, cols);
    DeviceBuffer blocks(nbytes, device);
    size_t at = 0;
    for (int p : parts) {  // the GGUF block stream of the stacked rows is the parts' streams in order
      NormalKernel<<<1184, kThreads>>>(tmp.floats(), (size_t)p * cols, 0.02f, seed, stream_id++);
      Check(cudaGetLastError(), "random weights");
      const size_t pb = mq_quantized_bytes(type, p, cols);
      CheckMq(mq_quantize_device(device, type, tmp.floats(), p, cols, static_cast<uint8_t *>(blocks.get()) + at, pb,
                                 nullptr),
              "quantize");
      at += pb;
    }
    mq_weight *h = nullptr;
    CheckMq(mq_weight_create(device, type, rows, cols, blocks.get(), nbytes, 1, nullptr, &h), "upload weight");
    Check(cudaDeviceSynchronize(), "upload weight");
    gpu->handles.push_back(h);
    gpu->uploaded_bytes += nbytes;
    w.packed = h;
    return w;
  };
  auto weight = [&](int rows, int cols) { return stacked({rows}, cols); };
  gpu->embedding = dense((size_t)c.vocab_size * c.dim, 1.0f, false);
  gpu->final_norm = dense(c.dim, 1.0f, true);
  for (int i = 0; i < c.n_layers; ++i) {
    CudaModelState::Layer l;
    l.norm = dense(c.dim, 1.0f, true);
    l.ffn_norm = dense(c.dim, 1.0f, true);
    l.qkv = stacked({c.dim, (int)kv_dim, (int)kv_dim}, c.dim);
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
    if (g.qkv.packed || g.qkv.dense) {  // split the stacked weight back into q, k, v
      const Tensor all = matrix(g.qkv);
      const int kv = c.n_kv_heads * c.head_dim, rows[3] = {c.dim, kv, kv};
      Tensor *dst[3] = {&l.wq, &l.wk, &l.wv};
      size_t at = 0;
      for (int j = 0; j < 3; ++j) {
        if (all.quantized) {
          const QuantizedStorage &qs = *all.quantized;
          const size_t row_bytes = qs.bytes.size() / qs.rows;
          std::vector<uint8_t> part(qs.bytes.begin() + at, qs.bytes.begin() + at + row_bytes * rows[j]);
          at += row_bytes * rows[j];
          *dst[j] = TensorFromQuantized(std::move(part), rows[j], qs.cols, qs.type);
        } else {
          Tensor t({rows[j], c.dim});
          std::copy(all.data.begin() + at, all.data.begin() + at + t.data.size(), t.data.begin());
          at += t.data.size();
          *dst[j] = std::move(t);
        }
      }
    } else {
      l.wq = matrix(g.q);
      l.wk = matrix(g.k);
      l.wv = matrix(g.v);
    }
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
