// mini_ai's CUDA backend (include/mini_llama/backend.h: EnableCuda,
// CudaDeviceInfo, CudaStats, ForwardCuda) rebuilt over the mq_b200 C ABI.
//
// This file takes the place of the reference's src/cuda_backend.cu in a
// mini_ai build: forward.cc calls ForwardCuda for a model that EnableCuda
// uploaded (src/forward.cc:160), and every projection of the token forward
// (q, k, v, o, gate, up, down and lm_head) goes through include/mq_b200.h:
//   - quantized weights (QuantizeModel / GGUF Q8_0, Q4_0, Q4_1) are uploaded
//     with mq_weight_create from their packed blocks (UploadWeight,
//     src/cuda_backend.cu:275-283) and multiplied by mq_linear (q/k/v with
//     their biases), mq_linear_residual (wo and w_down, the residual adds of
//     src/cuda_backend.cu:426-434 in the same kernel) and mq_linear_swiglu
//     (gate/up with SwiGluKernel, src/cuda_backend.cu:241-245);
//   - F32 weights, the embedding, RMSNorm, RoPE, the KV cache and attention
//     run on the small kernels below (the reference's EmbedKernel, NormKernel,
//     RopeKernel, StoreKvKernel, Scores/Softmax/AttentionKernel,
//     src/cuda_backend.cu:112-234), following the CPU forward's formulas
//     (src/forward.cc, src/ops.cc).
// Errors are C++ exceptions as in the reference: a failing CUDA call or ABI
// call throws std::runtime_error("<operation>: <message>") (Check,
// src/cuda_backend.cu:17-21). CudaStats reports the same counters as the
// reference (src/cuda_backend.cu:446-460).
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <limits>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

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

__global__ void EmbedKernel(const float *embedding, int token, int dim, float *out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dim) out[i] = embedding[(size_t)token * dim + i];
}

// RmsNorm (src/ops.cc): x * 1 / sqrt(mean(x^2) + eps) * w, one CTA.
__global__ void NormKernel(const float *x, const float *w, int dim, float eps, float *out) {
  __shared__ float part[kThreads / 32];
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
__global__ void RopeKernel(float *x, int heads, int hd, int pos, float theta, bool neox) {
  const int pair = blockIdx.x * blockDim.x + threadIdx.x;
  if (pair >= heads * (hd / 2)) return;
  const int head = pair / (hd / 2), i = 2 * (pair % (hd / 2));
  const float freq = 1.0f / powf(theta, (float)i / (float)hd);
  const float angle = (float)pos * freq;
  const float c = cosf(angle), s = sinf(angle);
  const int a = head * hd + (neox ? i / 2 : i);
  const int b = neox ? a + hd / 2 : a + 1;
  const float x0 = x[a], x1 = x[b];
  x[a] = x0 * c - x1 * s;
  x[b] = x0 * s + x1 * c;
}

__global__ void StoreKvKernel(const float *k, const float *v, float *keys, float *values, size_t offset, int count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) {
    keys[offset + i] = k[i];
    values[offset + i] = v[i];
  }
}

// Attention of one query head over positions 0..pos (AttentionForward,
// src/forward.cc): scores = q . k_t / sqrt(hd), softmax, weighted sum of v_t.
// One CTA per head; the scores live in dynamic shared memory.
__global__ void AttentionKernel(const float *q, const float *keys, const float *values, float *out, int pos, int hd,
                                int heads, int kv_heads, int max_seq, int layer) {
  extern __shared__ float scores[];
  __shared__ float red[kThreads / 32];
  const int h = blockIdx.x, kh = h / (heads / kv_heads);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const float scale = 1.0f / sqrtf((float)hd);
  for (int t = warp; t <= pos; t += nwarps) {
    const float *kp = keys + (((size_t)layer * max_seq + t) * kv_heads + kh) * hd;
    float dot = 0.0f;
    for (int d = lane; d < hd; d += 32) dot += q[h * hd + d] * kp[d];
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) scores[t] = dot * scale;
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int t = threadIdx.x; t <= pos; t += blockDim.x) mx = fmaxf(mx, scores[t]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < nwarps; ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.0f;
  for (int t = threadIdx.x; t <= pos; t += blockDim.x) {
    const float e = expf(scores[t] - mx);
    scores[t] = e;
    sum += e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.0f;
  for (int i = 0; i < nwarps; ++i) sum += red[i];
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int t = 0; t <= pos; ++t)
      acc += (scores[t] / sum) * values[(((size_t)layer * max_seq + t) * kv_heads + kh) * hd + d];
    out[h * hd + d] = acc;
  }
}

// F32 projection: y[n] = W[n] . x (+ bias[n]) (+ residual[n]), one warp per row.
__global__ void LinearF32Kernel(const float *x, const float *w, int rows, int cols, const float *bias,
                                const float *residual, float *y) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *wr = w + (size_t)row * cols;
  float dot = 0.0f;
  for (int c = lane; c < cols; c += 32) dot += wr[c] * x[c];
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) {
    float v = dot + (bias ? bias[row] : 0.0f);
    if (residual) v += residual[row];
    y[row] = v;
  }
}

// SwiGlu (src/ops.cc): g * sigmoid(g) * u, in place on the gate.
__global__ void SwiGluKernel(float *gate, const float *up, int count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) {
    const float g = gate[i];
    gate[i] = g * (1.0f / (1.0f + expf(-g))) * up[i];
  }
}

int Grid(int count) { return (count + kThreads - 1) / kThreads; }

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
};

struct CudaContextState {
  std::shared_ptr<CudaModelState> owner;
  DeviceBuffer keys, values, x, norm, q, k, v, attention, gate, up, logits;
  unsigned long long linear_calls = 0, activation_calls = 0, attention_calls = 0, d2h_bytes = 0;

  CudaContextState(const std::shared_ptr<CudaModelState> &model, const ModelConfig &c) : owner(model) {
    const size_t kv_dim = static_cast<size_t>(c.n_kv_heads) * c.head_dim;
    if (kv_dim > std::numeric_limits<size_t>::max() / c.n_layers / c.max_seq_len)
      throw std::runtime_error("CUDA KV cache size overflow");
    const size_t elements = kv_dim * c.n_layers * c.max_seq_len;
    if (elements > std::numeric_limits<size_t>::max() / sizeof(float))
      throw std::runtime_error("CUDA KV cache size overflow");
    auto alloc = [&](size_t n) { return DeviceBuffer(n * sizeof(float), model->device); };
    keys = alloc(elements);
    values = alloc(elements);
    Check(cudaMemset(keys.get(), 0, elements * sizeof(float)), "clear keys");
    Check(cudaMemset(values.get(), 0, elements * sizeof(float)), "clear values");
    x = alloc(c.dim);
    norm = alloc(c.dim);
    q = alloc(c.dim);
    k = alloc(kv_dim);
    v = alloc(kv_dim);
    attention = alloc(c.dim);
    gate = alloc(c.hidden_dim);
    up = alloc(c.hidden_dim);
    logits = alloc(c.vocab_size);
  }
};

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
  const auto &c = model.config;
  Check(cudaSetDevice(model.cuda->device), "cudaSetDevice");
  if (!context.cuda) context.cuda = std::make_shared<CudaContextState>(model.cuda, c);
  auto &st = *context.cuda;
  if (st.owner != model.cuda) throw std::runtime_error("CUDA context belongs to another model");
  const auto &gpu = *model.cuda;
  const int kv_dim = c.n_kv_heads * c.head_dim;
  // y = W x (+ bias) (+ residual; y may be the residual).
  auto linear = [&](const DeviceWeight &w, const float *x, float *y, const float *bias, const float *residual) {
    if (w.packed) {
      if (residual)
        CheckMq(mq_linear_residual(w.packed, x, 1, w.cols, bias, residual, y, w.rows, nullptr), "CUDA linear");
      else
        CheckMq(mq_linear(w.packed, x, 1, w.cols, bias, y, w.rows, nullptr), "CUDA linear");
    } else {
      LinearF32Kernel<<<(w.rows + 7) / 8, 256>>>(x, w.dense, w.rows, w.cols, bias, residual, y);
    }
    ++st.linear_calls;
  };
  auto norm = [&](const float *input, const float *weight, float *output) {
    NormKernel<<<1, kThreads>>>(input, weight, c.dim, c.rms_norm_eps, output);
    ++st.activation_calls;
  };
  EmbedKernel<<<Grid(c.dim), kThreads>>>(gpu.embedding, token, c.dim, st.x.floats());
  const bool neox = c.rope_type == RopeType::kNeoX;
  for (int i = 0; i < c.n_layers; ++i) {
    const auto &layer = gpu.layers[i];
    norm(st.x.floats(), layer.norm, st.norm.floats());
    linear(layer.q, st.norm.floats(), st.q.floats(), layer.bq, nullptr);
    linear(layer.k, st.norm.floats(), st.k.floats(), layer.bk, nullptr);
    linear(layer.v, st.norm.floats(), st.v.floats(), layer.bv, nullptr);
    RopeKernel<<<Grid(c.dim / 2), kThreads>>>(st.q.floats(), c.n_heads, c.head_dim, context.pos, c.rope_theta, neox);
    RopeKernel<<<Grid(kv_dim / 2), kThreads>>>(st.k.floats(), c.n_kv_heads, c.head_dim, context.pos, c.rope_theta,
                                                neox);
    const size_t offset = (static_cast<size_t>(i) * c.max_seq_len + context.pos) * kv_dim;
    StoreKvKernel<<<Grid(kv_dim), kThreads>>>(st.k.floats(), st.v.floats(), st.keys.floats(), st.values.floats(),
                                              offset, kv_dim);
    AttentionKernel<<<c.n_heads, kThreads, (size_t)(context.pos + 1) * sizeof(float)>>>(
        st.q.floats(), st.keys.floats(), st.values.floats(), st.attention.floats(), context.pos, c.head_dim,
        c.n_heads, c.n_kv_heads, c.max_seq_len, i);
    ++st.attention_calls;
    linear(layer.o, st.attention.floats(), st.x.floats(), nullptr, st.x.floats());  // x += wo . attn
    norm(st.x.floats(), layer.ffn_norm, st.norm.floats());
    if (layer.gate.packed && layer.up.packed) {  // SwiGlu(gate, up) fused into the up product's output
      CheckMq(mq_linear_swiglu(layer.gate.packed, layer.up.packed, st.norm.floats(), 1, c.dim, st.gate.floats(),
                               layer.up.rows, nullptr),
              "CUDA linear");
      st.linear_calls += 2;
    } else {
      linear(layer.gate, st.norm.floats(), st.gate.floats(), nullptr, nullptr);
      linear(layer.up, st.norm.floats(), st.up.floats(), nullptr, nullptr);
      SwiGluKernel<<<Grid(c.hidden_dim), kThreads>>>(st.gate.floats(), st.up.floats(), c.hidden_dim);
    }
    linear(layer.down, st.gate.floats(), st.x.floats(), nullptr, st.x.floats());  // x += w_down . h
    st.activation_calls += 5;
  }
  norm(st.x.floats(), gpu.final_norm, st.norm.floats());
  linear(gpu.output, st.norm.floats(), st.logits.floats(), nullptr, nullptr);
  Check(cudaGetLastError(), "CUDA forward kernel launch");
  Tensor output({c.vocab_size});
  // Sampling stays on the CPU: only the final logits come back, as in the reference.
  Check(cudaMemcpy(output.data.data(), st.logits.get(), output.size() * sizeof(float), cudaMemcpyDeviceToHost),
        "download logits");
  st.d2h_bytes += output.size() * sizeof(float);
  return output;
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
