// The B200 backend's surface beyond include/mini_llama/backend.h.
//
// backend.h (EnableCuda, CudaDeviceInfo, CudaStats, ForwardCuda) is served by
// b200_backend.cu as the reference's src/cuda_backend.cu serves it. These
// declarations add what that interface has no room for: several requests'
// tokens through each projection at once, the model-level quantizer over the
// engine's packer, and a device-generated random model for the full-size
// forward workload.
#ifndef MINI_AI_B200_ADAPTER_B200_BACKEND_H_
#define MINI_AI_B200_ADAPTER_B200_BACKEND_H_

#include <cstdint>
#include <vector>

#include "mini_llama/batch.h"
#include "mini_llama/context.h"
#include "mini_llama/model.h"
#include "mini_llama/quantized_tensor.h"
#include "mini_llama/tensor.h"

namespace mini_llama {

// ForwardBatch (src/forward.cc:175-203) for several requests at once on a
// model that EnableCuda (or RandomCudaModel) uploaded: contexts[r] runs
// batches[r], its tokens at their positions. All tokens of all requests form
// one ragged row block that goes through every projection in one call
// (mq_linear_ragged for q/k/v, mq_linear_residual for wo and w_down,
// mq_linear_swiglu for gate/up), so a prefill is a tensor-core GEMM and a
// decode step of R requests is an R-row decode product. Positions within a
// batch must increase (a token attends to its request's positions 0..pos,
// with every K/V of the batch stored first). Returns the logits of the last
// token of every batch, in request order, and updates every context as
// ForwardBatch does (pos, token_history, n_prefill_tokens /
// n_decode_tokens). Throws std::runtime_error / std::out_of_range on the
// inputs ForwardBatch and ForwardToken reject.
std::vector<Tensor> ForwardBatchCuda(const std::vector<MiniLlamaContext *> &contexts, const MiniLlamaModel &model,
                                     const std::vector<MiniBatch> &batches);

// Allocates the device KV cache of `context` for `model` now instead of at its
// first forward (so that a timed region does not include the allocation).
void PrepareCudaContext(MiniLlamaContext &context, const MiniLlamaModel &model);

// QuantizeModel (src/quantized_tensor.cc:208-219) over the engine's threaded
// packer (mq_quantize): byte-identical storage, and the same refusal once the
// model is uploaded.
void QuantizeModelB200(MiniLlamaModel &model, QuantType type);

// A model of the given shape whose weights are generated on `device` and never
// exist on the host: embeddings ~N(0, 1), norms 1, projections ~N(0, 0.02)
// packed to `type` by the device quantizer (bit-exact with QuantizeTensor) or
// kept F32 (type 0). Deterministic in `seed`. The returned model has
// loaded = true and `cuda` set; its host tensors are empty.
MiniLlamaModel RandomCudaModel(const ModelConfig &config, int type, uint64_t seed, int device = 0);

// Host copies of the first `layers` layers, the embedding, the final norm and
// the lm_head of a RandomCudaModel (packed weights exported bit-exactly with
// mq_weight_export), as a CPU model of `layers` layers: the reference's CPU
// forward can then be timed on part of the same weights.
MiniLlamaModel HostCopyOfCudaModel(const MiniLlamaModel &model, int layers);

}  // namespace mini_llama

#endif  // MINI_AI_B200_ADAPTER_B200_BACKEND_H_
