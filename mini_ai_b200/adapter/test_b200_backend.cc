// Tests of the B200 backend's surface beyond backend.h, registered in
// mini_ai's own test runner (tests/test_main.cc) and linked with its suite
// by mini_ai_b200/adapter/Makefile. They need a B200.
//
//   b200_batched_forward_matches_cpu   ForwardBatchCuda on several requests at
//       once (ragged prompts, then greedy decode steps of all requests in one
//       call) against the reference CPU ForwardBatch (src/forward.cc:175-203)
//       run request by request: logits within 1e-4 (the tolerance of
//       tests/test_cuda.cc), same context bookkeeping. Tiny model x {normal,
//       NeoX} x {F32, Q8_0, Q4_0, Q4_1}; a 60-row prompt block reaches the
//       tensor-core prefill GEMM, the others the decode kernels.
//   b200_batched_forward_rejects_bad_input   the inputs ForwardBatch and
//       ForwardToken reject, and the batched form's own rules.
//   b200_quantize_model_matches_reference   QuantizeModelB200 against
//       QuantizeModel (src/quantized_tensor.cc:208-219): identical bytes,
//       re-quantization of packed weights, the refusal after EnableCuda.
//   b200_gguf_quantized_model_forward   a GGUF file whose linears are Q8_0 /
//       Q4_0 / Q4_1 blocks, loaded by LoadGgufModel's packed branch
//       (src/gguf_loader.cc:539-545), uploaded from those blocks, and run
//       batched against the CPU forward of the same loaded model.
#include <cstdint>
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "b200_backend.h"
#include "mini_llama/backend.h"
#include "mini_llama/context.h"
#include "mini_llama/forward.h"
#include "mini_llama/gguf.h"
#include "mini_llama/gguf_loader.h"
#include "mini_llama/loader.h"
#include "mini_llama/ops.h"
#include "mini_llama/quantized_tensor.h"
#include "tests/gguf_loader_fixture.h"
#include "tests/test_main.h"

using namespace mini_llama;

namespace {

// Deterministic pseudo-random values in [-scale, scale).
struct Lcg {
  uint64_t s;
  float Next(float scale) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return scale * (static_cast<float>((s >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f);
  }
  int Token(int vocab) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return static_cast<int>((s >> 33) % static_cast<uint64_t>(vocab));
  }
};

bool SameLogits(const Tensor &actual, const Tensor &expected) {
  MINI_LLAMA_ASSERT_EQ(actual.size(), expected.size());
  for (size_t i = 0; i < expected.size(); ++i) MINI_LLAMA_ASSERT_NEAR(actual.data[i], expected.data[i], 1e-4f);
  return true;
}

// Prefill every prompt, then `steps` greedy decode steps of all requests, on
// the CPU model request by request and on the GPU model all at once.
bool RunRequests(const MiniLlamaModel &cpu, const MiniLlamaModel &gpu, const std::vector<std::vector<int>> &prompts,
                 int steps) {
  const size_t R = prompts.size();
  std::vector<MiniLlamaContext> a, b;
  for (size_t r = 0; r < R; ++r) {
    a.emplace_back(&cpu);
    b.emplace_back(&gpu);
  }
  std::vector<MiniLlamaContext *> ctx;
  std::vector<MiniBatch> batches;
  for (size_t r = 0; r < R; ++r) {
    ctx.push_back(&b[r]);
    batches.push_back(MiniBatch::FromTokens(prompts[r], 0));
  }
  std::vector<Tensor> expected(R);
  for (size_t r = 0; r < R; ++r) expected[r] = ForwardBatch(a[r], cpu, batches[r]);
  std::vector<Tensor> actual = ForwardBatchCuda(ctx, gpu, batches);
  MINI_LLAMA_ASSERT_EQ(actual.size(), R);
  for (int step = 0; step <= steps; ++step) {
    for (size_t r = 0; r < R; ++r) {
      if (!SameLogits(actual[r], expected[r])) return false;
      MINI_LLAMA_ASSERT_EQ(a[r].pos, b[r].pos);
      MINI_LLAMA_ASSERT_TRUE(a[r].token_history == b[r].token_history);
      MINI_LLAMA_ASSERT_EQ(a[r].n_prefill_tokens, b[r].n_prefill_tokens);
      MINI_LLAMA_ASSERT_EQ(a[r].n_decode_tokens, b[r].n_decode_tokens);
    }
    if (step == steps) break;
    batches.clear();
    for (size_t r = 0; r < R; ++r) {  // greedy, from the CPU logits
      const int next = ArgMax(expected[r]);
      batches.push_back(MiniBatch::Single(next, a[r].pos + 1));
      expected[r] = ForwardBatch(a[r], cpu, batches[r]);
    }
    actual = ForwardBatchCuda(ctx, gpu, batches);
  }
  return true;
}

std::vector<std::vector<int>> Prompts(const std::vector<int> &lengths, int vocab, uint64_t seed) {
  Lcg g{seed};
  std::vector<std::vector<int>> out;
  for (int n : lengths) {
    std::vector<int> p;
    for (int i = 0; i < n; ++i) p.push_back(g.Token(vocab));
    out.push_back(p);
  }
  return out;
}

bool TestBatchedForward() {
  for (RopeType layout : {RopeType::kNormal, RopeType::kNeoX}) {
    for (int type : {0, 8, 2, 3}) {
      auto cpu = LoadModel("models/tiny/model.json", "models/tiny/model.bin");
      MINI_LLAMA_ASSERT_TRUE(cpu.loaded);
      cpu.config.rope_type = layout;
      for (auto &layer : cpu.layers) {  // biases as tests/test_cuda.cc sets them
        layer.bq = Tensor({cpu.config.dim}, 0.1f);
        const int kv = cpu.config.n_kv_heads * cpu.config.head_dim;
        layer.bk = Tensor({kv}, -0.2f);
        layer.bv = Tensor({kv}, 0.3f);
      }
      if (type) QuantizeModel(cpu, static_cast<QuantType>(type));
      auto gpu = cpu;
      EnableCuda(gpu);
      const int V = cpu.config.vocab_size;
      if (!RunRequests(cpu, gpu, Prompts({5, 1, 9}, V, 11 + type), 4)) return false;  // decode kernels
      if (!RunRequests(cpu, gpu, Prompts({40, 3, 17}, V, 23 + type), 2)) return false;  // 60 rows: prefill GEMM
    }
  }
  return true;
}

template <typename F>
bool Throws(F &&f) {
  try {
    f();
  } catch (const std::exception &) {
    return true;
  }
  return false;
}

bool TestBatchedForwardRejects() {
  auto model = LoadModel("models/tiny/model.json", "models/tiny/model.bin");
  MINI_LLAMA_ASSERT_TRUE(model.loaded);
  QuantizeModel(model, QuantType::kQ80);
  EnableCuda(model);
  MiniLlamaContext c1(&model), c2(&model);
  const int V = model.config.vocab_size, S = model.config.max_seq_len;
  auto run = [&](std::vector<MiniLlamaContext *> ctx, std::vector<MiniBatch> b) { ForwardBatchCuda(ctx, model, b); };
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1}, {MiniBatch{}}); }));                                // empty batch
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1}, {MiniBatch{{1, 2}, {0}}}); }));                     // size mismatch
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1}, {MiniBatch::Single(V, 0)}); }));                    // token range
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1}, {MiniBatch::Single(1, S)}); }));                    // position range
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1}, {MiniBatch{{1, 2}, {3, 3}}}); }));                  // not increasing
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1, &c1}, {MiniBatch::Single(1, 0), MiniBatch::Single(2, 1)}); }));
  MINI_LLAMA_ASSERT_TRUE(Throws([&] { run({&c1, &c2}, {MiniBatch::Single(1, 0)}); }));               // count mismatch
  auto cpu_only = LoadModel("models/tiny/model.json", "models/tiny/model.bin");
  MINI_LLAMA_ASSERT_TRUE(Throws([&] {
    MiniLlamaContext c(&cpu_only);
    std::vector<MiniLlamaContext *> ctx{&c};
    ForwardBatchCuda(ctx, cpu_only, {MiniBatch::Single(1, 0)});
  }));
  MINI_LLAMA_ASSERT_EQ(c1.token_history.size(), 0u);  // rejected calls leave the contexts alone
  return true;
}

bool SameStorage(const Tensor &a, const Tensor &b) {
  MINI_LLAMA_ASSERT_TRUE(a.quantized && b.quantized);
  MINI_LLAMA_ASSERT_EQ(static_cast<int>(a.quantized->type), static_cast<int>(b.quantized->type));
  MINI_LLAMA_ASSERT_EQ(a.quantized->rows, b.quantized->rows);
  MINI_LLAMA_ASSERT_EQ(a.quantized->cols, b.quantized->cols);
  MINI_LLAMA_ASSERT_TRUE(a.quantized->bytes == b.quantized->bytes);
  MINI_LLAMA_ASSERT_TRUE(a.shape == b.shape);
  return true;
}

bool SameModelWeights(const MiniLlamaModel &x, const MiniLlamaModel &y) {
  for (size_t i = 0; i < x.layers.size(); ++i) {
    const auto &p = x.layers[i], &q = y.layers[i];
    for (auto pair : {std::make_pair(&p.wq, &q.wq), std::make_pair(&p.wk, &q.wk), std::make_pair(&p.wv, &q.wv),
                      std::make_pair(&p.wo, &q.wo), std::make_pair(&p.w_gate, &q.w_gate),
                      std::make_pair(&p.w_up, &q.w_up), std::make_pair(&p.w_down, &q.w_down)})
      if (!SameStorage(*pair.first, *pair.second)) return false;
  }
  return SameStorage(x.lm_head, y.lm_head);
}

bool TestQuantizeModel() {
  for (auto type : {QuantType::kQ80, QuantType::kQ40, QuantType::kQ41}) {
    auto ref = LoadModel("models/tiny/model.json", "models/tiny/model.bin");
    auto ours = ref;
    QuantizeModel(ref, type);
    QuantizeModelB200(ours, type);
    if (!SameModelWeights(ref, ours)) return false;
    for (auto again : {QuantType::kQ80, QuantType::kQ41}) {  // packed -> decoded -> packed
      auto r2 = ref, o2 = ours;
      QuantizeModel(r2, again);
      QuantizeModelB200(o2, again);
      if (!SameModelWeights(r2, o2)) return false;
    }
  }
  auto model = LoadModel("models/tiny/model.json", "models/tiny/model.bin");
  EnableCuda(model);
  bool refused = false;
  try {
    QuantizeModelB200(model, QuantType::kQ80);
  } catch (const std::runtime_error &e) {
    refused = std::string(e.what()) == "quantize weights before uploading the model to CUDA";
  }
  MINI_LLAMA_ASSERT_TRUE(refused);
  return true;
}

// A GGUF file (v3, "llama") of a small random model whose linears and lm_head
// are stored as `type` blocks; the other tensors F32. Written with the
// primitives of tests/gguf_loader_fixture.h.
std::filesystem::path WriteQuantizedGguf(const MiniLlamaModel &m, QuantType type, const std::string &name) {
  using namespace mini_llama::test;
  struct Entry {
    std::string name;
    std::vector<int> shape;
    uint32_t ggml_type;
    std::vector<char> bytes;
  };
  std::vector<Entry> entries;
  auto f32 = [&](const std::string &n, const Tensor &t) {
    const char *p = reinterpret_cast<const char *>(t.data.data());
    entries.push_back({n, t.shape, kGgmlTypeF32, std::vector<char>(p, p + t.data.size() * sizeof(float))});
  };
  auto packed = [&](const std::string &n, const Tensor &t) {
    const Tensor q = QuantizeTensor(t, type);
    const auto &b = q.quantized->bytes;
    entries.push_back({n, t.shape, static_cast<uint32_t>(type), std::vector<char>(b.begin(), b.end())});
  };
  f32("token_embd.weight", m.token_embedding);
  for (int l = 0; l < m.config.n_layers; ++l) {
    const auto &w = m.layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    f32(p + "attn_norm.weight", w.attention_norm);
    packed(p + "attn_q.weight", w.wq);
    packed(p + "attn_k.weight", w.wk);
    packed(p + "attn_v.weight", w.wv);
    packed(p + "attn_output.weight", w.wo);
    f32(p + "ffn_norm.weight", w.ffn_norm);
    packed(p + "ffn_gate.weight", w.w_gate);
    packed(p + "ffn_up.weight", w.w_up);
    packed(p + "ffn_down.weight", w.w_down);
  }
  f32("output_norm.weight", m.final_norm);
  packed("output.weight", m.lm_head);

  constexpr uint64_t kAlign = 32;
  std::vector<char> d = {'G', 'G', 'U', 'F'};
  AppendU32Le(d, 3);
  AppendU64Le(d, entries.size());
  AppendU64Le(d, 12);
  const ModelConfig &c = m.config;
  AppendMetadataString(d, "general.architecture", "llama");
  AppendMetadataString(d, "general.name", "mini-ai-b200-quantized-gguf-test");
  AppendMetadataU32(d, "general.alignment", kAlign);
  AppendMetadataU32(d, "llama.block_count", c.n_layers);
  AppendMetadataU32(d, "llama.context_length", c.max_seq_len);
  AppendMetadataU32(d, "llama.embedding_length", c.dim);
  AppendMetadataU32(d, "llama.feed_forward_length", c.hidden_dim);
  AppendMetadataU32(d, "llama.attention.head_count", c.n_heads);
  AppendMetadataU32(d, "llama.attention.head_count_kv", c.n_kv_heads);
  AppendMetadataF32(d, "llama.rope.freq_base", c.rope_theta);
  AppendMetadataF32(d, "llama.attention.layer_norm_rms_epsilon", c.rms_norm_eps);
  AppendMetadataTokens(d, c.vocab_size);
  uint64_t offset = 0;
  std::vector<uint64_t> offsets;
  for (const Entry &e : entries) {
    AppendString(d, e.name);
    AppendU32Le(d, static_cast<uint32_t>(e.shape.size()));
    if (e.shape.size() == 2) {  // GGUF order: ne0 = columns, ne1 = rows
      AppendU64Le(d, e.shape[1]);
      AppendU64Le(d, e.shape[0]);
    } else {
      for (int s : e.shape) AppendU64Le(d, s);
    }
    AppendU32Le(d, e.ggml_type);
    AppendU64Le(d, offset);
    offsets.push_back(offset);
    offset += (e.bytes.size() + kAlign - 1) / kAlign * kAlign;
  }
  d.insert(d.end(), (kAlign - d.size() % kAlign) % kAlign, '\0');
  for (const Entry &e : entries) {
    d.insert(d.end(), e.bytes.begin(), e.bytes.end());
    d.insert(d.end(), (kAlign - e.bytes.size() % kAlign) % kAlign, '\0');
  }
  const auto path = std::filesystem::temp_directory_path() / name;
  std::ofstream out(path, std::ios::binary);
  out.write(d.data(), static_cast<std::streamsize>(d.size()));
  return path;
}

bool TestGgufQuantizedModel() {
  ModelConfig c;
  c.vocab_size = 160;
  c.dim = 64;
  c.hidden_dim = 96;
  c.n_layers = 2;
  c.n_heads = 4;
  c.n_kv_heads = 2;
  c.head_dim = 16;
  c.max_seq_len = 64;
  c.rope_theta = 10000.0f;
  MiniLlamaModel src = MakeToyModel(c);
  Lcg g{7};
  auto fill = [&](Tensor &t, float scale, float bias) {
    for (float &v : t.data) v = bias + g.Next(scale);
  };
  fill(src.token_embedding, 1.0f, 0.0f);
  fill(src.final_norm, 0.1f, 1.0f);
  fill(src.lm_head, 0.2f, 0.0f);
  for (auto &l : src.layers) {
    fill(l.attention_norm, 0.1f, 1.0f);
    fill(l.ffn_norm, 0.1f, 1.0f);
    for (Tensor *w : {&l.wq, &l.wk, &l.wv, &l.wo, &l.w_gate, &l.w_up, &l.w_down}) fill(*w, 0.2f, 0.0f);
  }
  src.loaded = true;
  for (auto type : {QuantType::kQ80, QuantType::kQ40, QuantType::kQ41}) {
    const auto path = WriteQuantizedGguf(src, type, "mini_ai_b200_q" + std::to_string(static_cast<int>(type)) + ".gguf");
    MiniLlamaModel cpu = LoadGgufModel(path.string());
    std::filesystem::remove(path);
    MINI_LLAMA_ASSERT_TRUE(cpu.loaded);
    // The loader kept the file's blocks: they equal QuantizeTensor's.
    auto expected = src;
    QuantizeModel(expected, type);
    if (!SameModelWeights(cpu, expected)) return false;
    auto gpu = cpu;
    EnableCuda(gpu);
    if (!RunRequests(cpu, gpu, Prompts({7, 3}, c.vocab_size, 5), 3)) return false;
  }
  return true;
}

struct Registrar {
  Registrar() {
    RegisterTest("b200_batched_forward_matches_cpu", TestBatchedForward);
    RegisterTest("b200_batched_forward_rejects_bad_input", TestBatchedForwardRejects);
    RegisterTest("b200_quantize_model_matches_reference", TestQuantizeModel);
    RegisterTest("b200_gguf_quantized_model_forward", TestGgufQuantizedModel);
  }
} registrar;

}  // namespace
