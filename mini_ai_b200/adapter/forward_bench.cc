// Full LLaMA-style forward with random weights through the B200 backend:
// R requests with P-token uniform-random prompts, then D greedy decode steps
// each, as mini_ai serves them (prefill, then one token per step, greedy
// sampling on the host: src/main.cc:291-316), but with all requests of a step
// in one batched forward (ForwardBatchCuda): the prefill of all prompts is one
// ragged row block, every decode step one R-row block.
//
// Default shape: 32 layers, dim 4096, 32 query / 8 KV heads (head_dim 128),
// SwiGLU hidden 14336, RMSNorm eps 1e-5, NeoX RoPE theta 5e5, vocab 128256,
// Q8_0 linears and lm_head, F32 embeddings and norms, KV cache F32 on the
// device; 4 requests x 128 prompt tokens, 128 decode steps.
//
// The weights are generated and packed on the device (RandomCudaModel). The
// CPU baseline (--cpu-layers L > 0) runs the reference's own CPU forward
// (ForwardBatch, src/forward.cc:175-203, with every host thread) on host
// copies of the first L layers and the lm_head of the same weights, one
// token at a time as the reference does, and extrapolates to the full depth:
// t_token = t_head + n_layers * (t_L - t_head) / L, t_head timed alone.
//
// Prints one JSON line.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "b200_backend.h"
#include "mini_llama/forward.h"
#include "mini_llama/matmul_dispatch.h"
#include "mini_llama/ops.h"

using namespace mini_llama;

namespace {

double Now() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int Arg(int argc, char **argv, const char *name, int dflt) {
  for (int i = 1; i + 1 < argc; ++i)
    if (std::strcmp(argv[i], name) == 0) return std::atoi(argv[i + 1]);
  return dflt;
}
double ArgF(int argc, char **argv, const char *name, double dflt) {
  for (int i = 1; i + 1 < argc; ++i)
    if (std::strcmp(argv[i], name) == 0) return std::atof(argv[i + 1]);
  return dflt;
}

std::vector<std::vector<int>> Prompts(int requests, int length, int vocab, uint64_t seed) {
  uint64_t s = seed * 0x9e3779b97f4a7c15ull + 1;
  std::vector<std::vector<int>> out(requests);
  for (auto &p : out)
    for (int i = 0; i < length; ++i) {
      s = s * 6364136223846793005ull + 1442695040888963407ull;
      p.push_back(static_cast<int>((s >> 33) % static_cast<uint64_t>(vocab)));
    }
  return out;
}

struct RunTimes {
  double prefill_s = 0, decode_s = 0;
  std::vector<int> last_tokens;
};

// Prefill all prompts in one call, then `decode` greedy steps of all requests.
RunTimes Serve(const MiniLlamaModel &model, const std::vector<std::vector<int>> &prompts, int decode) {
  const size_t R = prompts.size();
  std::vector<MiniLlamaContext> ctx;
  for (size_t r = 0; r < R; ++r) ctx.emplace_back(&model);
  std::vector<MiniLlamaContext *> ptrs;
  for (auto &c : ctx) {
    PrepareCudaContext(c, model);
    ptrs.push_back(&c);
  }
  cudaDeviceSynchronize();
  RunTimes t;
  std::vector<MiniBatch> batches;
  for (const auto &p : prompts) batches.push_back(MiniBatch::FromTokens(p, 0));
  const double t0 = Now();
  std::vector<Tensor> logits = ForwardBatchCuda(ptrs, model, batches);
  std::vector<int> next(R);
  for (size_t r = 0; r < R; ++r) next[r] = ArgMax(logits[r]);
  const double t1 = Now();
  for (int step = 0; step < decode; ++step) {
    for (size_t r = 0; r < R; ++r) batches[r] = MiniBatch::Single(next[r], ctx[r].pos + 1);
    logits = ForwardBatchCuda(ptrs, model, batches);
    for (size_t r = 0; r < R; ++r) next[r] = ArgMax(logits[r]);
  }
  const double t2 = Now();
  t.prefill_s = t1 - t0;
  t.decode_s = t2 - t1;
  t.last_tokens = next;
  return t;
}

}  // namespace

int main(int argc, char **argv) {
  try {
    ModelConfig c;
    c.vocab_size = Arg(argc, argv, "--vocab", 128256);
    c.dim = Arg(argc, argv, "--dim", 4096);
    c.hidden_dim = Arg(argc, argv, "--hidden", 14336);
    c.n_layers = Arg(argc, argv, "--layers", 32);
    c.n_heads = Arg(argc, argv, "--heads", 32);
    c.n_kv_heads = Arg(argc, argv, "--kv-heads", 8);
    c.head_dim = c.dim / c.n_heads;
    c.rope_theta = 500000.0f;
    c.rms_norm_eps = 1e-5f;
    c.rope_type = RopeType::kNeoX;
    const int R = Arg(argc, argv, "--requests", 4), P = Arg(argc, argv, "--prompt", 128);
    const int D = Arg(argc, argv, "--decode", 128), type = Arg(argc, argv, "--type", 8);
    const int warmup = Arg(argc, argv, "--warmup", 3), seed = Arg(argc, argv, "--seed", 0);
    const int cpu_layers = Arg(argc, argv, "--cpu-layers", 0), cpu_tokens = Arg(argc, argv, "--cpu-tokens", 2);
    const double hbm_gbs = ArgF(argc, argv, "--hbm-gbs", 0.0);
    c.max_seq_len = P + D + 1;

    const double b0 = Now();
    MiniLlamaModel model = RandomCudaModel(c, type, static_cast<uint64_t>(seed), 0);
    const double build_s = Now() - b0;
    const auto prompts = Prompts(R, P, c.vocab_size, static_cast<uint64_t>(seed));
    // Warm-up: every row-block shape of the run reaches its captured graph
    // (plain, own stream, capture: three calls) before the timed requests.
    for (int w = 0; w < warmup; ++w) Serve(model, prompts, 3);
    const RunTimes t = Serve(model, prompts, D);

    // Packed bytes every decode step streams: all projections and the lm_head.
    const double kv = (double)c.n_kv_heads * c.head_dim;
    const double per_layer = (double)c.dim * c.dim * 2 + kv * c.dim * 2 + 3.0 * c.hidden_dim * c.dim;
    const double bpw = type == 8 ? 34.0 / 32 : type == 2 ? 18.0 / 32 : type == 3 ? 20.0 / 32 : 4.0;
    const double weight_bytes = (per_layer * c.n_layers + (double)c.vocab_size * c.dim) * bpw;
    const double step_s = t.decode_s / std::max(1, D);
    const double total_tokens = (double)R * P + (double)R * D;
    std::printf("{\"workload\": \"llama_forward_%s\", \"value\": %.2f, \"unit\": \"tokens/s\", ",
                type == 8 ? "q8_0" : type == 2 ? "q4_0" : type == 3 ? "q4_1" : "f32",
                total_tokens / (t.prefill_s + t.decode_s));
    std::printf("\"config\": {\"layers\": %d, \"dim\": %d, \"hidden\": %d, \"heads\": %d, \"kv_heads\": %d, "
                "\"vocab\": %d, \"rope\": \"neox\", \"rope_theta\": 500000, \"requests\": %d, \"prompt\": %d, "
                "\"decode\": %d, \"weights\": \"random, generated and packed on the device\"}, ",
                c.n_layers, c.dim, c.hidden_dim, c.n_heads, c.n_kv_heads, c.vocab_size, R, P, D);
    std::printf("\"tokens\": %.0f, \"seconds\": %.6f, \"prefill_s\": %.6f, \"decode_s\": %.6f, "
                "\"prefill_tokens_per_s\": %.1f, \"decode_tokens_per_s\": %.2f, \"ms_per_decode_step\": %.4f, ",
                total_tokens, t.prefill_s + t.decode_s, t.prefill_s, t.decode_s, (double)R * P / t.prefill_s,
                (double)R * D / t.decode_s, step_s * 1e3);
    std::printf("\"weight_bytes_per_decode_step\": %.0f, \"decode_gbs\": %.1f, ", weight_bytes,
                weight_bytes / step_s / 1e9);
    if (hbm_gbs > 0) std::printf("\"decode_frac_of_hbm\": %.4f, ", weight_bytes / step_s / 1e9 / hbm_gbs);
    std::printf("\"timing\": \"host wall clock around the served requests (logits to the host and greedy "
                "sampling on the host every step, as the reference serves); every step replays the CUDA graph of "
                "its row-block shape\", \"warmup\": %d, \"build_s\": %.2f", warmup, build_s);

    if (cpu_layers > 0) {
      const unsigned threads = std::max(1u, std::thread::hardware_concurrency());
      SetMatmulThreads(std::min(threads, 256u));
      MiniLlamaModel host = HostCopyOfCudaModel(model, cpu_layers);
      MiniLlamaContext ctx(&host);
      std::vector<int> toks(prompts[0].begin(), prompts[0].begin() + std::min(cpu_tokens, P));
      ForwardBatch(ctx, host, MiniBatch::Single(toks[0], 0));  // thread pool start-up, first touch
      MiniLlamaContext ctx2(&host);
      const double c0 = Now();
      ForwardBatch(ctx2, host, MiniBatch::FromTokens(toks, 0));
      const double t_l = (Now() - c0) / toks.size();
      Tensor x({c.dim}, 0.5f);
      const double h0 = Now();
      Tensor y = Linear(RmsNorm(x, host.final_norm, c.rms_norm_eps), host.lm_head);
      const double t_head = Now() - h0;
      const double t_token = t_head + c.n_layers * std::max(0.0, t_l - t_head) / cpu_layers;
      std::printf(", \"cpu_baseline\": {\"value\": %.5f, \"unit\": \"tokens/s\", \"cores\": %u, \"kind\": "
                  "\"reference\", \"sample\": \"the reference CPU forward (ForwardBatch, one token at a time) on "
                  "%d of %d layers + lm_head of the same weights, %zu tokens; %.3f s per token measured, lm_head "
                  "alone %.3f s; extrapolated to %d layers: %.2f s per token\"}",
                  1.0 / t_token, std::min(threads, 256u), cpu_layers, c.n_layers, toks.size(), t_l, t_head,
                  c.n_layers, t_token);
      (void)y;
    }
    std::printf("}\n");
    return 0;
  } catch (const std::exception &e) {
    std::printf("{\"error\": \"%s\"}\n", e.what());
    return 1;
  }
}
