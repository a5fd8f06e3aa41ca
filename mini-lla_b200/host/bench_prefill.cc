// Whole-model timing of the row-batched prefill driver (ForwardBatchCuda)
// and of decode steps, beside the reference's per-token GPU driver
// (src/cuda_forward.cc over this library's operators) and the reference's
// CPU forward pass (src/forward.cc + src/batch.cc, its thread pool at
// hardware_concurrency()), on a random-weight model of the given shape.
//
// Prints one JSON line.  Weights are random ggml blocks (scales uniform in
// [0.001, 0.05], codes uniform), activations stay finite; no checkpoint is
// needed.  Built by `make -C oracle dropin` next to the checks.
#include <cuda_runtime.h>

#include "mlb_ops.h"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "mini_llama/batch.h"
#include "mini_llama/cuda_batch.h"
#include "mini_llama/cuda_weights.h"
#include "mini_llama/forward.h"
#include "mini_llama/kv_cache.h"
#include "mini_llama/quant.h"
#include "mini_llama/thread_pool.h"

using namespace mini_lla;

namespace {

struct Args {
  int vocab = 128256, dim = 4096, hidden = 14336, layers = 4, heads = 32, kv_heads = 8;
  int max_seq = 4096;
  QuantType type = QuantType::kQ8_0;
  int tokens = 512;       // prompt rows per prefill
  int steps = 5, warmup = 2;
  int per_token = 64;     // tokens through the per-token GPU driver (0: skip)
  int decode = 32;        // decode steps after the prompt (0: skip)
  int cpu_tokens = 2;     // tokens through the CPU forward pass (0: skip)
  int max_rows = 512;
  int overlap = 1;        // programmatic dependent launch (mlb_set_launch_overlap)
};

uint16_t RandomScale(std::mt19937& rng) {
  std::uniform_real_distribution<float> u(0.001f, 0.05f);
  // fp16 bits of a normal value in [2^-10, 2^-4.3]: exponent and mantissa
  const float v = u(rng);
  int e = 0;
  const float m = std::frexp(v, &e);          // v = m * 2^e, m in [0.5, 1)
  const int exp16 = e - 1 + 15;               // biased fp16 exponent
  const int mant = static_cast<int>((m * 2.0f - 1.0f) * 1024.0f) & 1023;
  return static_cast<uint16_t>((exp16 << 10) | mant);
}

QuantizedTensor RandomWeight(int rows, int cols, QuantType type, std::mt19937& rng) {
  QuantizedTensor w;
  w.type = type;
  w.rows = rows;
  w.cols = cols;
  const size_t blocks = static_cast<size_t>(rows) * ((cols + 31) / 32);
  std::uniform_int_distribution<int> byte(0, 255);
  switch (type) {
    case QuantType::kF32: {
      Tensor t({rows, cols});
      std::normal_distribution<float> n(0.0f, 1.0f / std::sqrt(static_cast<float>(cols)));
      for (float& v : t.data) v = n(rng);
      return MakeF32Weight(std::move(t));
    }
    case QuantType::kQ8_0:
      w.q8_0.resize(blocks);
      for (BlockQ8_0& b : w.q8_0) {
        b.d = RandomScale(rng);
        for (int8_t& q : b.qs) q = static_cast<int8_t>(byte(rng) - 128);
      }
      break;
    case QuantType::kQ4_0:
      w.q4_0.resize(blocks);
      for (BlockQ4_0& b : w.q4_0) {
        b.d = RandomScale(rng);
        for (uint8_t& q : b.qs) q = static_cast<uint8_t>(byte(rng));
      }
      break;
    case QuantType::kQ4_1:
      w.q4_1.resize(blocks);
      for (BlockQ4_1& b : w.q4_1) {
        b.d = RandomScale(rng);
        b.m = static_cast<uint16_t>(RandomScale(rng) | 0x8000u);  // negative min
        for (uint8_t& q : b.qs) q = static_cast<uint8_t>(byte(rng));
      }
      break;
  }
  return w;
}

Tensor Norm(int n, std::mt19937& rng) {
  Tensor t({n});
  std::normal_distribution<float> d(1.0f, 0.1f);
  for (float& v : t.data) v = d(rng);
  return t;
}

Model BuildModel(const Args& a) {
  std::mt19937 rng(7);
  Model m;
  ModelConfig& c = m.config;
  c.vocab_size = a.vocab;
  c.dim = a.dim;
  c.hidden_dim = a.hidden;
  c.n_layers = a.layers;
  c.n_heads = a.heads;
  c.n_kv_heads = a.kv_heads;
  c.max_seq_len = a.max_seq;
  c.rope_theta = 500000.0f;
  c.rms_norm_eps = 1e-5f;
  ValidateConfig(c);
  m.token_embedding = RandomWeight(a.vocab, a.dim, a.type, rng);
  m.lm_head = RandomWeight(a.vocab, a.dim, a.type, rng);
  m.final_norm = Norm(a.dim, rng);
  m.layers.resize(static_cast<size_t>(a.layers));
  for (LayerWeights& l : m.layers) {
    l.attention_norm = Norm(a.dim, rng);
    l.wq = RandomWeight(c.attention_dim(), a.dim, a.type, rng);
    l.wk = RandomWeight(c.kv_dim(), a.dim, a.type, rng);
    l.wv = RandomWeight(c.kv_dim(), a.dim, a.type, rng);
    l.wo = RandomWeight(a.dim, c.attention_dim(), a.type, rng);
    l.ffn_norm = Norm(a.dim, rng);
    l.w_gate = RandomWeight(a.hidden, a.dim, a.type, rng);
    l.w_up = RandomWeight(a.hidden, a.dim, a.type, rng);
    l.w_down = RandomWeight(a.dim, a.hidden, a.type, rng);
  }
  return m;
}

double Seconds(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void Sync() {
  if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("device error");
}

QuantType ParseType(const std::string& s) {
  if (s == "F32") return QuantType::kF32;
  if (s == "Q8_0") return QuantType::kQ8_0;
  if (s == "Q4_0") return QuantType::kQ4_0;
  if (s == "Q4_1") return QuantType::kQ4_1;
  throw std::invalid_argument("unknown type " + s);
}

const char* TypeName(QuantType t) {
  switch (t) {
    case QuantType::kF32: return "F32";
    case QuantType::kQ8_0: return "Q8_0";
    case QuantType::kQ4_0: return "Q4_0";
    case QuantType::kQ4_1: return "Q4_1";
  }
  return "?";
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string k = argv[i];
    const std::string v = argv[i + 1];
    if (k == "--vocab") a.vocab = std::stoi(v);
    else if (k == "--dim") a.dim = std::stoi(v);
    else if (k == "--hidden") a.hidden = std::stoi(v);
    else if (k == "--layers") a.layers = std::stoi(v);
    else if (k == "--heads") a.heads = std::stoi(v);
    else if (k == "--kv-heads") a.kv_heads = std::stoi(v);
    else if (k == "--max-seq") a.max_seq = std::stoi(v);
    else if (k == "--type") a.type = ParseType(v);
    else if (k == "--tokens") a.tokens = std::stoi(v);
    else if (k == "--steps") a.steps = std::stoi(v);
    else if (k == "--warmup") a.warmup = std::stoi(v);
    else if (k == "--per-token") a.per_token = std::stoi(v);
    else if (k == "--decode") a.decode = std::stoi(v);
    else if (k == "--cpu-tokens") a.cpu_tokens = std::stoi(v);
    else if (k == "--max-rows") a.max_rows = std::stoi(v);
    else if (k == "--overlap") a.overlap = std::stoi(v);
    else {
      std::fprintf(stderr, "unknown flag %s\n", k.c_str());
      return 2;
    }
  }
  if (mlb_set_launch_overlap(a.overlap) != MLB_OK) {
    std::fprintf(stderr, "--overlap takes 0 or 1\n");
    return 2;
  }
  try {
    Model model = BuildModel(a);
    Model cpu_model = model;  // host-only copy for the CPU pass
    UploadModelWeights(&model, 0);
    std::mt19937 rng(11);
    std::uniform_int_distribution<int> tok(0, a.vocab - 1);
    std::vector<int> prompt(static_cast<size_t>(a.tokens));
    for (int& t : prompt) t = tok(rng);
    const MiniBatch batch = MiniBatch::FromTokens(prompt, 0);

    // prefill: ForwardBatchCuda over the whole prompt (wall clock, it ends
    // with the logits' download) and on-device time by events
    Context context(model.config);
    for (int i = 0; i < a.warmup; ++i) ForwardBatchCuda(context, model, batch, a.max_rows);
    Sync();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const auto t0 = std::chrono::steady_clock::now();
    cudaEventRecord(e0, nullptr);
    for (int i = 0; i < a.steps; ++i) ForwardBatchCuda(context, model, batch, a.max_rows);
    cudaEventRecord(e1, nullptr);
    Sync();
    const double prefill_s = Seconds(t0) / a.steps;
    float device_ms = 0;
    cudaEventElapsedTime(&device_ms, e0, e1);
    device_ms /= a.steps;

    // decode steps after the prompt
    double decode_s = 0;
    float decode_device_ms = 0;
    if (a.decode > 0) {
      const int start = a.tokens;
      for (int i = 0; i < 2; ++i) ForwardBatchCuda(context, model, MiniBatch::Single(tok(rng), start));
      Sync();
      const auto t1 = std::chrono::steady_clock::now();
      cudaEventRecord(e0, nullptr);
      for (int i = 0; i < a.decode && start + i < a.max_seq; ++i)
        ForwardBatchCuda(context, model, MiniBatch::Single(tok(rng), start + i));
      cudaEventRecord(e1, nullptr);
      Sync();
      decode_s = Seconds(t1) / a.decode;
      cudaEventElapsedTime(&decode_device_ms, e0, e1);
      decode_device_ms /= a.decode;
    }

    // the reference's per-token GPU driver (ForwardBatch -> ForwardTokenCuda)
    double per_token_s = 0;
    if (a.per_token > 0) {
      Context step(model.config);
      const std::vector<int> head(prompt.begin(),
                                  prompt.begin() + std::min(a.per_token, a.tokens));
      ForwardBatch(step, model, MiniBatch::FromTokens({head[0]}, 0));
      Sync();
      const auto t2 = std::chrono::steady_clock::now();
      ForwardBatch(step, model, MiniBatch::FromTokens(head, 0));
      Sync();
      per_token_s = Seconds(t2) / static_cast<double>(head.size());
    }

    // the reference's CPU forward pass on a few tokens
    double cpu_s = 0;
    const unsigned cores = std::thread::hardware_concurrency();
    if (a.cpu_tokens > 0) {
      SetThreadCount(static_cast<int>(cores));
      Context cpu(cpu_model.config);
      const std::vector<int> head(prompt.begin(),
                                  prompt.begin() + std::min(a.cpu_tokens, a.tokens));
      const auto t3 = std::chrono::steady_clock::now();
      ForwardBatch(cpu, cpu_model, MiniBatch::FromTokens(head, 0));
      cpu_s = Seconds(t3) / static_cast<double>(head.size());
    }

    std::printf(
        "{\"model\": {\"vocab\": %d, \"dim\": %d, \"hidden\": %d, \"layers\": %d, "
        "\"heads\": %d, \"kv_heads\": %d, \"type\": \"%s\"}, \"prompt_tokens\": %d, "
        "\"prefill_ms\": %.3f, \"prefill_device_ms\": %.3f, \"prefill_tokens_per_s\": %.1f, "
        "\"decode_ms_per_token\": %.4f, \"decode_device_ms_per_token\": %.4f, "
        "\"per_token_driver_ms_per_token\": %.4f, "
        "\"cpu_ms_per_token\": %.2f, \"cpu_threads\": %u, \"cpu_tokens\": %d, "
        "\"per_token_tokens\": %d, \"launch_overlap\": %d}\n",
        a.vocab, a.dim, a.hidden, a.layers, a.heads, a.kv_heads, TypeName(a.type),
        a.tokens, prefill_s * 1e3, device_ms, a.tokens / prefill_s, decode_s * 1e3,
        decode_device_ms, per_token_s * 1e3, cpu_s * 1e3, cores, a.cpu_tokens,
        std::min(a.per_token, a.tokens), a.overlap);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
