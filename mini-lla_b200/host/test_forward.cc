// Whole-model checks of the row-batched prefill driver (cuda_batch.h) and
// the device weight paths (cuda_weights.cc, cuda_gguf_upload.h), against the
// reference's own CPU forward pass (src/forward.cc ForwardToken,
// src/batch.cc ForwardBatch) on the same random models, and against the
// reference's per-token GPU driver (src/cuda_forward.cc, compiled unchanged
// over this library's operators).
//
// Built by `make -C oracle dropin`; prints one line per failed check and
// exits non-zero on failure.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf_fixture.h"  // the reference's GGUF test writer (tests/)
#include "mini_llama/batch.h"
#include "mini_llama/cuda_batch.h"
#include "mini_llama/cuda_gguf_upload.h"
#include "mini_llama/cuda_weights.h"
#include "mini_llama/forward.h"
#include "mini_llama/gguf_loader.h"
#include "mini_llama/kv_cache.h"
#include "mini_llama/quant.h"

using namespace mini_lla;

namespace {

int g_failures = 0;
int g_checks = 0;

void Expect(bool ok, const std::string& what) {
  ++g_checks;
  if (!ok) {
    ++g_failures;
    std::printf("FAIL: %s\n", what.c_str());
  }
}

// max |got - want| / max(max |want|, 1e-30): the logits of a multi-layer
// forward in another summation order differ from the reference's by a few
// fp32 ulps of the largest logit per layer.
double ScaledError(const std::vector<float>& got, const std::vector<float>& want) {
  if (got.size() != want.size() || got.empty()) return 1e30;
  double scale = 0, worst = 0;
  for (size_t i = 0; i < want.size(); ++i) {
    if (!std::isfinite(got[i])) return 1e30;
    scale = std::max(scale, std::fabs(double(want[i])));
    worst = std::max(worst, std::fabs(double(got[i]) - want[i]));
  }
  return worst / std::max(scale, 1e-30);
}

// Written into the test so a reader sees the bar: 2e-5 of the largest
// logit (measured errors are ~1e-6).
constexpr double kLogitTolerance = 2e-5;

Tensor Random(std::vector<int> shape, std::mt19937& rng, float scale, float shift = 0.0f) {
  Tensor t(shape);
  std::normal_distribution<float> n(0.0f, 1.0f);
  for (float& v : t.data) v = n(rng) * scale + shift;
  return t;
}

QuantizedTensor Linear(int rows, int cols, QuantType type, std::mt19937& rng) {
  Tensor w = Random({rows, cols}, rng, 1.0f / std::sqrt(static_cast<float>(cols)));
  return type == QuantType::kF32 ? MakeF32Weight(std::move(w)) : Quantize(w, type);
}

struct ModelSpec {
  const char* name;
  int vocab, dim, hidden, layers, heads, kv_heads, max_seq;
  QuantType type;
  RopeType rope;
  bool biases;
  bool tied;
};

Model RandomModel(const ModelSpec& s, std::mt19937& rng) {
  Model m;
  ModelConfig& c = m.config;
  c.vocab_size = s.vocab;
  c.dim = s.dim;
  c.hidden_dim = s.hidden;
  c.n_layers = s.layers;
  c.n_heads = s.heads;
  c.n_kv_heads = s.kv_heads;
  c.max_seq_len = s.max_seq;
  c.rope_theta = s.rope == RopeType::kNeoX ? 1e6f : 1e4f;
  c.rms_norm_eps = 1e-6f;
  c.rope_type = s.rope;
  ValidateConfig(c);
  m.token_embedding = Linear(s.vocab, s.dim, s.type, rng);
  m.final_norm = Random({s.dim}, rng, 0.1f, 1.0f);
  m.tied_lm_head = s.tied;
  if (!s.tied) m.lm_head = Linear(s.vocab, s.dim, s.type, rng);
  m.layers.resize(static_cast<size_t>(s.layers));
  for (LayerWeights& l : m.layers) {
    l.attention_norm = Random({s.dim}, rng, 0.1f, 1.0f);
    l.wq = Linear(c.attention_dim(), s.dim, s.type, rng);
    l.wk = Linear(c.kv_dim(), s.dim, s.type, rng);
    l.wv = Linear(c.kv_dim(), s.dim, s.type, rng);
    l.wo = Linear(s.dim, c.attention_dim(), s.type, rng);
    if (s.biases) {
      l.bq = Random({c.attention_dim()}, rng, 0.02f);
      l.bk = Random({c.kv_dim()}, rng, 0.02f);
      l.bv = Random({c.kv_dim()}, rng, 0.02f);
    }
    l.ffn_norm = Random({s.dim}, rng, 0.1f, 1.0f);
    l.w_gate = Linear(s.hidden, s.dim, s.type, rng);
    l.w_up = Linear(s.hidden, s.dim, s.type, rng);
    l.w_down = Linear(s.dim, s.hidden, s.type, rng);
  }
  return m;
}

std::vector<int> Tokens(int count, int vocab, std::mt19937& rng) {
  std::uniform_int_distribution<int> u(0, vocab - 1);
  std::vector<int> t(static_cast<size_t>(count));
  for (int& v : t) v = u(rng);
  return t;
}

std::vector<float> DeviceFloats(const float* p, size_t count) {
  std::vector<float> host(count);
  if (cudaMemcpy(host.data(), p, count * sizeof(float), cudaMemcpyDeviceToHost) !=
      cudaSuccess) {
    throw std::runtime_error("download failed");
  }
  return host;
}

// Prompt, then one decode token, then a batch whose positions jump back and
// forth: ForwardBatchCuda against the CPU ForwardBatch at every step, and the
// reference's per-token GPU driver on the prompt.
void TestModel(const ModelSpec& spec, std::mt19937& rng) {
  Model cpu = RandomModel(spec, rng);
  Model gpu = cpu;
  UploadModelWeights(&gpu, 0);
  const std::string tag = std::string(spec.name) + ": ";
  Expect(CudaWeightCount(gpu) ==
             3u - (spec.tied ? 1u : 0u) + spec.layers * (spec.biases ? 12u : 9u),
         tag + "weight count");

  // long enough for the tensor-core linears (48 tokens and more)
  const int prompt = std::min(100, spec.max_seq - 8);
  const std::vector<int> tokens = Tokens(prompt, spec.vocab, rng);
  Context c_cpu(cpu.config), c_gpu(gpu.config), c_step(gpu.config);

  const Tensor want = ForwardBatch(c_cpu, cpu, MiniBatch::FromTokens(tokens, 0));
  const Tensor got = ForwardBatchCuda(c_gpu, gpu, MiniBatch::FromTokens(tokens, 0));
  double err = ScaledError(got.data, want.data);
  Expect(err <= kLogitTolerance, tag + "prompt logits, error " + std::to_string(err));
  Expect(c_gpu.position == c_cpu.position, tag + "position after prompt");

  // the reference's per-token GPU driver over the same device weights
  const Tensor step = ForwardBatch(c_step, gpu, MiniBatch::FromTokens(tokens, 0));
  err = ScaledError(step.data, want.data);
  Expect(err <= kLogitTolerance, tag + "per-token GPU logits, error " + std::to_string(err));

  // the caches hold the same K/V (layer 0 and the last layer)
  const size_t per_layer = static_cast<size_t>(cpu.config.max_seq_len) *
                           cpu.config.n_kv_heads * cpu.config.head_dim();
  for (int layer : {0, spec.layers - 1}) {
    const std::vector<float> k = DeviceFloats(c_gpu.cuda_cache.Keys(layer), per_layer);
    const std::vector<float> v = DeviceFloats(c_gpu.cuda_cache.Values(layer), per_layer);
    const float* kc = c_cpu.cache.keys.data.data() + layer * per_layer;
    const float* vc = c_cpu.cache.values.data.data() + layer * per_layer;
    double worst = 0, scale = 0;
    for (size_t i = 0; i < per_layer; ++i) {
      scale = std::max({scale, std::fabs(double(kc[i])), std::fabs(double(vc[i]))});
      worst = std::max({worst, std::fabs(double(k[i]) - kc[i]), std::fabs(double(v[i]) - vc[i])});
    }
    Expect(worst <= kLogitTolerance * scale,
           tag + "KV cache layer " + std::to_string(layer) + ", error " +
               std::to_string(worst / scale));
  }

  // one decode token continues both caches
  const int next = Tokens(1, spec.vocab, rng)[0];
  const Tensor want_d = ForwardBatch(c_cpu, cpu, MiniBatch::Single(next, prompt));
  const Tensor got_d = ForwardBatchCuda(c_gpu, gpu, MiniBatch::Single(next, prompt));
  err = ScaledError(got_d.data, want_d.data);
  Expect(err <= kLogitTolerance, tag + "decode logits, error " + std::to_string(err));

  // positions that are not one run: rewrites earlier positions, then
  // continues; passes of at most 3 rows
  MiniBatch odd;
  odd.tokens = Tokens(9, spec.vocab, rng);
  odd.positions = {prompt + 1, prompt + 2, 5, 6, 7, 8, prompt + 3, 2, 3};
  const Tensor want_o = ForwardBatch(c_cpu, cpu, odd);
  const Tensor got_o = ForwardBatchCuda(c_gpu, gpu, odd, 3);
  err = ScaledError(got_o.data, want_o.data);
  Expect(err <= kLogitTolerance, tag + "jumping positions logits, error " + std::to_string(err));
  Expect(c_gpu.position == c_cpu.position && c_gpu.position == 4, tag + "position after jumps");
}

void TestValidation(std::mt19937& rng) {
  const ModelSpec spec{"validation", 50, 64, 128, 1, 4, 2, 16, QuantType::kQ8_0,
                       RopeType::kNormal, false, true};
  Model model = RandomModel(spec, rng);
  UploadModelWeights(&model, 0);
  Context context(model.config);
  auto throws = [&](const MiniBatch& b, bool out_of_range) {
    try {
      ForwardBatchCuda(context, model, b);
    } catch (const std::out_of_range&) {
      return out_of_range;
    } catch (const std::invalid_argument&) {
      return !out_of_range;
    }
    return false;
  };
  Expect(throws(MiniBatch(), false), "empty batch -> invalid_argument");
  MiniBatch mismatch = MiniBatch::FromTokens({1, 2}, 0);
  mismatch.positions.pop_back();
  Expect(throws(mismatch, false), "size mismatch -> invalid_argument");
  Expect(throws(MiniBatch::FromTokens({1, 50}, 0), true), "token id -> out_of_range");
  Expect(throws(MiniBatch::FromTokens({1, 2, 3}, 14), true), "position -> out_of_range");
  Expect(context.position == 0, "failed batches leave the position");
  Model cpu_only = model;
  cpu_only.cuda_weights.reset();
  bool threw = false;
  try {
    ForwardBatchCuda(context, cpu_only, MiniBatch::FromTokens({1}, 0));
  } catch (const std::runtime_error&) {
    threw = true;
  }
  Expect(threw, "no device weights -> runtime_error");
}

std::vector<uint8_t> DeviceBytes(const CudaWeight& w) {
  std::vector<uint8_t> host(w.buffer.size());
  w.buffer.Download(host.data(), host.size());
  return host;
}

bool SameBytes(const CudaWeight* a, const CudaWeight* b) {
  if (a == nullptr || b == nullptr) return a == b;
  return a->type == b->type && a->rows == b->rows && a->cols == b->cols &&
         a->linear == b->linear && DeviceBytes(*a) == DeviceBytes(*b);
}

// The reference's GGUF fixture (one qwen2 layer with Q8_0 / Q4_0 / Q4_1
// tensors and biases) loaded two ways: LoadGgufModel + UploadModelWeights,
// and LoadGgufModelToDevices.  Same names, types, shapes and bytes, and the
// same logits.
void TestGgufFixture() {
  const std::string path = "/tmp/mlb_forward_fixture.gguf";
  test::WriteFixtureGguf(path);
  Model host = LoadGgufModel(path);
  Model uploaded = host;
  UploadModelWeights(&uploaded, 0);
  const CudaGgufModel direct = LoadGgufModelToDevices(path, {0});
  const Model& device = direct.model;
  Expect(device.config.dim == host.config.dim && device.config.n_layers == host.config.n_layers &&
             device.config.n_kv_heads == host.config.n_kv_heads &&
             device.config.vocab_size == host.config.vocab_size &&
             device.config.max_seq_len == host.config.max_seq_len &&
             device.config.rope_type == host.config.rope_type &&
             device.config.rope_theta == host.config.rope_theta &&
             device.tied_lm_head == host.tied_lm_head,
         "GGUF config");
  Expect(CudaWeightCount(device) == CudaWeightCount(uploaded), "GGUF weight count");
  const char* names[] = {"token_embedding", "final_norm", "layers.0.attention_norm",
                         "layers.0.wq", "layers.0.wk", "layers.0.wv", "layers.0.wo",
                         "layers.0.bq", "layers.0.bk", "layers.0.bv", "layers.0.ffn_norm",
                         "layers.0.w_gate", "layers.0.w_up", "layers.0.w_down"};
  for (const char* name : names) {
    Expect(SameBytes(device.cuda_weights->Find(name), uploaded.cuda_weights->Find(name)),
           std::string("GGUF bytes of ") + name);
  }
  Context cpu(host.config), gpu(device.config), per_token(device.config);
  const MiniBatch batch = MiniBatch::FromTokens({1, 5, 7, 3, 9}, 0);
  const Tensor want = ForwardBatch(cpu, host, batch);
  const Tensor got = ForwardBatchCuda(gpu, device, batch);
  double err = ScaledError(got.data, want.data);
  Expect(err <= kLogitTolerance, "GGUF fixture logits, error " + std::to_string(err));
  // the reference's per-token GPU path accepts the device-only model too
  const Tensor step = ForwardBatch(per_token, device, batch);
  err = ScaledError(step.data, want.data);
  Expect(err <= kLogitTolerance, "GGUF fixture per-token logits, error " + std::to_string(err));

  bool threw = false;
  try {
    test::WriteFixtureGguf(path, false);
    LoadGgufModelToDevices(path, {0});
  } catch (const std::runtime_error&) {
    threw = true;
  }
  Expect(threw, "GGUF without tensors -> runtime_error");
  std::remove(path.c_str());
}

}  // namespace

int main() {
  std::mt19937 rng(20261202);
  try {
    const ModelSpec specs[] = {
        // bulk-copy GEMV path (k % 128 == 0), GQA 4, untied, normal RoPE
        {"q8_0 gqa", 300, 256, 512, 2, 8, 2, 128, QuantType::kQ8_0, RopeType::kNormal,
         false, false},
        // biases, NeoX, tied output, MHA
        {"q4_1 neox bias tied", 200, 128, 384, 2, 4, 4, 128, QuantType::kQ4_1,
         RopeType::kNeoX, true, true},
        // k % 128 != 0: the chunked GEMV form; group of 5
        {"q4_0 group5", 150, 160, 224, 2, 5, 1, 128, QuantType::kQ4_0, RopeType::kNormal,
         true, false},
        {"f32", 120, 128, 256, 1, 4, 2, 128, QuantType::kF32, RopeType::kNormal, false, false},
        // a short prompt (the GEMV linears) on a small context
        {"q8_0 short", 100, 128, 256, 1, 4, 1, 40, QuantType::kQ8_0, RopeType::kNeoX, true,
         true},
    };
    for (const ModelSpec& spec : specs) TestModel(spec, rng);
    TestValidation(rng);
    TestGgufFixture();
  } catch (const std::exception& e) {
    std::printf("FAIL: exception %s\n", e.what());
    return 1;
  }
  std::printf("%d checks, %d failures\n", g_checks, g_failures);
  if (g_failures != 0) return 1;
  std::printf("forward ok\n");
  return 0;
}
