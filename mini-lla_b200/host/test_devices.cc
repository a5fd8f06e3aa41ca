// Checks of the multi-device backend (cuda_backend.h) and of the per-device
// state under it (weight replicas, the caching pool, the RoPE table cache).
//
//   mlb_devices_test --cpu   device-list parsing and validation against a
//                            given device count; no CUDA call is made
//   mlb_devices_test         on a box with at least two GPUs: replicated
//                            uploads (host model and GGUF file) byte for byte,
//                            layer operators over token rows split across
//                            distinct devices against one device bit for bit,
//                            and requests spread over devices by
//                            ForwardBatchesCuda against ForwardBatchCuda on one
//                            device bit for bit; prints "devices skipped" and
//                            exits 0 with fewer than two GPUs
//
// Built by `make -C oracle dropin`; prints one line per failed check and
// exits non-zero on failure.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf_fixture.h"  // the reference's GGUF test writer (tests/)
#include "mini_llama/batch.h"
#include "mini_llama/cuda_backend.h"
#include "mini_llama/cuda_batch.h"
#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/cuda_weights.h"
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

template <typename E>
bool Throws(const std::function<void()>& fn) {
  try {
    fn();
  } catch (const E&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

bool BitEqual(const std::vector<float>& a, const std::vector<float>& b) {
  return a.size() == b.size() &&
         (a.empty() || std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0);
}

// ------------------------------------------------------------------ CPU

void TestParseAndValidate() {
  Expect(ParseCudaDevices("0,2,3", 8) == std::vector<int>({0, 2, 3}), "parse list");
  Expect(ParseCudaDevices("5", 8) == std::vector<int>({5}), "parse one id");
  Expect(ParseCudaDevices("all", 3) == std::vector<int>({0, 1, 2}), "parse all");
  for (const char* bad : {"", ",", "0,", ",1", "a", "-1", "1;2", "0,,1", "1234567890"}) {
    Expect(Throws<std::invalid_argument>([&] { ParseCudaDevices(bad, 8); }),
           std::string("parse rejects \"") + bad + "\"");
  }
  Expect(Throws<std::invalid_argument>([] { ParseCudaDevices("all", 0); }),
         "all with no device -> invalid_argument");

  BackendConfig cpu;
  BackendConfig cuda;
  cuda.kind = BackendKind::kCuda;
  ValidateBackendDevices(cpu, {}, 0);  // the reference's default: fine
  Expect(Throws<std::invalid_argument>([&] { ValidateBackendDevices(cpu, {0}, 4); }),
         "cpu backend with devices -> invalid_argument");
  BackendConfig cpu_device = cpu;
  cpu_device.device_set = true;
  Expect(Throws<std::invalid_argument>([&] { ValidateBackendDevices(cpu_device, {}, 4); }),
         "cpu backend with --device -> invalid_argument (backend.cc:28-31)");
  ValidateBackendDevices(cuda, {0, 1, 3}, 4);
  Expect(Throws<std::out_of_range>([&] { ValidateBackendDevices(cuda, {0, 4}, 4); }),
         "device == count -> out_of_range (backend.cc:37-41)");
  Expect(Throws<std::out_of_range>([&] { ValidateBackendDevices(cuda, {-1}, 4); }),
         "negative device -> out_of_range");
  Expect(Throws<std::out_of_range>([&] { ValidateBackendDevices(cuda, {0}, 0); }),
         "no visible device -> out_of_range");
  Expect(Throws<std::invalid_argument>([&] { ValidateBackendDevices(cuda, {}, 4); }),
         "empty list -> invalid_argument");
  Expect(Throws<std::invalid_argument>([&] { ValidateBackendDevices(cuda, {1, 2, 1}, 4); }),
         "duplicate -> invalid_argument");

  BackendConfig one = cuda;
  one.device = 3;
  Expect(SelectedDevices(one, {}) == std::vector<int>({3}), "no list -> the config's device");
  Expect(SelectedDevices(one, {1, 0}) == std::vector<int>({1, 0}), "list wins");
  Expect(BackendDevicesNote(one, {}) == "compute: cuda device 3", "note, one device");
  Expect(BackendDevicesNote(one, {0, 1}) == "compute: cuda devices 0,1 (weights replicated)",
         "note, two devices");
  Expect(BackendDevicesNote(cpu, {}) == "compute: cpu", "note, cpu");
  Expect(ShardRange(5, 2, 0) == std::make_pair(0, 3) && ShardRange(5, 2, 1) == std::make_pair(3, 5),
         "request ranges");
}

// ------------------------------------------------------------------ GPU

Tensor Random(std::vector<int> shape, std::mt19937& rng, float scale, float shift = 0.0f) {
  Tensor t(shape);
  std::normal_distribution<float> n(0.0f, 1.0f);
  for (float& v : t.data) v = n(rng) * scale + shift;
  return t;
}

Model RandomModel(std::mt19937& rng) {
  Model m;
  ModelConfig& c = m.config;
  c.vocab_size = 300;
  c.dim = 256;
  c.hidden_dim = 512;
  c.n_layers = 2;
  c.n_heads = 8;
  c.n_kv_heads = 2;
  c.max_seq_len = 256;
  c.rope_theta = 1e6f;
  c.rms_norm_eps = 1e-6f;
  c.rope_type = RopeType::kNeoX;
  ValidateConfig(c);
  auto linear = [&](int rows, int cols) {
    return Quantize(Random({rows, cols}, rng, 1.0f / std::sqrt(float(cols))), QuantType::kQ8_0);
  };
  m.token_embedding = linear(c.vocab_size, c.dim);
  m.final_norm = Random({c.dim}, rng, 0.1f, 1.0f);
  m.tied_lm_head = false;
  m.lm_head = linear(c.vocab_size, c.dim);
  m.layers.resize(static_cast<size_t>(c.n_layers));
  for (LayerWeights& l : m.layers) {
    l.attention_norm = Random({c.dim}, rng, 0.1f, 1.0f);
    l.wq = linear(c.attention_dim(), c.dim);
    l.wk = linear(c.kv_dim(), c.dim);
    l.wv = linear(c.kv_dim(), c.dim);
    l.wo = linear(c.dim, c.attention_dim());
    l.bq = Random({c.attention_dim()}, rng, 0.02f);
    l.bk = Random({c.kv_dim()}, rng, 0.02f);
    l.bv = Random({c.kv_dim()}, rng, 0.02f);
    l.ffn_norm = Random({c.dim}, rng, 0.1f, 1.0f);
    l.w_gate = linear(c.hidden_dim, c.dim);
    l.w_up = linear(c.hidden_dim, c.dim);
    l.w_down = linear(c.dim, c.hidden_dim);
  }
  return m;
}

std::vector<uint8_t> DeviceBytes(const CudaWeight& w) {
  std::vector<uint8_t> host(w.buffer.size());
  CudaDeviceScope scope(CudaPointerDevice(w.buffer.data()));
  w.buffer.Download(host.data(), host.size());
  return host;
}

const char* kWeightNames[] = {
    "token_embedding", "final_norm", "lm_head", "layers.0.attention_norm", "layers.0.wq",
    "layers.0.wk", "layers.0.wv", "layers.0.wo", "layers.0.bq", "layers.0.bk", "layers.0.bv",
    "layers.0.ffn_norm", "layers.0.w_gate", "layers.0.w_up", "layers.0.w_down"};

// Every replica holds the same bytes as `want` (a single-device upload), on
// its own device.
void CheckReplicas(const CudaModelReplicas& replicas, const CudaModelWeights& want,
                   const std::string& tag) {
  for (size_t i = 0; i < replicas.size(); ++i) {
    const CudaModelWeights& got = *replicas.weights[i];
    Expect(got.device() == replicas.devices[i] && got.Count() == want.Count(),
           tag + ": replica " + std::to_string(i) + " device and count");
    for (const char* name : kWeightNames) {
      const CudaWeight* a = got.Find(name);
      const CudaWeight* b = want.Find(name);
      if (a == nullptr || b == nullptr) {
        Expect(a == b, tag + ": presence of " + name);
        continue;
      }
      Expect(CudaPointerDevice(a->buffer.data()) == replicas.devices[i],
             tag + ": " + name + " lives on its replica's device");
      Expect(a->type == b->type && a->rows == b->rows && a->cols == b->cols &&
                 DeviceBytes(*a) == DeviceBytes(*b),
             tag + ": bytes of " + name + " on device " + std::to_string(replicas.devices[i]));
    }
  }
}

struct LayerOpInputs {
  int rows = 0;
  std::vector<int> tokens, positions;
  Tensor residual, q, k, gate, up;
};

struct LayerOpOutputs {
  std::vector<float> h, y, q, k, ffn;
};

// The layer-op chain of one prefill chunk (embedding -> residual RMSNorm ->
// bias + RoPE -> SwiGLU) over rows [begin, end) with replica `model`'s
// weights on the current device; results land in `out` at those rows.
void LayerOps(const Model& model, const LayerOpInputs& in, int begin, int end,
              LayerOpOutputs* out, std::mutex* m) {
  const ModelConfig& c = model.config;
  const CudaModelWeights& w = *model.cuda_weights;
  const int rows = end - begin, dim = c.dim, hidden = c.hidden_dim;
  const int qd = c.attention_dim(), kd = c.kv_dim();
  auto slice = [&](const Tensor& t, int width) {
    Tensor s({rows, width});
    std::copy(t.data.begin() + static_cast<size_t>(begin) * width,
              t.data.begin() + static_cast<size_t>(end) * width, s.data.begin());
    return CudaTensor::FromHost(s);
  };
  const std::vector<int> tokens(in.tokens.begin() + begin, in.tokens.begin() + end);
  const std::vector<int> positions(in.positions.begin() + begin, in.positions.begin() + end);
  const CudaTensor x = CudaEmbeddingRows(*w.Find("token_embedding"), tokens);
  const CudaTensor r = slice(in.residual, dim);
  CudaTensor h;
  const CudaTensor y = CudaAddRmsNormRows(x, &r, *w.Find("layers.0.attention_norm"),
                                          c.rms_norm_eps, &h);
  CudaTensor q = slice(in.q, qd), k = slice(in.k, kd);
  CudaRopeRows(&q, &k, w.Find("layers.0.bq"), w.Find("layers.0.bk"), positions, c.rope_theta,
               c.n_heads, c.n_kv_heads, c.head_dim(), c.rope_type);
  const CudaTensor ffn = CudaSwiGlu(slice(in.gate, hidden), slice(in.up, hidden));
  const Tensor hh = h.Download(), yy = y.Download(), qq = q.Download(), kk = k.Download(),
               ff = ffn.Download();
  std::lock_guard<std::mutex> lock(*m);
  std::copy(hh.data.begin(), hh.data.end(), out->h.begin() + static_cast<size_t>(begin) * dim);
  std::copy(yy.data.begin(), yy.data.end(), out->y.begin() + static_cast<size_t>(begin) * dim);
  std::copy(qq.data.begin(), qq.data.end(), out->q.begin() + static_cast<size_t>(begin) * qd);
  std::copy(kk.data.begin(), kk.data.end(), out->k.begin() + static_cast<size_t>(begin) * kd);
  std::copy(ff.data.begin(), ff.data.end(),
            out->ffn.begin() + static_cast<size_t>(begin) * hidden);
}

LayerOpOutputs ShardedLayerOps(const CudaModelReplicas& replicas, const std::vector<int>& devices,
                               const LayerOpInputs& in) {
  const ModelConfig& c = replicas.config;
  LayerOpOutputs out;
  out.h.resize(static_cast<size_t>(in.rows) * c.dim);
  out.y.resize(out.h.size());
  out.q.resize(static_cast<size_t>(in.rows) * c.attention_dim());
  out.k.resize(static_cast<size_t>(in.rows) * c.kv_dim());
  out.ffn.resize(static_cast<size_t>(in.rows) * c.hidden_dim);
  std::mutex m;
  CudaShardRows(in.rows, devices, [&](int device, int begin, int end) {
    size_t replica = 0;
    while (replicas.devices[replica] != device) ++replica;
    LayerOps(replicas.ForDevice(replica), in, begin, end, &out, &m);
  });
  return out;
}

void TestDevices() {
  const int count = CudaDeviceCount();
  std::mt19937 rng(20261203);
  Expect(ParseCudaDevices("all").size() == static_cast<size_t>(count), "all = every device");
  BackendConfig cuda;
  cuda.kind = BackendKind::kCuda;
  Expect(Throws<std::out_of_range>([&] { ValidateBackendDevices(cuda, {0, count}); }),
         "device == visible count -> out_of_range");
  const std::vector<int> two = {0, 1};

  // replicated upload of a host model, against a single-device upload
  Model model = RandomModel(rng);
  Model single = model;
  UploadModelWeights(&single, 0);
  const CudaModelReplicas replicas = UploadModelWeightsToDevices(&model, {1, 0});
  Expect(model.cuda_weights == replicas.weights[0] && model.cuda_weights->device() == 1,
         "model->cuda_weights is the first listed device's replica");
  CheckReplicas(replicas, *single.cuda_weights, "host model");
  Expect(Throws<std::out_of_range>([&] { UploadModelWeightsToDevices(&model, {0, count}); }),
         "upload to a missing device -> out_of_range");

  // replicated GGUF load, against LoadGgufModel + UploadModelWeights
  const std::string path = "/tmp/mlb_devices_fixture.gguf";
  test::WriteFixtureGguf(path);
  Model gguf_host = LoadGgufModel(path);
  UploadModelWeights(&gguf_host, 0);
  const CudaModelReplicas gguf = LoadGgufModelReplicas(path, {1, 0});
  CheckReplicas(gguf, *gguf_host.cuda_weights, "gguf");
  std::remove(path.c_str());

  // layer operators over token rows split across distinct devices
  LayerOpInputs in;
  in.rows = 1001;
  const ModelConfig& c = replicas.config;
  std::uniform_int_distribution<int> tok(0, c.vocab_size - 1);
  for (int i = 0; i < in.rows; ++i) {
    in.tokens.push_back(tok(rng));
    in.positions.push_back(i);
  }
  in.residual = Random({in.rows, c.dim}, rng, 1.0f);
  in.q = Random({in.rows, c.attention_dim()}, rng, 1.0f);
  in.k = Random({in.rows, c.kv_dim()}, rng, 1.0f);
  in.gate = Random({in.rows, c.hidden_dim}, rng, 1.0f);
  in.up = Random({in.rows, c.hidden_dim}, rng, 1.0f);
  CudaPoolRelease(1);
  const LayerOpOutputs want = ShardedLayerOps(replicas, {0}, in);
  for (const std::vector<int>& devices : {two, std::vector<int>({1, 0})}) {
    const LayerOpOutputs got = ShardedLayerOps(replicas, devices, in);
    const std::string tag = "layer ops split over devices " + std::to_string(devices[0]) + "," +
                            std::to_string(devices[1]);
    Expect(BitEqual(got.h, want.h) && BitEqual(got.y, want.y), tag + ": h, y bit-exact");
    Expect(BitEqual(got.q, want.q) && BitEqual(got.k, want.k), tag + ": q, k bit-exact");
    Expect(BitEqual(got.ffn, want.ffn), tag + ": SwiGLU bit-exact");
  }
  {
    CudaDeviceScope scope(1);
    Expect(CudaRopeTableRows(c.rope_theta, c.head_dim()) >= in.rows / 2,
           "device 1 holds its own RoPE table");
  }
  Expect(CudaPoolCachedBytes(1) > 0, "device 1's pool caches its freed blocks");

  // requests spread over devices by ForwardBatchesCuda, against one device
  const std::vector<std::vector<int>> prompts = {
      {1, 5, 7, 3, 9, 11, 13}, {2, 4}, {8, 6, 4, 2, 0, 1, 3, 5, 7, 9, 21, 22, 23}, {17}, {30, 31, 32}};
  const CudaModelReplicas one = UploadModelWeightsToDevices(&model, {0});
  std::vector<Context> spread_ctx, one_ctx;
  for (size_t i = 0; i < prompts.size(); ++i) {
    spread_ctx.emplace_back(c);
    one_ctx.emplace_back(c);
  }
  std::vector<Context*> spread_ptr, one_ptr;
  for (size_t i = 0; i < prompts.size(); ++i) {
    spread_ptr.push_back(&spread_ctx[i]);
    one_ptr.push_back(&one_ctx[i]);
  }
  std::vector<MiniBatch> prefill, decode;
  for (size_t i = 0; i < prompts.size(); ++i) {
    prefill.push_back(MiniBatch::FromTokens(prompts[i], 0));
    decode.push_back(MiniBatch::Single(40 + static_cast<int>(i),
                                       static_cast<int>(prompts[i].size())));
  }
  const CudaModelReplicas spread = UploadModelWeightsToDevices(&model, two);
  for (const auto* step : {&prefill, &decode}) {
    const std::vector<Tensor> got = ForwardBatchesCuda(spread_ptr, spread, *step);
    const std::vector<Tensor> want_l = ForwardBatchesCuda(one_ptr, one, *step);
    bool ok = got.size() == prompts.size();
    for (size_t i = 0; ok && i < prompts.size(); ++i) ok = BitEqual(got[i].data, want_l[i].data);
    Expect(ok, step == &prefill ? "ForwardBatchesCuda prefill over 2 devices bit-exact"
                                : "ForwardBatchesCuda decode over 2 devices bit-exact");
  }
  bool placed = true;
  for (size_t i = 0; i < prompts.size(); ++i) {
    const int expect = i < 3 ? 0 : 1;  // ShardRange(5, 2): [0, 3) and [3, 5)
    placed = placed && CudaPointerDevice(spread_ctx[i].cuda_cache.Keys(0)) == expect;
    placed = placed && spread_ctx[i].position == one_ctx[i].position;
  }
  Expect(placed, "each request's cache on its device, positions advanced");
  std::vector<Context*> reversed(spread_ptr.rbegin(), spread_ptr.rend());
  std::vector<MiniBatch> again(decode.rbegin(), decode.rend());
  Expect(Throws<std::invalid_argument>([&] { ForwardBatchesCuda(reversed, spread, again); }),
         "a context moved to another device -> invalid_argument");
  std::vector<Context*> twice = {spread_ptr[0], spread_ptr[0]};
  std::vector<MiniBatch> two_batches = {decode[0], decode[0]};
  Expect(Throws<std::invalid_argument>([&] { ForwardBatchesCuda(twice, spread, two_batches); }),
         "a context listed twice -> invalid_argument");
}

}  // namespace

int main(int argc, char** argv) {
  const bool cpu_only = argc > 1 && std::string(argv[1]) == "--cpu";
  try {
    TestParseAndValidate();
    if (!cpu_only) {
      int count = 0;
      if (cudaGetDeviceCount(&count) != cudaSuccess || count < 2) {
        std::printf("devices skipped: %d CUDA device(s), need 2\n", count);
        return g_failures == 0 ? 0 : 1;
      }
      TestDevices();
    }
  } catch (const std::exception& e) {
    std::printf("FAIL: exception %s\n", e.what());
    return 1;
  }
  std::printf("%d checks, %d failures\n", g_checks, g_failures);
  if (g_failures != 0) return 1;
  std::printf(cpu_only ? "devices cpu ok\n" : "devices ok\n");
  return 0;
}
