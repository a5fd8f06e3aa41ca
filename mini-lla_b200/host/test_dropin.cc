// Drop-in check of the C++ operator layer: mini-lla's own GPU API
// (cuda_ops.h, cuda_tensor.h, cuda_runtime.h of the reference), served by
// this library's cuda_ops.cc / cuda_runtime.cc over libmlb.so, compared with
// the reference's CPU operators (ops.cc, quant.cc) on the same inputs.
//
// Built by `make -C oracle dropin` against the reference's headers and CPU
// sources; prints one line per failed check and exits non-zero on failure.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <random>
#include <thread>
#include <stdexcept>
#include <string>
#include <vector>

#include "mini_llama/cuda_attention.h"
#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/cuda_matmul.h"
#include "mini_llama/kv_cache.h"
#include "mini_llama/cuda_ops.h"
#include "mini_llama/ops.h"
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

bool BitEqual(const std::vector<float>& a, const std::vector<float>& b) {
  if (a.size() != b.size()) return false;
  for (size_t i = 0; i < a.size(); ++i) {
    if (std::isnan(a[i]) && std::isnan(b[i])) continue;
    uint32_t x, y;
    std::memcpy(&x, &a[i], 4);
    std::memcpy(&y, &b[i], 4);
    if (x != y) return false;
  }
  return true;
}

double MaxRel(const std::vector<float>& got, const std::vector<float>& want) {
  if (got.size() != want.size()) return 1e30;
  double worst = 0;
  for (size_t i = 0; i < got.size(); ++i) {
    if (got[i] == want[i]) continue;
    worst = std::max(worst, std::fabs(double(got[i]) - want[i]) / std::fabs(double(want[i])));
  }
  return worst;
}

Tensor Random(std::vector<int> shape, std::mt19937& rng, float scale = 1.0f,
              float shift = 0.0f) {
  Tensor t(shape);
  std::normal_distribution<float> n(0.0f, 1.0f);
  for (float& v : t.data) v = n(rng) * scale + shift;
  return t;
}

// A norm/bias vector uploaded the way UploadVector does (cuda_weights.cc:65-77).
CudaWeight VectorWeight(const Tensor& t) {
  CudaWeight w;
  w.type = QuantType::kF32;
  w.rows = static_cast<int>(t.Size());
  w.cols = 1;
  w.linear = false;
  w.buffer.Reset(t.Size() * sizeof(float));
  w.buffer.Upload(t.data.data(), t.Size() * sizeof(float));
  return w;
}

// A table uploaded as raw blocks the way UploadQuantized does
// (cuda_weights.cc:33-62).
CudaWeight TableWeight(const QuantizedTensor& q) {
  CudaWeight w;
  w.type = q.type;
  w.rows = q.rows;
  w.cols = q.cols;
  const size_t bytes = QuantizedBytes(q);
  w.buffer.Reset(bytes);
  const void* src = q.type == QuantType::kF32 ? static_cast<const void*>(q.f32.data.data())
                    : q.type == QuantType::kQ8_0 ? static_cast<const void*>(q.q8_0.data())
                    : q.type == QuantType::kQ4_0 ? static_cast<const void*>(q.q4_0.data())
                                                 : static_cast<const void*>(q.q4_1.data());
  w.buffer.Upload(src, bytes);
  return w;
}

template <typename F>
bool Throws(F&& f) {
  try {
    f();
  } catch (const std::exception&) {
    return true;
  }
  return false;
}

void TestPerVectorOps(std::mt19937& rng) {
  for (int n : {3, 896, 4096, 3584, 37}) {
    const Tensor x = Random({n}, rng);
    const Tensor w = Random({n}, rng, 0.1f, 1.0f);
    const CudaWeight dw = VectorWeight(w);
    const CudaTensor dx = CudaTensor::FromHost(x);
    const Tensor y = CudaRmsNorm(dx, dw, 1e-5f).Download();
    Expect(MaxRel(y.data, RmsNorm(x, w, 1e-5f).data) <= 1e-5,
           "CudaRmsNorm n=" + std::to_string(n));
    const Tensor b = Random({n}, rng);
    const CudaTensor db = CudaTensor::FromHost(b);
    Expect(BitEqual(CudaAdd(dx, db).Download().data, Add(x, b).data),
           "CudaAdd n=" + std::to_string(n));
    Expect(MaxRel(CudaSilu(dx).Download().data, Silu(x).data) <= 1e-5,
           "CudaSilu n=" + std::to_string(n));
    Expect(MaxRel(CudaMul(CudaSilu(dx), db).Download().data, SwiGlu(x, b).data) <= 1e-5,
           "CudaSilu+CudaMul n=" + std::to_string(n));
    Expect(MaxRel(CudaSoftmax(dx).Download().data, Softmax(x).data) <= 1e-5,
           "CudaSoftmax n=" + std::to_string(n));
    Tensor biased = x;
    for (size_t i = 0; i < biased.Size(); ++i) biased.data[i] += b.data[i];
    const CudaWeight dbias = VectorWeight(b);
    Expect(BitEqual(CudaAddBias(dx, &dbias).Download().data, biased.data),
           "CudaAddBias n=" + std::to_string(n));
    Expect(BitEqual(CudaAddBias(dx, nullptr).Download().data, x.data),
           "CudaAddBias(null) n=" + std::to_string(n));
  }
  // reference tests/test_ops.cc:41 through the GPU path
  Tensor x({3});
  x.data = {1, 2, 3};
  const CudaWeight ones = VectorWeight(Tensor({3}, 1.0f));
  const float y0 = CudaRmsNorm(CudaTensor::FromHost(x), ones, 1e-5f).Download().data[0];
  Expect(std::fabs(y0 - 0.46291f) <= 1e-4, "CudaRmsNorm [1,2,3] constant");
  // error behaviour of cuda_ops.cu:196, 232, 243, 255
  const CudaTensor d3 = CudaTensor::FromHost(x);
  const CudaTensor d2 = CudaTensor::FromHost(Tensor({2}));
  Expect(Throws([&] { CudaRmsNorm(d2, ones, 1e-5f); }), "CudaRmsNorm mismatch throws");
  Expect(Throws([&] { CudaMul(d3, d2); }), "CudaMul mismatch throws");
  Expect(Throws([&] { CudaAdd(d3, d2); }), "CudaAdd mismatch throws");
  Expect(Throws([&] { CudaSoftmax(CudaTensor({2, 2})); }), "CudaSoftmax rank throws");
}

void TestRope(std::mt19937& rng) {
  struct Case { int nq, nk, hd; float theta; RopeType type; };
  const Case cases[] = {{14, 2, 64, 1e6f, RopeType::kNeoX},
                        {32, 8, 128, 5e5f, RopeType::kNormal},
                        {32, 32, 128, 1e4f, RopeType::kNormal},
                        {28, 4, 128, 1e6f, RopeType::kNeoX},
                        {3, 1, 6, 1e4f, RopeType::kNormal}};
  for (const Case& c : cases) {
    for (int position : {0, 1, 255, 2047, 16383, 65535}) {
      Tensor q = Random({c.nq, c.hd}, rng);
      Tensor k = Random({c.nk, c.hd}, rng);
      CudaTensor dq = CudaTensor::FromHost(q.Reshape({c.nq * c.hd}));
      CudaTensor dk = CudaTensor::FromHost(k.Reshape({c.nk * c.hd}));
      Rope(q, k, position, c.theta, c.type);
      CudaRope(&dq, &dk, position, c.theta, c.nq, c.nk, c.hd, c.type);
      Expect(BitEqual(dq.Download().data, q.data) && BitEqual(dk.Download().data, k.data),
             "CudaRope hd=" + std::to_string(c.hd) + " pos=" + std::to_string(position));
    }
  }
  // test_ops.cc:65-82 constants
  for (RopeType type : {RopeType::kNormal, RopeType::kNeoX}) {
    Tensor host({2});
    host.data = {1.0f, 0.0f};
    CudaTensor dq = CudaTensor::FromHost(host);
    CudaTensor dk = CudaTensor::FromHost(host);
    CudaRope(&dq, &dk, 1, 10000.0f, 1, 1, 2, type);
    const Tensor r = dq.Download();
    Expect(std::fabs(r.data[0] - std::cos(1.0f)) <= 1e-5 &&
               std::fabs(r.data[1] - std::sin(1.0f)) <= 1e-5,
           "CudaRope rotates by 1 rad");
  }
  CudaTensor dq({8}), dk({8});
  Expect(Throws([&] { CudaRope(&dq, &dk, -1, 1e4f, 1, 1, 8, RopeType::kNormal); }),
         "CudaRope negative position throws");
  Expect(Throws([&] { CudaRope(nullptr, &dk, 0, 1e4f, 1, 1, 8, RopeType::kNormal); }),
         "CudaRope null throws");
  Expect(CudaRopeTableRows(1e6f, 64) >= 65536, "RoPE table grown and cached");
}

void TestEmbedding(std::mt19937& rng) {
  for (QuantType type : {QuantType::kF32, QuantType::kQ8_0, QuantType::kQ4_0,
                         QuantType::kQ4_1}) {
    for (int cols : {896, 4096, 40, 38}) {
      const int vocab = 64;
      const Tensor values = Random({vocab, cols}, rng);
      const QuantizedTensor table = Quantize(values, type);
      const CudaWeight dt = TableWeight(table);
      std::vector<float> want(cols);
      for (int token : {0, 1, 31, vocab - 1}) {
        DequantizeRow(table, token, want.data());
        Expect(BitEqual(CudaEmbeddingRow(dt, token).Download().data, want),
               std::string("CudaEmbeddingRow ") + QuantTypeName(type) +
                   " cols=" + std::to_string(cols));
      }
      Expect(Throws([&] { CudaEmbeddingRow(dt, vocab); }) &&
                 Throws([&] { CudaEmbeddingRow(dt, -1); }),
             "CudaEmbeddingRow out of range throws");
      std::vector<int> tokens = {5, 0, 63, 5, 17};
      const Tensor rows = CudaEmbeddingRows(dt, tokens).Download();
      bool ok = true;
      for (size_t r = 0; r < tokens.size(); ++r) {
        DequantizeRow(table, tokens[r], want.data());
        std::vector<float> got(rows.data.begin() + r * cols,
                               rows.data.begin() + (r + 1) * cols);
        ok = ok && BitEqual(got, want);
      }
      Expect(ok, std::string("CudaEmbeddingRows ") + QuantTypeName(type));
    }
  }
}

void TestBatched(std::mt19937& rng) {
  const int rows = 33, cols = 4096;
  const Tensor x = Random({rows, cols}, rng);
  const Tensor r = Random({rows, cols}, rng);
  const Tensor w = Random({cols}, rng, 0.1f, 1.0f);
  const CudaWeight dw = VectorWeight(w);
  const CudaTensor dx = CudaTensor::FromHost(x);
  const CudaTensor dr = CudaTensor::FromHost(r);
  CudaTensor dh;
  const Tensor y = CudaAddRmsNormRows(dx, &dr, dw, 1e-5f, &dh).Download();
  const Tensor h = dh.Download();
  bool h_ok = true, y_ok = true;
  for (int i = 0; i < rows; ++i) {
    Tensor xi({cols}), ri({cols});
    std::copy(x.data.begin() + i * cols, x.data.begin() + (i + 1) * cols, xi.data.begin());
    std::copy(r.data.begin() + i * cols, r.data.begin() + (i + 1) * cols, ri.data.begin());
    const Tensor hi = Add(xi, ri);
    const Tensor yi = RmsNorm(hi, w, 1e-5f);
    h_ok = h_ok && BitEqual(std::vector<float>(h.data.begin() + i * cols, h.data.begin() + (i + 1) * cols), hi.data);
    y_ok = y_ok && MaxRel(std::vector<float>(y.data.begin() + i * cols, y.data.begin() + (i + 1) * cols), yi.data) <= 1e-5;
  }
  Expect(h_ok, "CudaAddRmsNormRows residual sum bit-exact");
  Expect(y_ok, "CudaAddRmsNormRows within 1e-5");

  const Tensor g = Random({rows, 14336}, rng, 3.0f);
  const Tensor u = Random({rows, 14336}, rng);
  Expect(MaxRel(CudaSwiGlu(CudaTensor::FromHost(g), CudaTensor::FromHost(u)).Download().data,
                SwiGlu(g, u).data) <= 1e-5,
         "CudaSwiGlu within 1e-5");

  const int nq = 28, nk = 4, hd = 128;
  Tensor q = Random({rows, nq * hd}, rng);
  Tensor k = Random({rows, nk * hd}, rng);
  const Tensor bq = Random({nq * hd}, rng, 0.02f);
  const Tensor bk = Random({nk * hd}, rng, 0.02f);
  const CudaWeight dbq = VectorWeight(bq), dbk = VectorWeight(bk);
  for (bool consecutive : {true, false}) {
    std::vector<int> positions(rows);
    for (int i = 0; i < rows; ++i) positions[i] = consecutive ? 1000 + i : (i * 7919) % 65536;
    CudaTensor dq = CudaTensor::FromHost(q), dk = CudaTensor::FromHost(k);
    CudaRopeRows(&dq, &dk, &dbq, &dbk, positions, 1e6f, nq, nk, hd, RopeType::kNeoX);
    const Tensor gq = dq.Download(), gk = dk.Download();
    bool ok = true;
    for (int i = 0; i < rows; ++i) {
      Tensor qi({nq, hd}), ki({nk, hd});
      for (int j = 0; j < nq * hd; ++j) qi.data[j] = q.data[i * nq * hd + j] + bq.data[j];
      for (int j = 0; j < nk * hd; ++j) ki.data[j] = k.data[i * nk * hd + j] + bk.data[j];
      Rope(qi, ki, positions[i], 1e6f, RopeType::kNeoX);
      ok = ok && BitEqual(std::vector<float>(gq.data.begin() + i * nq * hd, gq.data.begin() + (i + 1) * nq * hd), qi.data) &&
           BitEqual(std::vector<float>(gk.data.begin() + i * nk * hd, gk.data.begin() + (i + 1) * nk * hd), ki.data);
    }
    Expect(ok, consecutive ? "CudaRopeRows consecutive positions bit-exact"
                           : "CudaRopeRows scattered positions bit-exact");
  }

  const Tensor s = Random({rows, 256}, rng, 2.0f);
  std::vector<int> lengths(rows);
  for (int i = 0; i < rows; ++i) lengths[i] = i * 7 % 256 + 1;
  const Tensor p = CudaSoftmaxRows(CudaTensor::FromHost(s), &lengths).Download();
  bool ok = true;
  for (int i = 0; i < rows; ++i) {
    Tensor vis({lengths[i]});
    std::copy(s.data.begin() + i * 256, s.data.begin() + i * 256 + lengths[i], vis.data.begin());
    const Tensor want = Softmax(vis);
    std::vector<float> got(p.data.begin() + i * 256, p.data.begin() + i * 256 + lengths[i]);
    ok = ok && MaxRel(got, want.data) <= 1e-5;
    for (int j = lengths[i]; j < 256; ++j) ok = ok && p.data[i * 256 + j] == 0.0f;
  }
  Expect(ok, "CudaSoftmaxRows causal rows within 1e-5");
}

void TestRuntime() {
  int device = 0;
  cudaGetDevice(&device);
  // 22 MiB blocks (a size no other check allocates)
  const int n = (21 << 18) + 1;
  const size_t before = CudaPoolCachedBytes(device);
  {
    CudaTensor a({n});
    CudaTensor b({n});
  }
  Expect(CudaPoolCachedBytes(device) == before + (size_t{44} << 20),
         "pool keeps freed blocks");
  const size_t cached = CudaPoolCachedBytes(device);
  {
    CudaTensor c({n});
    Expect(CudaPoolCachedBytes(device) == cached - (size_t{22} << 20),
           "pool reuses a freed block");
  }
  Expect(CudaPoolCachedBytes(device) == cached, "pool takes the block back");
  // large transfers go through pinned staging and round-trip exactly
  std::vector<float> big(5 << 20);
  for (size_t i = 0; i < big.size(); ++i) big[i] = static_cast<float>(i) * 0.5f;
  Tensor host({static_cast<int>(big.size())});
  host.data = big;
  Expect(BitEqual(CudaTensor::FromHost(host).Download().data, big),
         "staged upload/download round trip");
  CudaPoolRelease(device);
  Expect(CudaPoolCachedBytes(device) == 0, "pool release");
  Expect(Throws([] { CudaSetDevice(1 << 20); }), "bad device index throws");
}

// CudaLinear (cuda_matmul.h) against the reference's quantised / F32 Linear.
void TestLinear(std::mt19937& rng) {
  for (QuantType type : {QuantType::kF32, QuantType::kQ8_0, QuantType::kQ4_0,
                         QuantType::kQ4_1}) {
    for (int cols : {4096, 896, 40}) {
      const int rows = 300;
      const Tensor values = Random({rows, cols}, rng);
      const QuantizedTensor w = Quantize(values, type);
      const CudaWeight dw = TableWeight(w);
      const Tensor x = Random({cols}, rng);
      const Tensor want = Linear(x, w);
      const Tensor got = CudaLinear(CudaTensor::FromHost(x), dw).Download();
      // |got - want| <= 1e-5 * sum_i |w_i x_i|
      std::vector<float> row(cols);
      bool ok = got.Size() == want.Size();
      for (int j = 0; ok && j < rows; ++j) {
        DequantizeRow(w, j, row.data());
        double mag = 0;
        for (int i = 0; i < cols; ++i) mag += std::fabs(double(row[i]) * x.data[i]);
        ok = std::fabs(double(got.data[j]) - want.data[j]) <= 1e-5 * mag + 1e-30;
      }
      Expect(ok, std::string("CudaLinear ") + QuantTypeName(type) +
                     " cols=" + std::to_string(cols));
    }
  }
  const CudaWeight dw = TableWeight(Quantize(Random({4, 64}, rng), QuantType::kQ8_0));
  Expect(Throws([&] { CudaLinear(CudaTensor({63}), dw); }), "CudaLinear size mismatch throws");
}

// CudaKvCache + CudaAttention against AttentionHead (forward.cc:50-67, in an
// anonymous namespace there, so its loop is restated over the reference's
// own KvCache and Softmax).
void TestAttention(std::mt19937& rng) {
  struct Case { int n_heads, n_kv, hd, layers, max_seq, position; };
  for (const Case& c : {Case{8, 2, 64, 2, 64, 37}, Case{32, 8, 128, 1, 512, 300},
                        Case{14, 2, 64, 3, 300, 255}, Case{4, 4, 32, 1, 8, 0}}) {
    KvCache host(c.layers, c.max_seq, c.n_kv, c.hd);
    CudaKvCache cache;
    cache.Reset(c.layers, c.max_seq, c.n_kv, c.hd);
    const int layer = c.layers - 1;
    for (int t = 0; t <= c.position; ++t) {
      const Tensor k = Random({c.n_kv, c.hd}, rng);
      const Tensor v = Random({c.n_kv, c.hd}, rng);
      host.Write(layer, t, k, v);
      cache.Write(layer, t, CudaTensor::FromHost(k.Reshape({c.n_kv * c.hd})),
                  CudaTensor::FromHost(v.Reshape({c.n_kv * c.hd})));
    }
    const Tensor q = Random({c.n_heads, c.hd}, rng);
    const Tensor got = CudaAttention(CudaTensor::FromHost(q.Reshape({c.n_heads * c.hd})),
                                     cache, layer, c.position, c.n_heads, c.n_kv, c.hd)
                           .Download();
    const int group = c.n_heads / c.n_kv;
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.hd));
    bool ok = true;
    for (int head = 0; head < c.n_heads; ++head) {
      Tensor scores({c.position + 1});
      for (int t = 0; t <= c.position; ++t) {
        const float* key = host.KeyPtr(layer, t, head / group);
        float dot = 0.0f;
        for (int i = 0; i < c.hd; ++i) dot += q.data[head * c.hd + i] * key[i];
        scores.data[t] = dot * scale;
      }
      const Tensor w = Softmax(scores);
      for (int i = 0; i < c.hd; ++i) {
        float want = 0.0f;
        double mag = 0.0;
        for (int t = 0; t <= c.position; ++t) {
          const float value = host.ValuePtr(layer, t, head / group)[i];
          want += w.data[t] * value;
          mag += w.data[t] * std::fabs(value);
        }
        ok = ok && std::fabs(double(got.data[head * c.hd + i]) - want) <= 1e-5 * mag + 1e-30;
      }
    }
    Expect(ok, "CudaAttention heads=" + std::to_string(c.n_heads) +
                   " pos=" + std::to_string(c.position));
    std::vector<float> keys_back(static_cast<size_t>(c.n_kv) * c.hd);
    cudaMemcpy(keys_back.data(),
               cache.Keys(layer) + static_cast<size_t>(c.position) * c.n_kv * c.hd,
               keys_back.size() * sizeof(float), cudaMemcpyDeviceToHost);
    Expect(std::memcmp(keys_back.data(), host.KeyPtr(layer, c.position, 0),
                       keys_back.size() * sizeof(float)) == 0,
           "CudaKvCache::Write copies bit-exact");
    Expect(Throws([&] { cache.Write(layer, c.max_seq, CudaTensor({c.n_kv * c.hd}),
                                    CudaTensor({c.n_kv * c.hd})); }),
           "CudaKvCache::Write out of range throws");
    const size_t at = static_cast<size_t>(c.position) * c.n_kv * c.hd;
    const CudaKvRows kv = CudaKvCacheRows(&cache, layer, c.position, 1);
    Expect(kv.keys == cache.Keys(layer) + at && kv.values == cache.Values(layer) + at,
           "CudaKvCacheRows addresses the cache's own rows");
    Expect(Throws([&] { CudaKvCacheRows(&cache, layer, c.max_seq - 1, 2); }) &&
               Throws([&] { CudaKvCacheRows(&cache, c.layers, 0, 1); }),
           "CudaKvCacheRows past the cache throws");
  }
}

// One host thread per "device" entry; a single-GPU box lists device 0 twice
// (independent token ranges, no waits between them).
void TestShardingAndWaits(std::mt19937& rng) {
  const int vocab = 100, cols = 896, total = 1001;
  const QuantizedTensor table = Quantize(Random({vocab, cols}, rng), QuantType::kQ8_0);
  std::vector<int> tokens(total);
  for (int i = 0; i < total; ++i) tokens[i] = (i * 37) % vocab;
  const std::vector<int> devices = {0, 0, 0};
  std::vector<std::vector<float>> parts(devices.size());
  std::vector<std::pair<int, int>> ranges(devices.size());
  std::mutex m;
  CudaShardRows(total, devices, [&](int, int begin, int end) {
    const CudaWeight dt = TableWeight(table);  // replicated per shard
    std::vector<int> mine(tokens.begin() + begin, tokens.begin() + end);
    const Tensor out = CudaEmbeddingRows(dt, mine).Download();
    std::lock_guard<std::mutex> lock(m);
    const size_t slot = begin == 0 ? 0 : (end == total ? devices.size() - 1 : 1);
    parts[slot] = out.data;
    ranges[slot] = {begin, end};
  });
  bool ok = ranges[0].first == 0 && ranges.back().second == total;
  std::vector<float> want(cols);
  for (size_t s = 0; s < parts.size(); ++s) {
    if (s > 0) ok = ok && ranges[s].first == ranges[s - 1].second;
    for (int r = ranges[s].first; r < ranges[s].second; ++r) {
      DequantizeRow(table, tokens[r], want.data());
      const size_t off = static_cast<size_t>(r - ranges[s].first) * cols;
      ok = ok && BitEqual(std::vector<float>(parts[s].begin() + off,
                                             parts[s].begin() + off + cols), want);
    }
  }
  Expect(ok, "CudaShardRows: contiguous ranges, gathered rows bit-exact");
  Expect(ShardRange(10, 3, 0) == std::make_pair(0, 4) &&
             ShardRange(10, 3, 2) == std::make_pair(7, 10),
         "ShardRange remainder rule");
  // A failing shard: every thread is joined and the first error surfaces.
  std::atomic<int> finished{0};
  const bool rethrown = Throws([&] {
    CudaShardRows(30, devices, [&](int, int begin, int) {
      if (begin == 10) throw std::runtime_error("injected shard failure");
      finished.fetch_add(1);
    });
  });
  Expect(rethrown && finished.load() == 2, "CudaShardRows rethrows after join");

  // Bounded wait: the stream is held by a host function (no GPU work is
  // stalled), the wait times out and returns false, then succeeds once the
  // host releases the stream.
  cudaStream_t stream;
  cudaEvent_t event;
  cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  cudaEventCreateWithFlags(&event, cudaEventDisableTiming);
  static std::atomic<bool> release{false};
  release.store(false);
  cudaLaunchHostFunc(stream, [](void*) {
    for (int i = 0; i < 20000 && !release.load(); ++i) {
      std::this_thread::sleep_for(std::chrono::microseconds(250));
    }
  }, nullptr);
  cudaEventRecord(event, stream);
  const bool early = CudaWaitEvent(event, 50.0);
  release.store(true);
  const bool late = CudaWaitEvent(event, 10000.0);
  Expect(!early && late, "CudaWaitEvent times out, then completes");
  cudaStreamSynchronize(stream);
  cudaEventDestroy(event);
  cudaStreamDestroy(stream);
}

// The row-batched entries that take host arrays (token ids, scattered
// positions, softmax lengths) queue their uploads instead of waiting for the
// device: with the legacy stream held by a host function they return at
// once, and their results are right once it is released.  Inputs, the pool
// blocks and the RoPE table are made beforehand (a first round of the same
// calls), since creating them copies synchronously.
void TestNoHostWait(std::mt19937& rng) {
  const int vocab = 64, cols = 512, rows = 300, nq = 4, nk = 2, hd = 64, width = 96;
  const QuantizedTensor table = Quantize(Random({vocab, cols}, rng), QuantType::kQ4_1);
  const CudaWeight dt = TableWeight(table);
  std::vector<int> tokens(rows), positions(rows), lengths(rows);
  for (int i = 0; i < rows; ++i) {
    tokens[i] = (i * 13) % vocab;
    positions[i] = (i * 7919) % 4096;
    lengths[i] = i % width + 1;
  }
  const Tensor q = Random({rows, nq * hd}, rng), k = Random({rows, nk * hd}, rng);
  const Tensor s = Random({rows, width}, rng, 2.0f);
  const CudaTensor ds = CudaTensor::FromHost(s);
  CudaTensor dq = CudaTensor::FromHost(q), dk = CudaTensor::FromHost(k);
  auto round = [&](CudaTensor* emb, CudaTensor* soft) {
    *emb = CudaEmbeddingRows(dt, tokens);
    CudaRopeRows(&dq, &dk, nullptr, nullptr, positions, 1e4f, nq, nk, hd, RopeType::kNormal);
    *soft = CudaSoftmaxRows(ds, &lengths);
  };
  {
    CudaTensor e, p;
    round(&e, &p);  // warm: pool blocks, RoPE table, pinned ring
  }
  CudaTensor qa = CudaTensor::FromHost(q), ka = CudaTensor::FromHost(k);
  dq = std::move(qa);
  dk = std::move(ka);
  cudaDeviceSynchronize();
  static std::atomic<bool> hold{false};
  hold.store(true);
  cudaLaunchHostFunc(cudaStreamLegacy, [](void*) {
    for (int i = 0; i < 40000 && hold.load(); ++i) {
      std::this_thread::sleep_for(std::chrono::microseconds(250));
    }
  }, nullptr);
  const auto t0 = std::chrono::steady_clock::now();
  CudaTensor emb, soft;
  round(&emb, &soft);
  const double ms = std::chrono::duration<double, std::milli>(
                        std::chrono::steady_clock::now() - t0).count();
  const bool held = cudaStreamQuery(cudaStreamLegacy) == cudaErrorNotReady;
  hold.store(false);
  Expect(held && ms < 2000.0,
         "CudaEmbeddingRows / CudaRopeRows / CudaSoftmaxRows return without waiting (" +
             std::to_string(ms) + " ms, stream held: " + (held ? "yes" : "no") + ")");
  const Tensor ge = emb.Download(), gq = dq.Download(), gs = soft.Download();
  bool ok = true;
  std::vector<float> want(cols);
  for (int i = 0; i < rows; ++i) {
    DequantizeRow(table, tokens[i], want.data());
    ok = ok && BitEqual(std::vector<float>(ge.data.begin() + i * cols,
                                           ge.data.begin() + (i + 1) * cols), want);
    Tensor qi({nq, hd}), ki({nk, hd});
    std::copy(q.data.begin() + i * nq * hd, q.data.begin() + (i + 1) * nq * hd, qi.data.begin());
    std::copy(k.data.begin() + i * nk * hd, k.data.begin() + (i + 1) * nk * hd, ki.data.begin());
    Rope(qi, ki, positions[i], 1e4f, RopeType::kNormal);
    ok = ok && BitEqual(std::vector<float>(gq.data.begin() + i * nq * hd,
                                           gq.data.begin() + (i + 1) * nq * hd), qi.data);
    Tensor vis({lengths[i]});
    std::copy(s.data.begin() + i * width, s.data.begin() + i * width + lengths[i], vis.data.begin());
    ok = ok && MaxRel(std::vector<float>(gs.data.begin() + i * width,
                                         gs.data.begin() + i * width + lengths[i]),
                      Softmax(vis).data) <= 1e-5;
  }
  Expect(ok, "queued uploads: gather bit-exact, RoPE bit-exact, softmax within 1e-5");
}

}  // namespace

int main() {
  std::mt19937 rng(20261201);
  try {
    TestPerVectorOps(rng);
    TestRope(rng);
    TestEmbedding(rng);
    TestBatched(rng);
    TestShardingAndWaits(rng);
    TestNoHostWait(rng);
    TestLinear(rng);
    TestAttention(rng);
    TestRuntime();
  } catch (const std::exception& e) {
    std::printf("FAIL: unexpected exception: %s\n", e.what());
    return 2;
  }
  std::printf("%s: %d checks, %d failures\n", g_failures ? "dropin FAILED" : "dropin ok",
              g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
