// C entry points over the reference's own CPU operators — TEST INFRASTRUCTURE.
//
// This file is compiled together with the unmodified reference sources
// (src/tensor.cc, src/ops.cc, src/matmul_optimized.cc, src/thread_pool.cc,
// src/quantized_tensor.cc, src/quant.cc of mini-lla, read where they lie) into
// oracle/_ref/libmlref.so by oracle/Makefile.  It serves two purposes:
//   1. pinning the C restatement (mlb_oracle.c) and generating the golden
//      fixtures: the mlref_*_rows functions run the reference's RmsNorm, Add,
//      SwiGlu, Softmax, Rope and DequantizeRow on raw row-major buffers;
//   2. the timed CPU baseline: mlref_bench_* run the same functions per token
//      row inside the reference's ParallelFor thread pool, on inputs prepared
//      as reference Tensors outside the timed region.
// It is never linked into, or called by, the product library.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <vector>

#include "mini_llama/kv_cache.h"
#include "mini_llama/ops.h"
#include "mini_llama/quant.h"
#include "mini_llama/quantized_tensor.h"
#include "mini_llama/tensor.h"
#include "mini_llama/thread_pool.h"

using mini_lla::QuantizedTensor;
using mini_lla::QuantType;
using mini_lla::RopeType;
using mini_lla::Tensor;

namespace {

Tensor RowTensor(const float* data, int64_t n) {
  Tensor t({static_cast<int>(n)});
  std::memcpy(t.data.data(), data, sizeof(float) * n);
  return t;
}

QuantType ToQuantType(int qtype) {
  switch (qtype) {
    case 0: return QuantType::kF32;
    case 1: return QuantType::kQ8_0;
    case 2: return QuantType::kQ4_0;
    case 3: return QuantType::kQ4_1;
  }
  throw std::invalid_argument("unknown qtype");
}

// Wraps raw ggml block bytes as a reference QuantizedTensor (the layout is
// the reference's own Block structs, quantized_tensor.h:19-35).
QuantizedTensor MakeTable(const void* table, int qtype, int64_t vocab,
                          int64_t cols) {
  QuantizedTensor w;
  w.type = ToQuantType(qtype);
  w.rows = static_cast<int>(vocab);
  w.cols = static_cast<int>(cols);
  const size_t blocks = static_cast<size_t>(vocab) * w.BlocksPerRow();
  switch (w.type) {
    case QuantType::kF32: {
      Tensor t({static_cast<int>(vocab), static_cast<int>(cols)});
      std::memcpy(t.data.data(), table, sizeof(float) * vocab * cols);
      w.f32 = std::move(t);
      break;
    }
    case QuantType::kQ8_0:
      w.q8_0.resize(blocks);
      std::memcpy(w.q8_0.data(), table, blocks * sizeof(mini_lla::BlockQ8_0));
      break;
    case QuantType::kQ4_0:
      w.q4_0.resize(blocks);
      std::memcpy(w.q4_0.data(), table, blocks * sizeof(mini_lla::BlockQ4_0));
      break;
    case QuantType::kQ4_1:
      w.q4_1.resize(blocks);
      std::memcpy(w.q4_1.data(), table, blocks * sizeof(mini_lla::BlockQ4_1));
      break;
  }
  return w;
}

// AddBias of src/forward.cc:36-47 sits in an anonymous namespace there; this
// is the same element-wise in-place add.
void AddBiasInPlace(Tensor* value, const float* bias) {
  if (bias == nullptr) return;
  for (size_t i = 0; i < value->Size(); ++i) value->data[i] += bias[i];
}

template <typename F>
int Guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::out_of_range&) {
    return 3;
  } catch (const std::exception&) {
    return 1;
  }
}

}  // namespace

extern "C" {

int mlref_thread_count() { return mini_lla::ThreadCount(); }
void mlref_set_thread_count(int n) { mini_lla::SetThreadCount(n); }

// y = RmsNorm(Add(x, residual)) per row; residual/h may be null.
int mlref_rmsnorm_rows(const float* x, const float* residual, float* h,
                       float* y, const float* w, int64_t rows, int64_t cols,
                       float eps) {
  return Guard([&] {
    const Tensor weight = RowTensor(w, cols);
    for (int64_t r = 0; r < rows; ++r) {
      Tensor xr = RowTensor(x + r * cols, cols);
      if (residual != nullptr) {
        xr = mini_lla::Add(xr, RowTensor(residual + r * cols, cols));
        if (h != nullptr) std::memcpy(h + r * cols, xr.data.data(), 4 * cols);
      }
      const Tensor yr = mini_lla::RmsNorm(xr, weight, eps);
      std::memcpy(y + r * cols, yr.data.data(), 4 * cols);
    }
  });
}

int mlref_swiglu_rows(const float* gate, const float* up, float* out,
                      int64_t rows, int64_t cols) {
  return Guard([&] {
    for (int64_t r = 0; r < rows; ++r) {
      const Tensor o = mini_lla::SwiGlu(RowTensor(gate + r * cols, cols),
                                        RowTensor(up + r * cols, cols));
      std::memcpy(out + r * cols, o.data.data(), 4 * cols);
    }
  });
}

int mlref_silu(const float* x, float* out, int64_t n) {
  return Guard([&] {
    const Tensor o = mini_lla::Silu(RowTensor(x, n));
    std::memcpy(out, o.data.data(), 4 * n);
  });
}

// Softmax of the first valid_len[r] entries, zeros after (valid_len may be
// null: full rows).
int mlref_softmax_rows(const float* x, float* y, int64_t rows, int64_t cols,
                       const int32_t* valid_len) {
  return Guard([&] {
    for (int64_t r = 0; r < rows; ++r) {
      const int64_t len = valid_len != nullptr ? valid_len[r] : cols;
      const Tensor o = mini_lla::Softmax(RowTensor(x + r * cols, len));
      std::memcpy(y + r * cols, o.data.data(), 4 * len);
      std::fill(y + r * cols + len, y + (r + 1) * cols, 0.0f);
    }
  });
}

// Bias add then Rope per token, q [rows, nq, hd], k [rows, nk, hd] in place.
int mlref_rope_rows(float* q, float* k, const float* bq, const float* bk,
                    const int32_t* positions, int64_t rows, int nq, int nk,
                    int hd, float theta, int neox) {
  return Guard([&] {
    for (int64_t t = 0; t < rows; ++t) {
      Tensor qt({nq, hd});
      Tensor kt({nk, hd});
      std::memcpy(qt.data.data(), q + t * nq * hd, 4 * nq * hd);
      std::memcpy(kt.data.data(), k + t * nk * hd, 4 * nk * hd);
      AddBiasInPlace(&qt, bq);
      AddBiasInPlace(&kt, bk);
      mini_lla::Rope(qt, kt, positions[t], theta,
                     neox ? RopeType::kNeoX : RopeType::kNormal);
      std::memcpy(q + t * nq * hd, qt.data.data(), 4 * nq * hd);
      std::memcpy(k + t * nk * hd, kt.data.data(), 4 * nk * hd);
    }
  });
}

int mlref_embedding_rows(const void* table, int qtype, int64_t vocab,
                         int64_t cols, const int32_t* tokens, int64_t rows,
                         float* out) {
  return Guard([&] {
    const QuantizedTensor w = MakeTable(table, qtype, vocab, cols);
    for (int64_t t = 0; t < rows; ++t) {
      mini_lla::DequantizeRow(w, tokens[t], out + t * cols);
    }
  });
}

// Linear layer through the reference (quant.cc:306-318 -> LinearWithBlocks,
// or the F32 LinearDispatch): x [t_rows, k] -> y [t_rows, n].
int mlref_linear(const void* table, int qtype, int64_t n, int64_t k,
                 const float* x, int64_t t_rows, float* y) {
  return Guard([&] {
    const QuantizedTensor w = MakeTable(table, qtype, n, k);
    Tensor input({static_cast<int>(t_rows), static_cast<int>(k)});
    std::memcpy(input.data.data(), x, 4 * t_rows * k);
    const Tensor out = mini_lla::Linear(input, w);
    std::memcpy(y, out.data.data(), 4 * t_rows * n);
  });
}

// Decode attention through the reference's KvCache (kv_cache.cc) and
// Softmax (ops.cc).  AttentionHead of src/forward.cc:50-67 sits in an
// anonymous namespace there; this is its loop, step for step, over the
// reference's own cache accessors.  keys/values: [visible, kv_heads, hd].
int mlref_attention_decode(const float* q, const float* keys,
                           const float* values, float* out, int64_t position,
                           int n_heads, int n_kv_heads, int hd) {
  return Guard([&] {
    const int visible = static_cast<int>(position) + 1;
    mini_lla::KvCache cache(1, visible, n_kv_heads, hd);
    for (int t = 0; t < visible; ++t) {
      Tensor k({n_kv_heads, hd}), v({n_kv_heads, hd});
      std::memcpy(k.data.data(), keys + static_cast<size_t>(t) * n_kv_heads * hd,
                  4 * n_kv_heads * hd);
      std::memcpy(v.data.data(), values + static_cast<size_t>(t) * n_kv_heads * hd,
                  4 * n_kv_heads * hd);
      cache.Write(0, t, k, v);
    }
    const int group = n_heads / n_kv_heads;
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    for (int head = 0; head < n_heads; ++head) {
      const int kv_head = head / group;
      Tensor scores({visible});
      for (int t = 0; t < visible; ++t) {
        const float* key = cache.KeyPtr(0, t, kv_head);
        float dot = 0.0f;
        for (int i = 0; i < hd; ++i) dot += q[head * hd + i] * key[i];
        scores.data[static_cast<size_t>(t)] = dot * scale;
      }
      const Tensor weights = mini_lla::Softmax(scores);
      float* output = out + head * hd;
      for (int i = 0; i < hd; ++i) output[i] = 0.0f;
      for (int t = 0; t < visible; ++t) {
        const float* value = cache.ValuePtr(0, t, kv_head);
        const float weight = weights.data[static_cast<size_t>(t)];
        for (int i = 0; i < hd; ++i) output[i] += weight * value[i];
      }
    }
  });
}

// Quantize through the reference's own quantisers (quant.cc:230-266); used
// only to build realistic fixtures.  out must hold the table's block bytes.
int mlref_quantize(const float* values, int64_t rows, int64_t cols, int qtype,
                   void* out) {
  return Guard([&] {
    Tensor t({static_cast<int>(rows), static_cast<int>(cols)});
    std::memcpy(t.data.data(), values, 4 * rows * cols);
    const QuantizedTensor q = mini_lla::Quantize(t, ToQuantType(qtype));
    switch (q.type) {
      case QuantType::kF32:
        std::memcpy(out, q.f32.data.data(), 4 * rows * cols);
        break;
      case QuantType::kQ8_0:
        std::memcpy(out, q.q8_0.data(), q.q8_0.size() * sizeof(q.q8_0[0]));
        break;
      case QuantType::kQ4_0:
        std::memcpy(out, q.q4_0.data(), q.q4_0.size() * sizeof(q.q4_0[0]));
        break;
      case QuantType::kQ4_1:
        std::memcpy(out, q.q4_1.data(), q.q4_1.size() * sizeof(q.q4_1[0]));
        break;
    }
  });
}

// ---------------------------------------------------------------------------
// Timed CPU baseline: inputs are prepared once as reference Tensors (the form
// the reference's callers hold), then each bench call fans the token rows out
// over the reference thread pool and calls the reference operator per row,
// allocating its output Tensor exactly as the reference does.

struct MlrefRows {
  std::vector<Tensor> rows;
};

void* mlref_rows_new(const float* data, int64_t rows, int64_t cols) {
  auto* h = new MlrefRows;
  h->rows.reserve(rows);
  for (int64_t r = 0; r < rows; ++r)
    h->rows.push_back(RowTensor(data + r * cols, cols));
  return h;
}

// Rows shaped [heads, hd] for RoPE.
void* mlref_heads_new(const float* data, int64_t rows, int heads, int hd) {
  auto* h = new MlrefRows;
  h->rows.reserve(rows);
  for (int64_t r = 0; r < rows; ++r) {
    Tensor t({heads, hd});
    std::memcpy(t.data.data(), data + r * heads * hd, 4 * heads * hd);
    h->rows.push_back(std::move(t));
  }
  return h;
}

void mlref_rows_free(void* h) { delete static_cast<MlrefRows*>(h); }

void* mlref_table_new(const void* table, int qtype, int64_t vocab,
                      int64_t cols) {
  return new QuantizedTensor(MakeTable(table, qtype, vocab, cols));
}

void mlref_table_free(void* h) { delete static_cast<QuantizedTensor*>(h); }

// (Add +) RmsNorm for every row (residual may be null: RmsNorm alone);
// returns a checksum so nothing is elided.
double mlref_bench_rmsnorm(void* x, void* residual, void* weight, float eps) {
  auto& xs = static_cast<MlrefRows*>(x)->rows;
  auto* rs = residual != nullptr ? &static_cast<MlrefRows*>(residual)->rows
                                 : nullptr;
  const Tensor& w = static_cast<MlrefRows*>(weight)->rows[0];
  std::vector<float> sink(xs.size());
  mini_lla::ParallelFor(static_cast<int>(xs.size()), [&](int b, int e) {
    for (int r = b; r < e; ++r) {
      if (rs != nullptr) {
        const Tensor h = mini_lla::Add(xs[r], (*rs)[r]);
        const Tensor y = mini_lla::RmsNorm(h, w, eps);
        sink[r] = y.data[0] + h.data[0];
      } else {
        const Tensor y = mini_lla::RmsNorm(xs[r], w, eps);
        sink[r] = y.data[0];
      }
    }
  });
  double s = 0;
  for (float v : sink) s += v;
  return s;
}

double mlref_bench_swiglu(void* gate, void* up) {
  auto& gs = static_cast<MlrefRows*>(gate)->rows;
  auto& us = static_cast<MlrefRows*>(up)->rows;
  std::vector<float> sink(gs.size());
  mini_lla::ParallelFor(static_cast<int>(gs.size()), [&](int b, int e) {
    for (int r = b; r < e; ++r) {
      const Tensor o = mini_lla::SwiGlu(gs[r], us[r]);
      sink[r] = o.data[0];
    }
  });
  double s = 0;
  for (float v : sink) s += v;
  return s;
}

// Bias add + Rope in place on the prepared [heads, hd] rows.
double mlref_bench_rope(void* q, void* k, const float* bq, const float* bk,
                        const int32_t* positions, float theta, int neox) {
  auto& qs = static_cast<MlrefRows*>(q)->rows;
  auto& ks = static_cast<MlrefRows*>(k)->rows;
  const RopeType type = neox ? RopeType::kNeoX : RopeType::kNormal;
  mini_lla::ParallelFor(static_cast<int>(qs.size()), [&](int b, int e) {
    for (int r = b; r < e; ++r) {
      AddBiasInPlace(&qs[r], bq);
      AddBiasInPlace(&ks[r], bk);
      mini_lla::Rope(qs[r], ks[r], positions[r], theta, type);
    }
  });
  return qs.empty() ? 0.0 : qs[0].data[0];
}

double mlref_bench_softmax(void* x, const int32_t* valid_len) {
  auto& xs = static_cast<MlrefRows*>(x)->rows;
  std::vector<float> sink(xs.size());
  mini_lla::ParallelFor(static_cast<int>(xs.size()), [&](int b, int e) {
    for (int r = b; r < e; ++r) {
      Tensor visible = xs[r];
      if (valid_len != nullptr) {
        visible.data.resize(valid_len[r]);
        visible.shape[0] = valid_len[r];
      }
      const Tensor o = mini_lla::Softmax(visible);
      sink[r] = o.data[0];
    }
  });
  double s = 0;
  for (float v : sink) s += v;
  return s;
}

// Embedding rows into a caller buffer [rows, cols] (the reference writes the
// dequantised row into the caller's vector, forward.cc:29-33).
double mlref_bench_embedding(void* table, const int32_t* tokens, int64_t rows,
                             float* out) {
  const QuantizedTensor& w = *static_cast<QuantizedTensor*>(table);
  const int64_t cols = w.cols;
  mini_lla::ParallelFor(static_cast<int>(rows), [&](int b, int e) {
    for (int r = b; r < e; ++r) {
      mini_lla::DequantizeRow(w, tokens[r], out + r * cols);
    }
  });
  return out[0];
}

}  // extern "C"
