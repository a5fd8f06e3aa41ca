// mini-lla's device KV cache and decode attention (the reference's
// include/mini_llama/cuda_attention.h) over libmlb.so.  This file takes the
// place of the reference's src/cuda_attention.cu: the cache keeps the
// reference's layout [layers, max_seq, kv_heads, head_dim] and API;
// attention runs as split-position (flash-decoding) kernels that read each kv
// head's K/V rows once for all query heads of its GQA group, with the slice
// partials in a pooled scratch buffer, instead of one CTA per query head
// holding every score in shared memory.
#include "mini_llama/cuda_attention.h"

#include <cstdint>
#include <stdexcept>
#include <string>

#include "mini_llama/cuda_layer_ops.h"
#include "mlb_ops.h"

namespace mini_lla {
namespace {

void Check(int rc, const char* caller) {
  if (rc == MLB_OK) return;
  const std::string message = std::string(caller) + ": " + mlb_last_error();
  if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
  if (rc == MLB_ERR_RANGE) throw std::out_of_range(message);
  throw std::runtime_error(message);
}

void CheckCache(const CudaKvCache& cache, int layer, int position) {
  if (layer < 0 || layer >= cache.layers()) {
    throw std::out_of_range("CudaKvCache: layer out of range");
  }
  if (position < 0 || position >= cache.max_seq()) {
    throw std::out_of_range("CudaKvCache: position out of range");
  }
}

size_t LayerFloats(const CudaKvCache& cache) {
  return static_cast<size_t>(cache.max_seq()) * cache.kv_heads() * cache.head_dim();
}

}  // namespace

void CudaKvCache::Reset(int layers, int max_seq, int kv_heads, int head_dim) {
  if (layers <= 0 || max_seq <= 0 || kv_heads <= 0 || head_dim <= 0) {
    throw std::invalid_argument("CudaKvCache::Reset: sizes must be positive");
  }
  layers_ = layers;
  max_seq_ = max_seq;
  kv_heads_ = kv_heads;
  head_dim_ = head_dim;
  const size_t count = static_cast<size_t>(layers) * max_seq * kv_heads * head_dim;
  keys_.Reset(count * sizeof(float));
  values_.Reset(count * sizeof(float));
  keys_.Zero();
  values_.Zero();
}

void CudaKvCache::Write(int layer, int position, const CudaTensor& key,
                        const CudaTensor& value) {
  CheckCache(*this, layer, position);
  const size_t count = static_cast<size_t>(kv_heads_) * head_dim_;
  if (key.Size() != count || value.Size() != count) {
    throw std::invalid_argument("CudaKvCache::Write: tensor shape mismatch");
  }
  float* keys = static_cast<float*>(keys_.data()) + layer * LayerFloats(*this);
  float* values = static_cast<float*>(values_.data()) + layer * LayerFloats(*this);
  Check(mlb_kv_write_f32(keys, values, key.data(), value.data(), position, 1,
                         max_seq_, kv_heads_, head_dim_, nullptr),
        "CudaKvCache::Write");
}

void CudaKvCache::Clear() {
  keys_.Clear();
  values_.Clear();
  layers_ = max_seq_ = kv_heads_ = head_dim_ = 0;
}

const float* CudaKvCache::Keys(int layer) const {
  CheckCache(*this, layer, 0);
  return static_cast<const float*>(keys_.data()) + layer * LayerFloats(*this);
}

const float* CudaKvCache::Values(int layer) const {
  CheckCache(*this, layer, 0);
  return static_cast<const float*>(values_.data()) + layer * LayerFloats(*this);
}

CudaTensor CudaAttention(const CudaTensor& q, const CudaKvCache& cache,
                         int layer, int position, int n_heads, int n_kv_heads,
                         int head_dim) {
  CheckCache(cache, layer, position);
  if (q.Size() != static_cast<size_t>(n_heads) * head_dim ||
      n_kv_heads != cache.kv_heads() || head_dim != cache.head_dim()) {
    throw std::invalid_argument("CudaAttention: shape mismatch");
  }
  CudaTensor output({n_heads * head_dim});
  const int64_t need =
      mlb_attention_scratch_floats(n_heads, n_kv_heads, head_dim, position);
  if (need < 0) throw std::invalid_argument("CudaAttention: bad sizes");
  DeviceBuffer scratch;  // pooled; reuse is ordered on the default stream
  scratch.Reset(static_cast<size_t>(need) * sizeof(float));
  Check(mlb_attention_decode_f32(q.data(), cache.Keys(layer), cache.Values(layer),
                                 output.data(), position, cache.max_seq(), n_heads,
                                 n_kv_heads, head_dim,
                                 static_cast<float*>(scratch.data()), need, nullptr),
        "CudaAttention");
  return output;
}

CudaKvRows CudaKvCacheRows(CudaKvCache* cache, int layer, int position, int rows) {
  if (cache == nullptr) throw std::invalid_argument("CudaKvCacheRows: null cache");
  if (rows < 1) throw std::invalid_argument("CudaKvCacheRows: rows < 1");
  CheckCache(*cache, layer, position);
  CheckCache(*cache, layer, position + rows - 1);
  const size_t offset = static_cast<size_t>(position) * cache->kv_heads() * cache->head_dim();
  // the cache's layer buffers are device memory it owns; Keys()/Values() hand
  // them out read-only, the writes go through the same addresses
  return {const_cast<float*>(cache->Keys(layer)) + offset,
          const_cast<float*>(cache->Values(layer)) + offset};
}

void CudaKvCacheWriteRows(CudaKvCache* cache, int layer, int position,
                          const CudaTensor& keys, const CudaTensor& values) {
  if (cache == nullptr) throw std::invalid_argument("CudaKvCacheWriteRows: null cache");
  CheckCache(*cache, layer, position);
  const size_t per = static_cast<size_t>(cache->kv_heads()) * cache->head_dim();
  if (keys.Size() != values.Size() || keys.Size() % per != 0) {
    throw std::invalid_argument("CudaKvCacheWriteRows: tensor shape mismatch");
  }
  const int64_t rows = static_cast<int64_t>(keys.Size() / per);
  // the cache's layer buffers are device memory it owns; Keys()/Values() hand
  // them out read-only, the write goes through the same addresses
  float* k_layer = const_cast<float*>(cache->Keys(layer));
  float* v_layer = const_cast<float*>(cache->Values(layer));
  Check(mlb_kv_write_f32(k_layer, v_layer, keys.data(), values.data(), position, rows,
                         cache->max_seq(), cache->kv_heads(), cache->head_dim(), nullptr),
        "CudaKvCacheWriteRows");
}

CudaTensor CudaAttentionRows(const CudaTensor& q, const CudaKvCache& cache,
                             int layer, int position, int n_heads,
                             int n_kv_heads, int head_dim) {
  CheckCache(cache, layer, position);
  const size_t per = static_cast<size_t>(n_heads) * head_dim;
  if (per == 0 || q.Size() % per != 0 || n_kv_heads != cache.kv_heads() ||
      head_dim != cache.head_dim()) {
    throw std::invalid_argument("CudaAttentionRows: shape mismatch");
  }
  const int rows = static_cast<int>(q.Size() / per);
  CudaTensor output({rows, n_heads * head_dim});
  if (rows == 0) return output;
  const int64_t need = mlb_attention_rows_scratch_floats(n_heads, n_kv_heads, head_dim,
                                                         position, rows);
  if (need < 0) throw std::invalid_argument("CudaAttentionRows: bad sizes");
  DeviceBuffer scratch;  // pooled; reuse is ordered on the default stream
  scratch.Reset(static_cast<size_t>(need) * sizeof(float));
  Check(mlb_attention_rows_f32(q.data(), cache.Keys(layer), cache.Values(layer),
                               output.data(), position, rows, cache.max_seq(), n_heads,
                               n_kv_heads, head_dim, static_cast<float*>(scratch.data()),
                               need, nullptr),
        "CudaAttentionRows");
  return output;
}

}  // namespace mini_lla
