// Row-batched layer operators and device helpers added next to mini-lla's
// per-vector GPU operator API (include/mini_llama/cuda_ops.h of the
// reference, whose eight functions this library also implements).
//
// Every function runs on the current device, on the legacy default stream,
// with the same synchronous-looking semantics and exception types as the
// reference's cuda_ops.cu: std::invalid_argument for a shape mismatch,
// std::out_of_range for a token id outside the table, std::runtime_error for
// a CUDA failure.  Outputs are fresh CudaTensors drawn from a per-device
// caching pool (see CudaPoolCachedBytes) instead of a cudaMalloc per call.
#ifndef MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_LAYER_OPS_H_
#define MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_LAYER_OPS_H_

#include <cstddef>
#include <cstdint>
#include <functional>
#include <utility>
#include <vector>

#include "mini_llama/cuda_attention.h"
#include "mini_llama/cuda_tensor.h"
#include "mini_llama/cuda_weights.h"
#include "mini_llama/ops.h"

namespace mini_lla {

// y[r] = RmsNorm(x[r] + residual[r]) for every row of x [rows, cols]; the
// residual may be null (plain RMSNorm of each row).  When h_out is given it
// receives the sum x + residual (the new residual stream), shaped like x.
// One pass over memory (forward.cc:122-124 fused).
CudaTensor CudaAddRmsNormRows(const CudaTensor& x, const CudaTensor* residual,
                              const CudaWeight& weight, float epsilon,
                              CudaTensor* h_out = nullptr);

// Silu(gate) * up in one pass (ops.cc:108-115); gate and up same shape.
CudaTensor CudaSwiGlu(const CudaTensor& gate, const CudaTensor& up);

// Bias add + RoPE in place for a batch of tokens: q holds rows x n_heads x
// head_dim values, k rows x n_kv_heads x head_dim, rows = positions.size().
// bq / bk may be null.  Bit-exact with Rope (ops.cc:126-142) after AddBias
// (forward.cc:36-47).  Throws std::invalid_argument for a negative position
// or odd head_dim, like Rope.
void CudaRopeRows(CudaTensor* q, CudaTensor* k, const CudaWeight* bq,
                  const CudaWeight* bk, const std::vector<int>& positions,
                  float theta, int n_heads, int n_kv_heads, int head_dim,
                  RopeType rope_type);

// CudaRopeRows on device memory the caller owns: q holds positions.size() x
// n_heads x head_dim floats, k positions.size() x n_kv_heads x head_dim (for
// instance the K rows of a KV cache, rotated where they are stored).
void CudaRopeRowsInPlace(float* q, float* k, const CudaWeight* bq, const CudaWeight* bk,
                         const std::vector<int>& positions, float theta, int n_heads,
                         int n_kv_heads, int head_dim, RopeType rope_type);

// Softmax of the first valid_len[r] entries of each row of x [rows, cols],
// zeros after; valid_len null means full rows.
CudaTensor CudaSoftmaxRows(const CudaTensor& x,
                           const std::vector<int>* valid_len = nullptr);

// One dequantised embedding row per token id -> [tokens.size(), cols].
CudaTensor CudaEmbeddingRows(const CudaWeight& embedding,
                             const std::vector<int>& tokens);

// y[r] = W . x[r] for every row of x [rows, weight.cols] -> [rows,
// weight.rows] (CudaLinear, cuda_matmul.h, for a batch of tokens).
CudaTensor CudaLinearRows(const CudaTensor& x, const CudaWeight& weight);

// CudaLinearRows for up to three weights applied to the same x (the q / k /
// v projections, the FFN gate / up) in one launch: one TF32 split of x and
// one grid for all of them.  The weights must share format and width
// (std::invalid_argument otherwise).
std::vector<CudaTensor> CudaLinearRowsGroup(const CudaTensor& x,
                                            const std::vector<const CudaWeight*>& weights);

// CudaLinearRowsGroup writing weight m's output to outputs[m], device memory
// of rows x weights[m]->rows floats that the caller owns (for instance K and
// V straight into their KV-cache rows).
void CudaLinearRowsGroupInto(const CudaTensor& x, const std::vector<const CudaWeight*>& weights,
                             const std::vector<float*>& outputs);

// value[r] + bias for every row of value [rows, bias size] (AddBias,
// forward.cc:36-47, for a batch of tokens); a null bias copies value.
CudaTensor CudaAddBiasRows(const CudaTensor& value, const CudaWeight* bias);

// The same add in place on rows x bias-size floats of device memory.
void CudaAddBiasRowsInPlace(float* value, int64_t rows, const CudaWeight& bias);

// Device addresses of rows [position, position + rows) of `layer` in the
// cache's K and V buffers (rows x kv_heads x head_dim floats each, owned by
// the cache), for kernels that write K / V where they are stored.
// std::out_of_range when the rows or the layer leave the cache.
struct CudaKvRows {
  float* keys;
  float* values;
};
CudaKvRows CudaKvCacheRows(CudaKvCache* cache, int layer, int position, int rows);

// Writes the K/V of rows consecutive tokens (keys, values [rows, kv_heads *
// head_dim]) to positions [position, position + rows) of `layer`
// (CudaKvCache::Write for a batch of tokens).  std::out_of_range when the
// positions or the layer leave the cache.
void CudaKvCacheWriteRows(CudaKvCache* cache, int layer, int position,
                          const CudaTensor& keys, const CudaTensor& values);

// Causal attention of q [rows, n_heads * head_dim] whose row r is the token
// at position + r, over `layer` of the cache (its K/V must be written for
// every position up to position + rows - 1) -> [rows, n_heads * head_dim];
// row r equals CudaAttention at position + r.
CudaTensor CudaAttentionRows(const CudaTensor& q, const CudaKvCache& cache,
                             int layer, int position, int n_heads,
                             int n_kv_heads, int head_dim);

// Makes `device` current for the scope and restores the previous device.
class CudaDeviceScope {
 public:
  explicit CudaDeviceScope(int device);
  ~CudaDeviceScope();
  CudaDeviceScope(const CudaDeviceScope&) = delete;
  CudaDeviceScope& operator=(const CudaDeviceScope&) = delete;

 private:
  int previous_ = 0;
};

// Bytes held by the caching pool of `device` (free blocks kept for reuse),
// and a call that returns them to the driver.
size_t CudaPoolCachedBytes(int device);
void CudaPoolRelease(int device);

// Number of (cos, sin) positions of the RoPE table cached on the current
// device for (theta, head_dim); 0 when none has been built.
int CudaRopeTableRows(float theta, int head_dim);

// Contiguous shard [begin, end) of `total` rows for shard `index` of
// `shards`; the first total % shards shards hold one extra row.
std::pair<int, int> ShardRange(int total, int shards, int index);

// Prefill sharding across GPUs: runs body(device, begin, end) on one host
// thread per entry of `devices`, each with its device current and its own
// contiguous token range of [0, total_rows).  Weights are replicated by the
// caller; no data moves between devices.  Every thread is joined before the
// call returns, and the first exception any body threw is rethrown here.
void CudaShardRows(int total_rows, const std::vector<int>& devices,
                   const std::function<void(int device, int begin, int end)>& body);

// Waits for a recorded cudaEvent_t (passed as void*) by polling it until
// `timeout_ms` has passed: true when the work before it finished, false on
// timeout (nothing is cancelled; the caller decides what to do).  Throws
// std::runtime_error if the event reports a CUDA error.
bool CudaWaitEvent(void* event, double timeout_ms);

}  // namespace mini_lla

#endif  // MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_LAYER_OPS_H_
