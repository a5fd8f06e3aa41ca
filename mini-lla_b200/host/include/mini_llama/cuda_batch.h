// Row-batched prefill on the GPU: the driver that replaces ForwardBatch's
// per-token loop (the reference's src/batch.cc:26-41 over ForwardToken /
// ForwardTokenCuda, src/cuda_forward.cc:37-93) for a model whose weights are
// on the device.
#ifndef MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BATCH_H_
#define MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BATCH_H_

#include "mini_llama/batch.h"
#include "mini_llama/kv_cache.h"
#include "mini_llama/model.h"
#include "mini_llama/tensor.h"

namespace mini_lla {

// Runs every token of `batch` through `model` (weights uploaded with
// UploadModelWeights) and returns the logits of the last one, like
// ForwardBatch: each token's K/V go to the cache at its position and
// context.position ends one past the last token's position.  Tokens whose
// positions are consecutive are processed together, up to `max_rows` rows
// per pass through the layers: embedding, RMSNorm, the q/k/v/o and FFN
// linears, bias + RoPE, the K/V write and causal attention each run once
// per pass over all of its rows, and residual adds are fused into the
// following RMSNorm.  A run of positions that is not consecutive starts a
// new pass, so the cache state every token sees is the one the per-token
// loop would give it.
//
// Differences from the per-token loop: the whole batch is validated before
// anything runs (an empty batch, mismatched sizes, a token id or a position
// out of range throw std::invalid_argument / std::out_of_range with the
// cache unchanged), and sums run in other orders (the result matches within
// floating-point tolerance, not bit for bit).
Tensor ForwardBatchCuda(Context& context, const Model& model,
                        const MiniBatch& batch, int max_rows = 512);

}  // namespace mini_lla

#endif  // MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BATCH_H_
