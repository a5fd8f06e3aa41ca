// Row-batched prefill driver (include/mini_llama/cuda_batch.h).
//
// The reference runs a prompt one token at a time (src/batch.cc:26-41):
// every token goes through ForwardToken -> ForwardTokenCuda
// (src/cuda_forward.cc:37-93), i.e. ~14 kernel launches per layer, each over
// one row, and every linear layer reads its whole weight matrix once per
// token.  Here a pass takes up to max_rows tokens of consecutive positions
// through the same steps as [rows, .] tensors: the linears read each weight
// on the tensor cores from 48 rows on (mlb_linear_rows_f32; q / k / v and
// gate / up as one grouped launch each, that q / k / v launch writing K and
// V straight into their KV-cache rows), RMSNorm / SwiGLU / bias + RoPE /
// causal attention run once per layer over all rows, and
// each residual add is fused into the RMSNorm that follows it.  Only the
// last row of the batch goes through the final norm and the output
// projection, since ForwardBatch returns the last token's logits.
#include "mini_llama/cuda_batch.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "mini_llama/cuda_attention.h"
#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/cuda_matmul.h"
#include "mini_llama/cuda_weights.h"
#include "mlb_ops.h"

namespace mini_lla {
namespace {

struct LayerRefs {
  const CudaWeight* attention_norm = nullptr;
  const CudaWeight* wq = nullptr;
  const CudaWeight* wk = nullptr;
  const CudaWeight* wv = nullptr;
  const CudaWeight* wo = nullptr;
  const CudaWeight* bq = nullptr;  // optional biases
  const CudaWeight* bk = nullptr;
  const CudaWeight* bv = nullptr;
  const CudaWeight* ffn_norm = nullptr;
  const CudaWeight* w_gate = nullptr;
  const CudaWeight* w_up = nullptr;
  const CudaWeight* w_down = nullptr;
};

struct ModelRefs {
  const CudaWeight* embedding = nullptr;
  const CudaWeight* final_norm = nullptr;
  const CudaWeight* output = nullptr;
  std::vector<LayerRefs> layers;
};

const CudaWeight* Require(const CudaModelWeights& weights, const std::string& name) {
  const CudaWeight* weight = weights.Find(name);
  if (weight == nullptr) {
    throw std::runtime_error("ForwardBatchCuda: weight missing on the GPU: " + name);
  }
  return weight;
}

// Looks every weight up once per call (CudaModelWeights::Find is a linear
// search by name), with the names UploadModelWeights gives them
// (cuda_weights.cc:81-111).
ModelRefs Resolve(const Model& model) {
  const CudaModelWeights& weights = *model.cuda_weights;
  ModelRefs refs;
  refs.embedding = Require(weights, "token_embedding");
  refs.final_norm = Require(weights, "final_norm");
  refs.output = model.tied_lm_head ? refs.embedding : Require(weights, "lm_head");
  refs.layers.resize(static_cast<size_t>(model.config.n_layers));
  for (int layer = 0; layer < model.config.n_layers; ++layer) {
    const std::string prefix = "layers." + std::to_string(layer) + ".";
    LayerRefs& l = refs.layers[static_cast<size_t>(layer)];
    l.attention_norm = Require(weights, prefix + "attention_norm");
    l.wq = Require(weights, prefix + "wq");
    l.wk = Require(weights, prefix + "wk");
    l.wv = Require(weights, prefix + "wv");
    l.wo = Require(weights, prefix + "wo");
    l.bq = weights.Find(prefix + "bq");
    l.bk = weights.Find(prefix + "bk");
    l.bv = weights.Find(prefix + "bv");
    l.ffn_norm = Require(weights, prefix + "ffn_norm");
    l.w_gate = Require(weights, prefix + "w_gate");
    l.w_up = Require(weights, prefix + "w_up");
    l.w_down = Require(weights, prefix + "w_down");
  }
  return refs;
}

// Weights that can share one grouped linear launch (same format and width).
bool SameShape(const CudaWeight& a, const CudaWeight& b) {
  return a.type == b.type && a.cols == b.cols;
}

void Check(int rc, const char* caller) {
  if (rc == MLB_OK) return;
  const std::string message = std::string(caller) + ": " + mlb_last_error();
  if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
  if (rc == MLB_ERR_RANGE) throw std::out_of_range(message);
  throw std::runtime_error(message);
}

}  // namespace

Tensor ForwardBatchCuda(Context& context, const Model& model, const MiniBatch& batch,
                        int max_rows) {
  if (model.cuda_weights == nullptr) {
    throw std::runtime_error("ForwardBatchCuda: model weights are not on the GPU");
  }
  // the reference's checks (batch.cc:30-35, forward.cc:16-26), all up front
  if (batch.Size() == 0) throw std::invalid_argument("ForwardBatch: empty batch");
  if (batch.tokens.size() != batch.positions.size()) {
    throw std::invalid_argument("ForwardBatch: token/position size mismatch");
  }
  if (max_rows < 1) throw std::invalid_argument("ForwardBatchCuda: max_rows must be positive");
  const ModelConfig& config = model.config;
  for (size_t i = 0; i < batch.tokens.size(); ++i) {
    if (batch.tokens[i] < 0 || batch.tokens[i] >= config.vocab_size) {
      throw std::out_of_range("forward: token id out of range");
    }
    if (batch.positions[i] < 0 || batch.positions[i] >= config.max_seq_len) {
      throw std::out_of_range("forward: position exceeds context length");
    }
  }

  CudaDeviceScope scope(model.cuda_weights->device());
  const ModelRefs refs = Resolve(model);
  const int dim = config.dim;
  const int head_dim = config.head_dim();
  const float eps = config.rms_norm_eps;
  if (context.cuda_cache.empty()) {
    context.cuda_cache.Reset(config.n_layers, config.max_seq_len, config.n_kv_heads,
                             head_dim);
  }

  Tensor logits;
  const size_t count = batch.tokens.size();
  size_t begin = 0;
  while (begin < count) {
    // one pass: consecutive positions, at most max_rows of them
    size_t end = begin + 1;
    while (end < count && end - begin < static_cast<size_t>(max_rows) &&
           batch.positions[end] == batch.positions[end - 1] + 1) {
      ++end;
    }
    const int rows = static_cast<int>(end - begin);
    const int position = batch.positions[begin];
    const std::vector<int> tokens(batch.tokens.begin() + begin, batch.tokens.begin() + end);
    const std::vector<int> positions(batch.positions.begin() + begin,
                                     batch.positions.begin() + end);

    CudaTensor x = CudaEmbeddingRows(*refs.embedding, tokens);  // [rows, dim]
    CudaTensor ffn;  // the previous layer's FFN output, added to x by the next norm
    for (int layer = 0; layer < config.n_layers; ++layer) {
      const LayerRefs& l = refs.layers[static_cast<size_t>(layer)];
      CudaTensor norm;
      if (layer == 0) {
        norm = CudaAddRmsNormRows(x, nullptr, *l.attention_norm, eps);
      } else {
        CudaTensor h;  // x + ffn: the residual stream entering this layer
        norm = CudaAddRmsNormRows(ffn, &x, *l.attention_norm, eps, &h);
        x = std::move(h);
      }
      CudaTensor q;
      if (SameShape(*l.wq, *l.wk) && SameShape(*l.wq, *l.wv)) {
        // one launch, K and V written straight into their cache rows (the
        // cache holds consecutive positions contiguously), where the bias
        // and RoPE are then applied: no separate K / V write
        const CudaKvRows kv = CudaKvCacheRows(&context.cuda_cache, layer, position, rows);
        q = CudaTensor(std::vector<int>{rows, l.wq->rows});
        CudaLinearRowsGroupInto(norm, {l.wq, l.wk, l.wv}, {q.data(), kv.keys, kv.values});
        if (l.bv != nullptr) CudaAddBiasRowsInPlace(kv.values, rows, *l.bv);
        CudaRopeRowsInPlace(q.data(), kv.keys, l.bq, l.bk, positions, config.rope_theta,
                            config.n_heads, config.n_kv_heads, head_dim, config.rope_type);
      } else {
        q = CudaLinearRows(norm, *l.wq);
        CudaTensor k = CudaLinearRows(norm, *l.wk);
        CudaTensor v = CudaLinearRows(norm, *l.wv);
        if (l.bv != nullptr) v = CudaAddBiasRows(v, l.bv);
        CudaRopeRows(&q, &k, l.bq, l.bk, positions, config.rope_theta, config.n_heads,
                     config.n_kv_heads, head_dim, config.rope_type);
        CudaKvCacheWriteRows(&context.cuda_cache, layer, position, k, v);
      }
      const CudaTensor attention =
          CudaAttentionRows(q, context.cuda_cache, layer, position, config.n_heads,
                            config.n_kv_heads, head_dim);
      const CudaTensor projected = CudaLinearRows(attention, *l.wo);
      CudaTensor x_attn;  // x + attention output
      const CudaTensor ffn_norm =
          CudaAddRmsNormRows(projected, &x, *l.ffn_norm, eps, &x_attn);
      CudaTensor act;
      if (SameShape(*l.w_gate, *l.w_up)) {
        const std::vector<CudaTensor> gate_up = CudaLinearRowsGroup(ffn_norm, {l.w_gate, l.w_up});
        act = CudaSwiGlu(gate_up[0], gate_up[1]);
      } else {
        act = CudaSwiGlu(CudaLinearRows(ffn_norm, *l.w_gate), CudaLinearRows(ffn_norm, *l.w_up));
      }
      ffn = CudaLinearRows(act, *l.w_down);
      x = std::move(x_attn);
    }

    if (end == count) {
      // logits of the batch's last token: final norm of its x + ffn, then
      // the output projection (cuda_forward.cc:86-90)
      const int64_t last = static_cast<int64_t>(rows - 1) * dim;
      CudaTensor final_norm({dim});
      Check(mlb_rmsnorm_f32(ffn.data() + last, x.data() + last, nullptr,
                            final_norm.data(),
                            static_cast<const float*>(refs.final_norm->buffer.data()), 1,
                            dim, eps, nullptr),
            "ForwardBatchCuda");
      logits = CudaLinear(final_norm, *refs.output).Download();
    }
    begin = end;
  }
  context.position = batch.positions.back() + 1;
  return logits;
}

}  // namespace mini_lla
