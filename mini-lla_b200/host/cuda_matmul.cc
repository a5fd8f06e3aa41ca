// mini-lla's device linear layer (the reference's
// include/mini_llama/cuda_matmul.h) over libmlb.so's mlb_linear_f32, and its
// row-batched form CudaLinearRows over mlb_linear_rows_f32.  This file takes
// the place of the reference's src/cuda_matmul.cu: the F32 path no longer
// needs cuBLAS, the Q8_0 / Q4_0 / Q4_1 decode paths stream each weight row
// through shared memory and reduce it across a warp instead of running one
// thread per output row, and prompt-sized batches run on the tensor cores.
#include "mini_llama/cuda_matmul.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "mini_llama/cuda_layer_ops.h"
#include "mlb_ops.h"

namespace mini_lla {

namespace {

int QType(QuantType type) {
  switch (type) {
    case QuantType::kF32: return MLB_F32;
    case QuantType::kQ8_0: return MLB_Q8_0;
    case QuantType::kQ4_0: return MLB_Q4_0;
    case QuantType::kQ4_1: return MLB_Q4_1;
  }
  throw std::invalid_argument("unknown quant type");
}

void Linear(const CudaTensor& x, const CudaWeight& weight, int64_t rows,
            CudaTensor* output, const char* caller) {
  const int rc = mlb_linear_f32(weight.buffer.data(), QType(weight.type), weight.rows,
                                weight.cols, x.data(), rows, output->data(), nullptr);
  if (rc != MLB_OK) {
    const std::string message = std::string(caller) + ": " + mlb_last_error();
    if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
    throw std::runtime_error(message);
  }
}

}  // namespace

CudaTensor CudaLinear(const CudaTensor& x, const CudaWeight& weight) {
  if (x.Size() != static_cast<size_t>(weight.cols)) {
    throw std::invalid_argument("CudaLinear: input size mismatch");
  }
  CudaTensor output({weight.rows});
  Linear(x, weight, 1, &output, "CudaLinear");
  return output;
}

CudaTensor CudaLinearRows(const CudaTensor& x, const CudaWeight& weight) {
  if (weight.cols <= 0 || x.shape().empty() || x.shape().back() != weight.cols) {
    throw std::invalid_argument("CudaLinearRows: input size mismatch");
  }
  const int rows = static_cast<int>(x.Size() / static_cast<size_t>(weight.cols));
  CudaTensor output({rows, weight.rows});
  if (rows == 0) return output;
  // prompt-sized batches run on the tensor cores; their scratch (x split
  // into TF32 head and tail) comes from the pool, ordered on the default
  // stream like every other operator's buffers
  const int64_t need = mlb_linear_rows_scratch_floats(weight.cols, rows);
  DeviceBuffer scratch;
  scratch.Reset(static_cast<size_t>(need) * sizeof(float));
  const int rc = mlb_linear_rows_f32(weight.buffer.data(), QType(weight.type), weight.rows,
                                     weight.cols, x.data(), rows, output.data(),
                                     static_cast<float*>(scratch.data()), need, nullptr);
  if (rc != MLB_OK) {
    const std::string message = std::string("CudaLinearRows: ") + mlb_last_error();
    if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
    throw std::runtime_error(message);
  }
  return output;
}

namespace {

// The checks and the launch of CudaLinearRowsGroup, writing weight m's
// output to y[m] (rows x weights[m]->rows floats).
void LinearRowsGroupTo(const CudaTensor& x, const std::vector<const CudaWeight*>& weights,
                       const std::vector<float*>& y) {
  if (weights.empty() || weights.size() > 3 || y.size() != weights.size()) {
    throw std::invalid_argument("CudaLinearRowsGroup: 1 to 3 weights");
  }
  const CudaWeight& first = *weights.front();
  for (const CudaWeight* w : weights) {
    if (w == nullptr || w->type != first.type || w->cols != first.cols) {
      throw std::invalid_argument("CudaLinearRowsGroup: weights differ in format or width");
    }
  }
  if (first.cols <= 0 || x.shape().empty() || x.shape().back() != first.cols) {
    throw std::invalid_argument("CudaLinearRowsGroup: input size mismatch");
  }
  const int rows = static_cast<int>(x.Size() / static_cast<size_t>(first.cols));
  if (rows == 0) return;
  const void* w[3];
  int64_t n[3];
  float* yy[3];
  for (size_t m = 0; m < weights.size(); ++m) {
    if (y[m] == nullptr) throw std::invalid_argument("CudaLinearRowsGroup: null output");
    w[m] = weights[m]->buffer.data();
    n[m] = weights[m]->rows;
    yy[m] = y[m];
  }
  const int64_t need = mlb_linear_rows_scratch_floats(first.cols, rows);
  DeviceBuffer scratch;
  scratch.Reset(static_cast<size_t>(need) * sizeof(float));
  const int rc = mlb_linear_rows_group_f32(
      static_cast<int>(weights.size()), w, QType(first.type), n, first.cols, x.data(), rows, yy,
      static_cast<float*>(scratch.data()), need, nullptr);
  if (rc != MLB_OK) {
    const std::string message = std::string("CudaLinearRowsGroup: ") + mlb_last_error();
    if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
    throw std::runtime_error(message);
  }
}

}  // namespace

std::vector<CudaTensor> CudaLinearRowsGroup(const CudaTensor& x,
                                            const std::vector<const CudaWeight*>& weights) {
  if (weights.empty() || weights.size() > 3) {
    throw std::invalid_argument("CudaLinearRowsGroup: 1 to 3 weights");
  }
  for (const CudaWeight* w : weights) {
    if (w == nullptr || w->cols <= 0) {
      throw std::invalid_argument("CudaLinearRowsGroup: weights differ in format or width");
    }
  }
  const int rows = static_cast<int>(x.Size() / static_cast<size_t>(weights.front()->cols));
  std::vector<CudaTensor> outputs;
  std::vector<float*> y;
  outputs.reserve(weights.size());
  for (const CudaWeight* w : weights) {
    outputs.emplace_back(std::vector<int>{rows, w->rows});
    y.push_back(outputs.back().data());
  }
  LinearRowsGroupTo(x, weights, y);
  return outputs;
}

void CudaLinearRowsGroupInto(const CudaTensor& x, const std::vector<const CudaWeight*>& weights,
                             const std::vector<float*>& outputs) {
  LinearRowsGroupTo(x, weights, outputs);
}

}  // namespace mini_lla
