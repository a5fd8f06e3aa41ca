// mini-lla's device linear layer (the reference's
// include/mini_llama/cuda_matmul.h) over libmlb.so's mlb_linear_f32.  This
// file takes the place of the reference's src/cuda_matmul.cu: the F32 path no
// longer needs cuBLAS, and the Q8_0 / Q4_0 / Q4_1 paths stage each weight
// row with 16-byte loads and reduce it across a warp instead of running one
// thread per output row.
#include "mini_llama/cuda_matmul.h"

#include <stdexcept>
#include <string>

#include "mlb_ops.h"

namespace mini_lla {

CudaTensor CudaLinear(const CudaTensor& x, const CudaWeight& weight) {
  if (x.Size() != static_cast<size_t>(weight.cols)) {
    throw std::invalid_argument("CudaLinear: input size mismatch");
  }
  CudaTensor output({weight.rows});
  int qtype = MLB_F32;
  switch (weight.type) {
    case QuantType::kF32: qtype = MLB_F32; break;
    case QuantType::kQ8_0: qtype = MLB_Q8_0; break;
    case QuantType::kQ4_0: qtype = MLB_Q4_0; break;
    case QuantType::kQ4_1: qtype = MLB_Q4_1; break;
  }
  const int rc = mlb_linear_f32(weight.buffer.data(), qtype, weight.rows,
                                weight.cols, x.data(), 1, output.data(), nullptr);
  if (rc != MLB_OK) {
    const std::string message = std::string("CudaLinear: ") + mlb_last_error();
    if (rc == MLB_ERR_ARG) throw std::invalid_argument(message);
    throw std::runtime_error(message);
  }
  return output;
}

}  // namespace mini_lla
