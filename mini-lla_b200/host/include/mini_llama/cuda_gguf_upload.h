// GGUF file -> device weights without host tensors.
//
// The reference loads a GGUF model into host QuantizedTensors
// (src/gguf_loader.cc:41-73 LoadBlocks, src/gguf.cc:293-305
// ReadGgufTensorInto) and UploadModelWeights (src/cuda_weights.cc:81-111)
// then copies every tensor to one device with a pageable cudaMemcpy.  Here
// the tensor bytes go from the file into pinned staging buffers and from
// there to every requested device, so a model is read from disk once however
// many replicas it gets, and no host copy of the weights is built.
#ifndef MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_GGUF_UPLOAD_H_
#define MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_GGUF_UPLOAD_H_

#include <memory>
#include <string>
#include <vector>

#include "mini_llama/cuda_weights.h"
#include "mini_llama/model.h"

namespace mini_lla {

// A GGUF model resident on one or more GPUs.
struct CudaGgufModel {
  // config and tied_lm_head as LoadGgufModel sets them (max_seq_len capped at
  // kMaxContextLength); the host tensors stay empty; cuda_weights is the
  // first replica.
  Model model;
  // one weight set per requested device, in the order of `devices`; use
  // `Model m = result.model; m.cuda_weights = replicas[i];` for device i.
  std::vector<std::shared_ptr<CudaModelWeights>> replicas;
};

// Reads `path` and uploads its weights to every device in `devices` under
// the names UploadModelWeights uses ("token_embedding", "final_norm",
// "lm_head", "layers.N.wq", ...), with the same types, shapes and bytes as
// LoadGgufModel followed by UploadModelWeights.  Throws std::runtime_error
// for a file that does not parse, a missing required tensor, an unsupported
// tensor type or a shape that does not match the metadata (the messages of
// LoadGgufModel's checks), std::invalid_argument for an empty device list.
CudaGgufModel LoadGgufModelToDevices(const std::string& path,
                                     const std::vector<int>& devices);

}  // namespace mini_lla

#endif  // MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_GGUF_UPLOAD_H_
