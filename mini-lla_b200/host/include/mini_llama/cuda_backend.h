// Several GPUs behind mini-lla's CUDA backend.
//
// The reference selects one GPU: BackendConfig{kind, device, device_set}
// (include/mini_llama/backend.h:12-16), ValidateBackend checks that device
// (src/backend.cc:26-42), and PrepareModel uploads every weight to it
// (src/main.cc:175-182 -> UploadModelWeights, src/cuda_weights.cc:81-111).
// Every layer operator is independent per token row and every request owns
// its KV cache, so work spreads over several GPUs that each hold a replica of
// the weights, with no data moving between them.  This header adds a device
// list to that flow; with a single device everything behaves as the
// reference's backend does.
#ifndef MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BACKEND_H_
#define MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BACKEND_H_

#include <memory>
#include <string>
#include <vector>

#include "mini_llama/backend.h"
#include "mini_llama/batch.h"
#include "mini_llama/cuda_weights.h"
#include "mini_llama/kv_cache.h"
#include "mini_llama/model.h"
#include "mini_llama/tensor.h"

namespace mini_lla {

// Parses a device list as a command line gives it: "all" (every visible
// device, 0 .. n-1) or comma-separated ids ("0,2,3"), in shard order.
// std::invalid_argument for empty text, an entry that is not a non-negative
// integer, or (for "all") no visible device.  The overload taking
// `visible` resolves "all" against that count instead of asking the driver.
std::vector<int> ParseCudaDevices(const std::string& text);
std::vector<int> ParseCudaDevices(const std::string& text, int visible);

// ValidateBackend (backend.cc:26-42) for a device list, with the same
// exception types: a CPU backend given devices -> std::invalid_argument (as
// --device without --backend cuda), a build without CUDA ->
// std::runtime_error, a device outside [0, visible) -> std::out_of_range.
// Also std::invalid_argument for an empty list (CUDA backend) or an id
// listed twice.  The overload taking `visible` checks against that device
// count instead of asking the driver.
void ValidateBackendDevices(const BackendConfig& config, const std::vector<int>& devices);
void ValidateBackendDevices(const BackendConfig& config, const std::vector<int>& devices,
                            int visible);

// The devices a run uses: `devices` when not empty, else the config's one
// device (the reference's behaviour).
std::vector<int> SelectedDevices(const BackendConfig& config,
                                 const std::vector<int>& devices);

// BackendNote (backend.cc:44-47) for a device list, e.g.
// "compute: cuda devices 0,1 (weights replicated)".
std::string BackendDevicesNote(const BackendConfig& config,
                               const std::vector<int>& devices);

// One model's weights on several devices.
struct CudaModelReplicas {
  ModelConfig config;
  bool tied_lm_head = false;
  std::vector<int> devices;
  // weights[i] lives on devices[i]
  std::vector<std::shared_ptr<CudaModelWeights>> weights;

  size_t size() const { return devices.size(); }
  // A model for the GPU path on replica i: config and output tying of the
  // source model, cuda_weights = weights[i], host tensors empty.
  Model ForDevice(size_t i) const;
};

// PrepareModel for a device list: the devices are validated as
// ValidateBackendDevices does for a CUDA backend, then the model's weights go
// to every device with UploadModelWeights, in list order.  model->cuda_weights
// is left on the first device's replica, so a caller of the single-device
// API sees what UploadModelWeights(model, devices[0]) gives.
CudaModelReplicas UploadModelWeightsToDevices(Model* model, const std::vector<int>& devices);

// The same for a GGUF file, read once and uploaded to every device without a
// host copy of the weights (LoadGgufModelToDevices).
CudaModelReplicas LoadGgufModelReplicas(const std::string& path,
                                        const std::vector<int>& devices);

// Runs independent requests — contexts[i] with batches[i] — through
// ForwardBatchCuda over the replicas: the requests are split into
// contiguous ranges (ShardRange over their count), one per device, and each
// device runs its requests in order on its own host thread (CudaShardRows).
// Returns every request's logits, in request order; each equals what
// ForwardBatchCuda gives for that request on a single device.
//
// Checked before anything runs: sizes that do not match, a null context, or
// a context whose device KV cache already lives on another device than the
// one its request is assigned to -> std::invalid_argument (a context keeps
// its device for its life; reuse the same request order).  A request that
// fails inside ForwardBatchCuda throws its exception here after every
// device's thread has finished.
//
// One sequence's prompt rows are not split across devices: causal attention
// at row r needs the K/V of every earlier row, which live in that context's
// cache on one device.  Rows of the stand-alone layer operators (embedding,
// RMSNorm, RoPE, SwiGLU) split freely with CudaShardRows.
std::vector<Tensor> ForwardBatchesCuda(const std::vector<Context*>& contexts,
                                       const CudaModelReplicas& model,
                                       const std::vector<MiniBatch>& batches,
                                       int max_rows = 512);

// Device that holds the memory at `pointer` (cudaPointerGetAttributes), or
// -1 for host or unknown memory.
int CudaPointerDevice(const void* pointer);

}  // namespace mini_lla

#endif  // MINI_LLA_INCLUDE_MINI_LLAMA_CUDA_BACKEND_H_
