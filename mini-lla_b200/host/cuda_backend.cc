// Device lists for mini-lla's CUDA backend (include/mini_llama/cuda_backend.h).
//
// Validation keeps the reference's rules and exception types
// (src/backend.cc:26-42) and applies them to each listed device; the weights
// are replicated with the reference's UploadModelWeights semantics
// (src/cuda_weights.cc:81-111) or straight from a GGUF file; requests are
// spread over the devices with CudaShardRows, one host thread per device.
#include "mini_llama/cuda_backend.h"

#include <cuda_runtime.h>

#include <cctype>
#include <set>
#include <stdexcept>
#include <string>
#include <utility>

#include "mini_llama/cuda_batch.h"
#include "mini_llama/cuda_gguf_upload.h"
#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/cuda_runtime.h"

namespace mini_lla {
namespace {

std::string Joined(const std::vector<int>& devices) {
  std::string text;
  for (size_t i = 0; i < devices.size(); ++i) {
    if (i > 0) text += ",";
    text += std::to_string(devices[i]);
  }
  return text;
}

}  // namespace

std::vector<int> ParseCudaDevices(const std::string& text, int visible) {
  if (text == "all") {
    if (visible <= 0) throw std::invalid_argument("--devices all: no visible CUDA device");
    std::vector<int> all(static_cast<size_t>(visible));
    for (int i = 0; i < visible; ++i) all[static_cast<size_t>(i)] = i;
    return all;
  }
  std::vector<int> devices;
  size_t begin = 0;
  while (true) {
    const size_t comma = text.find(',', begin);
    const std::string item =
        text.substr(begin, comma == std::string::npos ? std::string::npos : comma - begin);
    if (item.empty() || item.size() > 9) {
      throw std::invalid_argument("--devices: bad device list \"" + text + "\"");
    }
    int value = 0;
    for (const char c : item) {
      if (!std::isdigit(static_cast<unsigned char>(c))) {
        throw std::invalid_argument("--devices: bad device id \"" + item + "\"");
      }
      value = value * 10 + (c - '0');
    }
    devices.push_back(value);
    if (comma == std::string::npos) break;
    begin = comma + 1;
  }
  return devices;
}

std::vector<int> ParseCudaDevices(const std::string& text) {
  return ParseCudaDevices(text, text == "all" ? CudaDeviceCount() : 0);
}

void ValidateBackendDevices(const BackendConfig& config, const std::vector<int>& devices,
                            int visible) {
  if (config.kind == BackendKind::kCpu) {
    if (!devices.empty() || config.device_set) {
      throw std::invalid_argument("--devices / --device need --backend cuda");
    }
    return;
  }
  if (devices.empty()) throw std::invalid_argument("--devices: empty device list");
  std::set<int> seen;
  for (const int device : devices) {
    if (device < 0 || device >= visible) {
      throw std::out_of_range("CUDA device " + std::to_string(device) +
                              " out of range, visible devices: " + std::to_string(visible));
    }
    if (!seen.insert(device).second) {
      throw std::invalid_argument("--devices: device " + std::to_string(device) +
                                  " listed twice");
    }
  }
}

void ValidateBackendDevices(const BackendConfig& config, const std::vector<int>& devices) {
  if (config.kind == BackendKind::kCpu) {
    ValidateBackendDevices(config, devices, 0);
    return;
  }
  if (!CudaRuntimeBuilt()) {
    throw std::runtime_error("CUDA not enabled: rebuild with -DMINI_LLA_CUDA=ON");
  }
  ValidateBackendDevices(config, devices, CudaDeviceCount());
}

std::vector<int> SelectedDevices(const BackendConfig& config,
                                 const std::vector<int>& devices) {
  if (!devices.empty()) return devices;
  return {config.device};
}

std::string BackendDevicesNote(const BackendConfig& config,
                               const std::vector<int>& devices) {
  if (config.kind == BackendKind::kCpu) return "compute: cpu";
  const std::vector<int> used = SelectedDevices(config, devices);
  if (used.size() == 1) return "compute: cuda device " + std::to_string(used[0]);
  return "compute: cuda devices " + Joined(used) + " (weights replicated)";
}

Model CudaModelReplicas::ForDevice(size_t i) const {
  if (i >= weights.size()) throw std::out_of_range("CudaModelReplicas: no such replica");
  Model model;
  model.config = config;
  model.tied_lm_head = tied_lm_head;
  model.cuda_weights = weights[i];
  return model;
}

CudaModelReplicas UploadModelWeightsToDevices(Model* model, const std::vector<int>& devices) {
  if (model == nullptr) throw std::invalid_argument("UploadModelWeightsToDevices: null model");
  BackendConfig cuda;
  cuda.kind = BackendKind::kCuda;
  ValidateBackendDevices(cuda, devices);
  CudaModelReplicas replicas;
  replicas.config = model->config;
  replicas.tied_lm_head = model->tied_lm_head;
  replicas.devices = devices;
  // upload in reverse so that model->cuda_weights ends on devices[0]'s copy
  replicas.weights.resize(devices.size());
  for (size_t i = devices.size(); i-- > 0;) {
    UploadModelWeights(model, devices[i]);
    replicas.weights[i] = model->cuda_weights;
  }
  return replicas;
}

CudaModelReplicas LoadGgufModelReplicas(const std::string& path,
                                        const std::vector<int>& devices) {
  BackendConfig cuda;
  cuda.kind = BackendKind::kCuda;
  ValidateBackendDevices(cuda, devices);
  CudaGgufModel loaded = LoadGgufModelToDevices(path, devices);
  CudaModelReplicas replicas;
  replicas.config = loaded.model.config;
  replicas.tied_lm_head = loaded.model.tied_lm_head;
  replicas.devices = devices;
  replicas.weights = std::move(loaded.replicas);
  return replicas;
}

int CudaPointerDevice(const void* pointer) {
  if (pointer == nullptr) return -1;
  cudaPointerAttributes attributes{};
  if (cudaPointerGetAttributes(&attributes, pointer) != cudaSuccess) {
    cudaGetLastError();  // an unknown pointer leaves an error behind; clear it
    return -1;
  }
  return attributes.type == cudaMemoryTypeDevice ? attributes.device : -1;
}

std::vector<Tensor> ForwardBatchesCuda(const std::vector<Context*>& contexts,
                                       const CudaModelReplicas& model,
                                       const std::vector<MiniBatch>& batches,
                                       int max_rows) {
  if (contexts.size() != batches.size()) {
    throw std::invalid_argument("ForwardBatchesCuda: contexts and batches differ in size");
  }
  if (model.weights.empty() || model.weights.size() != model.devices.size()) {
    throw std::invalid_argument("ForwardBatchesCuda: no device replicas");
  }
  const int requests = static_cast<int>(contexts.size());
  std::vector<Tensor> logits(contexts.size());
  if (requests == 0) return logits;
  const int shards = static_cast<int>(model.devices.size());
  std::set<const Context*> distinct(contexts.begin(), contexts.end());
  if (distinct.size() != contexts.size()) {
    throw std::invalid_argument("ForwardBatchesCuda: a context is listed twice");
  }
  for (int s = 0; s < shards; ++s) {
    const std::pair<int, int> range = ShardRange(requests, shards, s);
    for (int i = range.first; i < range.second; ++i) {
      const Context* context = contexts[static_cast<size_t>(i)];
      if (context == nullptr) throw std::invalid_argument("ForwardBatchesCuda: null context");
      if (context->cuda_cache.empty()) continue;
      const int holder = CudaPointerDevice(context->cuda_cache.Keys(0));
      if (holder != model.devices[static_cast<size_t>(s)]) {
        throw std::invalid_argument(
            "ForwardBatchesCuda: request " + std::to_string(i) + " has its KV cache on device " +
            std::to_string(holder) + " but is assigned to device " +
            std::to_string(model.devices[static_cast<size_t>(s)]));
      }
    }
  }
  // CudaShardRows hands shard s the range ShardRange(requests, shards, s) and
  // runs it with devices[s] current; shards of equal device ids are told
  // apart by their range.
  CudaShardRows(requests, model.devices, [&](int, int begin, int end) {
    if (begin == end) return;
    int shard = 0;  // non-empty shards start at distinct rows
    while (ShardRange(requests, shards, shard).first != begin) ++shard;
    const Model replica = model.ForDevice(static_cast<size_t>(shard));
    for (int i = begin; i < end; ++i) {
      logits[static_cast<size_t>(i)] = ForwardBatchCuda(
          *contexts[static_cast<size_t>(i)], replica, batches[static_cast<size_t>(i)], max_rows);
    }
  });
  return logits;
}

}  // namespace mini_lla
