// mini-lla's device weight store (the reference's
// include/mini_llama/cuda_weights.h, whose src/cuda_weights.cc this file
// replaces) and the direct GGUF -> device path of cuda_gguf_upload.h.
//
// UploadModelWeights keeps the reference's names, order and layout
// (cuda_weights.cc:81-111): raw ggml blocks for the linears and the
// embedding, F32 vectors for norms and biases, empty optional vectors
// skipped.  Its copies go through DeviceBuffer::Upload, which stages large
// tensors through pinned double-buffered chunks.
//
// LoadGgufModelToDevices reads the tensor table with the reference's
// GgufReader (src/gguf.cc) and then moves each tensor's bytes from the file
// into two pinned 8 MiB staging buffers (pread, no intermediate host copy)
// and from them to every device with cudaMemcpyAsync on one stream per
// device; a staging buffer is refilled once all devices' copies of it have
// finished.  The config, the tensor-name mapping and the shape checks
// restate src/gguf_loader.cc (BuildConfig :132-158, LoadGgufModel :230-271,
// ValidateShapes :180-222).  Norms or biases stored quantized are
// dequantised on the device (mlb_embedding_row), matching LoadF32
// (:97-115), which dequantises on the host.
#include "mini_llama/cuda_weights.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "mini_llama/cuda_gguf_upload.h"
#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/gguf.h"
#include "mini_llama/gguf_loader.h"
#include "mini_llama/quant.h"
#include "mlb_ops.h"

namespace mini_lla {

const CudaWeight* CudaModelWeights::Find(const std::string& name) const {
  for (const CudaWeight& weight : weights_) {
    if (weight.name == name) return &weight;
  }
  return nullptr;
}

void CudaModelWeights::Add(CudaWeight weight) { weights_.push_back(std::move(weight)); }

size_t CudaModelWeights::Bytes() const {
  size_t bytes = 0;
  for (const CudaWeight& weight : weights_) bytes += weight.buffer.size();
  return bytes;
}

namespace {

void ThrowCuda(const std::string& what, cudaError_t error) {
  throw std::runtime_error(what + ": " + cudaGetErrorString(error));
}

const void* QuantizedData(const QuantizedTensor& weight) {
  switch (weight.type) {
    case QuantType::kF32: return weight.f32.data.data();
    case QuantType::kQ8_0: return weight.q8_0.data();
    case QuantType::kQ4_0: return weight.q4_0.data();
    case QuantType::kQ4_1: return weight.q4_1.data();
  }
  return nullptr;
}

void UploadQuantized(const std::string& name, const QuantizedTensor& weight,
                     CudaModelWeights* storage) {
  const size_t bytes = QuantizedBytes(weight);
  if (bytes == 0) throw std::runtime_error("UploadModelWeights: empty weight: " + name);
  CudaWeight uploaded;
  uploaded.name = name;
  uploaded.type = weight.type;
  uploaded.rows = weight.rows;
  uploaded.cols = weight.cols;
  uploaded.linear = true;
  uploaded.buffer.Reset(bytes);
  uploaded.buffer.Upload(QuantizedData(weight), bytes);
  storage->Add(std::move(uploaded));
}

void UploadVector(const std::string& name, const Tensor& tensor,
                  CudaModelWeights* storage) {
  if (tensor.Size() == 0) return;
  CudaWeight uploaded;
  uploaded.name = name;
  uploaded.type = QuantType::kF32;
  uploaded.rows = static_cast<int>(tensor.Size());
  uploaded.cols = 1;
  uploaded.linear = false;
  uploaded.buffer.Reset(tensor.Size() * sizeof(float));
  uploaded.buffer.Upload(tensor.data.data(), tensor.Size() * sizeof(float));
  storage->Add(std::move(uploaded));
}

}  // namespace

void UploadModelWeights(Model* model, int device) {
  if (model == nullptr) throw std::invalid_argument("UploadModelWeights: null model");
  CudaDeviceScope scope(device);
  auto storage = std::make_shared<CudaModelWeights>();
  storage->set_device(device);
  UploadQuantized("token_embedding", model->token_embedding, storage.get());
  UploadVector("final_norm", model->final_norm, storage.get());
  if (!model->tied_lm_head) UploadQuantized("lm_head", model->lm_head, storage.get());
  for (size_t layer = 0; layer < model->layers.size(); ++layer) {
    const LayerWeights& w = model->layers[layer];
    const std::string prefix = "layers." + std::to_string(layer) + ".";
    UploadVector(prefix + "attention_norm", w.attention_norm, storage.get());
    UploadQuantized(prefix + "wq", w.wq, storage.get());
    UploadQuantized(prefix + "wk", w.wk, storage.get());
    UploadQuantized(prefix + "wv", w.wv, storage.get());
    UploadQuantized(prefix + "wo", w.wo, storage.get());
    UploadVector(prefix + "bq", w.bq, storage.get());
    UploadVector(prefix + "bk", w.bk, storage.get());
    UploadVector(prefix + "bv", w.bv, storage.get());
    UploadVector(prefix + "ffn_norm", w.ffn_norm, storage.get());
    UploadQuantized(prefix + "w_gate", w.w_gate, storage.get());
    UploadQuantized(prefix + "w_up", w.w_up, storage.get());
    UploadQuantized(prefix + "w_down", w.w_down, storage.get());
  }
  model->cuda_weights = std::move(storage);
}

void ClearModelWeights(Model* model) {
  if (model != nullptr) model->cuda_weights.reset();
}

size_t CudaWeightCount(const Model& model) {
  return model.cuda_weights ? model.cuda_weights->Count() : 0;
}

size_t CudaWeightBytes(const Model& model) {
  return model.cuda_weights ? model.cuda_weights->Bytes() : 0;
}

// ---------------------------------------------------------------------------
// GGUF file -> devices.

namespace {

constexpr size_t kStageBytes = size_t{8} << 20;

// File bytes -> pinned staging -> every device.
class FileToDevices {
 public:
  FileToDevices(const std::string& path, const std::vector<int>& devices)
      : devices_(devices) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("GGUF open failed: " + path);
    for (int i = 0; i < 2; ++i) {
      const cudaError_t error =
          cudaHostAlloc(&stage_[i], kStageBytes, cudaHostAllocPortable);
      if (error != cudaSuccess) {
        Release();
        ThrowCuda("cudaHostAlloc", error);
      }
    }
    streams_.assign(devices.size(), nullptr);
    done_.assign(devices.size() * 2, nullptr);
    for (size_t d = 0; d < devices.size(); ++d) {
      CudaDeviceScope scope(devices[d]);
      cudaError_t error = cudaStreamCreateWithFlags(&streams_[d], cudaStreamNonBlocking);
      for (int i = 0; i < 2 && error == cudaSuccess; ++i)
        error = cudaEventCreateWithFlags(&done_[d * 2 + i], cudaEventDisableTiming);
      if (error != cudaSuccess) {
        Release();
        ThrowCuda("GGUF upload streams", error);
      }
    }
  }
  ~FileToDevices() { Release(); }
  FileToDevices(const FileToDevices&) = delete;
  FileToDevices& operator=(const FileToDevices&) = delete;

  // Copies file bytes [offset, offset + bytes) to dst[d] on devices[d].
  void Copy(uint64_t offset, size_t bytes, const std::vector<void*>& dst) {
    for (size_t off = 0; off < bytes; off += kStageBytes) {
      const int slot = static_cast<int>(next_ & 1);
      const size_t n = std::min(kStageBytes, bytes - off);
      if (used_[slot]) {
        for (size_t d = 0; d < devices_.size(); ++d) {
          const cudaError_t error = cudaEventSynchronize(done_[d * 2 + slot]);
          if (error != cudaSuccess) ThrowCuda("GGUF upload", error);
        }
      }
      ReadAt(stage_[slot], n, offset + off);
      for (size_t d = 0; d < devices_.size(); ++d) {
        CudaDeviceScope scope(devices_[d]);
        cudaError_t error = cudaMemcpyAsync(static_cast<char*>(dst[d]) + off, stage_[slot],
                                            n, cudaMemcpyHostToDevice, streams_[d]);
        if (error == cudaSuccess) error = cudaEventRecord(done_[d * 2 + slot], streams_[d]);
        if (error != cudaSuccess) ThrowCuda("GGUF upload", error);
      }
      used_[slot] = true;
      ++next_;
    }
  }

  // Waits for every copy issued so far.
  void Finish() {
    for (size_t d = 0; d < devices_.size(); ++d) {
      const cudaError_t error = cudaStreamSynchronize(streams_[d]);
      if (error != cudaSuccess) ThrowCuda("GGUF upload", error);
    }
  }

 private:
  void ReadAt(void* dst, size_t bytes, uint64_t offset) {
    char* p = static_cast<char*>(dst);
    while (bytes > 0) {
      const ssize_t got = ::pread(fd_, p, bytes, static_cast<off_t>(offset));
      if (got < 0 && errno == EINTR) continue;
      if (got <= 0) throw std::runtime_error("GGUF read failed (file truncated?)");
      p += got;
      bytes -= static_cast<size_t>(got);
      offset += static_cast<uint64_t>(got);
    }
  }

  void Release() {
    for (size_t d = 0; d < streams_.size(); ++d) {
      if (streams_[d] != nullptr) cudaStreamSynchronize(streams_[d]);
    }
    for (cudaEvent_t event : done_)
      if (event != nullptr) cudaEventDestroy(event);
    for (cudaStream_t stream : streams_)
      if (stream != nullptr) cudaStreamDestroy(stream);
    done_.clear();
    streams_.clear();
    for (void*& stage : stage_) {
      if (stage != nullptr) cudaFreeHost(stage);
      stage = nullptr;
    }
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
  }

  std::vector<int> devices_;
  int fd_ = -1;
  void* stage_[2] = {nullptr, nullptr};
  bool used_[2] = {false, false};
  size_t next_ = 0;
  std::vector<cudaStream_t> streams_;
  std::vector<cudaEvent_t> done_;  // [device][slot]
};

// The model config from GGUF metadata (gguf_loader.cc:132-158).
ModelConfig GgufConfig(const GgufReader& reader) {
  ModelConfig config;
  const std::string arch = reader.String("general.architecture", "llama");
  auto number = [&](const std::string& key, double fallback) {
    return reader.Number(arch + "." + key, fallback);
  };
  config.n_layers = static_cast<int>(number("block_count", 0));
  config.dim = static_cast<int>(number("embedding_length", 0));
  config.hidden_dim = static_cast<int>(number("feed_forward_length", 0));
  config.n_heads = static_cast<int>(number("attention.head_count", 0));
  config.n_kv_heads = static_cast<int>(number("attention.head_count_kv", config.n_heads));
  config.max_seq_len = static_cast<int>(number("context_length", 0));
  config.rope_theta = static_cast<float>(number("rope.freq_base", 10000.0));
  config.rms_norm_eps = static_cast<float>(number("attention.layer_norm_rms_epsilon", 1e-5));
  if (arch == "qwen2") config.rope_type = RopeType::kNeoX;
  std::vector<std::string> tokens;
  if (reader.Strings("tokenizer.ggml.tokens", &tokens)) {
    config.vocab_size = static_cast<int>(tokens.size());
  }
  ValidateConfig(config);
  config.max_seq_len = std::min(config.max_seq_len, kMaxContextLength);
  return config;
}

// One tensor to upload: where it is in the file and what it becomes.
struct Planned {
  std::string name;        // device weight name
  const GgufTensorInfo* info = nullptr;
  bool linear = true;      // false: an F32 vector (norm or bias)
  QuantType type = QuantType::kF32;  // storage type on the device
  int rows = 0;
  int cols = 0;
  uint64_t bytes = 0;      // file bytes
};

QuantType StorageType(GgmlType type, const std::string& name) {
  switch (type) {
    case GgmlType::kF32: return QuantType::kF32;
    case GgmlType::kQ8_0: return QuantType::kQ8_0;
    case GgmlType::kQ4_0: return QuantType::kQ4_0;
    case GgmlType::kQ4_1: return QuantType::kQ4_1;
    case GgmlType::kF16: break;
  }
  throw std::runtime_error("unsupported GGUF tensor type (F16): " + name);
}

// Logical [rows, cols] of a GGUF shape (first dimension fastest; the
// reference's MapShape swaps 2-D shapes, gguf_loader.cc:17-29).
void LogicalShape(const GgufTensorInfo& info, int* rows, int* cols) {
  if (info.shape.empty()) throw std::runtime_error("GGUF tensor without shape: " + info.name);
  uint64_t elements = 1;
  for (uint64_t d : info.shape) elements *= d;
  *cols = static_cast<int>(info.shape.size() == 2 ? info.shape[0] : info.shape.back());
  *rows = static_cast<int>(elements / static_cast<uint64_t>(*cols));
}

Planned Plan(const GgufReader& reader, const std::string& gguf_name,
             const std::string& name, bool linear, bool required) {
  Planned p;
  p.name = name;
  p.linear = linear;
  p.info = reader.FindTensor(gguf_name);
  if (p.info == nullptr) {
    if (required) throw std::runtime_error("GGUF is missing a required tensor: " + gguf_name);
    return p;
  }
  if (!GgufTensorDataSize(*p.info, &p.bytes)) {
    throw std::runtime_error("unsupported GGUF tensor: " + gguf_name);
  }
  p.type = StorageType(p.info->type, gguf_name);
  if (linear && p.info->shape.size() != 2) {
    throw std::runtime_error("GGUF linear weight must be 2-D: " + gguf_name);
  }
  LogicalShape(*p.info, &p.rows, &p.cols);
  return p;
}

void RequireShape(const Planned& p, int rows, int cols) {
  if (p.info == nullptr) return;
  if (p.linear ? (p.rows != rows || p.cols != cols)
               : (static_cast<int64_t>(p.rows) * p.cols != static_cast<int64_t>(rows))) {
    throw std::runtime_error("GGUF weight shape mismatch: " + p.name);
  }
}

int MlbType(QuantType type) {
  switch (type) {
    case QuantType::kF32: return MLB_F32;
    case QuantType::kQ8_0: return MLB_Q8_0;
    case QuantType::kQ4_0: return MLB_Q4_0;
    case QuantType::kQ4_1: return MLB_Q4_1;
  }
  return MLB_F32;
}

}  // namespace

CudaGgufModel LoadGgufModelToDevices(const std::string& path,
                                     const std::vector<int>& devices) {
  if (devices.empty()) throw std::invalid_argument("LoadGgufModelToDevices: no device");
  GgufReader reader;
  if (!reader.Load(path)) throw std::runtime_error("GGUF parse failed: " + reader.Error());

  CudaGgufModel result;
  Model& model = result.model;
  model.config = GgufConfig(reader);
  const ModelConfig& c = model.config;

  std::vector<Planned> plan;
  plan.push_back(Plan(reader, "token_embd.weight", "token_embedding", true, true));
  RequireShape(plan.back(), c.vocab_size, c.dim);
  plan.push_back(Plan(reader, "output_norm.weight", "final_norm", false, true));
  RequireShape(plan.back(), c.dim, 1);
  Planned output = Plan(reader, "output.weight", "lm_head", true, false);
  model.tied_lm_head = output.info == nullptr;
  if (!model.tied_lm_head) {
    RequireShape(output, c.vocab_size, c.dim);
    plan.push_back(output);
  }
  for (int layer = 0; layer < c.n_layers; ++layer) {
    const std::string g = "blk." + std::to_string(layer) + ".";
    const std::string n = "layers." + std::to_string(layer) + ".";
    const int attention = c.attention_dim();
    const int kv = c.kv_dim();
    struct Item { const char* gguf; const char* name; bool linear; bool required; int rows; int cols; };
    const Item items[] = {
        {"attn_norm.weight", "attention_norm", false, true, c.dim, 1},
        {"attn_q.weight", "wq", true, true, attention, c.dim},
        {"attn_k.weight", "wk", true, true, kv, c.dim},
        {"attn_v.weight", "wv", true, true, kv, c.dim},
        {"attn_output.weight", "wo", true, true, c.dim, attention},
        {"attn_q.bias", "bq", false, false, attention, 1},
        {"attn_k.bias", "bk", false, false, kv, 1},
        {"attn_v.bias", "bv", false, false, kv, 1},
        {"ffn_norm.weight", "ffn_norm", false, true, c.dim, 1},
        {"ffn_gate.weight", "w_gate", true, true, c.hidden_dim, c.dim},
        {"ffn_up.weight", "w_up", true, true, c.hidden_dim, c.dim},
        {"ffn_down.weight", "w_down", true, true, c.dim, c.hidden_dim},
    };
    for (const Item& item : items) {
      Planned p = Plan(reader, g + item.gguf, n + item.name, item.linear, item.required);
      if (p.info == nullptr) continue;  // optional bias absent
      RequireShape(p, item.rows, item.cols);
      plan.push_back(std::move(p));
    }
  }

  // device buffers for every replica; quantised vectors land in a
  // temporary block buffer and are dequantised afterwards
  const size_t count = devices.size();
  result.replicas.resize(count);
  std::vector<std::vector<CudaWeight>> weights(count);
  std::vector<std::vector<DeviceBuffer>> blocks(count);
  for (size_t d = 0; d < count; ++d) {
    CudaDeviceScope scope(devices[d]);
    result.replicas[d] = std::make_shared<CudaModelWeights>();
    result.replicas[d]->set_device(devices[d]);
    for (const Planned& p : plan) {
      CudaWeight w;
      w.name = p.name;
      w.linear = p.linear;
      if (p.linear) {
        w.type = p.type;
        w.rows = p.rows;
        w.cols = p.cols;
        w.buffer.Reset(p.bytes);
      } else {
        w.type = QuantType::kF32;
        w.rows = p.rows * p.cols;
        w.cols = 1;
        w.buffer.Reset(static_cast<size_t>(w.rows) * sizeof(float));
      }
      weights[d].push_back(std::move(w));
      blocks[d].emplace_back();
      if (!p.linear && p.type != QuantType::kF32) blocks[d].back().Reset(p.bytes);
    }
  }

  // the staging streams do not order with the legacy default stream: let
  // earlier work on these devices (which may still use recycled pool blocks)
  // finish before the copies start
  for (int device : devices) {
    CudaDeviceScope scope(device);
    const cudaError_t error = cudaDeviceSynchronize();
    if (error != cudaSuccess) ThrowCuda("GGUF upload", error);
  }
  // stream the file once, in file order
  std::vector<size_t> order(plan.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) {
    return plan[a].info->offset < plan[b].info->offset;
  });
  {
    FileToDevices copier(path, devices);
    std::vector<void*> dst(count);
    for (size_t i : order) {
      const Planned& p = plan[i];
      const bool staged = !p.linear && p.type != QuantType::kF32;
      for (size_t d = 0; d < count; ++d)
        dst[d] = staged ? blocks[d][i].data() : weights[d][i].buffer.data();
      copier.Copy(reader.DataOffset() + p.info->offset, static_cast<size_t>(p.bytes), dst);
    }
    copier.Finish();
  }
  for (size_t d = 0; d < count; ++d) {
    CudaDeviceScope scope(devices[d]);
    for (size_t i = 0; i < plan.size(); ++i) {
      const Planned& p = plan[i];
      if (p.linear || p.type == QuantType::kF32) continue;
      for (int r = 0; r < p.rows; ++r) {  // LoadF32 dequantises row by row
        const int rc = mlb_embedding_row(blocks[d][i].data(), MlbType(p.type), p.rows, p.cols,
                                         r, static_cast<float*>(weights[d][i].buffer.data()) +
                                                static_cast<int64_t>(r) * p.cols,
                                         nullptr);
        if (rc != MLB_OK) {
          throw std::runtime_error(std::string("GGUF vector dequantisation: ") +
                                   mlb_last_error());
        }
      }
    }
    const cudaError_t error = cudaDeviceSynchronize();
    if (error != cudaSuccess) ThrowCuda("GGUF upload", error);
    for (CudaWeight& w : weights[d]) result.replicas[d]->Add(std::move(w));
  }
  // empty host layers, so that the per-token path's layer-count check
  // (forward.cc:23-25) accepts the model too
  model.layers.resize(static_cast<size_t>(c.n_layers));
  model.cuda_weights = result.replicas.front();
  return result;
}

}  // namespace mini_lla
