// mini-lla's GPU operator API (the reference's include/mini_llama/cuda_ops.h)
// and the row-batched additions of cuda_layer_ops.h, implemented over the
// sm_100a kernels of libmlb.so through its C ABI (include/mlb_ops.h).  This
// file takes the place of the reference's src/cuda_ops.cu; callers such as
// src/cuda_forward.cc compile against the same header unchanged.
//
// Semantics kept from the reference (src/cuda_ops.cu:193-308):
//   - host-side shape checks throw std::invalid_argument, an out-of-range
//     token throws std::out_of_range, a CUDA failure std::runtime_error;
//   - outputs are fresh CudaTensors (now from the per-device pool);
//   - everything runs on the legacy default stream of the current device.
// Differences that callers can observe: RoPE is bit-exact with the CPU
// reference at every position (the (cos, sin) table is built on the host and
// cached per device; the reference's kernel evaluates powf/cosf/sinf on the
// device, cuda_ops.cu:69-74), RMSNorm uses an IEEE 1/sqrt instead of rsqrtf
// (cuda_ops.cu:54), and CudaAddBias / CudaRope reject mismatched sizes the
// reference kernels would read past.
#include "mini_llama/cuda_ops.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

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

const float* F32(const CudaWeight& w) {
  return static_cast<const float*>(w.buffer.data());
}

int QType(QuantType type) {
  switch (type) {
    case QuantType::kF32: return MLB_F32;
    case QuantType::kQ8_0: return MLB_Q8_0;
    case QuantType::kQ4_0: return MLB_Q4_0;
    case QuantType::kQ4_1: return MLB_Q4_1;
  }
  throw std::invalid_argument("unknown quant type");
}

size_t WeightSize(const CudaWeight& w) {
  return static_cast<size_t>(w.rows) * static_cast<size_t>(w.cols);
}

// Per-device cache of host-built RoPE (cos, sin) tables keyed by (theta,
// head_dim), grown by doubling to cover the largest position asked for.
class RopeTables {
 public:
  static RopeTables& Instance() {
    static RopeTables* tables = new RopeTables;
    return *tables;
  }

  // Returns the table of the current device covering positions [0, need).
  const float* Get(float theta, int head_dim, int64_t need, int64_t* rows) {
    int device = 0;
    cudaGetDevice(&device);
    uint32_t theta_bits = 0;
    std::memcpy(&theta_bits, &theta, sizeof(theta_bits));
    std::lock_guard<std::mutex> lock(mutex_);
    Entry& e = tables_[std::make_tuple(device, theta_bits, head_dim)];
    if (e.rows < need) {
      int64_t grow = e.rows > 0 ? e.rows * 2 : 4096;
      while (grow < need) grow *= 2;
      std::vector<float> host(static_cast<size_t>(grow) * head_dim);
      Check(mlb_rope_table_build_host(theta, head_dim, 0, grow, host.data()),
            "CudaRope: table");
      // The old table may still be read by queued kernels: the new one is a
      // separate block, and the old block goes back to the pool, whose reuse
      // is ordered on the legacy default stream after those kernels.
      DeviceBuffer fresh;
      fresh.Reset(host.size() * sizeof(float));
      fresh.Upload(host.data(), host.size() * sizeof(float));
      e.buffer = std::move(fresh);
      e.rows = grow;
    }
    *rows = e.rows;
    return static_cast<const float*>(e.buffer.data());
  }

  int Rows(float theta, int head_dim) {
    int device = 0;
    cudaGetDevice(&device);
    uint32_t theta_bits = 0;
    std::memcpy(&theta_bits, &theta, sizeof(theta_bits));
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = tables_.find(std::make_tuple(device, theta_bits, head_dim));
    return it == tables_.end() ? 0 : static_cast<int>(it->second.rows);
  }

 private:
  struct Entry {
    DeviceBuffer buffer;
    int64_t rows = 0;
  };
  std::mutex mutex_;
  std::map<std::tuple<int, uint32_t, int>, Entry> tables_;
};

// Small host arrays (token ids, positions, softmax lengths) reach the device
// without the host waiting for it: they are copied into a slot of pinned
// memory and moved by cudaMemcpyAsync on the legacy default stream, ordered
// before the kernel that reads them.  Every host thread has, per device, a
// ring of kSlots slots; a slot is refilled once the copy that last read it
// has completed (its event), so the host waits only when kSlots uploads are
// still queued on the device.  Arrays above kSlotBytes take the blocking
// DeviceBuffer::Upload.
class IntStaging {
 public:
  static constexpr size_t kSlotBytes = size_t{256} << 10;  // 65536 ints
  static constexpr int kSlots = 4;

  static DeviceBuffer Upload(const std::vector<int>& values) {
    static_assert(sizeof(int) == sizeof(int32_t), "int must be 32-bit");
    DeviceBuffer buffer;
    if (values.empty()) return buffer;
    const size_t bytes = values.size() * sizeof(int32_t);
    buffer.Reset(bytes);
    if (bytes > kSlotBytes) {
      buffer.Upload(values.data(), bytes);
      return buffer;
    }
    thread_local IntStaging staging;
    Ring& ring = staging.RingOf(CurrentDevice());
    const int slot = ring.next;
    ring.next = (ring.next + 1) % kSlots;
    if (ring.used[slot]) {
      const cudaError_t error = cudaEventSynchronize(ring.done[slot]);
      if (error != cudaSuccess) Throw("int upload", error);
    }
    char* pinned = ring.pinned + static_cast<size_t>(slot) * kSlotBytes;
    std::memcpy(pinned, values.data(), bytes);
    cudaError_t error = cudaMemcpyAsync(buffer.data(), pinned, bytes, cudaMemcpyHostToDevice,
                                        cudaStreamLegacy);
    if (error == cudaSuccess) error = cudaEventRecord(ring.done[slot], cudaStreamLegacy);
    if (error != cudaSuccess) Throw("int upload", error);
    ring.used[slot] = true;
    return buffer;
  }

  ~IntStaging() {
    for (auto& entry : rings_) {
      Ring& ring = entry.second;
      for (int i = 0; i < kSlots; ++i) {
        if (ring.used[i]) cudaEventSynchronize(ring.done[i]);
        if (ring.done[i] != nullptr) cudaEventDestroy(ring.done[i]);
      }
      if (ring.pinned != nullptr) cudaFreeHost(ring.pinned);
    }
  }

 private:
  struct Ring {
    char* pinned = nullptr;
    cudaEvent_t done[kSlots] = {};
    bool used[kSlots] = {};
    int next = 0;
  };

  static int CurrentDevice() {
    int device = 0;
    const cudaError_t error = cudaGetDevice(&device);
    if (error != cudaSuccess) Throw("cudaGetDevice", error);
    return device;
  }

  [[noreturn]] static void Throw(const char* what, cudaError_t error) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
  }

  // events belong to the device that was current when they were created
  Ring& RingOf(int device) {
    Ring& ring = rings_[device];
    if (ring.pinned != nullptr) return ring;
    cudaError_t error = cudaHostAlloc(reinterpret_cast<void**>(&ring.pinned),
                                      kSlots * kSlotBytes, cudaHostAllocPortable);
    if (error != cudaSuccess) Throw("cudaHostAlloc", error);
    for (int i = 0; i < kSlots; ++i) {
      error = cudaEventCreateWithFlags(&ring.done[i], cudaEventDisableTiming);
      if (error != cudaSuccess) Throw("cudaEventCreate", error);
    }
    return ring;
  }

  std::map<int, Ring> rings_;
};

DeviceBuffer UploadInts(const std::vector<int>& values) { return IntStaging::Upload(values); }

void RequireRope(float theta, int head_dim, const char* caller) {
  if (head_dim <= 0 || head_dim % 2 != 0) {
    throw std::invalid_argument(std::string(caller) +
                                ": expected [heads, even_dim]");
  }
  if (!(theta > 0.0f)) {
    throw std::invalid_argument(std::string(caller) + ": invalid theta");
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// The reference's per-vector API (cuda_ops.h:11-34).

CudaTensor CudaRmsNorm(const CudaTensor& x, const CudaWeight& weight,
                       float epsilon) {
  if (weight.rows != static_cast<int>(x.Size())) {
    throw std::invalid_argument("CudaRmsNorm: weight size mismatch");
  }
  CudaTensor output(x.shape());
  Check(mlb_rmsnorm_f32(x.data(), nullptr, nullptr, output.data(), F32(weight),
                        1, static_cast<int64_t>(x.Size()), epsilon, nullptr),
        "CudaRmsNorm");
  return output;
}

void CudaRope(CudaTensor* q, CudaTensor* k, int position, float theta,
              int n_heads, int n_kv_heads, int head_dim, RopeType rope_type) {
  if (q == nullptr || k == nullptr) {
    throw std::invalid_argument("CudaRope: null tensor");
  }
  RequireRope(theta, head_dim, "CudaRope");
  if (position < 0) throw std::invalid_argument("CudaRope: invalid position");
  if (q->Size() != static_cast<size_t>(n_heads) * head_dim ||
      k->Size() != static_cast<size_t>(n_kv_heads) * head_dim) {
    throw std::invalid_argument("CudaRope: q/k size mismatch");
  }
  int64_t rows = 0;
  const float* table =
      RopeTables::Instance().Get(theta, head_dim, int64_t{position} + 1, &rows);
  Check(mlb_rope_f32(q->data(), k->data(), nullptr, nullptr, nullptr, position,
                     table, rows, 1, n_heads, n_kv_heads, head_dim,
                     rope_type == RopeType::kNeoX ? 1 : 0, nullptr, nullptr),
        "CudaRope");
}

CudaTensor CudaSilu(const CudaTensor& x) {
  CudaTensor output(x.shape());
  Check(mlb_silu_f32(x.data(), output.data(), static_cast<int64_t>(x.Size()),
                     nullptr),
        "CudaSilu");
  return output;
}

CudaTensor CudaMul(const CudaTensor& a, const CudaTensor& b) {
  if (a.Size() != b.Size()) throw std::invalid_argument("CudaMul: size mismatch");
  CudaTensor output(a.shape());
  Check(mlb_mul_f32(a.data(), b.data(), output.data(),
                    static_cast<int64_t>(a.Size()), nullptr),
        "CudaMul");
  return output;
}

CudaTensor CudaAdd(const CudaTensor& a, const CudaTensor& b) {
  if (a.Size() != b.Size()) throw std::invalid_argument("CudaAdd: size mismatch");
  CudaTensor output(a.shape());
  Check(mlb_add_f32(a.data(), b.data(), output.data(),
                    static_cast<int64_t>(a.Size()), nullptr),
        "CudaAdd");
  return output;
}

CudaTensor CudaSoftmax(const CudaTensor& x) {
  if (x.shape().size() != 1 || x.Size() == 0) {
    throw std::invalid_argument("CudaSoftmax: expected a non-empty vector");
  }
  CudaTensor output(x.shape());
  Check(mlb_softmax_rows_f32(x.data(), output.data(), 1,
                             static_cast<int64_t>(x.Size()), nullptr, nullptr,
                             nullptr),
        "CudaSoftmax");
  return output;
}

CudaTensor CudaEmbeddingRow(const CudaWeight& embedding, int token) {
  if (token < 0 || token >= embedding.rows) {
    throw std::out_of_range("CudaEmbeddingRow: token out of range");
  }
  CudaTensor output({embedding.cols});
  Check(mlb_embedding_row(embedding.buffer.data(), QType(embedding.type),
                          embedding.rows, embedding.cols, token, output.data(),
                          nullptr),
        "CudaEmbeddingRow");
  return output;
}

CudaTensor CudaAddBias(const CudaTensor& value, const CudaWeight* bias) {
  if (bias != nullptr && WeightSize(*bias) != value.Size()) {
    throw std::invalid_argument("CudaAddBias: bias size mismatch");
  }
  CudaTensor output(value.shape());
  Check(mlb_add_bias_f32(value.data(), bias == nullptr ? nullptr : F32(*bias),
                         output.data(), 1, static_cast<int64_t>(value.Size()),
                         nullptr),
        "CudaAddBias");
  return output;
}

// ---------------------------------------------------------------------------
// Row-batched additions (cuda_layer_ops.h).

CudaTensor CudaAddRmsNormRows(const CudaTensor& x, const CudaTensor* residual,
                              const CudaWeight& weight, float epsilon,
                              CudaTensor* h_out) {
  const int cols = weight.rows;
  if (cols <= 0 || x.Size() % static_cast<size_t>(cols) != 0 ||
      x.shape().empty() || x.shape().back() != cols) {
    throw std::invalid_argument("CudaAddRmsNormRows: weight size mismatch");
  }
  if (residual != nullptr && residual->shape() != x.shape()) {
    throw std::invalid_argument("CudaAddRmsNormRows: residual shape mismatch");
  }
  if (h_out != nullptr && residual == nullptr) {
    throw std::invalid_argument("CudaAddRmsNormRows: h_out needs a residual");
  }
  if (h_out != nullptr && h_out->shape() != x.shape()) *h_out = CudaTensor(x.shape());
  CudaTensor output(x.shape());
  const int64_t rows = static_cast<int64_t>(x.Size() / cols);
  Check(mlb_rmsnorm_f32(x.data(), residual ? residual->data() : nullptr,
                        h_out ? h_out->data() : nullptr, output.data(),
                        F32(weight), rows, cols, epsilon, nullptr),
        "CudaAddRmsNormRows");
  return output;
}

CudaTensor CudaAddBiasRows(const CudaTensor& value, const CudaWeight* bias) {
  if (value.shape().empty()) {
    throw std::invalid_argument("CudaAddBiasRows: expected rows");
  }
  const int64_t cols = value.shape().back();
  if (bias != nullptr && WeightSize(*bias) != static_cast<size_t>(cols)) {
    throw std::invalid_argument("CudaAddBiasRows: bias size mismatch");
  }
  CudaTensor output(value.shape());
  if (value.Size() == 0) return output;
  Check(mlb_add_bias_f32(value.data(), bias == nullptr ? nullptr : F32(*bias),
                         output.data(), static_cast<int64_t>(value.Size()) / cols, cols,
                         nullptr),
        "CudaAddBiasRows");
  return output;
}

void CudaAddBiasRowsInPlace(float* value, int64_t rows, const CudaWeight& bias) {
  const int64_t cols = static_cast<int64_t>(WeightSize(bias));
  if (rows < 0 || cols <= 0) throw std::invalid_argument("CudaAddBiasRows: bad size");
  if (rows == 0) return;
  if (value == nullptr) throw std::invalid_argument("CudaAddBiasRows: null value");
  Check(mlb_add_bias_f32(value, F32(bias), value, rows, cols, nullptr), "CudaAddBiasRows");
}

CudaTensor CudaSwiGlu(const CudaTensor& gate, const CudaTensor& up) {
  if (gate.shape() != up.shape()) {
    throw std::invalid_argument("CudaSwiGlu: shape mismatch");
  }
  CudaTensor output(gate.shape());
  const int64_t cols = gate.shape().back();
  Check(mlb_swiglu_f32(gate.data(), up.data(), output.data(),
                       static_cast<int64_t>(gate.Size()) / cols, cols, nullptr),
        "CudaSwiGlu");
  return output;
}

void CudaRopeRows(CudaTensor* q, CudaTensor* k, const CudaWeight* bq,
                  const CudaWeight* bk, const std::vector<int>& positions,
                  float theta, int n_heads, int n_kv_heads, int head_dim,
                  RopeType rope_type) {
  if (q == nullptr || k == nullptr) {
    throw std::invalid_argument("CudaRopeRows: null tensor");
  }
  RequireRope(theta, head_dim, "CudaRopeRows");
  const size_t rows = positions.size();
  if (q->Size() != rows * n_heads * head_dim ||
      k->Size() != rows * n_kv_heads * head_dim) {
    throw std::invalid_argument("CudaRopeRows: q/k size mismatch");
  }
  CudaRopeRowsInPlace(q->data(), k->data(), bq, bk, positions, theta, n_heads, n_kv_heads,
                      head_dim, rope_type);
}

void CudaRopeRowsInPlace(float* q, float* k, const CudaWeight* bq, const CudaWeight* bk,
                         const std::vector<int>& positions, float theta, int n_heads,
                         int n_kv_heads, int head_dim, RopeType rope_type) {
  RequireRope(theta, head_dim, "CudaRopeRows");
  const size_t rows = positions.size();
  if (rows > 0 && (q == nullptr || (n_kv_heads > 0 && k == nullptr))) {
    throw std::invalid_argument("CudaRopeRows: null q or k");
  }
  if ((bq != nullptr && WeightSize(*bq) != static_cast<size_t>(n_heads) * head_dim) ||
      (bk != nullptr && WeightSize(*bk) != static_cast<size_t>(n_kv_heads) * head_dim)) {
    throw std::invalid_argument("CudaRopeRows: bias size mismatch");
  }
  if (rows == 0) return;
  int max_position = 0;
  bool consecutive = true;
  for (size_t i = 0; i < rows; ++i) {
    if (positions[i] < 0) {
      throw std::invalid_argument("CudaRopeRows: invalid position");
    }
    if (positions[i] > max_position) max_position = positions[i];
    if (positions[i] != positions[0] + static_cast<int>(i)) consecutive = false;
  }
  int64_t table_rows = 0;
  const float* table = RopeTables::Instance().Get(
      theta, head_dim, int64_t{max_position} + 1, &table_rows);
  const int neox = rope_type == RopeType::kNeoX ? 1 : 0;
  if (consecutive) {
    Check(mlb_rope_f32(q, k, bq ? F32(*bq) : nullptr,
                       bk ? F32(*bk) : nullptr, nullptr, positions[0], table,
                       table_rows, static_cast<int64_t>(rows), n_heads,
                       n_kv_heads, head_dim, neox, nullptr, nullptr),
          "CudaRopeRows");
    return;
  }
  const DeviceBuffer device_positions = UploadInts(positions);
  Check(mlb_rope_f32(q, k, bq ? F32(*bq) : nullptr,
                     bk ? F32(*bk) : nullptr,
                     static_cast<const int32_t*>(device_positions.data()), 0,
                     table, table_rows, static_cast<int64_t>(rows), n_heads,
                     n_kv_heads, head_dim, neox, nullptr, nullptr),
        "CudaRopeRows");
}

CudaTensor CudaSoftmaxRows(const CudaTensor& x,
                           const std::vector<int>* valid_len) {
  if (x.Size() == 0 || x.shape().empty()) {
    throw std::invalid_argument("CudaSoftmaxRows: expected non-empty rows");
  }
  const int cols = x.shape().back();
  const size_t rows = x.Size() / static_cast<size_t>(cols);
  DeviceBuffer lengths;
  if (valid_len != nullptr) {
    if (valid_len->size() != rows) {
      throw std::invalid_argument("CudaSoftmaxRows: valid_len size mismatch");
    }
    for (int len : *valid_len) {
      if (len < 1 || len > cols) {
        throw std::invalid_argument("CudaSoftmaxRows: expected a non-empty vector");
      }
    }
    lengths = UploadInts(*valid_len);
  }
  CudaTensor output(x.shape());
  Check(mlb_softmax_rows_f32(x.data(), output.data(),
                             static_cast<int64_t>(rows), cols,
                             static_cast<const int32_t*>(lengths.data()),
                             nullptr, nullptr),
        "CudaSoftmaxRows");
  return output;
}

CudaTensor CudaEmbeddingRows(const CudaWeight& embedding,
                             const std::vector<int>& tokens) {
  for (int token : tokens) {
    if (token < 0 || token >= embedding.rows) {
      throw std::out_of_range("CudaEmbeddingRows: token out of range");
    }
  }
  if (tokens.empty()) {
    throw std::invalid_argument("CudaEmbeddingRows: no tokens");
  }
  CudaTensor output({static_cast<int>(tokens.size()), embedding.cols});
  const DeviceBuffer ids = UploadInts(tokens);
  Check(mlb_embedding_gather(embedding.buffer.data(), QType(embedding.type),
                             embedding.rows, embedding.cols,
                             static_cast<const int32_t*>(ids.data()),
                             static_cast<int64_t>(tokens.size()), output.data(),
                             nullptr, nullptr),
        "CudaEmbeddingRows");
  return output;
}

int CudaRopeTableRows(float theta, int head_dim) {
  return RopeTables::Instance().Rows(theta, head_dim);
}

}  // namespace mini_lla
