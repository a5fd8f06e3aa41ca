// Device runtime for mini-lla's GPU path, implementing the reference's
// include/mini_llama/cuda_runtime.h (reference src/cuda_runtime.cc) with two
// changes behind the same API:
//   - DeviceBuffer memory comes from a per-device caching pool: Reset() reuses
//     a freed block of the same rounded size instead of calling cudaMalloc,
//     and Clear() returns the block to the pool of the device that owns it
//     (the reference allocates and frees on every operator call,
//     cuda_runtime.cc:88-105).  Reuse is safe for the reference's callers
//     because every operator runs on the legacy default stream, which orders
//     a later writer after an earlier reader of the same block.
//   - Upload / Download of more than kStageThreshold bytes go through a
//     per-thread pinned staging buffer in double-buffered chunks instead of
//     one pageable cudaMemcpy; both still return only when the copy is done.
// Device queries, CudaSetDevice and CudaCheckLastError keep the reference's
// behaviour and messages' meaning.
#include "mini_llama/cuda_runtime.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "mini_llama/cuda_layer_ops.h"

namespace mini_lla {
namespace {

[[noreturn]] void ThrowCuda(const std::string& what, cudaError_t error) {
  throw std::runtime_error(what + ": " + cudaGetErrorString(error));
}

int CurrentDevice() {
  int device = 0;
  const cudaError_t error = cudaGetDevice(&device);
  if (error != cudaSuccess) ThrowCuda("cudaGetDevice", error);
  return device;
}

// Blocks are rounded up to 512 bytes (small) or 2 MiB (large) so that the
// per-token sizes the layer loop asks for repeat exactly.
size_t RoundSize(size_t bytes) {
  const size_t unit = bytes < (size_t{1} << 21) ? 512 : (size_t{1} << 21);
  return (bytes + unit - 1) / unit * unit;
}

// Per-device free lists plus the owner map of live blocks.  Never destroyed
// (DeviceBuffers with static storage may be cleared during exit).
class Pool {
 public:
  static Pool& Instance() {
    static Pool* pool = new Pool;
    return *pool;
  }

  void* Allocate(size_t bytes, size_t* rounded) {
    const int device = CurrentDevice();
    *rounded = RoundSize(bytes);
    {
      std::lock_guard<std::mutex> lock(mutex_);
      auto& free_list = free_[Key(device, *rounded)];
      if (!free_list.empty()) {
        void* p = free_list.back();
        free_list.pop_back();
        cached_[device] -= *rounded;
        owner_[p] = {device, *rounded};
        return p;
      }
    }
    void* p = nullptr;
    cudaError_t error = cudaMalloc(&p, *rounded);
    if (error != cudaSuccess) {
      cudaGetLastError();
      Release(device);  // give cached blocks back and retry once
      error = cudaMalloc(&p, *rounded);
      if (error != cudaSuccess) ThrowCuda("cudaMalloc", error);
    }
    std::lock_guard<std::mutex> lock(mutex_);
    owner_[p] = {device, *rounded};
    return p;
  }

  void Free(void* p) {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = owner_.find(p);
    if (it == owner_.end()) return;
    const Block block = it->second;
    owner_.erase(it);
    if (cached_[block.device] + block.bytes > kMaxCachedBytes) {
      int current = 0;
      cudaGetDevice(&current);
      cudaSetDevice(block.device);
      cudaFree(p);
      cudaSetDevice(current);
      return;
    }
    free_[Key(block.device, block.bytes)].push_back(p);
    cached_[block.device] += block.bytes;
  }

  size_t Cached(int device) {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = cached_.find(device);
    return it == cached_.end() ? 0 : it->second;
  }

  void Release(int device) {
    std::vector<void*> blocks;
    {
      std::lock_guard<std::mutex> lock(mutex_);
      for (auto& entry : free_) {
        if (static_cast<int>(entry.first >> 56) != device) continue;
        blocks.insert(blocks.end(), entry.second.begin(), entry.second.end());
        entry.second.clear();
      }
      cached_[device] = 0;
    }
    if (blocks.empty()) return;
    int current = 0;
    cudaGetDevice(&current);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    for (void* p : blocks) cudaFree(p);
    cudaSetDevice(current);
  }

 private:
  struct Block {
    int device;
    size_t bytes;
  };
  static constexpr size_t kMaxCachedBytes = size_t{8} << 30;  // per device

  static uint64_t Key(int device, size_t bytes) {
    return (static_cast<uint64_t>(device) << 56) | bytes;
  }

  std::mutex mutex_;
  std::unordered_map<uint64_t, std::vector<void*>> free_;
  std::unordered_map<void*, Block> owner_;
  std::unordered_map<int, size_t> cached_;
};

// Per-thread pinned staging for large host<->device copies.
constexpr size_t kStageThreshold = size_t{1} << 20;
constexpr size_t kStageChunk = size_t{8} << 20;

struct Staging {
  void* buffer[2] = {nullptr, nullptr};
  cudaStream_t stream = nullptr;
  cudaEvent_t done[2] = {nullptr, nullptr};
  int device = -1;

  ~Staging() {
    for (int i = 0; i < 2; ++i) {
      if (buffer[i] != nullptr) cudaFreeHost(buffer[i]);
      if (done[i] != nullptr) cudaEventDestroy(done[i]);
    }
    if (stream != nullptr) cudaStreamDestroy(stream);
  }

  void Prepare() {
    const int current = CurrentDevice();
    if (buffer[0] != nullptr && device == current) return;
    if (stream != nullptr) {
      cudaStreamDestroy(stream);
      cudaEventDestroy(done[0]);
      cudaEventDestroy(done[1]);
    }
    for (int i = 0; i < 2; ++i) {
      if (buffer[i] == nullptr) {
        const cudaError_t error = cudaHostAlloc(&buffer[i], kStageChunk,
                                                cudaHostAllocPortable);
        if (error != cudaSuccess) ThrowCuda("cudaHostAlloc", error);
      }
    }
    // A blocking stream: ordered with the legacy default stream, so copies
    // see every earlier operator's writes and later operators see the copy.
    cudaError_t error = cudaStreamCreate(&stream);
    if (error != cudaSuccess) ThrowCuda("cudaStreamCreate", error);
    for (int i = 0; i < 2; ++i) {
      error = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
      if (error != cudaSuccess) ThrowCuda("cudaEventCreate", error);
    }
    device = current;
  }
};

Staging& ThreadStaging() {
  thread_local Staging staging;
  staging.Prepare();
  return staging;
}

void StagedUpload(void* device_dst, const void* host_src, size_t bytes) {
  Staging& st = ThreadStaging();
  const char* src = static_cast<const char*>(host_src);
  char* dst = static_cast<char*>(device_dst);
  for (size_t off = 0, i = 0; off < bytes; off += kStageChunk, ++i) {
    const int slot = static_cast<int>(i & 1);
    const size_t n = std::min(kStageChunk, bytes - off);
    if (i >= 2) {
      const cudaError_t error = cudaEventSynchronize(st.done[slot]);
      if (error != cudaSuccess) ThrowCuda("upload", error);
    }
    std::memcpy(st.buffer[slot], src + off, n);
    cudaError_t error = cudaMemcpyAsync(dst + off, st.buffer[slot], n,
                                        cudaMemcpyHostToDevice, st.stream);
    if (error == cudaSuccess) error = cudaEventRecord(st.done[slot], st.stream);
    if (error != cudaSuccess) ThrowCuda("upload", error);
  }
  const cudaError_t error = cudaStreamSynchronize(st.stream);
  if (error != cudaSuccess) ThrowCuda("upload", error);
}

void StagedDownload(void* host_dst, const void* device_src, size_t bytes) {
  Staging& st = ThreadStaging();
  const char* src = static_cast<const char*>(device_src);
  char* dst = static_cast<char*>(host_dst);
  const size_t chunks = (bytes + kStageChunk - 1) / kStageChunk;
  auto issue = [&](size_t i) {
    const int slot = static_cast<int>(i & 1);
    const size_t off = i * kStageChunk;
    const size_t n = std::min(kStageChunk, bytes - off);
    cudaError_t error = cudaMemcpyAsync(st.buffer[slot], src + off, n,
                                        cudaMemcpyDeviceToHost, st.stream);
    if (error == cudaSuccess) error = cudaEventRecord(st.done[slot], st.stream);
    if (error != cudaSuccess) ThrowCuda("download", error);
  };
  issue(0);
  for (size_t i = 0; i < chunks; ++i) {
    if (i + 1 < chunks) issue(i + 1);
    const int slot = static_cast<int>(i & 1);
    const cudaError_t error = cudaEventSynchronize(st.done[slot]);
    if (error != cudaSuccess) ThrowCuda("download", error);
    const size_t off = i * kStageChunk;
    std::memcpy(dst + off, st.buffer[slot], std::min(kStageChunk, bytes - off));
  }
}

}  // namespace

void CudaCheckLastError(const char* caller) {
  const cudaError_t error = cudaGetLastError();
  if (error == cudaSuccess) return;
  throw std::runtime_error(std::string(caller) + ": " + cudaGetErrorString(error));
}

bool CudaRuntimeBuilt() { return true; }

int CudaDeviceCount() {
  int count = 0;
  const cudaError_t error = cudaGetDeviceCount(&count);
  if (error != cudaSuccess) ThrowCuda("CudaDeviceCount", error);
  return count;
}

CudaDeviceInfo CudaGetDeviceInfo(int device) {
  cudaDeviceProp properties{};
  const cudaError_t error = cudaGetDeviceProperties(&properties, device);
  if (error != cudaSuccess) ThrowCuda("CudaGetDeviceInfo", error);
  CudaDeviceInfo info;
  info.id = device;
  info.name = properties.name;
  info.compute_major = properties.major;
  info.compute_minor = properties.minor;
  info.total_memory = static_cast<size_t>(properties.totalGlobalMem);
  cudaDriverGetVersion(&info.driver_version);
  cudaRuntimeGetVersion(&info.runtime_version);
  return info;
}

void CudaSetDevice(int device) {
  const cudaError_t error = cudaSetDevice(device);
  if (error != cudaSuccess) ThrowCuda("CudaSetDevice", error);
}

std::string CudaFormatDeviceInfo(const CudaDeviceInfo& info) {
  std::ostringstream text;
  text << "device " << info.id << ": " << info.name << ", compute "
       << info.compute_major << "." << info.compute_minor << ", "
       << (info.total_memory / (1024.0 * 1024.0)) << " MB, driver "
       << info.driver_version << ", runtime " << info.runtime_version;
  return text.str();
}

DeviceBuffer::~DeviceBuffer() { Clear(); }

DeviceBuffer::DeviceBuffer(DeviceBuffer&& other) noexcept
    : data_(other.data_), size_(other.size_) {
  other.data_ = nullptr;
  other.size_ = 0;
}

DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& other) noexcept {
  if (this != &other) {
    Clear();
    data_ = other.data_;
    size_ = other.size_;
    other.data_ = nullptr;
    other.size_ = 0;
  }
  return *this;
}

void DeviceBuffer::Reset(size_t bytes) {
  Clear();
  if (bytes == 0) return;
  size_t rounded = 0;
  data_ = Pool::Instance().Allocate(bytes, &rounded);
  size_ = bytes;
}

void DeviceBuffer::Clear() {
  if (data_ != nullptr) {
    Pool::Instance().Free(data_);
    data_ = nullptr;
  }
  size_ = 0;
}

void DeviceBuffer::Upload(const void* source, size_t bytes) {
  if (bytes > size_ || source == nullptr) {
    throw std::invalid_argument("DeviceBuffer::Upload: size mismatch");
  }
  if (bytes >= kStageThreshold) {
    StagedUpload(data_, source, bytes);
    return;
  }
  const cudaError_t error =
      cudaMemcpy(data_, source, bytes, cudaMemcpyHostToDevice);
  if (error != cudaSuccess) ThrowCuda("DeviceBuffer::Upload", error);
}

void DeviceBuffer::Download(void* destination, size_t bytes) const {
  if (bytes > size_ || destination == nullptr) {
    throw std::invalid_argument("DeviceBuffer::Download: size mismatch");
  }
  if (bytes >= kStageThreshold) {
    StagedDownload(destination, data_, bytes);
    return;
  }
  const cudaError_t error =
      cudaMemcpy(destination, data_, bytes, cudaMemcpyDeviceToHost);
  if (error != cudaSuccess) ThrowCuda("DeviceBuffer::Download", error);
}

void DeviceBuffer::Zero() {
  if (data_ == nullptr) return;
  const cudaError_t error = cudaMemset(data_, 0, size_);
  if (error != cudaSuccess) ThrowCuda("DeviceBuffer::Zero", error);
}

CudaDeviceScope::CudaDeviceScope(int device) {
  previous_ = CurrentDevice();
  CudaSetDevice(device);
}

CudaDeviceScope::~CudaDeviceScope() { cudaSetDevice(previous_); }

size_t CudaPoolCachedBytes(int device) { return Pool::Instance().Cached(device); }

void CudaPoolRelease(int device) { Pool::Instance().Release(device); }

}  // namespace mini_lla
