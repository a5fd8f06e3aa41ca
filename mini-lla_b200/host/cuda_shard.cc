// Multi-GPU prefill sharding and bounded waits for the layer-operator path.
//
// The reference runs on one device (README "不支持 ... 多 GPU"; its device is
// chosen once in backend.cc:26-42 / cuda_weights.cc:83).  Token rows are
// independent in every layer operator, so a large prefill batch splits into
// contiguous token ranges, one per GPU, with replicated weights and no
// collective.  CudaShardRows runs one host thread per device, like the
// reference's ParallelFor (thread_pool.cc:47-83) runs one chunk per worker,
// and rethrows the first failure on the caller (thread_pool.cc:102-107).
#include <cuda_runtime.h>

#include <chrono>
#include <exception>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "mini_llama/cuda_layer_ops.h"
#include "mini_llama/cuda_runtime.h"

namespace mini_lla {

std::pair<int, int> ShardRange(int total, int shards, int index) {
  if (total < 0 || shards <= 0 || index < 0 || index >= shards) {
    throw std::invalid_argument("ShardRange: bad shard");
  }
  const int base = total / shards;
  const int extra = total % shards;
  const int begin = index * base + (index < extra ? index : extra);
  return {begin, begin + base + (index < extra ? 1 : 0)};
}

void CudaShardRows(int total_rows, const std::vector<int>& devices,
                   const std::function<void(int, int, int)>& body) {
  if (devices.empty()) throw std::invalid_argument("CudaShardRows: no devices");
  std::mutex error_mutex;
  std::exception_ptr error;
  std::vector<std::thread> threads;
  threads.reserve(devices.size());
  for (size_t i = 0; i < devices.size(); ++i) {
    const auto range =
        ShardRange(total_rows, static_cast<int>(devices.size()), static_cast<int>(i));
    const int device = devices[i];
    threads.emplace_back([&, range, device] {
      try {
        CudaSetDevice(device);
        body(device, range.first, range.second);
      } catch (...) {
        std::lock_guard<std::mutex> lock(error_mutex);
        if (error == nullptr) error = std::current_exception();
      }
    });
  }
  for (std::thread& t : threads) t.join();
  if (error != nullptr) std::rethrow_exception(error);
}

bool CudaWaitEvent(void* event, double timeout_ms) {
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::duration<double, std::milli>(timeout_ms);
  cudaEvent_t e = static_cast<cudaEvent_t>(event);
  while (true) {
    const cudaError_t status = cudaEventQuery(e);
    if (status == cudaSuccess) return true;
    if (status != cudaErrorNotReady) {
      throw std::runtime_error(std::string("CudaWaitEvent: ") +
                               cudaGetErrorString(status));
    }
    if (std::chrono::steady_clock::now() >= deadline) return false;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace mini_lla
