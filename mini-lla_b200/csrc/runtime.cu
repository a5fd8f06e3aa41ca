// Host plumbing shared by every entry point: per-thread error text, launch
// checks, the per-device SM-count cache and the small C-ABI helpers.
#include <atomic>
#include <cstdio>
#include <string>

#include "common.cuh"

namespace mlb {
namespace {

thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

std::atomic<int> g_launch_overlap{1};

}  // namespace

bool LaunchOverlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }

void SetError(const std::string& message) { g_last_error = message; }

int Fail(int code, const std::string& message) {
  SetError(message);
  return code;
}

int CheckLaunch(const char* op) {
  const cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) return MLB_OK;
  return Fail(MLB_ERR_CUDA, std::string(op) + ": " + cudaGetErrorString(err));
}

int SmCount() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 ||
      device >= kMaxDevices) {
    return 148;
  }
  int cached = g_sm_count[device].load(std::memory_order_relaxed);
  if (cached > 0) return cached;
  int count = 0;
  if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) !=
          cudaSuccess ||
      count <= 0) {
    cudaGetLastError();
    return 148;
  }
  g_sm_count[device].store(count, std::memory_order_relaxed);
  return count;
}

}  // namespace mlb

extern "C" {

int mlb_version(void) { return 100; }

int mlb_set_launch_overlap(int on) {
  if (on != 0 && on != 1) return mlb::Fail(MLB_ERR_ARG, "mlb_set_launch_overlap: on must be 0 or 1");
  mlb::g_launch_overlap.store(on, std::memory_order_relaxed);
  return MLB_OK;
}

int mlb_launch_overlap(void) { return mlb::LaunchOverlap() ? 1 : 0; }

const char* mlb_last_error(void) { return mlb::g_last_error.c_str(); }

int64_t mlb_row_bytes(int qtype, int64_t cols) {
  if (cols < 0) return -1;
  const int64_t blocks = (cols + mlb::kBlock - 1) / mlb::kBlock;
  switch (qtype) {
    case MLB_F32: return cols * 4;
    case MLB_Q8_0: return blocks * 34;
    case MLB_Q4_0: return blocks * 18;
    case MLB_Q4_1: return blocks * 20;
    default: return -1;
  }
}

int mlb_status_check(const int32_t* status, int32_t* bits_host, void* stream) {
  if (status == nullptr) return mlb::Fail(MLB_ERR_ARG, "status_check: null status");
  int32_t bits = 0;
  cudaError_t err = cudaMemcpyAsync(&bits, status, sizeof(bits),
                                    cudaMemcpyDeviceToHost,
                                    mlb::AsStream(stream));
  if (err == cudaSuccess) err = cudaStreamSynchronize(mlb::AsStream(stream));
  if (err != cudaSuccess) {
    return mlb::Fail(MLB_ERR_CUDA,
                     std::string("status_check: ") + cudaGetErrorString(err));
  }
  if (bits_host != nullptr) *bits_host = bits;
  if (bits != 0) {
    char text[96];
    std::snprintf(text, sizeof(text), "device status bits 0x%x", bits);
    return mlb::Fail(MLB_ERR_RANGE, text);
  }
  return MLB_OK;
}

}  // extern "C"
