// Shared device helpers and host plumbing for the sm_100a layer operators.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "mlb_ops.h"

namespace mlb {

// ---------------------------------------------------------------------------
// Host side: per-thread error text, argument checks, per-device SM counts.

void SetError(const std::string& message);
int Fail(int code, const std::string& message);
int CheckLaunch(const char* op);

// Streaming-multiprocessor count of the current device (cached per device).
int SmCount();

inline bool Aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

inline cudaStream_t AsStream(void* s) { return static_cast<cudaStream_t>(s); }

// Programmatic dependent launch (on unless mlb_set_launch_overlap(0)): a
// kernel launched through Launch may start while the stream's previous kernel
// is still running, so that its launch and set-up overlap that kernel's
// tail.  Every kernel of this library begins with LaunchWait(), which returns
// once the previous kernel has completed and its writes are visible, before
// it reads or writes global memory; it then calls LaunchNext() so that the
// kernel after it may launch in turn.
bool LaunchOverlap();

template <typename... KArgs, typename... Args>
void Launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
            Args... args) {
  cudaLaunchConfig_t config{};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = LaunchOverlap() ? 1 : 0;
  // an error is left for CheckLaunch (cudaGetLastError), as with <<< >>>
  (void)cudaLaunchKernelEx(&config, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// Device side.

// Block size of the ggml formats: 32 values per block.
constexpr int kBlock = 32;

// The two halves of programmatic dependent launch (see Launch above).
__device__ __forceinline__ void LaunchWait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void LaunchNext() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// FP16 bit pattern -> F32 by integer decode.  Same mapping as the reference's
// Fp16ToFloat (src/quant.cc:44-71), including subnormal normalisation and the
// NaN payload (mantissa << 13, quiet bit not forced); the subnormal loop is
// replaced by a count-leading-zeros of the 10-bit mantissa.
__device__ __forceinline__ float Fp16BitsToF32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      const int top = 31 - __clz(m);  // highest set bit, 0..9
      const int shift = 10 - top;     // iterations of the reference loop
      m = (m << shift) & 0x3ffu;
      bits = sign | (static_cast<uint32_t>(1 - shift + 112) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  return __uint_as_float(bits);
}

// Streaming loads/stores (evict-first; each byte is touched once per pass).
__device__ __forceinline__ float4 LoadStream(const float4* p) {
  return __ldcs(p);
}
__device__ __forceinline__ void StoreStream(float4* p, const float4& v) {
  __stcs(p, v);
}

__device__ __forceinline__ float4 AddRn(const float4& a, const float4& b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y),
                     __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

__device__ __forceinline__ float WarpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float WarpMax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum whose result every thread receives.  `scratch` holds 32
// floats; callers alternate two scratch arrays between consecutive calls so
// that one barrier per reduction suffices.
__device__ __forceinline__ float BlockSum(float v, float* scratch) {
  v = WarpSum(v);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int warps = (blockDim.x + 31) >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < warps ? scratch[lane] : 0.0f;
  return WarpSum(t);
}

__device__ __forceinline__ float BlockMax(float v, float* scratch) {
  v = WarpMax(v);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int warps = (blockDim.x + 31) >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < warps ? scratch[lane] : -INFINITY;
  return WarpMax(t);
}

// 16-byte global -> shared copies that bypass registers (cp.async).
__device__ __forceinline__ void CopyAsync16(void* smem_dst, const void* gmem_src) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst),
               "l"(gmem_src));
}
__device__ __forceinline__ void CopyAsyncCommit() {
  asm volatile("cp.async.commit_group;\n" ::);
}
template <int N>
__device__ __forceinline__ void CopyAsyncWait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

}  // namespace mlb
