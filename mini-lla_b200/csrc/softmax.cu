// Row softmax with a per-row valid length (causal attention rows).
//
// Reference arithmetic (src/ops.cc:83-98 Softmax, applied per head to the
// pos+1 visible scores at src/forward.cc:53-63):
//   m = max(x[0:L]);  e_i = exp(x_i - m);  y_i = e_i / sum(e)
// Entries at and beyond the row's valid length L are written as 0.  The sum
// is a warp/block tree instead of the reference's sequential loop and exp is
// CUDA's expf, so results agree within a few ulp (1e-5 relative bound).
//
// Layout: x, y [rows, cols] fp32 row-major; valid_len [rows] int32 or NULL.
// Kernels:
//   SoftmaxWarpKernel  — cols <= 1024: one warp per row, row in registers,
//                        only the visible float4s are read.
//   SoftmaxBlockKernel — cols <= 32768: one CTA per row, registers.
//   SoftmaxScalarKernel— any other shape: three passes over the row.
// HBM roofline: 4 * sum(L) bytes read + 4 * rows * cols written.
#include <climits>

#include "common.cuh"

namespace mlb {
namespace {

struct SoftmaxArgs {
  const float* x;
  float* y;
  const int32_t* valid_len;
  int64_t rows;
  int cols;
  int32_t* status;
};

__device__ __forceinline__ int RowLength(const SoftmaxArgs& a, int64_t row,
                                         bool* bad) {
  const int len = a.valid_len != nullptr ? __ldg(a.valid_len + row) : a.cols;
  *bad = len < 1 || len > a.cols;
  return len;
}

// Loads the visible float4s of a row (masked entries set to -inf).
__device__ __forceinline__ float4 LoadMasked(const float4* p, int i4, int len) {
  const float ninf = -INFINITY;
  if (4 * i4 >= len) return make_float4(ninf, ninf, ninf, ninf);
  float4 v = LoadStream(p + i4);
  const int base = 4 * i4;
  if (base + 1 >= len) v.y = ninf;
  if (base + 2 >= len) v.z = ninf;
  if (base + 3 >= len) v.w = ninf;
  return v;
}

__device__ __forceinline__ float Max4(const float4& v, float m) {
  return fmaxf(fmaxf(fmaxf(m, v.x), fmaxf(v.y, v.z)), v.w);
}

// exp(x - m) for visible entries, 0 for masked ones (x == -inf).
__device__ __forceinline__ float Exp1(float x, float m) {
  return x == -INFINITY ? 0.0f : expf(__fsub_rn(x, m));
}

__device__ __forceinline__ float4 Exp4(const float4& v, float m) {
  return make_float4(Exp1(v.x, m), Exp1(v.y, m), Exp1(v.z, m), Exp1(v.w, m));
}

// e / total for the visible entries of float4 number i4, 0 beyond the row's
// valid length (also when every visible entry was -inf and total is 0).
__device__ __forceinline__ float4 Div4(const float4& e, float total, int i4,
                                       int len) {
  const int b = 4 * i4;
  return make_float4(b < len ? __fdiv_rn(e.x, total) : 0.0f,
                     b + 1 < len ? __fdiv_rn(e.y, total) : 0.0f,
                     b + 2 < len ? __fdiv_rn(e.z, total) : 0.0f,
                     b + 3 < len ? __fdiv_rn(e.w, total) : 0.0f);
}

template <int NV>
__global__ void __launch_bounds__(256) SoftmaxWarpKernel(SoftmaxArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int c4 = a.cols >> 2;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
       row < a.rows; row += static_cast<int64_t>(gridDim.x) * warps) {
    bool bad;
    const int len = RowLength(a, row, &bad);
    float4* y4 = reinterpret_cast<float4*>(a.y) + static_cast<size_t>(row) * c4;
    if (bad) {
      if (lane == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_LENGTH);
      for (int i = lane; i < c4; i += 32)
        StoreStream(y4 + i, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const float4* x4 =
        reinterpret_cast<const float4*>(a.x) + static_cast<size_t>(row) * c4;
    float4 v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      v[k] = i < c4 ? LoadMasked(x4, i, len)
                    : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      m = Max4(v[k], m);
    }
    m = WarpMax(m);
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      v[k] = Exp4(v[k], m);
      total += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    total = WarpSum(total);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < c4) StoreStream(y4 + i, Div4(v[k], total, i, len));
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(1024) SoftmaxBlockKernel(SoftmaxArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float scratch[2][32];
  const int c4 = a.cols >> 2;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    bool bad;
    const int len = RowLength(a, row, &bad);
    float4* y4 = reinterpret_cast<float4*>(a.y) + static_cast<size_t>(row) * c4;
    if (bad) {
      if (threadIdx.x == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_LENGTH);
      for (int i = threadIdx.x; i < c4; i += blockDim.x)
        StoreStream(y4 + i, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const float4* x4 =
        reinterpret_cast<const float4*>(a.x) + static_cast<size_t>(row) * c4;
    float4 v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + blockDim.x * k;
      v[k] = i < c4 ? LoadMasked(x4, i, len)
                    : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      m = Max4(v[k], m);
    }
    m = BlockMax(m, scratch[0]);
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      v[k] = Exp4(v[k], m);
      total += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    total = BlockSum(total, scratch[1]);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + blockDim.x * k;
      if (i < c4) StoreStream(y4 + i, Div4(v[k], total, i, len));
    }
    // scratch[0] is rewritten by the next row's max only after every thread
    // has passed this row's sum barrier, which follows its read of
    // scratch[0]; scratch[1] likewise waits behind the next max barrier.
  }
}

__global__ void __launch_bounds__(256) SoftmaxScalarKernel(SoftmaxArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float scratch[2][32];
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    bool bad;
    const int len = RowLength(a, row, &bad);
    const float* xr = a.x + static_cast<size_t>(row) * a.cols;
    float* yr = a.y + static_cast<size_t>(row) * a.cols;
    if (bad) {
      if (threadIdx.x == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_LENGTH);
      for (int i = threadIdx.x; i < a.cols; i += blockDim.x) yr[i] = 0.0f;
      continue;
    }
    float m = -INFINITY;
    for (int i = threadIdx.x; i < len; i += blockDim.x) m = fmaxf(m, xr[i]);
    m = BlockMax(m, scratch[0]);
    float total = 0.0f;
    for (int i = threadIdx.x; i < len; i += blockDim.x)
      total += expf(__fsub_rn(xr[i], m));
    total = BlockSum(total, scratch[1]);
    // y may alias x: each index is read and written by the same thread.
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x)
      yr[i] = i < len ? __fdiv_rn(expf(__fsub_rn(xr[i], m)), total) : 0.0f;
  }
}

constexpr int64_t kMaxGrid = 1 << 24;

}  // namespace
}  // namespace mlb

extern "C" int mlb_softmax_rows_f32(const float* x, float* y, int64_t rows,
                                    int64_t cols, const int32_t* valid_len,
                                    int32_t* status, void* stream) {
  using namespace mlb;
  if (x == nullptr || y == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_softmax_rows_f32: null x or y");
  if (rows < 0 || cols <= 0 || cols > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_softmax_rows_f32: bad shape");
  if (rows == 0) return MLB_OK;
  SoftmaxArgs a{x, y, valid_len, rows, static_cast<int>(cols), status};
  cudaStream_t s = AsStream(stream);
  const bool vec = (cols % 4) == 0 && Aligned16(x) && Aligned16(y);
  const int64_t c4 = cols / 4;
  if (vec && cols <= 1024) {
    const int nv = static_cast<int>((c4 + 31) / 32);
    // up to 8 rows (warps) per CTA; fewer when rows are too few to fill
    // every SM twice
    int64_t wpc = rows / (2 * static_cast<int64_t>(SmCount()));
    wpc = wpc < 1 ? 1 : (wpc > 8 ? 8 : wpc);
    const int64_t blocks = (rows + wpc - 1) / wpc;
    const int threads = static_cast<int>(32 * wpc);
    const dim3 grid(static_cast<unsigned>(blocks < kMaxGrid ? blocks : kMaxGrid));
    switch (nv) {
#define MLB_CASE(N) \
  case N: Launch(SoftmaxWarpKernel<N>, grid, threads, 0, s, a); break;
      MLB_CASE(1) MLB_CASE(2) MLB_CASE(3) MLB_CASE(4)
      MLB_CASE(5) MLB_CASE(6) MLB_CASE(7) MLB_CASE(8)
#undef MLB_CASE
    }
    return CheckLaunch("mlb_softmax_rows_f32");
  }
  const dim3 grid(static_cast<unsigned>(rows < kMaxGrid ? rows : kMaxGrid));
  if (vec && cols <= 32768) {
    int nv = static_cast<int>((c4 + 255) / 256);
    if (nv > 8) nv = 8;
    int threads = static_cast<int>((c4 + nv - 1) / nv);
    threads = (threads + 31) / 32 * 32;
    switch (nv) {
#define MLB_CASE(N) \
  case N: Launch(SoftmaxBlockKernel<N>, grid, threads, 0, s, a); break;
      MLB_CASE(1) MLB_CASE(2) MLB_CASE(3) MLB_CASE(4)
      MLB_CASE(5) MLB_CASE(6) MLB_CASE(7) MLB_CASE(8)
#undef MLB_CASE
    }
    return CheckLaunch("mlb_softmax_rows_f32");
  }
  Launch(SoftmaxScalarKernel, grid, 256, 0, s, a);
  return CheckLaunch("mlb_softmax_rows_f32");
}
