// (Residual-add +) RMSNorm over token rows, one pass over memory.
//
// Reference arithmetic (src/ops.cc:68-81 RmsNorm, :117-124 Add, composed at
// src/forward.cc:122-124):
//   h   = x + r                                   (one fp32 add, bit-exact)
//   inv = 1.0f / sqrt(sum(h^2) / (float)n + eps)  (IEEE divide and sqrt)
//   y   = (h * inv) * w                           (two separate roundings)
// Only the order of the sum of squares differs from the reference's
// sequential loop (a warp/block tree here), which moves inv by a few 1e-7
// relative at the hidden sizes in use.
//
// Layout: x, r, h, y are [rows, cols] fp32 row-major; w is [cols].
// Kernels:
//   RmsNormWarpKernel  — cols <= 1024: one warp per row, row in registers,
//                        shuffle-only reduction, up to 8 rows per CTA.
//   RmsNormBlockKernel — cols <= 32768: one CTA per row, NV float4 per
//                        thread held in registers, warp shuffle + one smem
//                        exchange per row.
//   RmsNormClusterKernel — few rows (a decode batch, rows < 2 x SMs) with
//                        cols > 1024: a thread-block cluster of S <= 8 CTAs
//                        shares each row; every CTA reduces its column slice
//                        and pushes its partial sum of squares into the
//                        other CTAs' shared memory (one barrier), so S times
//                        more SMs work on the batch.
//   RmsNormScalarKernel— any other shape/alignment: two passes, the second
//                        re-reading the row (from L2 for realistic sizes).
// HBM roofline: 16*rows*cols + 4*cols bytes with a residual (read x, r;
// write h, y), 8*rows*cols + 4*cols without.
#include <climits>

#include <cooperative_groups.h>

#include "common.cuh"

namespace mlb {
namespace {

struct RmsArgs {
  const float* x;
  const float* res;
  float* h;
  float* y;
  const float* w;
  int64_t rows;
  int cols;
  float n_f;
  float eps;
};

// 1.0f / std::sqrt(square_sum / (float)n + eps), src/ops.cc:74-75.
__device__ __forceinline__ float InvRms(float ss, float n_f, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, n_f), eps)));
}

// x * inverse_rms * weight, left to right, src/ops.cc:78.
__device__ __forceinline__ float4 Scale(const float4& v, float inv,
                                        const float4& w) {
  return make_float4(__fmul_rn(__fmul_rn(v.x, inv), w.x),
                     __fmul_rn(__fmul_rn(v.y, inv), w.y),
                     __fmul_rn(__fmul_rn(v.z, inv), w.z),
                     __fmul_rn(__fmul_rn(v.w, inv), w.w));
}

__device__ __forceinline__ float SumSq(const float4& v, float acc) {
  acc = fmaf(v.x, v.x, acc);
  acc = fmaf(v.y, v.y, acc);
  acc = fmaf(v.z, v.z, acc);
  return fmaf(v.w, v.w, acc);
}

template <int NV, bool RES>
__global__ void __launch_bounds__(256) RmsNormWarpKernel(RmsArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int c4 = a.cols >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
       row < a.rows; row += static_cast<int64_t>(gridDim.x) * warps) {
    const size_t off = static_cast<size_t>(row) * c4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x) + off;
    float4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      v[k] = i < c4 ? LoadStream(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (RES) {
      const float4* r4 = reinterpret_cast<const float4*>(a.res) + off;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int i = lane + 32 * k;
        if (i < c4) v[k] = AddRn(v[k], LoadStream(r4 + i));
      }
      if (a.h != nullptr) {
        float4* h4 = reinterpret_cast<float4*>(a.h) + off;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int i = lane + 32 * k;
          if (i < c4) StoreStream(h4 + i, v[k]);
        }
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) ss = SumSq(v[k], ss);
    const float inv = InvRms(WarpSum(ss), a.n_f, a.eps);
    float4* y4 = reinterpret_cast<float4*>(a.y) + off;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < c4) StoreStream(y4 + i, Scale(v[k], inv, __ldg(w4 + i)));
    }
  }
}

template <int NV, bool RES>
__global__ void __launch_bounds__(1024) RmsNormBlockKernel(RmsArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float scratch[2][32];
  const int c4 = a.cols >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  int parity = 0;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const size_t off = static_cast<size_t>(row) * c4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x) + off;
    float4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + blockDim.x * k;
      v[k] = i < c4 ? LoadStream(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (RES) {
      const float4* r4 = reinterpret_cast<const float4*>(a.res) + off;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + blockDim.x * k;
        if (i < c4) v[k] = AddRn(v[k], LoadStream(r4 + i));
      }
      if (a.h != nullptr) {
        float4* h4 = reinterpret_cast<float4*>(a.h) + off;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int i = threadIdx.x + blockDim.x * k;
          if (i < c4) StoreStream(h4 + i, v[k]);
        }
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) ss = SumSq(v[k], ss);
    const float inv = InvRms(BlockSum(ss, scratch[parity]), a.n_f, a.eps);
    parity ^= 1;
    float4* y4 = reinterpret_cast<float4*>(a.y) + off;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + blockDim.x * k;
      if (i < c4) StoreStream(y4 + i, Scale(v[k], inv, __ldg(w4 + i)));
    }
  }
}

// barrier.cluster in its two halves: Arrive marks this thread's arrival
// (relaxed: nothing to publish yet, or release: its shared-memory writes to
// other CTAs are published), Wait blocks until every thread of every CTA in
// the cluster has arrived (acquire).
__device__ __forceinline__ void ClusterArriveRelaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void ClusterArriveRelease() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void ClusterWait() {
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

// One row per cluster (blockIdx.x = row), S = cluster size CTAs along y.
// CTA rank r owns float4 columns [r*chunk, min((r+1)*chunk, c4)), NV per
// thread; its weight slice is loaded with the row.  Each CTA pushes its
// partial sum of squares into slot r of every CTA's `partials`, so one
// barrier delivers them all and no CTA reads another's memory afterwards
// (it may then exit at once).  A first barrier phase, arrived at on entry
// and waited on only before the pushes, guarantees that every CTA of the
// cluster is running when its shared memory is written.  The partials are
// summed in rank order (deterministic).
template <int NV, bool RES>
__global__ void __launch_bounds__(256) RmsNormClusterKernel(RmsArgs a, int chunk) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  ClusterArriveRelaxed();  // this CTA has started
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float scratch[32];
  __shared__ float partials[8];
  const int c4 = a.cols >> 2;
  const int rank = static_cast<int>(cluster.block_rank());
  const int ranks = static_cast<int>(cluster.num_blocks());
  const int c_begin = rank * chunk;
  const int c_end = min(c4, c_begin + chunk);
  const int64_t row = blockIdx.x;
  const size_t off = static_cast<size_t>(row) * c4;
  const float4* x4 = reinterpret_cast<const float4*>(a.x) + off;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  float4 v[NV], wv[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = c_begin + threadIdx.x + blockDim.x * k;
    v[k] = i < c_end ? LoadStream(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[k] = i < c_end ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (RES) {
    const float4* r4 = reinterpret_cast<const float4*>(a.res) + off;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = c_begin + threadIdx.x + blockDim.x * k;
      if (i < c_end) v[k] = AddRn(v[k], LoadStream(r4 + i));
    }
    if (a.h != nullptr) {
      float4* h4 = reinterpret_cast<float4*>(a.h) + off;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int i = c_begin + threadIdx.x + blockDim.x * k;
        if (i < c_end) StoreStream(h4 + i, v[k]);
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) ss = SumSq(v[k], ss);
  ss = BlockSum(ss, scratch);
  ClusterWait();  // every CTA of the cluster has started
  if (static_cast<int>(threadIdx.x) < ranks)
    *cluster.map_shared_rank(&partials[rank], static_cast<int>(threadIdx.x)) = ss;
  ClusterArriveRelease();
  ClusterWait();  // every CTA's partial is in this CTA's `partials`
  float total = 0.0f;
  for (int r = 0; r < ranks; ++r) total += partials[r];
  const float inv = InvRms(total, a.n_f, a.eps);
  float4* y4 = reinterpret_cast<float4*>(a.y) + off;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = c_begin + threadIdx.x + blockDim.x * k;
    if (i < c_end) StoreStream(y4 + i, Scale(v[k], inv, wv[k]));
  }
}

template <bool RES>
__global__ void __launch_bounds__(256) RmsNormScalarKernel(RmsArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float scratch[2][32];
  int parity = 0;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const size_t off = static_cast<size_t>(row) * a.cols;
    const float* xr = a.x + off;
    const float* rr = RES ? a.res + off : nullptr;
    float* hr = (RES && a.h != nullptr) ? a.h + off : nullptr;
    float* yr = a.y + off;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) {
      float v = xr[i];
      if (RES) {
        v = __fadd_rn(v, rr[i]);
        if (hr != nullptr) hr[i] = v;
      }
      ss = fmaf(v, v, ss);
    }
    const float inv = InvRms(BlockSum(ss, scratch[parity]), a.n_f, a.eps);
    parity ^= 1;
    // Each thread revisits exactly the indices it wrote in the first loop.
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) {
      float v;
      if (RES) {
        v = hr != nullptr ? hr[i] : __fadd_rn(xr[i], rr[i]);
      } else {
        v = xr[i];
      }
      yr[i] = __fmul_rn(__fmul_rn(v, inv), a.w[i]);
    }
  }
}

constexpr int64_t kMaxGrid = 1 << 24;

// Warps per CTA for the warp-per-row kernels: 8 when there are rows enough
// to fill every SM twice over, fewer for small batches so that the rows
// spread over more SMs (256 rows at cols 896 -> 256 one-warp CTAs).
int WarpsPerCta(int64_t rows) {
  const int64_t fill = 2 * static_cast<int64_t>(SmCount());
  int64_t w = rows / fill;
  if (w < 1) w = 1;
  if (w > 8) w = 8;
  return static_cast<int>(w);
}

template <bool RES>
int LaunchWarp(const RmsArgs& a, int nv, cudaStream_t s) {
  const int wpc = WarpsPerCta(a.rows);
  const int threads = 32 * wpc;
  const int64_t blocks = (a.rows + wpc - 1) / wpc;
  const dim3 grid(static_cast<unsigned>(blocks < kMaxGrid ? blocks : kMaxGrid));
  switch (nv) {
#define MLB_CASE(N) \
  case N: Launch(RmsNormWarpKernel<N, RES>, grid, threads, 0, s, a); break;
    MLB_CASE(1) MLB_CASE(2) MLB_CASE(3) MLB_CASE(4)
    MLB_CASE(5) MLB_CASE(6) MLB_CASE(7) MLB_CASE(8)
#undef MLB_CASE
    default: return Fail(MLB_ERR_ARG, "rmsnorm: bad warp width");
  }
  return CheckLaunch("mlb_rmsnorm_f32");
}

template <bool RES>
int LaunchBlock(const RmsArgs& a, int nv, int threads, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.rows < kMaxGrid ? a.rows : kMaxGrid));
  switch (nv) {
#define MLB_CASE(N) \
  case N: Launch(RmsNormBlockKernel<N, RES>, grid, threads, 0, s, a); break;
    MLB_CASE(1) MLB_CASE(2) MLB_CASE(3) MLB_CASE(4)
    MLB_CASE(5) MLB_CASE(6) MLB_CASE(7) MLB_CASE(8)
#undef MLB_CASE
    default: return Fail(MLB_ERR_ARG, "rmsnorm: bad block width");
  }
  return CheckLaunch("mlb_rmsnorm_f32");
}

// Few long rows: a cluster of `ranks` CTAs per row (rows <= 65535 so the
// row index fits blockIdx.x of a y-clustered grid).
template <bool RES>
int LaunchCluster(const RmsArgs& a, int ranks, cudaStream_t s) {
  const int c4 = a.cols / 4;
  const int chunk = (c4 + ranks - 1) / ranks;
  int nv = (chunk + 255) / 256;
  int threads = (chunk + nv - 1) / nv;
  threads = (threads + 31) / 32 * 32;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(a.rows), static_cast<unsigned>(ranks), 1);
  config.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  config.dynamicSmemBytes = 0;
  config.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(ranks);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see Launch
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = LaunchOverlap() ? 2 : 1;
  cudaError_t err = cudaErrorInvalidValue;
  switch (nv) {
    case 1: err = cudaLaunchKernelEx(&config, RmsNormClusterKernel<1, RES>, a, chunk); break;
    case 2: err = cudaLaunchKernelEx(&config, RmsNormClusterKernel<2, RES>, a, chunk); break;
    case 3: err = cudaLaunchKernelEx(&config, RmsNormClusterKernel<3, RES>, a, chunk); break;
    case 4: err = cudaLaunchKernelEx(&config, RmsNormClusterKernel<4, RES>, a, chunk); break;
    default: return Fail(MLB_ERR_ARG, "rmsnorm: bad cluster width");
  }
  if (err != cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, std::string("mlb_rmsnorm_f32: ") + cudaGetErrorString(err));
  }
  return CheckLaunch("mlb_rmsnorm_f32");
}

template <bool RES>
int LaunchScalar(const RmsArgs& a, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.rows < kMaxGrid ? a.rows : kMaxGrid));
  Launch(RmsNormScalarKernel<RES>, grid, 256, 0, s, a);
  return CheckLaunch("mlb_rmsnorm_f32");
}

}  // namespace
}  // namespace mlb

extern "C" int mlb_rmsnorm_f32(const float* x, const float* residual,
                               float* h_out, float* y, const float* w,
                               int64_t rows, int64_t cols, float eps,
                               void* stream) {
  using namespace mlb;
  if (x == nullptr || y == nullptr || w == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_rmsnorm_f32: null x, y or w");
  if (rows < 0 || cols <= 0 || cols > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_rmsnorm_f32: bad shape");
  if (rows == 0) return MLB_OK;
  RmsArgs a{x, residual, residual != nullptr ? h_out : nullptr, y, w, rows,
            static_cast<int>(cols), static_cast<float>(cols), eps};
  const bool res = residual != nullptr;
  bool vec = (cols % 4) == 0 && Aligned16(x) && Aligned16(y) && Aligned16(w);
  if (res) vec = vec && Aligned16(residual);
  if (a.h != nullptr) vec = vec && Aligned16(a.h);
  cudaStream_t s = AsStream(stream);
  const int64_t c4 = cols / 4;
  if (vec && cols <= 1024) {
    const int nv = static_cast<int>((c4 + 31) / 32);
    return res ? LaunchWarp<true>(a, nv, s) : LaunchWarp<false>(a, nv, s);
  }
  // few long rows: spread each row over a cluster of up to 8 CTAs
  const int64_t fill = 2 * static_cast<int64_t>(SmCount());
  if (vec && cols > 1024 && cols <= 32768 && rows < fill) {
    int64_t ranks = (fill + rows - 1) / rows;
    if (ranks > 8) ranks = 8;  // portable cluster size
    // each CTA holds at most 1024 float4s of its row (4 per thread x 256)
    if (ranks > 1 && (c4 + ranks - 1) / ranks <= 1024) {
      const int r = static_cast<int>(ranks);
      return res ? LaunchCluster<true>(a, r, s) : LaunchCluster<false>(a, r, s);
    }
  }
  if (vec && cols <= 32768) {
    int nv = static_cast<int>((c4 + 255) / 256);
    if (nv > 8) nv = 8;
    int threads = static_cast<int>((c4 + nv - 1) / nv);
    threads = (threads + 31) / 32 * 32;
    return res ? LaunchBlock<true>(a, nv, threads, s)
               : LaunchBlock<false>(a, nv, threads, s);
  }
  return res ? LaunchScalar<true>(a, s) : LaunchScalar<false>(a, s);
}
