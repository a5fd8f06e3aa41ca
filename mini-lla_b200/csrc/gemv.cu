// Quantised linear layer for decode-sized batches: y[t] = W · x[t] for t < T
// (T <= 8 per launch group), W [n, k] in the reference's ggml blocks or F32.
//
// Reference arithmetic (src/quant.cc:171-185 DotQuantizedRow, :202-226
// LinearWithBlocks; F32: src/matmul_optimized.cc:95-117): a sequential fp32
// sum of dequant(w_i) * x_i per output.  Here each block's 32 products are
// summed first and scaled once (d * Σ q_i x_i, plus m * Σ x_i for Q4_1), and
// the block sums are reduced across a warp — the same value up to rounding:
// |y - y_ref| <= 1e-5 * Σ|w_i x_i| in the tests.  The reference GPU kernels
// (cuda_matmul.cu:41-101) run one thread per output row over the whole row;
// its F32 path calls cuBLAS SGEMV (:122-133).
//
// Design (memory-bound on W at T = 1):
//   - one warp per output row, 8 rows per 256-thread CTA;
//   - the CTA walks k in chunks of kChunk = 1024 columns (32 blocks): all
//     threads stage x[:, chunk] for every token in shared memory (reused by
//     the CTA's 8 rows), each warp stages its row's 32 blocks with 16-byte
//     loads of the aligned window, and each lane decodes one block;
//   - block sums go to T fp32 accumulators per lane, reduced by shuffles.
// HBM roofline per launch: n * row_bytes (weights) + 4 * T * (k + n).
#include <climits>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kChunk = 1024;  // columns per k chunk = 32 blocks
constexpr int kWarpsPerCta = 8;
constexpr int kMaxTokens = 8;

struct GemvArgs {
  const uint8_t* w;
  int64_t n;
  int k;
  int64_t row_bytes;
  int64_t table_bytes;
  const float* x;
  float* y;
};

__device__ __forceinline__ uint32_t Smem16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

// 16-byte loads of table bytes [window, window + 16 * chunks) into dst; bytes
// past the end of the table are not read.
__device__ __forceinline__ void StageBytes(uint8_t* dst, const uint8_t* table,
                                           int64_t window, int chunks,
                                           int64_t table_bytes, int lane) {
  for (int c = lane; c < chunks; c += 32) {
    const int64_t off = window + 16 * static_cast<int64_t>(c);
    if (off + 16 <= table_bytes) {
      *reinterpret_cast<uint4*>(dst + 16 * c) =
          __ldg(reinterpret_cast<const uint4*>(table + off));
    } else {
      for (int b = 0; b < 16; ++b)
        dst[16 * c + b] = off + b < table_bytes ? table[off + b] : 0;
    }
  }
}

// Four quant values of one block (elements e..e+3), as floats.
template <int QT>
__device__ __forceinline__ float4 QuantValues(const uint8_t* blk, int e) {
  if (QT == MLB_Q8_0) {
    const uint32_t q = Smem16(blk + 2 + e) | (Smem16(blk + 4 + e) << 16);
    return make_float4(static_cast<float>(static_cast<int8_t>(q & 0xffu)),
                       static_cast<float>(static_cast<int8_t>((q >> 8) & 0xffu)),
                       static_cast<float>(static_cast<int8_t>((q >> 16) & 0xffu)),
                       static_cast<float>(static_cast<int8_t>(q >> 24)));
  }
  uint32_t q;
  if (QT == MLB_Q4_0) {
    q = Smem16(blk + 2 + (e & 15)) | (Smem16(blk + 4 + (e & 15)) << 16);
  } else {
    q = *reinterpret_cast<const uint32_t*>(blk + 4 + (e & 15));
  }
  if (e >= 16) q >>= 4;
  const float bias = QT == MLB_Q4_0 ? 8.0f : 0.0f;
  return make_float4(static_cast<float>(q & 15u) - bias,
                     static_cast<float>((q >> 8) & 15u) - bias,
                     static_cast<float>((q >> 16) & 15u) - bias,
                     static_cast<float>((q >> 24) & 15u) - bias);
}

__device__ __forceinline__ float Dot4(const float4& a, const float4& b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// Dynamic shared memory: x chunk [T][kChunk] floats, then one weight-staging
// slice of `slice` bytes per warp.
template <int QT, int T>
__global__ void __launch_bounds__(256) GemvKernel(GemvArgs a, int slice) {
  extern __shared__ __align__(16) uint8_t smem[];
  float4* xs = reinterpret_cast<float4*>(smem);
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint8_t* mine = smem + T * kChunk * 4 + warp * slice;
  const int64_t j = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + warp;
  const bool valid = j < a.n;
  const int k4 = a.k >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(a.x);
  float acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0.0f;

  for (int c0 = 0; c0 < a.k; c0 += kChunk) {
    const int cols = min(kChunk, a.k - c0);  // a multiple of 32
    const int c4 = cols >> 2;
    __syncthreads();  // the previous chunk is consumed
    for (int i = threadIdx.x; i < T * c4; i += blockDim.x) {
      const int t = i / c4;
      const int c = i - t * c4;
      xs[t * (kChunk / 4) + c] = __ldg(x4 + static_cast<int64_t>(t) * k4 + (c0 >> 2) + c);
    }
    int64_t start = 0, window = 0;
    if (QT != MLB_F32 && valid) {
      start = j * a.row_bytes + static_cast<int64_t>(c0 / 32) * kBB;
      window = start & ~int64_t{15};
      const int64_t end = start + static_cast<int64_t>(cols / 32) * kBB;
      StageBytes(mine, a.w, window, static_cast<int>((end - window + 15) >> 4),
                 a.table_bytes, lane);
    }
    __syncthreads();
    if (!valid) continue;
    if (QT == MLB_F32) {
      const float4* wrow =
          reinterpret_cast<const float4*>(a.w + j * a.row_bytes) + (c0 >> 2);
      for (int c = lane; c < c4; c += 32) {
        const float4 w = __ldg(wrow + c);
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = Dot4(w, xs[t * (kChunk / 4) + c], acc[t]);
      }
    } else {
      const uint8_t* blocks = mine + (start - window);
      for (int bl = lane; bl < (cols >> 5); bl += 32) {
        const uint8_t* blk = blocks + bl * kBB;
        const uint32_t scale = QT == MLB_Q4_1
                                   ? *reinterpret_cast<const uint32_t*>(blk)
                                   : Smem16(blk);
        float part[T], xsum[T];
#pragma unroll
        for (int t = 0; t < T; ++t) part[t] = xsum[t] = 0.0f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const float4 q = QuantValues<QT>(blk, g * 4);
#pragma unroll
          for (int t = 0; t < T; ++t) {
            const float4 xv = xs[t * (kChunk / 4) + bl * 8 + g];
            part[t] = Dot4(q, xv, part[t]);
            if (QT == MLB_Q4_1) xsum[t] += (xv.x + xv.y) + (xv.z + xv.w);
          }
        }
        const float d = Fp16BitsToF32(scale & 0xffffu);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          acc[t] = fmaf(d, part[t], acc[t]);
          if (QT == MLB_Q4_1) acc[t] = fmaf(Fp16BitsToF32(scale >> 16), xsum[t], acc[t]);
        }
      }
    }
  }
  if (!valid) return;
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const float s = WarpSum(acc[t]);
    if (lane == t) a.y[static_cast<int64_t>(t) * a.n + j] = s;
  }
}

// Any k / alignment: one thread per output element, the reference's
// sequential sum of dequant(w_i) * x_i (cuda_matmul.cu:41-101 shape).
__global__ void __launch_bounds__(256)
    GemvScalarKernel(GemvArgs a, int qt, int64_t t_rows) {
  const int64_t total = t_rows * a.n;
  const int bb = qt == MLB_Q8_0 ? 34 : (qt == MLB_Q4_0 ? 18 : 20);
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / a.n;
    const int64_t j = idx - t * a.n;
    const uint8_t* row = a.w + j * a.row_bytes;
    const float* xt = a.x + t * a.k;
    float sum = 0.0f;
    for (int i = 0; i < a.k; ++i) {
      float w;
      if (qt == MLB_F32) {
        w = reinterpret_cast<const float*>(row)[i];
      } else {
        const uint8_t* blk = row + (i >> 5) * bb;
        const int e = i & 31;
        const float d = Fp16BitsToF32(blk[0] | (blk[1] << 8));
        if (qt == MLB_Q8_0) {
          w = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[2 + e])));
        } else {
          const uint8_t* qs = blk + (qt == MLB_Q4_0 ? 2 : 4);
          const int nib = e < 16 ? (qs[e] & 15) : (qs[e - 16] >> 4);
          w = qt == MLB_Q4_0
                  ? __fmul_rn(d, static_cast<float>(nib - 8))
                  : __fadd_rn(__fmul_rn(d, static_cast<float>(nib)),
                              Fp16BitsToF32(blk[2] | (blk[3] << 8)));
        }
      }
      sum = __fadd_rn(sum, __fmul_rn(w, xt[i]));
    }
    a.y[t * a.n + j] = sum;
  }
}

template <int QT>
int LaunchVec(const GemvArgs& a, int t_rows, cudaStream_t s) {
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int slice = QT == MLB_F32 ? 0 : (32 * kBB + 15 + 15) / 16 * 16;
  const size_t shm = static_cast<size_t>(t_rows) * kChunk * 4 +
                     static_cast<size_t>(slice) * kWarpsPerCta;
  const dim3 grid(static_cast<unsigned>((a.n + kWarpsPerCta - 1) / kWarpsPerCta));
  switch (t_rows) {
#define MLB_T(N) \
  case N: GemvKernel<QT, N><<<grid, 256, shm, s>>>(a, slice); break;
    MLB_T(1) MLB_T(2) MLB_T(3) MLB_T(4) MLB_T(5) MLB_T(6) MLB_T(7) MLB_T(8)
#undef MLB_T
    default: return Fail(MLB_ERR_ARG, "mlb_linear_f32: bad token group");
  }
  return CheckLaunch("mlb_linear_f32");
}

}  // namespace
}  // namespace mlb

extern "C" int mlb_linear_f32(const void* w, int qtype, int64_t n, int64_t k,
                              const float* x, int64_t t_rows, float* y,
                              void* stream) {
  using namespace mlb;
  if (qtype < MLB_F32 || qtype > MLB_Q4_1)
    return Fail(MLB_ERR_ARG, "mlb_linear_f32: unknown qtype");
  if (n < 0 || k <= 0 || k > INT_MAX || t_rows < 0 || n > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_linear_f32: bad shape");
  if (n == 0 || t_rows == 0) return MLB_OK;
  if (w == nullptr || x == nullptr || y == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_linear_f32: null pointer");
  const uintptr_t wp = reinterpret_cast<uintptr_t>(w);
  if ((wp & (qtype == MLB_F32 || qtype == MLB_Q4_1 ? 3u : 1u)) != 0)
    return Fail(MLB_ERR_ARG, "mlb_linear_f32: weights misaligned");
  const int64_t row_bytes = mlb_row_bytes(qtype, k);
  cudaStream_t s = AsStream(stream);
  const bool vec = (k % 32) == 0 && Aligned16(x) &&
                   (qtype != MLB_F32 || (wp & 15u) == 0);
  if (!vec) {
    GemvArgs a{static_cast<const uint8_t*>(w), n, static_cast<int>(k), row_bytes,
               n * row_bytes, x, y};
    const int64_t total = n * t_rows;
    const int64_t blocks = (total + 255) / 256;
    GemvScalarKernel<<<static_cast<unsigned>(blocks < 65535 * 64 ? blocks : 65535 * 64),
                       256, 0, s>>>(a, qtype, t_rows);
    return CheckLaunch("mlb_linear_f32");
  }
  // token groups of up to kMaxTokens reuse each staged weight chunk
  for (int64_t t0 = 0; t0 < t_rows; t0 += kMaxTokens) {
    const int tg = static_cast<int>(t_rows - t0 < kMaxTokens ? t_rows - t0 : kMaxTokens);
    GemvArgs a{static_cast<const uint8_t*>(w), n, static_cast<int>(k), row_bytes,
               n * row_bytes, x + t0 * k, y + t0 * n};
    int rc = MLB_OK;
    switch (qtype) {
      case MLB_F32: rc = LaunchVec<MLB_F32>(a, tg, s); break;
      case MLB_Q8_0: rc = LaunchVec<MLB_Q8_0>(a, tg, s); break;
      case MLB_Q4_0: rc = LaunchVec<MLB_Q4_0>(a, tg, s); break;
      case MLB_Q4_1: rc = LaunchVec<MLB_Q4_1>(a, tg, s); break;
    }
    if (rc != MLB_OK) return rc;
  }
  return MLB_OK;
}
