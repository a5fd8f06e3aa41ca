// Quantised linear layer for decode-sized batches: y[t] = W · x[t] for t < T
// (T <= 8 per launch group), W [n, k] in the reference's ggml blocks or F32.
//
// Reference arithmetic (src/quant.cc:171-185 DotQuantizedRow, :202-226
// LinearWithBlocks; F32: src/matmul_optimized.cc:95-117): a sequential fp32
// sum of dequant(w_i) * x_i per output.  Here every 4 products of a block are
// summed and scaled at once (d * Σ q_i x_i, plus m * Σ x_i for Q4_1), and the
// partial sums are reduced across a warp — the same value up to rounding:
// |y - y_ref| <= 1e-5 * Σ|w_i x_i| in the tests.  The reference GPU kernels
// (cuda_matmul.cu:41-101) run one thread per output row over the whole row;
// its F32 path calls cuBLAS SGEMV (:122-133).
//
// Design (memory-bound on W at T = 1):
//   - streaming form (x of all tokens fits in 96 KB of shared memory):
//     persistent CTAs of 8 warps copy x once; each warp streams its rows in
//     1024-column segments through a 4-deep cp.async ring (no CTA barrier on
//     the weight stream);
//   - chunked form otherwise: one warp per output row, 8 rows per CTA;
//   - the CTA walks k in chunks of kChunk = 1024 columns (32 blocks): all
//     threads copy x[:, chunk] for every token into shared memory (reused by
//     the CTA's 8 rows), each warp copies its row's 32 blocks (the 16-byte
//     aligned window) — both with cp.async, double-buffered so that chunk
//     c + 1 is in flight while chunk c is computed — and lane l decodes the
//     float4 groups l, l + 32, ... (8 lanes per block, conflict-free x reads);
//   - block sums go to T fp32 accumulators per lane, reduced by shuffles.
// HBM roofline per launch: n * row_bytes (weights) + 4 * T * (k + n).
#include <climits>

#include <cuda_fp16.h>

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

// Four bytes -> four exact floats without I2F (a quarter-rate pipe): each
// byte goes into the low mantissa bits of 2^23 with a byte permute, and one
// subtract removes 2^23 (plus the byte bias).  `bias` = 2^23 + 128 for signed
// int8 stored as b ^ 0x80, 2^23 for 4-bit values, 2^23 + 8 for Q4_0's n - 8.
__device__ __forceinline__ float4 BytesToFloat4(uint32_t u, float bias) {
  return make_float4(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - bias,
                     __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - bias,
                     __int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - bias,
                     __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - bias);
}

// Four quant values of one block (elements e..e+3), as exact floats.
template <int QT>
__device__ __forceinline__ float4 QuantValues(const uint8_t* blk, int e) {
  if (QT == MLB_Q8_0) {
    const uint32_t q = Smem16(blk + 2 + e) | (Smem16(blk + 4 + e) << 16);
    return BytesToFloat4(q ^ 0x80808080u, 8388736.0f);
  }
  uint32_t q;
  if (QT == MLB_Q4_0) {
    q = Smem16(blk + 2 + (e & 15)) | (Smem16(blk + 4 + (e & 15)) << 16);
  } else {
    q = *reinterpret_cast<const uint32_t*>(blk + 4 + (e & 15));
  }
  if (e >= 16) q >>= 4;
  return BytesToFloat4(q & 0x0F0F0F0Fu, QT == MLB_Q4_0 ? 8388616.0f : 8388608.0f);
}

// fp16 scale bits -> f32 with the hardware conversion (exact for every
// non-NaN pattern; this path is checked to a tolerance, not bit for bit).
__device__ __forceinline__ float HalfBits(uint32_t bits) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}

__device__ __forceinline__ float Dot4(const float4& a, const float4& b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// 16-byte global -> shared copies that bypass registers (cp.async), so a
// lane keeps every copy of a chunk in flight at once.
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

// Dynamic shared memory holds two stages; a stage is the x chunk
// [T][kChunk] floats followed by one weight slice of `slice` bytes per warp.
// Chunk c + 1 is copied in (cp.async) while chunk c is computed.
template <int QT, int T>
__global__ void __launch_bounds__(256) GemvKernel(GemvArgs a, int slice) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int stage_bytes = T * kChunk * 4 + kWarpsPerCta * slice;
  const int64_t j = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + warp;
  const bool valid = j < a.n;
  const int k4 = a.k >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(a.x);
  const int chunks = (a.k + kChunk - 1) / kChunk;

  // Issues the copies of chunk `c` into stage `c & 1`; returns the byte
  // offset of this warp's row start inside its weight slice.
  auto stage_in = [&](int c) -> int {
    uint8_t* st = smem + (c & 1) * stage_bytes;
    const int c0 = c * kChunk;
    const int c4 = min(kChunk, a.k - c0) >> 2;
    float4* xs = reinterpret_cast<float4*>(st);
    for (int i = threadIdx.x; i < T * c4; i += blockDim.x) {
      const int t = i / c4;
      const int q = i - t * c4;
      CopyAsync16(xs + t * (kChunk / 4) + q,
                  x4 + static_cast<int64_t>(t) * k4 + (c0 >> 2) + q);
    }
    if (QT == MLB_F32 || !valid) return 0;
    uint8_t* mine = st + T * kChunk * 4 + warp * slice;
    const int64_t start = j * a.row_bytes + static_cast<int64_t>(c0 / 32) * kBB;
    const int64_t window = start & ~int64_t{15};
    const int64_t end = start + static_cast<int64_t>((c4 * 4) / 32) * kBB;
    const int n16 = static_cast<int>((end - window + 15) >> 4);
    for (int q = lane; q < n16; q += 32) {
      const int64_t off = window + 16 * static_cast<int64_t>(q);
      if (off + 16 <= a.table_bytes) {
        CopyAsync16(mine + 16 * q, a.w + off);
      } else {
        for (int b = 0; b < 16; ++b)
          mine[16 * q + b] = off + b < a.table_bytes ? a.w[off + b] : 0;
      }
    }
    return static_cast<int>(start - window);
  };

  float acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0.0f;

  int lead = stage_in(0);
  CopyAsyncCommit();
  for (int c = 0; c < chunks; ++c) {
    int next_lead = 0;
    if (c + 1 < chunks) next_lead = stage_in(c + 1);
    CopyAsyncCommit();   // (an empty group on the last chunk)
    CopyAsyncWait<1>();  // chunk c has landed for this thread ...
    __syncthreads();     // ... and for every thread of the CTA
    if (valid) {
      const uint8_t* st = smem + (c & 1) * stage_bytes;
      const float4* xs = reinterpret_cast<const float4*>(st);
      const int c0 = c * kChunk;
      const int cols = min(kChunk, a.k - c0);  // a multiple of 32
      if (QT == MLB_F32) {
        const float4* wrow =
            reinterpret_cast<const float4*>(a.w + j * a.row_bytes) + (c0 >> 2);
        for (int q = lane; q < (cols >> 2); q += 32) {
          const float4 w = __ldg(wrow + q);
#pragma unroll
          for (int t = 0; t < T; ++t) acc[t] = Dot4(w, xs[t * (kChunk / 4) + q], acc[t]);
        }
      } else {
        // Lane l takes float4 group o = l, l + 32, ...: 4 values of block
        // o / 8.  Consecutive lanes read consecutive x float4s (no bank
        // conflicts) and 8 lanes share one block's scale.
        const uint8_t* blocks = st + T * kChunk * 4 + warp * slice + lead;
        for (int o = lane; o < (cols >> 2); o += 32) {
          const uint8_t* blk = blocks + (o >> 3) * kBB;
          const float4 q = QuantValues<QT>(blk, (o & 7) * 4);
          const uint32_t scale = QT == MLB_Q4_1
                                     ? *reinterpret_cast<const uint32_t*>(blk)
                                     : Smem16(blk);
          const float d = HalfBits(scale & 0xffffu);
          const float m = QT == MLB_Q4_1 ? HalfBits(scale >> 16) : 0.0f;
#pragma unroll
          for (int t = 0; t < T; ++t) {
            const float4 xv = xs[t * (kChunk / 4) + o];
            acc[t] = fmaf(d, Dot4(q, xv, 0.0f), acc[t]);
            if (QT == MLB_Q4_1) acc[t] = fmaf(m, (xv.x + xv.y) + (xv.z + xv.w), acc[t]);
          }
        }
      }
    }
    __syncthreads();  // stage c & 1 is free for chunk c + 2
    lead = next_lead;
  }
  CopyAsyncWait<0>();
  if (!valid) return;
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const float s = WarpSum(acc[t]);
    if (lane == t) a.y[static_cast<int64_t>(t) * a.n + j] = s;
  }
}

// Streaming form, used when x for all T tokens fits in shared memory:
// persistent CTAs copy x once; then every warp walks its rows segment by
// segment (kChunk columns each) through a ring of kStages per-warp buffers
// filled by cp.async kStages - 1 segments ahead.  No CTA-wide barrier sits
// on the weight stream, so each warp keeps ~3 segments of weights in flight.
constexpr int kStages = 4;
constexpr int64_t kMaxResidentX = 96 * 1024;  // bytes of x kept in smem
constexpr int64_t kMaxStreamSmem = 200 * 1024; // whole CTA (227 KB is the cap)

template <int QT, int T>
__global__ void __launch_bounds__(256) GemvStreamKernel(GemvArgs a, int slice,
                                                        int rows_per_warp) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int k4 = a.k >> 2;
  float4* xs = reinterpret_cast<float4*>(smem);
  uint8_t* ring = smem + static_cast<size_t>(T) * a.k * 4 +
                  static_cast<size_t>(warp) * kStages * slice;
  // x for every token, once per CTA
  const float4* x4 = reinterpret_cast<const float4*>(a.x);
  for (int i = threadIdx.x; i < T * k4; i += blockDim.x) CopyAsync16(xs + i, x4 + i);
  CopyAsyncCommit();
  CopyAsyncWait<0>();
  __syncthreads();

  const int nseg = (a.k + kChunk - 1) / kChunk;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + warp) *
                       rows_per_warp;
  int64_t rows = a.n - row0;
  if (rows > rows_per_warp) rows = rows_per_warp;
  const int items = rows > 0 ? static_cast<int>(rows) * nseg : 0;

  // byte offset of item i's segment in the weight table
  auto seg_start = [&](int i) -> int64_t {
    const int64_t j = row0 + i / nseg;
    const int sg = i % nseg;
    return j * a.row_bytes + (QT == MLB_F32 ? static_cast<int64_t>(sg) * kChunk * 4
                                            : static_cast<int64_t>(sg) * 32 * kBB);
  };
  auto seg_bytes = [&](int i) -> int64_t {
    const int cols = min(kChunk, a.k - (i % nseg) * kChunk);
    return QT == MLB_F32 ? static_cast<int64_t>(cols) * 4
                         : static_cast<int64_t>(cols / 32) * kBB;
  };
  auto issue = [&](int i) {
    uint8_t* dst = ring + (i % kStages) * slice;
    const int64_t start = seg_start(i);
    const int64_t window = start & ~int64_t{15};
    const int n16 = static_cast<int>((start + seg_bytes(i) - window + 15) >> 4);
    for (int q = lane; q < n16; q += 32) {
      const int64_t off = window + 16 * static_cast<int64_t>(q);
      if (off + 16 <= a.table_bytes) {
        CopyAsync16(dst + 16 * q, a.w + off);
      } else {
        for (int b = 0; b < 16; ++b)
          dst[16 * q + b] = off + b < a.table_bytes ? a.w[off + b] : 0;
      }
    }
  };

  for (int i = 0; i < kStages - 1; ++i) {
    if (i < items) issue(i);
    CopyAsyncCommit();
  }
  float acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0.0f;
  for (int i = 0; i < items; ++i) {
    if (i + kStages - 1 < items) issue(i + kStages - 1);
    CopyAsyncCommit();
    CopyAsyncWait<kStages - 1>();  // item i's copies (this lane's) landed
    __syncwarp();                  // ... and every lane's
    const int sg = i % nseg;
    const int c4 = min(kChunk, a.k - sg * kChunk) >> 2;
    const int64_t start = seg_start(i);
    const uint8_t* seg = ring + (i % kStages) * slice + (start & 15);
    const float4* xseg = xs + sg * (kChunk / 4);
    if (QT == MLB_F32) {
      const float4* w4 = reinterpret_cast<const float4*>(seg);
      for (int o = lane; o < c4; o += 32) {
        const float4 w = w4[o];
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = Dot4(w, xseg[t * k4 + o], acc[t]);
      }
    } else {
      for (int o = lane; o < c4; o += 32) {
        const uint8_t* blk = seg + (o >> 3) * kBB;
        const float4 q = QuantValues<QT>(blk, (o & 7) * 4);
        const uint32_t scale = QT == MLB_Q4_1
                                   ? *reinterpret_cast<const uint32_t*>(blk)
                                   : Smem16(blk);
        const float d = HalfBits(scale & 0xffffu);
        const float m = QT == MLB_Q4_1 ? HalfBits(scale >> 16) : 0.0f;
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float4 xv = xseg[t * k4 + o];
          acc[t] = fmaf(d, Dot4(q, xv, 0.0f), acc[t]);
          if (QT == MLB_Q4_1) acc[t] = fmaf(m, (xv.x + xv.y) + (xv.z + xv.w), acc[t]);
        }
      }
    }
    if (sg == nseg - 1) {
      const int64_t j = row0 + i / nseg;
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float sum = WarpSum(acc[t]);
        if (lane == t) a.y[static_cast<int64_t>(t) * a.n + j] = sum;
        acc[t] = 0.0f;
      }
    }
    __syncwarp();  // the slot is read by every lane before it is refilled
  }
  CopyAsyncWait<0>();
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

// Opts a kernel in to more than 48 KB of dynamic shared memory (two stages
// of up to 8 x 4 KB of x plus 8 weight slices need up to 82 KB).
template <typename K>
bool AllowSmem(K kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return true;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(bytes)) == cudaSuccess;
}

template <int QT, int T>
int LaunchStream(const GemvArgs& a, cudaStream_t s) {
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int seg = QT == MLB_F32 ? kChunk * 4 : 32 * kBB;
  const int slice = (seg + 15 + 15) / 16 * 16;
  const size_t shm = static_cast<size_t>(T) * a.k * 4 +
                     static_cast<size_t>(kWarpsPerCta) * kStages * slice;
  auto kernel = GemvStreamKernel<QT, T>;
  if (!AllowSmem(kernel, shm))
    return Fail(MLB_ERR_CUDA, "mlb_linear_f32: shared memory opt-in");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, shm) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  // spread rows evenly: every warp gets rows_per_warp consecutive rows
  const int64_t max_warps = static_cast<int64_t>(per_sm) * SmCount() * kWarpsPerCta;
  const int64_t rows_per_warp = (a.n + max_warps - 1) / max_warps;
  const int64_t warps = (a.n + rows_per_warp - 1) / rows_per_warp;
  const int64_t blocks = (warps + kWarpsPerCta - 1) / kWarpsPerCta;
  kernel<<<static_cast<unsigned>(blocks), 256, shm, s>>>(a, slice,
                                                        static_cast<int>(rows_per_warp));
  return CheckLaunch("mlb_linear_f32");
}

template <int QT>
int LaunchVec(const GemvArgs& a, int t_rows, cudaStream_t s) {
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int64_t ring = static_cast<int64_t>(kWarpsPerCta) * kStages *
                       (((QT == MLB_F32 ? kChunk * 4 : 32 * kBB) + 30) / 16 * 16);
  const int64_t x_bytes = static_cast<int64_t>(t_rows) * a.k * 4;
  if (x_bytes <= kMaxResidentX && x_bytes + ring <= kMaxStreamSmem) {
    switch (t_rows) {
      case 1: return LaunchStream<QT, 1>(a, s);
      case 2: return LaunchStream<QT, 2>(a, s);
      case 3: return LaunchStream<QT, 3>(a, s);
      case 4: return LaunchStream<QT, 4>(a, s);
      case 5: return LaunchStream<QT, 5>(a, s);
      case 6: return LaunchStream<QT, 6>(a, s);
      case 7: return LaunchStream<QT, 7>(a, s);
      case 8: return LaunchStream<QT, 8>(a, s);
    }
  }
  const int slice = QT == MLB_F32 ? 0 : (32 * kBB + 15 + 15) / 16 * 16;
  const size_t shm = 2 * (static_cast<size_t>(t_rows) * kChunk * 4 +
                          static_cast<size_t>(slice) * kWarpsPerCta);
  const dim3 grid(static_cast<unsigned>((a.n + kWarpsPerCta - 1) / kWarpsPerCta));
  switch (t_rows) {
#define MLB_T(N)                                                     \
  case N:                                                            \
    if (!AllowSmem(GemvKernel<QT, N>, shm))                          \
      return Fail(MLB_ERR_CUDA, "mlb_linear_f32: shared memory opt-in"); \
    GemvKernel<QT, N><<<grid, 256, shm, s>>>(a, slice);              \
    break;
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
