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
//   - streaming form (x of all tokens fits in shared memory next to the
//     weight rings; k % 128 == 0; 16-byte aligned table): persistent CTAs
//     copy x once; each warp owns a contiguous run of rows and streams its
//     weight blocks in ~2 KB segments, one bulk copy (cp.async.bulk +
//     mbarrier) per segment, 3 segments ahead; products in packed fp32 pairs;
//   - chunked form otherwise: one warp per output row, 8 rows per CTA;
//     the CTA walks k in chunks of kChunk = 1024 columns (32 blocks): all
//     threads copy x[:, chunk] for every token into shared memory (reused by
//     the CTA's 8 rows), each warp copies its row's 32 blocks (the 16-byte
//     aligned window) — both with cp.async, double-buffered so that chunk
//     c + 1 is in flight while chunk c is computed;
//   - in both, lane l decodes float4 group l % 8 of block l / 8 (8 lanes per
//     block, conflict-free x reads) and block sums go to T fp32 accumulators
//     per lane, reduced by shuffles.
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

// Dynamic shared memory holds two stages; a stage is the x chunk
// [T][kChunk] floats followed by one weight slice of `slice` bytes per warp.
// Chunk c + 1 is copied in (cp.async) while chunk c is computed.
template <int QT, int T>
__global__ void __launch_bounds__(256) GemvKernel(GemvArgs a, int slice) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
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

// Packed fp32 pairs (sm_100 f32x2 instructions: two IEEE fp32 lanes per
// instruction, each rounded like its scalar form).
__device__ __forceinline__ uint64_t Pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float SumPair(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
__device__ __forceinline__ uint64_t Add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t Mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t Fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Four bytes -> two exact float pairs (the byte-permute conversion of
// BytesToFloat4 with the bias subtracted two lanes at a time).
__device__ __forceinline__ void BytesToPairs(uint32_t u, float bias, uint64_t& p01,
                                             uint64_t& p23) {
  const uint64_t nb = Pack2(-bias, -bias);
  p01 = Add2(Pack2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                   __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), nb);
  p23 = Add2(Pack2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                   __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), nb);
}

template <int QT>
__device__ __forceinline__ void QuantPairs(const uint8_t* blk, int e, uint64_t& p01,
                                           uint64_t& p23) {
  if (QT == MLB_Q8_0) {
    const uint32_t q = Smem16(blk + 2 + e) | (Smem16(blk + 4 + e) << 16);
    BytesToPairs(q ^ 0x80808080u, 8388736.0f, p01, p23);
    return;
  }
  uint32_t q;
  if (QT == MLB_Q4_0) {
    q = Smem16(blk + 2 + (e & 15)) | (Smem16(blk + 4 + (e & 15)) << 16);
  } else {
    q = *reinterpret_cast<const uint32_t*>(blk + 4 + (e & 15));
  }
  if (e >= 16) q >>= 4;
  BytesToPairs(q & 0x0F0F0F0Fu, QT == MLB_Q4_0 ? 8388616.0f : 8388608.0f, p01, p23);
}

// mbarrier + bulk-copy helpers (one elected lane issues, the warp waits).
__device__ __forceinline__ unsigned SmemAddr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void BarInit(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(SmemAddr(bar)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void BarExpectTx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(
                   SmemAddr(bar)),
               "r"(bytes)
               : "memory");
}
// One poll suspends the thread for at most ~kSuspendNs (it resumes as soon
// as the phase completes).
constexpr int kSuspendNs = 1000;
__device__ __forceinline__ bool BarTryWait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(SmemAddr(bar)), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after kWaitLimit polls, ~2 s (a copy that never
// lands must not hang the device).  A warp that gives up first waits, again
// bounded, for its copies still in flight; if one of those waits gives up
// too, the warp leaves with a copy pending into shared memory that its CTA
// no longer owns once it exits, which g_wait_abandoned records (and
// mlb_wait_timeouts reports as an error).
constexpr int kWaitLimit = 1 << 21;
__device__ __forceinline__ bool BarWait(uint64_t* bar, unsigned parity) {
  for (int i = 0; i < kWaitLimit; ++i)
    if (BarTryWait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void BulkCopy(void* dst, const void* src, unsigned bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];\n" ::"r"(SmemAddr(dst)),
      "l"(src), "r"(bytes), "r"(SmemAddr(bar))
      : "memory");
}

}  // namespace

// Waits that gave up (a bulk copy that did not land in time), and warps that
// left with copies still pending after their bounded drain; read by
// mlb_wait_timeouts.
__device__ unsigned int g_wait_timeouts;
__device__ unsigned int g_wait_abandoned;

namespace {

// Streaming form, used when x for all T tokens fits in shared memory next
// to the weight rings.  Persistent CTAs copy x once; the rows are split
// evenly over CTAs and then over each CTA's warps, so a warp owns a
// contiguous run of rows = a contiguous run of weight blocks.  The warp
// streams that run in segments of `sb` blocks (a multiple of 8, so every
// segment starts 16-byte aligned: 8 blocks are 272 / 144 / 160 bytes)
// through a ring of kBulkStages slots: lane 0 issues one bulk copy per
// segment (cp.async.bulk, completion on the slot's mbarrier) kBulkStages - 1
// segments ahead.  Lane l decodes float4 group l % 8 of block l / 8 of each
// group of 4 blocks (conflict-free x reads; the row length in blocks is a
// multiple of 4, so a group never straddles two rows) and accumulates in
// packed fp32 pairs.
constexpr int kBulkStages = 4;
constexpr int kBulkMaxWarps = 16;
constexpr int kBarBytes = kBulkMaxWarps * kBulkStages * 8;
constexpr int64_t kMaxBulkSmem = 220 * 1024;

template <int QT>
__host__ __device__ constexpr int BlockBytes() {  // bytes per 32 columns
  return QT == MLB_F32 ? 128 : (QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20));
}

// One group of 4 blocks: lane l takes float4 group l % 8 of block l / 8
// (blk already points at the lane's block, x at its x float4 of token 0).
template <int QT, int T>
__device__ __forceinline__ void BulkGroup(const uint8_t* blk, const float4* x, int k4,
                                          int lane, uint64_t (&acc)[T]) {
  if (QT == MLB_F32) {
    const float4 w = *reinterpret_cast<const float4*>(blk + (lane & 7) * 16);
    const uint64_t w01 = Pack2(w.x, w.y), w23 = Pack2(w.z, w.w);
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float4 xv = x[t * k4];
      acc[t] = Fma2(w01, Pack2(xv.x, xv.y), acc[t]);
      acc[t] = Fma2(w23, Pack2(xv.z, xv.w), acc[t]);
    }
  } else {
    uint64_t q01, q23;
    QuantPairs<QT>(blk, (lane & 7) * 4, q01, q23);
    const uint32_t scale =
        QT == MLB_Q4_1 ? *reinterpret_cast<const uint32_t*>(blk) : Smem16(blk);
    const float d = HalfBits(scale & 0xffffu);
    const uint64_t d2 = Pack2(d, d);
    const float m = QT == MLB_Q4_1 ? HalfBits(scale >> 16) : 0.0f;
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float4 xv = x[t * k4];
      const uint64_t x01 = Pack2(xv.x, xv.y), x23 = Pack2(xv.z, xv.w);
      const uint64_t p = Fma2(q23, x23, Mul2(q01, x01));
      acc[t] = Fma2(d2, p, acc[t]);
      if (QT == MLB_Q4_1) acc[t] = Fma2(Pack2(m, m), Add2(x01, x23), acc[t]);
    }
  }
}

// One group of 8 blocks for the ggml formats: lane l takes block l / 4 and
// its float4 chunks j = l % 4 and j + 4 (values 4j .. 4j + 3 and
// 16 + 4j .. 16 + 4j + 3; for Q4 both come from the same 4 code bytes).  x
// of an odd block is staged with its chunk halves swapped, so xa / xb (this
// lane's two x chunks of token 0) are conflict-free across a quarter-warp.
template <int QT, int T>
__device__ __forceinline__ void BulkGroup8(const uint8_t* blk, const float4* xa,
                                           const float4* xb, int k4, int j,
                                           uint64_t (&acc)[T]) {
  uint32_t lo, hi;  // code words of chunks j and j + 4
  float bias;
  if (QT == MLB_Q8_0) {
    lo = (Smem16(blk + 2 + 4 * j) | (Smem16(blk + 4 + 4 * j) << 16)) ^ 0x80808080u;
    hi = (Smem16(blk + 18 + 4 * j) | (Smem16(blk + 20 + 4 * j) << 16)) ^ 0x80808080u;
    bias = 8388736.0f;
  } else {
    const uint32_t u = QT == MLB_Q4_1 ? *reinterpret_cast<const uint32_t*>(blk + 4 + 4 * j)
                                      : (Smem16(blk + 2 + 4 * j) | (Smem16(blk + 4 + 4 * j) << 16));
    lo = u & 0x0F0F0F0Fu;
    hi = (u >> 4) & 0x0F0F0F0Fu;
    bias = QT == MLB_Q4_0 ? 8388616.0f : 8388608.0f;
  }
  uint64_t a01, a23, b01, b23;
  BytesToPairs(lo, bias, a01, a23);
  BytesToPairs(hi, bias, b01, b23);
  const uint32_t scale = QT == MLB_Q4_1 ? *reinterpret_cast<const uint32_t*>(blk) : Smem16(blk);
  const float d = HalfBits(scale & 0xffffu);
  const uint64_t d2 = Pack2(d, d);
  const float m = QT == MLB_Q4_1 ? HalfBits(scale >> 16) : 0.0f;
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const float4 va = xa[t * k4], vb = xb[t * k4];
    const uint64_t xa01 = Pack2(va.x, va.y), xa23 = Pack2(va.z, va.w);
    const uint64_t xb01 = Pack2(vb.x, vb.y), xb23 = Pack2(vb.z, vb.w);
    uint64_t p = Mul2(a01, xa01);
    p = Fma2(a23, xa23, p);
    p = Fma2(b01, xb01, p);
    p = Fma2(b23, xb23, p);
    acc[t] = Fma2(d2, p, acc[t]);
    if (QT == MLB_Q4_1)
      acc[t] = Fma2(Pack2(m, m), Add2(Add2(xa01, xa23), Add2(xb01, xb23)), acc[t]);
  }
}

template <int QT, int T>
__global__ void __launch_bounds__(kBulkMaxWarps * 32, 1)
    GemvBulkKernel(GemvArgs a, int sb, int slot_bytes) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int kBB = BlockBytes<QT>();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int k4 = a.k >> 2;
  const int nb = a.k >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kBulkStages;
  const float4* xs = reinterpret_cast<const float4*>(smem + kBarBytes);
  uint8_t* ring = smem + kBarBytes + static_cast<size_t>(T) * a.k * 4 +
                  static_cast<size_t>(warp) * kBulkStages * slot_bytes;

  {  // x for every token, once per CTA (ggml formats: odd blocks' chunk
     // halves swapped, see BulkGroup8)
    float4* xd = reinterpret_cast<float4*>(smem + kBarBytes);
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    for (int i = threadIdx.x; i < T * k4; i += blockDim.x)
      CopyAsync16(xd + (QT == MLB_F32 ? i : (i ^ ((i & 8) >> 1))), x4 + i);
    CopyAsyncCommit();
  }
  if (lane == 0) {
    for (int s = 0; s < kBulkStages; ++s) BarInit(bars + s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  CopyAsyncWait<0>();
  __syncthreads();

  const int64_t c0 = a.n * blockIdx.x / gridDim.x;
  const int64_t c1 = a.n * (blockIdx.x + 1) / gridDim.x;
  const int64_t w0 = c0 + (c1 - c0) * warp / warps;
  const int64_t w1 = c0 + (c1 - c0) * (warp + 1) / warps;
  if (w0 >= w1) return;
  const int64_t first = w0 * nb;               // this warp's first block
  const int64_t b0 = first & ~int64_t{7};      // segment grid start (aligned)
  const int64_t b1 = w1 * nb;
  const int nseg = static_cast<int>((b1 - b0 + sb - 1) / sb);

  auto issue = [&](int s) {
    if (lane != 0) return;
    const int64_t gb = b0 + static_cast<int64_t>(s) * sb;
    const int64_t ge = gb + sb < b1 ? gb + sb : b1;
    const int64_t start = gb * kBB;
    const int64_t bytes = (ge - gb) * kBB;
    int64_t copy = (bytes + 15) & ~int64_t{15};
    const int64_t room = (a.table_bytes - start) & ~int64_t{15};
    if (copy > room) copy = room;  // the table's last < 16 bytes: plain loads
    uint8_t* dst = ring + (s % kBulkStages) * slot_bytes;
    uint64_t* bar = bars + s % kBulkStages;
    if (copy < bytes) {
      for (int64_t b = copy; b < bytes; ++b) dst[b] = a.w[start + b];
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    BarExpectTx(bar, static_cast<unsigned>(copy));
    if (copy > 0) BulkCopy(dst, a.w + start, static_cast<unsigned>(copy), bar);
  };

  for (int s = 0; s < kBulkStages - 1 && s < nseg; ++s) issue(s);
  uint64_t acc[T], acc2[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = acc2[t] = 0;  // (+0.0f, +0.0f)
  int64_t row = w0;
  int kb = 0;  // block index of the current group inside `row`
  for (int s = 0; s < nseg; ++s) {
    if (s + kBulkStages - 1 < nseg) issue(s + kBulkStages - 1);
    if (!BarWait(bars + s % kBulkStages, (s / kBulkStages) & 1)) {
      // give up: count it, let the copies in flight land (bounded), and
      // leave NaN in the rows this warp did not finish
      if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
      const int last = s + kBulkStages - 1 < nseg ? s + kBulkStages - 1 : nseg - 1;
      bool drained = true;
      for (int r = s; r <= last; ++r)
        drained = BarWait(bars + r % kBulkStages, (r / kBulkStages) & 1) && drained;
      if (!drained && lane == 0) atomicAdd(&g_wait_abandoned, 1u);
      for (int64_t j = row; j < w1; ++j)
        if (lane < T) a.y[static_cast<int64_t>(lane) * a.n + j] = __int_as_float(0x7fc00000);
      return;
    }
    const int64_t gb = b0 + static_cast<int64_t>(s) * sb;
    const int count = static_cast<int>((gb + sb < b1 ? gb + sb : b1) - gb);
    const uint8_t* slot = ring + (s % kBulkStages) * slot_bytes;
    int b = s == 0 ? static_cast<int>(first - b0) : 0;
    while (b < count) {
      // blocks left in this segment and in the current row (multiples of 4)
      const int run = count - b < nb - kb ? count - b : nb - kb;
      int i = 0;
      if (QT == MLB_F32) {
        const uint8_t* blk = slot + (b + (lane >> 3)) * kBB;
        const float4* xg = xs + kb * 8 + lane;  // this lane's x float4
        // two independent groups of 4 blocks per step (ILP across the chains)
        for (; i + 8 <= run; i += 8) {
          BulkGroup<QT, T>(blk + i * kBB, xg + i * 8, k4, lane, acc);
          BulkGroup<QT, T>(blk + (i + 4) * kBB, xg + (i + 4) * 8, k4, lane, acc2);
        }
        if (i < run) BulkGroup<QT, T>(blk + i * kBB, xg + i * 8, k4, lane, acc);
      } else {
        // groups of 8 blocks, 4 lanes per block (kb is even here: block
        // parity = (lane / 4) & 1)
        const int j = lane & 3;
        const int par = (lane >> 2) & 1;
        const uint8_t* blk8 = slot + (b + (lane >> 2)) * kBB;
        const float4* xa = xs + (kb + (lane >> 2)) * 8 + j + 4 * par;
        const float4* xb = xs + (kb + (lane >> 2)) * 8 + j + 4 * (1 - par);
        for (; i + 16 <= run; i += 16) {
          BulkGroup8<QT, T>(blk8 + i * kBB, xa + i * 8, xb + i * 8, k4, j, acc);
          BulkGroup8<QT, T>(blk8 + (i + 8) * kBB, xa + (i + 8) * 8, xb + (i + 8) * 8, k4, j,
                            acc2);
        }
        if (i + 8 <= run) {
          BulkGroup8<QT, T>(blk8 + i * kBB, xa + i * 8, xb + i * 8, k4, j, acc);
          i += 8;
        }
        if (i < run) {  // 4 blocks left: 8 lanes per block
          const float4* xg = xs + (kb + i + (lane >> 3)) * 8 +
                             ((lane & 7) ^ (((lane >> 3) & 1) << 2));
          BulkGroup<QT, T>(slot + (b + i + (lane >> 3)) * kBB, xg, k4, lane, acc);
        }
      }
      b += run;
      kb += run;
      if (kb == nb) {
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float sum = WarpSum(SumPair(Add2(acc[t], acc2[t])));
          if (lane == t) a.y[static_cast<int64_t>(t) * a.n + row] = sum;
          acc[t] = 0;
          acc2[t] = 0;
        }
        ++row;
        kb = 0;
      }
    }
    __syncwarp();  // the slot is read by every lane before lane 0 refills it
  }
}

// Any k / alignment: one thread per output element, the reference's
// sequential sum of dequant(w_i) * x_i (cuda_matmul.cu:41-101 shape).
__global__ void __launch_bounds__(256)
    GemvScalarKernel(GemvArgs a, int qt, int64_t t_rows) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
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
int LaunchBulk(const GemvArgs& a, int warps, int sb, int slot, cudaStream_t s) {
  const size_t shm = kBarBytes + static_cast<size_t>(T) * a.k * 4 +
                     static_cast<size_t>(warps) * kBulkStages * slot;
  auto kernel = GemvBulkKernel<QT, T>;
  if (!AllowSmem(kernel, shm))
    return Fail(MLB_ERR_CUDA, "mlb_linear_f32: shared memory opt-in");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, warps * 32, shm) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  int64_t blocks = static_cast<int64_t>(per_sm) * SmCount();
  const int64_t needed = (a.n + warps - 1) / warps;  // at least a row per warp
  if (blocks > needed) blocks = needed;
  Launch(kernel, static_cast<unsigned>(blocks), warps * 32, shm, s, a, sb, slot);
  return CheckLaunch("mlb_linear_f32");
}

template <int QT>
int LaunchVec(const GemvArgs& a, int t_rows, bool bulk_ok, cudaStream_t s) {
  constexpr int kBB = BlockBytes<QT>();
  // segments of ~2 KB: 16 F32 blocks, 64 Q8_0 blocks, 128 Q4 blocks
  const int sb = QT == MLB_F32 ? 16 : (QT == MLB_Q8_0 ? 64 : 128);
  const int slot = (sb * kBB + 15) / 16 * 16;
  const int64_t x_bytes = static_cast<int64_t>(t_rows) * a.k * 4;
  // warps per CTA: enough CTAs to spread few rows over the SMs, at most 16,
  // at least 4, and all rings plus x inside the shared-memory budget
  int warps = static_cast<int>((a.n + SmCount() - 1) / SmCount());
  warps = warps < 4 ? 4 : (warps > kBulkMaxWarps ? kBulkMaxWarps : warps);
  while (warps > 4 && kBarBytes + x_bytes + int64_t{warps} * kBulkStages * slot > kMaxBulkSmem)
    --warps;
  if (bulk_ok && (a.k % 128) == 0 &&
      kBarBytes + x_bytes + int64_t{warps} * kBulkStages * slot <= kMaxBulkSmem) {
    switch (t_rows) {
      case 1: return LaunchBulk<QT, 1>(a, warps, sb, slot, s);
      case 2: return LaunchBulk<QT, 2>(a, warps, sb, slot, s);
      case 3: return LaunchBulk<QT, 3>(a, warps, sb, slot, s);
      case 4: return LaunchBulk<QT, 4>(a, warps, sb, slot, s);
      case 5: return LaunchBulk<QT, 5>(a, warps, sb, slot, s);
      case 6: return LaunchBulk<QT, 6>(a, warps, sb, slot, s);
      case 7: return LaunchBulk<QT, 7>(a, warps, sb, slot, s);
      case 8: return LaunchBulk<QT, 8>(a, warps, sb, slot, s);
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
    Launch(GemvKernel<QT, N>, grid, 256, shm, s, a, slice);              \
    break;
    MLB_T(1) MLB_T(2) MLB_T(3) MLB_T(4) MLB_T(5) MLB_T(6) MLB_T(7) MLB_T(8)
#undef MLB_T
    default: return Fail(MLB_ERR_ARG, "mlb_linear_f32: bad token group");
  }
  return CheckLaunch("mlb_linear_f32");
}

}  // namespace
}  // namespace mlb

namespace mlb {
unsigned int TcWaitTimeouts();  // linear_tc.cu
// gemv_tc.cu
int GemvTcSplit(int qtype, int count, const void* const* w, const int64_t* n, int64_t k,
                int tokens);
int GemvTc(int qtype, int count, const void* const* w, const int64_t* n, int64_t k,
           const float* x, int tokens, float* const* y, int split, cudaStream_t s);
unsigned int GemvTcWaitTimeouts();
unsigned int LinearF16WaitTimeouts();  // linear_f16.cu
unsigned int AttnTcWaitTimeouts();     // attention_tc.cu
}  // namespace mlb

namespace {
// mlb_set_gemv_path: 0 automatic, 1 CUDA cores only, 2 tensor cores where allowed
int g_gemv_path = 0;
// Automatic choice, by the launch's weight blocks (rows x k / 32, all its
// matrices): the tensor-core GEMV from kGemvTcMinBlocks1 blocks for one Q8_0
// matrix at one token (kGemvTcMinBlocks1Q4 / kGemvTcMinBlocks2Q4 for one
// 4-bit matrix at one / two tokens), from kGemvTcMinBlocks otherwise (a
// group at one token would take one CUDA-core launch per matrix).  Measured on B200, Q8_0, one
// call per weight copy in a CUDA graph (tensor cores / CUDA cores): one
// token: 14336 x 4096 18.2 / 22.2 us, 4096 x 14336 18.9 / 22.0, 11008 x 4096
// 17.4 / 17.4, 6144 x 4096 12.3 / 11.5, 4096 x 4096 9.8 / 8.6; two tokens:
// 4096 x 14336 19.3 / 32.3, 4096 x 4096 9.9 / 10.3, 2048 x 4096 11.7 / 6.9;
// four tokens: 4096 x 4096 10.1 / 14.3, 2048 x 4096 12.2 / 8.9.  The 4-bit
// formats halve the CUDA-core form's bytes but not the tensor-core form's
// per-tile cost, so one matrix stays on the CUDA cores longer: Q4_0 at one
// token 14336 x 4096 17.8 / 16.9 us, 11008 x 4096 17.5 / 13.6; at two
// tokens 6144 x 4096 12.9 / 12.4, 14336 x 4096 19.3 / 23.9 (Q4_1 alike).
constexpr int64_t kGemvTcMinBlocks1 = 1200 * 1024;
constexpr int64_t kGemvTcMinBlocks1Q4 = 2400 * 1024;
constexpr int64_t kGemvTcMinBlocks2Q4 = 1200 * 1024;
constexpr int64_t kGemvTcMinBlocks = 400 * 1024;
constexpr int kGemvTcTokens = 4;  // tokens per tensor-core pass
}  // namespace

namespace mlb {
// W[m] . x[t] for m < count, t < t_rows (< 48) on the int8 tensor cores,
// one launch per 4 tokens for all matrices, when they qualify; returns -1
// (nothing launched) when the caller should take the CUDA-core GEMV.
int GemvTcGroup(int count, const void* const* w, int qtype, const int64_t* n, int64_t k,
                const float* x, int64_t t_rows, float* const* y, cudaStream_t s) {
  if (g_gemv_path == 1 || t_rows < 1 || !Aligned16(x)) return -1;
  const int first = static_cast<int>(t_rows < kGemvTcTokens ? t_rows : kGemvTcTokens);
  if (GemvTcSplit(qtype, count, w, n, k, first) <= 0) return -1;
  if (g_gemv_path != 2) {
    int64_t rows = 0;
    for (int m = 0; m < count; ++m) rows += n[m];
    const int64_t blocks = rows * ((k + 31) / 32);
    const bool q4 = qtype != MLB_Q8_0;
    int64_t need = kGemvTcMinBlocks;
    if (count == 1 && t_rows == 1) need = q4 ? kGemvTcMinBlocks1Q4 : kGemvTcMinBlocks1;
    if (count == 1 && t_rows == 2 && q4) need = kGemvTcMinBlocks2Q4;
    if (blocks < need) return -1;
  }
  float* yy[3];
  for (int64_t t0 = 0; t0 < t_rows; t0 += kGemvTcTokens) {
    const int tg = static_cast<int>(t_rows - t0 < kGemvTcTokens ? t_rows - t0 : kGemvTcTokens);
    const int split = GemvTcSplit(qtype, count, w, n, k, tg);
    if (split <= 0) return Fail(MLB_ERR_ARG, "mlb_linear_f32: no tensor-core split");
    for (int m = 0; m < count; ++m) yy[m] = y[m] + t0 * n[m];
    const int rc = GemvTc(qtype, count, w, n, k, x + t0 * k, tg, yy, split, s);
    if (rc != MLB_OK) return rc;
  }
  return MLB_OK;
}
}  // namespace mlb

extern "C" int mlb_set_gemv_path(int path) {
  if (path < 0 || path > 2) return mlb::Fail(MLB_ERR_ARG, "mlb_set_gemv_path: bad path");
  g_gemv_path = path;
  return MLB_OK;
}

extern "C" int mlb_gemv_path(void) { return g_gemv_path; }

extern "C" int mlb_wait_timeouts(unsigned int* count) {
  using namespace mlb;
  if (count == nullptr) return Fail(MLB_ERR_ARG, "mlb_wait_timeouts: null pointer");
  unsigned int abandoned = 0;
  if (cudaMemcpyFromSymbol(count, g_wait_timeouts, sizeof(unsigned int)) != cudaSuccess ||
      cudaMemcpyFromSymbol(&abandoned, g_wait_abandoned, sizeof(unsigned int)) != cudaSuccess)
    return Fail(MLB_ERR_CUDA, "mlb_wait_timeouts: read failed");
  *count += TcWaitTimeouts() + GemvTcWaitTimeouts() + LinearF16WaitTimeouts() +
            AttnTcWaitTimeouts();
  if (abandoned != 0)
    return Fail(MLB_ERR_CUDA, "mlb_wait_timeouts: " + std::to_string(abandoned) +
                                  " warp(s) gave up with bulk copies still pending into "
                                  "shared memory; results on this device since then are "
                                  "undefined");
  return MLB_OK;
}

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
    Launch(GemvScalarKernel, static_cast<unsigned>(blocks < 65535 * 64 ? blocks : 65535 * 64), 256, 0, s, a, qtype, t_rows);
    return CheckLaunch("mlb_linear_f32");
  }
  // wide ggml matrices: int8 tensor cores, kGemvTcTokens tokens per pass
  {
    const int rc = GemvTcGroup(1, &w, qtype, &n, k, x, t_rows, &y, s);
    if (rc != -1) return rc;
  }
  // bulk copies need a 16-byte aligned table (segments start on 8-block,
  // i.e. 16-byte, boundaries of it)
  const bool bulk_ok = (wp & 15u) == 0;
  // token groups of up to kMaxTokens reuse each staged weight chunk
  for (int64_t t0 = 0; t0 < t_rows; t0 += kMaxTokens) {
    const int tg = static_cast<int>(t_rows - t0 < kMaxTokens ? t_rows - t0 : kMaxTokens);
    GemvArgs a{static_cast<const uint8_t*>(w), n, static_cast<int>(k), row_bytes,
               n * row_bytes, x + t0 * k, y + t0 * n};
    int rc = MLB_OK;
    switch (qtype) {
      case MLB_F32: rc = LaunchVec<MLB_F32>(a, tg, bulk_ok, s); break;
      case MLB_Q8_0: rc = LaunchVec<MLB_Q8_0>(a, tg, bulk_ok, s); break;
      case MLB_Q4_0: rc = LaunchVec<MLB_Q4_0>(a, tg, bulk_ok, s); break;
      case MLB_Q4_1: rc = LaunchVec<MLB_Q4_1>(a, tg, bulk_ok, s); break;
    }
    if (rc != MLB_OK) return rc;
  }
  return MLB_OK;
}
