// Token-embedding gather with in-register ggml block dequantisation.
//
// Reference arithmetic (src/forward.cc:29-33 Embedding -> src/quant.cc:278-304
// DequantizeRow -> :187-199 -> :148-167 DequantizeElement, fp16 decode
// :44-71):
//   F32 : copy
//   Q8_0: f16(d) * (float)qs[i]
//   Q4_0: f16(d) * (float)(nib - 8), nib = i < 16 ? qs[i] & 15 : qs[i-16] >> 4
//   Q4_1: f16(d) * (float)nib + f16(m)
// Every product is exact in fp32 and the Q4_1 add is one IEEE rounding
// (__fadd_rn, never contracted into an FMA), so the output is bit-exact.
//
// Block layouts (quantized_tensor.h:19-35): Q8_0 {u16 d; i8 qs[32]} 34 B,
// Q4_0 {u16 d; u8 qs[16]} 18 B, Q4_1 {u16 d, m; u8 qs[16]} 20 B.  A table row
// is ceil(cols/32) blocks, so rows are only 2-byte aligned in general
// (cols = 896, Q8_0: 952 B per row).
//
// Kernels (cols % 4 == 0, 16-byte aligned output): two token rows per CTA
// (one warp per row when rows are short).  Quantised tables stage each row's
// bytes in shared memory — the 16-byte-aligned window of the table's address
// space that covers the row, copied with cp.async — and decode float4s (4
// consecutive values of one block) from there; F32 tables copy the row with
// float4 loads.  Output stores are 16-byte and fully coalesced.  Any other
// shape takes the scalar kernel (one value per thread).
// HBM roofline per row: row_bytes read + 4 * cols written (+ 4 for the id).
#include <climits>

#include <cuda_fp16.h>

#include "common.cuh"

namespace mlb {
namespace {

// Rows up to this many bytes are staged one per warp when there are rows
// enough to fill every SM (B200 sweep: Q8_0 at cols 2048 1.08 vs 0.79 of the
// copy peak, Q4_1 at cols 4096 1.03 vs 0.88; Q8_0 at cols 4096 — 4352-byte
// rows — is faster one row per CTA).
constexpr int64_t kWarpRowBytes = 2560;

// Largest staged window of one row (bytes of dynamic shared memory per row;
// two rows per CTA stay under the 48 KB available without an opt-in): Q8_0
// rows up to cols ~ 22000.  Longer rows are split over several CTAs.
constexpr int64_t kMaxStagedBytes = 24 * 1024;

struct EmbArgs {
  const uint8_t* table;
  int64_t vocab;
  int cols;
  int64_t row_bytes;
  const int32_t* tokens;  // NULL: every row gathers `token`
  int32_t token;
  int64_t rows;
  float* out;
  int32_t* status;
};

__device__ __forceinline__ uint32_t LoadU16(const uint8_t* p) {
  return __ldg(reinterpret_cast<const unsigned short*>(p));
}

__device__ __forceinline__ uint32_t Smem16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

// fp16 bits -> fp32 by the hardware conversion, which is exact for every
// finite, infinite and subnormal input — the value quant.cc:44-71 computes.
// (A NaN scale's payload may differ, but every product or sum of it is the
// GPU's canonical NaN either way.)
__device__ __forceinline__ float HalfBits(uint32_t bits) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}

// Byte j (selector 0x7540 + j) of `codes` as an exact float: the byte goes
// into the low mantissa bits of 2^23 (0x4B000000) and `bias` = 2^23 + offset
// is subtracted (offset 128 for int8 codes stored ^ 0x80, 8 for Q4_0
// nibbles, 0 for Q4_1).  No int->float conversion instruction is needed.
__device__ __forceinline__ float CodeAt(uint32_t codes, uint32_t sel, float bias) {
  return __fsub_rn(__uint_as_float(__byte_perm(codes, 0x4B000000u, sel)), bias);
}

// Decodes output float4 number o of a row (block b = o / 8, values e..e+3
// with e = (o % 8) * 4) from the row's bytes staged in shared memory.  The
// staged copy keeps the table's address modulo 16, so block starts are
// 2-byte aligned (Q8_0, Q4_0: 34 B and 18 B blocks) or 4-byte aligned (Q4_1:
// 20 B blocks, 4-byte aligned tables): the scale and the four code bytes are
// read as u16 + two u16 (Q8_0, Q4_0) or two u32 (Q4_1) shared loads.
template <int QT>
__device__ __forceinline__ float4 DecodeStaged(const uint8_t* row, int o) {
  const int e = (o & 7) << 2;
  if (QT == MLB_Q8_0) {
    const uint8_t* blk = row + (o >> 3) * 34;
    const float d = HalfBits(Smem16(blk));
    const uint32_t q = (Smem16(blk + 2 + e) | (Smem16(blk + 4 + e) << 16)) ^ 0x80808080u;
    return make_float4(__fmul_rn(d, CodeAt(q, 0x7540, 8388736.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7541, 8388736.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7542, 8388736.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7543, 8388736.0f)));
  }
  uint32_t scale, q;
  if (QT == MLB_Q4_0) {
    const uint8_t* blk = row + (o >> 3) * 18;
    scale = Smem16(blk);
    q = Smem16(blk + 2 + (e & 15)) | (Smem16(blk + 4 + (e & 15)) << 16);
  } else {
    const uint8_t* blk = row + (o >> 3) * 20;
    scale = *reinterpret_cast<const uint32_t*>(blk);               // d | m << 16
    q = *reinterpret_cast<const uint32_t*>(blk + 4 + (e & 15));
  }
  if (e >= 16) q >>= 4;  // the last 16 values sit in the high nibbles
  q &= 0x0F0F0F0Fu;
  const float d = HalfBits(scale & 0xffffu);
  if (QT == MLB_Q4_0) {  // d * (nib - 8); nib - 8 is exact
    return make_float4(__fmul_rn(d, CodeAt(q, 0x7540, 8388616.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7541, 8388616.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7542, 8388616.0f)),
                       __fmul_rn(d, CodeAt(q, 0x7543, 8388616.0f)));
  }
  const float m = HalfBits(scale >> 16);
  return make_float4(__fadd_rn(__fmul_rn(d, CodeAt(q, 0x7540, 8388608.0f)), m),
                     __fadd_rn(__fmul_rn(d, CodeAt(q, 0x7541, 8388608.0f)), m),
                     __fadd_rn(__fmul_rn(d, CodeAt(q, 0x7542, 8388608.0f)), m),
                     __fadd_rn(__fmul_rn(d, CodeAt(q, 0x7543, 8388608.0f)), m));
}

// The table's address range [lo, hi).  A staged window starts at a 16-byte
// boundary of the address space, so it may begin before the table (a table
// that is only 2-byte aligned) or end after it (the last row); only bytes
// inside the range are ever read.
struct TableSpan {
  uintptr_t lo, hi;
};

// Copies window chunks [first, chunks) stepping by `step` (16 bytes each,
// starting at address `win`) into dst: whole in-table chunks with cp.async
// (ASYNC) or one 16-byte load each, the in-table bytes of a chunk that
// straddles the table's start or end one by one.  With ASYNC the caller
// commits and waits for the copies.
template <bool ASYNC>
__device__ __forceinline__ void StageWindow(uint8_t* dst, uintptr_t win, int chunks,
                                            TableSpan span, int first, int step) {
  for (int c = first; c < chunks; c += step) {
    const uintptr_t p = win + 16 * static_cast<uintptr_t>(c);
    if (p >= span.lo && p + 16 <= span.hi) {
      if (ASYNC) CopyAsync16(dst + 16 * c, reinterpret_cast<const void*>(p));
      else
        *reinterpret_cast<uint4*>(dst + 16 * c) = __ldg(reinterpret_cast<const uint4*>(p));
    } else {
      for (int b = 0; b < 16; ++b)
        if (p + b >= span.lo && p + b < span.hi)
          dst[16 * c + b] = *reinterpret_cast<const uint8_t*>(p + b);
    }
  }
}

// Quantised tables, R token rows per CTA iteration: the CTA copies the R
// rows' windows into shared memory (cp.async, every copy of the R rows in
// flight at once), waits, then decodes float4s from shared memory and
// streams them out.  (Measured on B200, Q8_0 [128256, 4096], 16384 random
// tokens: 0.054 ms alone = 0.98 of the copy peak with R = 2; one row per CTA
// with 16-byte register loads 0.062 ms; four rows per CTA, a warp-specialised
// ring of bulk copies, and bulk-copy stores of the decoded rows were all
// slower than R = 2.)
// With few tokens (a decode batch) each row is split over gridDim.y CTAs of
// `per_cta` output float4s each (a multiple of 8: whole blocks); a CTA stages
// only the blocks it decodes.  `slice` = shared bytes per staged row.
template <int QT, int R>
__global__ void __launch_bounds__(256) EmbeddingStagedKernel(EmbArgs a, TableSpan span,
                                                             int per_cta, int slice) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  extern __shared__ __align__(16) uint8_t staged[];
  constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
  const int groups = a.cols >> 2;
  const int g0 = blockIdx.y * per_cta;
  const int g1 = min(groups, g0 + per_cta);
  if (g0 >= groups) return;
  const int b0 = g0 >> 3;             // first block of this CTA
  const int b1 = (g1 + 7) >> 3;       // one past its last block
  for (int64_t t0 = static_cast<int64_t>(blockIdx.x) * R; t0 < a.rows;
       t0 += static_cast<int64_t>(gridDim.x) * R) {
    uintptr_t first[R];  // address of block b0 of each row; 0: no valid row
    __syncthreads();     // the previous rows' decode is done with `staged`
#pragma unroll
    for (int r = 0; r < R; ++r) {
      first[r] = 0;
      const int64_t t = t0 + r;
      if (t >= a.rows) continue;
      const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
      if (token < 0 || token >= a.vocab) continue;
      first[r] = span.lo + static_cast<uint64_t>(token) * a.row_bytes +
                 static_cast<uint64_t>(b0) * kBB;
      const uintptr_t end = first[r] + static_cast<uint64_t>(b1 - b0) * kBB;
      const uintptr_t win = first[r] & ~uintptr_t{15};
      const int chunks = static_cast<int>((end - win + 15) >> 4);
      StageWindow<true>(staged + r * slice, win, chunks, span, threadIdx.x, blockDim.x);
    }
    CopyAsyncCommit();
    CopyAsyncWait<0>();
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t t = t0 + r;
      if (t >= a.rows) continue;
      float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
      if (first[r] == 0) {  // id outside the table: zero row, status bit
        if (threadIdx.x == 0 && blockIdx.y == 0 && a.status != nullptr)
          atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
        for (int o = g0 + threadIdx.x; o < g1; o += blockDim.x)
          StoreStream(out + o, make_float4(0.f, 0.f, 0.f, 0.f));
        continue;
      }
      // `row` addresses block 0 of the row; only blocks [b0, b1) are staged
      const uint8_t* row = staged + r * slice + (first[r] & 15) -
                           static_cast<int64_t>(b0) * kBB;
      for (int o = g0 + threadIdx.x; o < g1; o += blockDim.x)
        StoreStream(out + o, DecodeStaged<QT>(row, o));
    }
  }
}

// Short rows (cols <= 1024, or rows of at most kWarpRowBytes in a large
// batch): one warp per token row, up to 8 rows per CTA, each warp staging its
// own row in its slice of shared memory (`slice` bytes) — a CTA per short
// row would be mostly launch and barrier overhead.
template <int QT>
__global__ void __launch_bounds__(256) EmbeddingStagedWarpKernel(EmbArgs a, TableSpan span,
                                                                 int slice) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  extern __shared__ __align__(16) uint8_t staged[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int groups = a.cols >> 2;
  uint8_t* mine = staged + warp * slice;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * warps + warp; t < a.rows;
       t += static_cast<int64_t>(gridDim.x) * warps) {
    const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
    float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
    if (token < 0 || token >= a.vocab) {
      if (lane == 0 && a.status != nullptr) atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
      for (int o = lane; o < groups; o += 32)
        StoreStream(out + o, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const uintptr_t start = span.lo + static_cast<uint64_t>(token) * a.row_bytes;
    const uintptr_t win = start & ~uintptr_t{15};
    const int chunks = static_cast<int>((start + a.row_bytes - win + 15) >> 4);
    __syncwarp();  // the previous row's decode is done with `mine`
    StageWindow<false>(mine, win, chunks, span, lane, 32);
    __syncwarp();
    const uint8_t* row = mine + (start & 15);
    for (int o = lane; o < groups; o += 32)
      StoreStream(out + o, DecodeStaged<QT>(row, o));
  }
}

// F32 tables with 16-byte aligned rows: a plain row copy, one CTA per token.
__global__ void __launch_bounds__(256) EmbeddingF32Kernel(EmbArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int groups = a.cols >> 2;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
    float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
    const bool ok = token >= 0 && token < a.vocab;
    if (!ok && threadIdx.x == 0 && a.status != nullptr)
      atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
    const float4* src = reinterpret_cast<const float4*>(
        a.table + static_cast<size_t>(ok ? token : 0) * a.row_bytes);
    for (int o = threadIdx.x; o < groups; o += blockDim.x)
      StoreStream(out + o, ok ? __ldg(src + o) : make_float4(0.f, 0.f, 0.f, 0.f));
  }
}

__device__ __forceinline__ float DecodeOne(int qt, const uint8_t* row, int i) {
  if (qt == MLB_F32) {
    float v;
    memcpy(&v, row + 4 * static_cast<size_t>(i), 4);
    return v;
  }
  const int b = i >> 5;
  const int e = i & 31;
  if (qt == MLB_Q8_0) {
    const uint8_t* blk = row + b * 34;
    return __fmul_rn(Fp16BitsToF32(LoadU16(blk)),
                     static_cast<float>(static_cast<int8_t>(blk[2 + e])));
  }
  const uint8_t* blk = row + b * (qt == MLB_Q4_0 ? 18 : 20);
  const uint8_t* qs = blk + (qt == MLB_Q4_0 ? 2 : 4);
  const int nib = e < 16 ? (qs[e] & 15) : (qs[e - 16] >> 4);
  const float d = Fp16BitsToF32(LoadU16(blk));
  if (qt == MLB_Q4_0) return __fmul_rn(d, static_cast<float>(nib - 8));
  return __fadd_rn(__fmul_rn(d, static_cast<float>(nib)),
                   Fp16BitsToF32(LoadU16(blk + 2)));
}

__global__ void __launch_bounds__(256) EmbeddingScalarKernel(EmbArgs a, int qt) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int32_t token = a.tokens != nullptr ? a.tokens[t] : a.token;
    float* out = a.out + static_cast<size_t>(t) * a.cols;
    if (token < 0 || token >= a.vocab) {
      if (threadIdx.x == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
      for (int i = threadIdx.x; i < a.cols; i += blockDim.x) out[i] = 0.0f;
      continue;
    }
    const uint8_t* row = a.table + static_cast<size_t>(token) * a.row_bytes;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x)
      out[i] = DecodeOne(qt, row, i);
  }
}

}  // namespace
}  // namespace mlb

namespace mlb {
namespace {

int LaunchEmbedding(const void* table, int qtype, int64_t vocab, int64_t cols,
                    const int32_t* tokens, int32_t token, int64_t rows,
                    float* out, int32_t* status, void* stream, const char* op) {
  if (qtype < MLB_F32 || qtype > MLB_Q4_1)
    return Fail(MLB_ERR_ARG, std::string(op) + ": unknown qtype");
  if (rows < 0 || cols <= 0 || cols > INT_MAX || vocab < 0 || vocab > INT_MAX)
    return Fail(MLB_ERR_ARG, std::string(op) + ": bad shape");
  if (rows == 0) return MLB_OK;
  if (table == nullptr || out == nullptr)
    return Fail(MLB_ERR_ARG, std::string(op) + ": null pointer");
  const uintptr_t tbl = reinterpret_cast<uintptr_t>(table);
  if (qtype != MLB_F32 && (tbl & (qtype == MLB_Q4_1 ? 3u : 1u)) != 0)
    return Fail(MLB_ERR_ARG, std::string(op) + ": table misaligned");
  if (qtype == MLB_F32 && (tbl & 3u) != 0)
    return Fail(MLB_ERR_ARG, std::string(op) + ": table misaligned");
  EmbArgs a{static_cast<const uint8_t*>(table), vocab, static_cast<int>(cols),
            mlb_row_bytes(qtype, cols), tokens, token, rows, out, status};
  const int64_t cap = 1 << 24;
  const dim3 grid(static_cast<unsigned>(rows < cap ? rows : cap));
  const int groups = static_cast<int>(cols / 4);
  int threads = groups < 256 ? (groups + 31) / 32 * 32 : 256;
  if (threads < 32) threads = 32;
  cudaStream_t s = AsStream(stream);
  const int64_t row_bytes = a.row_bytes;
  const bool vec = (cols % 4) == 0 && Aligned16(out);
  const TableSpan span{tbl, tbl + static_cast<uintptr_t>(vocab * row_bytes)};
  const int bb = qtype == MLB_Q8_0 ? 34 : (qtype == MLB_Q4_0 ? 18 : 20);
  // Rows split over CTAs when tokens cannot fill every SM twice, or when a
  // row's window would not fit kMaxStagedBytes; each CTA takes a whole
  // number of blocks (8 float4s per block).
  const int64_t fill = 2 * static_cast<int64_t>(SmCount());
  const int64_t blocks_per_row = (groups + 7) / 8;
  int64_t split = rows < fill ? (fill + rows - 1) / rows : 1;
  const int64_t max_blocks = (kMaxStagedBytes - 30) / bb;
  if (split < (blocks_per_row + max_blocks - 1) / max_blocks)
    split = (blocks_per_row + max_blocks - 1) / max_blocks;
  if (split > blocks_per_row) split = blocks_per_row;
  if (split < 1) split = 1;
  const int64_t per_cta = (blocks_per_row + split - 1) / split * 8;
  split = (groups + per_cta - 1) / per_cta;
  // staged window of one row: up to 15 leading bytes + the CTA's blocks,
  // rounded up to 16
  const int slice = static_cast<int>((per_cta / 8 * bb + 15 + 15) / 16 * 16);
  if (vec && qtype == MLB_F32 && (tbl & 15u) == 0) {
    Launch(EmbeddingF32Kernel, grid, threads, 0, s, a);
  } else if (vec && qtype != MLB_F32 &&
             (cols <= 1024 || (rows >= fill && row_bytes <= kWarpRowBytes))) {
    // warp per row; 8 rows per CTA unless rows are too few to fill the SMs
    int64_t wpc = rows / fill;
    wpc = wpc < 1 ? 1 : (wpc > 8 ? 8 : wpc);
    const int wslice = static_cast<int>((row_bytes + 15 + 15) / 16 * 16);
    const int64_t nblk = (rows + wpc - 1) / wpc;
    const dim3 wgrid(static_cast<unsigned>(nblk < cap ? nblk : cap));
    const int wthreads = static_cast<int>(32 * wpc);
    const size_t shm = static_cast<size_t>(wslice) * wpc;
    switch (qtype) {
      case MLB_Q8_0:
        Launch(EmbeddingStagedWarpKernel<MLB_Q8_0>, wgrid, wthreads, shm, s, a, span, wslice);
        break;
      case MLB_Q4_0:
        Launch(EmbeddingStagedWarpKernel<MLB_Q4_0>, wgrid, wthreads, shm, s, a, span, wslice);
        break;
      case MLB_Q4_1:
        Launch(EmbeddingStagedWarpKernel<MLB_Q4_1>, wgrid, wthreads, shm, s, a, span, wslice);
        break;
    }
  } else if (vec && qtype != MLB_F32) {
    // two rows per CTA once the halved grid still fills every SM's eight
    // CTA slots (2 x 4 x fill rows)
    const bool two = split == 1 && rows >= 8 * fill;
    const int64_t nrow = two ? (rows + 1) / 2 : rows;
    const dim3 grid2(static_cast<unsigned>(nrow < cap ? nrow : cap),
                     static_cast<unsigned>(split));
    const size_t shm = static_cast<size_t>(slice) * (two ? 2 : 1);
    int cta_threads = per_cta < 256 ? static_cast<int>((per_cta + 31) / 32 * 32) : 256;
    if (cta_threads > threads) cta_threads = threads;
    const int pc = static_cast<int>(per_cta);
    switch (qtype) {
      case MLB_Q8_0:
        if (two) Launch(EmbeddingStagedKernel<MLB_Q8_0, 2>, grid2, cta_threads, shm, s, a, span, pc, slice);
        else Launch(EmbeddingStagedKernel<MLB_Q8_0, 1>, grid2, cta_threads, shm, s, a, span, pc, slice);
        break;
      case MLB_Q4_0:
        if (two) Launch(EmbeddingStagedKernel<MLB_Q4_0, 2>, grid2, cta_threads, shm, s, a, span, pc, slice);
        else Launch(EmbeddingStagedKernel<MLB_Q4_0, 1>, grid2, cta_threads, shm, s, a, span, pc, slice);
        break;
      case MLB_Q4_1:
        if (two) Launch(EmbeddingStagedKernel<MLB_Q4_1, 2>, grid2, cta_threads, shm, s, a, span, pc, slice);
        else Launch(EmbeddingStagedKernel<MLB_Q4_1, 1>, grid2, cta_threads, shm, s, a, span, pc, slice);
        break;
    }
  } else {
    Launch(EmbeddingScalarKernel, grid, 256, 0, s, a, qtype);
  }
  return CheckLaunch(op);
}

}  // namespace
}  // namespace mlb

extern "C" int mlb_embedding_gather(const void* table, int qtype, int64_t vocab,
                                    int64_t cols, const int32_t* tokens,
                                    int64_t rows, float* out, int32_t* status,
                                    void* stream) {
  if (rows > 0 && tokens == nullptr)
    return mlb::Fail(MLB_ERR_ARG, "mlb_embedding_gather: null tokens");
  return mlb::LaunchEmbedding(table, qtype, vocab, cols, tokens, 0, rows, out,
                              status, stream, "mlb_embedding_gather");
}

extern "C" int mlb_embedding_row(const void* table, int qtype, int64_t vocab,
                                 int64_t cols, int32_t token, float* out,
                                 void* stream) {
  if (token < 0 || token >= vocab)
    return mlb::Fail(MLB_ERR_RANGE, "mlb_embedding_row: token out of range");
  return mlb::LaunchEmbedding(table, qtype, vocab, cols, nullptr, token, 1, out,
                              nullptr, stream, "mlb_embedding_row");
}
