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
// Kernels (cols % 4 == 0, 16-byte aligned output): one CTA per token row
// (one warp per row when cols <= 1024).  Quantised tables stage the row's
// bytes in shared memory with 16-byte loads and decode float4s — 4
// consecutive values of one block — from there; F32 tables copy the row with
// float4 loads.  Output stores are 16-byte and fully
// coalesced.  Any other shape takes the scalar kernel (one value per thread).
// HBM roofline per row: row_bytes read + 4 * cols written (+ 4 for the id).
#include <climits>

#include "common.cuh"

namespace mlb {
namespace {

// Rows up to this many bytes are staged one per warp when there are rows
// enough to fill every SM (B200 sweep: Q8_0 at cols 2048 1.08 vs 0.79 of the
// copy peak, Q4_1 at cols 4096 1.03 vs 0.88; Q8_0 at cols 4096 — 4352-byte
// rows — is faster one row per CTA).
constexpr int64_t kWarpRowBytes = 2560;

// Largest staged row (bytes of dynamic shared memory without an opt-in):
// Q8_0 rows up to cols ~ 45000.  Longer rows take the scalar kernel.
constexpr int64_t kMaxStagedBytes = 48 * 1024;

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

// Decodes output float4 number o of a row (block b = o / 8, values e..e+3
// with e = (o % 8) * 4) from the row's bytes staged in shared memory.  The
// staged copy keeps the table's alignment modulo 16, so block starts are
// 2-byte aligned (Q8_0, Q4_0: 34 B and 18 B blocks) or 4-byte aligned (Q4_1:
// 20 B blocks): the scale and the four quant bytes are read as two u16 + one
// u16 (Q8_0, Q4_0) or two u32 (Q4_1) shared loads.
__device__ __forceinline__ uint32_t Smem16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

template <int QT>
__device__ __forceinline__ float4 DecodeStaged(const uint8_t* row, int o) {
  const int e = (o & 7) << 2;
  if (QT == MLB_Q8_0) {
    const uint8_t* blk = row + (o >> 3) * 34;
    const float d = Fp16BitsToF32(Smem16(blk));
    const uint32_t q = Smem16(blk + 2 + e) | (Smem16(blk + 4 + e) << 16);
    return make_float4(
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 8) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 16) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q >> 24))));
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
  const float n0 = static_cast<float>(q & 15u);
  const float n1 = static_cast<float>((q >> 8) & 15u);
  const float n2 = static_cast<float>((q >> 16) & 15u);
  const float n3 = static_cast<float>((q >> 24) & 15u);
  const float d = Fp16BitsToF32(scale & 0xffffu);
  if (QT == MLB_Q4_0) {
    return make_float4(__fmul_rn(d, n0 - 8.0f), __fmul_rn(d, n1 - 8.0f),
                       __fmul_rn(d, n2 - 8.0f), __fmul_rn(d, n3 - 8.0f));
  }
  const float m = Fp16BitsToF32(scale >> 16);
  return make_float4(__fadd_rn(__fmul_rn(d, n0), m), __fadd_rn(__fmul_rn(d, n1), m),
                     __fadd_rn(__fmul_rn(d, n2), m), __fadd_rn(__fmul_rn(d, n3), m));
}

// Copies table bytes [window, window + 16 * chunks) into `dst` with 16-byte
// loads, lane `first` stepping by `step`; bytes past the end of the table are
// never read (they are written as 0 and never decoded).
__device__ __forceinline__ void StageWindow(uint8_t* dst, const uint8_t* table,
                                            int64_t window, int chunks,
                                            int64_t table_bytes, int first,
                                            int step) {
  for (int c = first; c < chunks; c += step) {
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

// Quantised tables: one CTA per token row.  The CTA first copies the row's
// bytes into shared memory with 16-byte loads over the 16-byte-aligned window
// that covers it (ggml rows are only 2-byte aligned: 952 B per Q8_0 row at
// cols 896), then decodes float4s from shared memory and streams them out.
// Bytes of the window that lie past the end of the table are never read.
// (Measured on B200, Q8_0 [128256, 4096], 16384 tokens: 5.63 TB/s, against
// 5.49 TB/s decoding straight from 2-byte global loads with every load of a
// thread issued first, and 3.4-4.6 TB/s for flat or serial-loop forms.)
// With few tokens (a decode batch) each row is split over gridDim.y CTAs of
// `per_cta` output float4s each (a multiple of 8: whole blocks); a CTA stages
// only the blocks it decodes.
template <int QT>
__global__ void __launch_bounds__(256) EmbeddingStagedKernel(EmbArgs a,
                                                             int64_t table_bytes,
                                                             int per_cta) {
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
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
    float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
    if (token < 0 || token >= a.vocab) {
      if (threadIdx.x == 0 && blockIdx.y == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
      for (int o = g0 + threadIdx.x; o < g1; o += blockDim.x)
        StoreStream(out + o, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const int64_t start = static_cast<int64_t>(token) * a.row_bytes +
                          static_cast<int64_t>(b0) * kBB;
    const int64_t end = start + static_cast<int64_t>(b1 - b0) * kBB;
    const int64_t window = start & ~int64_t{15};
    const int chunks = static_cast<int>((end - window + 15) >> 4);
    __syncthreads();  // the previous row's decode is done with `staged`
    StageWindow(staged, a.table, window, chunks, table_bytes, threadIdx.x,
                blockDim.x);
    __syncthreads();
    // `row` addresses block 0 of the row; only blocks [b0, b1) are staged
    const uint8_t* row = staged + (start - window) - static_cast<int64_t>(b0) * kBB;
    for (int o = g0 + threadIdx.x; o < g1; o += blockDim.x)
      StoreStream(out + o, DecodeStaged<QT>(row, o));
  }
}

// Short rows (cols <= 1024, or rows of at most kWarpRowBytes in a large
// batch): one warp per token row, up to 8 rows per CTA, each warp staging its
// own row in its slice of shared memory (`slice` bytes) — a CTA per short
// row would be mostly launch and barrier overhead.
template <int QT>
__global__ void __launch_bounds__(256) EmbeddingStagedWarpKernel(EmbArgs a,
                                                                 int64_t table_bytes,
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
    const int64_t start = static_cast<int64_t>(token) * a.row_bytes;
    const int64_t window = start & ~int64_t{15};
    const int chunks = static_cast<int>((start + a.row_bytes - window + 15) >> 4);
    __syncwarp();  // the previous row's decode is done with `mine`
    StageWindow(mine, a.table, window, chunks, table_bytes, lane, 32);
    __syncwarp();
    const uint8_t* row = mine + (start - window);
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
  // Rows split over CTAs when tokens cannot fill every SM twice; each CTA
  // takes a whole number of blocks (8 float4s per block).
  const int64_t fill = 2 * static_cast<int64_t>(SmCount());
  int64_t split = rows < fill ? (fill + rows - 1) / rows : 1;
  const int64_t blocks_per_row = (groups + 7) / 8;
  if (split > blocks_per_row) split = blocks_per_row;
  if (split < 1) split = 1;
  const int64_t per_cta = (blocks_per_row + split - 1) / split * 8;
  split = (groups + per_cta - 1) / per_cta;
  const int bb = qtype == MLB_Q8_0 ? 34 : (qtype == MLB_Q4_0 ? 18 : 20);
  // staged window: up to 15 leading bytes + the CTA's blocks, rounded to 16
  const int64_t smem = (per_cta / 8 * bb + 15 + 15) / 16 * 16;
  const int64_t table_bytes_all = vocab * row_bytes;
  if (vec && qtype == MLB_F32 && (tbl & 15u) == 0) {
    Launch(EmbeddingF32Kernel, grid, threads, 0, s, a);
  } else if (vec && qtype != MLB_F32 &&
             (cols <= 1024 || (rows >= fill && row_bytes <= kWarpRowBytes))) {
    // warp per row; 8 rows per CTA unless rows are too few to fill the SMs
    int64_t wpc = rows / fill;
    wpc = wpc < 1 ? 1 : (wpc > 8 ? 8 : wpc);
    const int slice = static_cast<int>((row_bytes + 15 + 15) / 16 * 16);
    const int64_t nblk = (rows + wpc - 1) / wpc;
    const dim3 wgrid(static_cast<unsigned>(nblk < cap ? nblk : cap));
    const int wthreads = static_cast<int>(32 * wpc);
    const size_t shm = static_cast<size_t>(slice) * wpc;
    switch (qtype) {
      case MLB_Q8_0:
        Launch(EmbeddingStagedWarpKernel<MLB_Q8_0>, wgrid, wthreads, shm, s, a, table_bytes_all, slice);
        break;
      case MLB_Q4_0:
        Launch(EmbeddingStagedWarpKernel<MLB_Q4_0>, wgrid, wthreads, shm, s, a, table_bytes_all, slice);
        break;
      case MLB_Q4_1:
        Launch(EmbeddingStagedWarpKernel<MLB_Q4_1>, wgrid, wthreads, shm, s, a, table_bytes_all, slice);
        break;
    }
  } else if (vec && qtype != MLB_F32 && smem <= kMaxStagedBytes) {
    const int64_t table_bytes = vocab * row_bytes;
    const size_t shm = static_cast<size_t>(smem);
    const dim3 grid2(grid.x, static_cast<unsigned>(split));
    int cta_threads = per_cta < 256 ? static_cast<int>((per_cta + 31) / 32 * 32) : 256;
    if (cta_threads > threads) cta_threads = threads;
    const int pc = static_cast<int>(per_cta);
    switch (qtype) {
      case MLB_Q8_0:
        Launch(EmbeddingStagedKernel<MLB_Q8_0>, grid2, cta_threads, shm, s, a, table_bytes, pc);
        break;
      case MLB_Q4_0:
        Launch(EmbeddingStagedKernel<MLB_Q4_0>, grid2, cta_threads, shm, s, a, table_bytes, pc);
        break;
      case MLB_Q4_1:
        Launch(EmbeddingStagedKernel<MLB_Q4_1>, grid2, cta_threads, shm, s, a, table_bytes, pc);
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
