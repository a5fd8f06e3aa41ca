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
// Vector kernels (cols % 4 == 0): each thread produces float4s of output —
// 4 consecutive values of one block — from the block's 2-byte scale
// (broadcast across the 8 threads of the block) and 4 quant bytes read as two
// aligned u16 (Q8_0/Q4_0) or one u32 (Q4_1).  The flat kernel gives every
// thread one float4 of the [rows, cols] output; the row-per-CTA kernel (for
// more than 2^32 float4s) gives a thread NG of them, all loaded before any is
// decoded.  Output stores are 16-byte and fully coalesced.  Scalar kernel
// otherwise.
// HBM roofline per row: row_bytes read + 4 * cols written (+ 4 for the id).
#include <climits>

#include "common.cuh"

namespace mlb {
namespace {

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

// Four consecutive quant bytes starting at a 2-byte aligned address.
__device__ __forceinline__ uint32_t Load4Bytes2(const uint8_t* p) {
  return LoadU16(p) | (LoadU16(p + 2) << 16);
}

// Raw bytes of one output float4 (block b = o / 8, values e..e+3 with
// e = (o % 8) * 4): the block's scale word and four quant bytes.
struct RawGroup {
  uint32_t scale;  // d (Q8_0, Q4_0) or d | m << 16 (Q4_1)
  uint32_t quants; // 4 quant bytes, or the high-nibble bytes pre-shifted
};

template <int QT>
__device__ __forceinline__ RawGroup LoadGroup(const uint8_t* row, int o) {
  const int b = o >> 3;
  const int e = (o & 7) << 2;
  RawGroup g;
  if (QT == MLB_Q8_0) {
    const uint8_t* blk = row + b * 34;
    g.scale = LoadU16(blk);
    g.quants = Load4Bytes2(blk + 2 + e);
  } else if (QT == MLB_Q4_0) {
    const uint8_t* blk = row + b * 18;
    g.scale = LoadU16(blk);
    g.quants = Load4Bytes2(blk + 2 + (e & 15));
  } else {  // MLB_Q4_1
    const uint8_t* blk = row + b * 20;
    g.scale = __ldg(reinterpret_cast<const unsigned int*>(blk));
    g.quants = __ldg(reinterpret_cast<const unsigned int*>(blk + 4 + (e & 15)));
  }
  if (QT != MLB_Q8_0 && e >= 16) g.quants >>= 4;  // high nibbles: last 16
  return g;
}

template <int QT>
__device__ __forceinline__ float4 DecodeGroup(const RawGroup& g) {
  const uint32_t q = g.quants;
  if (QT == MLB_Q8_0) {
    const float d = Fp16BitsToF32(g.scale);
    return make_float4(
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 8) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 16) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q >> 24))));
  } else if (QT == MLB_Q4_0) {
    const float d = Fp16BitsToF32(g.scale);
    return make_float4(
        __fmul_rn(d, static_cast<float>(static_cast<int>(q & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 8) & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 16) & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 24) & 15u) - 8)));
  } else {  // MLB_Q4_1
    const float d = Fp16BitsToF32(g.scale & 0xffffu);
    const float m = Fp16BitsToF32(g.scale >> 16);
    return make_float4(
        __fadd_rn(__fmul_rn(d, static_cast<float>(q & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 8) & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 16) & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 24) & 15u)), m));
  }
}

// One CTA per token row.  Each thread owns NG output float4s of a chunk of
// blockDim * NG float4s and issues every load of the chunk before decoding,
// so a row costs one memory latency instead of NG serial ones.
template <int QT, int NG>
__global__ void __launch_bounds__(256) EmbeddingVecKernel(EmbArgs a) {
  const int groups = a.cols >> 2;
  const int chunk = blockDim.x * NG;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
    float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
    if (token < 0 || token >= a.vocab) {
      if (threadIdx.x == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
      for (int o = threadIdx.x; o < groups; o += blockDim.x)
        StoreStream(out + o, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const uint8_t* row = a.table + static_cast<size_t>(token) * a.row_bytes;
    for (int base = 0; base < groups; base += chunk) {
      if (QT == MLB_F32) {
        const float4* src = reinterpret_cast<const float4*>(row);
        float4 v[NG];
#pragma unroll
        for (int k = 0; k < NG; ++k) {
          const int o = base + threadIdx.x + k * blockDim.x;
          if (o < groups) v[k] = __ldg(src + o);
        }
#pragma unroll
        for (int k = 0; k < NG; ++k) {
          const int o = base + threadIdx.x + k * blockDim.x;
          if (o < groups) StoreStream(out + o, v[k]);
        }
      } else {
        RawGroup g[NG];
#pragma unroll
        for (int k = 0; k < NG; ++k) {
          const int o = base + threadIdx.x + k * blockDim.x;
          if (o < groups) g[k] = LoadGroup<QT>(row, o);
        }
#pragma unroll
        for (int k = 0; k < NG; ++k) {
          const int o = base + threadIdx.x + k * blockDim.x;
          if (o < groups) StoreStream(out + o, DecodeGroup<QT>(g[k]));
        }
      }
    }
  }
}

// Flat form: one output float4 per thread over rows * cols/4 items, so the
// output stream is written in address order by consecutive CTAs.  Used while
// the item count fits 32 bits; the row-per-CTA kernel above covers the rest.
template <int QT>
__global__ void __launch_bounds__(256)
    EmbeddingFlatKernel(EmbArgs a, uint32_t groups, uint32_t total) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const uint32_t t = idx / groups;
  const int o = static_cast<int>(idx - t * groups);
  const int32_t token = a.tokens != nullptr ? __ldg(a.tokens + t) : a.token;
  float4* out = reinterpret_cast<float4*>(a.out) + idx;
  if (token < 0 || token >= a.vocab) {
    if (o == 0 && a.status != nullptr) atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
    StoreStream(out, make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }
  const uint8_t* row = a.table + static_cast<size_t>(token) * a.row_bytes;
  if (QT == MLB_F32) {
    StoreStream(out, __ldg(reinterpret_cast<const float4*>(row) + o));
  } else {
    StoreStream(out, DecodeGroup<QT>(LoadGroup<QT>(row, o)));
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
  const bool vec = (cols % 4) == 0 && Aligned16(out) &&
                   (qtype != MLB_F32 || (tbl & 15u) == 0);
  const int64_t total = rows * static_cast<int64_t>(groups);
  if (vec && total <= 0xffffffffLL - 256) {
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    const uint32_t g32 = static_cast<uint32_t>(groups);
    const uint32_t t32 = static_cast<uint32_t>(total);
    switch (qtype) {
      case MLB_F32: EmbeddingFlatKernel<MLB_F32><<<blocks, 256, 0, s>>>(a, g32, t32); break;
      case MLB_Q8_0: EmbeddingFlatKernel<MLB_Q8_0><<<blocks, 256, 0, s>>>(a, g32, t32); break;
      case MLB_Q4_0: EmbeddingFlatKernel<MLB_Q4_0><<<blocks, 256, 0, s>>>(a, g32, t32); break;
      case MLB_Q4_1: EmbeddingFlatKernel<MLB_Q4_1><<<blocks, 256, 0, s>>>(a, g32, t32); break;
    }
  } else if (vec) {
    int ng = (groups + threads - 1) / threads;
    if (ng > 8) ng = 8;
    switch (ng) {
#define MLB_NG(N)                                                            \
  case N:                                                                    \
    switch (qtype) {                                                         \
      case MLB_F32: EmbeddingVecKernel<MLB_F32, N><<<grid, threads, 0, s>>>(a); break;  \
      case MLB_Q8_0: EmbeddingVecKernel<MLB_Q8_0, N><<<grid, threads, 0, s>>>(a); break; \
      case MLB_Q4_0: EmbeddingVecKernel<MLB_Q4_0, N><<<grid, threads, 0, s>>>(a); break; \
      case MLB_Q4_1: EmbeddingVecKernel<MLB_Q4_1, N><<<grid, threads, 0, s>>>(a); break; \
    }                                                                        \
    break;
      MLB_NG(1) MLB_NG(2) MLB_NG(3) MLB_NG(4) MLB_NG(5) MLB_NG(6) MLB_NG(7)
      MLB_NG(8)
#undef MLB_NG
    }
  } else {
    EmbeddingScalarKernel<<<grid, 256, 0, s>>>(a, qtype);
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
