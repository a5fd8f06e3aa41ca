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
// Vector kernel (cols % 4 == 0): one CTA per token row; each thread produces
// one float4 of output per item — 4 consecutive values of one block — from
// the block's 2-byte scale (broadcast across the 8 threads of the block) and
// 4 quant bytes read as two aligned u16 (Q8_0/Q4_0) or one u32 (Q4_1).
// Output stores are 16-byte, fully coalesced.  Scalar kernel otherwise.
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
  const int32_t* tokens;
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

template <int QT>
__device__ __forceinline__ float4 DecodeGroup(const uint8_t* row, int o) {
  // o = index of the float4 within the row; block b, first value e.
  const int b = o >> 3;
  const int e = (o & 7) << 2;
  if (QT == MLB_Q8_0) {
    const uint8_t* blk = row + b * 34;
    const float d = Fp16BitsToF32(LoadU16(blk));
    const uint32_t q = Load4Bytes2(blk + 2 + e);
    return make_float4(
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 8) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> 16) & 0xffu))),
        __fmul_rn(d, static_cast<float>(static_cast<int8_t>(q >> 24))));
  } else if (QT == MLB_Q4_0) {
    const uint8_t* blk = row + b * 18;
    const float d = Fp16BitsToF32(LoadU16(blk));
    uint32_t q = Load4Bytes2(blk + 2 + (e & 15));
    if (e >= 16) q >>= 4;
    return make_float4(
        __fmul_rn(d, static_cast<float>(static_cast<int>(q & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 8) & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 16) & 15u) - 8)),
        __fmul_rn(d, static_cast<float>(static_cast<int>((q >> 24) & 15u) - 8)));
  } else {  // MLB_Q4_1
    const uint8_t* blk = row + b * 20;
    const uint32_t dm = __ldg(reinterpret_cast<const unsigned int*>(blk));
    const float d = Fp16BitsToF32(dm & 0xffffu);
    const float m = Fp16BitsToF32(dm >> 16);
    uint32_t q = __ldg(reinterpret_cast<const unsigned int*>(blk + 4 + (e & 15)));
    if (e >= 16) q >>= 4;
    return make_float4(
        __fadd_rn(__fmul_rn(d, static_cast<float>(q & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 8) & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 16) & 15u)), m),
        __fadd_rn(__fmul_rn(d, static_cast<float>((q >> 24) & 15u)), m));
  }
}

template <int QT>
__global__ void __launch_bounds__(256) EmbeddingVecKernel(EmbArgs a) {
  const int groups = a.cols >> 2;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int32_t token = __ldg(a.tokens + t);
    float4* out = reinterpret_cast<float4*>(a.out + static_cast<size_t>(t) * a.cols);
    if (token < 0 || token >= a.vocab) {
      if (threadIdx.x == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_TOKEN);
      for (int o = threadIdx.x; o < groups; o += blockDim.x)
        StoreStream(out + o, make_float4(0.f, 0.f, 0.f, 0.f));
      continue;
    }
    const uint8_t* row = a.table + static_cast<size_t>(token) * a.row_bytes;
    if (QT == MLB_F32) {
      const float4* src = reinterpret_cast<const float4*>(row);
      for (int o = threadIdx.x; o < groups; o += blockDim.x)
        StoreStream(out + o, __ldg(src + o));
    } else {
      for (int o = threadIdx.x; o < groups; o += blockDim.x)
        StoreStream(out + o, DecodeGroup<QT>(row, o));
    }
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
    const int32_t token = a.tokens[t];
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

extern "C" int mlb_embedding_gather(const void* table, int qtype, int64_t vocab,
                                    int64_t cols, const int32_t* tokens,
                                    int64_t rows, float* out, int32_t* status,
                                    void* stream) {
  using namespace mlb;
  if (qtype < MLB_F32 || qtype > MLB_Q4_1)
    return Fail(MLB_ERR_ARG, "mlb_embedding_gather: unknown qtype");
  if (rows < 0 || cols <= 0 || cols > INT_MAX || vocab < 0 || vocab > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_embedding_gather: bad shape");
  if (rows == 0) return MLB_OK;
  if (table == nullptr || tokens == nullptr || out == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_embedding_gather: null pointer");
  const uintptr_t tbl = reinterpret_cast<uintptr_t>(table);
  if (qtype != MLB_F32 && (tbl & (qtype == MLB_Q4_1 ? 3u : 1u)) != 0)
    return Fail(MLB_ERR_ARG, "mlb_embedding_gather: table misaligned");
  if (qtype == MLB_F32 && (tbl & 3u) != 0)
    return Fail(MLB_ERR_ARG, "mlb_embedding_gather: table misaligned");
  EmbArgs a{static_cast<const uint8_t*>(table), vocab, static_cast<int>(cols),
            mlb_row_bytes(qtype, cols), tokens, rows, out, status};
  const int64_t cap = 1 << 24;
  const dim3 grid(static_cast<unsigned>(rows < cap ? rows : cap));
  const int groups = static_cast<int>(cols / 4);
  int threads = groups < 256 ? (groups + 31) / 32 * 32 : 256;
  if (threads < 32) threads = 32;
  cudaStream_t s = AsStream(stream);
  const bool vec = (cols % 4) == 0 && Aligned16(out) &&
                   (qtype != MLB_F32 || (tbl & 15u) == 0);
  if (vec) {
    switch (qtype) {
      case MLB_F32: EmbeddingVecKernel<MLB_F32><<<grid, threads, 0, s>>>(a); break;
      case MLB_Q8_0: EmbeddingVecKernel<MLB_Q8_0><<<grid, threads, 0, s>>>(a); break;
      case MLB_Q4_0: EmbeddingVecKernel<MLB_Q4_0><<<grid, threads, 0, s>>>(a); break;
      case MLB_Q4_1: EmbeddingVecKernel<MLB_Q4_1><<<grid, threads, 0, s>>>(a); break;
    }
  } else {
    EmbeddingScalarKernel<<<grid, 256, 0, s>>>(a, qtype);
  }
  return CheckLaunch("mlb_embedding_gather");
}
