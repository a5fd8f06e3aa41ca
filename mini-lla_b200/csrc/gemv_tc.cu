// Decode-sized quantised linear layers on the int8 tensor cores:
// y[t] = W . x[t] for t < T <= 4 per launch, W [n, k] in the reference's
// ggml Q8_0 / Q4_0 / Q4_1 blocks, x and y fp32.
//
// Reference arithmetic (src/quant.cc:171-226 LinearWithBlocks): per output
// a sequential fp32 sum of dequant(w_i) * x_i, dequant = d * q (Q8_0),
// d * (n - 8) (Q4_0), d * n + m (Q4_1).
//
// Method: exact integer products, no dequantisation of W.
//   - the weight codes go to the MMA as stored: Q8_0's int8 q as signed
//     bytes, the Q4 formats' 4-bit n as unsigned bytes;
//   - each block of 32 values of x[t] is written as
//       x_i = s * (D0_i + D1_i / 128 + D2_i / 128^2 + D3_i / 128^3) + r_i,
//     s = 2^(e - 6) with 2^(e-1) <= max_i |x_i| < 2^e, integer digits
//     |Dj_i| <= 64 (each the rounding of an exactly computed fp32
//     remainder) and |r_i| <= 2^-22 s <= 2^-27 max_i |x_i|;
//   - per (row, block, token, digit) the tensor core forms
//     A_j = sum_i q_i Dj_i exactly in int32 (tcgen05.mma kind::i8,
//     M = 128 rows, N = 16 = 4 tokens x 4 digits, K = 32 = one block);
//   - the epilogue adds d * s * (A0 + A1/128 + A2/128^2 + A3/128^3) to the
//     row's fp32 sum (Q4_0 first takes 8 * sum_i Dj_i off each A_j: the
//     codes are n, the values n - 8; Q4_1 adds m * sum_i x_i).
// Error per output: the fp32 roundings of ~5 operations per block plus
// sum_b sum_i |w_i| 2^-27 max_b |x| — orders of magnitude inside the tests'
// |y - y_ref| <= 1e-5 * sum_i |w_i x_i| unless a block of x mixes values
// ~2^20 apart.  A block of x holding Inf or NaN makes its outputs NaN.
//
// Design (one CTA per SM, 320 threads; persistent clusters of `split` CTAs,
// each cluster taking 128-row tiles, rank r of a cluster taking 1 / split of
// every row's blocks):
//   - warp 8, one lane: TMA producer.  A stage is 8 (Q8_0) or 16 (Q4)
//     consecutive blocks of the tile's 128 rows — 272 / 288 / 320 bytes per
//     row, loaded as 5 boxes of 64 bytes x 128 rows from a 2-D uint8 tensor
//     map over [n, row_bytes] (64-byte swizzle, so per-row reads are
//     bank-conflict free); 3 stages in flight;
//   - warps 0-3 (movers; thread = weight row = tensor-memory lane): copy a
//     chunk's (8 blocks') codes from the raw stage into tensor memory
//     (tcgen05.st; the A operand, 8 columns per block) and its block scales
//     into shared memory;
//   - warp 9: allocates tensor memory; one lane issues the chunk's 8 MMAs
//     (B from the resident digit tiles, one result slot per chunk) and
//     commits them;
//   - warps 4-7 (epilogue; thread = row): read a chunk's int32 results
//     (tcgen05.ld) and accumulate d * s * digits-sum per block and token;
//     at a tile's end rank r > 0 sends its 128 x 4 partial sums into rank
//     0's shared memory (st.async, counted on rank 0's mbarrier) and rank 0
//     adds them in rank order (deterministic) and writes y;
//   - before the loop, warps 0-7 write x's digits (the rank's share of k)
//     into shared memory in the K-major 128-byte-swizzled layout the MMA
//     reads (one thread per block of 32 values and token).
// Tensor memory (512 columns): T <= 2: N = 8, 3 code slots of 64 columns and
// 5 result slots of 64; T = 4: N = 16, 2 + 3 slots of 64 / 128 columns.
// Measured on B200: an i8 MMA of 128 x 32 x N costs ~60-110 cycles whatever
// N <= 64, so the tensor pipe, not HBM, bounds a 128 x 4096 tile (~128
// MMAs); wide matrices (the FFN, the output projection) gain most.
// Every wait is bounded: a wait that gives up is counted (mlb_wait_timeouts)
// and the CTA writes NaN to its outputs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kGtRows = 128;            // weight rows per tile (MMA M)
constexpr int kGtThreads = 320;         // 8 mover/epilogue warps, producer, MMA
constexpr int kGtMovers = 256;
constexpr int kGtBox = 64;              // bytes per box row
constexpr int kGtBoxes = 5;             // boxes per stage
constexpr int kGtBoxBytes = kGtBox * kGtRows;
constexpr int kGtStageBytes = kGtBoxes * kGtBoxBytes;
constexpr int kGtRawStages = 3;
constexpr int kGtMaxTokens = 4;
constexpr int kGtChunk = 8;             // blocks per chunk (one MMA each)
constexpr int kGtAColumns = 64;         // a chunk's codes: 8 blocks x 8 columns (4 codes each)
constexpr int kGtMaxSlots = 5;          // largest code / result ring
constexpr int kGtTmemColumns = 512;
constexpr int kGtMaxDigitBytes = 64 * 1024;  // x digits resident in shared memory

// Per token count T (1, 2 or 4): MMA N = 4 digits x tokens (8 for T <= 2,
// 16 for T = 4) and the tensor-memory rings (code slots of 64 columns,
// result slots of 8 N columns; 512 columns in all).
__host__ __device__ constexpr int GtN(int t) { return t <= 2 ? 8 : 16; }
__host__ __device__ constexpr int GtASlots(int t) { return t <= 2 ? 3 : 2; }
__host__ __device__ constexpr int GtDSlots(int t) { return t <= 2 ? 5 : 3; }

__host__ __device__ constexpr int GtBlockBytes(int qt) {
  return qt == MLB_Q8_0 ? 34 : (qt == MLB_Q4_0 ? 18 : 20);
}
__host__ __device__ constexpr int GtStageBlocks(int qt) { return qt == MLB_Q8_0 ? 8 : 16; }

// Shared-memory layout (offsets from a 1024-byte aligned base) for a CTA
// whose share of a row has `nb` blocks, in clusters of `split` ranks.
struct GtLayout {
  int digits;  // [nb / 4 chunks][16 rows][128 bytes], 128-byte swizzle
  int raw;     // kGtRawStages x kGtStageBytes
  int xscale;  // float [nb][4 tokens]
  int xcorr;   // Q4_0: int [nb][4 tokens][4 digits]; Q4_1: float [nb][4]
  int scales;  // uint32 [result slots][8 blocks][128 rows]: d | m << 16 (fp16 bits)
  int red;     // float [2][split][128 rows][4 tokens]: ranks' partials (rank 0)
  int bars;
  int total;
};

// raw_full / raw_empty per stage, a_full / a_empty per code slot, d_full /
// d_empty per result slot, b_ready, mma_done, red_full / red_empty x 2
constexpr int kGtBarriers = 2 * kGtRawStages + 4 * kGtMaxSlots + 2 + 4;

__host__ __device__ inline GtLayout MakeGtLayout(int qt, int nb, int split, int tokens) {
  GtLayout l{};
  l.digits = 0;
  l.raw = nb / 4 * GtN(tokens) * 128;  // (a multiple of 1024)
  l.xscale = l.raw + kGtRawStages * kGtStageBytes;
  l.xcorr = l.xscale + nb * kGtMaxTokens * 4;
  l.scales = l.xcorr + (qt == MLB_Q4_0 ? nb * kGtMaxTokens * 4 * 4
                                       : (qt == MLB_Q4_1 ? nb * kGtMaxTokens * 4 : 0));
  l.red = l.scales + GtDSlots(tokens) * kGtChunk * kGtRows * 4;
  l.bars = l.red + (split > 1 ? 2 * split * kGtRows * kGtMaxTokens * 4 : 0);
  l.total = l.bars + 8 * kGtBarriers + 16;  // + the TMEM address and the abort flag
  return l;
}

__device__ __forceinline__ uint32_t GtSmem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void GtBarInit(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void GtExpectTx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void GtArrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool GtTryWait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(1000)
      : "memory");
  return ok != 0;
}
// ~2 s at most (each poll suspends for at most ~1 us)
__device__ __forceinline__ bool GtWait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 21); ++i)
    if (GtTryWait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void GtTmaLoad(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major operand, 128-byte swizzle, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t GtDesc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor: D int32, A u8 (Q4) or s8 (Q8_0), B s8, both
// K-major, N, M = 128.
template <int QT, int N>
__host__ __device__ constexpr uint32_t GtInstrDesc() {
  return (2u << 4) | ((QT == MLB_Q8_0 ? 1u : 0u) << 7) | (1u << 10) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(kGtRows >> 4) << 24);
}

// D[d] = A[a] . B[b]^T (no accumulation: one block per result), A in
// tensor memory (row m in lane m, 4 codes per column).
__device__ __forceinline__ void GtMma(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void GtCommit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void GtStore32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void GtLoad8(uint32_t taddr, int (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr));
}
__device__ __forceinline__ void GtLoad16(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// Bytes [b, b + 4) of the words w (b a constant once the callers' loops
// are unrolled, so w stays in registers).
template <int NW>
__device__ __forceinline__ uint32_t GtWord(const uint32_t (&w)[NW], int b) {
  if ((b & 3) == 0) return w[b >> 2];
  return __funnelshift_r(w[b >> 2], w[(b >> 2) + 1], 8 * (b & 3));
}

// Codes and scale of block J of a chunk whose bytes start at byte REL of
// the loaded words: 8 code words (A columns 8J .. 8J + 7) and the scale
// word (d | m << 16).
template <int QT, int REL, int J, int NW>
__device__ __forceinline__ void GtTakeBlock(const uint32_t (&w)[NW], uint32_t (&codes)[32],
                                            uint32_t& scale) {
  constexpr int b = REL + J * GtBlockBytes(QT);
  if constexpr (QT == MLB_Q8_0) {
    scale = GtWord<NW>(w, b) & 0xFFFFu;
#pragma unroll
    for (int i = 0; i < 8; ++i) codes[8 * J + i] = GtWord<NW>(w, b + 2 + 4 * i);
  } else if constexpr (QT == MLB_Q4_0) {
    scale = GtWord<NW>(w, b) & 0xFFFFu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = GtWord<NW>(w, b + 2 + 4 * i);
      codes[8 * J + i] = u & 0x0F0F0F0Fu;             // values 4i .. 4i + 3
      codes[8 * J + 4 + i] = (u >> 4) & 0x0F0F0F0Fu;  // values 16 + 4i ..
    }
  } else {
    scale = GtWord<NW>(w, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = GtWord<NW>(w, b + 4 + 4 * i);
      codes[8 * J + i] = u & 0x0F0F0F0Fu;
      codes[8 * J + 4 + i] = (u >> 4) & 0x0F0F0F0Fu;
    }
  }
}

// Reads row m's bytes of chunk POS of a raw stage (blocks 4 POS .. 4 POS + 3
// of the stage) and returns its 32 code words and 4 scale words.
template <int QT, int POS>
__device__ __forceinline__ void GtReadChunk(const uint8_t* stage, int m, uint32_t (&codes)[32],
                                            uint32_t (&scales)[4]) {
  constexpr int kBB = GtBlockBytes(QT);
  constexpr int off = POS * 4 * kBB;                  // chunk's first byte in the stage
  constexpr int q0 = off / 16;                        // first 16-byte piece
  constexpr int rel = off - 16 * q0;
  constexpr int pieces = (rel + 4 * kBB + 15) / 16;   // pieces covering the chunk
  constexpr int NW = 4 * pieces + 1;                  // (+1: funnel-shift slack)
  uint32_t w[NW];
#pragma unroll
  for (int p = 0; p < pieces; ++p) {
    const int q = q0 + p;
    const int box = q >> 2;
    const int phys = (q & 3) ^ ((m >> 1) & 3);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + box * kGtBoxBytes + m * kGtBox +
                                                    16 * phys);
    w[4 * p] = v.x;
    w[4 * p + 1] = v.y;
    w[4 * p + 2] = v.z;
    w[4 * p + 3] = v.w;
  }
  w[NW - 1] = 0;
  GtTakeBlock<QT, rel, 0, NW>(w, codes, scales[0]);
  GtTakeBlock<QT, rel, 1, NW>(w, codes, scales[1]);
  GtTakeBlock<QT, rel, 2, NW>(w, codes, scales[2]);
  GtTakeBlock<QT, rel, 3, NW>(w, codes, scales[3]);
}

template <int QT>
__device__ __forceinline__ void GtReadChunkAt(int pos, const uint8_t* stage, int m,
                                              uint32_t (&codes)[32], uint32_t (&scales)[4]) {
  if constexpr (QT == MLB_Q8_0) {
    if (pos == 0) GtReadChunk<QT, 0>(stage, m, codes, scales);
    else GtReadChunk<QT, 1>(stage, m, codes, scales);
  } else {
    switch (pos) {
      case 0: GtReadChunk<QT, 0>(stage, m, codes, scales); break;
      case 1: GtReadChunk<QT, 1>(stage, m, codes, scales); break;
      case 2: GtReadChunk<QT, 2>(stage, m, codes, scales); break;
      default: GtReadChunk<QT, 3>(stage, m, codes, scales); break;
    }
  }
}

// Up to kGtMaxGroup matrices of one format and width applied to the same x
// in one launch (the q / k / v projections, the FFN gate / up): their
// 128-row tiles are numbered matrix by matrix.
constexpr int kGtMaxGroup = 3;

struct GtArgs {
  CUtensorMap w[kGtMaxGroup];  // raw weight bytes [n, row_bytes] of each matrix
  float* y[kGtMaxGroup];       // [tokens, n] each
  int n[kGtMaxGroup];
  int tile_begin[kGtMaxGroup + 1];  // first tile of each matrix; [count] = all tiles
  int count;
  const float* x;    // [tokens, k]
  int k;
  int tokens;        // <= kGtMaxTokens
  int tiles;
  int split;         // CTAs per cluster: each takes 1 / split of k
  int nbl;           // most blocks of one rank's share of a row
};

// Matrix of global tile `tile` (tiles are numbered matrix by matrix).
__device__ __forceinline__ int GtMatrixOf(const GtArgs& a, int tile) {
  int mat = 0;
  while (mat + 1 < a.count && tile >= a.tile_begin[mat + 1]) ++mat;
  return mat;
}

__device__ __forceinline__ uint32_t GtMapRank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void GtClusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// 16 bytes into another CTA's shared memory, counted on its mbarrier.
__device__ __forceinline__ void GtSendRemote(uint32_t raddr, const float (&v)[4], uint32_t rbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];\n"
      ::"r"(raddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
      "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(rbar)
      : "memory");
}
__device__ __forceinline__ void GtArriveRemote(uint32_t rbar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(rbar)
               : "memory");
}


// x's digits for one block of 32 values of one token (thread-local): the
// block scale s = 2^(e - 6) (2^(e-1) <= max|x| < 2^e), four int8 digit rows
// written into the digit tile (row 4 t + j, bytes 32 (bl % 4) ..), the scale
// and the format's correction term (Q4_0: per-digit sums; Q4_1: sum of x).
// Rounding: r + 1.5 * 2^23 rounds r (|r| <= 64) to the nearest integer D,
// and the low byte of that float's bits is D as an int8.
template <int QT, int N>
__device__ __forceinline__ void GtDigitBlock(const float* __restrict__ xb, int bl, int t,
                                             uint8_t* digits, float* xscale, int* xcorr_i,
                                             float* xcorr_f) {
  float v[32];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(xb) + q);
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
  float mx = 0.0f;
  bool nan = false;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    mx = fmaxf(mx, fabsf(v[i]));
    nan |= v[i] != v[i];
  }
  const bool finite = !nan && mx <= 3.402823466e38f;
  int e = 0;
  frexpf(finite ? mx : 0.0f, &e);  // mx < 2^e (e = 0 for mx = 0)
  // r = x * 2^(6 - e) exactly, as two power-of-two factors (6 - e <= 155)
  const int sh = 6 - e;
  const float f1 = __int_as_float((127 + (sh < 127 ? sh : 127)) << 23);
  const float f2 = __int_as_float((127 + (sh > 127 ? sh - 127 : 0)) << 23);
  constexpr float kM = 12582912.0f;  // 1.5 * 2^23
  uint32_t dw[4][8];
  float dsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    uint32_t b[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float r = finite ? (v[4 * w + u] * f1) * f2 : 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float tb = r + kM;
        const float q = tb - kM;
        b[j][u] = __float_as_uint(tb);
        if constexpr (QT == MLB_Q4_0) dsum[j] += q;
        r = (r - q) * 128.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      dw[j][w] = __byte_perm(__byte_perm(b[j][0], b[j][1], 0x0040),
                             __byte_perm(b[j][2], b[j][3], 0x0040), 0x5410);
  }
  uint8_t* tilep = digits + (bl >> 2) * (N * 128);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = 4 * t + j;
    uint8_t* row = tilep + (n >> 3) * 1024 + (n & 7) * 128;
    const int c0 = 2 * (bl & 3);  // the block's two 16-byte chunks of the row
    *reinterpret_cast<uint4*>(row + ((c0 ^ (n & 7)) << 4)) =
        make_uint4(dw[j][0], dw[j][1], dw[j][2], dw[j][3]);
    *reinterpret_cast<uint4*>(row + (((c0 + 1) ^ (n & 7)) << 4)) =
        make_uint4(dw[j][4], dw[j][5], dw[j][6], dw[j][7]);
  }
  xscale[bl * kGtMaxTokens + t] = finite ? ldexpf(1.0f, e - 6) : __int_as_float(0x7fc00000);
  if constexpr (QT == MLB_Q4_0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) xcorr_i[(bl * kGtMaxTokens + t) * 4 + j] = static_cast<int>(dsum[j]);
  } else if constexpr (QT == MLB_Q4_1) {
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sum += v[i];
    xcorr_f[bl * kGtMaxTokens + t] = sum;
  }
}

}  // namespace

// Bounded waits of the tensor-core GEMV that gave up.
__device__ unsigned int g_gt_wait_timeouts;

namespace {

template <int QT, int T>  // T: tokens this instance computes (1, 2 or 4; a.tokens <= T)
__global__ void __launch_bounds__(kGtThreads, 1) GemvTcKernel(const __grid_constant__ GtArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  constexpr int SB = GtStageBlocks(QT);
  constexpr int CPS = SB / kGtChunk;  // chunks per stage (1 or 2)
  constexpr int N = GtN(T);
  constexpr int RA = GtASlots(T), RD = GtDSlots(T);
  constexpr int kDColumns = kGtChunk * N;
  constexpr uint32_t kIdesc = GtInstrDesc<QT, N>();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw_addr = GtSmem(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = GtSmem(base);
  const GtLayout lay = MakeGtLayout(QT, a.nbl, a.split, T);
  uint8_t* digits = base + lay.digits;
  uint8_t* raw = base + lay.raw;
  float* xscale = reinterpret_cast<float*>(base + lay.xscale);
  int* xcorr_i = reinterpret_cast<int*>(base + lay.xcorr);
  float* xcorr_f = reinterpret_cast<float*>(base + lay.xcorr);
  uint32_t* scale_ring = reinterpret_cast<uint32_t*>(base + lay.scales);
  float* red = reinterpret_cast<float*>(base + lay.red);
  const uint32_t bars = sbase + lay.bars;
  auto raw_full = [&](int s) { return bars + 8 * s; };
  auto raw_empty = [&](int s) { return bars + 8 * (kGtRawStages + s); };
  auto a_full = [&](int s) { return bars + 8 * (2 * kGtRawStages + s); };
  auto a_empty = [&](int s) { return bars + 8 * (2 * kGtRawStages + kGtMaxSlots + s); };
  auto d_full = [&](int s) { return bars + 8 * (2 * kGtRawStages + 2 * kGtMaxSlots + s); };
  auto d_empty = [&](int s) { return bars + 8 * (2 * kGtRawStages + 3 * kGtMaxSlots + s); };
  const uint32_t b_ready = bars + 8 * (2 * kGtRawStages + 4 * kGtMaxSlots);
  const uint32_t mma_done = b_ready + 8;
  auto red_full = [&](int p) { return b_ready + 8 * (2 + p); };   // on rank 0
  auto red_empty = [&](int p) { return b_ready + 8 * (4 + p); };  // on ranks 1..
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + lay.bars) + 2 * kGtBarriers;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // cluster of `split` CTAs per tile; rank r takes stages [s0, s0 + spt) of every row
  const int split = a.split;
  const int rank = static_cast<int>(blockIdx.x) % split;
  const int cluster = static_cast<int>(blockIdx.x) / split;
  const int clusters = static_cast<int>(gridDim.x) / split;
  const int spt_all = (a.k >> 5) / SB;
  const int s0 = rank * spt_all / split;
  const int spt = (rank + 1) * spt_all / split - s0;  // stages per tile (>= 1)
  const int kb0 = s0 * SB;                             // first block of the share
  const int nbl = spt * SB;
  const int cpt = nbl / kGtChunk;                      // chunks per tile
  const int my_tiles = cluster < a.tiles ? (a.tiles - cluster + clusters - 1) / clusters : 0;
  const int stages = my_tiles * spt;
  const int chunks = my_tiles * cpt;
  constexpr uint32_t kRedBytes = kGtRows * kGtMaxTokens * 4;  // one rank's partials

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGtRawStages; ++s) {
      GtBarInit(raw_full(s), 1);
      GtBarInit(raw_empty(s), 4);
    }
    for (int s = 0; s < RA; ++s) {
      GtBarInit(a_full(s), 4);
      GtBarInit(a_empty(s), 1);
    }
    for (int s = 0; s < RD; ++s) {
      GtBarInit(d_full(s), 1);
      GtBarInit(d_empty(s), 4);
    }
    GtBarInit(b_ready, 1);
    GtBarInit(mma_done, 1);
    for (int p = 0; p < 2; ++p) {
      GtBarInit(red_full(p), 1);
      GtBarInit(red_empty(p), kGtRows);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    // rank 0 expects the other ranks' partials of the first two tiles
    if (split > 1 && rank == 0)
      for (int p = 0; p < 2; ++p) GtExpectTx(red_full(p), (split - 1) * kRedBytes);
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     GtSmem(tmem_slot)),
                 "r"(kGtTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (split > 1) GtClusterSync();  // every rank's barriers exist before any remote access
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  auto a_col = [&](int s) { return static_cast<uint32_t>(s * kGtAColumns); };
  auto d_col = [&](int s) { return static_cast<uint32_t>(RA * kGtAColumns + s * kDColumns); };
  auto tile_of = [&](int iter) { return cluster + iter * clusters; };

  int issued = 0;  // producer: stages whose loads were issued
  if (warp == 8) {
    if (lane == 0) {
      for (int g = 0; g < stages; ++g) {
        const int st = g % kGtRawStages;
        if (!GtWait(raw_empty(st), ((g / kGtRawStages) & 1) ^ 1) || *abort_flag) {
          atomicAdd(&g_gt_wait_timeouts, 1u);
          *abort_flag = 1;
          break;
        }
        const int x0 = (s0 + g % spt) * SB * GtBlockBytes(QT);
        const int tile = tile_of(g / spt);
        const int mat = GtMatrixOf(a, tile);
        GtExpectTx(raw_full(st), kGtStageBytes);
        for (int b = 0; b < kGtBoxes; ++b)
          GtTmaLoad(GtSmem(raw + st * kGtStageBytes + b * kGtBoxBytes), &a.w[mat],
                    x0 + kGtBox * b, (tile - a.tile_begin[mat]) * kGtRows, raw_full(st));
        issued = g + 1;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      bool ok = GtWait(b_ready, 0) && !*abort_flag;
      if (!ok) {
        atomicAdd(&g_gt_wait_timeouts, 1u);
        *abort_flag = 1;
      }
      for (int c = 0; ok && c < chunks; ++c) {
        const int as = c % RA, ds = c % RD;
        if (!GtWait(a_full(as), (c / RA) & 1) || !GtWait(d_empty(ds), ((c / RD) & 1) ^ 1) ||
            *abort_flag) {
          atomicAdd(&g_gt_wait_timeouts, 1u);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        // block bl = 8 (c % cpt) + j: digit tile bl / 4, 32-byte k slice bl % 4
        const uint32_t bchunk = GtSmem(digits) + (c % cpt) * 2 * (N * 128);
#pragma unroll
        for (int j = 0; j < kGtChunk; ++j)
          GtMma(tmem + d_col(ds) + N * j, tmem + a_col(as) + 8 * j,
                GtDesc(bchunk + (j >> 2) * (N * 128) + 32 * (j & 3)), kIdesc);
        GtCommit(d_full(ds));   // results ready for the epilogue
        GtCommit(a_empty(as));  // codes consumed
      }
      GtCommit(mma_done);  // every MMA issued so far has finished
    }
  } else {
    // ---- x digits of this rank's share of k, written once (warps 0-7) ----
    for (int item = static_cast<int>(threadIdx.x); item < nbl * a.tokens; item += kGtMovers) {
      const int t = item / nbl, bl = item - t * nbl;  // neighbours read neighbouring blocks
      GtDigitBlock<QT, N>(a.x + static_cast<int64_t>(t) * a.k + (kb0 + bl) * 32, bl, t, digits,
                          xscale, xcorr_i, xcorr_f);
    }
    // digits are read by the tensor core (async proxy), the rest by warps 4-7
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    asm volatile("bar.sync 1, %0;\n" ::"n"(kGtMovers) : "memory");
    if (threadIdx.x == 0) GtArrive(b_ready);

    const int m = threadIdx.x & (kGtRows - 1);  // weight row within the tile (TMEM lane)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    bool ok = true;
    if (warp < 4) {
      // ---- movers: codes of chunk c -> tensor memory, scales -> shared ----
      for (int c = 0; c < chunks; ++c) {
        const int gs = c / CPS;  // stage index in this CTA's sequence
        const int st = gs % kGtRawStages;
        const int pos = c % CPS;  // which half of a 16-block stage (Q4)
        const int as = c % RA, ds = c % RD;
        if ((pos == 0 && !GtWait(raw_full(st), (gs / kGtRawStages) & 1)) ||
            !GtWait(a_empty(as), ((c / RA) & 1) ^ 1) ||
            !GtWait(d_empty(ds), ((c / RD) & 1) ^ 1) || *abort_flag) {
          ok = false;
          break;
        }
        const uint8_t* stage = raw + st * kGtStageBytes;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 4 blocks at a time
          uint32_t codes[32], sc[4];
          GtReadChunkAt<QT>(2 * pos + h, stage, m, codes, sc);
          GtStore32(lane_base + a_col(as) + 32 * h, codes);
#pragma unroll
          for (int j = 0; j < 4; ++j) scale_ring[(ds * kGtChunk + 4 * h + j) * kGtRows + m] = sc[j];
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          GtArrive(a_full(as));
          if (pos == CPS - 1) GtArrive(raw_empty(st));  // stage fully read
        }
      }
    } else {
      // ---- epilogue: chunk c's int32 results -> the rows' fp32 sums ----
      float acc[kGtMaxTokens] = {0.0f, 0.0f, 0.0f, 0.0f};
      int tile_iter = 0;
      for (int c = 0; c < chunks; ++c) {
        const int ds = c % RD;
        if (!GtWait(d_full(ds), (c / RD) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const int cl = c % cpt;
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 4 blocks at a time
          int r[4][N];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (N == 8) GtLoad8(lane_base + d_col(ds) + N * (4 * h + j), r[j]);
            else GtLoad16(lane_base + d_col(ds) + N * (4 * h + j), r[j]);
          }
          uint32_t sw[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) sw[j] = scale_ring[(ds * kGtChunk + 4 * h + j) * kGtRows + m];
          asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
          if (h == 1) {  // both halves read: the slot may be refilled
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) GtArrive(d_empty(ds));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int bl = kGtChunk * cl + 4 * h + j;
            const float d =
                __half2float(__ushort_as_half(static_cast<unsigned short>(sw[j] & 0xFFFFu)));
#pragma unroll
            for (int t = 0; t < T; ++t) {
              int q0 = r[j][4 * t], q1 = r[j][4 * t + 1], q2 = r[j][4 * t + 2],
                  q3 = r[j][4 * t + 3];
              if constexpr (QT == MLB_Q4_0) {
                const int4 s4 =
                    *reinterpret_cast<const int4*>(xcorr_i + (bl * kGtMaxTokens + t) * 4);
                q0 -= 8 * s4.x;
                q1 -= 8 * s4.y;
                q2 -= 8 * s4.z;
                q3 -= 8 * s4.w;
              }
              float hv = fmaf(static_cast<float>(q3), 0.0078125f, static_cast<float>(q2));
              hv = fmaf(hv, 0.0078125f, static_cast<float>(q1));
              hv = fmaf(hv, 0.0078125f, static_cast<float>(q0));
              acc[t] = fmaf(d * xscale[bl * kGtMaxTokens + t], hv, acc[t]);
              if constexpr (QT == MLB_Q4_1) {
                const float mn =
                    __half2float(__ushort_as_half(static_cast<unsigned short>(sw[j] >> 16)));
                acc[t] = fmaf(mn, xcorr_f[bl * kGtMaxTokens + t], acc[t]);
              }
            }
          }
        }
        if (cl == cpt - 1) {  // the tile's last chunk: its rows are done
          const int p = tile_iter & 1;
          const uint32_t par = (tile_iter >> 1) & 1;
          float tot[kGtMaxTokens];
#pragma unroll
          for (int t = 0; t < kGtMaxTokens; ++t) tot[t] = acc[t];
          if (rank > 0) {  // this rank's partials -> rank 0
            if (!GtWait(red_empty(p), par ^ 1)) {
              ok = false;
              break;
            }
            const uint32_t slot_addr =
                GtSmem(red + ((p * split + rank) * kGtRows + m) * kGtMaxTokens);
            GtSendRemote(GtMapRank(slot_addr, 0), tot, GtMapRank(red_full(p), 0));
          } else {
            if (split > 1) {  // add ranks 1 .. split-1 in order
              if (!GtWait(red_full(p), par)) {
                ok = false;
                break;
              }
              for (int q = 1; q < split; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(
                    red + ((p * split + q) * kGtRows + m) * kGtMaxTokens);
                tot[0] += v.x;
                tot[1] += v.y;
                tot[2] += v.z;
                tot[3] += v.w;
              }
              // the next use of this buffer: expect the bytes again, then let
              // every rank write it
              if (m == 0) GtExpectTx(red_full(p), (split - 1) * kRedBytes);
              for (int q = 1; q < split; ++q)
                GtArriveRemote(GtMapRank(red_empty(p), static_cast<uint32_t>(q)));
            }
            const int tile = tile_of(tile_iter);
            const int mat = GtMatrixOf(a, tile);
            const int n = a.n[mat];
            const int row = (tile - a.tile_begin[mat]) * kGtRows + m;
            if (row < n) {
              for (int t = 0; t < a.tokens; ++t) a.y[mat][static_cast<int64_t>(t) * n + row] = tot[t];
            }
          }
#pragma unroll
          for (int t = 0; t < kGtMaxTokens; ++t) acc[t] = 0.0f;
          ++tile_iter;
        }
      }
    }
    if (!ok) {
      if (lane == 0) atomicAdd(&g_gt_wait_timeouts, 1u);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // let loads and MMAs in flight finish, then mark every output of this
    // cluster's tiles as failed
    if (warp == 8 && lane == 0) {
      for (int g = issued - kGtRawStages > 0 ? issued - kGtRawStages : 0; g < issued; ++g)
        GtWait(raw_full(g % kGtRawStages), (g / kGtRawStages) & 1);
    }
    if (warp < 4) {
      for (int ti = 0; ti < my_tiles; ++ti) {
        const int tile = tile_of(ti);
        const int mat = GtMatrixOf(a, tile);
        const int n = a.n[mat];
        const int row = (tile - a.tile_begin[mat]) * kGtRows + static_cast<int>(threadIdx.x);
        if (row < n)
          for (int t = 0; t < a.tokens; ++t)
            a.y[mat][static_cast<int64_t>(t) * n + row] = __int_as_float(0x7fc00000);
      }
    }
  }
  if (warp == 9 && lane == 0) GtWait(mma_done, 0);
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  // no rank leaves while another may still write to its shared memory
  if (split > 1) GtClusterSync();
  if (warp == 9) {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kGtTmemColumns)
                 : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 GtEncodeFn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// Ranks per tile (1, 2, 4 or 8) for `tiles` 128-row tiles of width k: as
// many as keep one cluster per tile within one wave of CTAs, each rank with
// at least one stage, and enough that a rank's digits of x fit in shared
// memory; 0 when no split works.
int GtSplit(int qtype, int64_t tiles, int64_t k, int tokens) {
  const int sb = GtStageBlocks(qtype);
  const int64_t spt = k / 32 / sb;
  const int digit_bytes = GtN(tokens) * 32;  // per block
  int split = 1;
  while (split < 8 && tiles * split * 2 <= SmCount() && spt >= 2 * split) split *= 2;
  auto share_blocks = [&](int s) { return (spt + s - 1) / s * sb; };
  while (split < 8 && share_blocks(split) * digit_bytes > kGtMaxDigitBytes && spt >= 2 * split)
    split *= 2;
  if (share_blocks(split) * digit_bytes > kGtMaxDigitBytes) return 0;
  if (MakeGtLayout(qtype, static_cast<int>(share_blocks(split)), split, tokens).total + 1024 >
      227 * 1024)
    return 0;
  return split;
}

int64_t GtTiles(int count, const int64_t* n) {
  int64_t tiles = 0;
  for (int m = 0; m < count; ++m) tiles += (n[m] + kGtRows - 1) / kGtRows;
  return tiles;
}

int GtTokenClass(int tokens) { return tokens <= 1 ? 1 : (tokens <= 2 ? 2 : 4); }

template <int QT>
int LaunchGemvTc(int count, const void* const* w, const int64_t* n, int64_t k, const float* x,
                 int tokens, float* const* y, int split, cudaStream_t s) {
  GtArgs a{};
  const int64_t row_bytes = mlb_row_bytes(QT, k);
  PFN_cuTensorMapEncodeTiled_v12000 encode = GtEncodeFn();
  if (encode == nullptr) return Fail(MLB_ERR_CUDA, "mlb_linear_f32: tensor map encoding failed");
  int tiles = 0;
  for (int m = 0; m < count; ++m) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes),
                                static_cast<cuuint64_t>(n[m])};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {kGtBox, kGtRows};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&a.w[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w[m]), dims, strides,
               box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return Fail(MLB_ERR_CUDA, "mlb_linear_f32: tensor map encoding failed");
    a.y[m] = y[m];
    a.n[m] = static_cast<int>(n[m]);
    a.tile_begin[m] = tiles;
    tiles += static_cast<int>((n[m] + kGtRows - 1) / kGtRows);
  }
  a.tile_begin[count] = tiles;
  a.count = count;
  constexpr int sb = GtStageBlocks(QT);
  const int spt = static_cast<int>(k / 32 / sb);
  a.x = x;
  a.k = static_cast<int>(k);
  a.tokens = tokens;
  a.tiles = tiles;
  a.split = split;
  a.nbl = (spt + split - 1) / split * sb;
  const int tclass = GtTokenClass(tokens);
  const int shm = MakeGtLayout(QT, a.nbl, split, tclass).total + 1024;
  auto kernel = tclass == 1 ? GemvTcKernel<QT, 1>
                            : (tclass == 2 ? GemvTcKernel<QT, 2> : GemvTcKernel<QT, 4>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, shm) !=
      cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "mlb_linear_f32: shared memory opt-in");
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(split));
  cfg.blockDim = dim3(kGtThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(shm);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see Launch
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent clusters: as many as fit on the GPU at once (one CTA per SM),
  // found once per format and split size
  static int resident[3][4] = {};
  int& fit = resident[QT - MLB_Q8_0][split == 1 ? 0 : (split == 2 ? 1 : (split == 4 ? 2 : 3))];
  if (fit <= 0) {
    int found = 0;
    if (cudaOccupancyMaxActiveClusters(&found, kernel, &cfg) != cudaSuccess || found < 1) {
      cudaGetLastError();
      found = SmCount() / split > 0 ? SmCount() / split : 1;
    }
    fit = found;
  }
  const int clusters = fit < tiles ? fit : tiles;
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * split));
  cfg.numAttrs = LaunchOverlap() ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kernel, a) != cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "mlb_linear_f32: launch failed");
  }
  return CheckLaunch("mlb_linear_f32");
}

}  // namespace

// Ranks per 128-row tile the tensor-core GEMV would use for the `count`
// matrices W[m] [n[m], k] of format qtype (1, 2, 4 or 8) with `tokens`
// tokens per pass, or 0 when it does not take them: ggml blocks only,
// 16-byte aligned tables, whole stages per row, x's digits of a rank's
// share of k within the shared-memory budget.
int GemvTcSplit(int qtype, int count, const void* const* w, const int64_t* n, int64_t k,
                int tokens) {
  if (qtype != MLB_Q8_0 && qtype != MLB_Q4_0 && qtype != MLB_Q4_1) return 0;
  if (count < 1 || count > kGtMaxGroup || k > INT_MAX) return 0;
  for (int m = 0; m < count; ++m)
    if ((reinterpret_cast<uintptr_t>(w[m]) & 15u) != 0 || n[m] <= 0 || n[m] > INT_MAX) return 0;
  if (k % (32 * GtStageBlocks(qtype)) != 0) return 0;
  const int64_t tiles = GtTiles(count, n);
  if (tiles > INT_MAX / 2) return 0;
  return GtSplit(qtype, tiles, k, GtTokenClass(tokens));
}


// y[m][t] = W[m] . x[t] for t < tokens (1..4) and m < count on the tensor
// cores, `split` ranks per tile (from GemvTcSplit).
int GemvTc(int qtype, int count, const void* const* w, const int64_t* n, int64_t k,
           const float* x, int tokens, float* const* y, int split, cudaStream_t s) {
  if (tokens < 1 || tokens > kGtMaxTokens)
    return Fail(MLB_ERR_ARG, "mlb_linear_f32: bad token group");
  switch (qtype) {
    case MLB_Q8_0: return LaunchGemvTc<MLB_Q8_0>(count, w, n, k, x, tokens, y, split, s);
    case MLB_Q4_0: return LaunchGemvTc<MLB_Q4_0>(count, w, n, k, x, tokens, y, split, s);
    default: return LaunchGemvTc<MLB_Q4_1>(count, w, n, k, x, tokens, y, split, s);
  }
}

unsigned int GemvTcWaitTimeouts() {
  unsigned int count = 0;
  if (cudaMemcpyFromSymbol(&count, g_gt_wait_timeouts, sizeof(count)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count;
}

}  // namespace mlb
