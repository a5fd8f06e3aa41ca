// Prompt-sized Q8_0 / Q4_0 linear layers on the fp16 tensor cores:
// y[t] = W . x[t], W [n, k] in ggml blocks, x [T, k] fp32 — the form
// mlb_linear_rows_f32 takes for these two formats.
//
// Reference arithmetic (src/quant.cc:171-226 LinearWithBlocks): per output a
// sequential fp32 sum of (d * q_i) * x_i, with q_i the int8 code (Q8_0) or
// n_i - 8 (Q4_0) and d the block's fp16 scale.
//
// Method: a dequantised weight w = d * q is split into two fp16 pieces
// without error.  d is an fp16 number, so d and q * d (|q| <= 128) are
// integer multiples of 2^-24, fp16's smallest step; hi = RN_fp16(q * d) is one
// too, and the remainder lo = q * d - hi is a multiple of 2^-24 with at most 8
// significant bits — an fp16 number.  Both come from two packed fp16
// operations: hi by a rounded multiply, lo by a fused multiply-add of q, d
// and -hi (exact because its result is representable).  That holds while
// |q * d| <= 65504, i.e. |d| < 512; a tile that meets a larger or non-finite
// block scale is recomputed on the CUDA cores (below).  Each token row of x
// is scaled by a power of two s_t (its largest magnitude lands in
// [2^14, 2^15)) and split into two fp16 pieces, x / s_t = xh + xl + r,
// |r| <= 2^-22 |x / s_t| (plus 2^-25 below fp16's normal range, i.e. 2^-39
// of the row's largest value).  Per (128-row, 128-token) tile the tensor core
// sums hi.xh + hi.xl + lo.xh over the whole of k into one fp32 accumulator
// (tcgen05.mma kind::f16, K = 16: 3 MMAs per 16 values; every product is
// exact, the dropped lo.xl is below 2^-23 of each term), and the epilogue
// multiplies by s_t.  No per-block rescaling interrupts the accumulation, so
// the MMAs of consecutive stages queue back to back.  Results stay within
// the tests' 1e-5 * sum |w_i x_i| of the reference.  A row of x holding Inf
// or NaN keeps s_t = 1, so the non-finite values reach its outputs.
//
// Design (one CTA = 128 weight rows x 128 tokens, k in stages of two blocks;
// 320 threads in warp roles):
//   - warp 8, one lane: TMA producer.  Per stage: the raw bytes of the 128
//     rows' two blocks (a 2-D uint8 map over [n, row_bytes], box 128 bytes
//     from the stage's byte offset rounded down to 16, which covers two 34-
//     or 18-byte blocks) and the two 128-token x 64-value fp16 tiles of x's
//     pieces, all with a 128-byte swizzle (bank-conflict-free row reads; the
//     MMA descriptors use the same layout); 4 stages of 48 KB in flight;
//   - warps 0-7, two threads per weight row (= tensor-memory lane), warps
//     0-3 the stage's first block and 4-7 its second: turn the block's codes
//     into fp16 pairs (a byte permute builds 1024 + byte in both halves, one
//     packed subtract), form hi and lo, and store them into tensor memory
//     (tcgen05.st, the A operands: 16 columns each per block); at the end
//     the same warps read the accumulator (tcgen05.ld) and store s_t * sum;
//   - warp 9: allocates tensor memory; one lane issues the 12 MMAs of each
//     stage into the accumulator and commits the stage's buffers.
// Every wait is bounded: a wait that gives up is counted (mlb_wait_timeouts)
// and the CTA writes NaN instead of its tile.
//
// CUDA-core tile (block scales with |d| >= 512, Inf or NaN): the movers flag
// such a block; the CTA then computes each of its outputs as the GEMV does —
// per block the fp32 sum of q_i x_i, times d, summed over the blocks — which
// keeps the reference's Inf / NaN behaviour.  Real model weights have
// |d| far below 512; the path exists so that no input gives a wrong result.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kHfRows = 128;        // weight rows (MMA M)
constexpr int kHfTokens = 128;      // tokens (MMA N)
constexpr int kHfStageK = 64;       // values per stage: two ggml blocks
constexpr int kHfStages = 4;
constexpr int kHfPieces = 2;        // fp16 pieces of x
constexpr int kHfMovers = 8;        // warps 0-7: A operands, then the epilogue
constexpr int kHfThreads = 320;     // movers 0-7, producer 8, MMA 9
constexpr int kHfRawBytes = kHfRows * 128;               // raw weight box per stage
constexpr int kHfPieceBytes = kHfTokens * kHfStageK * 2; // one fp16 x piece per stage
constexpr int kHfStageBytes = kHfRawBytes + kHfPieces * kHfPieceBytes;
constexpr int kHfTmemColumns = 512;
constexpr int kHfAccColumns = kHfTokens;  // the fp32 accumulator
constexpr int kHfAColumns = 64;           // per stage: hi (2 blocks x 16), then lo
constexpr int kHfMaxGroup = 3;

__host__ __device__ constexpr int HfBlockBytes(int qt) { return qt == MLB_Q8_0 ? 34 : 18; }

// Shared memory from a 1024-byte aligned base: kHfStages stages (raw box,
// then x's pieces), the barriers, the TMEM address and two flags.
constexpr int kHfBarOffset = kHfStages * kHfStageBytes;
// raw_full / raw_empty / a_full / a_empty per stage, acc_full, mma_done
constexpr int kHfBarriers = 4 * kHfStages + 2;
constexpr int kHfSmemBytes = kHfBarOffset + 8 * kHfBarriers + 16 + 1024;

__device__ __forceinline__ uint32_t HfSmem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void HfBarInit(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void HfExpectTx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void HfArrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool HfTryWait(uint32_t bar, uint32_t parity) {
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
__device__ __forceinline__ bool HfWait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 21); ++i)
    if (HfTryWait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void HfTmaLoad(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// K-major operand, 128-byte swizzle, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t HfDesc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// Instruction descriptor: D fp32, A and B fp16, both K-major, N = 128, M = 128.
constexpr uint32_t kHfInstrDesc = (1u << 4) | (0u << 7) | (0u << 10) |
                                  (static_cast<uint32_t>(kHfTokens >> 3) << 17) |
                                  (static_cast<uint32_t>(kHfRows >> 4) << 24);
__device__ __forceinline__ void HfMma(uint32_t d, uint32_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(kHfInstrDesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void HfCommit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void HfStore16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void HfLoad32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Four byte values of u -> two fp16 pairs (values 0, 1 and 2, 3): a byte
// permute puts 0x64 above each byte, i.e. the fp16 1024 + byte, and one
// packed subtract of `bias` (1024 + offset) leaves byte - offset, exact.
__device__ __forceinline__ void HfWordPairs(uint32_t u, uint32_t bias2, uint32_t& p0,
                                            uint32_t& p1) {
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);  // bytes 0, 1
  const uint32_t b = __byte_perm(u, 0x64646464u, 0x5342);  // bytes 2, 3
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(p0) : "r"(a), "r"(bias2));
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(p1) : "r"(b), "r"(bias2));
}
constexpr uint32_t kHfBiasQ8 = 0x64806480u;  // fp16 pair (1152, 1152): 1024 + 128
constexpr uint32_t kHfBiasQ4 = 0x64086408u;  // fp16 pair (1032, 1032): 1024 + 8

// A code pair q (fp16 x2) and the block scale pair (d, d), -d: the exact
// pieces hi = RN(q d) and lo = q d - hi (see the top of the file).
__device__ __forceinline__ void HfSplitPair(uint32_t q, uint32_t d2, uint32_t nd2, uint32_t& hi,
                                            uint32_t& lo) {
  uint32_t nh;
  asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(nh) : "r"(q), "r"(nd2));         // -hi
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(lo) : "r"(q), "r"(d2), "r"(nh));
  hi = nh ^ 0x80008000u;
}

// Block J (0 or 1) of a raw stage, row m (its 128-byte swizzled box row; the
// stage's first block starts at byte 4R): the 16 hi and 16 lo A columns (fp16
// pairs in K order) and the block scale's bits.
template <int QT, int R, int J>
__device__ __forceinline__ void HfTakeBlock(const uint8_t* raw_row, int m, uint32_t (&hi)[16],
                                            uint32_t (&lo)[16], uint32_t& dbits) {
  // 16-byte chunks holding the block: Q8_0 bytes [4R + 34J, 4R + 34J + 34),
  // Q4_0 bytes [4R + 18J, 4R + 18J + 18), R <= 3
  constexpr int kC0 = QT == MLB_Q8_0 ? 2 * J : J;
  constexpr int kC1 = QT == MLB_Q8_0 ? 2 * J + 2 : J + 1;
  uint32_t w[4 * kC1 + 4];
#pragma unroll
  for (int c = kC0; c <= kC1; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(raw_row + 16 * (c ^ (m & 7)));
    w[4 * c] = v.x;
    w[4 * c + 1] = v.y;
    w[4 * c + 2] = v.z;
    w[4 * c + 3] = v.w;
  }
  uint32_t q[16];
  if constexpr (QT == MLB_Q8_0) {
    // block 0: scale in the low half of word R, codes from byte 4R + 2 (a
    // half-word shift); block 1 (byte 4R + 34): scale in the high half of
    // word R + 8, codes word-aligned from word R + 9
    dbits = J == 0 ? (w[R] & 0xFFFFu) : (w[R + 8] >> 16);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t c = J == 0 ? __funnelshift_r(w[R + i], w[R + i + 1], 16) : w[R + 9 + i];
      HfWordPairs(c ^ 0x80808080u, kHfBiasQ8, q[2 * i], q[2 * i + 1]);
    }
  } else {
    // Q4_0: block 0 nibbles from byte 4R + 2, block 1 (byte 4R + 18): scale
    // in the high half of word R + 4, nibbles word-aligned from word R + 5;
    // values 0-15 are the low nibbles, 16-31 the high ones
    dbits = J == 0 ? (w[R] & 0xFFFFu) : (w[R + 4] >> 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = J == 0 ? __funnelshift_r(w[R + i], w[R + i + 1], 16) : w[R + 5 + i];
      HfWordPairs(u & 0x0F0F0F0Fu, kHfBiasQ4, q[2 * i], q[2 * i + 1]);
      HfWordPairs((u >> 4) & 0x0F0F0F0Fu, kHfBiasQ4, q[8 + 2 * i], q[8 + 2 * i + 1]);
    }
  }
  const uint32_t d2 = dbits | (dbits << 16);
  const uint32_t nd2 = d2 ^ 0x80008000u;
#pragma unroll
  for (int i = 0; i < 16; ++i) HfSplitPair(q[i], d2, nd2, hi[i], lo[i]);
}

template <int QT, int J>
__device__ __forceinline__ void HfTakeBlockAt(int r, const uint8_t* raw_row, int m,
                                              uint32_t (&hi)[16], uint32_t (&lo)[16],
                                              uint32_t& dbits) {
  switch (r) {
    case 0: HfTakeBlock<QT, 0, J>(raw_row, m, hi, lo, dbits); break;
    case 1: HfTakeBlock<QT, 1, J>(raw_row, m, hi, lo, dbits); break;
    case 2: HfTakeBlock<QT, 2, J>(raw_row, m, hi, lo, dbits); break;
    default: HfTakeBlock<QT, 3, J>(raw_row, m, hi, lo, dbits); break;
  }
}

struct HfGroup {
  CUtensorMap w[kHfMaxGroup];  // raw weight bytes of each matrix
  CUtensorMap x[kHfPieces];    // x's fp16 pieces [T, k]
  const uint8_t* wp[kHfMaxGroup];  // the same weights, for the CUDA-core tile
  float* y[kHfMaxGroup];
  const float* x32;            // x [T, k] fp32, for the CUDA-core tile
  const float* row_scale;      // s_t per token
  int64_t row_bytes;
  int n[kHfMaxGroup];
  int tile_begin[kHfMaxGroup + 1];  // first tile of each matrix; [count] = total
  int count;
  int t_tiles;
  int t_rows;
  int k;
};

// The tile's outputs on the CUDA cores: per output and block the fp32 sum
// of q_i x_i, times d, summed over the blocks (lanes take blocks, then a
// warp reduction).
template <int QT>
__device__ void HfCudaCoreTile(const HfGroup& grp, int mat, int n0, int t0) {
  constexpr int kBB = HfBlockBytes(QT);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nb = grp.k / 32;
  const int n = grp.n[mat];
  for (int r = warp; r < kHfRows && n0 + r < n; r += kHfThreads / 32) {
    const uint8_t* wrow = grp.wp[mat] + static_cast<int64_t>(n0 + r) * grp.row_bytes;
    for (int t = t0; t < t0 + kHfTokens && t < grp.t_rows; ++t) {
      const float* xr = grp.x32 + static_cast<int64_t>(t) * grp.k;
      float acc = 0.0f;
      for (int b = lane; b < nb; b += 32) {
        const uint8_t* blk = wrow + b * kBB;
        const float d = __half2float(*reinterpret_cast<const __half*>(blk));
        const float* xb = xr + 32 * b;
        float sum = 0.0f;
        if constexpr (QT == MLB_Q8_0) {
#pragma unroll 8
          for (int i = 0; i < 32; ++i)
            sum = fmaf(static_cast<float>(static_cast<int8_t>(blk[2 + i])), xb[i], sum);
        } else {
#pragma unroll 8
          for (int i = 0; i < 16; ++i)
            sum = fmaf(static_cast<float>((blk[2 + i] & 15) - 8), xb[i], sum);
#pragma unroll 8
          for (int i = 0; i < 16; ++i)
            sum = fmaf(static_cast<float>((blk[2 + i] >> 4) - 8), xb[16 + i], sum);
        }
        acc = fmaf(d, sum, acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) grp.y[mat][static_cast<int64_t>(t) * n + n0 + r] = acc;
    }
  }
}

}  // namespace

// Bounded waits of this file's kernel that gave up.
__device__ unsigned int g_hf_wait_timeouts;

namespace {

template <int QT>
__global__ void __launch_bounds__(kHfThreads, 1)
    LinearF16Kernel(const __grid_constant__ HfGroup grp) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  constexpr int kBB = HfBlockBytes(QT);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw_addr = HfSmem(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = HfSmem(base);
  auto stage_base = [&](int s) { return base + s * kHfStageBytes; };
  const uint32_t bars = sbase + kHfBarOffset;
  auto raw_full = [&](int s) { return bars + 8 * s; };
  auto raw_empty = [&](int s) { return bars + 8 * (kHfStages + s); };
  auto a_full = [&](int s) { return bars + 8 * (2 * kHfStages + s); };
  auto a_empty = [&](int s) { return bars + 8 * (3 * kHfStages + s); };
  const uint32_t acc_full = bars + 8 * (4 * kHfStages);
  const uint32_t mma_done = bars + 8 * (4 * kHfStages + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kHfBarOffset + 8 * kHfBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* cuda_core_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int mat = 0;
  while (mat + 1 < grp.count && static_cast<int>(blockIdx.x) >= grp.tile_begin[mat + 1]) ++mat;
  const int local = static_cast<int>(blockIdx.x) - grp.tile_begin[mat];
  const int n0 = (local / grp.t_tiles) * kHfRows;
  const int t0 = (local % grp.t_tiles) * kHfTokens;
  const int n = grp.n[mat];
  const int stages = grp.k / kHfStageK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHfStages; ++s) {
      HfBarInit(raw_full(s), 1);
      HfBarInit(raw_empty(s), kHfMovers + 1);  // the mover warps + the MMA commit
      HfBarInit(a_full(s), kHfMovers);
      HfBarInit(a_empty(s), 1);
    }
    HfBarInit(acc_full, 1);
    HfBarInit(mma_done, 1);
    *abort_flag = 0;
    *cuda_core_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     HfSmem(tmem_slot)),
                 "r"(kHfTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // tensor-memory columns: the accumulator, then the A ring
  auto a_col = [&](int s) { return static_cast<uint32_t>(kHfAccColumns + s * kHfAColumns); };

  int issued = 0;  // producer: stages whose loads were issued
  if (warp == 8) {
    if (lane == 0) {
      for (int s = 0; s < stages; ++s) {
        const int st = s % kHfStages;
        if (!HfWait(raw_empty(st), ((s / kHfStages) & 1) ^ 1) || *abort_flag) {
          atomicAdd(&g_hf_wait_timeouts, 1u);
          *abort_flag = 1;
          break;
        }
        uint8_t* sb = stage_base(st);
        HfExpectTx(raw_full(st), kHfStageBytes);
        const int xw = (s * 2 * kBB) & ~15;  // the two blocks' bytes, from the 16-byte floor
        HfTmaLoad(HfSmem(sb), &grp.w[mat], xw, n0, raw_full(st));
        for (int p = 0; p < kHfPieces; ++p)
          HfTmaLoad(HfSmem(sb + kHfRawBytes + p * kHfPieceBytes), &grp.x[p], s * kHfStageK, t0,
                    raw_full(st));
        issued = s + 1;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // shared-memory descriptors are built once: an offset below 256 KB adds
      // to the descriptor's 14-bit address field (in 16-byte units)
      const uint64_t desc0 = HfDesc(HfSmem(stage_base(0) + kHfRawBytes));
      bool ok = true;
      for (int s = 0; s < stages; ++s) {
        const int st = s % kHfStages;
        if (!HfWait(raw_full(st), (s / kHfStages) & 1) ||
            !HfWait(a_full(st), (s / kHfStages) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint64_t desc = desc0 + static_cast<uint64_t>(st * (kHfStageBytes >> 4));
        const uint32_t a_st = tmem + a_col(st);
#pragma unroll
        for (int j = 0; j < 2; ++j)      // the stage's two blocks
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // K = 16 per MMA: 32 bytes of the 128-byte rows
            const uint32_t a_hi = a_st + 16 * j + 8 * h;
            const uint64_t bh = desc + ((64 * j + 32 * h) >> 4);
            const uint64_t bl = desc + ((kHfPieceBytes + 64 * j + 32 * h) >> 4);
            HfMma(tmem, a_hi, bh, (s | j | h) != 0);
            HfMma(tmem, a_hi, bl, 1);
            HfMma(tmem, a_hi + 32, bh, 1);
          }
        HfCommit(a_empty(st));
        HfCommit(raw_empty(st));
      }
      if (ok) {
        HfCommit(acc_full);
      } else {
        atomicAdd(&g_hf_wait_timeouts, 1u);
        *abort_flag = 1;
      }
    }
  } else {
    // ---- movers: block j of each stage -> hi / lo pairs in tensor memory ----
    const int j = warp >> 2;                  // the stage's block
    const int m = (warp & 3) * 32 + lane;     // weight row within the tile (TMEM lane)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t big = 0;
    for (int s = 0; s < stages; ++s) {
      const int st = s % kHfStages;
      // one decision per warp: the tensor-memory stores below need all lanes
      const bool ready = HfWait(raw_full(st), (s / kHfStages) & 1) &&
                         HfWait(a_empty(st), ((s / kHfStages) & 1) ^ 1) && !*abort_flag;
      if (!__all_sync(0xffffffffu, ready)) {
        if (lane == 0) atomicAdd(&g_hf_wait_timeouts, 1u);
        *abort_flag = 1;
        break;
      }
      uint32_t hi[16], lo[16], dbits;
      const int r = ((s * 2 * kBB) & 15) >> 2;
      if (j == 0)
        HfTakeBlockAt<QT, 0>(r, stage_base(st) + m * 128, m, hi, lo, dbits);
      else
        HfTakeBlockAt<QT, 1>(r, stage_base(st) + m * 128, m, hi, lo, dbits);
      big |= (dbits & 0x7FFFu) >= 0x6000u;  // |d| >= 512, Inf or NaN
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      HfStore16(lane_base + a_col(st) + 16 * j, hi);
      HfStore16(lane_base + a_col(st) + 32 + 16 * j, lo);
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        HfArrive(a_full(st));
        HfArrive(raw_empty(st));  // this warp is done with the raw box
      }
    }
    if (__any_sync(0xffffffffu, big) && lane == 0) *cuda_core_flag = 1;
  }

  __syncthreads();
  const bool cuda_core = *cuda_core_flag != 0;
  if (warp < kHfMovers && !*abort_flag && !cuda_core) {
    // ---- epilogue: warps w and w + 4 share lanes 32 (w & 3).., 64 tokens each ----
    if (!__all_sync(0xffffffffu, HfWait(acc_full, 0))) {
      if (lane == 0) atomicAdd(&g_hf_wait_timeouts, 1u);
      *abort_flag = 1;
    } else {
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const int q = warp & 3;
      const int half = warp >> 2;
      const int row = n0 + q * 32 + lane;
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
      float* y = grp.y[mat];
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 32 tokens at a time
        float v[32];
        HfLoad32(lane_base + 64 * half + 32 * c, v);
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        if (row < n) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = t0 + 64 * half + 32 * c + i;
            if (t < grp.t_rows)
              y[static_cast<int64_t>(t) * n + row] = v[i] * __ldg(grp.row_scale + t);
          }
        }
      }
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // let the loads in flight land and mark the whole tile as failed
    if (warp == 8 && lane == 0) {
      for (int s = issued - kHfStages > 0 ? issued - kHfStages : 0; s < issued; ++s)
        HfWait(raw_full(s % kHfStages), (s / kHfStages) & 1);
    }
    if (warp < 4) {
      const int row = n0 + static_cast<int>(threadIdx.x);
      if (row < n)
        for (int t = t0; t < t0 + kHfTokens && t < grp.t_rows; ++t)
          grp.y[mat][static_cast<int64_t>(t) * n + row] = __int_as_float(0x7fc00000);
    }
  } else if (cuda_core) {
    HfCudaCoreTile<QT>(grp, mat, n0, t0);
  }
  if (warp == 9 && lane == 0) {
    // every MMA issued has finished before the tensor memory is released
    HfCommit(mma_done);
    HfWait(mma_done, 0);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 9) {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kHfTmemColumns)
                 : "memory");
  }
}

// One token row of x -> its power-of-two scale s_t (largest |x| / s_t in
// [2^14, 2^15); 1 for an all-zero or non-finite row) and the two fp16
// pieces of x / s_t.  One CTA per row.
__global__ void __launch_bounds__(256)
    SplitF16Kernel(const float* __restrict__ x, __half* __restrict__ xh, __half* __restrict__ xl,
                   float* __restrict__ row_scale, int k) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float red[8];
  __shared__ int bad_row;
  const int64_t t = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + t * k);
  const int k4 = k >> 2;
  float mx = 0.0f;
  int bad = 0;
  for (int i = threadIdx.x; i < k4; i += blockDim.x) {
    const float4 v = xr[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    bad |= !(fabsf(v.x) <= 3.402823466e38f) | !(fabsf(v.y) <= 3.402823466e38f) |
           !(fabsf(v.z) <= 3.402823466e38f) | !(fabsf(v.w) <= 3.402823466e38f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  bad = __any_sync(0xffffffffu, bad);
  if (threadIdx.x == 0) bad_row = 0;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = mx;
    if (bad) bad_row = 1;
  }
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < (blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  // s = 2^(e - 15) with mx < 2^e: mx / s in [2^14, 2^15); e is kept >= -111
  // so that s and 1 / s stay normal (rows below 2^-112 land lower)
  int e = 0;
  frexpf(mx, &e);
  e = e < -111 ? -111 : e;
  const bool plain = bad_row || mx == 0.0f;
  const float s = plain ? 1.0f : ldexpf(1.0f, e - 15);
  const float inv = plain ? 1.0f : ldexpf(1.0f, 15 - e);
  if (threadIdx.x == 0) row_scale[t] = s;
  __half2* h2 = reinterpret_cast<__half2*>(xh + t * k);
  __half2* l2 = reinterpret_cast<__half2*>(xl + t * k);
  for (int i = threadIdx.x; i < k4; i += blockDim.x) {
    const float4 v = xr[i];
    const float a[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};  // exact
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hi[j] = __float2half_rn(a[j]);
      lo[j] = __float2half_rn(a[j] - __half2float(hi[j]));  // exact remainder
    }
    h2[2 * i] = __halves2half2(hi[0], hi[1]);
    h2[2 * i + 1] = __halves2half2(hi[2], hi[3]);
    l2[2 * i] = __halves2half2(lo[0], lo[1]);
    l2[2 * i + 1] = __halves2half2(lo[2], lo[3]);
  }
}

// The same split with the row held in registers (NV float4 per thread of
// 512, rows of up to 16384 values): x is read once.
template <int NV>
__global__ void __launch_bounds__(512)
    SplitF16RegKernel(const float* __restrict__ x, __half* __restrict__ xh,
                      __half* __restrict__ xl, float* __restrict__ row_scale, int k) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float red[16];
  __shared__ int bad_row;
  const int64_t t = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + t * k);
  const int k4 = k >> 2;
  float4 v[NV];
  float mx = 0.0f;
  int bad = 0;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = static_cast<int>(threadIdx.x) + 512 * j;
    v[j] = i < k4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    bad |= !(fabsf(v[j].x) <= 3.402823466e38f) | !(fabsf(v[j].y) <= 3.402823466e38f) |
           !(fabsf(v[j].z) <= 3.402823466e38f) | !(fabsf(v[j].w) <= 3.402823466e38f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  bad = __any_sync(0xffffffffu, bad);
  if (threadIdx.x == 0) bad_row = 0;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = mx;
    if (bad) bad_row = 1;
  }
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < 16; ++i) mx = fmaxf(mx, red[i]);
  // as SplitF16Kernel: s = 2^(e - 15) with mx < 2^e, e kept >= -111
  int e = 0;
  frexpf(mx, &e);
  e = e < -111 ? -111 : e;
  const bool plain = bad_row || mx == 0.0f;
  const float inv = plain ? 1.0f : ldexpf(1.0f, 15 - e);
  if (threadIdx.x == 0) row_scale[t] = plain ? 1.0f : ldexpf(1.0f, e - 15);
  __half2* h2 = reinterpret_cast<__half2*>(xh + t * k);
  __half2* l2 = reinterpret_cast<__half2*>(xl + t * k);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = static_cast<int>(threadIdx.x) + 512 * j;
    if (i < k4) {
      const float a[4] = {v[j].x * inv, v[j].y * inv, v[j].z * inv, v[j].w * inv};  // exact
      __half hi[4], lo[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        hi[q] = __float2half_rn(a[q]);
        lo[q] = __float2half_rn(a[q] - __half2float(hi[q]));  // exact remainder
      }
      h2[2 * i] = __halves2half2(hi[0], hi[1]);
      h2[2 * i + 1] = __halves2half2(hi[2], hi[3]);
      l2[2 * i] = __halves2half2(lo[0], lo[1]);
      l2[2 * i + 1] = __halves2half2(lo[2], lo[3]);
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 HfEncodeFn() {
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

// 2-D map with a 128-byte swizzle (128-byte box rows).
bool HfMap2D(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner,
             uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = HfEncodeFn();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Whether LinearF16 takes the matrices: Q8_0 / Q4_0, whole stages of two
// blocks, 16-byte aligned rows (the TMA map's stride).
bool LinearF16Eligible(int qtype, int64_t k, int64_t row_bytes) {
  return (qtype == MLB_Q8_0 || qtype == MLB_Q4_0) && k % kHfStageK == 0 && row_bytes % 16 == 0;
}

// y[m] [t_rows, n[m]] = x . W[m]^T for m < count; scratch (16-byte aligned)
// holds k t_rows + t_rows floats: x's two fp16 pieces and the row scales.
// The caller checked LinearF16Eligible, the pointers and the alignment.
int LinearF16(int count, const void* const* w, int qtype, const int64_t* n, int64_t k,
              int64_t row_bytes, const float* x, int64_t t_rows, float* const* y,
              float* scratch, cudaStream_t s) {
  HfGroup grp{};
  grp.count = count;
  grp.t_tiles = static_cast<int>((t_rows + kHfTokens - 1) / kHfTokens);
  grp.t_rows = static_cast<int>(t_rows);
  grp.k = static_cast<int>(k);
  int64_t tiles = 0;
  for (int m = 0; m < count; ++m) {
    if (!HfMap2D(&grp.w[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, w[m], static_cast<uint64_t>(row_bytes),
                 static_cast<uint64_t>(n[m]), static_cast<uint64_t>(row_bytes), 128, kHfRows))
      return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: tensor map encoding failed");
    grp.wp[m] = static_cast<const uint8_t*>(w[m]);
    grp.y[m] = y[m];
    grp.n[m] = static_cast<int>(n[m]);
    grp.tile_begin[m] = static_cast<int>(tiles);
    tiles += (n[m] + kHfRows - 1) / kHfRows * grp.t_tiles;
  }
  grp.tile_begin[count] = static_cast<int>(tiles);
  if (tiles > INT_MAX) return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: too many tiles");
  // x's pieces: two [t_rows, k] fp16 arrays, then the row scales
  __half* xh = reinterpret_cast<__half*>(scratch);
  __half* xl = xh + k * t_rows;  // k % 64 == 0: still 16-byte aligned
  float* row_scale = reinterpret_cast<float*>(xl + k * t_rows);
  switch ((k / 4 + 511) / 512) {  // float4 per thread of 512
    case 1: Launch(SplitF16RegKernel<1>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 2: Launch(SplitF16RegKernel<2>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 3: Launch(SplitF16RegKernel<3>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 4: Launch(SplitF16RegKernel<4>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 5: Launch(SplitF16RegKernel<5>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 6: Launch(SplitF16RegKernel<6>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 7: Launch(SplitF16RegKernel<7>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    case 8: Launch(SplitF16RegKernel<8>, static_cast<unsigned>(t_rows), 512, 0, s, x, xh, xl, row_scale, static_cast<int>(k)); break;
    default:  // longer rows: two passes over x
      Launch(SplitF16Kernel, static_cast<unsigned>(t_rows), 256, 0, s, x, xh, xl, row_scale,
             static_cast<int>(k));
  }
  int rc = CheckLaunch("mlb_linear_rows_f32");
  if (rc != MLB_OK) return rc;
  if (!HfMap2D(&grp.x[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, static_cast<uint64_t>(k),
               static_cast<uint64_t>(t_rows), static_cast<uint64_t>(k) * 2, kHfStageK,
               kHfTokens) ||
      !HfMap2D(&grp.x[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xl, static_cast<uint64_t>(k),
               static_cast<uint64_t>(t_rows), static_cast<uint64_t>(k) * 2, kHfStageK,
               kHfTokens))
    return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: tensor map encoding failed");
  grp.row_scale = row_scale;
  grp.x32 = x;
  grp.row_bytes = row_bytes;
  auto kernel = qtype == MLB_Q8_0 ? LinearF16Kernel<MLB_Q8_0> : LinearF16Kernel<MLB_Q4_0>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHfSmemBytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: shared memory opt-in");
  }
  Launch(kernel, static_cast<unsigned>(tiles), kHfThreads, kHfSmemBytes, s, grp);
  return CheckLaunch("mlb_linear_rows_f32");
}

unsigned int LinearF16WaitTimeouts() {
  unsigned int count = 0;
  if (cudaMemcpyFromSymbol(&count, g_hf_wait_timeouts, sizeof(count)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count;
}

}  // namespace mlb
