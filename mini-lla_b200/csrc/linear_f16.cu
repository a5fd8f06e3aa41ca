// Prompt-sized Q8_0 / Q4_0 linear layers on the fp16 tensor cores with the
// weight codes as exact operands: y[t] = W . x[t], W [n, k] in ggml blocks,
// x [T, k] fp32 — the form mlb_linear_rows_f32 takes for these two formats.
//
// Reference arithmetic (src/quant.cc:171-226 LinearWithBlocks): per output a
// sequential fp32 sum of (d * q_i) * x_i, with q_i the int8 code (Q8_0) or
// n_i - 8 (Q4_0) and d the block's fp16 scale.
//
// Method: every code q (|q| <= 128) is exact in fp16.  Each token row of x is
// scaled by a power of two s_t (its largest magnitude lands in [2^14, 2^15))
// and split into two fp16 pieces, x / s_t = xh + xl + r, each piece the fp16
// rounding of the exact fp32 remainder, |r| <= 2^-22 |x / s_t| (plus 2^-25
// below fp16's normal range, i.e. 2^-39 of the row's largest value).  Per
// (128-row, 128-token) tile and ggml block the tensor core sums
// q_i * (xh_i + xl_i) into an fp32 accumulator — every product is exact
// (8 x 11 significant bits) — with 4 MMAs (tcgen05.mma kind::f16, fp16 A
// and B, K = 16: two pieces x two halves of the block).  The epilogue adds
// d * block sum to each output in fp32 registers and finally multiplies by
// s_t: the block scale never enters the tensor core, so no weight is
// dequantised or split.  Against the TF32 form (w and x split into head +
// tail, 3 products of K = 8 per 8 values) this is a third of the tensor-core
// work per block.  Results stay within the tests' 1e-5 * sum |w_i x_i| of the
// reference.  A row of x holding Inf or NaN keeps s_t = 1, so the
// non-finite values reach its outputs.
//
// Design (one CTA = 128 weight rows x 128 tokens, k in stages of two blocks;
// 448 threads in warp roles):
//   - warp 4, one lane: TMA producer.  Per stage: the raw bytes of the 128
//     rows' two blocks (a 2-D uint8 map over [n, row_bytes], box 128 bytes
//     from the stage's byte offset rounded down to 16, which covers two 34-
//     or 18-byte blocks) and the two 128-token x 64-value fp16 tiles of x's
//     pieces, all with a 128-byte swizzle (bank-conflict-free row reads; the
//     MMA descriptors use the same layout); 4 stages of 48 KB in flight;
//   - warps 0-3 (thread = weight row = tensor-memory lane): turn the two
//     blocks' codes into fp16 pairs (one byte permute builds 1024 + byte in
//     both halves, one packed subtract — exact) and store them into tensor
//     memory (tcgen05.st, the A operand; 16 columns per block); the block
//     scales go to a shared ring;
//   - warp 5: allocates tensor memory; one lane issues the 4 MMAs of each
//     block into one of two 128-column fp32 accumulators and commits;
//   - warps 6-13 (two per tensor-memory lane quarter, 64 tokens each): read
//     a block's accumulator (tcgen05.ld), add d * sum to 64 fp32 sums per
//     thread, and at the end store s_t * sum.
// Every wait is bounded: a wait that gives up is counted (mlb_wait_timeouts)
// and the CTA writes NaN instead of its tile.
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
constexpr int kHfThreads = 448;     // movers 0-3, producer 4, MMA 5, epilogue 6-13
constexpr int kHfRawBytes = kHfRows * 128;               // raw weight box per stage
constexpr int kHfPieceBytes = kHfTokens * kHfStageK * 2; // one fp16 x piece per stage
constexpr int kHfStageBytes = kHfRawBytes + kHfPieces * kHfPieceBytes;
constexpr int kHfScaleSlots = 8;    // stages of block scales kept for the epilogue
constexpr int kHfTmemColumns = 512;
constexpr int kHfAccColumns = kHfTokens;  // one fp32 accumulator
constexpr int kHfAColumns = 32;           // two blocks x 16 columns (2 fp16 each)
constexpr int kHfMaxGroup = 3;

__host__ __device__ constexpr int HfBlockBytes(int qt) { return qt == MLB_Q8_0 ? 34 : 18; }

// Shared memory from a 1024-byte aligned base: kHfStages stages (raw box,
// then x's pieces), the scale ring, the barriers, the TMEM address.
constexpr int kHfScaleOffset = kHfStages * kHfStageBytes;
constexpr int kHfBarOffset = kHfScaleOffset + kHfScaleSlots * 2 * kHfRows * 4;
// raw_full / raw_empty / a_full / a_empty per stage, d_full / d_empty x 2,
// sc_full / sc_empty per scale slot, mma_done
constexpr int kHfBarriers = 4 * kHfStages + 4 + 2 * kHfScaleSlots + 1;
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
__device__ __forceinline__ void HfStore32(uint32_t taddr, const uint32_t (&v)[32]) {
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

// Row m's two blocks of a raw stage (byte `rel` = 4 R of its 128-byte
// swizzled box row): 32 A columns (fp16 pairs, K order) and the two fp16
// scales.
template <int QT, int R>
__device__ __forceinline__ void HfTakeStage(const uint8_t* raw_row, int m, uint32_t (&cols)[32],
                                            uint32_t (&scale)[2]) {
  constexpr int kChunks = QT == MLB_Q8_0 ? 5 : 3;  // 16-byte pieces covering rel + 2 blocks
  uint32_t w[4 * kChunks + 1];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(raw_row + 16 * (c ^ (m & 7)));
    w[4 * c] = v.x;
    w[4 * c + 1] = v.y;
    w[4 * c + 2] = v.z;
    w[4 * c + 3] = v.w;
  }
  w[4 * kChunks] = 0;
  if constexpr (QT == MLB_Q8_0) {
    // block 0 at byte 4R: scale in the low half of word R, codes from byte
    // 4R + 2 (a half-word shift); block 1 at 4R + 34: scale in the high half
    // of word R + 8, codes word-aligned from word R + 9
    scale[0] = w[R] & 0xFFFFu;
    scale[1] = w[R + 8] >> 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t c0 = __funnelshift_r(w[R + i], w[R + i + 1], 16) ^ 0x80808080u;
      const uint32_t c1 = w[R + 9 + i] ^ 0x80808080u;
      HfWordPairs(c0, kHfBiasQ8, cols[2 * i], cols[2 * i + 1]);
      HfWordPairs(c1, kHfBiasQ8, cols[16 + 2 * i], cols[16 + 2 * i + 1]);
    }
  } else {
    // Q4_0 18-byte blocks: block 0 at 4R (nibbles from 4R + 2), block 1 at
    // 4R + 18 (scale in the high half of word R + 4, nibbles word-aligned
    // from word R + 5); values 0-15 are the low nibbles, 16-31 the high ones
    scale[0] = w[R] & 0xFFFFu;
    scale[1] = w[R + 4] >> 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u0 = __funnelshift_r(w[R + i], w[R + i + 1], 16);
      const uint32_t u1 = w[R + 5 + i];
      HfWordPairs(u0 & 0x0F0F0F0Fu, kHfBiasQ4, cols[2 * i], cols[2 * i + 1]);
      HfWordPairs((u0 >> 4) & 0x0F0F0F0Fu, kHfBiasQ4, cols[8 + 2 * i], cols[8 + 2 * i + 1]);
      HfWordPairs(u1 & 0x0F0F0F0Fu, kHfBiasQ4, cols[16 + 2 * i], cols[16 + 2 * i + 1]);
      HfWordPairs((u1 >> 4) & 0x0F0F0F0Fu, kHfBiasQ4, cols[24 + 2 * i], cols[24 + 2 * i + 1]);
    }
  }
}

template <int QT>
__device__ __forceinline__ void HfTakeStageAt(int r, const uint8_t* raw_row, int m,
                                              uint32_t (&cols)[32], uint32_t (&scale)[2]) {
  switch (r) {
    case 0: HfTakeStage<QT, 0>(raw_row, m, cols, scale); break;
    case 1: HfTakeStage<QT, 1>(raw_row, m, cols, scale); break;
    case 2: HfTakeStage<QT, 2>(raw_row, m, cols, scale); break;
    default: HfTakeStage<QT, 3>(raw_row, m, cols, scale); break;
  }
}

struct HfGroup {
  CUtensorMap w[kHfMaxGroup];  // raw weight bytes of each matrix
  CUtensorMap x[kHfPieces];    // x's fp16 pieces [T, k]
  float* y[kHfMaxGroup];
  const float* row_scale;      // s_t per token
  int n[kHfMaxGroup];
  int tile_begin[kHfMaxGroup + 1];  // first tile of each matrix; [count] = total
  int count;
  int t_tiles;
  int t_rows;
  int k;
};

}  // namespace

// Bounded waits of this file's kernel that gave up.
__device__ unsigned int g_hf_wait_timeouts;

namespace {

template <int QT>
__global__ void __launch_bounds__(kHfThreads, 1)
    LinearF16Kernel(const __grid_constant__ HfGroup grp) {
  constexpr int kBB = HfBlockBytes(QT);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw_addr = HfSmem(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = HfSmem(base);
  auto stage_base = [&](int s) { return base + s * kHfStageBytes; };
  float* scales = reinterpret_cast<float*>(base + kHfScaleOffset);
  const uint32_t bars = sbase + kHfBarOffset;
  auto raw_full = [&](int s) { return bars + 8 * s; };
  auto raw_empty = [&](int s) { return bars + 8 * (kHfStages + s); };
  auto a_full = [&](int s) { return bars + 8 * (2 * kHfStages + s); };
  auto a_empty = [&](int s) { return bars + 8 * (3 * kHfStages + s); };
  auto d_full = [&](int s) { return bars + 8 * (4 * kHfStages + s); };
  auto d_empty = [&](int s) { return bars + 8 * (4 * kHfStages + 2 + s); };
  auto sc_full = [&](int s) { return bars + 8 * (4 * kHfStages + 4 + s); };
  auto sc_empty = [&](int s) { return bars + 8 * (4 * kHfStages + 4 + kHfScaleSlots + s); };
  const uint32_t mma_done = bars + 8 * (4 * kHfStages + 4 + 2 * kHfScaleSlots);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kHfBarOffset + 8 * kHfBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
      HfBarInit(raw_empty(s), 5);  // the 4 mover warps + the MMA commit
      HfBarInit(a_full(s), 4);
      HfBarInit(a_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      HfBarInit(d_full(s), 1);
      HfBarInit(d_empty(s), 8);
    }
    for (int s = 0; s < kHfScaleSlots; ++s) {
      HfBarInit(sc_full(s), 4);
      HfBarInit(sc_empty(s), 8);
    }
    HfBarInit(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 5) {
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
  // tensor-memory columns: two accumulators, then the A ring
  auto acc_col = [&](int b) { return static_cast<uint32_t>(b * kHfAccColumns); };
  auto a_col = [&](int s) { return static_cast<uint32_t>(2 * kHfAccColumns + s * kHfAColumns); };

  int issued = 0;  // producer: stages whose loads were issued
  if (warp == 4) {
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
  } else if (warp == 5) {
    if (lane == 0) {
      bool ok = true;
      for (int s = 0; ok && s < stages; ++s) {
        const int st = s % kHfStages;
        if (!HfWait(raw_full(st), (s / kHfStages) & 1) ||
            !HfWait(a_full(st), (s / kHfStages) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        const uint32_t pieces = HfSmem(stage_base(st) + kHfRawBytes);
#pragma unroll
        for (int j = 0; j < 2; ++j) {  // the stage's two blocks
          const int b = 2 * s + j;
          if (!HfWait(d_empty(b & 1), ((b >> 1) & 1) ^ 1) || *abort_flag) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll
          for (int p = 0; p < kHfPieces; ++p)
#pragma unroll
            for (int h = 0; h < 2; ++h)  // K = 16 per MMA: 32 bytes of the 128-byte rows
              HfMma(tmem + acc_col(b & 1), tmem + a_col(st) + 16 * j + 8 * h,
                    HfDesc(pieces + p * kHfPieceBytes + 64 * j + 32 * h), (p | h) != 0);
          HfCommit(d_full(b & 1));
        }
        if (!ok) break;
        HfCommit(a_empty(st));
        HfCommit(raw_empty(st));
      }
      if (!ok) {
        atomicAdd(&g_hf_wait_timeouts, 1u);
        *abort_flag = 1;
      }
    }
  } else if (warp < 4) {
    // ---- movers: codes -> fp16 pairs in tensor memory, scales -> shared ----
    const int m = threadIdx.x;  // weight row within the tile (TMEM lane)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    for (int s = 0; s < stages; ++s) {
      const int st = s % kHfStages;
      const int ss = s % kHfScaleSlots;
      if (!HfWait(raw_full(st), (s / kHfStages) & 1) ||
          !HfWait(a_empty(st), ((s / kHfStages) & 1) ^ 1) ||
          !HfWait(sc_empty(ss), ((s / kHfScaleSlots) & 1) ^ 1) || *abort_flag) {
        atomicAdd(&g_hf_wait_timeouts, 1u);
        *abort_flag = 1;
        break;
      }
      uint32_t cols[32], sc[2];
      HfTakeStageAt<QT>(((s * 2 * kBB) & 15) >> 2, stage_base(st) + m * 128, m, cols, sc);
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      HfStore32(lane_base + a_col(st), cols);
      float* sl = scales + ss * 2 * kHfRows;
      sl[m] = __half2float(__ushort_as_half(static_cast<unsigned short>(sc[0])));
      sl[kHfRows + m] = __half2float(__ushort_as_half(static_cast<unsigned short>(sc[1])));
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        HfArrive(a_full(st));
        HfArrive(sc_full(ss));
        HfArrive(raw_empty(st));  // this warp is done with the raw box
      }
    }
  } else {
    // ---- epilogue: block sums * d -> 64 fp32 sums per thread ----
    const int q = warp & 3;            // tensor-memory lane quarter
    const int half = (warp - 6) >> 2;  // tokens [64 half, 64 half + 64)
    const int m = q * 32 + lane;       // weight row
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
    bool ok = true;
    for (int b = 0; b < 2 * stages; ++b) {
      const int ss = (b >> 1) % kHfScaleSlots;
      if (((b & 1) == 0 && !HfWait(sc_full(ss), ((b >> 1) / kHfScaleSlots) & 1)) ||
          !HfWait(d_full(b & 1), (b >> 1) & 1) || *abort_flag) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const float d = scales[ss * 2 * kHfRows + (b & 1) * kHfRows + m];
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 32 tokens at a time
        float v[32];
        HfLoad32(lane_base + acc_col(b & 1) + 64 * half + 32 * c, v);
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[32 * c + i] = fmaf(d, v[i], acc[32 * c + i]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        HfArrive(d_empty(b & 1));
        if (b & 1) HfArrive(sc_empty(ss));  // both blocks of the stage read
      }
    }
    if (!ok) {
      if (lane == 0) atomicAdd(&g_hf_wait_timeouts, 1u);
      *abort_flag = 1;
    }
    const int row = n0 + m;
    if (row < n) {
      float* y = grp.y[mat];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int t = t0 + 64 * half + i;
        if (t < grp.t_rows)
          y[static_cast<int64_t>(t) * n + row] =
              ok ? acc[i] * __ldg(grp.row_scale + t) : __int_as_float(0x7fc00000);
      }
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // let the loads in flight land and mark the whole tile as failed
    if (warp == 4 && lane == 0) {
      for (int s = issued - kHfStages > 0 ? issued - kHfStages : 0; s < issued; ++s)
        HfWait(raw_full(s % kHfStages), (s / kHfStages) & 1);
    }
    if (warp < 4) {
      const int row = n0 + static_cast<int>(threadIdx.x);
      if (row < n)
        for (int t = t0; t < t0 + kHfTokens && t < grp.t_rows; ++t)
          grp.y[mat][static_cast<int64_t>(t) * n + row] = __int_as_float(0x7fc00000);
    }
  }
  if (warp == 5 && lane == 0) {
    // every MMA issued has finished before the tensor memory is released
    HfCommit(mma_done);
    HfWait(mma_done, 0);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 5) {
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
  SplitF16Kernel<<<static_cast<unsigned>(t_rows), 256, 0, s>>>(x, xh, xl, row_scale,
                                                              static_cast<int>(k));
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
  auto kernel = qtype == MLB_Q8_0 ? LinearF16Kernel<MLB_Q8_0> : LinearF16Kernel<MLB_Q4_0>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHfSmemBytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: shared memory opt-in");
  }
  kernel<<<static_cast<unsigned>(tiles), kHfThreads, kHfSmemBytes, s>>>(grp);
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
