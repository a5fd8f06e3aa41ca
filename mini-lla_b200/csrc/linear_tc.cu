// Prompt-sized linear layers on the 5th-generation tensor cores:
// y[t] = W . x[t] for t < T with W [n, k] in the reference's ggml blocks
// (Q8_0 / Q4_0 / Q4_1) or F32 and x [T, k] fp32.
//
// Reference arithmetic: src/quant.cc:171-226 (LinearWithBlocks) and
// src/matmul_optimized.cc:95-117 (F32), a sequential fp32 sum of
// dequant(w_i) * x_i per output; the reference runs it once per token.
//
// Accuracy on TF32 tensor cores: every operand is split into a TF32 head
// (its top 19 bits) and the exact remainder, w = wh + wl and x = xh + xl,
// and each tile accumulates wh.xh + wh.xl + wl.xh in fp32 (the dropped
// wl.xl term and the TF32 reading of the tails are ~2^-21 of each product).
// A dequantised ggml weight d * q has at most 19 significant bits, so its
// tail is exact in TF32 too.  Results
// match the reference within 1e-5 * sum_i |w_i x_i| (tests).
//
// Design (one CTA = 128 weight rows x 128 tokens, k in steps of 32 = one
// ggml block; 352 threads in warp roles):
//   - warp 8, one lane: TMA producer.  Per step it loads the raw weight
//     bytes of the 128 rows (a 2-D uint8 tensor map over [n, row_bytes];
//     the box starts at the block's byte offset rounded down to 16 and is
//     64 bytes wide, which covers any 34 / 18 / 20-byte block; 64-byte
//     swizzle so the per-row reads are bank-conflict free) and the
//     128 x 32 tiles of xh and xl (fp32 tensor maps, 128-byte swizzle);
//   - warps 0-7: dequantisers, two threads per weight row (16 values each).
//     A thread decodes its half of row m's block (byte permutes into the
//     mantissa of 2^23 instead of int->float conversions, packed f32x2
//     arithmetic), splits each value into its TF32 head (the top 19 bits,
//     a mask) and the exact remainder, and stores both straight into tensor
//     memory (tcgen05.st; row m is lane m, one value per column) — the MMA
//     reads its A operand from there, so shared memory only carries the
//     raw weights and the x tiles;
//   - warp 9, one lane: MMA issuer.  Per step 4 k-slices x 3 products of
//     tcgen05.mma.cta_group::1.kind::tf32 (M = 128, N = 128, K = 8; A from
//     tensor memory, B from shared memory) into a 128-column fp32
//     accumulator in tensor memory; tcgen05.commit frees the stage's
//     buffers;
//   - warp 10 allocates / frees the tensor memory; warps 0-7 finally read
//     the accumulator (tcgen05.ld, lane = weight row; warps w and w + 4
//     share TMEM lanes 32w.. and take one half of the tokens each) and store
//     y[t, row], 32 consecutive rows per warp store.
// Stages form a ring (5 for the quantised formats, 4 for F32) tracked by
// mbarriers; every wait is bounded (a wait that gives up is counted in
// g_tc_wait_timeouts and the CTA writes NaN instead of its tile).
// x is split into xh / xl by a small kernel first (caller scratch).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>
#include <mutex>
#include <string>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kTileRows = 128;    // weight rows (MMA M)
constexpr int kTileTokens = 128;  // tokens (MMA N)
constexpr int kStepK = 32;        // k per stage: one ggml block
constexpr int kTcThreads = 352;       // 8 dequant/epilogue warps + producer, MMA, TMEM
constexpr int kDequantThreads = 256;  // two per weight row
constexpr int kTileBytes = kTileRows * kStepK * 4;  // one 128 x 32 fp32 tile
constexpr int kTmemColumns = 512;  // accumulator (128) + the A ring (64 per stage)
constexpr int kAccColumns = kTileTokens;
constexpr int kATileColumns = kStepK;  // one TF32 per column, row m in lane m

__host__ __device__ constexpr int TcBlockBytes(int qt) {
  return qt == MLB_F32 ? 128 : (qt == MLB_Q8_0 ? 34 : (qt == MLB_Q4_0 ? 18 : 20));
}
__host__ __device__ constexpr int TcRawBytes(int qt) { return qt == MLB_F32 ? 128 : 64; }
__host__ __device__ constexpr int TcStages(int qt) { return qt == MLB_F32 ? 4 : 5; }

// Shared-memory layout from a 1024-byte aligned base: per stage two tiles
// (B head, B tail), then the raw weight tiles, then the mbarriers (full,
// dequantised, empty per stage; accumulator ready) and the tensor-memory
// address.  The A tiles live in tensor memory.
__host__ __device__ constexpr int TcRawOffset(int qt) { return TcStages(qt) * 2 * kTileBytes; }
__host__ __device__ constexpr int TcBarOffset(int qt) {
  return TcRawOffset(qt) + TcStages(qt) * kTileRows * TcRawBytes(qt);
}
__host__ __device__ constexpr int TcSmemBytes(int qt) {
  return TcBarOffset(qt) + 8 * (3 * TcStages(qt) + 1) + 16 + 1024;  // + alignment slack
}

__device__ __forceinline__ uint32_t SmemU32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void MbarInit(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void MbarExpectTx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void MbarArrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool MbarTryWait(uint32_t bar, uint32_t parity) {
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
__device__ __forceinline__ bool MbarWait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 21); ++i)
    if (MbarTryWait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void TmaLoad2D(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle,
// 8-row atoms of 128-byte rows 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t SmemDesc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;            // LBO (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // SBO
  d |= static_cast<uint64_t>(1) << 46;            // descriptor version
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D fp32, A and B TF32, both K-major, N = 128, M = 128.
constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) |
                                (static_cast<uint32_t>(kTileTokens >> 3) << 17) |
                                (static_cast<uint32_t>(kTileRows >> 4) << 24);

// D[tmem] (+)= A[a_tmem] . B[b_desc]^T, A read from tensor memory (row m in
// lane m, one TF32 per column), B from shared memory.
__device__ __forceinline__ void MmaTf32(uint32_t tmem, uint32_t a_tmem, uint64_t b,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem),
      "r"(a_tmem), "l"(b), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void TmemStore16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void MmaCommit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
      : "memory");
}

// TF32 head of an fp32 value: sign, exponent and the top 10 mantissa bits
// (truncation).  The tail v - head is exact and has at most 13 significant
// bits; the tensor core reads it as TF32 (dropping at most 2^-11 of it).
__device__ __forceinline__ uint32_t Tf32Head(uint32_t bits) { return bits & 0xFFFFE000u; }

__device__ __forceinline__ uint64_t Pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 Unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
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

// Four bytes -> four exact floats (byte permuted into the low mantissa of
// 2^23, then `bias` = 2^23 + offset subtracted, two lanes at a time).
__device__ __forceinline__ void BytesToFloats(uint32_t u, float bias, uint64_t& p01,
                                              uint64_t& p23) {
  const uint64_t nb = Pack2(-bias, -bias);
  p01 = Add2(Pack2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                   __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), nb);
  p23 = Add2(Pack2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                   __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), nb);
}

// The raw weight tile holds one 64-byte row per weight row (128 bytes for
// F32), written by TMA with a 64-byte (128-byte) swizzle: logical 16-byte
// chunk c of row m sits at chunk c ^ ((m >> 1) & 3) (c ^ (m & 7)).  A
// thread reads its row with 16-byte loads, which the swizzle spreads over
// all banks for the 8 rows of a quarter-warp.
template <int QT>
__device__ __forceinline__ uint4 RawChunk(const uint8_t* row, int m, int c) {
  const int phys = QT == MLB_F32 ? (c ^ (m & 7)) : (c ^ ((m >> 1) & 3));
  return *reinterpret_cast<const uint4*>(row + 16 * phys);
}

// Words 0..8 of a block starting at byte `off` of the 16 raw words:
// out[k] = bytes off + 4k .. off + 4k + 3.
template <int Q>
__device__ __forceinline__ void TakeWords(const uint32_t (&w)[16], uint32_t sh,
                                          uint32_t (&out)[9]) {
#pragma unroll
  for (int k = 0; k < 9; ++k) out[k] = __funnelshift_r(w[Q + k], w[Q + k + 1], sh);
}

template <int QT>
__device__ __forceinline__ void DequantBlockHalf(const uint8_t* row, int m, int off, int half,
                                                 float (&w)[16]);

// Half `half` (values 16 * half .. 16 * half + 15) of row m's block at
// byte `off` of its raw row, as the reference dequantises them (d * q,
// d * (n - 8), d * n + m, or the F32 value).
template <int QT>
__device__ __forceinline__ void DequantHalf(const uint8_t* row, int m, int off, int half,
                                            float (&w)[16]) {
  if constexpr (QT == MLB_F32) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = RawChunk<QT>(row, m, 4 * half + c);
      w[4 * c] = __uint_as_float(v.x);
      w[4 * c + 1] = __uint_as_float(v.y);
      w[4 * c + 2] = __uint_as_float(v.z);
      w[4 * c + 3] = __uint_as_float(v.w);
    }
  } else {
    DequantBlockHalf<QT>(row, m, off, half, w);
  }
}

template <int QT>
__device__ __forceinline__ void DequantBlockHalf(const uint8_t* row, int m, int off, int half,
                                                 float (&w)[16]) {
  uint32_t raw[16];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = RawChunk<QT>(row, m, c);
    raw[4 * c] = v.x;
    raw[4 * c + 1] = v.y;
    raw[4 * c + 2] = v.z;
    raw[4 * c + 3] = v.w;
  }
  // the block's first 36 bytes as aligned words (off is the same for the
  // whole CTA at a given step, so the switch does not diverge)
  uint32_t blk[9];
  const uint32_t sh = 8u * (off & 3);
  switch (off >> 2) {
    case 0: TakeWords<0>(raw, sh, blk); break;
    case 1: TakeWords<1>(raw, sh, blk); break;
    case 2: TakeWords<2>(raw, sh, blk); break;
    default: TakeWords<3>(raw, sh, blk); break;
  }
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] & 0xFFFFu)));
  const uint64_t d2 = Pack2(d, d);
  uint32_t words[4];
  if (QT == MLB_Q8_0) {  // codes at bytes 2 + 16 * half ..
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // (selects, not an indexed load: blk stays in registers)
      const uint32_t lo = half ? blk[4 + i] : blk[i];
      const uint32_t hi = half ? blk[5 + i] : blk[1 + i];
      words[i] = __funnelshift_r(lo, hi, 16) ^ 0x80808080u;
    }
  } else if (QT == MLB_Q4_0) {  // nibbles at bytes 2 .. 17
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = __funnelshift_r(blk[i], blk[i + 1], 16);
      words[i] = (half ? u >> 4 : u) & 0x0F0F0F0Fu;
    }
  } else {  // Q4_1: nibbles at bytes 4 .. 19
#pragma unroll
    for (int i = 0; i < 4; ++i) words[i] = (half ? blk[1 + i] >> 4 : blk[1 + i]) & 0x0F0F0F0Fu;
  }
  const float bias = QT == MLB_Q8_0 ? 8388736.0f : (QT == MLB_Q4_0 ? 8388616.0f : 8388608.0f);
  const float mn =
      QT == MLB_Q4_1 ? __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] >> 16)))
                     : 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t a, b;
    BytesToFloats(words[i], bias, a, b);
    a = Mul2(a, d2);  // exact: 11-bit scale times a code of at most 8 bits
    b = Mul2(b, d2);
    if (QT == MLB_Q4_1) {  // d * n + m, rounded like the reference's sum
      const uint64_t m2 = Pack2(mn, mn);
      a = Add2(a, m2);
      b = Add2(b, m2);
    }
    const float2 fa = Unpack2(a), fb = Unpack2(b);
    w[4 * i] = fa.x;
    w[4 * i + 1] = fa.y;
    w[4 * i + 2] = fb.x;
    w[4 * i + 3] = fb.y;
  }
}

}  // namespace

// Bounded waits of the tensor-core linear kernel that gave up.
__device__ unsigned int g_tc_wait_timeouts;

namespace {

// Up to kMaxGroup weight matrices applied to the same x in one launch (the
// q / k / v projections, the FFN gate / up): CTA i takes tile i of the
// concatenated tile list, matrix by matrix, the token tile fastest so that
// consecutive CTAs share a weight tile in L2.
constexpr int kMaxGroup = 3;

struct TcGroup {
  CUtensorMap w[kMaxGroup];     // raw weight bytes of each matrix
  CUtensorMap xh, xl;           // x's TF32 head and tail
  float* y[kMaxGroup];
  int n[kMaxGroup];
  int tile_begin[kMaxGroup + 1];  // first tile of each matrix; [count] = total
  int count;
  int t_tiles;
  int t_rows;
  int k;
};

template <int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
    LinearTcKernel(const __grid_constant__ TcGroup grp) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  constexpr int S = TcStages(QT);
  constexpr int kRaw = TcRawBytes(QT);
  constexpr int kBB = TcBlockBytes(QT);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // 1024-byte aligned base (the swizzled tiles need it)
  const uint32_t raw_addr = SmemU32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = SmemU32(base);
  auto b_hi = [&](int s) { return sbase + s * 2 * kTileBytes; };
  auto b_lo = [&](int s) { return sbase + s * 2 * kTileBytes + kTileBytes; };
  // tensor-memory columns of stage s's A head and tail tiles
  auto a_hi_col = [&](int s) { return kAccColumns + s * 2 * kATileColumns; };
  auto a_lo_col = [&](int s) { return kAccColumns + s * 2 * kATileColumns + kATileColumns; };
  uint8_t* raw = base + TcRawOffset(QT);
  const uint32_t bars = sbase + TcBarOffset(QT);
  auto full = [&](int s) { return bars + 8 * s; };
  auto dequantised = [&](int s) { return bars + 8 * (S + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * S + s); };
  const uint32_t acc_ready = bars + 8 * (3 * S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + TcBarOffset(QT) + 8 * (3 * S + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int mat = 0;
  while (mat + 1 < grp.count && static_cast<int>(blockIdx.x) >= grp.tile_begin[mat + 1]) ++mat;
  const int local = static_cast<int>(blockIdx.x) - grp.tile_begin[mat];
  const int n0 = (local / grp.t_tiles) * kTileRows;
  const int t0 = (local % grp.t_tiles) * kTileTokens;
  const int n = grp.n[mat];
  const int t_rows = grp.t_rows;
  float* __restrict__ y = grp.y[mat];
  const CUtensorMap* wmap = &grp.w[mat];
  const int steps = grp.k / kStepK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      MbarInit(full(s), 1);
      MbarInit(dequantised(s), kDequantThreads);
      MbarInit(empty(s), 1);
    }
    MbarInit(acc_ready, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 10) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     SmemU32(tmem_slot)),
                 "r"(kTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  int issued = 0;  // producer: stages whose loads were issued
  if (warp == 8) {
    if (lane == 0) {
      for (int s = 0; s < steps; ++s) {
        const int slot = s % S;
        if (!MbarWait(empty(slot), ((s / S) & 1) ^ 1) || *abort_flag) {
          atomicAdd(&g_tc_wait_timeouts, 1u);
          *abort_flag = 1;
          break;
        }
        MbarExpectTx(full(slot), kTileRows * kRaw + 2 * kTileBytes);
        const int xw = (s * kBB) & ~15;  // byte column of the block, rounded down
        TmaLoad2D(SmemU32(raw + slot * kTileRows * kRaw), wmap, xw, n0, full(slot));
        TmaLoad2D(b_hi(slot), &grp.xh, s * kStepK, t0, full(slot));
        TmaLoad2D(b_lo(slot), &grp.xl, s * kStepK, t0, full(slot));
        issued = s + 1;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      for (int s = 0; s < steps; ++s) {
        const int slot = s % S;
        if (!MbarWait(dequantised(slot), (s / S) & 1) || *abort_flag) {
          atomicAdd(&g_tc_wait_timeouts, 1u);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll
        for (int j = 0; j < kStepK / 8; ++j) {  // K = 8 TF32 = 32 bytes per MMA
          const uint32_t ah = tmem + a_hi_col(slot) + 8 * j;
          const uint32_t al = tmem + a_lo_col(slot) + 8 * j;
          const uint64_t bh = SmemDesc(b_hi(slot) + 32 * j);
          const uint64_t bl = SmemDesc(b_lo(slot) + 32 * j);
          MmaTf32(tmem, ah, bh, (s | j) != 0 ? 1u : 0u);
          MmaTf32(tmem, ah, bl, 1u);
          MmaTf32(tmem, al, bh, 1u);
        }
        MmaCommit(empty(slot));  // the stage's buffers are free once these finish
      }
      MmaCommit(acc_ready);  // every MMA issued so far has finished
    }
  } else if (warp < 8) {
    const int m = threadIdx.x & (kTileRows - 1);  // weight row within the tile
    const int half = threadIdx.x >> 7;             // which 16 values of the block
    for (int s = 0; s < steps; ++s) {
      const int slot = s % S;
      if (!MbarWait(full(slot), (s / S) & 1) || *abort_flag) {
        atomicAdd(&g_tc_wait_timeouts, 1u);
        *abort_flag = 1;
        break;
      }
      float w[16];
      DequantHalf<QT>(raw + slot * kTileRows * kRaw + m * kRaw, m, (s * kBB) & 15, half, w);
      uint32_t h[16], l[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        h[i] = Tf32Head(__float_as_uint(w[i]));
        l[i] = __float_as_uint(w[i] - __uint_as_float(h[i]));
      }
      // (the MMAs that last read this slot's A tiles finished before its
      // loads were issued; order the stores after that)
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      // this warp's 32 lanes (rows), 16 columns each for its half of the block
      const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      TmemStore16(lane_base + a_hi_col(slot) + 16 * half, h);
      TmemStore16(lane_base + a_lo_col(slot) + 16 * half, l);
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      MbarArrive(dequantised(slot));
    }
    // epilogue: lane = weight row, column = token; warps w and w + 4 read
    // the same TMEM lanes (32 (w % 4) ..) and split the tokens
    const bool ok = MbarWait(acc_ready, 0) && !*abort_flag;
    if (!ok && lane == 0) atomicAdd(&g_tc_wait_timeouts, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const int row = n0 + m;
    const uint32_t taddr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll 1
    for (int c = half * (kTileTokens / 2); c < (half + 1) * (kTileTokens / 2); c += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32"
          " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
            "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
            "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr + c));
      asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
      if (row < n) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = t0 + c + j;
          if (t < t_rows)
            y[static_cast<int64_t>(t) * n + row] =
                ok ? __uint_as_float(v[j]) : __int_as_float(0x7fc00000);
        }
      }
    }
  }
  // let any load still in flight land before the CTA leaves (only after a
  // timeout can a consumer have stopped early)
  __syncthreads();
  if (warp == 8 && lane == 0 && *abort_flag) {
    for (int s = issued - S > 0 ? issued - S : 0; s < issued; ++s)
      MbarWait(full(s % S), (s / S) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 10) {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kTmemColumns)
                 : "memory");
  }
}

// x -> TF32 head and exact tail, one float4 per thread.
__global__ void __launch_bounds__(256)
    SplitTf32Kernel(const float4* __restrict__ x, uint4* __restrict__ xh,
                    uint4* __restrict__ xl, int64_t count4) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= count4) return;
  const float4 v = x[i];
  uint4 h, l;
  h.x = Tf32Head(__float_as_uint(v.x));
  h.y = Tf32Head(__float_as_uint(v.y));
  h.z = Tf32Head(__float_as_uint(v.z));
  h.w = Tf32Head(__float_as_uint(v.w));
  l.x = __float_as_uint(v.x - __uint_as_float(h.x));
  l.y = __float_as_uint(v.y - __uint_as_float(h.y));
  l.z = __float_as_uint(v.z - __uint_as_float(h.z));
  l.w = __float_as_uint(v.w - __uint_as_float(h.w));
  xh[i] = h;
  xl[i] = l;
}

PFN_cuTensorMapEncodeTiled_v12000 EncodeFn() {
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

bool Map2D(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner,
           uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
           CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = EncodeFn();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int QT>
int LaunchTc(int count, const void* const* w, const int64_t* n, int64_t k, int64_t row_bytes,
             const float* xh, const float* xl, int64_t t_rows, float* const* y,
             cudaStream_t s) {
  TcGroup grp{};
  grp.count = count;
  grp.t_tiles = static_cast<int>((t_rows + kTileTokens - 1) / kTileTokens);
  grp.t_rows = static_cast<int>(t_rows);
  grp.k = static_cast<int>(k);
  int64_t tiles = 0;
  for (int m = 0; m < count; ++m) {
    if (!Map2D(&grp.w[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, w[m],
               static_cast<uint64_t>(row_bytes), static_cast<uint64_t>(n[m]),
               static_cast<uint64_t>(row_bytes), TcRawBytes(QT), kTileRows,
               QT == MLB_F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: tensor map encoding failed");
    grp.y[m] = y[m];
    grp.n[m] = static_cast<int>(n[m]);
    grp.tile_begin[m] = static_cast<int>(tiles);
    tiles += (n[m] + kTileRows - 1) / kTileRows * grp.t_tiles;
  }
  grp.tile_begin[count] = static_cast<int>(tiles);
  if (tiles > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: too many tiles");
  if (!Map2D(&grp.xh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xh, static_cast<uint64_t>(k),
             static_cast<uint64_t>(t_rows), static_cast<uint64_t>(k) * 4, kStepK, kTileTokens,
             CU_TENSOR_MAP_SWIZZLE_128B) ||
      !Map2D(&grp.xl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xl, static_cast<uint64_t>(k),
             static_cast<uint64_t>(t_rows), static_cast<uint64_t>(k) * 4, kStepK, kTileTokens,
             CU_TENSOR_MAP_SWIZZLE_128B))
    return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: tensor map encoding failed");
  auto kernel = LinearTcKernel<QT>;
  constexpr int shm = TcSmemBytes(QT);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, shm) !=
      cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "mlb_linear_rows_f32: shared memory opt-in");
  }
  Launch(kernel, static_cast<unsigned>(tiles), kTcThreads, shm, s, grp);
  return CheckLaunch("mlb_linear_rows_f32");
}

}  // namespace

// Host side of mlb_wait_timeouts for this file's kernels.
unsigned int TcWaitTimeouts() {
  unsigned int count = 0;
  if (cudaMemcpyFromSymbol(&count, g_tc_wait_timeouts, sizeof(count)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count;
}

}  // namespace mlb

// Token counts from which the tensor-core form is used (below it the GEMV
// form of mlb_linear_f32 reads every weight once per 8 tokens and wins).
static constexpr int64_t kTcMinTokens = 48;

namespace mlb {
int GemvTcGroup(int count, const void* const* w, int qtype, const int64_t* n, int64_t k,
                const float* x, int64_t t_rows, float* const* y, cudaStream_t s);  // gemv.cu
// linear_f16.cu
bool LinearF16Eligible(int qtype, int64_t k, int64_t row_bytes);
int LinearF16(int count, const void* const* w, int qtype, const int64_t* n, int64_t k,
              int64_t row_bytes, const float* x, int64_t t_rows, float* const* y,
              float* scratch, cudaStream_t s);
}  // namespace mlb

extern "C" int64_t mlb_linear_rows_scratch_floats(int64_t k, int64_t t_rows) {
  if (k <= 0 || t_rows < 0) return -1;
  return 2 * k * t_rows + 8;  // xh, xl (+ room to align each to 16 bytes)
}

namespace {

// Shared by the single and grouped entries: W_m . x for m < count, all
// matrices of the same format and width k.
int LinearRowsGroup(int count, const void* const* w, int qtype, const int64_t* n, int64_t k,
                    const float* x, int64_t t_rows, float* const* y, float* scratch,
                    int64_t scratch_floats, void* stream) {
  using namespace mlb;
  if (qtype < MLB_F32 || qtype > MLB_Q4_1)
    return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: unknown qtype");
  if (count < 1 || count > kMaxGroup || w == nullptr || n == nullptr || y == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: bad group");
  if (k <= 0 || k > INT_MAX || t_rows < 0 || t_rows > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: bad shape");
  for (int m = 0; m < count; ++m)
    if (n[m] < 0 || n[m] > INT_MAX) return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: bad shape");
  if (t_rows == 0) return MLB_OK;
  const int64_t row_bytes = mlb_row_bytes(qtype, k);
  bool tc = t_rows >= kTcMinTokens && (k % kStepK) == 0 && (row_bytes % 16) == 0 &&
            x != nullptr && Aligned16(x);
  for (int m = 0; m < count; ++m)
    tc = tc && w[m] != nullptr && (reinterpret_cast<uintptr_t>(w[m]) & 15u) == 0;
  if (!tc) {  // the GEMV form: all matrices in one tensor-core launch when
              // they qualify, else matrix by matrix on the CUDA cores
    if (t_rows < kTcMinTokens && x != nullptr) {
      const void* ws[kMaxGroup];
      int64_t ns[kMaxGroup];
      float* ys[kMaxGroup];
      int used = 0;
      bool ok = true;
      for (int m = 0; m < count; ++m) {
        if (n[m] == 0) continue;
        ok = ok && w[m] != nullptr && y[m] != nullptr;
        ws[used] = w[m];
        ns[used] = n[m];
        ys[used] = y[m];
        ++used;
      }
      if (ok && used == 0) return MLB_OK;
      if (ok) {
        const int rc = GemvTcGroup(used, ws, qtype, ns, k, x, t_rows, ys, AsStream(stream));
        if (rc != -1) return rc;
      }
    }
    for (int m = 0; m < count; ++m) {
      if (n[m] == 0) continue;
      const int rc = mlb_linear_f32(w[m], qtype, n[m], k, x, t_rows, y[m], stream);
      if (rc != MLB_OK) return rc;
    }
    return MLB_OK;
  }
  for (int m = 0; m < count; ++m)
    if (y[m] == nullptr && n[m] > 0) return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: null pointer");
  if (scratch == nullptr || scratch_floats < mlb_linear_rows_scratch_floats(k, t_rows))
    return Fail(MLB_ERR_ARG, "mlb_linear_rows_f32: scratch too small");
  // matrices with rows (an empty one adds no tile)
  const void* ws[kMaxGroup];
  int64_t ns[kMaxGroup];
  float* ys[kMaxGroup];
  int used = 0;
  for (int m = 0; m < count; ++m) {
    if (n[m] == 0) continue;
    ws[used] = w[m];
    ns[used] = n[m];
    ys[used] = y[m];
    ++used;
  }
  if (used == 0) return MLB_OK;
  float* xh = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(scratch) + 15) & ~uintptr_t{15});
  float* xl = xh + k * t_rows;  // k % 32 == 0: still 16-byte aligned
  cudaStream_t s = AsStream(stream);
  // Q8_0 / Q4_0: d * q and x in exact fp16 pieces (linear_f16.cu)
  if (LinearF16Eligible(qtype, k, row_bytes))
    return LinearF16(used, ws, qtype, ns, k, row_bytes, x, t_rows, ys, xh, s);
  const int64_t count4 = k * t_rows / 4;
  Launch(SplitTf32Kernel, static_cast<unsigned>((count4 + 255) / 256), 256, 0, s, reinterpret_cast<const float4*>(x), reinterpret_cast<uint4*>(xh),
      reinterpret_cast<uint4*>(xl), count4);
  const int rc = CheckLaunch("mlb_linear_rows_f32");
  if (rc != MLB_OK) return rc;
  switch (qtype) {
    case MLB_F32: return LaunchTc<MLB_F32>(used, ws, ns, k, row_bytes, xh, xl, t_rows, ys, s);
    case MLB_Q8_0: return LaunchTc<MLB_Q8_0>(used, ws, ns, k, row_bytes, xh, xl, t_rows, ys, s);
    case MLB_Q4_0: return LaunchTc<MLB_Q4_0>(used, ws, ns, k, row_bytes, xh, xl, t_rows, ys, s);
    default: return LaunchTc<MLB_Q4_1>(used, ws, ns, k, row_bytes, xh, xl, t_rows, ys, s);
  }
}

}  // namespace

extern "C" int mlb_linear_rows_f32(const void* w, int qtype, int64_t n, int64_t k,
                                   const float* x, int64_t t_rows, float* y, float* scratch,
                                   int64_t scratch_floats, void* stream) {
  return LinearRowsGroup(1, &w, qtype, &n, k, x, t_rows, &y, scratch, scratch_floats, stream);
}

extern "C" int mlb_linear_rows_group_f32(int count, const void* const* w, int qtype,
                                         const int64_t* n, int64_t k, const float* x,
                                         int64_t t_rows, float* const* y, float* scratch,
                                         int64_t scratch_floats, void* stream) {
  return LinearRowsGroup(count, w, qtype, n, k, x, t_rows, y, scratch, scratch_floats, stream);
}
