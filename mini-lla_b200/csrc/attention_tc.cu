// Causal attention of prompt rows on the 5th-generation tensor cores.
//
// Reference arithmetic (src/forward.cc:50-95 AttentionHead / Attention), per
// query row r (the token at position + r) and query head h reading kv head
// h / G (GQA, G = n_heads / n_kv_heads):
//   score_t = dot(q, k_t) * (1 / sqrt(hd)) for t <= position + r
//   w = softmax(score);  out = sum_t w_t * v_t
// with fp32 dot products and sums.  The CUDA-core tile kernel (attention.cu)
// computes the same thing on the FMA pipes.
//
// Accuracy on TF32 tensor cores: operands are split into TF32 pieces,
// each rounded to 11 significant bits: a = ah + al + e with |e| <= 2^-22 |a|
// (Q, P, V), and K into three, k = kh + km + kl + e' with |e'| <= 2^-33 |k|.
// S = Q K^T accumulates qh.kh in one fp32 accumulator and the small cross
// terms qh.km + ql.kh + qh.kl + ql.km in a second, added once at the end —
// the large sum then sees one rounding per 8 dimensions, and what is
// dropped (ql.kl, Q's residual) is ~2^-22 of each product, so a score is as
// close to the exact dot product as the reference's sequential fp32 sum.
// O = P V accumulates ph.vh + ph.vl + pl.vh (P's and V's residuals ~2^-22).
// Results match the reference within the attention tests' bar, 1e-5 *
// sum_t w_t |v_t[i]| per output, and stay within the reference's own error
// when scores spread widely.
//
// Design: CTA = (kv head g, 128 query vectors: 128 / G consecutive rows x G
// heads of the group); the visible keys in blocks of 32; 288 threads:
//   - warps 0-3, thread = query vector = tensor-memory lane: write the tile's
//     Q pieces into tensor memory once (the A operand of S = Q K^T); per
//     block read S (tcgen05.ld, 32 columns), apply the scale and the causal
//     mask, keep the online softmax (running reference max m, sum l) and
//     write P's pieces into shared memory (the A operand of O += P V);
//     the reference max moves only when a block's max exceeds it by more
//     than 8 (p stays below e^8), and then O is rescaled in tensor memory;
//     finally O / l to global memory;
//   - warps 4-7: copy each block's K and V rows of kv head g from global
//     memory, split them into pieces and store them in the 128-byte-swizzled
//     K-major layouts the MMA reads (K as [keys][hd], V transposed to
//     [hd][keys]); keys past the tile's last visible one are zeros;
//   - warp 8: allocates tensor memory; one lane issues the MMAs — per block
//     5 x hd/8 MMAs (M 128, N 32, K 8) for S into one of two S buffers
//     (head and cross-term accumulators), and after the softmax of the
//     previous block 3 x 4 MMAs (M 128, N hd, K 8) accumulating P V into O
//     — and commits each group to its barrier.
// Two stages of K / V pieces and of P pieces; every wait is bounded (a wait
// that gives up is counted in mlb_wait_timeouts and the CTA writes NaN in
// place of its outputs).
#include <cuda.h>

#include <climits>
#include <cmath>
#include <cstdint>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kAtVectors = 128;  // query vectors per CTA (MMA M, tensor-memory lanes)
constexpr int kAtKeys = 32;      // keys per block (S's N, P V's K)
constexpr int kAtThreads = 288;  // 4 softmax warps, 4 loader warps, 1 MMA warp
constexpr int kAtTmemColumns = 512;
constexpr int kAtOCol = 0;       // O accumulator: hd columns
constexpr int kAtSCol = 128;     // two S buffers: 32 head + 32 cross-term columns each
constexpr int kAtQhCol = 256;    // Q head: hd columns
constexpr int kAtQlCol = 384;    // Q tail: hd columns
constexpr float kAtRescale = 8.0f;  // reference max moves when exceeded by this

// Shared-memory layout from a 1024-byte aligned base, for head_dim HD:
// per stage K's three pieces ([HD / 32 sub-tiles][32 keys][128 B] each),
// V's two ([HD rows][128 B]); then per stage P head, P tail ([128][128 B]);
// then the barriers and the tensor-memory address (225 KB at HD = 128).
template <int HD>
struct AtLayout {
  static constexpr int kKBytes = HD * kAtKeys * 4;   // one piece of K (or V)
  static constexpr int kStageBytes = 5 * kKBytes;    // Kh, Km, Kl, Vh, Vl
  static constexpr int kPBytes = kAtVectors * kAtKeys * 4;
  static constexpr int kPOffset = 2 * kStageBytes;
  static constexpr int kBarOffset = kPOffset + 4 * kPBytes;
  // q_full, kv_full[2], s_full[2], s_empty[2], p_full[2], pv_done[2], o_final
  static constexpr int kBarriers = 12;
  static constexpr int kSmemBytes = kBarOffset + 8 * kBarriers + 16 + 1024;
};

__device__ __forceinline__ uint32_t AtSmem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void AtBarInit(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void AtArrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool AtTryWait(uint32_t bar, uint32_t parity) {
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
__device__ __forceinline__ bool AtWait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 21); ++i)
    if (AtTryWait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void AtCommit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row
// atoms of 128-byte rows 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t AtDesc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;          // LBO (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // SBO
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version
  d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
  return d;
}
// Instruction descriptor: D fp32, A and B TF32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t AtInstr(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kAtVectors >> 4) << 24);
}
// D[tmem] (+)= A[a_tmem] . B[b]^T, A read from tensor memory.
__device__ __forceinline__ void AtMmaTs(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[a] . B[b]^T, both from shared memory.
__device__ __forceinline__ void AtMmaSs(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void AtLd32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void AtSt32(uint32_t taddr, const uint32_t (&v)[32]) {
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

// TF32 head of an fp32 value, rounded to the nearest 11-significant-bit
// value (ties away from zero); the remainder v - head is exact and at most
// 2^-11 |v|.  Infinities and NaNs pass through as heads (their remainders
// are NaN, which keeps a non-finite input visible in the result).
__device__ __forceinline__ float Tf32Round(float v) {
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}
// The two pieces the MMAs read: head = Tf32Round(v) and tail =
// Tf32Round(v - head), both exact TF32 values (the tensor core reads them
// without loss); v - head - tail is at most 2^-22 |v| and is dropped.
__device__ __forceinline__ void Tf32Split(float v, float& head, float& tail) {
  head = Tf32Round(v);
  tail = Tf32Round(v - head);
}
// Three exact TF32 pieces: what is left, v - head - mid - low, is at most
// 2^-33 |v|.
__device__ __forceinline__ void Tf32Split3(float v, float& head, float& mid, float& low) {
  head = Tf32Round(v);
  const float r = v - head;
  mid = Tf32Round(r);
  low = Tf32Round(r - mid);
}

// Byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled tile
// of 128-byte rows (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t AtSwz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace

// Bounded waits of the tensor-core attention kernel that gave up.
__device__ unsigned int g_at_wait_timeouts;

namespace {

struct AtArgs {
  const float* q;       // [rows, n_heads, hd]
  const float* keys;    // [max_seq, n_kv_heads, hd]
  const float* values;
  float* out;           // [rows, n_heads, hd]
  int64_t position;     // query row r is the token at position + r
  int64_t rows;
  int n_heads;
  int n_kv_heads;
  float scale;
};

template <int G, int HD>
__global__ void __launch_bounds__(kAtThreads, 1) AttnTcKernel(const AtArgs a) {
  using L = AtLayout<HD>;
  constexpr int QR = kAtVectors / G;  // query rows per CTA
  constexpr int QV = QR * G;          // used vectors (<= 128)
  constexpr int KSTEPS = HD / 8;      // K = 8 TF32 per MMA over hd
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  extern __shared__ __align__(16) uint8_t at_raw[];
  const uint32_t raw_addr = AtSmem(at_raw);
  uint8_t* base = at_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = AtSmem(base);
  auto kh = [&](int s) { return sbase + s * L::kStageBytes; };
  auto km = [&](int s) { return sbase + s * L::kStageBytes + L::kKBytes; };
  auto kl = [&](int s) { return sbase + s * L::kStageBytes + 2 * L::kKBytes; };
  auto vh = [&](int s) { return sbase + s * L::kStageBytes + 3 * L::kKBytes; };
  auto vl = [&](int s) { return sbase + s * L::kStageBytes + 4 * L::kKBytes; };
  auto ph = [&](int s) { return sbase + L::kPOffset + s * 2 * L::kPBytes; };
  auto pl = [&](int s) { return sbase + L::kPOffset + s * 2 * L::kPBytes + L::kPBytes; };
  const uint32_t bars = sbase + L::kBarOffset;
  const uint32_t q_full = bars;
  auto kv_full = [&](int s) { return bars + 8 * (1 + s); };
  auto s_full = [&](int s) { return bars + 8 * (3 + s); };
  auto s_empty = [&](int s) { return bars + 8 * (5 + s); };
  auto p_full = [&](int s) { return bars + 8 * (7 + s); };
  auto pv_done = [&](int s) { return bars + 8 * (9 + s); };
  const uint32_t o_final = bars + 8 * 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::kBarOffset + 8 * L::kBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x;  // kv head
  // the last row tiles see the most keys: schedule them first
  const int64_t r0 = static_cast<int64_t>(gridDim.y - 1 - blockIdx.y) * QR;
  const int64_t last_row = r0 + QR - 1 < a.rows - 1 ? r0 + QR - 1 : a.rows - 1;
  const int64_t kv_limit = a.position + last_row + 1;  // keys any row of the tile sees
  const int nb = static_cast<int>((kv_limit + kAtKeys - 1) / kAtKeys);
  const int64_t q_stride = static_cast<int64_t>(a.n_heads) * HD;
  const int64_t kv_stride = static_cast<int64_t>(a.n_kv_heads) * HD;

  if (threadIdx.x == 0) {
    AtBarInit(q_full, 128);
    for (int s = 0; s < 2; ++s) {
      AtBarInit(kv_full(s), 128);
      AtBarInit(s_full(s), 1);
      AtBarInit(s_empty(s), 128);
      AtBarInit(p_full(s), 128);
      AtBarInit(pv_done(s), 1);
    }
    AtBarInit(o_final, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     AtSmem(tmem_slot)),
                 "r"(kAtTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  auto give_up = [&]() {
    if (!*abort_flag) atomicAdd(&g_at_wait_timeouts, 1u);
    *abort_flag = 1;
  };
  // warps 0-7: a wait whose outcome every lane of the warp shares (the
  // tensor-memory loads and stores after it are warp-collective)
  auto warp_wait = [&](uint32_t bar, uint32_t parity) {
    const bool ok = AtWait(bar, parity) && !*abort_flag;
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = AtWait(q_full, 0) && !*abort_flag;
      if (!ok) give_up();
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      for (int b = 0; ok && b <= nb; ++b) {
        if (b < nb) {  // S(b) = Q K_b^T into S buffer b % 2
          const int s = b & 1;
          ok = AtWait(kv_full(s), (b >> 1) & 1) &&
               (b < 2 || AtWait(s_empty(s), ((b - 2) >> 1) & 1)) && !*abort_flag;
          if (!ok) {
            give_up();
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
          const uint32_t dh = tmem + kAtSCol + 2 * kAtKeys * s;  // qh.kh
          const uint32_t dx = dh + kAtKeys;                       // cross terms
#pragma unroll 4
          for (int j = 0; j < KSTEPS; ++j) {
            const uint32_t off = static_cast<uint32_t>((j >> 2) * (kAtKeys * 128) + (j & 3) * 32);
            const uint64_t bh = AtDesc(kh(s) + off);
            const uint64_t bm = AtDesc(km(s) + off);
            const uint64_t bl = AtDesc(kl(s) + off);
            const uint32_t qh = tmem + kAtQhCol + 8 * j, ql = tmem + kAtQlCol + 8 * j;
            AtMmaTs(dh, qh, bh, AtInstr(kAtKeys), j != 0 ? 1u : 0u);
            AtMmaTs(dx, qh, bm, AtInstr(kAtKeys), j != 0 ? 1u : 0u);
            AtMmaTs(dx, ql, bh, AtInstr(kAtKeys), 1u);
            AtMmaTs(dx, qh, bl, AtInstr(kAtKeys), 1u);
            AtMmaTs(dx, ql, bm, AtInstr(kAtKeys), 1u);
          }
          AtCommit(s_full(s));
        }
        if (b >= 1) {  // O += P(b-1) V(b-1)
          const int jb = b - 1, s = jb & 1;
          ok = AtWait(p_full(s), (jb >> 1) & 1) && !*abort_flag;
          if (!ok) {
            give_up();
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll
          for (int j = 0; j < kAtKeys / 8; ++j) {
            const uint64_t ah = AtDesc(ph(s) + 32 * j);
            const uint64_t al = AtDesc(pl(s) + 32 * j);
            const uint64_t bh = AtDesc(vh(s) + 32 * j);
            const uint64_t bl = AtDesc(vl(s) + 32 * j);
            AtMmaSs(tmem + kAtOCol, ah, bh, AtInstr(HD), (jb | j) != 0 ? 1u : 0u);
            AtMmaSs(tmem + kAtOCol, ah, bl, AtInstr(HD), 1u);
            AtMmaSs(tmem + kAtOCol, al, bh, AtInstr(HD), 1u);
          }
          AtCommit(pv_done(s));
        }
      }
      AtCommit(o_final);  // every MMA issued so far has finished
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ loaders
    // Block b + 1's rows are loaded into registers as soon as block b's
    // pieces are stored, so their latency passes while the loader waits for
    // the next stage to be free; all of a block's loads are in flight at
    // once.  K: lane = float4 chunk along hd, keys lw, lw + 4, ...; V: lane =
    // key, float4 chunks lw, lw + 4, ... of hd (stored transposed).
    constexpr int KR = kAtKeys / 4;  // keys per loader warp
    constexpr int VC = HD / 16;      // V float4 chunks per lane
    const int lw = warp - 4;
    float4 kx[KR], vx[VC];
    auto load_block = [&](int b) {
#pragma unroll
      for (int i = 0; i < KR; ++i) {
        const int64_t t = static_cast<int64_t>(b) * kAtKeys + lw + 4 * i;
        kx[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane < HD / 4 && t < kv_limit)
          kx[i] = *reinterpret_cast<const float4*>(a.keys + t * kv_stride +
                                                   static_cast<int64_t>(g) * HD + 4 * lane);
      }
      const int64_t t = static_cast<int64_t>(b) * kAtKeys + lane;
      const float* vrow = a.values + t * kv_stride + static_cast<int64_t>(g) * HD;
#pragma unroll
      for (int i = 0; i < VC; ++i) {
        vx[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < kv_limit) vx[i] = *reinterpret_cast<const float4*>(vrow + 4 * (lw + 4 * i));
      }
    };
    if (nb > 0) load_block(0);
    for (int b = 0; b < nb; ++b) {
      const int s = b & 1;
      if (b >= 2 && !warp_wait(pv_done(s), ((b - 2) >> 1) & 1)) {
        give_up();
        break;
      }
      uint8_t* khp = base + (kh(s) - sbase);
      uint8_t* kmp = base + (km(s) - sbase);
      uint8_t* klp = base + (kl(s) - sbase);
      uint8_t* vhp = base + (vh(s) - sbase);
      uint8_t* vlp = base + (vl(s) - sbase);
      if (lane < HD / 4) {
        const int st = lane >> 3, ch = lane & 7;
#pragma unroll
        for (int i = 0; i < KR; ++i) {
          const int key = lw + 4 * i;
          float4 h, mid, r;
          Tf32Split3(kx[i].x, h.x, mid.x, r.x);
          Tf32Split3(kx[i].y, h.y, mid.y, r.y);
          Tf32Split3(kx[i].z, h.z, mid.z, r.z);
          Tf32Split3(kx[i].w, h.w, mid.w, r.w);
          const uint32_t off = static_cast<uint32_t>(st * (kAtKeys * 128)) + AtSwz(key, ch);
          *reinterpret_cast<float4*>(khp + off) = h;
          *reinterpret_cast<float4*>(kmp + off) = mid;
          *reinterpret_cast<float4*>(klp + off) = r;
        }
      }
      {
        const int ch = lane >> 2, w = lane & 3;
#pragma unroll
        for (int i = 0; i < VC; ++i) {
          const int c4 = lw + 4 * i;
          const float xs[4] = {vx[i].x, vx[i].y, vx[i].z, vx[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = 4 * c4 + e;
            float hv, tv;
            Tf32Split(xs[e], hv, tv);
            const uint32_t off = AtSwz(d, ch) + 4 * w;
            *reinterpret_cast<float*>(vhp + off) = hv;
            *reinterpret_cast<float*>(vlp + off) = tv;
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      AtArrive(kv_full(s));
      if (b + 1 < nb) load_block(b + 1);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int v = threadIdx.x;  // query vector = tensor-memory lane
    const int64_t row = r0 + v / G;
    const bool live = v < QV && row < a.rows;
    const int64_t qpos = live ? a.position + row : -1;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    {  // the vector's Q pieces into tensor memory (A of S = Q K^T)
      const float* qv = a.q + row * q_stride + static_cast<int64_t>(g * G + v % G) * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t hv[32], lv[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live) x = *reinterpret_cast<const float4*>(qv + 32 * c + 4 * i);
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float h, t;
            Tf32Split(xs[e], h, t);
            hv[4 * i + e] = __float_as_uint(h);
            lv[4 * i + e] = __float_as_uint(t);
          }
        }
        AtSt32(lane_base + kAtQhCol + 32 * c, hv);
        AtSt32(lane_base + kAtQlCol + 32 * c, lv);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      AtArrive(q_full);
    }
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    uint8_t* prow_h[2] = {base + (ph(0) - sbase), base + (ph(1) - sbase)};
    uint8_t* prow_l[2] = {base + (pl(0) - sbase), base + (pl(1) - sbase)};
    for (int b = 0; b < nb; ++b) {
      const int s = b & 1;
      if (!warp_wait(s_full(s), (b >> 1) & 1)) {
        give_up();
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      uint32_t sv[32], sx[32];
      AtLd32(lane_base + kAtSCol + 2 * kAtKeys * s, sv);
      AtLd32(lane_base + kAtSCol + 2 * kAtKeys * s + kAtKeys, sx);
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      AtArrive(s_empty(s));
      const int64_t t0 = static_cast<int64_t>(b) * kAtKeys;
      float sc[32];
      float bm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float dot = __fadd_rn(__uint_as_float(sv[j]), __uint_as_float(sx[j]));
        sc[j] = t0 + j <= qpos ? __fmul_rn(dot, a.scale) : -INFINITY;
        bm = fmaxf(bm, sc[j]);
      }
      // the reference max moves when the block's max exceeds it by more than
      // kAtRescale (or on the first visible key); O and l are then rescaled
      // by exp(m - m_new).  The tensor-memory loads and stores are
      // warp-collective, so the warp rescales together when any of its
      // vectors needs it, each lane by its own factor (1 if it needs none).
      const bool move = bm != -INFINITY && (m == -INFINITY || bm > m + kAtRescale);
      const bool scale_o = move && m != -INFINITY;  // O holds earlier blocks (b >= 1)
      const float al = scale_o ? expf(m - bm) : 1.0f;
      if (__any_sync(0xffffffffu, scale_o)) {
        if (!warp_wait(pv_done((b - 1) & 1), ((b - 1) >> 1) & 1)) {
          give_up();
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t ov[32];
          AtLd32(lane_base + kAtOCol + 32 * c, ov);
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * al);
          AtSt32(lane_base + kAtOCol + 32 * c, ov);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      }
      l *= al;
      if (move) m = bm;
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        sc[j] = sc[j] == -INFINITY ? 0.0f : expf(sc[j] - m);  // now p
        sum += sc[j];
      }
      l += sum;
      // P buffer s was last read by P V of block b - 2
      if (b >= 2 && !warp_wait(pv_done(s), ((b - 2) >> 1) & 1)) {
        give_up();
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float4 h, r;
        Tf32Split(sc[4 * c], h.x, r.x);
        Tf32Split(sc[4 * c + 1], h.y, r.y);
        Tf32Split(sc[4 * c + 2], h.z, r.z);
        Tf32Split(sc[4 * c + 3], h.w, r.w);
        *reinterpret_cast<float4*>(prow_h[s] + AtSwz(v, c)) = h;
        *reinterpret_cast<float4*>(prow_l[s] + AtSwz(v, c)) = r;
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      AtArrive(p_full(s));
    }
    // O / l to global memory
    ok = __all_sync(0xffffffffu, ok);
    ok = ok && warp_wait(o_final, 0);
    if (!ok) give_up();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    float* o = a.out + row * q_stride + static_cast<int64_t>(g * G + v % G) * HD;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t ov[32];
      AtLd32(lane_base + kAtOCol + 32 * c, ov);
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 y =
              ok ? make_float4(__fdiv_rn(__uint_as_float(ov[4 * i]), l),
                               __fdiv_rn(__uint_as_float(ov[4 * i + 1]), l),
                               __fdiv_rn(__uint_as_float(ov[4 * i + 2]), l),
                               __fdiv_rn(__uint_as_float(ov[4 * i + 3]), l))
                 : make_float4(NAN, NAN, NAN, NAN);
          *reinterpret_cast<float4*>(o + 32 * c + 4 * i) = y;
        }
      }
    }
  }
  // every role has left its loop; once the MMAs in flight have finished
  // (o_final, bounded) the tensor memory goes back
  if (threadIdx.x == 8 * 32 && *abort_flag) AtWait(o_final, 0);
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 8) {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kAtTmemColumns)
                 : "memory");
  }
}

template <int G, int HD>
int LaunchAttnTc(const AtArgs& a, cudaStream_t s) {
  constexpr int QR = kAtVectors / G;
  constexpr int smem = AtLayout<HD>::kSmemBytes;
  auto kernel = AttnTcKernel<G, HD>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "attention (tensor cores): shared memory opt-in");
  }
  const dim3 grid(static_cast<unsigned>(a.n_kv_heads),
                  static_cast<unsigned>((a.rows + QR - 1) / QR));
  Launch(kernel, grid, kAtThreads, static_cast<size_t>(smem), s, a);
  return CheckLaunch("attention (tensor cores)");
}

template <int HD>
int LaunchAttnTcGroup(const AtArgs& a, int group, cudaStream_t s) {
  switch (group) {
    case 1: return LaunchAttnTc<1, HD>(a, s);
    case 2: return LaunchAttnTc<2, HD>(a, s);
    case 3: return LaunchAttnTc<3, HD>(a, s);
    case 4: return LaunchAttnTc<4, HD>(a, s);
    case 5: return LaunchAttnTc<5, HD>(a, s);
    case 6: return LaunchAttnTc<6, HD>(a, s);
    case 7: return LaunchAttnTc<7, HD>(a, s);
    default: return LaunchAttnTc<8, HD>(a, s);
  }
}

}  // namespace

// Prompt rows on the tensor cores: group 1 .. 8, head_dim 64 or 128, 16-byte
// aligned q / keys / values / out; -1 when the shape is not covered.  The
// caller checked the sizes and the position range.
int AttentionRowsTc(const float* q, const float* keys, const float* values, float* out,
                    int64_t position, int64_t rows, int n_heads, int n_kv_heads, int hd,
                    cudaStream_t s) {
  const int group = n_heads / n_kv_heads;
  if (group < 1 || group > 8 || (hd != 64 && hd != 128) || !Aligned16(q) || !Aligned16(keys) ||
      !Aligned16(values) || !Aligned16(out) || rows > 65535LL * (kAtVectors / group))
    return -1;
  AtArgs a{q, keys, values, out, position, rows, n_heads, n_kv_heads,
           1.0f / std::sqrt(static_cast<float>(hd))};
  return hd == 64 ? LaunchAttnTcGroup<64>(a, group, s) : LaunchAttnTcGroup<128>(a, group, s);
}

unsigned int AttnTcWaitTimeouts() {
  unsigned int count = 0;
  if (cudaMemcpyFromSymbol(&count, g_at_wait_timeouts, sizeof(count)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count;
}

}  // namespace mlb
