// Decode attention over the KV cache, and the KV-cache write.
//
// Reference arithmetic (src/forward.cc:50-95 AttentionHead / Attention, and
// src/kv_cache.cc:25-40 Write; GPU src/cuda_attention.cu:13-106):
//   score_t = dot(q_h, k_t) * (1 / sqrt(hd))        for t <= position
//   w = softmax(score);  out_h = sum_t w_t * v_t
// with query head h reading kv head h / (n_heads / n_kv_heads) (GQA).  The
// reference runs one CTA per query head, serial over positions with a block
// reduction per position; scores for all positions live in shared memory.
//
// Here (flash-decoding): the visible positions are split into S slices; CTA
// (g, s) takes kv head g with all of its query heads — K and V rows are read
// from HBM once per group, not once per query head — and slice s, keeping an
// online softmax (running max m, sum l, accumulator acc) per query head.
// Slice partials (m, l, acc[hd]) go to caller-provided scratch; a second
// kernel rescales and sums them.  Sums run in a different order than the
// reference and exp is CUDA's expf, so the output matches within
// 1e-5 * sum_t w_t |v_t[i]| (tests).
//
// Layout: keys / values of one layer [max_seq, n_kv_heads, hd] fp32 (the
// reference's CudaKvCache per layer); q, out [n_heads, hd].
// HBM roofline: 8 * (position + 1) * n_kv_heads * hd bytes of K and V, plus
// q and out.
#include <climits>
#include <cmath>
#include <mutex>
#include <string>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kMaxGroup = 8;      // query heads per kv head handled per CTA
constexpr int kMaxHdVec = 2;      // float4 per lane: hd <= 256
constexpr int kMinSlice = 128;    // positions per slice at least (but see Splits)
// A slice partial is (m, l, two unused floats, acc[hd]): acc rows start
// 16 bytes after the record, so they stay 16-byte aligned for the combine's
// cp.async copies.
constexpr int kPartHead = 4;

struct AttnArgs {
  const float* q;
  const float* keys;
  const float* values;
  float* out;
  float* scratch;  // [rows][n_heads][splits][kPartHead + hd]
  int64_t visible; // visible positions of query row 0 (row r sees visible + r)
  int n_heads;
  int n_kv_heads;
  int hd;
  int splits;
  int64_t slice;   // positions per slice
  float scale;
};

// Number of position slices for a launch of `rows` query rows (of the
// longest row's positions), the largest of: slices of kMinSlice positions up
// to the kSliceCtasPerSm CTAs that every SM holds at once (the slice
// kernel's shared-memory limit at head_dim 128; rounded down so that no CTA
// waits for a second wave); slices of 64 positions up to 2 CTAs per SM; of
// 32 positions up to one CTA per SM.  Short caches get more, shorter
// slices while the grid is small; long ones keep slices of 128 positions or
// more.  Measured on B200 (a CUDA graph of calls over cache copies), 32 / 8
// heads x 128, slices of 128 / 64 / 32 positions: position 511 8.8 / 6.7 /
// 5.9 us, 2047 9.8 / 9.4 / 11.2 (440 CTAs of 37 positions: fixed costs
// dominate), 4095 with 74-position slices at 3 CTAs per SM 14.5 against
// 12.8; 16383 30.7 (55 slices, 3 CTAs per SM; 37 slices at 2 per SM were
// slower).
constexpr int kSliceCtasPerSm = 3;
int Splits(int n_kv_heads, int64_t visible, int64_t rows = 1) {
  const int64_t ctas = static_cast<int64_t>(n_kv_heads) * rows;
  const int64_t sms = SmCount();
  const auto slices = [&](int64_t positions, int64_t per_sm) {
    const int64_t by_length = (visible + positions - 1) / positions;
    const int64_t by_grid = per_sm * sms / ctas;
    return by_length < by_grid ? by_length : by_grid;
  };
  int64_t s = slices(kMinSlice, kSliceCtasPerSm);
  const int64_t mid = slices(64, 2), small = slices(32, 1);
  if (mid > s) s = mid;
  if (small > s) s = small;
  if (s < 1) s = 1;
  return static_cast<int>(s);
}

template <int G, int NV>
__global__ void __launch_bounds__(kAttnWarps * 32) AttnPartialKernel(AttnArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  __shared__ float sm_m[kAttnWarps][G];
  __shared__ float sm_l[kAttnWarps][G];
  __shared__ float4 sm_acc[kAttnWarps][G][32 * NV];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = blockIdx.x;   // kv head
  const int s = blockIdx.y;   // slice
  const int64_t row = blockIdx.z;
  const int hd4 = a.hd >> 2;
  const int64_t t_begin = s * a.slice;
  const int64_t t_end = min(a.visible + row, t_begin + a.slice);  // may be empty
  const float* q_row = a.q + row * a.n_heads * a.hd;
  float* scratch_row = a.scratch + row * a.n_heads * a.splits * (a.hd + kPartHead);
  const int64_t stride4 = static_cast<int64_t>(a.n_kv_heads) * hd4;

  float4 q[G][NV];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int i = lane + 32 * v;
      q[h][v] = i < hd4 ? __ldg(reinterpret_cast<const float4*>(q_row) +
                                (static_cast<int64_t>(g) * G + h) * hd4 + i)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  float m[G], l[G];
  float4 acc[G][NV];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[h][v] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float4* k4 = reinterpret_cast<const float4*>(a.keys) + static_cast<int64_t>(g) * hd4;
  const float4* v4 = reinterpret_cast<const float4*>(a.values) + static_cast<int64_t>(g) * hd4;
  for (int64_t t = t_begin + warp; t < t_end; t += kAttnWarps) {
    float4 kk[NV], vv[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int i = lane + 32 * v;
      kk[v] = i < hd4 ? __ldg(k4 + t * stride4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      vv[v] = i < hd4 ? __ldg(v4 + t * stride4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float dot = 0.0f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        dot = fmaf(q[h][v].x, kk[v].x, dot);
        dot = fmaf(q[h][v].y, kk[v].y, dot);
        dot = fmaf(q[h][v].z, kk[v].z, dot);
        dot = fmaf(q[h][v].w, kk[v].w, dot);
      }
      const float score = __fmul_rn(WarpSum(dot), a.scale);
      const float m_new = fmaxf(m[h], score);
      const float alpha = expf(m[h] - m_new);  // 0 on the first position
      const float p = expf(score - m_new);
      l[h] = fmaf(l[h], alpha, p);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        acc[h][v].x = fmaf(acc[h][v].x, alpha, p * vv[v].x);
        acc[h][v].y = fmaf(acc[h][v].y, alpha, p * vv[v].y);
        acc[h][v].z = fmaf(acc[h][v].z, alpha, p * vv[v].z);
        acc[h][v].w = fmaf(acc[h][v].w, alpha, p * vv[v].w);
      }
      m[h] = m_new;
    }
  }
  // combine the warps of this CTA, then write the slice partial
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      sm_m[warp][h] = m[h];
      sm_l[warp][h] = l[h];
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) sm_acc[warp][h][lane + 32 * v] = acc[h][v];
  }
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sm_m[w][h]);
    float ll = 0.0f;
    float4 aa[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) aa[v] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = sm_m[w][h] == -INFINITY ? 0.0f : expf(sm_m[w][h] - mm);
      ll = fmaf(sm_l[w][h], f, ll);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const float4 x = sm_acc[w][h][lane + 32 * v];
        aa[v].x = fmaf(x.x, f, aa[v].x);
        aa[v].y = fmaf(x.y, f, aa[v].y);
        aa[v].z = fmaf(x.z, f, aa[v].z);
        aa[v].w = fmaf(x.w, f, aa[v].w);
      }
    }
    const int head = g * G + h;
    float* part = scratch_row + (static_cast<int64_t>(head) * a.splits + s) * (a.hd + kPartHead);
    if (lane == 0) {
      part[0] = mm;
      part[1] = ll;
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int i = lane + 32 * v;
      if (i < hd4) {
        part[kPartHead + 4 * i + 0] = aa[v].x;
        part[kPartHead + 4 * i + 1] = aa[v].y;
        part[kPartHead + 4 * i + 2] = aa[v].z;
        part[kPartHead + 4 * i + 3] = aa[v].w;
      }
    }
  }
}

// out[h][i] = sum_s acc_s[i] * f_s / sum_s l_s * f_s, f_s = e^(m_s - M),
// M = max_s m_s (f_s = 0 for a slice that saw no position).  The CTA's
// threads take the slices in parallel for M and for the factors (kept in
// shared memory) and sum l_s * f_s as a block tree; thread i then adds its
// output's terms in slice order.  STAGED (hd % 4 == 0, scratch 16-byte
// aligned): the slices' acc rows pass through shared memory in chunks of
// `chunk` slices, two buffers, copied with cp.async — the first chunk's
// copies issued before the (m, l) loads and chunk k + 1's while chunk k is
// summed — so a combine of one chunk waits for a single round trip of
// loads; otherwise thread i reads its terms from global memory, eight loads
// in flight.  (Measured on B200, 32 heads x 128, cold: 6.7 us at 16 slices
// for per-thread slice loops of dependent loads, 3.6 us staged; 25.4 us at
// 111 slices, 28 heads, for the global-memory loop.)
constexpr int kCombineSmemBytes = 96 * 1024;

template <bool STAGED>
__global__ void __launch_bounds__(256) AttnCombineKernel(AttnArgs a, int chunk) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  extern __shared__ __align__(16) float csm[];
  __shared__ float scratch[2][32];
  const int splits = a.splits;
  const int hd = a.hd;
  const int stride = hd + kPartHead;
  const int head = blockIdx.x;
  const int64_t row = blockIdx.y;
  const float* base = a.scratch + (row * a.n_heads + head) * static_cast<int64_t>(splits) * stride;
  float* factor = csm;                          // [splits]
  float* bufs = csm + ((splits + 3) & ~3);      // [2][chunk][hd] when STAGED
  // copies the acc rows of slices [c0, c0 + chunk) into buffer b, one group
  const auto stage = [&](int c0, int b) {
    const int hd4 = hd >> 2;
    const int n = min(chunk, splits - c0);
    float* dst = bufs + static_cast<int64_t>(b) * chunk * hd;
    for (int i = threadIdx.x; i < n * hd4; i += blockDim.x) {
      const int sl = i / hd4, c = i - sl * hd4;
      CopyAsync16(dst + sl * hd + 4 * c,
                  base + static_cast<int64_t>(c0 + sl) * stride + kPartHead + 4 * c);
    }
    CopyAsyncCommit();
  };
  if (STAGED) stage(0, 0);
  float mm = -INFINITY;
  for (int s = threadIdx.x; s < splits; s += blockDim.x)
    mm = fmaxf(mm, base[static_cast<int64_t>(s) * stride]);
  mm = BlockMax(mm, scratch[0]);
  float ll = 0.0f;
  for (int s = threadIdx.x; s < splits; s += blockDim.x) {
    const float ms = base[static_cast<int64_t>(s) * stride];
    const float f = ms == -INFINITY ? 0.0f : expf(ms - mm);
    factor[s] = f;
    ll = fmaf(base[static_cast<int64_t>(s) * stride + 1], f, ll);
  }
  ll = BlockSum(ll, scratch[1]);  // its barrier also publishes factor[]
  // thread i < hd owns output i (blockDim >= hd when STAGED; the launch
  // gives hd <= 256 threads of one output each)
  const int i = threadIdx.x;
  float sum = 0.0f;
  if (STAGED) {
    for (int c0 = 0, b = 0; c0 < splits; c0 += chunk, b ^= 1) {
      if (c0 + chunk < splits) stage(c0 + chunk, b ^ 1);
      else CopyAsyncCommit();  // an empty group keeps the count uniform
      CopyAsyncWait<1>();
      __syncthreads();  // chunk c0's copies, by every thread, have landed
      if (i < hd) {
        const float* acc = bufs + static_cast<int64_t>(b) * chunk * hd + i;
        const int n = min(chunk, splits - c0);
        for (int s = 0; s < n; ++s) sum = fmaf(acc[s * hd], factor[c0 + s], sum);
      }
      __syncthreads();  // buffer b is read before it is refilled
    }
    if (i < hd) a.out[(row * a.n_heads + head) * a.hd + i] = __fdiv_rn(sum, ll);
  } else {
    for (int o = i; o < hd; o += blockDim.x) {
      const float* acc = base + kPartHead + o;
      float t = 0.0f;
#pragma unroll 8
      for (int s = 0; s < splits; ++s)
        t = fmaf(acc[static_cast<int64_t>(s) * stride], factor[s], t);
      a.out[(row * a.n_heads + head) * a.hd + o] = __fdiv_rn(t, ll);
    }
  }
}

// Position-parallel form of the slice kernel (head_dim 64 or 128).  Each
// warp walks its slice's positions kQuadBlock = 8 at a time, double-buffered:
// the K and V rows of its next block are copied into shared memory with
// cp.async while the current block is computed (2 x ~8.7 KB per warp, so
// 3 CTAs share an SM).  Lanes 4r .. 4r + 3 score position r of the block
// against all G query heads, one quarter of the dimensions each, and add
// the quarters with two shuffles.  Bank layout: chunk c (16 bytes) of
// quarter j of a K row, and of each q vector, is stored at Q * j + (c ^ j)
// (Q chunks per quarter) and K rows are padded by 16 floats, so the 8 lanes
// of a quarter-warp (2 positions x 4 quarters) read 8 distinct bank groups
// and the q reads are 4-address broadcasts.  Per block and head the online
// softmax takes 3 shuffles for the max and 3 for the sum (the 4 lanes of a
// position hold the same score); P.V walks the block's rows with the G
// probabilities of a row broadcast from shared memory and each lane
// accumulating DPL = hd / 32 dimensions of the V row.  The 4 warps' states
// are merged and written as the slice partial, as in AttnPartialKernel.
// (Measured on B200, 32 / 8 heads x 128 at position 16383: the form before,
// 2 lanes per position over 16-position blocks loaded and then computed,
// spent ~40 % of each block waiting for its own copies.)
constexpr int kQuadBlock = 8;

template <int HD4>
__host__ __device__ constexpr int QuadKRowFloats() { return 4 * HD4 + 16; }
template <int HD4>
__host__ __device__ constexpr int QuadStageFloats() {  // one block: K rows + V rows
  return kQuadBlock * (QuadKRowFloats<HD4>() + 4 * HD4);
}

template <int G, int HD4>
__global__ void __launch_bounds__(kAttnWarps * 32) AttnQuadPartialKernel(AttnArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  constexpr int HD = 4 * HD4;
  constexpr int DPL = HD / 32;        // dimensions per lane in P.V (2 or 4)
  constexpr int Q = HD4 / 4;          // 16-byte chunks per quarter (4 or 8)
  constexpr int KRF = QuadKRowFloats<HD4>();
  constexpr int SF = QuadStageFloats<HD4>();
  static_assert(Q == 4 || Q == 8, "head_dim 64 or 128");
  // dynamic: q of the G heads, then per warp two staged blocks of K and V
  // rows (the warps' final accumulators reuse that area once the loop is done)
  extern __shared__ __align__(16) float lsm[];
  float* qs = lsm;                   // [G][HD], quarter-swizzled
  float* stages = lsm + G * HD;      // [kAttnWarps][2][K rows | V rows]
  __shared__ __align__(16) float sm_p[kAttnWarps][kQuadBlock][G];  // a block's probabilities
  __shared__ float sm_m[kAttnWarps][G];
  __shared__ float sm_l[kAttnWarps][G];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = blockIdx.x;
  const int s = blockIdx.y;
  const int64_t row = blockIdx.z;
  const int64_t t_begin = s * a.slice;
  const int64_t t_end = min(a.visible + row, t_begin + a.slice);
  const float* q_row = a.q + row * a.n_heads * HD;
  float* scratch_row = a.scratch + row * a.n_heads * a.splits * (HD + kPartHead);
  const int64_t kv_stride = static_cast<int64_t>(a.n_kv_heads) * HD;
  const float* kbase = a.keys + static_cast<int64_t>(g) * HD;
  const float* vbase = a.values + static_cast<int64_t>(g) * HD;

  for (int i = threadIdx.x; i < G * HD4; i += blockDim.x) {
    const int h = i / HD4, c = i - h * HD4;
    const int j = c / Q, cq = c - j * Q;
    reinterpret_cast<float4*>(qs)[h * HD4 + Q * j + (cq ^ j)] =
        __ldg(reinterpret_cast<const float4*>(q_row + static_cast<int64_t>(g) * G * HD) + i);
  }
  __syncthreads();

  const int pos = lane >> 2;      // position of this lane quad in the block
  const int quarter = lane & 3;   // which quarter of the dimensions it scores
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[h][e] = 0.0f;
  }
  float* wst = stages + warp * 2 * SF;
  // copies rows blk .. blk + n - 1 into stage `buf` (coalesced 16-byte
  // chunks; K chunks quarter-swizzled into padded rows) as one cp.async group
  // (a warp covers RPI rows per pass; lane l always copies chunk l % HD4 of
  // rows l / HD4 + RPI * pass, so its offsets are fixed)
  constexpr int RPI = 32 / HD4;
  const int sc_c = lane % HD4;
  const int sc_r0 = lane / HD4;
  const int sc_kdst = 4 * (Q * (sc_c / Q) + ((sc_c % Q) ^ (sc_c / Q)));
  const auto stage = [&](int buf, int64_t blk, int n) {
    float* kw = wst + buf * SF + sc_kdst;
    float* vw = wst + buf * SF + kQuadBlock * KRF + 4 * sc_c;
    const float* ks = kbase + 4 * sc_c;
    const float* vs = vbase + 4 * sc_c;
#pragma unroll
    for (int it = 0; it < kQuadBlock / RPI; ++it) {
      const int r = sc_r0 + RPI * it;
      if (r < n) {
        const int64_t off = (blk + r) * kv_stride;
        CopyAsync16(kw + r * KRF, ks + off);
        CopyAsync16(vw + r * HD, vs + off);
      }
    }
    CopyAsyncCommit();
  };
  // positions of the block that starts at b (b < t_end)
  const auto block_len = [t_end](int64_t b) {
    return static_cast<int>(t_end - b < kQuadBlock ? t_end - b : kQuadBlock);
  };
  constexpr int64_t kStep = static_cast<int64_t>(kAttnWarps) * kQuadBlock;
  int64_t blk = t_begin + static_cast<int64_t>(warp) * kQuadBlock;
  if (blk < t_end) stage(0, blk, block_len(blk));
  for (int buf = 0; blk < t_end; blk += kStep, buf ^= 1) {
    const int n = block_len(blk);
    const int64_t next = blk + kStep;
    if (next < t_end)
      stage(buf ^ 1, next, block_len(next));
    else
      CopyAsyncCommit();  // an empty group keeps the count below uniform
    CopyAsyncWait<1>();   // this block's copies have landed
    __syncwarp();
    const float* kw = wst + buf * SF;
    const float* vw = kw + kQuadBlock * KRF;
    // this quarter's part of the scores of position blk + pos, its chunks
    // in order (the physical slot of chunk c of quarter j is c ^ j)
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.0f;
    if (pos < n) {
      const float* kr = kw + pos * KRF + 4 * Q * quarter;
      const float* qq = qs + 4 * Q * quarter;
#pragma unroll
      for (int c = 0; c < Q; ++c) {
        const int pc = c ^ quarter;
        const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * pc);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float4 qv = *reinterpret_cast<const float4*>(qq + h * HD + 4 * pc);
          sc[h] = fmaf(qv.x, kv.x, sc[h]);
          sc[h] = fmaf(qv.y, kv.y, sc[h]);
          sc[h] = fmaf(qv.z, kv.z, sc[h]);
          sc[h] = fmaf(qv.w, kv.w, sc[h]);
        }
      }
    }
    // full dot products on all 4 lanes of a position, then the block's
    // online softmax over its 8 positions (heads interleaved per shuffle)
    float p[G], score[G], bm[G], ps[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float dot = sc[h] + __shfl_xor_sync(0xffffffffu, sc[h], 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      score[h] = pos < n ? __fmul_rn(dot, a.scale) : -INFINITY;
      bm[h] = score[h];
    }
#pragma unroll
    for (int o = 16; o >= 4; o >>= 1)
#pragma unroll
      for (int h = 0; h < G; ++h) bm[h] = fmaxf(bm[h], __shfl_xor_sync(0xffffffffu, bm[h], o));
    float alpha[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float m_new = fmaxf(m[h], bm[h]);
      alpha[h] = expf(m[h] - m_new);  // 0 on the first block
      p[h] = pos < n ? expf(score[h] - m_new) : 0.0f;
      m[h] = m_new;
      ps[h] = p[h];
    }
#pragma unroll
    for (int o = 16; o >= 4; o >>= 1)
#pragma unroll
      for (int h = 0; h < G; ++h) ps[h] += __shfl_xor_sync(0xffffffffu, ps[h], o);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      l[h] = fmaf(l[h], alpha[h], ps[h]);
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[h][e] *= alpha[h];
    }
    // the block's probabilities, G per position, for every lane's P.V
    if (quarter == 0 && pos < n) {
#pragma unroll
      for (int h = 0; h < G; ++h) sm_p[warp][pos][h] = p[h];
    }
    __syncwarp();
    // P.V over the block's positions (V row r: lane owns dims DPL * lane ..)
#pragma unroll
    for (int r = 0; r < kQuadBlock; ++r) {
      if (r >= n) break;
      const float* vr = vw + r * HD + DPL * lane;
      float v[DPL];
      if (DPL == 4) {
        const float4 x = *reinterpret_cast<const float4*>(vr);
        v[0] = x.x; v[1] = x.y; v[2 % DPL] = x.z; v[3 % DPL] = x.w;
      } else {
        const float2 x = *reinterpret_cast<const float2*>(vr);
        v[0] = x.x; v[1] = x.y;
      }
      float pr[G];  // position r's probabilities (a shared-memory broadcast)
      if constexpr (G % 4 == 0) {
#pragma unroll
        for (int h4 = 0; h4 < G; h4 += 4) {
          const float4 p4 = *reinterpret_cast<const float4*>(&sm_p[warp][r][h4]);
          pr[h4] = p4.x;
          pr[h4 + 1] = p4.y;
          pr[h4 + 2] = p4.z;
          pr[h4 + 3] = p4.w;
        }
      } else {
#pragma unroll
        for (int h = 0; h < G; ++h) pr[h] = sm_p[warp][r][h];
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[h][e] = fmaf(pr[h], v[e], acc[h][e]);
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
  }
  // merge the 4 warps, then write the slice partial
  __syncthreads();  // every warp is done with its stages: reuse the area
  float* sm_acc = stages;  // [kAttnWarps][G][HD]
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      sm_m[warp][h] = m[h];
      sm_l[warp][h] = l[h];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) sm_acc[(warp * G + h) * HD + DPL * lane + e] = acc[h][e];
  }
  __syncthreads();
  for (int h = warp; h < G; h += kAttnWarps) {
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sm_m[w][h]);
    float ll = 0.0f, aa[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) aa[e] = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = sm_m[w][h] == -INFINITY ? 0.0f : expf(sm_m[w][h] - mm);
      ll = fmaf(sm_l[w][h], f, ll);
#pragma unroll
      for (int e = 0; e < DPL; ++e) aa[e] = fmaf(sm_acc[(w * G + h) * HD + DPL * lane + e], f, aa[e]);
    }
    float* part = scratch_row + (static_cast<int64_t>(g * G + h) * a.splits + s) * (HD + kPartHead);
    if (lane == 0) {
      part[0] = mm;
      part[1] = ll;
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) part[kPartHead + DPL * lane + e] = aa[e];
  }
}

template <int G, int HD4>
int LaunchQuad(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  constexpr size_t kStage = static_cast<size_t>(kAttnWarps) * 2 * QuadStageFloats<HD4>();
  constexpr size_t kAcc = static_cast<size_t>(kAttnWarps) * G * 4 * HD4;
  static_assert(kAcc <= kStage, "the merge reuses the stage area");
  constexpr size_t shm = sizeof(float) * (G * 4 * HD4 + kStage);
  auto kernel = AttnQuadPartialKernel<G, HD4>;
  if (shm > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(shm)) != cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "attention: shared memory opt-in");
  }
  Launch(kernel, grid, kAttnWarps * 32, shm, s, a);
  return CheckLaunch("mlb_attention_decode_f32");
}

template <int G>
int LaunchPartial(const AttnArgs& a, int64_t rows, int nv, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.n_kv_heads), static_cast<unsigned>(a.splits),
                  static_cast<unsigned>(rows));
  if (a.hd == 128) {
    return LaunchQuad<G, 32>(a, grid, s);
  } else if (a.hd == 64) {
    return LaunchQuad<G, 16>(a, grid, s);
  } else if (nv == 1) {
    Launch(AttnPartialKernel<G, 1>, grid, kAttnWarps * 32, 0, s, a);
  } else {
    Launch(AttnPartialKernel<G, 2>, grid, kAttnWarps * 32, 0, s, a);
  }
  return CheckLaunch("mlb_attention_decode_f32");
}

__global__ void __launch_bounds__(256)
    KvWriteKernel(float* keys, float* values, const float* k, const float* v,
                  int64_t base, int64_t count) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < count; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    keys[base + i] = k[i];
    values[base + i] = v[i];
  }
}

int ValidateAttention(const float* q, const float* keys, const float* values,
                      const float* out, int64_t position, int64_t max_seq,
                      int n_heads, int n_kv_heads, int hd) {
  if (q == nullptr || keys == nullptr || values == nullptr || out == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_attention_decode_f32: null pointer");
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 ||
      n_heads / n_kv_heads > kMaxGroup || hd <= 0 || hd % 4 != 0 ||
      hd > 128 * kMaxHdVec)
    return Fail(MLB_ERR_ARG,
                "mlb_attention_decode_f32: heads must divide, group <= 8, "
                "hd % 4 == 0, hd <= 256");
  if (!Aligned16(q) || !Aligned16(keys) || !Aligned16(values))
    return Fail(MLB_ERR_ARG, "mlb_attention_decode_f32: q/keys/values misaligned");
  if (position < 0 || position >= max_seq)
    return Fail(MLB_ERR_RANGE, "mlb_attention_decode_f32: position out of range");
  return MLB_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Prompt chunks: tiles of query rows.
//
// CTA (kv head g, tile of QR = 64 / G consecutive query rows; tiles of the
// most keys first) holds the QV = QR * G <= 64 query vectors of its rows and
// group in shared memory and walks
// the visible positions in blocks of 64 keys: every K/V block is staged once
// (cp.async, double-buffered) for all QV query vectors instead of once per
// query row.  256 threads, each owning 4 query vectors x 4 keys of the score
// tile (thread (a = tid / 16, b = tid % 16): vectors 4a .. 4a + 3, keys
// b, b + 16, b + 32, b + 48): 8 shared loads feed 64 FMAs per 4 dimensions.
// Rows are padded by 16 bytes so the 8 keys of a quarter-warp sit on
// distinct banks.  The online softmax of a vector is reduced over the 16
// threads that share it; the probabilities go to shared memory transposed
// ([key][vector]) so that P.V reads the 4 probabilities of a thread's
// vectors with one 16-byte load, and each thread accumulates its 4 vectors
// x float4 columns c, c + 16, ... of the output.  Future keys score -inf;
// no slice partials.
constexpr int kTileKeys = 64;
constexpr int kTileQv = 64;
constexpr int kTileThreads = 256;
constexpr int kPsStride = kTileQv + 4;  // transposed probability tile row

struct AttnTileArgs {
  const float* q;
  const float* keys;
  const float* values;
  float* out;
  int64_t position;  // query row r is the token at position + r
  int64_t rows;
  int64_t max_seq;
  int n_heads;
  int n_kv_heads;
  float scale;
};

template <int HD4>
__host__ __device__ constexpr int TileRowFloats() { return 4 * HD4 + 4; }  // one padded row

template <int G, int HD4>
constexpr size_t TileSmemBytes() {
  return sizeof(float) * (static_cast<size_t>(kTileQv + 4 * kTileKeys) * TileRowFloats<HD4>() +
                          static_cast<size_t>(kTileKeys) * kPsStride);
}

template <int G, int HD4>
__global__ void __launch_bounds__(kTileThreads, 1) AttnRowTileKernel(AttnTileArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  constexpr int QR = kTileQv / G;  // query rows per CTA
  constexpr int QV = QR * G;
  constexpr int RF = TileRowFloats<HD4>();
  constexpr int HD = 4 * HD4;
  constexpr int CPT = HD4 / 16;    // float4 columns per thread in P.V (1 or 2)
  extern __shared__ __align__(16) float tsm[];
  float* qs = tsm;                           // [QV][RF]
  float* ks = qs + kTileQv * RF;             // [2][kTileKeys][RF]
  float* vs = ks + 2 * kTileKeys * RF;       // [2][kTileKeys][RF]
  float* ps = vs + 2 * kTileKeys * RF;       // [kTileKeys][kPsStride]

  const int g = blockIdx.x;
  // the last row tiles see the most keys: schedule them first
  const int64_t r0 = static_cast<int64_t>(gridDim.y - 1 - blockIdx.y) * QR;
  const int tid = threadIdx.x;
  const int qa = tid >> 4;   // vectors 4 qa .. 4 qa + 3
  const int kb4 = tid & 15;  // keys kb4 + 16 j (scores); float4 columns kb4 + 16 c (P.V)
  const int64_t row_stride = static_cast<int64_t>(a.n_heads) * HD;
  const int64_t kv_stride = static_cast<int64_t>(a.n_kv_heads) * HD;

  // the tile's query vectors (rows beyond the chunk read as zeros)
  for (int i = tid; i < kTileQv * HD4; i += kTileThreads) {
    const int v = i / HD4, d4 = i - v * HD4;
    const int64_t row = r0 + v / G;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < QV && row < a.rows)
      x = *reinterpret_cast<const float4*>(a.q + row * row_stride +
                                           static_cast<int64_t>(g * G + v % G) * HD + 4 * d4);
    *reinterpret_cast<float4*>(qs + v * RF + 4 * d4) = x;
  }
  const int64_t last_row = r0 + QR - 1 < a.rows - 1 ? r0 + QR - 1 : a.rows - 1;
  const int64_t visible = a.position + last_row + 1;  // keys any row of the tile sees
  const int blocks = static_cast<int>((visible + kTileKeys - 1) / kTileKeys);

  auto stage = [&](int b) {
    float* kd = ks + (b & 1) * kTileKeys * RF;
    float* vd = vs + (b & 1) * kTileKeys * RF;
    for (int i = tid; i < kTileKeys * HD4; i += kTileThreads) {
      const int key = i / HD4, d4 = i - key * HD4;
      const int64_t t = static_cast<int64_t>(b) * kTileKeys + key;
      if (t < a.max_seq) {
        const int64_t off = t * kv_stride + static_cast<int64_t>(g) * HD + 4 * d4;
        CopyAsync16(kd + key * RF + 4 * d4, a.keys + off);
        CopyAsync16(vd + key * RF + 4 * d4, a.values + off);
      }
    }
  };

  int64_t qpos[4];
  float m[4], l[4];
  float4 acc[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * qa + i;
    qpos[i] = v < QV ? a.position + r0 + v / G : -1;  // padding vectors see nothing
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  stage(0);
  CopyAsyncCommit();
  for (int b = 0; b < blocks; ++b) {
    if (b + 1 < blocks) stage(b + 1);
    CopyAsyncCommit();
    CopyAsyncWait<1>();
    __syncthreads();  // block b (and, on b == 0, the query tile) in place
    const float* kb = ks + (b & 1) * kTileKeys * RF;
    const float* vb = vs + (b & 1) * kTileKeys * RF;
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
#pragma unroll 2
    for (int d4 = 0; d4 < HD4; ++d4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qv[i] = *reinterpret_cast<const float4*>(qs + (4 * qa + i) * RF + 4 * d4);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        kv[j] = *reinterpret_cast<const float4*>(kb + (kb4 + 16 * j) * RF + 4 * d4);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[i][j] = fmaf(qv[i].x, kv[j].x, sc[i][j]);
          sc[i][j] = fmaf(qv[i].y, kv[j].y, sc[i][j]);
          sc[i][j] = fmaf(qv[i].z, kv[j].z, sc[i][j]);
          sc[i][j] = fmaf(qv[i].w, kv[j].w, sc[i][j]);
        }
    }
    // online softmax of each of the 4 vectors over the block's 64 keys
    // (16 threads share a vector: lanes 0-15 or 16-31 of a warp)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t t = static_cast<int64_t>(b) * kTileKeys + kb4 + 16 * j;
        sc[i][j] = t <= qpos[i] ? __fmul_rn(sc[i][j], a.scale) : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float nm = fmaxf(m[i], mx);
      // a vector with no visible key yet keeps p = 0 (no -inf - -inf)
      const float al = nm == -INFINITY ? 1.0f : expf(m[i] - nm);
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[i][j] = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - nm);  // now p
        sum += sc[i][j];
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l[i] = fmaf(l[i], al, sum);
      m[i] = nm;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        acc[i][c].x *= al;
        acc[i][c].y *= al;
        acc[i][c].z *= al;
        acc[i][c].w *= al;
      }
    }
    // probabilities, transposed: ps[key][vector]
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(ps + (kb4 + 16 * j) * kPsStride + 4 * qa) =
          make_float4(sc[0][j], sc[1][j], sc[2][j], sc[3][j]);
    __syncthreads();  // every vector's probabilities are in place
#pragma unroll 4
    for (int key = 0; key < kTileKeys; ++key) {
      const float4 p = *reinterpret_cast<const float4*>(ps + key * kPsStride + 4 * qa);
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const float4 vv = *reinterpret_cast<const float4*>(vb + key * RF + 4 * (kb4 + 16 * c));
        acc[0][c].x = fmaf(p.x, vv.x, acc[0][c].x);
        acc[0][c].y = fmaf(p.x, vv.y, acc[0][c].y);
        acc[0][c].z = fmaf(p.x, vv.z, acc[0][c].z);
        acc[0][c].w = fmaf(p.x, vv.w, acc[0][c].w);
        acc[1][c].x = fmaf(p.y, vv.x, acc[1][c].x);
        acc[1][c].y = fmaf(p.y, vv.y, acc[1][c].y);
        acc[1][c].z = fmaf(p.y, vv.z, acc[1][c].z);
        acc[1][c].w = fmaf(p.y, vv.w, acc[1][c].w);
        acc[2][c].x = fmaf(p.z, vv.x, acc[2][c].x);
        acc[2][c].y = fmaf(p.z, vv.y, acc[2][c].y);
        acc[2][c].z = fmaf(p.z, vv.z, acc[2][c].z);
        acc[2][c].w = fmaf(p.z, vv.w, acc[2][c].w);
        acc[3][c].x = fmaf(p.w, vv.x, acc[3][c].x);
        acc[3][c].y = fmaf(p.w, vv.y, acc[3][c].y);
        acc[3][c].z = fmaf(p.w, vv.z, acc[3][c].z);
        acc[3][c].w = fmaf(p.w, vv.w, acc[3][c].w);
      }
    }
    __syncthreads();  // buffers of block b and the probability tile are free
  }
  CopyAsyncWait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * qa + i;
    const int64_t row = r0 + v / G;
    if (v >= QV || row >= a.rows) continue;
    float* o = a.out + row * row_stride + static_cast<int64_t>(g * G + v % G) * HD;
#pragma unroll
    for (int c = 0; c < CPT; ++c)
      *reinterpret_cast<float4*>(o + 4 * (kb4 + 16 * c)) =
          make_float4(__fdiv_rn(acc[i][c].x, l[i]), __fdiv_rn(acc[i][c].y, l[i]),
                      __fdiv_rn(acc[i][c].z, l[i]), __fdiv_rn(acc[i][c].w, l[i]));
  }
}

template <int G, int HD4>
int LaunchRowTile(const AttnTileArgs& a, cudaStream_t s) {
  constexpr int QR = kTileQv / G;
  constexpr size_t shm = TileSmemBytes<G, HD4>();
  auto kernel = AttnRowTileKernel<G, HD4>;
  if (shm > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(shm)) != cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "attention: shared memory opt-in");
  }
  const dim3 grid(static_cast<unsigned>(a.n_kv_heads),
                  static_cast<unsigned>((a.rows + QR - 1) / QR));
  Launch(kernel, grid, kTileThreads, shm, s, a);
  return CheckLaunch("attention (row tiles)");
}

// Row tiles when they fill the GPU (n_kv_heads x row tiles >= half the SMs),
// group 1 .. 8, head_dim 64 or 128; -1 when the shape does not fit.
template <int HD4>
int LaunchRowTiles(const AttnTileArgs& a, int group, cudaStream_t s) {
  switch (group) {
    case 1: return LaunchRowTile<1, HD4>(a, s);
    case 2: return LaunchRowTile<2, HD4>(a, s);
    case 3: return LaunchRowTile<3, HD4>(a, s);
    case 4: return LaunchRowTile<4, HD4>(a, s);
    case 5: return LaunchRowTile<5, HD4>(a, s);
    case 6: return LaunchRowTile<6, HD4>(a, s);
    case 7: return LaunchRowTile<7, HD4>(a, s);
    default: return LaunchRowTile<8, HD4>(a, s);
  }
}

// attention_tc.cu: prompt rows on the tensor cores (-1: shape not covered)
int AttentionRowsTc(const float* q, const float* keys, const float* values, float* out,
                    int64_t position, int64_t rows, int n_heads, int n_kv_heads, int hd,
                    cudaStream_t s);

// Kernel choice for prompt rows (mlb_set_attention_path): 0 automatic, 1 the
// CUDA-core kernels, 2 the tensor cores wherever the shape allows.
int g_attention_path = 0;

int AttentionRowTiles(const float* q, const float* keys, const float* values, float* out,
                      int64_t position, int64_t rows, int64_t max_seq, int n_heads,
                      int n_kv_heads, int hd, cudaStream_t s) {
  const int group = n_heads / n_kv_heads;
  if (group < 1 || group > 8 || (hd != 64 && hd != 128) || !Aligned16(out) ||
      rows > 65535LL * (kTileQv / group))
    return -1;
  if (static_cast<int64_t>(n_kv_heads) * ((rows + kTileQv / group - 1) / (kTileQv / group)) <
      SmCount() / 2)
    return -1;
  AttnTileArgs a{q, keys, values, out, position, rows, max_seq, n_heads, n_kv_heads,
                 1.0f / std::sqrt(static_cast<float>(hd))};
  return hd == 64 ? LaunchRowTiles<16>(a, group, s) : LaunchRowTiles<32>(a, group, s);
}

// The slice combine of `rows` query rows: staged through shared memory
// (chunks of as many slices as two buffers of kCombineSmemBytes hold) when
// hd <= 256 is a multiple of 4 and the scratch is 16-byte aligned.
int LaunchCombine(const AttnArgs& a, const float* scratch, int64_t rows, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.n_heads), static_cast<unsigned>(rows));
  const int threads = a.hd < 256 ? ((a.hd + 31) / 32) * 32 : 256;
  const size_t factors = sizeof(float) * ((a.splits + 3) & ~3);
  if ((a.hd % 4) == 0 && a.hd <= 256 && Aligned16(scratch)) {
    int chunk = static_cast<int>((kCombineSmemBytes - factors) / (2 * sizeof(float) * a.hd));
    if (chunk > a.splits) chunk = a.splits;
    if (chunk >= 1) {
      const size_t shm = factors + 2 * sizeof(float) * static_cast<size_t>(chunk) * a.hd;
      if (shm > 48 * 1024 &&
          cudaFuncSetAttribute(AttnCombineKernel<true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(shm)) != cudaSuccess) {
        cudaGetLastError();
        return Fail(MLB_ERR_CUDA, "attention: shared memory opt-in");
      }
      Launch(AttnCombineKernel<true>, grid, threads, shm, s, a, chunk);
      return CheckLaunch("attention");
    }
  }
  Launch(AttnCombineKernel<false>, grid, threads, factors, s, a, 0);
  return CheckLaunch("attention");
}

// Shared by the entry points: scratch must hold AttentionScratchFloats() for
// `rows` query rows, row r seeing visible + r positions.
int64_t AttentionScratchFloats(int n_heads, int n_kv_heads, int hd, int64_t visible,
                               int64_t rows) {
  return rows * n_heads * Splits(n_kv_heads, visible + rows - 1, rows) * (hd + kPartHead);
}

// Query rows [0, rows) at positions position + r (row r attends to cache
// positions 0 .. position + r); q, out [rows, n_heads, hd].
int AttentionRows(const float* q, const float* keys, const float* values, float* out,
                  int64_t position, int64_t rows, int64_t max_seq, int n_heads,
                  int n_kv_heads, int hd, float* scratch, void* stream) {
  int rc = ValidateAttention(q, keys, values, out, position, max_seq, n_heads,
                             n_kv_heads, hd);
  if (rc != MLB_OK) return rc;
  if (rows < 1 || position + rows > max_seq)
    return Fail(MLB_ERR_RANGE, "attention: rows leave the cache");
  cudaStream_t s = AsStream(stream);
  // the tensor cores from 512 query rows (automatic: measured on B200 at
  // 32 / 8 heads x 128, 2048 rows 0.52 ms against 1.09 on the CUDA cores, 512
  // rows 0.083 against 0.086, fewer rows slower), or for any prompt chunk of
  // two rows or more (path 2)
  if (rows > 1 && g_attention_path != 1 && (g_attention_path == 2 || rows >= 512)) {
    rc = AttentionRowsTc(q, keys, values, out, position, rows, n_heads, n_kv_heads, hd, s);
    if (rc >= 0) return rc;  // -1: shape not covered
  }
  if (rows > 1) {
    rc = AttentionRowTiles(q, keys, values, out, position, rows, max_seq, n_heads,
                           n_kv_heads, hd, s);
    if (rc >= 0) return rc;  // -1: shape not covered, use the split form
  }
  AttnArgs a{};
  a.keys = keys;
  a.values = values;
  a.scratch = scratch;
  a.n_heads = n_heads;
  a.n_kv_heads = n_kv_heads;
  a.hd = hd;
  a.splits = Splits(n_kv_heads, position + rows, rows);
  a.slice = (position + rows + a.splits - 1) / a.splits;
  // 1 / std::sqrt((float)head_dim) as the reference computes it (forward.cc:75)
  a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
  const int nv = (hd / 4 + 31) / 32;
  const int64_t per_row = static_cast<int64_t>(n_heads) * hd;
  constexpr int64_t kMaxRowsPerLaunch = 65535;  // grid.z
  for (int64_t r0 = 0; r0 < rows; r0 += kMaxRowsPerLaunch) {
    const int64_t rc_rows = rows - r0 < kMaxRowsPerLaunch ? rows - r0 : kMaxRowsPerLaunch;
    a.q = q + r0 * per_row;
    a.out = out + r0 * per_row;
    a.visible = position + r0 + 1;
    switch (n_heads / n_kv_heads) {
      case 1: rc = LaunchPartial<1>(a, rc_rows, nv, s); break;
      case 2: rc = LaunchPartial<2>(a, rc_rows, nv, s); break;
      case 3: rc = LaunchPartial<3>(a, rc_rows, nv, s); break;
      case 4: rc = LaunchPartial<4>(a, rc_rows, nv, s); break;
      case 5: rc = LaunchPartial<5>(a, rc_rows, nv, s); break;
      case 6: rc = LaunchPartial<6>(a, rc_rows, nv, s); break;
      case 7: rc = LaunchPartial<7>(a, rc_rows, nv, s); break;
      case 8: rc = LaunchPartial<8>(a, rc_rows, nv, s); break;
    }
    if (rc != MLB_OK) return rc;
    rc = LaunchCombine(a, scratch, rc_rows, s);
    if (rc != MLB_OK) return rc;
  }
  return MLB_OK;
}

int AttentionDecode(const float* q, const float* keys, const float* values,
                    float* out, int64_t position, int64_t max_seq, int n_heads,
                    int n_kv_heads, int hd, float* scratch, void* stream) {
  return AttentionRows(q, keys, values, out, position, 1, max_seq, n_heads, n_kv_heads,
                       hd, scratch, stream);
}

}  // namespace mlb

extern "C" int mlb_set_attention_path(int path) {
  if (path < 0 || path > 2)
    return mlb::Fail(MLB_ERR_ARG, "mlb_set_attention_path: bad path");
  mlb::g_attention_path = path;
  return MLB_OK;
}

extern "C" int mlb_attention_path(void) { return mlb::g_attention_path; }

extern "C" int64_t mlb_attention_scratch_floats(int n_heads, int n_kv_heads,
                                                int head_dim, int64_t position) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || position < 0) return -1;
  return mlb::AttentionScratchFloats(n_heads, n_kv_heads, head_dim, position + 1, 1);
}

extern "C" int mlb_attention_decode_f32(const float* q, const float* keys,
                                        const float* values, float* out,
                                        int64_t position, int64_t max_seq,
                                        int n_heads, int n_kv_heads, int head_dim,
                                        float* scratch, int64_t scratch_floats,
                                        void* stream) {
  using namespace mlb;
  if (scratch == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_attention_decode_f32: null scratch");
  if (n_heads > 0 && n_kv_heads > 0 && head_dim > 0 && position >= 0 &&
      scratch_floats < AttentionScratchFloats(n_heads, n_kv_heads, head_dim, position + 1, 1))
    return Fail(MLB_ERR_ARG, "mlb_attention_decode_f32: scratch too small");
  return AttentionDecode(q, keys, values, out, position, max_seq, n_heads,
                         n_kv_heads, head_dim, scratch, stream);
}

extern "C" int64_t mlb_attention_rows_scratch_floats(int n_heads, int n_kv_heads,
                                                     int head_dim, int64_t position,
                                                     int64_t rows) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || position < 0 || rows < 1)
    return -1;
  return mlb::AttentionScratchFloats(n_heads, n_kv_heads, head_dim, position + 1, rows);
}

extern "C" int mlb_attention_rows_f32(const float* q, const float* keys,
                                      const float* values, float* out, int64_t position,
                                      int64_t rows, int64_t max_seq, int n_heads,
                                      int n_kv_heads, int head_dim, float* scratch,
                                      int64_t scratch_floats, void* stream) {
  using namespace mlb;
  if (rows == 0) return MLB_OK;
  if (rows < 0) return Fail(MLB_ERR_ARG, "mlb_attention_rows_f32: rows < 0");
  if (scratch == nullptr) return Fail(MLB_ERR_ARG, "mlb_attention_rows_f32: null scratch");
  if (n_heads > 0 && n_kv_heads > 0 && head_dim > 0 && position >= 0 &&
      scratch_floats < AttentionScratchFloats(n_heads, n_kv_heads, head_dim, position + 1, rows))
    return Fail(MLB_ERR_ARG, "mlb_attention_rows_f32: scratch too small");
  return AttentionRows(q, keys, values, out, position, rows, max_seq, n_heads, n_kv_heads,
                       head_dim, scratch, stream);
}

extern "C" int mlb_kv_write_f32(float* keys, float* values, const float* k,
                                const float* v, int64_t position, int64_t rows,
                                int64_t max_seq, int n_kv_heads, int head_dim,
                                void* stream) {
  using namespace mlb;
  if (keys == nullptr || values == nullptr || k == nullptr || v == nullptr)
    return Fail(MLB_ERR_ARG, "mlb_kv_write_f32: null pointer");
  if (rows < 0 || n_kv_heads <= 0 || head_dim <= 0 || max_seq <= 0)
    return Fail(MLB_ERR_ARG, "mlb_kv_write_f32: bad shape");
  if (position < 0 || position + rows > max_seq)
    return Fail(MLB_ERR_RANGE, "mlb_kv_write_f32: position out of range");
  if (rows == 0) return MLB_OK;
  const int64_t per = static_cast<int64_t>(n_kv_heads) * head_dim;
  const int64_t count = rows * per;
  const int64_t blocks = (count + 255) / 256;
  Launch(KvWriteKernel, static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16), 256, 0, AsStream(stream), keys, values, k, v, position * per,
                                              count);
  return CheckLaunch("mlb_kv_write_f32");
}

// ---------------------------------------------------------------------------
// Attention without any allocation by the caller or the library.
//
// Some callers cannot hand the library device memory for scratch: a plugin
// inside a host framework that owns every device allocation (its allocator,
// its memory budget), or a token loop that must not call cudaMalloc /
// cudaFree, which can synchronise the whole device.  For them the slice
// partials live in this file-scope device array instead of caller scratch.
// It is part of the library's device code: every GPU on which the library's
// kernels are loaded holds it (4 MiB) until the process exits.
namespace mlb {
namespace {

constexpr int64_t kNoAllocScratchFloats = int64_t{1} << 20;  // 4 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// The array's device address differs per context (each context loads the
// library's device code on its own), so the looked-up addresses are kept per
// (context, device) — a caller that makes its own contexts (cuCtxCreate)
// besides the primary one gets the address of each.  A cudaDeviceReset keeps
// the primary context's handle but loads the code again, possibly elsewhere,
// so an address kept from before a reset is not used again after it: the
// entry point's contract asks callers not to reset a device they use it on.
constexpr int kMaxNoAllocEntries = 64;
struct NoAllocEntry {
  void* context;
  int device;
  float* address;
};
std::mutex g_noalloc_mutex;
NoAllocEntry g_noalloc_entries[kMaxNoAllocEntries] = {};
int g_noalloc_count = 0;

// cuCtxGetCurrent through the runtime's driver entry point (no link against
// the driver library); null when the driver does not offer it.
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn CtxGetCurrent() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// Device address of g_noalloc_scratch in the current context.  In host code
// the array's name only stands in for the symbol, so the address is looked up
// with cudaGetSymbolAddress once per (context, device), with that device
// current, and kept.
int NoAllocScratch(float** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess)
    return Fail(MLB_ERR_CUDA, std::string("attention (no alloc): ") + cudaGetErrorString(err));
  auto current = []() -> void* {  // null before any context is current
    void* context = nullptr;
    if (CtxGetCurrent() == nullptr || CtxGetCurrent()(&context) != 0) return nullptr;
    return context;
  };
  void* context = current();
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  for (int i = 0; context != nullptr && i < g_noalloc_count; ++i) {
    if (g_noalloc_entries[i].context == context && g_noalloc_entries[i].device == device) {
      *out = g_noalloc_entries[i].address;
      return MLB_OK;
    }
  }
  if (g_noalloc_count == kMaxNoAllocEntries)
    return Fail(MLB_ERR_ARG, "attention (no alloc): more than 64 (context, device) pairs");
  void* address = nullptr;
  err = cudaGetSymbolAddress(&address, g_noalloc_scratch);  // makes a context current
  if (err != cudaSuccess || address == nullptr) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, std::string("attention (no alloc): scratch address: ") +
                                  cudaGetErrorString(err));
  }
  context = current();
  bool known = false;
  for (int i = 0; i < g_noalloc_count; ++i)
    known = known || (g_noalloc_entries[i].context == context && g_noalloc_entries[i].device == device);
  if (!known && context != nullptr)
    g_noalloc_entries[g_noalloc_count++] = {context, device, static_cast<float*>(address)};
  *out = static_cast<float*>(address);
  return MLB_OK;
}

}  // namespace
}  // namespace mlb

extern "C" int mlb_attention_decode_noalloc_f32(const float* q, const float* keys,
                                                const float* values, float* out,
                                                int64_t position, int64_t max_seq,
                                                int n_heads, int n_kv_heads,
                                                int head_dim, void* stream) {
  using namespace mlb;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || position < 0)
    return Fail(MLB_ERR_ARG, "mlb_attention_decode_noalloc_f32: bad sizes");
  const int64_t need = AttentionScratchFloats(n_heads, n_kv_heads, head_dim, position + 1, 1);
  if (need > kNoAllocScratchFloats) {
    return Fail(MLB_ERR_ARG,
                "mlb_attention_decode_noalloc_f32: these sizes need " +
                    std::to_string(need) + " floats of scratch, more than the " +
                    std::to_string(kNoAllocScratchFloats) +
                    " (4 MiB) this entry point holds; use mlb_attention_decode_f32 "
                    "with caller-provided scratch");
  }
  float* scratch = nullptr;
  const int rc = NoAllocScratch(&scratch);
  if (rc != MLB_OK) return rc;
  // Every scratch slot the combine kernel reads is written first by the
  // partial kernel of the same call, so nothing needs clearing.
  return AttentionDecode(q, keys, values, out, position, max_seq, n_heads,
                         n_kv_heads, head_dim, scratch, stream);
}
