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
constexpr int kMinSlice = 128;    // positions per slice at least (4 warps x 32)

struct AttnArgs {
  const float* q;
  const float* keys;
  const float* values;
  float* out;
  float* scratch;  // [rows][n_heads][splits][hd + 2]
  int64_t visible; // visible positions of query row 0 (row r sees visible + r)
  int n_heads;
  int n_kv_heads;
  int hd;
  int splits;
  int64_t slice;   // positions per slice
  float scale;
};

// Number of position slices for a launch of `rows` query rows: enough CTAs
// to cover every SM twice, at least kMinSlice positions per slice (of the
// longest row).
int Splits(int n_kv_heads, int64_t visible, int64_t rows = 1) {
  const int64_t ctas = static_cast<int64_t>(n_kv_heads) * rows;
  const int64_t want = (2 * static_cast<int64_t>(SmCount()) + ctas - 1) / ctas;
  const int64_t most = (visible + kMinSlice - 1) / kMinSlice;
  int64_t s = want < most ? want : most;
  if (s < 1) s = 1;
  return static_cast<int>(s);
}

template <int G, int NV>
__global__ void __launch_bounds__(kAttnWarps * 32) AttnPartialKernel(AttnArgs a) {
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
  float* scratch_row = a.scratch + row * a.n_heads * a.splits * (a.hd + 2);
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
    float* part = scratch_row + (static_cast<int64_t>(head) * a.splits + s) * (a.hd + 2);
    if (lane == 0) {
      part[0] = mm;
      part[1] = ll;
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int i = lane + 32 * v;
      if (i < hd4) {
        part[2 + 4 * i + 0] = aa[v].x;
        part[2 + 4 * i + 1] = aa[v].y;
        part[2 + 4 * i + 2] = aa[v].z;
        part[2 + 4 * i + 3] = aa[v].w;
      }
    }
  }
}

// out[h][i] = sum_s acc_s[i] * e^(m_s - M) / sum_s l_s * e^(m_s - M).
__global__ void __launch_bounds__(256) AttnCombineKernel(AttnArgs a) {
  const int head = blockIdx.x;
  const int64_t row = blockIdx.y;
  const float* base = a.scratch + (row * a.n_heads + head) * a.splits * (a.hd + 2);
  float mm = -INFINITY;
  for (int s = 0; s < a.splits; ++s) mm = fmaxf(mm, base[s * (a.hd + 2)]);
  float ll = 0.0f;
  for (int s = 0; s < a.splits; ++s) {
    const float ms = base[s * (a.hd + 2)];
    if (ms != -INFINITY) ll = fmaf(base[s * (a.hd + 2) + 1], expf(ms - mm), ll);
  }
  for (int i = threadIdx.x; i < a.hd; i += blockDim.x) {
    float sum = 0.0f;
    for (int s = 0; s < a.splits; ++s) {
      const float ms = base[s * (a.hd + 2)];
      if (ms != -INFINITY) sum = fmaf(base[s * (a.hd + 2) + 2 + i], expf(ms - mm), sum);
    }
    a.out[(row * a.n_heads + head) * a.hd + i] = __fdiv_rn(sum, ll);
  }
}

// Lane-per-position form of the slice kernel (head_dim 64 or 128): each
// warp takes its slice's positions 32 at a time, stages those 32 K rows in
// shared memory (cp.async, rows padded by 16 bytes so that a lane reading
// its own row stays on distinct banks), and lane l scores position
// block + l against all G query heads with plain FMAs — no cross-lane
// reduction per dot product.  One warp max / sum per block and head feeds
// the online softmax; P.V then walks the block's positions with the
// probabilities broadcast by shuffles and each lane accumulating DPL = hd / 32
// dimensions of a coalesced V row.  The 4 warps' states are merged and
// written as the slice partial, as in AttnPartialKernel.
constexpr int kLaneBlock = 32;

template <int HD4>
__host__ __device__ constexpr int LaneRowFloats() { return 4 * HD4 + 4; }

template <int G, int HD4>
__global__ void __launch_bounds__(kAttnWarps * 32) AttnLanePartialKernel(AttnArgs a) {
  constexpr int HD = 4 * HD4;
  constexpr int DPL = HD / 32;        // dimensions per lane in P.V (2 or 4)
  constexpr int RF = LaneRowFloats<HD4>();
  // dynamic: q of the G heads, then per warp a staged block of K rows (the
  // warps' final accumulators reuse the K area once the loop is done)
  extern __shared__ __align__(16) float lsm[];
  float* qs = lsm;                   // [G][HD]
  float* ks_all = lsm + G * HD;      // [kAttnWarps][kLaneBlock][RF]
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
  float* scratch_row = a.scratch + row * a.n_heads * a.splits * (HD + 2);
  const int64_t kv_stride = static_cast<int64_t>(a.n_kv_heads) * HD;
  const float* kbase = a.keys + static_cast<int64_t>(g) * HD;
  const float* vbase = a.values + static_cast<int64_t>(g) * HD;

  for (int i = threadIdx.x; i < G * HD4; i += blockDim.x)
    reinterpret_cast<float4*>(qs)[i] =
        __ldg(reinterpret_cast<const float4*>(q_row + static_cast<int64_t>(g) * G * HD) + i);
  __syncthreads();

  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[h][e] = 0.0f;
  }
  float* kw = ks_all + warp * kLaneBlock * RF;
  for (int64_t blk = t_begin + static_cast<int64_t>(warp) * kLaneBlock; blk < t_end;
       blk += kAttnWarps * kLaneBlock) {
    const int n = static_cast<int>(t_end - blk < kLaneBlock ? t_end - blk : kLaneBlock);
    // stage K rows blk .. blk + n - 1 (coalesced: lane l copies float4 l, l + 32, ...)
    for (int i = lane; i < n * HD4; i += 32) {
      const int r = i / HD4, c = i - r * HD4;
      CopyAsync16(kw + r * RF + 4 * c, kbase + (blk + r) * kv_stride + 4 * c);
    }
    CopyAsyncCommit();
    CopyAsyncWait<0>();
    __syncwarp();
    // scores of position blk + lane for the G heads
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.0f;
    if (lane < n) {
      const float* kr = kw + lane * RF;
#pragma unroll 8
      for (int c = 0; c < HD4; ++c) {
        const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * c);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float4 qv = *reinterpret_cast<const float4*>(qs + h * HD + 4 * c);
          sc[h] = fmaf(qv.x, kv.x, sc[h]);
          sc[h] = fmaf(qv.y, kv.y, sc[h]);
          sc[h] = fmaf(qv.z, kv.z, sc[h]);
          sc[h] = fmaf(qv.w, kv.w, sc[h]);
        }
      }
    }
    float p[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float score = lane < n ? __fmul_rn(sc[h], a.scale) : -INFINITY;
      const float m_new = fmaxf(m[h], WarpMax(score));
      const float alpha = expf(m[h] - m_new);  // 0 on the first block
      p[h] = lane < n ? expf(score - m_new) : 0.0f;
      l[h] = fmaf(l[h], alpha, WarpSum(p[h]));
      m[h] = m_new;
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[h][e] *= alpha;
    }
    // P.V over the block's positions (V row r: lane owns dims DPL * lane ..)
    for (int r = 0; r < n; ++r) {
      const float* vr = vbase + (blk + r) * kv_stride + DPL * lane;
      float v[DPL];
      if (DPL == 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(vr));
        v[0] = x.x; v[1] = x.y; v[2 % DPL] = x.z; v[3 % DPL] = x.w;
      } else {
        const float2 x = __ldg(reinterpret_cast<const float2*>(vr));
        v[0] = x.x; v[1] = x.y;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pr = __shfl_sync(0xffffffffu, p[h], r);
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[h][e] = fmaf(pr, v[e], acc[h][e]);
      }
    }
    __syncwarp();  // every lane is done with kw before it is restaged
  }
  // merge the 4 warps, then write the slice partial
  __syncthreads();  // every warp is done with its K rows: reuse them
  float* sm_acc = ks_all;  // [kAttnWarps][G][HD]
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
    float* part = scratch_row + (static_cast<int64_t>(g * G + h) * a.splits + s) * (HD + 2);
    if (lane == 0) {
      part[0] = mm;
      part[1] = ll;
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) part[2 + DPL * lane + e] = aa[e];
  }
}

template <int G, int HD4>
int LaunchLane(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  constexpr size_t kStage = static_cast<size_t>(kAttnWarps) * kLaneBlock * LaneRowFloats<HD4>();
  constexpr size_t kAcc = static_cast<size_t>(kAttnWarps) * G * 4 * HD4;
  constexpr size_t shm = sizeof(float) * (G * 4 * HD4 + (kStage > kAcc ? kStage : kAcc));
  auto kernel = AttnLanePartialKernel<G, HD4>;
  if (shm > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(shm)) != cudaSuccess) {
    cudaGetLastError();
    return Fail(MLB_ERR_CUDA, "attention: shared memory opt-in");
  }
  kernel<<<grid, kAttnWarps * 32, shm, s>>>(a);
  return CheckLaunch("mlb_attention_decode_f32");
}

template <int G>
int LaunchPartial(const AttnArgs& a, int64_t rows, int nv, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.n_kv_heads), static_cast<unsigned>(a.splits),
                  static_cast<unsigned>(rows));
  if (a.hd == 128) {
    return LaunchLane<G, 32>(a, grid, s);
  } else if (a.hd == 64) {
    return LaunchLane<G, 16>(a, grid, s);
  } else if (nv == 1) {
    AttnPartialKernel<G, 1><<<grid, kAttnWarps * 32, 0, s>>>(a);
  } else {
    AttnPartialKernel<G, 2><<<grid, kAttnWarps * 32, 0, s>>>(a);
  }
  return CheckLaunch("mlb_attention_decode_f32");
}

__global__ void __launch_bounds__(256)
    KvWriteKernel(float* keys, float* values, const float* k, const float* v,
                  int64_t base, int64_t count) {
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
// CTA (kv head g, tile of QR = 64 / G consecutive query rows) holds the
// QV = QR * G query vectors of its rows and group in shared memory and walks
// the visible positions in blocks of 32 keys: every K/V block is staged once
// (cp.async, double-buffered) for all QV query vectors instead of once per
// query row.  256 threads; thread (pair p = tid / 8, j = tid % 8) scores
// query vectors 2p, 2p + 1 against keys j, j + 8, j + 16, j + 24 of a block
// (rows padded by 16 bytes so those reads hit distinct banks), keeps the
// online softmax of its two vectors (max / sum reduced over the 8 threads of
// the pair) and accumulates P.V for float4 columns j, j + 8, ... of them.
// Masked (future) keys score -inf; no slice partials, no combine kernel.
constexpr int kTileKeys = 32;
constexpr int kTileQv = 64;
constexpr int kTileThreads = 256;

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
                          static_cast<size_t>(kTileQv) * (kTileKeys + 1));
}

template <int G, int HD4>
__global__ void __launch_bounds__(kTileThreads) AttnRowTileKernel(AttnTileArgs a) {
  constexpr int QR = kTileQv / G;  // query rows per CTA
  constexpr int QV = QR * G;
  constexpr int RF = TileRowFloats<HD4>();
  constexpr int HD = 4 * HD4;
  constexpr int CPT = HD4 / 8;     // float4 columns per thread in P.V
  extern __shared__ __align__(16) float tsm[];
  float* qs = tsm;                           // [QV][RF]
  float* ks = qs + kTileQv * RF;             // [2][kTileKeys][RF]
  float* vs = ks + 2 * kTileKeys * RF;       // [2][kTileKeys][RF]
  float* ps = vs + 2 * kTileKeys * RF;       // [QV][kTileKeys + 1]

  const int g = blockIdx.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * QR;
  const int tid = threadIdx.x;
  const int pair = tid >> 3;
  const int j = tid & 7;
  const int v0 = 2 * pair, v1 = 2 * pair + 1;
  const bool active = v1 < QV;  // (QV is even: both or neither)
  const int64_t row_stride = static_cast<int64_t>(a.n_heads) * HD;
  const int64_t kv_stride = static_cast<int64_t>(a.n_kv_heads) * HD;

  // the tile's query vectors (rows beyond the chunk read as zeros)
  for (int i = tid; i < QV * HD4; i += kTileThreads) {
    const int v = i / HD4, d4 = i - v * HD4;
    const int64_t row = r0 + v / G;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < a.rows)
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

  const int64_t qpos0 = a.position + r0 + v0 / G;  // positions of the two vectors
  const int64_t qpos1 = a.position + r0 + v1 / G;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  float4 acc0[CPT], acc1[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    acc0[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    acc1[c] = make_float4(0.f, 0.f, 0.f, 0.f);
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
    if (active) {
      float s0[4], s1[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) s0[i] = s1[i] = 0.0f;
#pragma unroll 4
      for (int d4 = 0; d4 < HD4; ++d4) {
        const float4 qa = *reinterpret_cast<const float4*>(qs + v0 * RF + 4 * d4);
        const float4 qb = *reinterpret_cast<const float4*>(qs + v1 * RF + 4 * d4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 kk = *reinterpret_cast<const float4*>(kb + (j + 8 * i) * RF + 4 * d4);
          s0[i] = fmaf(qa.x, kk.x, s0[i]);
          s0[i] = fmaf(qa.y, kk.y, s0[i]);
          s0[i] = fmaf(qa.z, kk.z, s0[i]);
          s0[i] = fmaf(qa.w, kk.w, s0[i]);
          s1[i] = fmaf(qb.x, kk.x, s1[i]);
          s1[i] = fmaf(qb.y, kk.y, s1[i]);
          s1[i] = fmaf(qb.z, kk.z, s1[i]);
          s1[i] = fmaf(qb.w, kk.w, s1[i]);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t t = static_cast<int64_t>(b) * kTileKeys + j + 8 * i;
        s0[i] = t <= qpos0 ? __fmul_rn(s0[i], a.scale) : -INFINITY;
        s1[i] = t <= qpos1 ? __fmul_rn(s1[i], a.scale) : -INFINITY;
        mx0 = fmaxf(mx0, s0[i]);
        mx1 = fmaxf(mx1, s1[i]);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      // a vector with no visible key yet keeps p = 0 (no -inf - -inf)
      const float al0 = n0 == -INFINITY ? 1.0f : expf(m0 - n0);
      const float al1 = n1 == -INFINITY ? 1.0f : expf(m1 - n1);
      float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p0 = s0[i] == -INFINITY ? 0.0f : expf(s0[i] - n0);
        const float p1 = s1[i] == -INFINITY ? 0.0f : expf(s1[i] - n1);
        ps[v0 * (kTileKeys + 1) + j + 8 * i] = p0;
        ps[v1 * (kTileKeys + 1) + j + 8 * i] = p1;
        sum0 += p0;
        sum1 += p1;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, o);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, o);
      }
      l0 = fmaf(l0, al0, sum0);
      l1 = fmaf(l1, al1, sum1);
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        acc0[c].x *= al0; acc0[c].y *= al0; acc0[c].z *= al0; acc0[c].w *= al0;
        acc1[c].x *= al1; acc1[c].y *= al1; acc1[c].z *= al1; acc1[c].w *= al1;
      }
      __syncwarp();  // the pair's p values are in place (the 8 threads share a warp)
#pragma unroll 4
      for (int key = 0; key < kTileKeys; ++key) {
        const float p0 = ps[v0 * (kTileKeys + 1) + key];
        const float p1 = ps[v1 * (kTileKeys + 1) + key];
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          const float4 vv = *reinterpret_cast<const float4*>(vb + key * RF + 4 * (j + 8 * c));
          acc0[c].x = fmaf(p0, vv.x, acc0[c].x);
          acc0[c].y = fmaf(p0, vv.y, acc0[c].y);
          acc0[c].z = fmaf(p0, vv.z, acc0[c].z);
          acc0[c].w = fmaf(p0, vv.w, acc0[c].w);
          acc1[c].x = fmaf(p1, vv.x, acc1[c].x);
          acc1[c].y = fmaf(p1, vv.y, acc1[c].y);
          acc1[c].z = fmaf(p1, vv.z, acc1[c].z);
          acc1[c].w = fmaf(p1, vv.w, acc1[c].w);
        }
      }
    }
    __syncthreads();  // buffers of block b are free for block b + 2
  }
  CopyAsyncWait<0>();
  if (!active) return;
  const int64_t row0 = r0 + v0 / G, row1 = r0 + v1 / G;
  float* o0 = a.out + row0 * row_stride + static_cast<int64_t>(g * G + v0 % G) * HD;
  float* o1 = a.out + row1 * row_stride + static_cast<int64_t>(g * G + v1 % G) * HD;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int col = 4 * (j + 8 * c);
    if (row0 < a.rows)
      *reinterpret_cast<float4*>(o0 + col) =
          make_float4(__fdiv_rn(acc0[c].x, l0), __fdiv_rn(acc0[c].y, l0),
                      __fdiv_rn(acc0[c].z, l0), __fdiv_rn(acc0[c].w, l0));
    if (row1 < a.rows)
      *reinterpret_cast<float4*>(o1 + col) =
          make_float4(__fdiv_rn(acc1[c].x, l1), __fdiv_rn(acc1[c].y, l1),
                      __fdiv_rn(acc1[c].z, l1), __fdiv_rn(acc1[c].w, l1));
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
  kernel<<<grid, kTileThreads, shm, s>>>(a);
  return CheckLaunch("attention (row tiles)");
}

// Row tiles when they fill the GPU (n_kv_heads x row tiles >= half the SMs),
// group 1 / 2 / 4 / 8, head_dim 64 or 128; -1 when the shape does not fit.
int AttentionRowTiles(const float* q, const float* keys, const float* values, float* out,
                      int64_t position, int64_t rows, int64_t max_seq, int n_heads,
                      int n_kv_heads, int hd, cudaStream_t s) {
  const int group = n_heads / n_kv_heads;
  if ((group != 1 && group != 2 && group != 4 && group != 8) || (hd != 64 && hd != 128) ||
      !Aligned16(out) || rows > 65535LL * (kTileQv / group))
    return -1;
  if (static_cast<int64_t>(n_kv_heads) * ((rows + kTileQv / group - 1) / (kTileQv / group)) <
      SmCount() / 2)
    return -1;
  AttnTileArgs a{q, keys, values, out, position, rows, max_seq, n_heads, n_kv_heads,
                 1.0f / std::sqrt(static_cast<float>(hd))};
  if (hd == 64) {
    switch (group) {
      case 1: return LaunchRowTile<1, 16>(a, s);
      case 2: return LaunchRowTile<2, 16>(a, s);
      case 4: return LaunchRowTile<4, 16>(a, s);
      default: return LaunchRowTile<8, 16>(a, s);
    }
  }
  switch (group) {
    case 1: return LaunchRowTile<1, 32>(a, s);
    case 2: return LaunchRowTile<2, 32>(a, s);
    case 4: return LaunchRowTile<4, 32>(a, s);
    default: return LaunchRowTile<8, 32>(a, s);
  }
}

// Shared by the entry points: scratch must hold AttentionScratchFloats() for
// `rows` query rows, row r seeing visible + r positions.
int64_t AttentionScratchFloats(int n_heads, int n_kv_heads, int hd, int64_t visible,
                               int64_t rows) {
  return rows * n_heads * Splits(n_kv_heads, visible + rows - 1, rows) * (hd + 2);
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
    AttnCombineKernel<<<dim3(n_heads, static_cast<unsigned>(rc_rows)),
                        hd < 256 ? ((hd + 31) / 32) * 32 : 256, 0, s>>>(a);
    rc = CheckLaunch("attention");
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
  KvWriteKernel<<<static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16),
                  256, 0, AsStream(stream)>>>(keys, values, k, v, position * per,
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

constexpr int kMaxNoAllocDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_address[kMaxNoAllocDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name only stands in for the symbol, so the address is looked up
// once per device (with that device current) and cached.
int NoAllocScratch(float** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess)
    return Fail(MLB_ERR_CUDA, std::string("attention (no alloc): ") + cudaGetErrorString(err));
  if (device < 0 || device >= kMaxNoAllocDevices)
    return Fail(MLB_ERR_ARG, "attention (no alloc): device index beyond 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[device] == nullptr) {
    void* address = nullptr;
    err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (err != cudaSuccess || address == nullptr) {
      cudaGetLastError();
      return Fail(MLB_ERR_CUDA, std::string("attention (no alloc): scratch address: ") +
                                    cudaGetErrorString(err));
    }
    g_noalloc_address[device] = static_cast<float*>(address);
  }
  *out = g_noalloc_address[device];
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
