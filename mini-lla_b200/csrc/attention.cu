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
constexpr int kMinSlice = 64;     // positions per slice at least

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

template <int G>
int LaunchPartial(const AttnArgs& a, int64_t rows, int nv, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(a.n_kv_heads), static_cast<unsigned>(a.splits),
                  static_cast<unsigned>(rows));
  if (nv == 1) {
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
  cudaStream_t s = AsStream(stream);
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
