// Attention-bias add + rotary position embedding, in place, for a batch of
// tokens, Q and K in one launch.
//
// Reference arithmetic (src/forward.cc:113-119 AddBias then src/ops.cc:126-142
// Rope -> ApplyRopeNormal :22-37 / ApplyRopeNeoX :40-56):
//   q += bq; k += bk                      (skipped when the bias is absent)
//   x0' = x0*cos - x1*sin;  x1' = x0*sin + x1*cos
// pairs (2j, 2j+1) in the normal layout, (j, j + hd/2) in NeoX.  cos/sin come
// from a table built on the host with the reference's own expressions
// (rope_table.cc), so device code never evaluates powf/cosf/sinf and the
// result is bit-exact: the multiplies and the add/subtract are separate
// IEEE roundings (__fmul_rn / __fadd_rn / __fsub_rn, no contraction).
//
// Layout: q [rows, nq, hd], k [rows, nk, hd] fp32; positions [rows] int32;
// table [table_rows, hd/2] of (cos, sin) float pairs (8 MB at 16384
// positions x hd 128, which stays resident in the 126 MB L2).
// Work item = one token x one head x one group of 4 rotated floats pairs:
//   normal: a float4 holds pairs 2g, 2g+1 -> table float4 (c,s,c,s)
//   NeoX:   float4s at g*4 and hd/2 + g*4 hold pairs 4g..4g+3 -> two table
//           float4s
// One CTA walks the (head, group) items of a token and grid-strides tokens;
// with too few tokens to fill every SM twice, RopeSplitKernel spreads each
// token's items over several CTAs, one item per thread.
// HBM roofline: 8 bytes per rotated float plus the position (and the bias
// vectors once, L2-resident afterwards).
#include <climits>

#include "common.cuh"

namespace mlb {
namespace {

struct RopeArgs {
  float* q;
  float* k;
  const float* bq;
  const float* bk;
  const int32_t* positions;  // NULL: position_base + t
  int64_t position_base;
  const float* table;
  int64_t table_rows;
  int64_t rows;
  int nq;
  int nk;
  int hd;
  int32_t* status;
};

__device__ __forceinline__ void Rotate(float& x0, float& x1, float c, float s) {
  const float first = x0;
  const float second = x1;
  x0 = __fsub_rn(__fmul_rn(first, c), __fmul_rn(second, s));
  x1 = __fadd_rn(__fmul_rn(first, s), __fmul_rn(second, c));
}

// Vector path: hd % 8 == 0 (NeoX) or hd % 4 == 0 (normal), 16-byte aligned.
// One CTA per token: its threads walk the token's (head, group) items, so
// every CTA streams one contiguous q row and one k row.  (Measured on B200
// at 40 heads x 128: 6.27 TB/s, against 5.83 TB/s for one item per thread
// over a flat grid and 5.73 TB/s for a 2-D token x chunk grid.)
// (Launched for heads wider than 256 float4 groups; few tokens go to
// RopeSplitKernel, narrower heads to RopeRowsKernel.)
template <bool NEOX>
__global__ void __launch_bounds__(256) RopeVecKernel(RopeArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int half = a.hd >> 1;
  const int groups = NEOX ? (a.hd >> 3) : (a.hd >> 2);  // per head
  const int items = (a.nq + a.nk) * groups;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int64_t pos =
        a.positions != nullptr ? __ldg(a.positions + t) : a.position_base + t;
    const bool ok = pos >= 0 && pos < a.table_rows;
    if (!ok && threadIdx.x == 0 && a.status != nullptr)
      atomicOr(a.status, MLB_STATUS_BAD_POSITION);
    const float4* trow = reinterpret_cast<const float4*>(
        a.table + static_cast<size_t>(ok ? pos : 0) * a.hd);
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
      const int head = it / groups;
      const int g = it - head * groups;
      const bool is_q = head < a.nq;
      const int h = is_q ? head : head - a.nq;
      float* base = is_q ? a.q + (static_cast<size_t>(t) * a.nq + h) * a.hd
                         : a.k + (static_cast<size_t>(t) * a.nk + h) * a.hd;
      const float* bias = is_q ? a.bq : a.bk;
      float4* lo = reinterpret_cast<float4*>(base + 4 * g);
      float4 x0 = LoadStream(lo);
      if (NEOX) {
        float4* hi = reinterpret_cast<float4*>(base + half + 4 * g);
        float4 x1 = LoadStream(hi);
        if (bias != nullptr) {
          const float* bh = bias + static_cast<size_t>(h) * a.hd;
          x0 = AddRn(x0, __ldg(reinterpret_cast<const float4*>(bh + 4 * g)));
          x1 = AddRn(x1, __ldg(reinterpret_cast<const float4*>(bh + half + 4 * g)));
        }
        if (ok) {
          const float4 cs0 = __ldg(trow + 2 * g);      // pairs 4g, 4g+1
          const float4 cs1 = __ldg(trow + 2 * g + 1);  // pairs 4g+2, 4g+3
          Rotate(x0.x, x1.x, cs0.x, cs0.y);
          Rotate(x0.y, x1.y, cs0.z, cs0.w);
          Rotate(x0.z, x1.z, cs1.x, cs1.y);
          Rotate(x0.w, x1.w, cs1.z, cs1.w);
        }
        StoreStream(lo, x0);
        StoreStream(hi, x1);
      } else {
        if (bias != nullptr) {
          const float* bh = bias + static_cast<size_t>(h) * a.hd;
          x0 = AddRn(x0, __ldg(reinterpret_cast<const float4*>(bh + 4 * g)));
        }
        if (ok) {
          const float4 cs = __ldg(trow + g);  // pairs 2g, 2g+1
          Rotate(x0.x, x0.y, cs.x, cs.y);
          Rotate(x0.z, x0.w, cs.z, cs.w);
        }
        StoreStream(lo, x0);
      }
    }
  }
}

// Few tokens (a decode batch): token t's (head, group) items are spread
// over gridDim.y CTAs, one item per thread (the launch makes gridDim.y *
// blockDim.x cover the items; a longer item range is walked in steps).  The
// item's q / k (and bias) loads are issued before the position load, so a
// thread waits for two DRAM round trips, position then (cos, sin), with its
// data in flight alongside, and never for a load that follows a store.  The
// bad-position status is set after the item is written, so that no branch
// on the position stands between the loads and their uses.
template <bool NEOX>
__global__ void __launch_bounds__(256) RopeSplitKernel(RopeArgs a) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int half = a.hd >> 1;
  const int groups = NEOX ? (a.hd >> 3) : (a.hd >> 2);  // per head
  const int items = (a.nq + a.nk) * groups;
  const int first = blockIdx.y * blockDim.x + threadIdx.x;
  const int step = gridDim.y * blockDim.x;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    for (int it = first; it < items; it += step) {
      const int head = it / groups;
      const int g = it - head * groups;
      const bool is_q = head < a.nq;
      const int h = is_q ? head : head - a.nq;
      float* base = is_q ? a.q + (static_cast<size_t>(t) * a.nq + h) * a.hd
                         : a.k + (static_cast<size_t>(t) * a.nk + h) * a.hd;
      float4* lo = reinterpret_cast<float4*>(base + 4 * g);
      float4* hi = reinterpret_cast<float4*>(base + half + 4 * g);
      float4 x0 = LoadStream(lo);
      float4 x1 = NEOX ? LoadStream(hi) : x0;
      const float* bias = is_q ? a.bq : a.bk;
      if (bias != nullptr) {
        const float* bh = bias + static_cast<size_t>(h) * a.hd;
        x0 = AddRn(x0, __ldg(reinterpret_cast<const float4*>(bh + 4 * g)));
        if (NEOX)
          x1 = AddRn(x1, __ldg(reinterpret_cast<const float4*>(bh + half + 4 * g)));
      }
      const int64_t pos =
          a.positions != nullptr ? __ldg(a.positions + t) : a.position_base + t;
      const bool ok = pos >= 0 && pos < a.table_rows;
      if (ok) {
        const float4* trow =
            reinterpret_cast<const float4*>(a.table + static_cast<size_t>(pos) * a.hd);
        if (NEOX) {
          const float4 cs0 = __ldg(trow + 2 * g);      // pairs 4g, 4g+1
          const float4 cs1 = __ldg(trow + 2 * g + 1);  // pairs 4g+2, 4g+3
          Rotate(x0.x, x1.x, cs0.x, cs0.y);
          Rotate(x0.y, x1.y, cs0.z, cs0.w);
          Rotate(x0.z, x1.z, cs1.x, cs1.y);
          Rotate(x0.w, x1.w, cs1.z, cs1.w);
        } else {
          const float4 cs = __ldg(trow + g);  // pairs 2g, 2g+1
          Rotate(x0.x, x0.y, cs.x, cs.y);
          Rotate(x0.z, x0.w, cs.z, cs.w);
        }
      }
      StoreStream(lo, x0);
      if (NEOX) StoreStream(hi, x1);
      if (!ok && it == 0 && a.status != nullptr)
        atomicOr(a.status, MLB_STATUS_BAD_POSITION);
    }
  }
}

// Large batches (the unsplit vector path): one CTA per token, thread
// (h0, g) = (tid / G, tid % G) with G = float4 groups per head (hd / 4
// normal, hd / 8 NeoX), so a thread's (cos, sin) float4s are the same for
// every head it takes and are loaded once per token; it takes heads h0,
// h0 + hpp, ... (hpp = heads per pass = blockDim / G), MAXI of them at a
// time, issuing every load of the MAXI heads before the first rotation and
// store.  No index division in the loop.  Launched with MAXI = 1: measured
// on B200 at 40 heads x 128, 16384 tokens with a positions array, inside
// the layer-op step (after the residual RMSNorm), MAXI = 1 / 3 took 0.117 /
// 0.123 ms against 0.118 for the item loop above — more loads in flight
// compete with the write-back of the previous kernel's dirty L2 lines — and
// 0.108 / 0.107 / 0.109 ms alone (256-thread CTAs; see the launch for the
// CTA size).
template <bool NEOX, int MAXI>
__global__ void __launch_bounds__(256) RopeRowsKernel(RopeArgs a, int G) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int half = a.hd >> 1;
  const int g = threadIdx.x % G;
  const int h0 = threadIdx.x / G;
  const int hpp = blockDim.x / G;
  const int heads = a.nq + a.nk;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int64_t pos =
        a.positions != nullptr ? __ldg(a.positions + t) : a.position_base + t;
    const bool ok = pos >= 0 && pos < a.table_rows;
    if (!ok && threadIdx.x == 0 && a.status != nullptr)
      atomicOr(a.status, MLB_STATUS_BAD_POSITION);
    const float4* trow = reinterpret_cast<const float4*>(
        a.table + static_cast<size_t>(ok ? pos : 0) * a.hd);
    float4 cs0 = make_float4(1.f, 0.f, 1.f, 0.f), cs1 = cs0;
    if (ok) {
      cs0 = __ldg(trow + (NEOX ? 2 * g : g));
      if (NEOX) cs1 = __ldg(trow + 2 * g + 1);
    }
    float* qrow = a.q + static_cast<size_t>(t) * a.nq * a.hd;
    float* krow = a.k + static_cast<size_t>(t) * a.nk * a.hd;
    for (int hb = h0; hb < heads; hb += MAXI * hpp) {
      float4 x0[MAXI], x1[MAXI];
#pragma unroll
      for (int i = 0; i < MAXI; ++i) {
        const int head = hb + i * hpp;
        if (head < heads) {
          const float* base = head < a.nq ? qrow + head * a.hd : krow + (head - a.nq) * a.hd;
          x0[i] = LoadStream(reinterpret_cast<const float4*>(base + 4 * g));
          if (NEOX) x1[i] = LoadStream(reinterpret_cast<const float4*>(base + half + 4 * g));
        }
      }
#pragma unroll
      for (int i = 0; i < MAXI; ++i) {
        const int head = hb + i * hpp;
        if (head >= heads) continue;
        const bool is_q = head < a.nq;
        const int h = is_q ? head : head - a.nq;
        float* base = is_q ? qrow + head * a.hd : krow + h * a.hd;
        const float* bias = is_q ? a.bq : a.bk;
        if (bias != nullptr) {
          const float* bh = bias + static_cast<size_t>(h) * a.hd;
          x0[i] = AddRn(x0[i], __ldg(reinterpret_cast<const float4*>(bh + 4 * g)));
          if (NEOX)
            x1[i] = AddRn(x1[i], __ldg(reinterpret_cast<const float4*>(bh + half + 4 * g)));
        }
        if (ok) {
          if (NEOX) {
            Rotate(x0[i].x, x1[i].x, cs0.x, cs0.y);
            Rotate(x0[i].y, x1[i].y, cs0.z, cs0.w);
            Rotate(x0[i].z, x1[i].z, cs1.x, cs1.y);
            Rotate(x0[i].w, x1[i].w, cs1.z, cs1.w);
          } else {
            Rotate(x0[i].x, x0[i].y, cs0.x, cs0.y);
            Rotate(x0[i].z, x0[i].w, cs0.z, cs0.w);
          }
        }
        StoreStream(reinterpret_cast<float4*>(base + 4 * g), x0[i]);
        if (NEOX) StoreStream(reinterpret_cast<float4*>(base + half + 4 * g), x1[i]);
      }
    }
  }
}

// Any even hd / alignment: one item per rotated pair.
__global__ void __launch_bounds__(256) RopeScalarKernel(RopeArgs a, int neox) {
  LaunchWait();  // the previous kernel on the stream has completed
  LaunchNext();
  const int half = a.hd >> 1;
  const int heads = a.nq + a.nk;
  const int items = heads * half;
  for (int64_t t = blockIdx.x; t < a.rows; t += gridDim.x) {
    const int64_t pos =
        a.positions != nullptr ? a.positions[t] : a.position_base + t;
    const bool ok = pos >= 0 && pos < a.table_rows;
    if (!ok && threadIdx.x == 0 && a.status != nullptr)
      atomicOr(a.status, MLB_STATUS_BAD_POSITION);
    const float* trow = a.table + static_cast<size_t>(ok ? pos : 0) * a.hd;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
      const int head = it / half;
      const int j = it - head * half;
      const bool is_q = head < a.nq;
      const int h = is_q ? head : head - a.nq;
      float* base = is_q ? a.q + (static_cast<size_t>(t) * a.nq + h) * a.hd
                         : a.k + (static_cast<size_t>(t) * a.nk + h) * a.hd;
      const float* bias = is_q ? a.bq : a.bk;
      const int i0 = neox ? j : 2 * j;
      const int i1 = neox ? j + half : 2 * j + 1;
      float x0 = base[i0];
      float x1 = base[i1];
      if (bias != nullptr) {
        const float* bh = bias + static_cast<size_t>(h) * a.hd;
        x0 = __fadd_rn(x0, bh[i0]);
        x1 = __fadd_rn(x1, bh[i1]);
      }
      if (ok) Rotate(x0, x1, trow[2 * j], trow[2 * j + 1]);
      base[i0] = x0;
      base[i1] = x1;
    }
  }
}

}  // namespace
}  // namespace mlb

extern "C" int mlb_rope_f32(float* q, float* k, const float* bq,
                            const float* bk, const int32_t* positions,
                            int64_t position_base, const float* cos_sin,
                            int64_t table_rows, int64_t rows, int nq, int nk,
                            int hd, int neox, int32_t* status, void* stream) {
  using namespace mlb;
  if (rows < 0 || nq < 0 || nk < 0 || hd <= 0 || (hd % 2) != 0 ||
      table_rows < 0)
    return Fail(MLB_ERR_ARG, "mlb_rope_f32: bad shape (hd must be even)");
  if (static_cast<int64_t>(nq + static_cast<int64_t>(nk)) * hd > INT_MAX)
    return Fail(MLB_ERR_ARG, "mlb_rope_f32: too many heads");
  if (rows == 0 || nq + nk == 0) return MLB_OK;
  if (cos_sin == nullptr || (nq > 0 && q == nullptr) || (nk > 0 && k == nullptr))
    return Fail(MLB_ERR_ARG, "mlb_rope_f32: null pointer");
  if (positions == nullptr &&
      (position_base < 0 || position_base > table_rows - rows))
    return Fail(MLB_ERR_RANGE, "mlb_rope_f32: positions outside the table");
  RopeArgs a{q, k, bq, bk, positions, position_base, cos_sin, table_rows, rows,
             nq, nk, hd, status};
  const bool aligned = (nq == 0 || Aligned16(q)) && (nk == 0 || Aligned16(k)) &&
                       (bq == nullptr || Aligned16(bq)) &&
                       (bk == nullptr || Aligned16(bk)) && Aligned16(cos_sin);
  const bool vec = aligned && (neox ? (hd % 8) == 0 : (hd % 4) == 0);
  const int64_t cap = 1 << 24;
  const dim3 grid(static_cast<unsigned>(rows < cap ? rows : cap));
  const int items = (nq + nk) * (neox ? hd / 8 : hd / 4);
  int threads = items < 256 ? (items + 31) / 32 * 32 : 256;
  if (threads < 32) threads = 32;
  cudaStream_t s = AsStream(stream);
  if (vec) {
    // split tokens over several CTAs when they cannot fill every SM twice
    const int64_t fill = 2 * static_cast<int64_t>(SmCount());
    // (one item per thread: as many CTAs per token as its items need)
    int64_t split = rows < fill ? (items + threads - 1) / threads : 1;
    if (split > 65535) split = 65535;
    const dim3 grid2(grid.x, static_cast<unsigned>(split));
    const int G = neox ? hd / 8 : hd / 4;  // float4 groups per head
    if (split > 1) {
      if (neox) Launch(RopeSplitKernel<true>, grid2, threads, 0, s, a);
      else Launch(RopeSplitKernel<false>, grid2, threads, 0, s, a);
    } else if (G <= 256) {
      // heads per pass: as many as fit 128 threads (at least one), no more
      // than there are.  Measured on B200 in the layer-op step: 128-thread
      // CTAs beat 256 (40 heads x 128 normal, 16384 tokens: 0.114 against
      // 0.116 ms; 28 + 4 heads x 128 NeoX with bias, 65536 tokens: 0.339
      // against 0.405 ms; the item loop above 0.117 / 0.360 ms at 256)
      int hpp = G <= 128 ? 128 / G : 1;
      if (hpp > nq + nk) hpp = nq + nk;
      const int rthreads = hpp * G;
      if (neox) Launch(RopeRowsKernel<true, 1>, grid, rthreads, 0, s, a, G);
      else Launch(RopeRowsKernel<false, 1>, grid, rthreads, 0, s, a, G);
    } else {
      if (neox) Launch(RopeVecKernel<true>, grid, threads, 0, s, a);
      else Launch(RopeVecKernel<false>, grid, threads, 0, s, a);
    }
  } else {
    Launch(RopeScalarKernel, grid, 256, 0, s, a, neox);
  }
  return CheckLaunch("mlb_rope_f32");
}
