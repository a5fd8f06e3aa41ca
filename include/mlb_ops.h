/*
 * mlb_ops.h — C ABI of the B200 (sm_100a) layer-operator library libmlb.so.
 *
 * These entry points are what mini-lla's GPU operator layer binds to in place
 * of its per-vector kernels (reference src/cuda_ops.cu and the declarations
 * in include/mini_llama/cuda_ops.h:11-34).  The C++17 wrappers that keep the
 * reference's CudaRmsNorm / CudaRope / ... signatures call them with rows = 1;
 * row-batched callers (prefill) call them with rows = T.
 *
 * Conventions (all entries):
 *   - Every pointer argument is a DEVICE pointer unless the name ends in
 *     _host; the caller owns every buffer.  Nothing here allocates device
 *     memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Calls are asynchronous on that stream and run on the device
 *     that is current on the calling thread; the stream must belong to it.
 *   - Return value: MLB_OK, or MLB_ERR_ARG for a rejected argument (nothing is
 *     launched), MLB_ERR_RANGE for a host-checked id or position outside its
 *     table (nothing is launched), or MLB_ERR_CUDA when the launch failed.  The message of the
 *     last failure on the calling thread is mlb_last_error().
 *   - Conditions only the device can see (a token id outside the table, a
 *     position outside the RoPE table, a softmax row length outside [1, cols])
 *     are reported through an optional device status word: the kernel ORs the
 *     MLB_STATUS_* bits into *status (the caller zeroes it and reads it after
 *     the stream synchronises).  The affected rows are skipped (RoPE) or
 *     written as zeros (embedding, softmax); other rows are unaffected.
 *   - Element counts are int64_t; fp32 tensors are row-major and contiguous.
 *   - Floating-point results follow the reference CPU arithmetic of
 *     src/ops.cc and src/quant.cc: bit-exact for the embedding gather, the
 *     residual sum and RoPE; within 1e-5 relative error for RMSNorm's output,
 *     SiLU/SwiGLU and softmax (whose sums are reduced in a different order and
 *     whose exponential is CUDA's expf).
 *   - No entry point falls back to the CPU.
 */
#ifndef MLB_OPS_H_
#define MLB_OPS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MLB_OK = 0,
  MLB_ERR_ARG = 1,
  MLB_ERR_CUDA = 2,
  MLB_ERR_RANGE = 3 /* a token id or position checked on the host is out of
                       range, or mlb_status_check found a status bit set */
};

/* Status bits written by kernels into the optional device status word. */
enum {
  MLB_STATUS_BAD_TOKEN = 1,    /* embedding: token id < 0 or >= vocab      */
  MLB_STATUS_BAD_POSITION = 2, /* rope: position < 0 or >= table rows     */
  MLB_STATUS_BAD_LENGTH = 4    /* softmax: valid length outside [1, cols] */
};

/* Table formats; same order as the reference's QuantType
 * (include/mini_llama/quantized_tensor.h:13) and its ggml block layouts
 * (quantized_tensor.h:19-35): Q8_0 34 B, Q4_0 18 B, Q4_1 20 B per 32 values. */
enum { MLB_F32 = 0, MLB_Q8_0 = 1, MLB_Q4_0 = 2, MLB_Q4_1 = 3 };

/* Library version (major * 10000 + minor * 100 + patch). */
int mlb_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* mlb_last_error(void);

/* Bytes of one table row: ceil(cols / 32) blocks, or cols floats for F32. */
int64_t mlb_row_bytes(int qtype, int64_t cols);

/*
 * (Residual-add +) RMSNorm over rows.
 * Replaces CudaRmsNorm (cuda_ops.h:12-13, cuda_ops.cu:193-204) and, fused,
 * the CudaAdd that precedes it in the layer (cuda_forward.cc:72-77, 83;
 * CPU composition forward.cc:122-124 -> ops.cc:117-124, 68-81):
 *   h[r] = x[r] + residual[r]            (bit-exact; skipped if residual NULL)
 *   y[r] = h[r] * (1 / sqrt(sum(h[r]^2) / cols + eps)) * w
 * residual and h_out may be NULL; with residual NULL the norm is of x.
 * x, residual, h_out and y are [rows, cols]; w is [cols].  h_out may alias x
 * or residual; y may alias x.  One pass over memory.
 */
int mlb_rmsnorm_f32(const float* x, const float* residual, float* h_out,
                    float* y, const float* w, int64_t rows, int64_t cols,
                    float eps, void* stream);

/*
 * SwiGLU over n = rows * cols elements: out = (g / (1 + exp(-g))) * u.
 * Replaces CudaSilu + CudaMul (cuda_ops.h:19-22, cuda_ops.cu:222-240, used
 * together at cuda_forward.cc:80-82; CPU ops.cc:100-115).  One pass.
 * out may alias gate or up.
 */
int mlb_swiglu_f32(const float* gate, const float* up, float* out,
                   int64_t rows, int64_t cols, void* stream);

/* SiLU alone, out = x / (1 + exp(-x)); replaces CudaSilu (cuda_ops.h:19). */
int mlb_silu_f32(const float* x, float* out, int64_t n, void* stream);

/* Element-wise product; replaces CudaMul (cuda_ops.h:22). */
int mlb_mul_f32(const float* a, const float* b, float* out, int64_t n,
                void* stream);

/* Element-wise sum; replaces CudaAdd (cuda_ops.h:25). Bit-exact. */
int mlb_add_f32(const float* a, const float* b, float* out, int64_t n,
                void* stream);

/*
 * Bias add over rows: out[r] = value[r] + bias (a copy when bias is NULL).
 * Replaces CudaAddBias (cuda_ops.h:34, cuda_ops.cu:298-308). Bit-exact.
 */
int mlb_add_bias_f32(const float* value, const float* bias, float* out,
                     int64_t rows, int64_t cols, void* stream);

/*
 * Host-side (cos, sin) table for RoPE, bit-identical to the values the
 * reference computes inline (ops.cc:26-31 normal, :45-50 NeoX; the two
 * exponent expressions give the same float):
 *   angle(p, j) = (float)p / powf(theta, (float)(2j) / (float)hd)
 *   out_host[((p - pos_begin) * hd/2 + j) * 2 + {0,1}] = {cosf, sinf}(angle)
 * for p in [pos_begin, pos_end), j in [0, hd/2).  Computed with the host's
 * libm so it matches the reference CPU path on the same machine.
 */
int mlb_rope_table_build_host(float theta, int hd, int64_t pos_begin,
                              int64_t pos_end, float* out_host);

/*
 * Attention-bias add + rotary embedding, in place, for a batch of tokens.
 * Replaces CudaAddBias(q/k) + CudaRope (cuda_ops.h:15-17, 34;
 * cuda_ops.cu:206-220, 298-308; CPU forward.cc:113-119 -> ops.cc:126-142).
 *   q: [rows, nq, hd], k: [rows, nk, hd]  (k may be NULL when nk == 0)
 *   bq: [nq*hd] or NULL, bk: [nk*hd] or NULL (added before rotation)
 *   positions: [rows] int32 device array, or NULL for consecutive
 *   positions: token t then sits at position_base + t (a prefill chunk, or
 *   the single token of a decode step with rows = 1).
 *   cos_sin: table from mlb_rope_table_build_host with table_rows positions
 *   starting at position 0.
 *   neox = 0: pairs (2j, 2j+1); neox = 1: pairs (j, j + hd/2).
 * x0' = x0*c - x1*s, x1' = x0*s + x1*c with separate roundings: bit-exact.
 * With a positions array, a token whose position is outside [0, table_rows)
 * gets its bias added but is not rotated, and MLB_STATUS_BAD_POSITION is
 * raised.  Without one, the range [position_base, position_base + rows) is
 * checked on the host and MLB_ERR_RANGE returned (nothing launched) if it
 * leaves the table, as the reference throws for a negative position
 * (ops.cc:132-134).
 */
int mlb_rope_f32(float* q, float* k, const float* bq, const float* bk,
                 const int32_t* positions, int64_t position_base,
                 const float* cos_sin, int64_t table_rows, int64_t rows,
                 int nq, int nk, int hd, int neox, int32_t* status,
                 void* stream);

/*
 * Row softmax over the first valid_len[r] entries of each row, zeros after
 * (valid_len NULL = full rows).  Replaces CudaSoftmax (cuda_ops.h:28,
 * cuda_ops.cu:253-262; CPU ops.cc:83-98) and the per-head softmax of the
 * causal attention rows (forward.cc:53-63).  x, y: [rows, cols]; y may
 * alias x.  A row whose length is outside [1, cols] is written as zeros and
 * raises MLB_STATUS_BAD_LENGTH.
 */
int mlb_softmax_rows_f32(const float* x, float* y, int64_t rows, int64_t cols,
                         const int32_t* valid_len, int32_t* status,
                         void* stream);

/*
 * Token-embedding gather with in-register block dequantisation.
 * Replaces CudaEmbeddingRow (cuda_ops.h:31, cuda_ops.cu:146-189, 264-296;
 * CPU forward.cc:29-33 -> quant.cc:278-304).
 *   table: vocab rows of mlb_row_bytes(qtype, cols) bytes, ggml blocks as
 *   the reference stores them (a partial tail block when cols % 32 != 0).
 *   tokens: [rows] int32; out: [rows, cols] fp32.
 *   Q8_0: d*q;  Q4_0: d*(nib-8);  Q4_1: d*nib + m  (fp16 d, m decoded as in
 *   quant.cc:44-71).  Bit-exact with the reference.
 * A token outside [0, vocab) writes a zero row and raises
 * MLB_STATUS_BAD_TOKEN.
 */
int mlb_embedding_gather(const void* table, int qtype, int64_t vocab,
                         int64_t cols, const int32_t* tokens, int64_t rows,
                         float* out, int32_t* status, void* stream);

/*
 * One embedding row for a token id held on the host: the per-token form of
 * mlb_embedding_gather that CudaEmbeddingRow (cuda_ops.cu:264-296) maps to.
 * The id is range-checked on the host: MLB_ERR_RANGE (nothing launched) when
 * it is outside [0, vocab), as the reference throws std::out_of_range
 * (cuda_ops.cu:265-267, quant.cc:279-281).  out: [cols] fp32.
 */
int mlb_embedding_row(const void* table, int qtype, int64_t vocab,
                      int64_t cols, int32_t token, float* out, void* stream);

/*
 * Linear layer for decode-sized batches: y[t] = W · x[t] for t < t_rows.
 * Replaces CudaLinear (include/mini_llama/cuda_matmul.h:11, cuda_matmul.cu:
 * 41-101 block GEMV kernels and the cuBLAS SGEMV F32 path :122-133; CPU
 * quant.cc:171-226 LinearWithBlocks, matmul_optimized.cc:95-117).
 *   w: n rows of mlb_row_bytes(qtype, k) bytes (ggml blocks or F32), the
 *   reference's weight layout; x: [t_rows, k]; y: [t_rows, n].
 * Every block's 32 products are summed before its scale is applied and the
 * row is reduced across a warp, so y matches the reference's sequential sum
 * within |y - y_ref| <= 1e-5 * sum_i |w_i x_i|.  Weights are read once per
 * group of 8 tokens; k % 32 != 0 or unaligned x take a scalar path that keeps
 * the reference's summation order.
 * Large ggml launches (Q8_0: k % 256 == 0, Q4_0 / Q4_1: k % 512 == 0,
 * 16-byte aligned table; long rows split over a cluster of up to 8 CTAs)
 * run on the int8 tensor cores instead once they hold enough weight blocks
 * (rows x k / 32: for one matrix 1.2 M at one token in Q8_0, 2.4 M / 1.2 M
 * at one / two tokens in Q4_0 / Q4_1; 400 K otherwise), up
 * to 4 tokens per pass: the codes enter the MMA as stored and x as four
 * exact int8 digits per value relative to a power-of-two block scale
 * (|x_i - digits| <= 2^-27 max|x| of its block), within the same bound.
 */
int mlb_linear_f32(const void* w, int qtype, int64_t n, int64_t k,
                   const float* x, int64_t t_rows, float* y, void* stream);

/*
 * Kernel choice of mlb_linear_f32 for ggml formats: 0 = automatic (the
 * default), 1 = always the CUDA-core GEMV, 2 = the tensor-core GEMV wherever
 * its shape rules allow.  Process-wide; for benchmarks and tests.  Returns
 * MLB_OK, or MLB_ERR_ARG for another value.  mlb_gemv_path returns the
 * current setting.  No counterpart in the reference.
 */
int mlb_set_gemv_path(int path);
int mlb_gemv_path(void);

/*
 * Launch overlap: 1 (the default) launches every kernel with programmatic
 * dependent launch, so that a kernel's launch and set-up overlap the tail of
 * the stream's previous kernel (each kernel first waits, on the device, for
 * the previous one to complete and its writes to be visible); 0 launches them
 * one after another.  Results are the same either way.  Process-wide; for
 * benchmarks and tests.  Returns MLB_OK, or MLB_ERR_ARG for another value;
 * mlb_launch_overlap returns the current setting.  No counterpart in the
 * reference.
 */
int mlb_set_launch_overlap(int on);
int mlb_launch_overlap(void);

/* Floats of scratch mlb_linear_rows_f32 needs for t_rows tokens of k values
 * (-1 for bad arguments). */
int64_t mlb_linear_rows_scratch_floats(int64_t k, int64_t t_rows);

/*
 * Linear layer for prompt-sized batches: y[t] = W . x[t] for t < t_rows, the
 * reference's CudaLinear / Linear (cuda_matmul.cu, quant.cc:171-226) applied
 * to every token of a prompt at once.  From 48 tokens on (k % 32 == 0,
 * row_bytes % 16 == 0, 16-byte aligned table and x) it runs on the tensor
 * cores.  Q8_0 / Q4_0 (k % 64 == 0): each dequantised weight d * q is split
 * into two fp16 pieces without error (|d| < 512; a 128 x 128 tile with a
 * larger or non-finite block scale is computed on the CUDA cores), x,
 * scaled per token by a power of two, into two fp16 pieces, and one fp32
 * accumulator spans the whole of k.  Q4_1 / F32: tcgen05 TF32 MMAs
 * with W dequantised and both operands split into TF32 head + tail (three
 * products per tile).  Either way the result stays within 1e-5 * sum|w x|
 * of the reference's fp32 sum; `scratch` (caller-owned device memory of
 * mlb_linear_rows_scratch_floats(k, t_rows) floats) holds x's split.
 * Otherwise it is mlb_linear_f32 (scratch unused).
 * x [t_rows, k], y [t_rows, n].
 */
int mlb_linear_rows_f32(const void* w, int qtype, int64_t n, int64_t k,
                        const float* x, int64_t t_rows, float* y, float* scratch,
                        int64_t scratch_floats, void* stream);

/*
 * mlb_linear_rows_f32 for `count` (1..3) weight matrices applied to the same
 * x in one launch — the q / k / v projections of a layer, or its FFN gate
 * and up — sharing one split of x and one grid (small matrices no longer
 * leave SMs idle): y[m] [t_rows, n[m]] = x . W[m]^T.  All matrices have
 * format `qtype` and width k; scratch as for mlb_linear_rows_f32.
 */
int mlb_linear_rows_group_f32(int count, const void* const* w, int qtype,
                              const int64_t* n, int64_t k, const float* x,
                              int64_t t_rows, float* const* y, float* scratch,
                              int64_t scratch_floats, void* stream);

/*
 * Number of bounded device-side waits (a bulk weight copy that did not land
 * within the kernel's poll limit) that gave up on the current device since
 * the library was loaded.  A kernel that gives up leaves NaN in the outputs
 * it did not finish instead of hanging.  Returns MLB_ERR_CUDA (with *count
 * still set) when a waiting warp also gave up on copies it had in flight, so
 * that a copy may have landed in shared memory after its block exited: the
 * device's results since then are undefined.  Synchronous.  Diagnostic only:
 * no counterpart in the reference.
 */
int mlb_wait_timeouts(unsigned int* count);

/*
 * KV-cache write: rows tokens' k and v ([rows, n_kv_heads * head_dim]) go to
 * positions [position, position + rows) of one layer's cache, laid out as the
 * reference's CudaKvCache layer [max_seq, n_kv_heads, head_dim]
 * (cuda_attention.h:8-40; CudaKvCache::Write / KvWriteKernel
 * cuda_attention.cu:13-23, 128-145; CPU kv_cache.cc:25-40).  Bit-exact copy.
 * MLB_ERR_RANGE when the positions leave [0, max_seq).
 */
int mlb_kv_write_f32(float* keys, float* values, const float* k, const float* v,
                     int64_t position, int64_t rows, int64_t max_seq,
                     int n_kv_heads, int head_dim, void* stream);

/* Floats of scratch mlb_attention_decode_f32 needs for these sizes and
 * position (-1 for bad arguments). */
int64_t mlb_attention_scratch_floats(int n_heads, int n_kv_heads, int head_dim,
                                     int64_t position);

/*
 * Decode attention of one token at `position` over one layer's cache:
 *   out[h] = softmax_t(q[h] . k_t / sqrt(head_dim)) . v_t,  t = 0..position,
 * kv head h / (n_heads / n_kv_heads) for query head h (GQA, group <= 8).
 * Replaces CudaAttention (cuda_attention.h:43-45, cuda_attention.cu:26-106,
 * 147-195; CPU forward.cc:50-95).  q, out: [n_heads, head_dim]; keys, values:
 * the layer's [max_seq, n_kv_heads, head_dim]; head_dim % 4 == 0, <= 256.
 * The visible positions are split over CTAs (flash-decoding); each CTA reads
 * a kv head's K/V rows once for all of its query heads and writes a partial
 * softmax state to `scratch` (caller-owned device memory of at least
 * mlb_attention_scratch_floats(...) floats), which a second kernel combines
 * (through shared memory when the scratch is 16-byte aligned, as every
 * cudaMalloc / torch allocation is; from global memory otherwise).
 * Within 1e-5 * sum_t w_t |v_t| of the reference.  MLB_ERR_RANGE when
 * position is outside [0, max_seq).
 */
int mlb_attention_decode_f32(const float* q, const float* keys,
                             const float* values, float* out, int64_t position,
                             int64_t max_seq, int n_heads, int n_kv_heads,
                             int head_dim, float* scratch,
                             int64_t scratch_floats, void* stream);

/* Floats of scratch mlb_attention_rows_f32 needs (-1 for bad arguments). */
int64_t mlb_attention_rows_scratch_floats(int n_heads, int n_kv_heads,
                                          int head_dim, int64_t position,
                                          int64_t rows);

/*
 * Causal attention of `rows` consecutive query tokens (a prompt chunk) over
 * one layer's cache: row r is the token at position + r and attends to cache
 * positions 0 .. position + r, exactly as if the reference's per-token
 * CudaAttention (cuda_attention.cu:147-195) were called for each row in
 * order after its K/V were written.  This is the attention step of the
 * row-batched prefill driver, which replaces ForwardBatch's per-token loop
 * (batch.cc:26-41); write the rows' K/V first (mlb_kv_write_f32 with the same
 * position and rows).  q, out: [rows, n_heads, head_dim]; other arguments and
 * the tolerance as mlb_attention_decode_f32 (which is this call with
 * rows = 1).  MLB_ERR_RANGE when position + rows > max_seq.
 */
int mlb_attention_rows_f32(const float* q, const float* keys,
                           const float* values, float* out, int64_t position,
                           int64_t rows, int64_t max_seq, int n_heads,
                           int n_kv_heads, int head_dim, float* scratch,
                           int64_t scratch_floats, void* stream);

/*
 * Kernel choice of mlb_attention_rows_f32 for prompt chunks (two rows or
 * more): 0 = automatic (the default: the tensor cores from 512 rows),
 * 1 = always the CUDA-core
 * kernels, 2 = the tensor cores wherever the shape allows (group 1 .. 8,
 * head_dim 64 or 128, 16-byte aligned tensors).  Process-wide; for benchmarks
 * and tests.  Returns MLB_OK, or MLB_ERR_ARG for another value;
 * mlb_attention_path returns the current setting.  No counterpart in the
 * reference.
 */
int mlb_set_attention_path(int path);
int mlb_attention_path(void);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference:
 * it is mlb_attention_decode_f32 for callers that cannot provide device
 * scratch — a plugin inside a host framework that owns every device
 * allocation, or a token loop that must not call cudaMalloc / cudaFree
 * (those can synchronise the whole device).  The slice partials live in a
 * file-scope device array of the library, 1 Mi floats (4 MiB), held on every
 * GPU where the library's kernels are loaded until the process exits.
 *   - Sizes whose mlb_attention_scratch_floats(...) exceeds 1 Mi floats are
 *     rejected with MLB_ERR_ARG and a message naming the need.
 *   - The first call on a device looks up the array's device address (once
 *     per device and context, with that device current) and keeps it; make
 *     that first call before any stream capture.  A context created with
 *     cuCtxCreate gets its own lookup.  Do not call it again on a device
 *     after cudaDeviceReset of that device: the library's device code is
 *     loaded anew there and the kept address may no longer be the array's.
 *   - Every call shares the one array and it keeps the last call's contents
 *     (nothing in it needs to start at zero): calls that overlap on the GPU —
 *     on different streams, or from several host threads — race.
 * Arguments and results as for mlb_attention_decode_f32.
 */
int mlb_attention_decode_noalloc_f32(const float* q, const float* keys,
                                     const float* values, float* out,
                                     int64_t position, int64_t max_seq,
                                     int n_heads, int n_kv_heads, int head_dim,
                                     void* stream);

/*
 * Helper for synchronous callers: waits for `stream`, copies the device
 * status word to the host, and returns MLB_OK when it is zero, MLB_ERR_RANGE
 * when a bit is set (the bits are stored in *bits_host when non-NULL), or
 * MLB_ERR_CUDA.  Does not clear the word.
 */
int mlb_status_check(const int32_t* status, int32_t* bits_host, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLB_OPS_H_ */
