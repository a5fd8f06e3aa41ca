/*
 * CPU oracle for the mini-lla layer operators — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference CPU arithmetic of mini-lla's
 * per-layer operators (src/ops.cc, src/quant.cc, src/forward.cc of the
 * reference project).  It is the checker that the CUDA kernels of the
 * product library are compared against.  Only tests, the smoke check and the
 * CPU-baseline leg of bench.py may load it; the product path never does.
 *
 * Every floating-point expression keeps the reference's evaluation order and
 * its separate roundings: the file is compiled with -ffp-contract=off and
 * without -ffast-math, and it calls the same libm entry points (powf, cosf,
 * sinf, expf, sqrtf) that the reference's std:: overloads resolve to.
 *
 * Parity pin: the test suite compares every function here bit-for-bit with
 * the reference's own ops.cc / quant.cc compiled from source
 * (oracle/ref_shim.cc), and with the golden fixtures under tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define MLBO_BLOCK 32

/* Block byte sizes, quantized_tensor.h:19-39 (BlockQ8_0 34 B, BlockQ4_0 18 B,
 * BlockQ4_1 20 B); F32 rows are plain floats. */
enum { MLBO_F32 = 0, MLBO_Q8_0 = 1, MLBO_Q4_0 = 2, MLBO_Q4_1 = 3 };

int mlbo_block_bytes(int qtype) {
  switch (qtype) {
    case MLBO_F32: return 4 * MLBO_BLOCK;
    case MLBO_Q8_0: return 34;
    case MLBO_Q4_0: return 18;
    case MLBO_Q4_1: return 20;
    default: return -1;
  }
}

/* Bytes of one table row: ceil(cols/32) blocks (quantized_tensor.h:56);
 * F32 rows are exactly cols floats. */
int64_t mlbo_row_bytes(int qtype, int64_t cols) {
  if (qtype == MLBO_F32) return cols * 4;
  const int64_t blocks = (cols + MLBO_BLOCK - 1) / MLBO_BLOCK;
  return blocks * mlbo_block_bytes(qtype);
}

static uint16_t load_u16(const uint8_t* p) {
  uint16_t v;
  memcpy(&v, p, sizeof(v));
  return v;
}

/* FP16 bit pattern -> F32, integer decode with the subnormal normalisation
 * loop; reference src/quant.cc:44-71 (Fp16ToFloat). */
float mlbo_fp16_to_f32(uint16_t value) {
  const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t mantissa = value & 0x03ffu;
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa != 0) {
      exponent = 1;
      while ((mantissa & 0x0400u) == 0) {
        mantissa <<= 1;
        --exponent;
      }
      mantissa &= 0x03ffu;
      bits = sign | ((exponent + (127 - 15)) << 23) | (mantissa << 13);
    } else {
      bits = sign;
    }
  } else if (exponent == 31) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | ((exponent + (127 - 15)) << 23) | (mantissa << 13);
  }
  float result;
  memcpy(&result, &bits, sizeof(result));
  return result;
}

/* One element of one block; reference src/quant.cc:148-167
 * (DequantizeElement for Q8_0, Q4_0, Q4_1). */
static float dequant_element(int qtype, const uint8_t* block, int index) {
  const float d = mlbo_fp16_to_f32(load_u16(block));
  if (qtype == MLBO_Q8_0) {
    const int8_t q = (int8_t)block[2 + index];
    return d * (float)q;
  }
  const uint8_t* qs = block + (qtype == MLBO_Q4_1 ? 4 : 2);
  const int packed = index < MLBO_BLOCK / 2 ? (qs[index] & 0x0f)
                                            : (qs[index - MLBO_BLOCK / 2] >> 4);
  if (qtype == MLBO_Q4_0) return d * (float)(packed - 8);
  const float m = mlbo_fp16_to_f32(load_u16(block + 2));
  return d * (float)packed + m;
}

/* Embedding gather: out[t] = DequantizeRow(table, tokens[t]); reference
 * src/forward.cc:29-33 -> src/quant.cc:278-304 -> :187-199.  Returns the
 * number of out-of-range tokens (their rows are left untouched), where the
 * reference throws std::out_of_range (quant.cc:279-281). */
int64_t mlbo_embedding_rows(const void* table, int qtype, int64_t vocab,
                            int64_t cols, const int32_t* tokens, int64_t rows,
                            float* out) {
  const uint8_t* base = (const uint8_t*)table;
  const int64_t row_bytes = mlbo_row_bytes(qtype, cols);
  const int bb = mlbo_block_bytes(qtype);
  int64_t bad = 0;
  for (int64_t t = 0; t < rows; ++t) {
    const int64_t token = tokens[t];
    float* dst = out + t * cols;
    if (token < 0 || token >= vocab) {
      ++bad;
      continue;
    }
    const uint8_t* row = base + token * row_bytes;
    if (qtype == MLBO_F32) {
      memcpy(dst, row, (size_t)cols * sizeof(float));
      continue;
    }
    const int64_t blocks = (cols + MLBO_BLOCK - 1) / MLBO_BLOCK;
    for (int64_t b = 0; b < blocks; ++b) {
      const int64_t begin = b * MLBO_BLOCK;
      const int64_t end = begin + MLBO_BLOCK < cols ? begin + MLBO_BLOCK : cols;
      for (int64_t i = begin; i < end; ++i) {
        dst[i] = dequant_element(qtype, row + b * bb, (int)(i - begin));
      }
    }
  }
  return bad;
}

/* Element-wise residual add a + b; reference src/ops.cc:117-124 (Add). */
void mlbo_add(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* One RMSNorm row: sequential fp32 sum of squares, IEEE divide and sqrt,
 * y = (x * inv) * w; reference src/ops.cc:68-81 (RmsNorm). */
void mlbo_rmsnorm_row(const float* x, const float* w, float* y, int64_t n,
                      float eps) {
  float square_sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) square_sum += x[i] * x[i];
  const float inverse_rms = 1.0f / sqrtf(square_sum / (float)n + eps);
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * inverse_rms * w[i];
}

/* Row-batched (residual-add +) RMSNorm, as the reference composes it at
 * src/forward.cc:122-124: h = Add(x, residual); y = RmsNorm(h, w, eps).
 * residual may be NULL (plain RMSNorm of x); h may be NULL. */
void mlbo_rmsnorm_rows(const float* x, const float* residual, float* h,
                       float* y, const float* w, int64_t rows, int64_t cols,
                       float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float* yr = y + r * cols;
    if (residual != NULL) {
      float* hr = h != NULL ? h + r * cols : yr; /* y doubles as scratch */
      mlbo_add(xr, residual + r * cols, hr, cols);
      mlbo_rmsnorm_row(hr, w, yr, cols, eps);
    } else {
      mlbo_rmsnorm_row(xr, w, yr, cols, eps);
    }
  }
}

/* SwiGLU: Silu(g) * u with Silu = g / (1 + exp(-g)); reference
 * src/ops.cc:100-115 (Silu, SwiGlu). */
void mlbo_swiglu(const float* gate, const float* up, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float s = gate[i] / (1.0f + expf(-gate[i]));
    s *= up[i];
    out[i] = s;
  }
}

/* Silu alone; reference src/ops.cc:100-106. */
void mlbo_silu(const float* x, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}

/* Softmax of one vector: max, exp(x - max) with a sequential sum, divide;
 * reference src/ops.cc:83-98. */
void mlbo_softmax_row(const float* x, float* y, int64_t n) {
  float maximum = x[0];
  for (int64_t i = 1; i < n; ++i)
    if (x[i] > maximum) maximum = x[i];
  float total = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    y[i] = expf(x[i] - maximum);
    total += y[i];
  }
  for (int64_t i = 0; i < n; ++i) y[i] /= total;
}

/* Row softmax over the first valid_len[r] entries of each row, zeros after
 * (the causal use at src/forward.cc:53-63 softmaxes the pos+1 visible
 * scores).  valid_len NULL means every row is full.  Returns the number of
 * rows whose valid length is outside [1, cols] (written as zeros), where the
 * reference throws on an empty vector (ops.cc:84-86). */
int64_t mlbo_softmax_rows(const float* x, float* y, int64_t rows, int64_t cols,
                          const int32_t* valid_len) {
  int64_t bad = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t len = valid_len != NULL ? valid_len[r] : cols;
    float* yr = y + r * cols;
    if (len < 1 || len > cols) {
      ++bad;
      for (int64_t i = 0; i < cols; ++i) yr[i] = 0.0f;
      continue;
    }
    mlbo_softmax_row(x + r * cols, yr, len);
    for (int64_t i = len; i < cols; ++i) yr[i] = 0.0f;
  }
  return bad;
}

/* The rotation angle of pair j at a position.  Normal layout,
 * src/ops.cc:26-28: pos / pow(theta, (float)i / (float)hd) with i = 2j.
 * NeoX layout, src/ops.cc:45-47: pos / pow(theta, 2.0f * (float)j / (float)hd).
 * 2.0f * (float)j and (float)(2j) are the same float, so the two agree. */
static float rope_angle(int64_t position, float theta, int pair, int hd,
                        int neox) {
  const float exponent = neox ? 2.0f * (float)pair / (float)hd
                              : (float)(2 * pair) / (float)hd;
  return (float)position / powf(theta, exponent);
}

/* Host-built per-position (cos, sin) table: out[(p - pos_begin) * hd/2 + j]
 * = {cos(angle), sin(angle)} — the same values ops.cc computes inline. */
void mlbo_rope_table(float theta, int hd, int64_t pos_begin, int64_t pos_end,
                     float* out) {
  const int half = hd / 2;
  for (int64_t p = pos_begin; p < pos_end; ++p) {
    for (int j = 0; j < half; ++j) {
      const float angle = rope_angle(p, theta, j, hd, 0);
      float* slot = out + ((p - pos_begin) * half + j) * 2;
      slot[0] = cosf(angle);
      slot[1] = sinf(angle);
    }
  }
}

/* Rotate the heads of one token in place; reference src/ops.cc:22-56
 * (ApplyRopeNormal pairs (2j, 2j+1), ApplyRopeNeoX pairs (j, j + hd/2)):
 * x0' = x0*c - x1*s, x1' = x0*s + x1*c. */
static void rope_heads(float* x, int heads, int hd, int64_t position,
                       float theta, int neox) {
  const int half = hd / 2;
  for (int head = 0; head < heads; ++head) {
    float* v = x + (int64_t)head * hd;
    for (int j = 0; j < half; ++j) {
      const float angle = rope_angle(position, theta, j, hd, neox);
      const float cosine = cosf(angle);
      const float sine = sinf(angle);
      const int a = neox ? j : 2 * j;
      const int b = neox ? j + half : 2 * j + 1;
      const float first = v[a];
      const float second = v[b];
      v[a] = first * cosine - second * sine;
      v[b] = first * sine + second * cosine;
    }
  }
}

/* Row-batched attention-bias add + RoPE: for every token t, q[t] += bq,
 * k[t] += bk (src/forward.cc:36-47, 113-118; skipped when NULL), then
 * Rope(q[t], k[t], positions[t], theta) (src/ops.cc:126-142).
 * q is [rows, nq, hd], k is [rows, nk, hd], both rotated in place.
 * Returns the number of tokens with a negative position (left unrotated),
 * where the reference throws (ops.cc:132-134). */
int64_t mlbo_rope_rows(float* q, float* k, const float* bq, const float* bk,
                       const int32_t* positions, int64_t rows, int nq, int nk,
                       int hd, float theta, int neox) {
  int64_t bad = 0;
  for (int64_t t = 0; t < rows; ++t) {
    float* qt = q + t * (int64_t)nq * hd;
    float* kt = k + t * (int64_t)nk * hd;
    if (bq != NULL) mlbo_add(qt, bq, qt, (int64_t)nq * hd);
    if (bk != NULL) mlbo_add(kt, bk, kt, (int64_t)nk * hd);
    if (positions[t] < 0) {
      ++bad;
      continue;
    }
    rope_heads(qt, nq, hd, positions[t], theta, neox);
    rope_heads(kt, nk, hd, positions[t], theta, neox);
  }
  return bad;
}

/* Linear layer y[t] = W · x[t] over a table of `n` rows x `k` columns (the
 * weight layout of the embedding table: ggml blocks or F32 rows).
 * Quantised: reference src/quant.cc:171-185 (DotQuantizedRow: sequential
 * sum of DequantizeElement(w) * x, each product and partial sum rounded) and
 * :202-226 (LinearWithBlocks, one dot per (row, output)).
 * F32: src/matmul_optimized.cc:95-117 (LinearOptimized: sum += x[k] * w[k]).
 * x is [t_rows, k], y is [t_rows, n]. */
void mlbo_linear_rows(const void* table, int qtype, int64_t n, int64_t k,
                      const float* x, int64_t t_rows, float* y) {
  const uint8_t* base = (const uint8_t*)table;
  const int64_t row_bytes = mlbo_row_bytes(qtype, k);
  const int bb = mlbo_block_bytes(qtype);
  for (int64_t t = 0; t < t_rows; ++t) {
    const float* xt = x + t * k;
    for (int64_t j = 0; j < n; ++j) {
      const uint8_t* row = base + j * row_bytes;
      float sum = 0.0f;
      if (qtype == MLBO_F32) {
        const float* w = (const float*)row;
        for (int64_t i = 0; i < k; ++i) sum += xt[i] * w[i];
      } else {
        const int64_t blocks = (k + MLBO_BLOCK - 1) / MLBO_BLOCK;
        for (int64_t b = 0; b < blocks; ++b) {
          const int64_t begin = b * MLBO_BLOCK;
          const int64_t end = begin + MLBO_BLOCK < k ? begin + MLBO_BLOCK : k;
          for (int64_t i = begin; i < end; ++i)
            sum += dequant_element(qtype, row + b * bb, (int)(i - begin)) * xt[i];
        }
      }
      y[t * n + j] = sum;
    }
  }
}

/* Decode attention of one token at `position` over one layer's cache
 * [max_seq, n_kv_heads, hd]; reference src/forward.cc:50-95 (AttentionHead,
 * Attention): per query head h (kv head h / group), score_t = dot(q, k_t) *
 * scale with a sequential dot and scale = 1 / sqrt(hd) (forward.cc:75),
 * w = Softmax(score) (ops.cc:83-98), out[i] += w_t * v_t[i] in t order.
 * scores must hold position + 1 floats. */
void mlbo_attention_decode(const float* q, const float* keys,
                           const float* values, float* out, int64_t position,
                           int n_heads, int n_kv_heads, int hd, float* scores) {
  const int group = n_heads / n_kv_heads;
  const float scale = 1.0f / sqrtf((float)hd);
  const int64_t visible = position + 1;
  const int64_t stride = (int64_t)n_kv_heads * hd;
  for (int h = 0; h < n_heads; ++h) {
    const int kvh = h / group;
    const float* qh = q + (int64_t)h * hd;
    for (int64_t t = 0; t < visible; ++t) {
      const float* key = keys + t * stride + (int64_t)kvh * hd;
      float dot = 0.0f;
      for (int i = 0; i < hd; ++i) dot += qh[i] * key[i];
      scores[t] = dot * scale;
    }
    mlbo_softmax_row(scores, scores, visible);
    float* oh = out + (int64_t)h * hd;
    for (int i = 0; i < hd; ++i) oh[i] = 0.0f;
    for (int64_t t = 0; t < visible; ++t) {
      const float* value = values + t * stride + (int64_t)kvh * hd;
      const float w = scores[t];
      for (int i = 0; i < hd; ++i) oh[i] += w * value[i];
    }
  }
}
