/*
 * kllm_oracle.c — CPU restatement of LittleLLM's reference CPU operators
 * (src/op/cpu/ sources, src/base/half.cpp, src/model/weights.cpp).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library's parity tests,
 * smoke check and the benchmark's CPU-baseline leg. Nothing in the product
 * links or calls this file.
 *
 * The reference stores activations in a DType-tagged Tensor and every CPU op
 * reads/writes through read_cpu/write_cpu (include/kllm/op/detail/
 * cpu_helpers.h:23-50). These functions are the F32 instance of each op:
 * plain float arrays, same loop nest, same operation order, same libm calls,
 * so a build with the reference's flags (-O3, no -march, hence no FMA
 * contraction on x86-64) gives bit-identical fp32 results. The parity of
 * this file with the compiled reference is itself checked by the tests
 * (oracle vs. golden vectors produced by the reference).
 */
#include "kllm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* fp16 <-> fp32 conversion                                                */
/* ---------------------------------------------------------------------- */

/* Follows float_to_half (src/base/half.cpp:38-61). Bit-exact parity needs
 * the same steps, including the two non-IEEE behaviours:
 *  - rounding adds half an fp16 ulp (0x1000 in fp32 fraction units) and
 *    truncates, so ties round away from zero;
 *  - in the normal range the rounded 10-bit fraction is OR-ed into the
 *    exponent field instead of added, so a fraction that carries out
 *    (0x400) is lost when the fp16 exponent is odd.
 * Magnitudes with fp16 exponent >= 31 (including inf and NaN) become inf;
 * magnitudes below 2^-25 become signed zero. */
uint16_t kllm_oracle_float_to_half(float value) {
  uint32_t bits;
  memcpy(&bits, &value, sizeof bits);
  const uint32_t sign16 = (bits >> 16) & 0x8000u;
  const int32_t exp16 = (int32_t)((bits >> 23) & 0xffu) - 112; /* rebias 127 -> 15 */
  const uint32_t frac = bits & 0x007fffffu;

  if (exp16 <= 0) {
    if (exp16 < -10) {
      return (uint16_t)sign16;
    }
    const uint32_t denorm = (frac | 0x00800000u) >> (uint32_t)(1 - exp16);
    return (uint16_t)(sign16 | ((denorm + 0x1000u) >> 13));
  }
  if (exp16 >= 31) {
    return (uint16_t)(sign16 | 0x7c00u);
  }
  return (uint16_t)(sign16 | ((uint32_t)exp16 << 10) | ((frac + 0x1000u) >> 13));
}

/* Same mapping as half_to_float (src/base/half.cpp:7-36): exact for every
 * finite fp16 value; fp16 subnormals are m * 2^-24, inf/NaN keep the
 * payload shifted into the fp32 fraction. */
float kllm_oracle_half_to_float(uint16_t value) {
  const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  const uint32_t exp5 = (value >> 10) & 0x1fu;
  const uint32_t frac = value & 0x03ffu;
  uint32_t bits;
  if (exp5 == 0) {
    const float mag = (float)frac * 0x1p-24f; /* exact: frac < 2^10 */
    memcpy(&bits, &mag, sizeof bits);
    bits |= sign;
  } else if (exp5 == 0x1fu) {
    bits = sign | 0x7f800000u | (frac << 13);
  } else {
    bits = sign | ((exp5 + 112u) << 23) | (frac << 13);
  }
  float out;
  memcpy(&out, &bits, sizeof out);
  return out;
}

void kllm_oracle_float_to_half_array(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = kllm_oracle_float_to_half(in[i]);
}

void kllm_oracle_half_to_float_array(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = kllm_oracle_half_to_float(in[i]);
}

/* ---------------------------------------------------------------------- */
/* Operators                                                               */
/* ---------------------------------------------------------------------- */

/* cpu_embedding (src/op/cpu/embedding.cpp:9-29): the id is checked before
 * its row is copied; rows before a bad id are already written. */
int kllm_oracle_embedding(const float* table, int64_t vocab, int64_t hidden,
                          const int32_t* ids, int64_t n_tokens, float* out, int64_t* bad) {
  for (int64_t t = 0; t < n_tokens; ++t) {
    const int32_t token = ids[t];
    if (token < 0 || token >= vocab) {
      if (bad) *bad = t;
      return -1;
    }
    memcpy(out + t * hidden, table + (int64_t)token * hidden, (size_t)hidden * sizeof(float));
  }
  return 0;
}

/* cpu_rms_norm (src/op/cpu/rms_norm.cpp:9-29): sequential fp32 sum of
 * squares, scale = 1 / sqrt(sum / hidden + eps), out = (x * scale) * w. */
void kllm_oracle_rms_norm(const float* x, const float* weight, float* out, int64_t rows,
                          int64_t hidden, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * hidden;
    float sum_sq = 0.0f;
    for (int64_t c = 0; c < hidden; ++c) {
      const float v = xr[c];
      sum_sq += v * v;
    }
    const float scale = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
    float* orow = out + r * hidden;
    for (int64_t c = 0; c < hidden; ++c) {
      orow[c] = xr[c] * scale * weight[c];
    }
  }
}

/* cpu_add_inplace (src/op/cpu/add.cpp:26-35). */
void kllm_oracle_add_inplace(float* x, const float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] + y[i];
}

/* cpu_add_bias_inplace (src/op/cpu/add.cpp:9-24); a NULL bias is a no-op. */
void kllm_oracle_add_bias_inplace(float* x, const float* bias, int64_t rows, int64_t cols) {
  if (bias == NULL) return;
  for (int64_t r = 0; r < rows; ++r) {
    float* xr = x + r * cols;
    for (int64_t c = 0; c < cols; ++c) xr[c] = xr[c] + bias[c];
  }
}

/* cpu_select_last_row (src/op/cpu/add.cpp:37-49). */
void kllm_oracle_select_last_row(const float* x, int64_t rows, int64_t cols, float* out) {
  memcpy(out, x + (rows - 1) * cols, (size_t)cols * sizeof(float));
}

/* cpu_matmul (src/op/cpu/matmul.cpp:9-33): out[r, c] = sum over i = 0..k-1,
 * in that order, of a[r, i] * b[c, i], accumulated in one fp32 variable
 * (b is [n, k]: the weight layout linear() passes, src/model/llama.cpp:12-24). */
void kllm_oracle_matmul(const float* a, const float* b, float* out, int64_t m, int64_t n, int64_t k) {
  for (int64_t r = 0; r < m; ++r) {
    const float* ar = a + r * k;
    for (int64_t c = 0; c < n; ++c) {
      const float* bc = b + c * k;
      float sum = 0.0f;
      for (int64_t i = 0; i < k; ++i) sum += ar[i] * bc[i];
      out[r * n + c] = sum;
    }
  }
}

/* cpu_silu_mul (src/op/cpu/silu.cpp:9-20) with sigmoid from
 * include/kllm/op/detail/cpu_helpers.h:19-21: (g * (1 / (1 + exp(-g)))) * u. */
void kllm_oracle_silu_mul(const float* gate, const float* up, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float g = gate[i];
    const float sig = 1.0f / (1.0f + expf(-g));
    out[i] = g * sig * up[i];
  }
}

/* cpu_rope_inplace (src/op/cpu/rope.cpp:10-37): rotate-half over pairs
 * (d, d + head_dim/2) at position past_len + t; the frequency exponent is
 * formed in float as (-2 * d) / head_dim and passed to powf. */
void kllm_oracle_rope_inplace(float* x, int64_t seq, int64_t heads, int64_t head_dim,
                              int32_t past_len, float theta) {
  const int64_t half = head_dim / 2;
  for (int64_t t = 0; t < seq; ++t) {
    const int32_t position = past_len + (int32_t)t;
    for (int64_t h = 0; h < heads; ++h) {
      float* base = x + (t * heads + h) * head_dim;
      for (int64_t d = 0; d < half; ++d) {
        const float inv_freq = powf(theta, -2.0f * (float)d / (float)head_dim);
        const float angle = (float)position * inv_freq;
        const float c = cosf(angle);
        const float s = sinf(angle);
        const float x1 = base[d];
        const float x2 = base[d + half];
        base[d] = x1 * c - x2 * s;
        base[d + half] = x2 * c + x1 * s;
      }
    }
  }
}

/* cpu_copy_kv_to_cache (src/op/cpu/kv_cache.cpp:9-32): caches are
 * [max_seq, kv_heads, head_dim]; rows past_len.. receive k/v rows. */
int kllm_oracle_copy_kv_to_cache(const float* k, const float* v, int64_t seq,
                                 int64_t kv_heads, int64_t head_dim, float* k_cache,
                                 float* v_cache, int64_t max_seq, int32_t past_len) {
  if (past_len + seq > max_seq) return -1;
  const int64_t row = kv_heads * head_dim;
  for (int64_t t = 0; t < seq; ++t) {
    const int64_t dst = ((int64_t)past_len + t) * row;
    memcpy(k_cache + dst, k + t * row, (size_t)row * sizeof(float));
    memcpy(v_cache + dst, v + t * row, (size_t)row * sizeof(float));
  }
  return 0;
}

/* cpu::dequantize_int8 (src/op/cpu/quantize.cpp:37-48) and the fp32 step of
 * the weight loader (src/model/weights.cpp:139-141): one fp32 multiply. */
void kllm_oracle_dequantize_int8_f32(const int8_t* q, int64_t n, float scale, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)q[i] * scale;
}

/* The fp16 weight-load path (src/model/weights.cpp:139-148): fp32 product,
 * then the reference float_to_half. */
void kllm_oracle_dequantize_int8_f16(const int8_t* q, int64_t n, float scale, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = kllm_oracle_float_to_half((float)q[i] * scale);
}

/* ---------------------------------------------------------------------- */
/* Compositions used as the oracle of the fused / batched operators        */
/* ---------------------------------------------------------------------- */

/* add_inplace then rms_norm, the sequence at src/model/llama.cpp:135-143
 * (delta == NULL: rms_norm alone, residual unchanged). */
void kllm_oracle_add_rms_norm(float* residual, const float* delta, const float* weight,
                              float* out, int64_t rows, int64_t hidden, float eps) {
  if (delta != NULL) kllm_oracle_add_inplace(residual, delta, rows * hidden);
  kllm_oracle_rms_norm(residual, weight, out, rows, hidden, eps);
}

/* The reference runs one sequence with a scalar past_len; a batch of tokens
 * with per-token positions and cache slots is the same ops applied to each
 * token as its own [1, heads, head_dim] call with past_len = position
 * (add_bias_inplace x3, rope_inplace x2, copy_kv_to_cache;
 * src/model/llama.cpp:89-114). The reference cache of one sequence is
 * [max_seq, kv_heads, head_dim]; element [pos, h, d] of slot s lands at
 * [s, h, pos, d] of the head-major [n_slots, kv_heads, max_seq, head_dim]
 * layer plane written here. */
int64_t kllm_oracle_qkv_bias_rope_kv_append(
    float* q, const float* k, const float* v, const float* bq, const float* bk,
    const float* bv, const int32_t* positions, const int32_t* slots, int64_t n_tokens,
    int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float theta, float* k_cache,
    float* v_cache, int64_t n_slots, int64_t max_seq) {
  const int64_t q_row = n_heads * head_dim;
  const int64_t kv_row = n_kv_heads * head_dim;
  float k_tmp[64 * 256];
  float v_tmp[64 * 256];
  int64_t skipped = 0;
  if (kv_row > 64 * 256) return -1;
  for (int64_t t = 0; t < n_tokens; ++t) {
    const int32_t pos = positions[t];
    const int32_t slot = slots[t];
    float* qt = q + t * q_row;
    memcpy(k_tmp, k + t * kv_row, (size_t)kv_row * sizeof(float));
    memcpy(v_tmp, v + t * kv_row, (size_t)kv_row * sizeof(float));
    kllm_oracle_add_bias_inplace(qt, bq, 1, q_row);
    kllm_oracle_add_bias_inplace(k_tmp, bk, 1, kv_row);
    kllm_oracle_add_bias_inplace(v_tmp, bv, 1, kv_row);
    kllm_oracle_rope_inplace(qt, 1, n_heads, head_dim, pos, theta);
    kllm_oracle_rope_inplace(k_tmp, 1, n_kv_heads, head_dim, pos, theta);
    if (pos < 0 || pos >= max_seq || slot < 0 || slot >= n_slots) {
      ++skipped;
      continue;
    }
    for (int64_t h = 0; h < n_kv_heads; ++h) {
      const int64_t dst = (((int64_t)slot * n_kv_heads + h) * max_seq + pos) * head_dim;
      memcpy(k_cache + dst, k_tmp + h * head_dim, (size_t)head_dim * sizeof(float));
      memcpy(v_cache + dst, v_tmp + h * head_dim, (size_t)head_dim * sizeof(float));
    }
  }
  return skipped;
}

/* select_last_row applied to each sequence of a packed batch
 * (src/op/cpu/add.cpp:37-49 on rows [start_b, end_b)). */
int kllm_oracle_select_last_rows(const float* x, int64_t rows, int64_t cols,
                                 const int32_t* seq_ends, int64_t seq_len, int64_t n_seqs,
                                 float* out) {
  int status = 0;
  for (int64_t b = 0; b < n_seqs; ++b) {
    const int64_t end = seq_ends ? (int64_t)seq_ends[b] : (b + 1) * seq_len;
    if (end < 1 || end > rows) {
      memset(out + b * cols, 0, (size_t)cols * sizeof(float));
      status = -1;
      continue;
    }
    kllm_oracle_select_last_row(x, end, cols, out + b * cols);
  }
  return status;
}

/* ---------------------------------------------------------------------- */
/* Attention (scope row f1)                                                */
/* ---------------------------------------------------------------------- */

/* One (token, head) of cpu_attention (src/op/cpu/attention.cpp:31-64):
 * scores over keys 0..key_limit-1 scaled by 1/sqrt(head_dim), max, exp,
 * the sum of exps, then out[d] = sum_pos (score[pos] / denom) * v[pos][d],
 * every sum in key order. k_row(pos) = k + pos * pos_stride (same for v). */
static void oracle_attend_row(const float* q_row, const float* k, const float* v,
                              int64_t pos_stride, int64_t key_limit, int64_t head_dim,
                              float* scores, float* out_row) {
  const float scale = 1.0f / sqrtf((float)head_dim);
  float max_score = -INFINITY;
  for (int64_t pos = 0; pos < key_limit; ++pos) {
    const float* k_row = k + pos * pos_stride;
    float dot = 0.0f;
    for (int64_t d = 0; d < head_dim; ++d) dot += q_row[d] * k_row[d];
    scores[pos] = dot * scale;
    if (scores[pos] > max_score) max_score = scores[pos];
  }
  float denom = 0.0f;
  for (int64_t pos = 0; pos < key_limit; ++pos) {
    scores[pos] = expf(scores[pos] - max_score);
    denom += scores[pos];
  }
  for (int64_t d = 0; d < head_dim; ++d) {
    float value = 0.0f;
    for (int64_t pos = 0; pos < key_limit; ++pos) {
      const float prob = scores[pos] / denom;
      value += prob * v[pos * pos_stride + d];
    }
    out_row[d] = value;
  }
}

/* cpu_attention (src/op/cpu/attention.cpp:12-67): q/out [seq, num_heads,
 * head_dim], caches [max_seq, num_kv_heads, head_dim]; token t attends to
 * keys 0..past_len+t, head h reads kv head h / (num_heads / num_kv_heads). */
void kllm_oracle_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                           int64_t seq, int32_t past_len, int64_t num_heads, int64_t num_kv_heads,
                           int64_t head_dim) {
  const int64_t groups = num_heads / num_kv_heads;
  float* scores = (float*)malloc((size_t)(past_len + seq + 1) * sizeof(float));
  if (!scores) return;
  for (int64_t t = 0; t < seq; ++t) {
    const int64_t key_limit = past_len + t + 1;
    for (int64_t h = 0; h < num_heads; ++h) {
      const int64_t kv_h = h / groups;
      oracle_attend_row(q + (t * num_heads + h) * head_dim, k_cache + kv_h * head_dim,
                        v_cache + kv_h * head_dim, num_kv_heads * head_dim, key_limit, head_dim,
                        scores, out + (t * num_heads + h) * head_dim);
    }
  }
  free(scores);
}

/* The same per-row computation over the head-major cache [n_slots,
 * num_kv_heads, max_seq, head_dim] of one layer: token t attends to
 * positions 0..positions[t] of sequence slot slots[t]. Rows of tokens with
 * a position outside [0, max_seq) or a slot outside [0, n_slots) are zero.
 * Returns the number of such tokens. */
int64_t kllm_oracle_attention_head_major(const float* q, const float* k_cache, const float* v_cache,
                                         float* out, const int32_t* positions, const int32_t* slots,
                                         int64_t n_tokens, int64_t num_heads, int64_t num_kv_heads,
                                         int64_t head_dim, int64_t n_slots, int64_t max_seq) {
  const int64_t groups = num_heads / num_kv_heads;
  int64_t bad = 0;
  float* scores = (float*)malloc((size_t)(max_seq + 1) * sizeof(float));
  if (!scores) return -1;
  for (int64_t t = 0; t < n_tokens; ++t) {
    const int64_t pos = positions[t], slot = slots[t];
    float* out_t = out + t * num_heads * head_dim;
    if (pos < 0 || pos >= max_seq || slot < 0 || slot >= n_slots) {
      memset(out_t, 0, (size_t)(num_heads * head_dim) * sizeof(float));
      ++bad;
      continue;
    }
    for (int64_t h = 0; h < num_heads; ++h) {
      const int64_t kv_h = h / groups;
      const int64_t base = ((slot * num_kv_heads + kv_h) * max_seq) * head_dim;
      oracle_attend_row(q + (t * num_heads + h) * head_dim, k_cache + base, v_cache + base, head_dim,
                        pos + 1, head_dim, scores, out_t + h * head_dim);
    }
  }
  free(scores);
  return bad;
}
