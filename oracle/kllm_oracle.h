/*
 * kllm_oracle.h — CPU restatement of LittleLLM's reference CPU operators.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the parity tests, the smoke
 * check and the CPU-baseline leg of the benchmark compare against; the
 * product (the CUDA library) never links or calls it.
 *
 * Every function follows one reference function (cited at its definition in
 * kllm_oracle.c) in fp32, with the same operation order, so that its results
 * are bit-identical to the reference CPU backend built with the same
 * compiler flags (no FMA contraction, sequential reductions, libm
 * powf/cosf/sinf/expf/sqrtf).
 */
#ifndef KLLM_ORACLE_H_
#define KLLM_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t kllm_oracle_float_to_half(float value);
float kllm_oracle_half_to_float(uint16_t value);
void kllm_oracle_float_to_half_array(const float* in, uint16_t* out, int64_t n);
void kllm_oracle_half_to_float_array(const uint16_t* in, float* out, int64_t n);

/* Return 0, or -1 with the failing index in *bad (token id out of range). */
int kllm_oracle_embedding(const float* table, int64_t vocab, int64_t hidden,
                          const int32_t* ids, int64_t n_tokens, float* out, int64_t* bad);
void kllm_oracle_rms_norm(const float* x, const float* weight, float* out, int64_t rows,
                          int64_t hidden, float eps);
void kllm_oracle_add_inplace(float* x, const float* y, int64_t n);
void kllm_oracle_add_bias_inplace(float* x, const float* bias, int64_t rows, int64_t cols);
void kllm_oracle_select_last_row(const float* x, int64_t rows, int64_t cols, float* out);
void kllm_oracle_matmul(const float* a, const float* b, float* out, int64_t m, int64_t n, int64_t k);
void kllm_oracle_silu_mul(const float* gate, const float* up, float* out, int64_t n);
void kllm_oracle_rope_inplace(float* x, int64_t seq, int64_t heads, int64_t head_dim,
                              int32_t past_len, float theta);
/* Return 0, or -1 when past_len + seq > max_seq (capacity). */
int kllm_oracle_copy_kv_to_cache(const float* k, const float* v, int64_t seq,
                                 int64_t kv_heads, int64_t head_dim, float* k_cache,
                                 float* v_cache, int64_t max_seq, int32_t past_len);
void kllm_oracle_dequantize_int8_f32(const int8_t* q, int64_t n, float scale, float* out);
void kllm_oracle_dequantize_int8_f16(const int8_t* q, int64_t n, float scale, uint16_t* out);

/* Batched / per-row-position compositions of the functions above. */
void kllm_oracle_add_rms_norm(float* residual, const float* delta, const float* weight,
                              float* out, int64_t rows, int64_t hidden, float eps);
/* Returns the number of tokens whose cache write was skipped (bad pos/slot). */
int64_t kllm_oracle_qkv_bias_rope_kv_append(
    float* q, const float* k, const float* v, const float* bq, const float* bk,
    const float* bv, const int32_t* positions, const int32_t* slots, int64_t n_tokens,
    int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float theta, float* k_cache,
    float* v_cache, int64_t n_slots, int64_t max_seq);
/* Returns 0, or -1 if an end index is outside [1, rows]. */
int kllm_oracle_select_last_rows(const float* x, int64_t rows, int64_t cols,
                                 const int32_t* seq_ends, int64_t seq_len, int64_t n_seqs,
                                 float* out);

/* Attention: the reference layout (caches [max_seq, kv_heads, head_dim]) and
 * the head-major cache [n_slots, kv_heads, max_seq, head_dim] with per-token
 * positions and slots (returns the number of tokens zeroed as invalid). */
void kllm_oracle_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                           int64_t seq, int32_t past_len, int64_t num_heads, int64_t num_kv_heads,
                           int64_t head_dim);
int64_t kllm_oracle_attention_head_major(const float* q, const float* k_cache, const float* v_cache,
                                         float* out, const int32_t* positions, const int32_t* slots,
                                         int64_t n_tokens, int64_t num_heads, int64_t num_kv_heads,
                                         int64_t head_dim, int64_t n_slots, int64_t max_seq);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_ORACLE_H_ */
