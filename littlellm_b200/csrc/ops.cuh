// ops.cuh — internal (C++) launchers behind the C ABI; the chain runner
// calls these directly with its own LaunchOpts (stream, PDL).
#pragma once

#include "common.cuh"

namespace kb {

int embedding(const void* table, int64_t vocab, int64_t hidden, int table_dtype, const int32_t* ids,
              int64_t n_tokens, void* out, int out_dtype, int32_t* err_flags, const LaunchOpts& o);

int add_rms_norm(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                 int64_t hidden, float eps, int act_dtype, int weight_dtype, const LaunchOpts& o);

// add_rms_norm (fp16 rows) that also copies the last row of each of n_seqs
// sequences of seq_len rows to last_rows (select_last_rows fused into the
// final norm); two launches where the fast path does not apply.
int add_rms_norm_last_rows(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                           int64_t hidden, float eps, int weight_dtype, void* last_rows, int64_t seq_len,
                           int64_t n_seqs, int32_t* err_flags, const LaunchOpts& o, int* n_launched);

// residual = table[ids] (fp16 rows, bit-exact) and out = rms_norm(residual) * weight in one launch
// (embedding + layer 0's input norm).
int embedding_rms_norm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n_tokens,
                       const void* weight, int weight_dtype, float eps, void* residual, void* out,
                       int32_t* err_flags, const LaunchOpts& o);

int silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype, const LaunchOpts& o);

int add_inplace(void* x, const void* y, int64_t n, int x_dtype, int y_dtype, const LaunchOpts& o);

int add_bias_inplace(void* x, const void* bias, int64_t rows, int64_t cols, int x_dtype, int bias_dtype,
                     const LaunchOpts& o);

int qkv_bias_rope_kv_append(void* q, const void* k, const void* v, const void* bq, const void* bk,
                            const void* bv, int bias_dtype, const int32_t* positions, const int32_t* slots,
                            int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                            float theta, void* k_cache, void* v_cache, int64_t n_slots, int64_t max_seq,
                            int32_t* err_flags, const LaunchOpts& o);

// RoPE frequency table inv_freq[d] = theta^(-2d / head_dim), d < head_dim / 2
// (host, fp32; shared by every RoPE path).
void rope_inv_freq(float* inv_freq, int head_dim, float theta);

int dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n, int out_dtype,
                    const LaunchOpts& o);

// The same with the scale passed by value (host-side scale, e.g. read from a file).
int dequantize_int8_value(const int8_t* data, float scale, void* out, int64_t n, int out_dtype,
                          const LaunchOpts& o);

int dequantize_int8_rne(const int8_t* data, const float* scale, void* out, int64_t n,
                        unsigned long long* mismatches, const LaunchOpts& o);

int select_last_rows(const void* x, int64_t rows, int64_t cols, const int32_t* seq_ends, int64_t seq_len,
                     int64_t n_seqs, void* out, int dtype, int32_t* err_flags, const LaunchOpts& o);

// out = fp16(fp16(x . w^T) + bias) on tcgen05 (gemm.cu).
int linear(const void* x, const void* w, const void* bias, int bias_dtype, void* out, int64_t m, int64_t n,
           int64_t k, int32_t* err_flags, const LaunchOpts& o);

// out = silu_mul(linear(x, w_gate, b_gate), linear(x, w_up, b_up)) in one kernel (gemm.cu).
int linear_swiglu(const void* x, const void* w_gate, const void* w_up, const void* b_gate, const void* b_up,
                  int bias_dtype, void* out, int64_t m, int64_t n, int64_t k, int32_t* err_flags,
                  const LaunchOpts& o);

// q, k, v = x . wq^T, wk^T, wv^T as one tcgen05 GEMM whose epilogue adds the
// biases, applies RoPE to q and k and appends k and v to the head-major
// caches: linear x3 + qkv_bias_rope_kv_append in one kernel (gemm.cu).
int qkv_linear_rope_kv_append(const void* x, const void* wq, const void* wk, const void* wv, const void* bq,
                              const void* bk, const void* bv, int bias_dtype, const int32_t* positions,
                              const int32_t* slots, int64_t n_tokens, int64_t hidden, int64_t n_heads,
                              int64_t n_kv_heads, int64_t head_dim, float theta, void* q_out, void* k_cache,
                              void* v_cache, int64_t n_slots, int64_t max_seq, int32_t* err_flags,
                              const LaunchOpts& o);

int attention_workspace_bytes(int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                              int64_t max_seq, int64_t* bytes);

int attention_head_major(const void* q, const void* k_cache, const void* v_cache, void* out,
                         const int32_t* positions, const int32_t* slots, int64_t n_tokens, int64_t seq_len,
                         int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t n_slots, int64_t max_seq,
                         int dtype, void* workspace, int64_t workspace_bytes, int32_t* err_flags,
                         const LaunchOpts& o, int* n_launched = nullptr);

}  // namespace kb
