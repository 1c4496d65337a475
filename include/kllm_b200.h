/*
 * kllm_b200.h — C ABI of the B200 (sm_100a) backend for LittleLLM's non-GEMM
 * decoder-layer operators.
 *
 * Every entry point takes plain device pointers, element counts, scalar
 * parameters and a CUDA stream handle (passed as `void*`; NULL means the
 * legacy default stream, which is what the reference backend uses). Nothing
 * here allocates device memory, synchronises the host, or keeps per-call
 * state: every call is stream-ordered and re-entrant.
 *
 * Return value: KLLM_B200_OK (0) or a negative KLLM_B200_ERR_* code. The text
 * of the most recent failure on the calling thread is returned by
 * kllm_b200_last_error(). A C++ caller turns a non-zero code into
 * std::runtime_error, the same convention the reference uses for CUDA errors
 * (include/kllm/op/detail/cuda_helpers.cuh:11-15).
 *
 * Element types use the reference's DType numbering
 * (include/kllm/base/tensor.h:13-18): F32 = 0, F16 = 1, I32 = 2, I8 = 3.
 *
 * Values that only the device can check (token ids, positions, cache slots
 * held in device memory) are checked in the kernel: an offending row is
 * skipped (embedding rows are zero-filled) and, when the caller passes a
 * device word `err_flags`, the matching KLLM_B200_FLAG_* bit is OR-ed into it.
 * No kernel traps, asserts or spins.
 */
#ifndef KLLM_B200_H_
#define KLLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element types (reference DType, include/kllm/base/tensor.h:13-18) ---- */
enum {
  KLLM_B200_F32 = 0,
  KLLM_B200_F16 = 1,
  KLLM_B200_I32 = 2,
  KLLM_B200_I8 = 3
};

/* ---- status codes ---- */
enum {
  KLLM_B200_OK = 0,
  KLLM_B200_ERR_INVALID_ARG = -1, /* null pointer where one is required, negative size */
  KLLM_B200_ERR_SHAPE = -2,       /* inconsistent or unsupported shape */
  KLLM_B200_ERR_DTYPE = -3,       /* unsupported element-type combination */
  KLLM_B200_ERR_ALIGN = -4,       /* pointer alignment a kernel requires is not met */
  KLLM_B200_ERR_RANGE = -5,       /* host-visible id / position out of range */
  KLLM_B200_ERR_CAPACITY = -6,    /* KV cache capacity exceeded */
  KLLM_B200_ERR_CUDA = -7,        /* CUDA runtime / launch error */
  KLLM_B200_ERR_IO = -8,          /* file open / read error */
  KLLM_B200_ERR_FORMAT = -9       /* malformed .kllm file */
};

/* ---- bits OR-ed into the optional device word `err_flags` ---- */
enum {
  KLLM_B200_FLAG_BAD_TOKEN = 1,    /* embedding id outside [0, vocab) */
  KLLM_B200_FLAG_BAD_POSITION = 2, /* RoPE/KV position outside [0, max_seq) */
  KLLM_B200_FLAG_BAD_SLOT = 4,     /* KV cache slot outside [0, n_slots) */
  KLLM_B200_FLAG_BAD_SEQ_END = 8,  /* select_last_rows end index outside [1, rows] */
  KLLM_B200_FLAG_TIMEOUT = 16      /* a kernel's bounded wait on its tensor-core work ran out;
                                      that launch's outputs are incomplete */
};

/* Copies the calling thread's most recent error message into buf (always
 * NUL-terminated when len > 0). Returns the full message length. */
size_t kllm_b200_last_error(char* buf, size_t len);

/* Static text for a status code. */
const char* kllm_b200_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int kllm_b200_version(void);

/* Launch mode of the individual operator entry points, for the calling host
 * thread (default off; kllm_b200_chain_run follows its descriptor's use_pdl
 * instead, and the .kllm loader and the no-allocation dequant never use it).
 * With enable != 0 the entry points launch with programmatic dependent launch:
 * a kernel's CTAs may be scheduled while the previous kernel on the stream
 * drains, and they wait for it to complete (griddepcontrol.wait) before their
 * first global read (before it they only ask L2 to prefetch, a hint that
 * returns no data), so the mode is correct whatever the previous kernel
 * wrote. (Only kllm_b200_chain_run, which knows what each of its launches
 * writes, also reads weights, biases, positions, slots, tables and ids before
 * that wait.) A runner that calls the operators one by one (the C++ binding
 * of LittleLLM's kllm::op::cuda_*) overlaps each operator's launch and
 * scheduling with its predecessor's tail. Returns the previous mode. No
 * reference counterpart (launch configuration only). */
int kllm_b200_set_pdl(int enable);

/* ======================================================================== *
 *  Reference-compatible operators (same semantics as kllm::op::cuda_*)      *
 * ======================================================================== */

/* out[t, :] = table[ids[t], :].
 * Replaces cuda_embedding (src/op/cuda/embedding.cu:83-108); the reference
 * copies host ids with a blocking cudaMemcpy on every call, here `ids` is
 * already a device array of n_tokens int32. table_dtype/out_dtype in {F32,F16};
 * equal dtypes are a bit-exact copy, mixed dtypes convert (F32->F16 rounds to
 * nearest even, like the reference kernel's __float2half). Ids outside
 * [0, vocab) zero-fill the row and set KLLM_B200_FLAG_BAD_TOKEN. */
int kllm_b200_embedding(const void* table, int64_t vocab, int64_t hidden, int table_dtype,
                        const int32_t* ids, int64_t n_tokens, void* out, int out_dtype,
                        int32_t* err_flags, void* stream);

/* kllm_b200_embedding with the ids in HOST memory, as cuda_embedding takes
 * them (a std::vector<int>, src/op/cuda/embedding.cu:83-108). The ids travel
 * inside the kernel launches' parameters (up to KLLM_B200_PARAM_IDS per
 * launch; longer lists take several launches), so there is no device
 * buffer, no allocation and no blocking copy: the call returns once the
 * launches are enqueued and host_ids may be reused at once. Same copy
 * semantics, flags and dtypes as kllm_b200_embedding. */
#define KLLM_B200_PARAM_IDS 7680
int kllm_b200_embedding_host_ids(const void* table, int64_t vocab, int64_t hidden, int table_dtype,
                                 const int32_t* host_ids, int64_t n_tokens, void* out, int out_dtype,
                                 int32_t* err_flags, void* stream);

/* out = x * (mean(x^2) + eps)^-1/2 * weight, per row of `hidden` elements.
 * Replaces cuda_rms_norm (src/op/cuda/rms_norm.cu:177-188). x/out share
 * act_dtype in {F32,F16}; weight_dtype in {F32,F16}; fp32 accumulation. */
int kllm_b200_rms_norm(const void* x, const void* weight, void* out, int64_t rows,
                       int64_t hidden, float eps, int act_dtype, int weight_dtype,
                       void* stream);

/* x[i] += y[i] for n elements (add_inplace, src/op/cuda/add.cu:71-76).
 * x_dtype, y_dtype in {F32,F16}. */
int kllm_b200_add_inplace(void* x, const void* y, int64_t n, int x_dtype, int y_dtype,
                          void* stream);

/* x[r, c] += bias[c] for a [rows, cols] matrix (add_bias_inplace,
 * src/op/cuda/add.cu:59-69). A NULL bias is a no-op, as in the reference. */
int kllm_b200_add_bias_inplace(void* x, const void* bias, int64_t rows, int64_t cols,
                               int x_dtype, int bias_dtype, void* stream);

/* out[0, :] = x[rows-1, :] (select_last_row, src/op/cuda/add.cu:78-84). */
int kllm_b200_select_last_row(const void* x, int64_t rows, int64_t cols, void* out,
                              int dtype, void* stream);

/* out = silu(gate) * up = gate * sigmoid(gate) * up, n elements
 * (silu_mul, src/op/cuda/silu.cu:30-36). All three share dtype in {F32,F16}. */
int kllm_b200_silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype,
                       void* stream);

/* Rotate-half RoPE in place on x[seq, heads, head_dim] at positions
 * past_len + t, angle = pos * theta^(-2d/head_dim)
 * (rope_inplace, src/op/cuda/rope.cu:188-201). head_dim must be even. */
int kllm_b200_rope_inplace(void* x, int64_t seq, int64_t heads, int64_t head_dim,
                           int32_t past_len, float theta, int dtype, void* stream);

/* k_cache[past_len + t, :, :] = k[t, :, :], same for v, with caches laid out
 * [max_seq, kv_heads, head_dim] (copy_kv_to_cache,
 * src/op/cuda/kv_cache.cu:32-41). Fails with KLLM_B200_ERR_CAPACITY when
 * past_len + seq > max_seq, as the reference CPU path does
 * (src/op/cpu/kv_cache.cpp:19-21). One launch covers K and V. */
int kllm_b200_copy_kv_to_cache(const void* k, const void* v, int64_t seq, int64_t kv_heads,
                               int64_t head_dim, void* k_cache, void* v_cache,
                               int64_t max_seq, int32_t past_len, int src_dtype,
                               int cache_dtype, void* stream);

/* INT8 per-tensor dequantisation: out[i] = q[i] * scale[0].
 *  - out_dtype F32: the reference GPU op (src/op/cuda/quantize.cu:110-121).
 *  - out_dtype F16: the reference weight-load path
 *    (src/model/weights.cpp:139-148): the product is formed in fp32 and
 *    rounded with the reference's own float_to_half (src/base/half.cpp:38-61),
 *    bit for bit, including its tie and carry behaviour.
 * `scale` points to one float in device memory. */
int kllm_b200_dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n,
                              int out_dtype, void* stream);

/* Opt-in IEEE rounding of the INT8 -> fp16 dequant: out[i] is
 * float(data[i]) * scale[0] rounded to nearest even (__float2half_rn)
 * instead of by the reference loader's float_to_half (src/base/half.cpp:
 * 38-61, which rounds ties away from zero and drops a carry into an odd
 * exponent). If `mismatches` (a device uint64) is given, the number of
 * elements where the two roundings differ is ADDED to it; zero it first.
 * Same alignment rules and fast path as kllm_b200_dequantize_int8. */
int kllm_b200_dequantize_int8_rne(const int8_t* data, const float* scale, void* out, int64_t n,
                                  unsigned long long* mismatches, void* stream);

/* ======================================================================== *
 *  Fused / batched operators (additive to include/kllm/op/ops.h)           *
 * ======================================================================== */

/* Many INT8 tensors in one launch: for each i, outs[i][j] = data[i][j] *
 * scales[i][0], rounded exactly as kllm_b200_dequantize_int8 rounds for
 * out_dtype. This is the dequant step of the weight loader
 * (src/model/weights.cpp:95-154, which dequantises record by record on the
 * host) applied to a whole checkpoint on the device. data/scales/outs/counts
 * are HOST arrays of n_tensors entries holding device pointers and element
 * counts; they are read during the call only. Tensors whose data or output
 * is not 16-byte aligned are dequantised by single-tensor launches. */
int kllm_b200_dequantize_int8_batched(const int8_t* const* data, const float* const* scales,
                                      void* const* outs, const int64_t* counts, int n_tensors,
                                      int out_dtype, void* stream);

/* Residual add fused with RMSNorm, the pair at src/model/llama.cpp:135-143
 * (and :166 -> :83 across layers, :176 at the end):
 *     residual[r, :] = fp16(residual[r, :] + delta[r, :])   (stored)
 *     out[r, :]      = residual[r, :] * (mean(residual^2) + eps)^-1/2 * weight
 * The norm reads the stored (rounded) residual, exactly as the reference's
 * separate add_inplace then rms_norm do. delta == NULL gives a plain RMSNorm
 * of `residual` (left unmodified). act_dtype in {F32,F16}. */
int kllm_b200_add_rms_norm(void* residual, const void* delta, const void* weight, void* out,
                           int64_t rows, int64_t hidden, float eps, int act_dtype,
                           int weight_dtype, void* stream);

/* The embedding gather fused with the RMSNorm that reads it (layer 0's input
 * norm): src/model/llama.cpp:84 (cuda_embedding) and :83-87 of the first
 * layer (cuda_rms_norm), in one launch:
 *     residual_out[t, :] = table[ids[t], :]                (bit-exact copy)
 *     norm_out[t, :]     = rms_norm(residual_out[t, :]) * weight
 * fp16 table and outputs; weight_dtype in {F32,F16}; ids a device array.
 * Bit-identical to kllm_b200_embedding followed by kllm_b200_rms_norm; the
 * gathered rows are not re-read from HBM. Ids outside [0, vocab) give zero
 * rows (both outputs) and set KLLM_B200_FLAG_BAD_TOKEN. */
int kllm_b200_embedding_rms_norm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids,
                                 int64_t n_tokens, const void* weight, int weight_dtype, float eps,
                                 void* residual_out, void* norm_out, int32_t* err_flags, void* stream);

/* q/k/v bias add + rotate-half RoPE + KV-cache append, one launch.
 * Replaces, per layer, add_bias_inplace x3 (src/model/llama.cpp:89-106 via
 * :22), rope_inplace x2 (:111-112) and copy_kv_to_cache (:114).
 *   q  [n_tokens, n_heads,    head_dim] fp16, rotated in place (after +bq)
 *   k  [n_tokens, n_kv_heads, head_dim] fp16, read only
 *   v  [n_tokens, n_kv_heads, head_dim] fp16, read only
 *   bq/bk/bv: [heads*head_dim] biases of bias_dtype (F32/F16), each may be NULL
 *   positions[t], slots[t]: device int32 per token (position in its sequence,
 *       sequence slot in the cache)
 *   k_cache, v_cache: this layer's planes, [n_slots, n_kv_heads, max_seq,
 *       head_dim] fp16 (the [layer, k/v, slot, kv_head, max_seq, head_dim]
 *       cache indexed at one layer).
 * Written: q (rotated), k_cache[slot, h, pos, :] = rope(k + bk),
 * v_cache[slot, h, pos, :] = fp16(v + bv). The biased values are rounded to
 * fp16 before the rotation, as the reference's separate bias-add writes them.
 * Tokens with an out-of-range position or slot skip the cache write and set
 * KLLM_B200_FLAG_BAD_POSITION / _BAD_SLOT in *err_flags (if given).
 * head_dim must be even and at most 256. */
int kllm_b200_qkv_bias_rope_kv_append(void* q, const void* k, const void* v, const void* bq,
                                      const void* bk, const void* bv, int bias_dtype,
                                      const int32_t* positions, const int32_t* slots,
                                      int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads,
                                      int64_t head_dim, float theta, void* k_cache,
                                      void* v_cache, int64_t n_slots, int64_t max_seq,
                                      int32_t* err_flags, void* stream);

/* Batched select_last_row (src/op/cuda/add.cu:78-84, called at
 * src/model/llama.cpp:178): out[b, :] = x[end_b - 1, :] with
 * end_b = seq_ends[b] when seq_ends (device int32[n_seqs]) is given, else
 * end_b = (b + 1) * seq_len. Out-of-range ends zero-fill the row and set
 * KLLM_B200_FLAG_BAD_SEQ_END. */
int kllm_b200_select_last_rows(const void* x, int64_t rows, int64_t cols,
                               const int32_t* seq_ends, int64_t seq_len, int64_t n_seqs,
                               void* out, int dtype, int32_t* err_flags, void* stream);

/* Attention over the head-major cache (replaces cuda_attention,
 * src/op/cuda/attention.cu:224-263, for a runner that keeps the cache
 * [n_slots, n_kv_heads, max_seq, head_dim] per layer that
 * kllm_b200_qkv_bias_rope_kv_append fills). For token t and query head h:
 * out[t, h, :] = sum_j p_j * v_cache[slots[t], h / G, j, :] over positions
 * j = 0..positions[t], with p = softmax_j(q[t, h, :] . k_cache[slots[t], h / G,
 * j, :] / sqrt(head_dim)) and G = n_heads / n_kv_heads, as cpu_attention
 * (src/op/cpu/attention.cpp:12-67) computes it with past_len + t equal to
 * positions[t]. q and out are [n_tokens, n_heads, head_dim]. F16 only;
 * head_dim 64 or 128; G <= 16. seq_len: tokens arrive in runs of seq_len
 * consecutive rows of one sequence (1 for decode); it selects the kernel,
 * and the rows of one run must then share a slot. A token whose position
 * or slot is out of range gets zero rows and sets KLLM_B200_FLAG_BAD_POSITION
 * / _BAD_SLOT. workspace (device, 16-byte aligned) holds split-sequence
 * partials; kllm_b200_attention_workspace_bytes gives the size for the best
 * split, and a smaller (or NULL) workspace gives coarser splits with the
 * same results. Nothing is allocated; the workspace needs no clearing, and
 * calls sharing one workspace must not overlap on the GPU. */
int kllm_b200_attention_workspace_bytes(int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads,
                                        int64_t head_dim, int64_t max_seq, int64_t* bytes);
int kllm_b200_attention_head_major(const void* q, const void* k_cache, const void* v_cache,
                                   void* out, const int32_t* positions, const int32_t* slots,
                                   int64_t n_tokens, int64_t seq_len, int64_t n_heads,
                                   int64_t n_kv_heads, int64_t head_dim, int64_t n_slots,
                                   int64_t max_seq, int dtype, void* workspace,
                                   int64_t workspace_bytes, int32_t* err_flags, void* stream);

/* ======================================================================== *
 *  GEMM with fused epilogues (tcgen05)                                      *
 * ======================================================================== */

/* linear() of src/model/llama.cpp:12-24, i.e. matmul (cuda_matmul,
 * src/op/cuda/matmul.cu:130-160; cpu_matmul, src/op/cpu/matmul.cpp:9-33)
 * followed by add_bias_inplace (src/op/cuda/add.cu:59-69), in one kernel:
 * out[i, j] = fp16(fp16(sum_c x[i, c] * w[j, c]) + bias[j]), fp32
 * accumulation, both roundings to nearest even. x [m, k], w [n, k] and
 * out [m, n] are fp16, row-major, 16-byte aligned; k must be a positive
 * multiple of 8. bias (F16 or F32, 4-byte aligned) may be NULL (plain
 * matmul). out must not overlap x or w. A bounded wait that runs out inside
 * the kernel sets KLLM_B200_FLAG_TIMEOUT in err_flags (optional). */
int kllm_b200_linear(const void* x, const void* w, const void* bias, int bias_dtype, void* out,
                     int64_t m, int64_t n, int64_t k, int32_t* err_flags, void* stream);

/* The MLP's gate and up linears and silu_mul (src/model/llama.cpp:145-158)
 * in one kernel: out = silu_mul(linear(x, w_gate, b_gate),
 * linear(x, w_up, b_up)), with the gate and up values rounded to fp16
 * (plus bias, rounded again) exactly as the separate ops store them, then
 * silu(g) * u in fp32 rounded to fp16 as kllm_b200_silu_mul computes it.
 * w_gate and w_up are [n, k] (n = intermediate size); out is [m, n]; the
 * biases share bias_dtype and may each be NULL. Gate and up never reach
 * memory. Same requirements and error flag as kllm_b200_linear. */
int kllm_b200_linear_swiglu(const void* x, const void* w_gate, const void* w_up,
                            const void* b_gate, const void* b_up, int bias_dtype, void* out,
                            int64_t m, int64_t n, int64_t k, int32_t* err_flags, void* stream);

/* The attention block's projections and their epilogue in one kernel: q, k,
 * v = x . wq^T, x . wk^T, x . wv^T (linear() x3, src/model/llama.cpp:89-106),
 * then the work of kllm_b200_qkv_bias_rope_kv_append on them (bias, RoPE of
 * q and k at positions[t], k and v appended to the head-major caches
 * [n_slots, n_kv_heads, max_seq, head_dim] at slot slots[t]), bit for bit
 * as those separate calls compute it. q_out is [n_tokens, n_heads*head_dim];
 * k and v are never written elsewhere. x [n_tokens, hidden], wq
 * [n_heads*head_dim, hidden], wk and wv [n_kv_heads*head_dim, hidden], fp16,
 * 16-byte aligned; hidden a multiple of 8; head_dim 64 or 128. Out-of-range
 * positions or slots skip the token's cache rows and set
 * KLLM_B200_FLAG_BAD_POSITION / _BAD_SLOT. */
int kllm_b200_qkv_linear_rope_kv_append(const void* x, const void* wq, const void* wk, const void* wv,
                                        const void* bq, const void* bk, const void* bv, int bias_dtype,
                                        const int32_t* positions, const int32_t* slots, int64_t n_tokens,
                                        int64_t hidden, int64_t n_heads, int64_t n_kv_heads,
                                        int64_t head_dim, float theta, void* q_out, void* k_cache,
                                        void* v_cache, int64_t n_slots, int64_t max_seq,
                                        int32_t* err_flags, void* stream);

/* ======================================================================== *
 *  Layer-op chain executor                                                  *
 * ======================================================================== */

/* Per-layer buffers of the non-GEMM chain of LlamaRunner::forward
 * (src/model/llama.cpp:81-168). The GEMM outputs (q, k, v, attn_out, gate,
 * up, ffn_out) are inputs here; the norm / SwiGLU outputs feed the GEMMs. */
typedef struct kllm_b200_layer_buffers {
  void* q;                   /* [T, n_heads*head_dim] fp16, rotated in place */
  const void* k;             /* [T, n_kv_heads*head_dim] fp16 */
  const void* v;             /* [T, n_kv_heads*head_dim] fp16 */
  const void* q_bias;        /* [n_heads*head_dim] or NULL */
  const void* k_bias;        /* [n_kv_heads*head_dim] or NULL */
  const void* v_bias;        /* [n_kv_heads*head_dim] or NULL */
  const void* attn_out;      /* [T, hidden] o_proj output */
  const void* ffn_out;       /* [T, hidden] down_proj output */
  const void* gate;          /* [T, intermediate] */
  const void* up;            /* [T, intermediate] */
  const void* input_norm_w;  /* [hidden] */
  const void* post_norm_w;   /* [hidden] */
  void* attn_norm_out;       /* [T, hidden] */
  void* ffn_norm_out;        /* [T, hidden] */
  void* swiglu_out;          /* [T, intermediate] */
  void* k_cache;             /* [n_slots, n_kv_heads, max_seq, head_dim] */
  void* v_cache;             /* [n_slots, n_kv_heads, max_seq, head_dim] */
  void* attn_ctx;            /* [T, n_heads*head_dim] attention output (KLLM_B200_OP_ATTENTION) or NULL */
} kllm_b200_layer_buffers;

/* Per-layer weights of the GEMMs (KLLM_B200_OP_GEMM): fp16, [out, in]
 * row-major as linear() takes them (src/model/llama.cpp:12-24). Biases are
 * of the chain's weight_dtype and may be NULL; the q/k/v biases stay in
 * kllm_b200_layer_buffers (the fused RoPE op adds them). */
typedef struct kllm_b200_layer_weights {
  const void* wq;        /* [n_heads*head_dim, hidden] */
  const void* wk;        /* [n_kv_heads*head_dim, hidden] */
  const void* wv;        /* [n_kv_heads*head_dim, hidden] */
  const void* wo;        /* [hidden, n_heads*head_dim] */
  const void* w_gate;    /* [intermediate, hidden] */
  const void* w_up;      /* [intermediate, hidden] */
  const void* w_down;    /* [hidden, intermediate] */
  const void* o_bias;    /* [hidden] or NULL */
  const void* gate_bias; /* [intermediate] or NULL */
  const void* up_bias;   /* [intermediate] or NULL */
  const void* down_bias; /* [hidden] or NULL */
} kllm_b200_layer_weights;

/* op_mask bits of kllm_b200_chain */
enum {
  KLLM_B200_OP_EMBEDDING = 1,
  KLLM_B200_OP_INPUT_NORM = 2,  /* per layer: residual add (from layer 1) + RMSNorm */
  KLLM_B200_OP_QKV_ROPE = 4,    /* per layer: bias + RoPE + KV append */
  KLLM_B200_OP_POST_NORM = 8,   /* per layer: residual add + RMSNorm */
  KLLM_B200_OP_SWIGLU = 16,     /* per layer */
  KLLM_B200_OP_FINAL_NORM = 32,
  KLLM_B200_OP_SELECT = 64,
  /* per layer, after the RoPE/KV append: attention of q over the layer's
   * cache into attn_ctx (kllm_b200_attention_head_major; runs of seq_len
   * tokens, or single tokens when seq_ends is given). Not in op_mask 0:
   * the GEMM-free chain of the seven ops above stays the default. */
  KLLM_B200_OP_ATTENTION = 128,
  /* the GEMMs too, making the chain the whole forward step of
   * LlamaRunner::forward (src/model/llama.cpp:78-184): per layer the q, k
   * and v linears after the input norm with the bias + RoPE + KV append in
   * their epilogue (kllm_b200_qkv_linear_rope_kv_append: q rotated into q,
   * k and v straight into the caches), the o linear after
   * attention (into attn_out), the gate/up linears with SwiGLU fused (into
   * swiglu_out; replaces KLLM_B200_OP_SWIGLU's silu_mul), the down linear
   * (into ffn_out); after select, logits = last_rows . lm_head^T when
   * lm_head and logits are given. Needs KLLM_B200_OP_ATTENTION and weights. */
  KLLM_B200_OP_GEMM = 256
};

typedef struct kllm_b200_chain {
  int64_t n_tokens, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  int64_t n_layers, n_slots, max_seq, n_seqs, seq_len;
  float eps, theta;
  int weight_dtype;               /* F16 or F32 for norm weights and biases */
  int use_pdl;                    /* launch with programmatic dependent launch */
  int op_mask;                    /* 0 = the whole chain; else only the KLLM_B200_OP_* bits set
                                     (profiling: one op kind timed in chain context) */
  const void* embed_table;        /* [vocab, hidden] fp16 */
  const int32_t* ids;             /* [T] device */
  const int32_t* positions;       /* [T] device */
  const int32_t* slots;           /* [T] device */
  const int32_t* seq_ends;        /* [n_seqs] device, or NULL for uniform seq_len */
  void* residual;                 /* [T, hidden] fp16 running residual stream */
  const void* final_norm_w;       /* [hidden] */
  void* final_norm_out;           /* [T, hidden] */
  void* last_rows;                /* [n_seqs, hidden] */
  const kllm_b200_layer_buffers* layers; /* host array of n_layers entries */
  int32_t* err_flags;             /* device word or NULL */
  void* attn_workspace;           /* attention split workspace (KLLM_B200_OP_ATTENTION), or NULL */
  int64_t attn_workspace_bytes;
  const kllm_b200_layer_weights* weights; /* host array of n_layers entries (KLLM_B200_OP_GEMM) */
  const void* lm_head;            /* [vocab, hidden] fp16, or NULL */
  void* logits;                   /* [n_seqs, vocab] fp16, or NULL */
} kllm_b200_chain;

/* Launches the whole non-GEMM chain on `stream`: embedding, then per layer
 * add+RMSNorm, fused bias+RoPE+KV append, (attention, when its bit is set),
 * add+RMSNorm, SwiGLU, then the final add+RMSNorm and select_last_rows (the
 * op kinds selected by op_mask; 0 selects the seven ops without attention).
 * With KLLM_B200_OP_GEMM the layer's GEMMs run in between and the step is
 * the whole forward: q, attn_out and ffn_out are then written (k and v go
 * straight into the caches).
 * When both the embedding and the input norm run, they are one kernel
 * (kllm_b200_embedding_rms_norm for layer 0); when both the final norm and
 * select run and seq_ends is NULL, the final norm's kernel writes the last
 * rows. With use_pdl, every launch after the chain's first reads the inputs
 * that no launch of the chain writes (norm weights, q/k/v biases, positions,
 * slots, the embedding table and ids) before its grid-dependency wait, and an
 * add+RMSNorm whose previous launch left the residual alone reads the
 * residual rows there too (they were written two or more launches back, and
 * this library's kernels trigger their dependents only after their own wait).
 * The chain's first launch reads nothing before its wait, so the caller's
 * launch before chain_run may write any of the chain's inputs.
 * *n_launches (if given) receives the number of kernels launched. Can be
 * captured into a CUDA graph. */
int kllm_b200_chain_run(const kllm_b200_chain* chain, int* n_launches, void* stream);

/* ======================================================================== *
 *  .kllm weight files: index + streaming load with device-side dequant      *
 * ======================================================================== */

/* Model config of a .kllm file header (read by src/model/weights.cpp:65-79). */
typedef struct kllm_b200_kllm_config {
  uint32_t model_type; /* 0 llama, 1 qwen2 */
  int32_t vocab_size, hidden_size, intermediate_size, num_layers, num_heads, num_kv_heads;
  int32_t head_dim, max_seq_len;
  float rms_norm_eps, rope_theta;
  uint8_t tie_word_embeddings, qkv_bias, o_bias, mlp_bias;
} kllm_b200_kllm_config;

/* One tensor record of a .kllm file (src/model/weights.cpp:81-118). */
typedef struct kllm_b200_kllm_record {
  char name[192];
  int32_t dtype;        /* as stored: F32, F16, I32 or I8 */
  int32_t ndim;
  int64_t dims[8];
  int64_t numel;
  uint64_t data_offset; /* file offset of the record's bytes */
  uint64_t nbytes;      /* stored bytes; I8 records: numel int8 values + one fp32 scale */
  int32_t load_dtype;   /* dtype of the device tensor: I8 -> F16 (the reference's CUDA
                           load type, src/model/weights.cpp:122), others as stored */
  int32_t reserved;
  int64_t load_bytes;   /* bytes of the device tensor */
} kllm_b200_kllm_record;

/* Parses the header and record table of a .kllm file (magic "KLLM0001",
 * version 1) with the checks of ModelWeights::load (src/model/weights.cpp:
 * 47-118): magic, version, byte counts per dtype. Writes up to max_records
 * entries and the total count to *n_records (so a first call with
 * max_records = 0 sizes the array). Host only; no CUDA calls. */
int kllm_b200_kllm_read_index(const char* path, kllm_b200_kllm_config* config,
                              kllm_b200_kllm_record* records, int max_records, int* n_records);

/* Streams records into caller-allocated device tensors dst[i]
 * (records[i].load_bytes each): F32/F16/I32 records are copied as stored;
 * I8 records are copied to the device and dequantised there to fp16 with the
 * rounding of the reference loader (src/model/weights.cpp:120-154), bit for
 * bit. host_staging (pinned host memory, >= 64 KB) is used as two halves so
 * file reads overlap the copies; dev_staging (device memory, needed only
 * for I8 records, >= 64 KB) holds int8 chunks before dequant. Returns after
 * the stream has finished all copies and kernels of the call. */
int kllm_b200_kllm_load(const char* path, const kllm_b200_kllm_record* records, int n_records,
                        void* const* dst, void* host_staging, size_t host_staging_bytes,
                        void* dev_staging, size_t dev_staging_bytes, void* stream);

/* ======================================================================== *
 *  No device allocation                                                     *
 * ======================================================================== */

/* out[i] = host_data[i] * scale for n INT8 values that live in HOST memory,
 * with no device memory allocated anywhere: the int8 bytes are staged in a
 * 32 MiB device array built into the library (the staged dequant of
 * kllm_b200_kllm_load, which instead stages in device memory the caller
 * allocates). For callers that cannot call cudaMalloc, e.g. a plugin handed
 * only output buffers by its host application. Rounding as
 * kllm_b200_dequantize_int8 for out_dtype (F16: the reference loader's
 * float_to_half, bit for bit). n above 33554432 (32 MiB) fails with
 * KLLM_B200_ERR_CAPACITY before any GPU work. The array's device address
 * belongs to the CUDA context current at the call, so every call looks it up
 * (cudaGetSymbolAddress) in that context; the first call in a context loads
 * the library's module there. All calls share the array, so calls
 * that overlap on the GPU race; run them in one stream order. host_data must
 * not change until the stream has passed the copy (pinned memory is read
 * asynchronously). This entry point has no counterpart in the reference. */
int kllm_b200_dequantize_int8_host_static(const int8_t* host_data, float scale, void* out,
                                          int64_t n, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_B200_H_ */
