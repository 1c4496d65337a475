// chain.cu — the non-GEMM op chain of one forward step, launched natively.
//
// Mirrors the op order of LlamaRunner::forward (src/model/llama.cpp:78-178)
// with the GEMM outputs supplied as inputs:
//   embedding                               (llama.cpp:79)
//   per layer l:
//     add+RMSNorm  r += ffn_out[l-1]; attn_norm = norm(r)   (l=0: norm only; :83-87, :166)
//                  (the embedding and layer 0's norm are one kernel when both run)
//     bias+RoPE+KV q/k/v -> q rotated, cache[l] appended    (:89-114)
//     [attention   ctx = attn(q, cache[l]), when requested]  (:116-126)
//     add+RMSNorm  r += attn_out[l]; ffn_norm = norm(r)      (:135-143)
//     SwiGLU       swiglu = silu(gate) * up                  (:158)
//   add+RMSNorm  r += ffn_out[L-1]; normed = norm(r)         (:166, :171)
//   select_last_rows                                          (:173)
//                (written by the final norm's kernel when all sequences have seq_len rows)
// With KLLM_B200_OP_GEMM the GEMMs run in between (tcgen05, gemm.cu), and the
// step is the whole forward of llama.cpp:78-184:
//   after the input norm   q, k, v = linear(attn_norm, wq / wk / wv)   (:89-106), with
//                          bias + RoPE + KV append in the same kernel   (:108-114)
//   after attention        attn_out = linear(ctx, wo, o_bias)          (:129-134)
//   instead of SwiGLU      swiglu = silu_mul(linear(ffn_norm, w_gate), linear(ffn_norm, w_up)),
//                          one kernel                                   (:145-158)
//   then                   ffn_out = linear(swiglu, w_down, down_bias)  (:160-165)
//   after select           logits = linear(last_rows, lm_head)          (:175-183)
// Everything goes to one stream; with use_pdl every launch carries the
// programmatic-dependent-launch attribute so a kernel's CTAs are scheduled
// while its predecessor drains. The sequence contains no host sync and no
// allocation, so it can be captured into a CUDA graph.
#include "ops.cuh"

extern "C" int kllm_b200_chain_run(const kllm_b200_chain* c, int* n_launches, void* stream) {
  using namespace kb;
  if (n_launches) *n_launches = 0;
  if (c == nullptr || c->layers == nullptr) return fail(KLLM_B200_ERR_INVALID_ARG, "chain_run: null chain");
  if (c->n_tokens <= 0 || c->hidden <= 0 || c->n_layers <= 0 || c->n_seqs <= 0 || c->intermediate <= 0 ||
      c->n_heads <= 0 || c->head_dim <= 0) {
    return fail(KLLM_B200_ERR_SHAPE, "chain_run: all dimensions must be positive");
  }
  if (c->weight_dtype != KLLM_B200_F16 && c->weight_dtype != KLLM_B200_F32) {
    return fail(KLLM_B200_ERR_DTYPE, "chain_run: weight dtype %d not supported", c->weight_dtype);
  }
  LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  o.pdl = c->use_pdl != 0;
  const int64_t T = c->n_tokens, H = c->hidden;
  const int wdt = c->weight_dtype;
  const int mask = c->op_mask == 0 ? 0x7f : c->op_mask;
  if ((mask & KLLM_B200_OP_ATTENTION) != 0) {
    for (int64_t l = 0; l < c->n_layers; ++l) {
      if (c->layers[l].attn_ctx == nullptr) return fail(KLLM_B200_ERR_INVALID_ARG, "chain_run: layer %lld has no attn_ctx", (long long)l);
    }
  }
  const bool gemm = (mask & KLLM_B200_OP_GEMM) != 0;
  if (gemm) {
    if ((mask & KLLM_B200_OP_ATTENTION) == 0) {
      return fail(KLLM_B200_ERR_INVALID_ARG, "chain_run: the GEMM op needs the attention op (o_proj reads attn_ctx)");
    }
    if (c->weights == nullptr) return fail(KLLM_B200_ERR_INVALID_ARG, "chain_run: the GEMM op needs weights");
    for (int64_t l = 0; l < c->n_layers; ++l) {
      const kllm_b200_layer_weights& W = c->weights[l];
      if (!W.wq || !W.wk || !W.wv || !W.wo || !W.w_gate || !W.w_up || !W.w_down) {
        return fail(KLLM_B200_ERR_INVALID_ARG, "chain_run: layer %lld is missing a GEMM weight", (long long)l);
      }
    }
  }
  auto on = [mask](int bit) { return (mask & bit) != 0; };
  // Whether the launch before the next one wrote the residual. A residual
  // add may read its residual rows before its dependency wait (PDL) when the
  // launch before it did not write them: they were then written two or more
  // launches back, and every kernel of this library triggers its dependents
  // only after its own wait. Unknown (true) before the chain's first launch.
  bool prev_wrote_residual = true;
  int launched = 0;
  // Every launch after the chain's first may read the inputs no launch of the
  // chain writes (weights, biases, positions, slots, table, ids) before its
  // dependency wait. The first launch reads nothing before its wait: the
  // caller's launch before it may have written any of them.
  auto step_opts = [&]() {
    LaunchOpts n = o;
    n.early_inputs = o.pdl && launched > 0;
    return n;
  };
  auto norm_opts = [&]() {
    LaunchOpts n = step_opts();
    n.early_residual = o.pdl && !prev_wrote_residual;
    return n;
  };
  const int64_t qd = c->n_heads * c->head_dim, I = c->intermediate;
  int rc = KLLM_B200_OK;
  // the embedding and layer 0's input norm run as one kernel when both are on
  const bool fuse_embedding = on(KLLM_B200_OP_EMBEDDING) && on(KLLM_B200_OP_INPUT_NORM);
  if (fuse_embedding) {
    rc = embedding_rms_norm(c->embed_table, c->vocab, H, c->ids, T, c->layers[0].input_norm_w, wdt, c->eps,
                            c->residual, c->layers[0].attn_norm_out, c->err_flags, step_opts());
    if (rc != KLLM_B200_OK) return rc;
    ++launched;
    prev_wrote_residual = true;
  } else if (on(KLLM_B200_OP_EMBEDDING)) {
    rc = embedding(c->embed_table, c->vocab, H, KLLM_B200_F16, c->ids, T, c->residual, KLLM_B200_F16,
                   c->err_flags, step_opts());
    if (rc != KLLM_B200_OK) return rc;
    ++launched;
    prev_wrote_residual = true;
  }
  for (int64_t l = 0; l < c->n_layers; ++l) {
    const kllm_b200_layer_buffers& L = c->layers[l];
    const void* delta = l == 0 ? nullptr : c->layers[l - 1].ffn_out;
    if (on(KLLM_B200_OP_INPUT_NORM) && !(l == 0 && fuse_embedding)) {
      rc = add_rms_norm(c->residual, delta, L.input_norm_w, L.attn_norm_out, T, H, c->eps, KLLM_B200_F16, wdt,
                        norm_opts());
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = delta != nullptr;
    }
    if (gemm) {  // q/k/v projections with bias + RoPE + KV append in the GEMM's epilogue
      const kllm_b200_layer_weights& W = c->weights[l];
      rc = qkv_linear_rope_kv_append(L.attn_norm_out, W.wq, W.wk, W.wv, L.q_bias, L.k_bias, L.v_bias, wdt,
                                     c->positions, c->slots, T, H, c->n_heads, c->n_kv_heads, c->head_dim,
                                     c->theta, L.q, L.k_cache, L.v_cache, c->n_slots, c->max_seq, c->err_flags, o);
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = false;
    } else if (on(KLLM_B200_OP_QKV_ROPE)) {
      rc = qkv_bias_rope_kv_append(L.q, L.k, L.v, L.q_bias, L.k_bias, L.v_bias, wdt, c->positions, c->slots, T,
                                   c->n_heads, c->n_kv_heads, c->head_dim, c->theta, L.k_cache, L.v_cache,
                                   c->n_slots, c->max_seq, c->err_flags, step_opts());
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = false;
    }
    if (on(KLLM_B200_OP_ATTENTION)) {
      // runs of seq_len tokens of one sequence; single tokens for ragged batches
      const int64_t run = c->seq_ends == nullptr && c->seq_len >= 1 ? c->seq_len : 1;
      int n = 0;
      rc = attention_head_major(L.q, L.k_cache, L.v_cache, L.attn_ctx, c->positions, c->slots, T, run, c->n_heads,
                                c->n_kv_heads, c->head_dim, c->n_slots, c->max_seq, KLLM_B200_F16, c->attn_workspace,
                                c->attn_workspace_bytes, c->err_flags, o, &n);
      if (rc != KLLM_B200_OK) return rc;
      launched += n;
      if (n > 0) prev_wrote_residual = false;
    }
    if (gemm) {  // o projection of the attention output
      const kllm_b200_layer_weights& W = c->weights[l];
      rc = linear(L.attn_ctx, W.wo, W.o_bias, wdt, const_cast<void*>(L.attn_out), T, H, qd, c->err_flags, o);
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = false;
    }
    if (on(KLLM_B200_OP_POST_NORM)) {
      rc = add_rms_norm(c->residual, L.attn_out, L.post_norm_w, L.ffn_norm_out, T, H, c->eps, KLLM_B200_F16, wdt,
                        norm_opts());
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = true;
    }
    if (on(KLLM_B200_OP_SWIGLU) && !gemm) {
      rc = silu_mul(L.gate, L.up, L.swiglu_out, T * c->intermediate, KLLM_B200_F16, o);
      if (rc != KLLM_B200_OK) return rc;
      ++launched;
      prev_wrote_residual = false;
    }
    if (gemm) {  // gate/up projections with SwiGLU fused, then the down projection
      const kllm_b200_layer_weights& W = c->weights[l];
      rc = linear_swiglu(L.ffn_norm_out, W.w_gate, W.w_up, W.gate_bias, W.up_bias, wdt, L.swiglu_out, T, I, H,
                         c->err_flags, o);
      if (rc == KLLM_B200_OK) {
        rc = linear(L.swiglu_out, W.w_down, W.down_bias, wdt, const_cast<void*>(L.ffn_out), T, H, I, c->err_flags, o);
      }
      if (rc != KLLM_B200_OK) return rc;
      launched += 2;
      prev_wrote_residual = false;
    }
  }
  // the final norm also writes the last rows when every sequence has seq_len rows
  const bool fuse_select = on(KLLM_B200_OP_FINAL_NORM) && on(KLLM_B200_OP_SELECT) && c->seq_ends == nullptr &&
                           c->seq_len >= 1 && c->n_seqs * c->seq_len == T;
  if (fuse_select) {
    int n = 0;
    rc = add_rms_norm_last_rows(c->residual, c->layers[c->n_layers - 1].ffn_out, c->final_norm_w,
                                c->final_norm_out, T, H, c->eps, wdt, c->last_rows, c->seq_len, c->n_seqs,
                                c->err_flags, norm_opts(), &n);
    if (rc != KLLM_B200_OK) return rc;
    launched += n;
  } else if (on(KLLM_B200_OP_FINAL_NORM)) {
    rc = add_rms_norm(c->residual, c->layers[c->n_layers - 1].ffn_out, c->final_norm_w, c->final_norm_out, T, H,
                      c->eps, KLLM_B200_F16, wdt, norm_opts());
    if (rc != KLLM_B200_OK) return rc;
    ++launched;
  }
  if (on(KLLM_B200_OP_SELECT) && !fuse_select) {
    rc = select_last_rows(c->final_norm_out, T, H, c->seq_ends, c->seq_len, c->n_seqs, c->last_rows,
                          KLLM_B200_F16, c->err_flags, o);
    if (rc != KLLM_B200_OK) return rc;
    ++launched;
  }
  if (gemm && c->lm_head != nullptr && c->logits != nullptr) {
    rc = linear(c->last_rows, c->lm_head, nullptr, wdt, c->logits, c->n_seqs, c->vocab, H, c->err_flags, o);
    if (rc != KLLM_B200_OK) return rc;
    ++launched;
  }
  if (n_launches) *n_launches = launched;
  return KLLM_B200_OK;
}
