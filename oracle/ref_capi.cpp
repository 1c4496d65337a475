// ref_capi.cpp — C entry points over the reference's own CPU operators.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the reference's sources (src/base/{half,tensor}.cpp, src/op/dispatch.cpp,
// src/op/cpu/*.cpp, built in place from the read-only reference tree with the
// reference's Release flags) into oracle/_ref/libkllm_ref.so. The tests use it
// to pin the C restatement in kllm_oracle.c and to generate golden vectors;
// the benchmark's reference arm and CPU baseline time the reference's public
// kllm::op API through it. The CUDA product never links it.
//
// Each function builds CPU kllm::Tensor objects of the requested DType,
// copies the caller's bytes in, calls the reference operator through
// kllm::op (include/kllm/op/ops.h:10-35, dispatch at
// src/op/dispatch.cpp:43-194) and copies the result back.
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "kllm/base/half.h"
#include "kllm/base/tensor.h"
#include "kllm/model/llama.h"
#include "kllm/model/weights.h"
#include "kllm/op/ops.h"

namespace {

thread_local std::string g_error;

kllm::Tensor make_tensor(std::vector<std::int64_t> shape, int dtype, const void* src) {
  kllm::Tensor t(std::move(shape), static_cast<kllm::DType>(dtype), kllm::DeviceType::CPU);
  if (src != nullptr && t.nbytes() > 0) t.copy_from_host(src, t.nbytes());
  return t;
}

void read_back(const kllm::Tensor& t, void* dst) {
  if (dst != nullptr && t.nbytes() > 0) t.copy_to_host(dst, t.nbytes());
}

template <typename F>
int guarded(F&& body) {
  try {
    body();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

// Deterministic fill for the timing chain: splitmix64 + Box-Muller.
struct Fill {
  std::uint64_t state;
  std::uint64_t next() {
    std::uint64_t z = (state += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
  }
  float uniform() { return static_cast<float>((next() >> 40) + 1) * (1.0f / 16777217.0f); }
  float normal(float sigma) {
    const float u1 = uniform(), u2 = uniform();
    return sigma * std::sqrt(-2.0f * std::log(u1)) * std::cos(6.2831853f * u2);
  }
};

void fill_normal(kllm::Tensor& t, Fill& rng, float sigma) {
  float* p = t.data_as<float>();
  for (std::size_t i = 0; i < t.numel(); ++i) p[i] = rng.normal(sigma);
}

void fill_uniform(kllm::Tensor& t, Fill& rng, float lo, float hi) {
  float* p = t.data_as<float>();
  for (std::size_t i = 0; i < t.numel(); ++i) p[i] = lo + (hi - lo) * rng.uniform();
}

// One sequence of the reference's non-GEMM decoder chain in fp32 on the CPU,
// with the op order of LlamaRunner::forward (src/model/llama.cpp:78-178);
// GEMM outputs are pre-filled tensors.
struct RefChain {
  int T, H, Hq, Hkv, D, I, max_seq;
  float eps, theta;
  const kllm::Tensor* table;
  std::vector<int> ids;
  kllm::Tensor x, attn_norm, q, k, v, attn_out, ffn_norm, gate, up, swiglu, ffn_out;
  kllm::Tensor normed, last, w_in, w_post, w_final, bq, bk, bv, k_cache, v_cache;
};

}  // namespace

extern "C" {

const char* kref_last_error() { return g_error.c_str(); }

std::uint16_t kref_float_to_half(float v) { return kllm::float_to_half(v); }
float kref_half_to_float(std::uint16_t h) { return kllm::half_to_float(h); }

void kref_float_to_half_array(const float* in, std::uint16_t* out, std::int64_t n) {
  for (std::int64_t i = 0; i < n; ++i) out[i] = kllm::float_to_half(in[i]);
}

int kref_embedding(const void* table, std::int64_t vocab, std::int64_t hidden, int dtype,
                   const std::int32_t* ids, std::int64_t n, void* out) {
  return guarded([&] {
    auto t = make_tensor({vocab, hidden}, dtype, table);
    auto o = make_tensor({n, hidden}, dtype, nullptr);
    std::vector<int> id(ids, ids + n);
    kllm::op::embedding(t, id, o);
    read_back(o, out);
  });
}

int kref_rms_norm(const void* x, const void* w, void* out, std::int64_t rows,
                  std::int64_t hidden, float eps, int x_dtype, int w_dtype) {
  return guarded([&] {
    auto xt = make_tensor({rows, hidden}, x_dtype, x);
    auto wt = make_tensor({hidden}, w_dtype, w);
    auto ot = make_tensor({rows, hidden}, x_dtype, nullptr);
    kllm::op::rms_norm(xt, wt, ot, eps);
    read_back(ot, out);
  });
}

int kref_add_inplace(void* x, const void* y, std::int64_t n, int dtype) {
  return guarded([&] {
    auto xt = make_tensor({n}, dtype, x);
    auto yt = make_tensor({n}, dtype, y);
    kllm::op::add_inplace(xt, yt);
    read_back(xt, x);
  });
}

int kref_add_bias_inplace(void* x, const void* bias, std::int64_t rows, std::int64_t cols,
                          int dtype) {
  return guarded([&] {
    auto xt = make_tensor({rows, cols}, dtype, x);
    if (bias == nullptr) {
      kllm::op::add_bias_inplace(xt, nullptr);
    } else {
      auto bt = make_tensor({cols}, dtype, bias);
      kllm::op::add_bias_inplace(xt, &bt);
    }
    read_back(xt, x);
  });
}

int kref_select_last_row(const void* x, std::int64_t rows, std::int64_t cols, void* out,
                         int dtype) {
  return guarded([&] {
    auto xt = make_tensor({rows, cols}, dtype, x);
    auto ot = make_tensor({1, cols}, dtype, nullptr);
    kllm::op::select_last_row(xt, ot);
    read_back(ot, out);
  });
}

// kllm::op::matmul on the CPU (cpu_matmul, src/op/cpu/matmul.cpp:9-33):
// out [m, n] = a [m, k] * b [n, k]^T.
int kref_matmul(const void* a, const void* b, void* out, std::int64_t m, std::int64_t n, std::int64_t k,
                int dtype) {
  return guarded([&] {
    auto at = make_tensor({m, k}, dtype, a);
    auto bt = make_tensor({n, k}, dtype, b);
    auto ot = make_tensor({m, n}, dtype, nullptr);
    kllm::op::matmul(at, bt, ot);
    read_back(ot, out);
  });
}

int kref_silu_mul(const void* g, const void* u, void* out, std::int64_t n, int dtype) {
  return guarded([&] {
    auto gt = make_tensor({n}, dtype, g);
    auto ut = make_tensor({n}, dtype, u);
    auto ot = make_tensor({n}, dtype, nullptr);
    kllm::op::silu_mul(gt, ut, ot);
    read_back(ot, out);
  });
}

int kref_rope_inplace(void* x, std::int64_t seq, std::int64_t heads, std::int64_t head_dim,
                      int past_len, float theta, int dtype) {
  return guarded([&] {
    auto xt = make_tensor({seq, heads, head_dim}, dtype, x);
    kllm::op::rope_inplace(xt, past_len, theta);
    read_back(xt, x);
  });
}

int kref_copy_kv_to_cache(const void* k, const void* v, std::int64_t seq,
                          std::int64_t kv_heads, std::int64_t head_dim, void* k_cache,
                          void* v_cache, std::int64_t max_seq, int past_len, int dtype) {
  return guarded([&] {
    auto kt = make_tensor({seq, kv_heads, head_dim}, dtype, k);
    auto vt = make_tensor({seq, kv_heads, head_dim}, dtype, v);
    auto kc = make_tensor({max_seq, kv_heads, head_dim}, dtype, k_cache);
    auto vc = make_tensor({max_seq, kv_heads, head_dim}, dtype, v_cache);
    kllm::op::copy_kv_to_cache(kt, vt, kc, vc, past_len);
    read_back(kc, k_cache);
    read_back(vc, v_cache);
  });
}

// kllm::op::attention on CPU tensors: q/out [seq, heads, head_dim], caches
// [max_seq, kv_heads, head_dim]; keys 0..past_len+t for token t.
int kref_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                   std::int64_t seq, std::int64_t max_seq, int past_len, int heads, int kv_heads,
                   int head_dim, int dtype) {
  return guarded([&] {
    auto qt = make_tensor({seq, heads, head_dim}, dtype, q);
    auto kc = make_tensor({max_seq, kv_heads, head_dim}, dtype, k_cache);
    auto vc = make_tensor({max_seq, kv_heads, head_dim}, dtype, v_cache);
    auto ot = make_tensor({seq, heads, head_dim}, dtype, nullptr);
    kllm::op::attention(qt, kc, vc, ot, past_len, past_len + static_cast<int>(seq), heads, kv_heads,
                        head_dim);
    read_back(ot, out);
  });
}

int kref_dequantize_int8(const std::int8_t* q, std::int64_t n, float scale, float* out) {
  return guarded([&] {
    auto qt = make_tensor({n}, 3, q);
    auto st = make_tensor({1}, 0, &scale);
    auto ot = make_tensor({n}, 0, nullptr);
    kllm::op::dequantize_int8(qt, st, ot);
    read_back(ot, out);
  });
}

// fp16 weight-load dequant: the loop body of src/model/weights.cpp:139-148
// (fp32 product, then the reference float_to_half).
void kref_dequantize_int8_f16(const std::int8_t* q, std::int64_t n, float scale,
                              std::uint16_t* out) {
  for (std::int64_t i = 0; i < n; ++i) {
    const float deq = static_cast<float>(q[i]) * scale;
    out[i] = kllm::float_to_half(deq);
  }
}

// ---- the reference weight loader (src/model/weights.cpp) on the CPU --------

void* kref_weights_load(const char* path) {
  try {
    return new kllm::ModelWeights(kllm::ModelWeights::load(path, kllm::DeviceType::CPU));
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void kref_weights_free(void* w) { delete static_cast<kllm::ModelWeights*>(w); }

// Copies the named tensor as float values (its CPU dtype: F32 for F32 and
// I8 records, F16/I32 converted exactly); returns numel or -1.
std::int64_t kref_weights_get(void* w, const char* name, float* out, std::int64_t cap) {
  const kllm::Tensor* t = static_cast<kllm::ModelWeights*>(w)->find(name);
  if (t == nullptr) {
    g_error = std::string("no tensor ") + name;
    return -1;
  }
  const std::vector<float> v = t->to_float_vector();
  if (static_cast<std::int64_t>(v.size()) > cap) return -1;
  std::memcpy(out, v.data(), v.size() * sizeof(float));
  return static_cast<std::int64_t>(v.size());
}

int kref_weights_dtype(void* w, const char* name) {
  const kllm::Tensor* t = static_cast<kllm::ModelWeights*>(w)->find(name);
  return t == nullptr ? -1 : static_cast<int>(t->dtype());
}

// ---- the reference model runner (src/model/llama.cpp) on the CPU ----------

// LlamaRunner over a .kllm file loaded on the CPU (F32 activations).
void* kref_runner_create(const char* path, int max_seq) {
  try {
    return new kllm::LlamaRunner(kllm::ModelWeights::load(path, kllm::DeviceType::CPU), kllm::DeviceType::CPU,
                                 max_seq);
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void kref_runner_destroy(void* r) { delete static_cast<kllm::LlamaRunner*>(r); }

// One LlamaRunner::forward (src/model/llama.cpp:68-184) of n tokens at
// past_len; the last token's logits (vocab floats) go to `logits`.
int kref_runner_forward(void* r, const std::int32_t* ids, int n, int past_len, float* logits,
                        std::int64_t vocab) {
  return guarded([&] {
    std::vector<int> in(ids, ids + n);
    const kllm::Tensor out = static_cast<kllm::LlamaRunner*>(r)->forward(in, past_len);
    const std::vector<float> v = out.to_float_vector();
    if (static_cast<std::int64_t>(v.size()) != vocab) throw std::runtime_error("logits size mismatch");
    std::memcpy(logits, v.data(), v.size() * sizeof(float));
  });
}

// ---- timing chain -------------------------------------------------------

void* kref_table_create(std::int64_t vocab, std::int64_t hidden, std::uint64_t seed) {
  try {
    auto* t = new kllm::Tensor({vocab, hidden}, kllm::DType::F32, kllm::DeviceType::CPU);
    Fill rng{seed};
    fill_normal(*t, rng, 0.02f);
    return t;
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void kref_table_destroy(void* table) { delete static_cast<kllm::Tensor*>(table); }

void* kref_chain_create(const void* table, int T, int Hq, int Hkv, int D, int I,
                        int max_seq, float eps, float theta, std::uint64_t seed) {
  try {
    const auto* tab = static_cast<const kllm::Tensor*>(table);
    auto c = std::make_unique<RefChain>();
    const int H = static_cast<int>(tab->shape().at(1));
    const int vocab = static_cast<int>(tab->shape().at(0));
    c->T = T; c->H = H; c->Hq = Hq; c->Hkv = Hkv; c->D = D; c->I = I;
    c->max_seq = max_seq; c->eps = eps; c->theta = theta; c->table = tab;
    Fill rng{seed};
    c->ids.resize(T);
    for (int t = 0; t < T; ++t) c->ids[t] = static_cast<int>(rng.next() % vocab);
    auto f32 = [](std::vector<std::int64_t> s) {
      return kllm::Tensor(std::move(s), kllm::DType::F32, kllm::DeviceType::CPU);
    };
    c->x = f32({T, H});
    c->attn_norm = f32({T, H});
    c->ffn_norm = f32({T, H});
    c->normed = f32({T, H});
    c->last = f32({1, H});
    c->q = f32({T, Hq * D});
    c->k = f32({T, Hkv * D});
    c->v = f32({T, Hkv * D});
    c->attn_out = f32({T, H});
    c->ffn_out = f32({T, H});
    c->gate = f32({T, I});
    c->up = f32({T, I});
    c->swiglu = f32({T, I});
    c->w_in = f32({H});
    c->w_post = f32({H});
    c->w_final = f32({H});
    c->bq = f32({Hq * D});
    c->bk = f32({Hkv * D});
    c->bv = f32({Hkv * D});
    c->k_cache = f32({max_seq, Hkv, D});
    c->v_cache = f32({max_seq, Hkv, D});
    for (auto* t : {&c->q, &c->k, &c->v, &c->attn_out, &c->ffn_out, &c->gate, &c->up}) {
      fill_normal(*t, rng, 1.0f);
    }
    for (auto* t : {&c->bq, &c->bk, &c->bv}) fill_normal(*t, rng, 0.02f);
    for (auto* t : {&c->w_in, &c->w_post, &c->w_final}) fill_uniform(*t, rng, 0.5f, 1.5f);
    return c.release();
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void kref_chain_destroy(void* chain) { delete static_cast<RefChain*>(chain); }

// Runs embedding, n_layers decoder layers' non-GEMM ops and the final
// norm + select_last_row through the reference's public kllm::op API.
int kref_chain_run(void* chain, int n_layers) {
  auto* c = static_cast<RefChain*>(chain);
  return guarded([&] {
    namespace op = kllm::op;
    op::embedding(*c->table, c->ids, c->x);
    for (int l = 0; l < n_layers; ++l) {
      op::rms_norm(c->x, c->w_in, c->attn_norm, c->eps);
      op::add_bias_inplace(c->q, &c->bq);
      op::add_bias_inplace(c->k, &c->bk);
      op::add_bias_inplace(c->v, &c->bv);
      c->q.reshape({c->T, c->Hq, c->D});
      c->k.reshape({c->T, c->Hkv, c->D});
      c->v.reshape({c->T, c->Hkv, c->D});
      op::rope_inplace(c->q, 0, c->theta);
      op::rope_inplace(c->k, 0, c->theta);
      op::copy_kv_to_cache(c->k, c->v, c->k_cache, c->v_cache, 0);
      c->q.reshape({c->T, c->Hq * c->D});
      c->k.reshape({c->T, c->Hkv * c->D});
      c->v.reshape({c->T, c->Hkv * c->D});
      op::add_inplace(c->x, c->attn_out);
      op::rms_norm(c->x, c->w_post, c->ffn_norm, c->eps);
      op::silu_mul(c->gate, c->up, c->swiglu);
      op::add_inplace(c->x, c->ffn_out);
    }
    op::rms_norm(c->x, c->w_final, c->normed, c->eps);
    op::select_last_row(c->normed, c->last);
  });
}

}  // extern "C"
