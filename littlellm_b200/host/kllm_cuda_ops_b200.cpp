// kllm_cuda_ops_b200.cpp — LittleLLM's CUDA operator backend on the B200 C ABI.
//
// This file is the binding a LittleLLM build compiles in place of its own
// src/op/cuda/{embedding,rms_norm,add,rope,kv_cache,silu}.cu and the
// dequantize_int8 of src/op/cuda/quantize.cu: it defines the functions that
// include/kllm/op/cuda_ops.h declares (the ones src/op/dispatch.cpp:43-194
// routes CUDA tensors to) on top of libkllm_b200.so (include/kllm_b200.h).
// It is compiled against the reference's own headers (kllm/base/tensor.h,
// kllm/op/cuda_ops.h); GEMM, attention, int8 quantize and int8 GEMM stay with
// the reference's implementations.
//
// Conventions kept from the reference:
//  - shapes are read from the Tensor exactly as the reference kernels read
//    them (x.shape().at(0) rows, at(1) columns, ...);
//  - errors are thrown as std::runtime_error (include/kllm/op/detail/
//    cuda_helpers.cuh:11-15), with the library's message;
//  - launches go to the legacy default stream, so they are ordered with the
//    reference's other CUDA work (cuBLAS GEMMs, attention) exactly as before.
// Token ids arrive as a host std::vector; they are range-checked on the host
// (the reference CPU path's check, src/op/cpu/embedding.cpp:22-24, which its
// CUDA path lacks) and handed to kllm_b200_embedding_host_ids, which carries
// them in the kernel launches' parameters: no device buffer to grow (the
// reference's TokenIdBufferCache, src/op/cuda/embedding.cu:13-41) and no
// blocking copy.

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "kllm/base/tensor.h"
#include "kllm/op/cuda_ops.h"
#include "kllm_b200.h"

namespace kllm::op {

namespace {

void check(int status) {
  if (status != KLLM_B200_OK) {
    char msg[512];
    kllm_b200_last_error(msg, sizeof msg);
    throw std::runtime_error(msg);
  }
}

int dt(const Tensor& t) { return static_cast<int>(t.dtype()); }

}  // namespace

void cuda_embedding(const Tensor& table, const std::vector<int>& token_ids, Tensor& out) {
  const int64_t vocab = table.shape().at(0);
  const int64_t hidden = table.shape().at(1);
  if (out.shape().size() != 2 || out.shape()[0] != static_cast<int64_t>(token_ids.size()) ||
      out.shape()[1] != hidden) {
    throw std::runtime_error("embedding output shape mismatch");
  }
  for (int id : token_ids) {
    if (id < 0 || id >= vocab) throw std::runtime_error("token id out of vocabulary range");
  }
  if (token_ids.empty()) return;
  static_assert(sizeof(int) == sizeof(int32_t), "ids are passed as int32");
  check(kllm_b200_embedding_host_ids(table.data(), vocab, hidden, dt(table),
                                     reinterpret_cast<const int32_t*>(token_ids.data()),
                                     static_cast<int64_t>(token_ids.size()), out.data(), dt(out), nullptr, nullptr));
}

void cuda_rms_norm(const Tensor& x, const Tensor& weight, Tensor& out, float eps) {
  check(kllm_b200_rms_norm(x.data(), weight.data(), out.data(), x.shape().at(0), x.shape().at(1), eps, dt(x),
                           dt(weight), nullptr));
}

void cuda_add_bias_inplace(Tensor& x, const Tensor* bias) {
  if (bias == nullptr) return;
  check(kllm_b200_add_bias_inplace(x.data(), bias->data(), x.shape().at(0), x.shape().at(1), dt(x),
                                   dt(*bias), nullptr));
}

void cuda_add_inplace(Tensor& x, const Tensor& residual) {
  if (x.numel() != residual.numel()) throw std::runtime_error("add shape mismatch");
  check(kllm_b200_add_inplace(x.data(), residual.data(), static_cast<int64_t>(x.numel()), dt(x), dt(residual),
                              nullptr));
}

void cuda_select_last_row(const Tensor& x, Tensor& out) {
  const int64_t cols = x.shape().at(1);
  if (out.shape().size() != 2 || out.shape().at(0) != 1 || out.shape().at(1) != cols) {
    throw std::runtime_error("select_last_row output shape mismatch");
  }
  if (x.dtype() != out.dtype()) throw std::runtime_error("select_last_row dtype mismatch");
  check(kllm_b200_select_last_row(x.data(), x.shape().at(0), cols, out.data(), dt(x), nullptr));
}

void cuda_silu_mul(const Tensor& gate, const Tensor& up, Tensor& out) {
  if (gate.numel() != up.numel() || gate.numel() != out.numel()) {
    throw std::runtime_error("silu_mul shape mismatch");
  }
  if (gate.dtype() != up.dtype() || gate.dtype() != out.dtype()) {
    throw std::runtime_error("silu_mul dtype mismatch");
  }
  check(kllm_b200_silu_mul(gate.data(), up.data(), out.data(), static_cast<int64_t>(gate.numel()), dt(gate),
                           nullptr));
}

void cuda_rope_inplace(Tensor& q_or_k, int past_len, float theta) {
  check(kllm_b200_rope_inplace(q_or_k.data(), q_or_k.shape().at(0), q_or_k.shape().at(1), q_or_k.shape().at(2),
                               past_len, theta, dt(q_or_k), nullptr));
}

void cuda_copy_kv_to_cache(const Tensor& k, const Tensor& v, Tensor& k_cache, Tensor& v_cache, int past_len) {
  check(kllm_b200_copy_kv_to_cache(k.data(), v.data(), k.shape().at(0), k.shape().at(1), k.shape().at(2),
                                   k_cache.data(), v_cache.data(), k_cache.shape().at(0), past_len, dt(k),
                                   dt(k_cache), nullptr));
}

namespace cuda {

void dequantize_int8(const Tensor& data, const Tensor& scale, Tensor& output) {
  if (data.numel() != output.numel()) throw std::runtime_error("dequantize_int8 shape mismatch");
  check(kllm_b200_dequantize_int8(static_cast<const int8_t*>(data.data()), static_cast<const float*>(scale.data()),
                                  output.data(), static_cast<int64_t>(data.numel()), dt(output), nullptr));
}

}  // namespace cuda

}  // namespace kllm::op
