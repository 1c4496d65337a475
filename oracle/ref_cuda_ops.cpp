// ref_cuda_ops.cpp — times the reference's own CUDA operators on the GPU.
//
// TEST INFRASTRUCTURE ONLY (a baseline, never the product). Built by
// oracle/Makefile (target dropin) against the reference's sources with its
// CUDA backend: every src/op/cuda/*.cu compiled for sm_100a. It calls the
// reference's public CUDA operators (include/kllm/op/cuda_ops.h) on reference
// Tensors the way LlamaRunner::forward calls them per layer
// (src/model/llama.cpp:79-178):
//
//   embedding      cuda_embedding(table, ids, out)                  (:84)
//   add_rms_norm   cuda_add_inplace(r, delta); cuda_rms_norm(r, w)  (:135-143, :166 -> :83)
//   rms_norm       cuda_rms_norm(r, w) alone (layer 0's input norm, :83)
//   qkv_rope_kv    cuda_add_bias_inplace x3; cuda_rope_inplace x2;
//                  cuda_copy_kv_to_cache                             (:89-114)
//   silu_mul       cuda_silu_mul(gate, up, out)                      (:158)
//   select_last_row cuda_select_last_row(x_b, out), once per sequence (:173)
//   dequant_f32    cuda::dequantize_int8(q, scale, out_f32)          (src/op/cuda/quantize.cu:110-121)
//
// Every op kind is timed over `layers` calls per pass that cycle through
// `sets` distinct buffer sets (more bytes than the 126 MB L2), `reps` passes,
// with CUDA events on the legacy default stream the reference launches on;
// launches are eager (the reference API takes no stream, so nothing can be
// captured in a graph). The reference runner serves one sequence at a time,
// so RoPE runs at positions past_len + t (past_len = 0) over all T rows and
// the KV copy goes to one [T, kv_heads, head_dim] block: the same bytes as
// the batched per-row-position op it is compared with.
//
// Usage: ref_cuda_ops T hidden heads kv_heads head_dim intermediate vocab
//                     layers sets reps eps theta n_seqs dequant_rows dequant_cols
// Output: one line per op, "<op> <microseconds per call-group> <calls per group>".
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "kllm/base/half.h"
#include "kllm/base/tensor.h"
#include "kllm/op/cuda_ops.h"

namespace {

using kllm::DeviceType;
using kllm::DType;
using kllm::Tensor;

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Fills the fp16 tensor `t` from the prefix of `host`, a host array of
// random fp16 bit patterns at least as long as any tensor filled.
void fill(Tensor& t, const std::vector<uint16_t>& host) {
  if (t.dtype() != DType::F16 || t.numel() > host.size()) throw std::runtime_error("fill: bad tensor");
  t.copy_from_host(host.data(), t.numel() * 2);
}

struct Timer {
  cudaEvent_t a{}, b{};
  Timer() {
    cuda_check(cudaEventCreate(&a), "event");
    cuda_check(cudaEventCreate(&b), "event");
  }
  ~Timer() {
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  template <typename F>
  double us_per_group(int reps, int groups, F&& pass) {
    pass();  // warm: first-call set-up of the reference (inv_freq table, id buffer)
    cuda_check(cudaDeviceSynchronize(), "sync");
    cuda_check(cudaEventRecord(a, nullptr), "record");
    for (int r = 0; r < reps; ++r) pass();
    cuda_check(cudaEventRecord(b, nullptr), "record");
    cuda_check(cudaEventSynchronize(b), "sync");
    float ms = 0.f;
    cuda_check(cudaEventElapsedTime(&ms, a, b), "elapsed");
    return 1000.0 * ms / (static_cast<double>(reps) * groups);
  }
};

}  // namespace

int main(int argc, char** argv) {
  if (argc != 16) {
    std::fprintf(stderr,
                 "usage: %s T hidden heads kv_heads head_dim intermediate vocab layers sets reps eps theta "
                 "n_seqs dequant_rows dequant_cols\n",
                 argv[0]);
    return 2;
  }
  try {
    const int64_t T = std::atoll(argv[1]), H = std::atoll(argv[2]), Hq = std::atoll(argv[3]);
    const int64_t Hkv = std::atoll(argv[4]), D = std::atoll(argv[5]), I = std::atoll(argv[6]);
    const int64_t V = std::atoll(argv[7]);
    const int layers = std::atoi(argv[8]), sets = std::atoi(argv[9]), reps = std::atoi(argv[10]);
    const float eps = std::strtof(argv[11], nullptr), theta = std::strtof(argv[12], nullptr);
    const int64_t n_seqs = std::atoll(argv[13]), dq_rows = std::atoll(argv[14]), dq_cols = std::atoll(argv[15]);
    if (T <= 0 || H <= 0 || layers <= 0 || sets <= 0 || reps <= 0 || n_seqs <= 0 || T % n_seqs != 0) {
      throw std::runtime_error("bad arguments");
    }

    std::mt19937_64 rng(0x4B4C4C4D);
    std::normal_distribution<float> nrm(0.f, 1.f);
    std::vector<uint16_t> pool(1 << 20);
    for (auto& x : pool) x = kllm::float_to_half(nrm(rng));
    std::size_t biggest = static_cast<std::size_t>(std::max({T * I, T * H, T * Hq * D, V * H}));
    std::vector<uint16_t> host(biggest);
    for (std::size_t i = 0; i < biggest; i += pool.size()) {
      std::memcpy(host.data() + i, pool.data(), std::min(pool.size(), biggest - i) * 2);
    }
    auto dev = [](std::vector<int64_t> shape, DType dt) { return Tensor(std::move(shape), dt, DeviceType::CUDA); };

    struct Set {
      Tensor residual, delta, norm_w, norm_out, q, k, v, bq, bk, bv, kc, vc, gate, up, act;
    };
    std::vector<std::unique_ptr<Set>> S;
    for (int s = 0; s < sets; ++s) {
      auto p = std::make_unique<Set>();
      p->residual = dev({T, H}, DType::F16);
      p->delta = dev({T, H}, DType::F16);
      p->norm_w = dev({H}, DType::F16);
      p->norm_out = dev({T, H}, DType::F16);
      p->q = dev({T, Hq, D}, DType::F16);
      p->k = dev({T, Hkv, D}, DType::F16);
      p->v = dev({T, Hkv, D}, DType::F16);
      p->bq = dev({Hq * D}, DType::F16);
      p->bk = dev({Hkv * D}, DType::F16);
      p->bv = dev({Hkv * D}, DType::F16);
      p->kc = dev({T, Hkv, D}, DType::F16);
      p->vc = dev({T, Hkv, D}, DType::F16);
      p->gate = dev({T, I}, DType::F16);
      p->up = dev({T, I}, DType::F16);
      p->act = dev({T, I}, DType::F16);
      for (Tensor* t : {&p->residual, &p->delta, &p->norm_w, &p->q, &p->k, &p->v, &p->bq, &p->bk, &p->bv,
                        &p->gate, &p->up}) {
        fill(*t, host);
      }
      S.push_back(std::move(p));
    }
    Timer tm;
    const int64_t seq_len = T / n_seqs;

    // q/k/v views as the rope op wants them ([T, heads, D]) and as the bias add
    // wants them ([T, heads * D]): the reference's linear() output is 2-D and
    // llama.cpp reshapes it before rope (src/model/llama.cpp:108-110)
    double us = tm.us_per_group(reps, layers, [&] {
      for (int l = 0; l < layers; ++l) {
        Set& s = *S[l % sets];
        s.q.reshape({T, Hq * D});
        s.k.reshape({T, Hkv * D});
        s.v.reshape({T, Hkv * D});
        kllm::op::cuda_add_bias_inplace(s.q, &s.bq);
        kllm::op::cuda_add_bias_inplace(s.k, &s.bk);
        kllm::op::cuda_add_bias_inplace(s.v, &s.bv);
        s.q.reshape({T, Hq, D});
        s.k.reshape({T, Hkv, D});
        s.v.reshape({T, Hkv, D});
        kllm::op::cuda_rope_inplace(s.q, 0, theta);
        kllm::op::cuda_rope_inplace(s.k, 0, theta);
        kllm::op::cuda_copy_kv_to_cache(s.k, s.v, s.kc, s.vc, 0);
      }
    });
    std::printf("qkv_bias_rope_kv_append %.4f 7\n", us);

    us = tm.us_per_group(reps, layers, [&] {
      for (int l = 0; l < layers; ++l) {
        Set& s = *S[l % sets];
        kllm::op::cuda_add_inplace(s.residual, s.delta);
        kllm::op::cuda_rms_norm(s.residual, s.norm_w, s.norm_out, eps);
      }
    });
    std::printf("add_rms_norm %.4f 2\n", us);

    us = tm.us_per_group(reps, layers, [&] {
      for (int l = 0; l < layers; ++l) {
        Set& s = *S[l % sets];
        kllm::op::cuda_rms_norm(s.residual, s.norm_w, s.norm_out, eps);
      }
    });
    std::printf("rms_norm %.4f 1\n", us);

    us = tm.us_per_group(reps, layers, [&] {
      for (int l = 0; l < layers; ++l) {
        Set& s = *S[l % sets];
        kllm::op::cuda_silu_mul(s.gate, s.up, s.act);
      }
    });
    std::printf("silu_mul %.4f 1\n", us);

    // select_last_row: the runner picks one row per sequence; B sequences
    // are B calls on [seq_len, H] views... the reference Tensor owns its
    // memory, so each sequence's rows are a tensor of their own here
    {
      std::vector<std::unique_ptr<Tensor>> xs;
      for (int64_t b = 0; b < n_seqs; ++b) {
        xs.push_back(std::make_unique<Tensor>(std::vector<int64_t>{seq_len, H}, DType::F16, DeviceType::CUDA));
        fill(*xs.back(), host);
      }
      Tensor out = dev({1, H}, DType::F16);
      us = tm.us_per_group(reps, 1, [&] {
        for (auto& x : xs) kllm::op::cuda_select_last_row(*x, out);
      });
      std::printf("select_last_rows %.4f %lld\n", us, static_cast<long long>(n_seqs));
    }
    S.clear();

    {  // embedding: one call per step over all T tokens (its ids uploaded per call)
      Tensor table = dev({V, H}, DType::F16);
      fill(table, host);
      std::uniform_int_distribution<int> pick(0, static_cast<int>(V - 1));
      std::vector<std::vector<int>> ids(sets, std::vector<int>(T));
      for (auto& v : ids)
        for (auto& x : v) x = pick(rng);
      std::vector<std::unique_ptr<Tensor>> outs;
      for (int s = 0; s < sets; ++s) outs.push_back(std::make_unique<Tensor>(std::vector<int64_t>{T, H}, DType::F16, DeviceType::CUDA));
      us = tm.us_per_group(reps, sets, [&] {
        for (int s = 0; s < sets; ++s) kllm::op::cuda_embedding(table, ids[s], *outs[s]);
      });
      std::printf("embedding %.4f 1\n", us);
    }

    if (dq_rows > 0 && dq_cols > 0) {  // INT8 -> fp32 dequant of one weight-sized tensor per call
      std::vector<int8_t> hq(static_cast<std::size_t>(dq_rows * dq_cols));
      std::uniform_int_distribution<int> q8(-127, 127);
      for (auto& x : hq) x = static_cast<int8_t>(q8(rng));
      std::vector<std::unique_ptr<Tensor>> qs, outs;
      Tensor scale = dev({1}, DType::F32);
      const float sc = 0.0047f;
      scale.copy_from_host(&sc, 4);
      const int dq_sets = 4;
      for (int s = 0; s < dq_sets; ++s) {
        qs.push_back(std::make_unique<Tensor>(std::vector<int64_t>{dq_rows, dq_cols}, DType::I8, DeviceType::CUDA));
        qs.back()->copy_from_host(hq.data(), hq.size());
        outs.push_back(std::make_unique<Tensor>(std::vector<int64_t>{dq_rows, dq_cols}, DType::F32, DeviceType::CUDA));
      }
      us = tm.us_per_group(reps, dq_sets, [&] {
        for (int s = 0; s < dq_sets; ++s) kllm::op::cuda::dequantize_int8(*qs[s], scale, *outs[s]);
      });
      std::printf("dequant_f32 %.4f 1\n", us);
    }
    cuda_check(cudaDeviceSynchronize(), "final sync");
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ref_cuda_ops: %s\n", e.what());
    return 1;
  }
  return 0;
}
