// gather.cu — row gathers: embedding lookup and (batched) select_last_row.
//
// embedding replaces cuda_embedding (src/op/cuda/embedding.cu:83-108) with
// device-resident ids (no per-call host copy, no growing device buffer), and
// embedding_host_ids keeps its host std::vector<int> ids, carried in the
// launches' kernel parameters;
// select_last_rows generalises cuda_select_last_row (src/op/cuda/add.cu:78-84)
// to the last row of every sequence in a packed batch.
//
// Same-dtype rows whose byte length is a multiple of 16 are copied by one
// warp per row with 16-byte vectors, four vectors in flight per lane, so the
// output is a bit-exact copy of the source row. Mixed dtypes or odd sizes go
// through an element-per-thread kernel that converts (fp32->fp16 rounds to
// nearest even, as the reference kernel's __float2half does).
#include <cstring>

#include "ops.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Copies one row of nvec 16-byte vectors with the calling warp. The rows are
// read once (random table rows, last rows of sequences), so the loads do not
// allocate in L1.
__device__ __forceinline__ void warp_copy_row(const uint4* __restrict__ src, uint4* __restrict__ dst, int nvec,
                                              int lane) {
  for (int base = 0; base < nvec; base += 32 * 4) {
    uint4 buf[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = base + k * 32 + lane;
      if (i < nvec) buf[k] = ld_stream(src + i);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = base + k * 32 + lane;
      if (i < nvec) st_plain(dst + i, buf[k]);
    }
  }
}

__device__ __forceinline__ void warp_zero_row(uint4* dst, int nvec, int lane) {
  for (int i = lane; i < nvec; i += 32) st_plain(dst + i, make_uint4(0, 0, 0, 0));
}

// out[t] = table[ids[t]] with rows of nvec 16-byte vectors.
__global__ void __launch_bounds__(kThreads) embedding_vec_kernel(const uint4* __restrict__ table, int64_t vocab,
                                                                 const int32_t* __restrict__ ids, int64_t n_tokens,
                                                                 uint4* __restrict__ out, int nvec,
                                                                 int32_t* err_flags) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t t = warp_global; t < n_tokens; t += warp_stride) {
    const int32_t id = __ldg(ids + t);
    uint4* dst = out + t * nvec;
    if (id < 0 || id >= vocab) {
      warp_zero_row(dst, nvec, lane);
      if (lane == 0) set_flag(err_flags, KLLM_B200_FLAG_BAD_TOKEN);
      continue;
    }
    warp_copy_row(table + static_cast<int64_t>(id) * nvec, dst, nvec, lane);
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) embedding_generic_kernel(const TI* table, int64_t vocab, int64_t hidden,
                                                                     const int32_t* ids, int64_t n_tokens, TO* out,
                                                                     int32_t* err_flags) {
  grid_dep_wait();
  grid_dep_launch();
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    const int32_t id = ids[t];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && threadIdx.x == 0) set_flag(err_flags, KLLM_B200_FLAG_BAD_TOKEN);
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      out[t * hidden + c] = ok ? from_f<TO>(to_f(table[static_cast<int64_t>(id) * hidden + c])) : from_f<TO>(0.0f);
    }
  }
}

// Host ids carried in the kernel parameters: CUDA 12.1+ gives a kernel up to
// 32764 bytes of parameters, enough for KLLM_B200_PARAM_IDS int32 ids and the
// pointers, so cuda_embedding's std::vector<int> ids reach the GPU without a
// device buffer or a blocking copy.
struct ParamIds {
  const void* table;
  void* out;
  int32_t* err_flags;
  int64_t vocab;
  int64_t hidden;  // elements per row
  int n;           // ids in this launch
  int nvec;        // 16-byte vectors per row (same-dtype vector path)
  int32_t ids[KLLM_B200_PARAM_IDS];
};
static_assert(sizeof(ParamIds) <= 32764, "kernel parameters are limited to 32764 bytes");

// Vector path: one warp per token, as embedding_vec_kernel.
__global__ void __launch_bounds__(kThreads) embedding_param_vec_kernel(const __grid_constant__ ParamIds a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const uint4* table = static_cast<const uint4*>(a.table);
  uint4* out = static_cast<uint4*>(a.out);
  for (int t = blockIdx.x * kWarps + (threadIdx.x >> 5); t < a.n; t += gridDim.x * kWarps) {
    const int32_t id = a.ids[t];
    uint4* dst = out + static_cast<int64_t>(t) * a.nvec;
    if (id < 0 || id >= a.vocab) {
      warp_zero_row(dst, a.nvec, lane);
      if (lane == 0) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_TOKEN);
      continue;
    }
    warp_copy_row(table + static_cast<int64_t>(id) * a.nvec, dst, a.nvec, lane);
  }
}

// Any dtypes / row sizes: one CTA per token, element per thread.
template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) embedding_param_generic_kernel(const __grid_constant__ ParamIds a) {
  grid_dep_wait();
  grid_dep_launch();
  const TI* table = static_cast<const TI*>(a.table);
  TO* out = static_cast<TO*>(a.out);
  for (int t = blockIdx.x; t < a.n; t += gridDim.x) {
    const int32_t id = a.ids[t];
    const bool ok = id >= 0 && id < a.vocab;
    if (!ok && threadIdx.x == 0) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_TOKEN);
    for (int64_t c = threadIdx.x; c < a.hidden; c += blockDim.x) {
      out[t * a.hidden + c] = ok ? from_f<TO>(to_f(table[static_cast<int64_t>(id) * a.hidden + c])) : from_f<TO>(0.0f);
    }
  }
}

// out[b] = x[end_b - 1], end_b = seq_ends[b] or (b + 1) * seq_len.
__global__ void __launch_bounds__(kThreads) select_rows_vec_kernel(const uint4* __restrict__ x, int64_t rows,
                                                                   const int32_t* __restrict__ seq_ends,
                                                                   int64_t seq_len, int64_t n_seqs,
                                                                   uint4* __restrict__ out, int nvec,
                                                                   int32_t* err_flags) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t b = warp_global; b < n_seqs; b += warp_stride) {
    const int64_t end = seq_ends ? static_cast<int64_t>(__ldg(seq_ends + b)) : (b + 1) * seq_len;
    uint4* dst = out + b * nvec;
    if (end < 1 || end > rows) {
      warp_zero_row(dst, nvec, lane);
      if (lane == 0) set_flag(err_flags, KLLM_B200_FLAG_BAD_SEQ_END);
      continue;
    }
    warp_copy_row(x + (end - 1) * nvec, dst, nvec, lane);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) select_rows_generic_kernel(const T* x, int64_t rows, int64_t cols,
                                                                       const int32_t* seq_ends, int64_t seq_len,
                                                                       int64_t n_seqs, T* out, int32_t* err_flags) {
  grid_dep_wait();
  grid_dep_launch();
  for (int64_t b = blockIdx.x; b < n_seqs; b += gridDim.x) {
    const int64_t end = seq_ends ? static_cast<int64_t>(seq_ends[b]) : (b + 1) * seq_len;
    const bool ok = end >= 1 && end <= rows;
    if (!ok && threadIdx.x == 0) set_flag(err_flags, KLLM_B200_FLAG_BAD_SEQ_END);
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      out[b * cols + c] = ok ? x[(end - 1) * cols + c] : from_f<T>(0.0f);
    }
  }
}

template <typename TI, typename TO>
int launch_embedding_generic(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n,
                             void* out, int32_t* err_flags, const LaunchOpts& o) {
  auto k = embedding_generic_kernel<TI, TO>;
  const unsigned grid = persistent_grid(k, kThreads, 0, 1, n);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<const TI*>(table), vocab, hidden,
                              ids, n, static_cast<TO*>(out), err_flags),
                       "embedding");
}

}  // namespace

int embedding(const void* table, int64_t vocab, int64_t hidden, int table_dtype, const int32_t* ids,
              int64_t n_tokens, void* out, int out_dtype, int32_t* err_flags, const LaunchOpts& o) {
  if (vocab < 0 || hidden < 0 || n_tokens < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "embedding: negative size");
  if (n_tokens == 0 || hidden == 0) return KLLM_B200_OK;
  if (!table || !ids || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "embedding: null pointer");
  if (!is_float_dtype(table_dtype) || !is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "embedding: dtypes %d/%d not supported", table_dtype, out_dtype);
  }
  const int64_t row_bytes = hidden * dtype_size(table_dtype);
  if (table_dtype == out_dtype && row_bytes % 16 == 0 && aligned16(table) && aligned16(out) &&
      row_bytes / 16 < (int64_t)1 << 30) {
    const unsigned grid = persistent_grid(embedding_vec_kernel, kThreads, 0, kWarps, n_tokens);
    return launch_status(launch(embedding_vec_kernel, grid, kThreads, 0, o.stream, o.pdl,
                                static_cast<const uint4*>(table), vocab, ids, n_tokens, static_cast<uint4*>(out),
                                static_cast<int>(row_bytes / 16), err_flags),
                         "embedding");
  }
  if (table_dtype == KLLM_B200_F16) {
    return out_dtype == KLLM_B200_F16
               ? launch_embedding_generic<__half, __half>(table, vocab, hidden, ids, n_tokens, out, err_flags, o)
               : launch_embedding_generic<__half, float>(table, vocab, hidden, ids, n_tokens, out, err_flags, o);
  }
  return out_dtype == KLLM_B200_F16
             ? launch_embedding_generic<float, __half>(table, vocab, hidden, ids, n_tokens, out, err_flags, o)
             : launch_embedding_generic<float, float>(table, vocab, hidden, ids, n_tokens, out, err_flags, o);
}

int embedding_host_ids(const void* table, int64_t vocab, int64_t hidden, int table_dtype, const int32_t* host_ids,
                       int64_t n_tokens, void* out, int out_dtype, int32_t* err_flags, const LaunchOpts& o) {
  if (vocab < 0 || hidden < 0 || n_tokens < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "embedding_host_ids: negative size");
  }
  if (n_tokens == 0 || hidden == 0) return KLLM_B200_OK;
  if (!table || !host_ids || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "embedding_host_ids: null pointer");
  if (!is_float_dtype(table_dtype) || !is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "embedding_host_ids: dtypes %d/%d not supported", table_dtype, out_dtype);
  }
  const int64_t row_bytes = hidden * dtype_size(table_dtype);
  const int64_t out_row_bytes = hidden * dtype_size(out_dtype);
  const bool vec = table_dtype == out_dtype && row_bytes % 16 == 0 && aligned16(table) && aligned16(out) &&
                   row_bytes / 16 < (int64_t)1 << 30;
  ParamIds a;
  a.table = table;
  a.err_flags = err_flags;
  a.vocab = vocab;
  a.hidden = hidden;
  a.nvec = vec ? static_cast<int>(row_bytes / 16) : 0;
  for (int64_t start = 0; start < n_tokens; start += KLLM_B200_PARAM_IDS) {
    const int64_t left = n_tokens - start;
    a.n = static_cast<int>(left < KLLM_B200_PARAM_IDS ? left : KLLM_B200_PARAM_IDS);
    std::memcpy(a.ids, host_ids + start, static_cast<size_t>(a.n) * sizeof(int32_t));
    a.out = static_cast<char*>(out) + start * out_row_bytes;
    cudaError_t err;
    if (vec) {
      const unsigned grid = persistent_grid(embedding_param_vec_kernel, kThreads, 0, kWarps, a.n);
      err = launch(embedding_param_vec_kernel, grid, kThreads, 0, o.stream, o.pdl, a);
    } else {
      void (*k)(ParamIds);
      if (table_dtype == KLLM_B200_F16) {
        k = out_dtype == KLLM_B200_F16 ? embedding_param_generic_kernel<__half, __half>
                                       : embedding_param_generic_kernel<__half, float>;
      } else {
        k = out_dtype == KLLM_B200_F16 ? embedding_param_generic_kernel<float, __half>
                                       : embedding_param_generic_kernel<float, float>;
      }
      const unsigned grid = persistent_grid(k, kThreads, 0, 1, a.n);
      err = launch(k, grid, kThreads, 0, o.stream, o.pdl, a);
    }
    const int rc = launch_status(err, "embedding_host_ids");
    if (rc != KLLM_B200_OK) return rc;
  }
  return KLLM_B200_OK;
}

int select_last_rows(const void* x, int64_t rows, int64_t cols, const int32_t* seq_ends, int64_t seq_len,
                     int64_t n_seqs, void* out, int dtype, int32_t* err_flags, const LaunchOpts& o) {
  if (rows < 0 || cols < 0 || n_seqs < 0 || seq_len < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "select_last_rows: negative size");
  }
  if (n_seqs == 0 || cols == 0) return KLLM_B200_OK;
  if (!x || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "select_last_rows: null pointer");
  if (!is_float_dtype(dtype)) return fail(KLLM_B200_ERR_DTYPE, "select_last_rows: dtype %d not supported", dtype);
  if (seq_ends == nullptr && n_seqs * seq_len > rows) {
    return fail(KLLM_B200_ERR_SHAPE, "select_last_rows: %lld sequences of %lld rows exceed %lld rows",
                (long long)n_seqs, (long long)seq_len, (long long)rows);
  }
  const int64_t row_bytes = cols * dtype_size(dtype);
  if (row_bytes % 16 == 0 && aligned16(x) && aligned16(out) && row_bytes / 16 < (int64_t)1 << 30) {
    const unsigned grid = persistent_grid(select_rows_vec_kernel, kThreads, 0, kWarps, n_seqs);
    return launch_status(launch(select_rows_vec_kernel, grid, kThreads, 0, o.stream, o.pdl,
                                static_cast<const uint4*>(x), rows, seq_ends, seq_len, n_seqs,
                                static_cast<uint4*>(out), static_cast<int>(row_bytes / 16), err_flags),
                         "select_last_rows");
  }
  if (dtype == KLLM_B200_F16) {
    auto k = select_rows_generic_kernel<__half>;
    const unsigned grid = persistent_grid(k, kThreads, 0, 1, n_seqs);
    return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<const __half*>(x), rows, cols,
                                seq_ends, seq_len, n_seqs, static_cast<__half*>(out), err_flags),
                         "select_last_rows");
  }
  auto k = select_rows_generic_kernel<float>;
  const unsigned grid = persistent_grid(k, kThreads, 0, 1, n_seqs);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<const float*>(x), rows, cols,
                              seq_ends, seq_len, n_seqs, static_cast<float*>(out), err_flags),
                       "select_last_rows");
}

}  // namespace kb

extern "C" int kllm_b200_embedding(const void* table, int64_t vocab, int64_t hidden, int table_dtype,
                                   const int32_t* ids, int64_t n_tokens, void* out, int out_dtype,
                                   int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::embedding(table, vocab, hidden, table_dtype, ids, n_tokens, out, out_dtype, err_flags, o);
}

extern "C" int kllm_b200_embedding_host_ids(const void* table, int64_t vocab, int64_t hidden, int table_dtype,
                                            const int32_t* host_ids, int64_t n_tokens, void* out, int out_dtype,
                                            int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::embedding_host_ids(table, vocab, hidden, table_dtype, host_ids, n_tokens, out, out_dtype, err_flags,
                                o);
}

extern "C" int kllm_b200_select_last_rows(const void* x, int64_t rows, int64_t cols, const int32_t* seq_ends,
                                          int64_t seq_len, int64_t n_seqs, void* out, int dtype, int32_t* err_flags,
                                          void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::select_last_rows(x, rows, cols, seq_ends, seq_len, n_seqs, out, dtype, err_flags, o);
}

extern "C" int kllm_b200_select_last_row(const void* x, int64_t rows, int64_t cols, void* out, int dtype,
                                         void* stream) {
  if (rows < 1) return kb::fail(KLLM_B200_ERR_SHAPE, "select_last_row: rows must be positive");
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::select_last_rows(x, rows, cols, nullptr, rows, 1, out, dtype, nullptr, o);
}
