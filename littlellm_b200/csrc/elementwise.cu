// elementwise.cu — SwiGLU, residual add and row-broadcast bias add.
//
// Hot path: fp16 with 16-byte aligned buffers -> grid-stride kernels moving
// 16 B per load (8 halves), UNROLL independent vectors per thread in flight,
// grid = one wave of resident CTAs. Other dtypes or alignments take the
// generic element-per-thread kernels (same arithmetic). SwiGLU asks L2 for a
// CTA's first gate and up vectors before its grid-dependency wait (a hint
// that returns no data).
#include "common.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t silu_mul_h2(uint32_t g, uint32_t u) {
  const float2 gf = h2_to_f2(g), uf = h2_to_f2(u);
  return f2_to_h2(silu(gf.x) * uf.x, silu(gf.y) * uf.y);
}

__device__ __forceinline__ uint4 silu_mul_h8(uint4 g, uint4 u) {
  return make_uint4(silu_mul_h2(g.x, u.x), silu_mul_h2(g.y, u.y), silu_mul_h2(g.z, u.z),
                    silu_mul_h2(g.w, u.w));
}

// out = silu(gate) * up over nvec 16-byte vectors plus a scalar tail.
template <int UNROLL>
__global__ void __launch_bounds__(kThreads) silu_mul_f16_kernel(const __half* __restrict__ gate,
                                                                const __half* __restrict__ up,
                                                                __half* __restrict__ out, int64_t n) {
  const int64_t nvec = n >> 3;
  const uint4* g = reinterpret_cast<const uint4*>(gate);
  const uint4* u = reinterpret_cast<const uint4*>(up);
  uint4* y = reinterpret_cast<uint4*>(out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // this CTA's first gate and up vectors into L2 while the previous kernel
  // drains (a hint; they are read after the wait)
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      const int64_t v0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + k * stride;
      if (v0 < nvec) {
        const int64_t cnt = nvec - v0 < blockDim.x ? nvec - v0 : blockDim.x;
        prefetch_l2_bulk(g + v0, static_cast<uint32_t>(cnt * 16));
        prefetch_l2_bulk(u + v0, static_cast<uint32_t>(cnt * 16));
      }
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (UNROLL - 1) * stride < nvec; i += UNROLL * stride) {
    uint4 gv[UNROLL], uv[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
      gv[k] = ld_stream(g + i + k * stride);
      uv[k] = ld_stream(u + i + k * stride);
    }
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) st_plain(y + i + k * stride, silu_mul_h8(gv[k], uv[k]));
  }
  for (; i < nvec; i += stride) st_plain(y + i, silu_mul_h8(ld_stream(g + i), ld_stream(u + i)));
  if (blockIdx.x == 0) {
    for (int64_t j = (nvec << 3) + threadIdx.x; j < n; j += blockDim.x) {
      const float gf = __half2float(gate[j]);
      out[j] = __float2half_rn(silu(gf) * __half2float(up[j]));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) silu_mul_generic_kernel(const T* gate, const T* up, T* out,
                                                                    int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    out[i] = from_f<T>(silu(to_f(gate[i])) * to_f(up[i]));
  }
}

__device__ __forceinline__ uint32_t add_h2(uint32_t a, uint32_t b) {
  const float2 af = h2_to_f2(a), bf = h2_to_f2(b);
  return f2_to_h2(af.x + bf.x, af.y + bf.y);
}

__device__ __forceinline__ uint4 add_h8(uint4 a, uint4 b) {
  return make_uint4(add_h2(a.x, b.x), add_h2(a.y, b.y), add_h2(a.z, b.z), add_h2(a.w, b.w));
}

// x += y (fp16, vectorised).
__global__ void __launch_bounds__(kThreads) add_f16_kernel(__half* __restrict__ x, const __half* __restrict__ y,
                                                           int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t nvec = n >> 3;
  uint4* xv = reinterpret_cast<uint4*>(x);
  const uint4* yv = reinterpret_cast<const uint4*>(y);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    const uint4 a0 = ld_cg(xv + i), b0 = ld_stream(yv + i);
    const uint4 a1 = ld_cg(xv + i + stride), b1 = ld_stream(yv + i + stride);
    st_plain(xv + i, add_h8(a0, b0));
    st_plain(xv + i + stride, add_h8(a1, b1));
  }
  for (; i < nvec; i += stride) st_plain(xv + i, add_h8(ld_cg(xv + i), ld_stream(yv + i)));
  if (blockIdx.x == 0) {
    for (int64_t j = (nvec << 3) + threadIdx.x; j < n; j += blockDim.x) {
      x[j] = __float2half_rn(__half2float(x[j]) + __half2float(y[j]));
    }
  }
}

template <typename TX, typename TY>
__global__ void __launch_bounds__(kThreads) add_generic_kernel(TX* x, const TY* y, int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    x[i] = from_f<TX>(to_f(x[i]) + to_f(y[i]));
  }
}

// x[r, c] += bias[c] over a [rows, cols] matrix, cols % 8 == 0, fp16 x.
template <typename TB>
__global__ void __launch_bounds__(kThreads) add_bias_f16_kernel(__half* __restrict__ x,
                                                                const TB* __restrict__ bias,
                                                                int64_t rows, int64_t cols) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t vec_per_row = cols >> 3;
  const int64_t nvec = rows * vec_per_row;
  uint4* xv = reinterpret_cast<uint4*>(x);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const int64_t c0 = (i % vec_per_row) << 3;
    const uint4 a = ld_cg(xv + i);
    float b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) b[k] = to_f(bias[c0 + k]);
    const float2 a0 = h2_to_f2(a.x), a1 = h2_to_f2(a.y), a2 = h2_to_f2(a.z), a3 = h2_to_f2(a.w);
    st_plain(xv + i, make_uint4(f2_to_h2(a0.x + b[0], a0.y + b[1]), f2_to_h2(a1.x + b[2], a1.y + b[3]),
                                f2_to_h2(a2.x + b[4], a2.y + b[5]), f2_to_h2(a3.x + b[6], a3.y + b[7])));
  }
}

template <typename TX, typename TB>
__global__ void __launch_bounds__(kThreads) add_bias_generic_kernel(TX* x, const TB* bias, int64_t rows,
                                                                    int64_t cols) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t n = rows * cols;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    x[i] = from_f<TX>(to_f(x[i]) + to_f(bias[i % cols]));
  }
}

template <typename Kernel, typename... Args>
int run_generic(Kernel k, int64_t n, const LaunchOpts& o, const char* what, Args... args) {
  const unsigned grid = persistent_grid(k, kThreads, 0, kThreads * 4, n);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, args...), what);
}

}  // namespace

int silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype, const LaunchOpts& o) {
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "silu_mul: negative size %lld", (long long)n);
  if (n == 0) return KLLM_B200_OK;
  if (!gate || !up || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "silu_mul: null pointer");
  if (dtype == KLLM_B200_F16) {
    if (aligned16(gate) && aligned16(up) && aligned16(out)) {
      auto k = silu_mul_f16_kernel<2>;
      const unsigned grid = persistent_grid(k, kThreads, 0, kThreads * 2, (n >> 3) + 1);
      return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<const __half*>(gate),
                                  static_cast<const __half*>(up), static_cast<__half*>(out), n),
                           "silu_mul");
    }
    return run_generic(silu_mul_generic_kernel<__half>, n, o, "silu_mul", static_cast<const __half*>(gate),
                       static_cast<const __half*>(up), static_cast<__half*>(out), n);
  }
  if (dtype == KLLM_B200_F32) {
    return run_generic(silu_mul_generic_kernel<float>, n, o, "silu_mul", static_cast<const float*>(gate),
                       static_cast<const float*>(up), static_cast<float*>(out), n);
  }
  return fail(KLLM_B200_ERR_DTYPE, "silu_mul: dtype %d not supported (F32/F16)", dtype);
}

int add_inplace(void* x, const void* y, int64_t n, int x_dtype, int y_dtype, const LaunchOpts& o) {
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "add_inplace: negative size");
  if (n == 0) return KLLM_B200_OK;
  if (!x || !y) return fail(KLLM_B200_ERR_INVALID_ARG, "add_inplace: null pointer");
  if (!is_float_dtype(x_dtype) || !is_float_dtype(y_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "add_inplace: dtypes %d/%d not supported", x_dtype, y_dtype);
  }
  if (x_dtype == KLLM_B200_F16 && y_dtype == KLLM_B200_F16) {
    if (aligned16(x) && aligned16(y)) {
      const unsigned grid = persistent_grid(add_f16_kernel, kThreads, 0, kThreads * 2, (n >> 3) + 1);
      return launch_status(launch(add_f16_kernel, grid, kThreads, 0, o.stream, o.pdl, static_cast<__half*>(x),
                                  static_cast<const __half*>(y), n),
                           "add_inplace");
    }
    return run_generic(add_generic_kernel<__half, __half>, n, o, "add_inplace", static_cast<__half*>(x),
                       static_cast<const __half*>(y), n);
  }
  if (x_dtype == KLLM_B200_F16) {
    return run_generic(add_generic_kernel<__half, float>, n, o, "add_inplace", static_cast<__half*>(x),
                       static_cast<const float*>(y), n);
  }
  if (y_dtype == KLLM_B200_F16) {
    return run_generic(add_generic_kernel<float, __half>, n, o, "add_inplace", static_cast<float*>(x),
                       static_cast<const __half*>(y), n);
  }
  return run_generic(add_generic_kernel<float, float>, n, o, "add_inplace", static_cast<float*>(x),
                     static_cast<const float*>(y), n);
}

int add_bias_inplace(void* x, const void* bias, int64_t rows, int64_t cols, int x_dtype, int bias_dtype,
                     const LaunchOpts& o) {
  if (bias == nullptr) return KLLM_B200_OK;  // reference: a null bias is a no-op
  if (rows < 0 || cols < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "add_bias_inplace: negative size");
  if (rows == 0 || cols == 0) return KLLM_B200_OK;
  if (!x) return fail(KLLM_B200_ERR_INVALID_ARG, "add_bias_inplace: null x");
  if (!is_float_dtype(x_dtype) || !is_float_dtype(bias_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "add_bias_inplace: dtypes %d/%d not supported", x_dtype, bias_dtype);
  }
  const int64_t n = rows * cols;
  if (x_dtype == KLLM_B200_F16 && cols % 8 == 0 && aligned16(x)) {
    if (bias_dtype == KLLM_B200_F16) {
      auto k = add_bias_f16_kernel<__half>;
      const unsigned grid = persistent_grid(k, kThreads, 0, kThreads, n >> 3);
      return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<__half*>(x),
                                  static_cast<const __half*>(bias), rows, cols),
                           "add_bias_inplace");
    }
    auto k = add_bias_f16_kernel<float>;
    const unsigned grid = persistent_grid(k, kThreads, 0, kThreads, n >> 3);
    return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<__half*>(x),
                                static_cast<const float*>(bias), rows, cols),
                         "add_bias_inplace");
  }
  if (x_dtype == KLLM_B200_F16) {
    if (bias_dtype == KLLM_B200_F16)
      return run_generic(add_bias_generic_kernel<__half, __half>, n, o, "add_bias_inplace",
                         static_cast<__half*>(x), static_cast<const __half*>(bias), rows, cols);
    return run_generic(add_bias_generic_kernel<__half, float>, n, o, "add_bias_inplace", static_cast<__half*>(x),
                       static_cast<const float*>(bias), rows, cols);
  }
  if (bias_dtype == KLLM_B200_F16)
    return run_generic(add_bias_generic_kernel<float, __half>, n, o, "add_bias_inplace", static_cast<float*>(x),
                       static_cast<const __half*>(bias), rows, cols);
  return run_generic(add_bias_generic_kernel<float, float>, n, o, "add_bias_inplace", static_cast<float*>(x),
                     static_cast<const float*>(bias), rows, cols);
}

}  // namespace kb

extern "C" int kllm_b200_silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype,
                                  void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::silu_mul(gate, up, out, n, dtype, o);
}

extern "C" int kllm_b200_add_inplace(void* x, const void* y, int64_t n, int x_dtype, int y_dtype,
                                     void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::add_inplace(x, y, n, x_dtype, y_dtype, o);
}

extern "C" int kllm_b200_add_bias_inplace(void* x, const void* bias, int64_t rows, int64_t cols,
                                          int x_dtype, int bias_dtype, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::add_bias_inplace(x, bias, rows, cols, x_dtype, bias_dtype, o);
}
