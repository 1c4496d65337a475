// dequant.cu — INT8 per-tensor weight dequantisation.
//
// out_dtype F32: out = float(q) * scale, the reference GPU op
//   (src/op/cuda/quantize.cu:47-52,110-121) and cpu::dequantize_int8
//   (src/op/cpu/quantize.cpp:37-48).
// out_dtype F16: the reference weight loader's result
//   (src/model/weights.cpp:139-148): the fp32 product rounded by the
//   project's own float_to_half (src/base/half.cpp:38-61), bit for bit.
// Opt-in: fp16 rounded to nearest even (IEEE), with a count of the values
//   where that differs from the reference rounding.
//
// With one scale per tensor the fp16 result is a function of the int8 byte
// alone, so each CTA evaluates the reference rounding for all 256 byte
// values once and the streaming loop becomes a table lookup. The table is
// replicated per lane (lut[byte][lane], 32 KB) so the 32 lanes of a warp
// always read 32 different banks: no bank conflicts whatever the data. The
// stream itself moves 16 int8 in (one 16-byte load) and 16 fp16 out (two
// 16-byte stores) per vector.
#include "ops.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;

// The reference float_to_half (src/base/half.cpp:38-61) on fp32 bits. The
// steps must match for bit-exact results: add half an fp16 ulp and
// truncate (ties away from zero); in the normal range the rounded fraction is
// OR-ed into the exponent field, so a carry out of the fraction is dropped
// when the exponent is odd; fp16 exponent >= 31 (inf, NaN, overflow) -> inf;
// magnitudes below 2^-25 -> signed zero.
__device__ __forceinline__ uint32_t ref_float_to_half(float value) {
  const uint32_t bits = __float_as_uint(value);
  const uint32_t sign16 = (bits >> 16) & 0x8000u;
  const int32_t exp16 = static_cast<int32_t>((bits >> 23) & 0xffu) - 112;
  const uint32_t frac = bits & 0x007fffffu;
  if (exp16 <= 0) {
    if (exp16 < -10) return sign16;
    const uint32_t denorm = (frac | 0x00800000u) >> static_cast<uint32_t>(1 - exp16);
    return sign16 | ((denorm + 0x1000u) >> 13);
  }
  if (exp16 >= 31) return sign16 | 0x7c00u;
  return sign16 | (static_cast<uint32_t>(exp16) << 10) | ((frac + 0x1000u) >> 13);
}

__device__ __forceinline__ float dequant_value(uint32_t byte, float s) {
  return __fmul_rn(static_cast<float>(static_cast<int8_t>(byte)), s);
}

// Two fp16 results (bytes 0/1 or 2/3 of w) packed low-first.
__device__ __forceinline__ uint32_t lut2(const uint32_t* my, uint32_t w, int shift) {
  const uint32_t lo = my[((w >> shift) & 0xffu) << 5];
  const uint32_t hi = my[((w >> (shift + 8)) & 0xffu) << 5];
  return lo | (hi << 16);
}

__device__ __forceinline__ void lut16(const uint32_t* my, uint4 w, uint4& o0, uint4& o1) {
  o0 = make_uint4(lut2(my, w.x, 0), lut2(my, w.x, 16), lut2(my, w.y, 0), lut2(my, w.y, 16));
  o1 = make_uint4(lut2(my, w.z, 0), lut2(my, w.z, 16), lut2(my, w.w, 0), lut2(my, w.w, 16));
}

// `scale` points to the per-tensor scale in device memory; when it is null
// the scale comes by value in `scale_value` (the weight loader reads it from
// the file).
__global__ void __launch_bounds__(kThreads) dequant_f16_kernel(const int8_t* __restrict__ q,
                                                               const float* __restrict__ scale, float scale_value,
                                                               __half* __restrict__ out, int64_t n) {
  __shared__ uint32_t lut[256 * 32];
  grid_dep_wait();
  grid_dep_launch();
  const float s = scale != nullptr ? __ldg(scale) : scale_value;
  {
    // Thread b evaluates byte value b and writes its 32 lane copies,
    // rotating the lane so a warp's 32 stores hit 32 different banks.
    const uint32_t b = threadIdx.x;
    const uint32_t h = ref_float_to_half(dequant_value(b, s));
#pragma unroll 8
    for (int l = 0; l < 32; ++l) lut[b * 32 + ((l + b) & 31)] = h;
  }
  __syncthreads();
  const uint32_t* my = lut + (threadIdx.x & 31);

  const int64_t nvec = n >> 4;
  const uint4* src = reinterpret_cast<const uint4*>(q);
  uint4* dst = reinterpret_cast<uint4*>(out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // a thread's 16 results are 32 contiguous bytes: one 32-byte store when the
  // output is 32-byte aligned (a warp then writes 1 KB contiguously), else two
  const bool out32 = (reinterpret_cast<uintptr_t>(out) & 31u) == 0;
  auto store16 = [&](int64_t v, uint4 lo, uint4 hi) {
    if (out32) {
      st_plain32(dst + 2 * v, lo, hi);
    } else {
      st_plain(dst + 2 * v, lo);
      st_plain(dst + 2 * v + 1, hi);
    }
  };
  for (; i + stride < nvec; i += 2 * stride) {
    const uint4 w0 = ld_stream(src + i);
    const uint4 w1 = ld_stream(src + i + stride);
    uint4 a0, a1, b0, b1;
    lut16(my, w0, a0, a1);
    lut16(my, w1, b0, b1);
    store16(i, a0, a1);
    store16(i + stride, b0, b1);
  }
  for (; i < nvec; i += stride) {
    uint4 a0, a1;
    lut16(my, ld_stream(src + i), a0, a1);
    store16(i, a0, a1);
  }
  if (blockIdx.x == 0) {
    unsigned short* o16 = reinterpret_cast<unsigned short*>(out);
    for (int64_t j = (nvec << 4) + threadIdx.x; j < n; j += blockDim.x) {
      o16[j] = static_cast<unsigned short>(my[(static_cast<uint32_t>(static_cast<uint8_t>(q[j]))) << 5]);
    }
  }
}

// 4-byte load through the non-coherent path, not allocated in L1.
__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// fp32 output: one 4-value word per thread and float4 store, so a warp reads
// 128 contiguous bytes and writes 512 contiguous bytes per instruction; four
// words in flight per thread (a CTA covers 4 x 256 consecutive words per
// step).
constexpr int kF32Words = 4;

__global__ void __launch_bounds__(kThreads) dequant_f32_kernel(const int8_t* __restrict__ q,
                                                               const float* __restrict__ scale, float scale_value,
                                                               float* __restrict__ out, int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const float s = scale != nullptr ? __ldg(scale) : scale_value;
  const int64_t nw = n >> 2;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(q);
  float4* dst = reinterpret_cast<float4*>(out);
  const int64_t chunk = static_cast<int64_t>(blockDim.x) * kF32Words;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * chunk; base < nw; base += static_cast<int64_t>(gridDim.x) * chunk) {
    uint32_t w[kF32Words];
#pragma unroll
    for (int k = 0; k < kF32Words; ++k) {
      const int64_t i = base + k * blockDim.x + threadIdx.x;
      if (i < nw) w[k] = ld_stream_u32(src + i);
    }
#pragma unroll
    for (int k = 0; k < kF32Words; ++k) {
      const int64_t i = base + k * blockDim.x + threadIdx.x;
      if (i < nw) {
        const uint32_t x = w[k];
        dst[i] = make_float4(dequant_value(x & 0xffu, s), dequant_value((x >> 8) & 0xffu, s),
                             dequant_value((x >> 16) & 0xffu, s), dequant_value(x >> 24, s));
      }
    }
  }
  if (blockIdx.x == 0) {
    for (int64_t j = (nw << 2) + threadIdx.x; j < n; j += blockDim.x) {
      out[j] = __fmul_rn(static_cast<float>(q[j]), s);
    }
  }
}

// Unaligned buffers: element per thread, same arithmetic.
template <bool F16>
__global__ void __launch_bounds__(kThreads) dequant_generic_kernel(const int8_t* q, const float* scale,
                                                                   float scale_value, void* out, int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const float s = scale != nullptr ? __ldg(scale) : scale_value;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float val = __fmul_rn(static_cast<float>(q[i]), s);
    if (F16) {
      static_cast<unsigned short*>(out)[i] = static_cast<unsigned short>(ref_float_to_half(val));
    } else {
      static_cast<float*>(out)[i] = val;
    }
  }
}

// ---- opt-in IEEE rounding --------------------------------------------------
//
// The same dequant with round-to-nearest-even fp16 (__float2half_rn) in place
// of the reference loader's rounding, for callers that want IEEE results.
// Each table entry holds the RNE half in its low 16 bits and, in bit 16,
// whether it differs from the reference rounding of the same byte, so one
// lookup gives both the output and that element's contribution to the count
// of values the two roundings disagree on.

__device__ __forceinline__ uint32_t rne_entry(uint32_t b, float s) {
  const float v = dequant_value(b, s);
  const uint32_t rne = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v)));
  return rne | ((rne != ref_float_to_half(v)) ? 0x10000u : 0u);
}

// Two fp16 results (bytes 0/1 or 2/3 of w) packed low-first; their mismatch
// flags are added to `count`.
__device__ __forceinline__ uint32_t rne2(const uint32_t* my, uint32_t w, int shift, uint32_t& count) {
  const uint32_t lo = my[((w >> shift) & 0xffu) << 5];
  const uint32_t hi = my[((w >> (shift + 8)) & 0xffu) << 5];
  count += (lo >> 16) + (hi >> 16);
  return (lo & 0xffffu) | (hi << 16);
}

__global__ void __launch_bounds__(kThreads) dequant_f16_rne_kernel(const int8_t* __restrict__ q,
                                                                   const float* __restrict__ scale,
                                                                   __half* __restrict__ out, int64_t n,
                                                                   unsigned long long* mismatches) {
  __shared__ uint32_t lut[256 * 32];
  grid_dep_wait();
  grid_dep_launch();
  const float s = __ldg(scale);
  {
    const uint32_t b = threadIdx.x;
    const uint32_t e = rne_entry(b, s);
#pragma unroll 8
    for (int l = 0; l < 32; ++l) lut[b * 32 + ((l + b) & 31)] = e;
  }
  __syncthreads();
  const uint32_t* my = lut + (threadIdx.x & 31);
  uint32_t count = 0;
  const int64_t nvec = n >> 4;
  const uint4* src = reinterpret_cast<const uint4*>(q);
  uint4* dst = reinterpret_cast<uint4*>(out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 w = ld_stream(src + i);
    st_plain(dst + 2 * i, make_uint4(rne2(my, w.x, 0, count), rne2(my, w.x, 16, count), rne2(my, w.y, 0, count),
                                     rne2(my, w.y, 16, count)));
    st_plain(dst + 2 * i + 1, make_uint4(rne2(my, w.z, 0, count), rne2(my, w.z, 16, count),
                                         rne2(my, w.w, 0, count), rne2(my, w.w, 16, count)));
  }
  if (blockIdx.x == 0) {
    unsigned short* o16 = reinterpret_cast<unsigned short*>(out);
    for (int64_t j = (nvec << 4) + threadIdx.x; j < n; j += blockDim.x) {
      const uint32_t e = my[(static_cast<uint32_t>(static_cast<uint8_t>(q[j]))) << 5];
      o16[j] = static_cast<unsigned short>(e & 0xffffu);
      count += e >> 16;
    }
  }
  if (mismatches != nullptr) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) count += __shfl_xor_sync(0xffffffffu, count, off);
    if ((threadIdx.x & 31) == 0 && count != 0) atomicAdd(mismatches, static_cast<unsigned long long>(count));
  }
}

// Unaligned buffers: element per thread, same rounding and count.
__global__ void __launch_bounds__(kThreads) dequant_f16_rne_generic_kernel(const int8_t* q, const float* scale,
                                                                           unsigned short* out, int64_t n,
                                                                           unsigned long long* mismatches) {
  grid_dep_wait();
  grid_dep_launch();
  const float s = __ldg(scale);
  uint32_t count = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t e = rne_entry(static_cast<uint32_t>(static_cast<uint8_t>(q[i])), s);
    out[i] = static_cast<unsigned short>(e & 0xffffu);
    count += e >> 16;
  }
  if (mismatches != nullptr) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) count += __shfl_xor_sync(0xffffffffu, count, off);
    if ((threadIdx.x & 31) == 0 && count != 0) atomicAdd(mismatches, static_cast<unsigned long long>(count));
  }
}

// ---- many tensors in one launch -----------------------------------------
//
// The weight loader dequantises every INT8 record of a checkpoint
// (src/model/weights.cpp:95-154, one tensor at a time on the host). Here a
// whole batch of tensors is one persistent launch: each tensor is cut into
// chunks of kChunk int8 elements, the chunks of all tensors are numbered
// consecutively, and CTA b processes the contiguous chunk range
// [b * n / grid, (b + 1) * n / grid), so it meets only a few tensors and
// rebuilds its rounding table only when it crosses into the next one. The
// task table travels by value in the kernel parameters.

constexpr int kMaxTasks = 96;  // keeps the parameter block under the classic 4 KB limit
constexpr int kVecsPerThread = 4;
constexpr int kChunkVecs = kVecsPerThread * kThreads;  // 16-byte vectors per chunk
constexpr int64_t kChunk = 16 * kChunkVecs;    // int8 elements per chunk

struct DequantTask {
  const int8_t* q;
  const float* scale;
  void* out;
  int64_t n;            // elements
  int64_t first_chunk;  // index of the task's first chunk in the batch
};

struct DequantBatch {
  int n_tasks;
  int64_t n_chunks;
  DequantTask task[kMaxTasks];
};
static_assert(sizeof(DequantBatch) <= 4000, "kernel parameter block must stay below 4 KB");

__device__ __forceinline__ void build_lut(uint32_t* lut, float s) {
  const uint32_t b = threadIdx.x;
  const uint32_t h = ref_float_to_half(dequant_value(b, s));
#pragma unroll 8
  for (int l = 0; l < 32; ++l) lut[b * 32 + ((l + b) & 31)] = h;
}

template <bool F16>
__global__ void __launch_bounds__(kThreads) dequant_batched_kernel(const __grid_constant__ DequantBatch batch) {
  __shared__ uint32_t lut[256 * 32];
  grid_dep_wait();
  grid_dep_launch();
  const int64_t c_begin = batch.n_chunks * blockIdx.x / gridDim.x;
  const int64_t c_end = batch.n_chunks * (blockIdx.x + 1) / gridDim.x;
  if (c_begin >= c_end) return;
  // task holding chunk c_begin: last task whose first_chunk <= c_begin
  int lo = 0, hi = batch.n_tasks - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (batch.task[mid].first_chunk <= c_begin) lo = mid; else hi = mid - 1;
  }
  int ti = lo;
  float s = __ldg(batch.task[ti].scale);
  if (F16) build_lut(lut, s);
  __syncthreads();
  const uint32_t* my = lut + (threadIdx.x & 31);
  for (int64_t c = c_begin; c < c_end; ++c) {
    bool moved = false;
    while (ti + 1 < batch.n_tasks && batch.task[ti + 1].first_chunk <= c) {
      ++ti;
      moved = true;
    }
    if (moved) {
      s = __ldg(batch.task[ti].scale);
      if (F16) {
        __syncthreads();  // everyone is done with the previous table
        build_lut(lut, s);
        __syncthreads();
      }
    }
    const DequantTask& t = batch.task[ti];
    const int64_t e0 = (c - t.first_chunk) * kChunk;     // first element of this chunk
    // e0 * 2 bytes is a multiple of 32 (kChunk is), so the chunk's output is
    // 32-byte aligned exactly when the tensor's is
    const bool out32 = (reinterpret_cast<uintptr_t>(t.out) & 31u) == 0;
    const int64_t e1 = e0 + kChunk < t.n ? e0 + kChunk : t.n;
    const int64_t nvec = (e1 - e0) >> 4;
    const uint4* src = reinterpret_cast<const uint4*>(t.q + e0);
    uint4 w[kVecsPerThread];
#pragma unroll
    for (int k = 0; k < kVecsPerThread; ++k) {
      const int64_t i = threadIdx.x + k * kThreads;
      if (i < nvec) w[k] = ld_stream(src + i);
    }
#pragma unroll
    for (int k = 0; k < kVecsPerThread; ++k) {
      const int64_t i = threadIdx.x + k * kThreads;
      if (i >= nvec) continue;
      if (F16) {
        uint4 o0, o1;
        lut16(my, w[k], o0, o1);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(t.out) + e0);
        if (out32) {  // uniform per task: one 32-byte store per thread, 1 KB per warp
          st_plain32(dst + 2 * i, o0, o1);
        } else {
          st_plain(dst + 2 * i, o0);
          st_plain(dst + 2 * i + 1, o1);
        }
      } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(t.out) + e0);
        const uint32_t words[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const uint32_t x = words[m];
          dst[4 * i + m] = make_float4(dequant_value(x & 0xffu, s), dequant_value((x >> 8) & 0xffu, s),
                                       dequant_value((x >> 16) & 0xffu, s), dequant_value(x >> 24, s));
        }
      }
    }
    // scalar tail of the tensor's last chunk (fewer than 16 elements)
    for (int64_t j = e0 + (nvec << 4) + threadIdx.x; j < e1; j += blockDim.x) {
      if (F16) {
        static_cast<unsigned short*>(t.out)[j] =
            static_cast<unsigned short>(my[static_cast<uint32_t>(static_cast<uint8_t>(t.q[j])) << 5]);
      } else {
        static_cast<float*>(t.out)[j] = __fmul_rn(static_cast<float>(t.q[j]), s);
      }
    }
  }
}

}  // namespace

int dequantize_int8_impl(const int8_t* data, const float* scale, float scale_value, void* out, int64_t n,
                         int out_dtype, const LaunchOpts& o) {
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8: negative size");
  if (n == 0) return KLLM_B200_OK;
  if (!data || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8: null pointer");
  if (!is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "dequantize_int8: output dtype %d not supported (F32/F16)", out_dtype);
  }
  const bool vec = aligned16(data) && aligned16(out);
  if (out_dtype == KLLM_B200_F16 && vec) {
    const unsigned grid = persistent_grid(dequant_f16_kernel, kThreads, 0, kThreads * 2, (n >> 4) + 1);
    return launch_status(launch(dequant_f16_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale, scale_value,
                                static_cast<__half*>(out), n),
                         "dequantize_int8");
  }
  if (out_dtype == KLLM_B200_F32 && vec) {
    const unsigned grid = persistent_grid(dequant_f32_kernel, kThreads, 0, kThreads * kF32Words, (n >> 2) + 1);
    return launch_status(launch(dequant_f32_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale, scale_value,
                                static_cast<float*>(out), n),
                         "dequantize_int8");
  }
  auto k = out_dtype == KLLM_B200_F16 ? dequant_generic_kernel<true> : dequant_generic_kernel<false>;
  const unsigned grid = persistent_grid(k, kThreads, 0, kThreads * 4, n);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, data, scale, scale_value, out, n),
                       "dequantize_int8");
}

int dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n, int out_dtype,
                    const LaunchOpts& o) {
  if (n > 0 && !scale) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8: null scale");
  return dequantize_int8_impl(data, scale, 0.0f, out, n, out_dtype, o);
}

int dequantize_int8_value(const int8_t* data, float scale, void* out, int64_t n, int out_dtype,
                          const LaunchOpts& o) {
  return dequantize_int8_impl(data, nullptr, scale, out, n, out_dtype, o);
}

int dequantize_int8_rne(const int8_t* data, const float* scale, void* out, int64_t n,
                        unsigned long long* mismatches, const LaunchOpts& o) {
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_rne: negative size");
  if (n == 0) return KLLM_B200_OK;
  if (!data || !scale || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_rne: null pointer");
  if (aligned16(data) && aligned16(out)) {
    const unsigned grid = persistent_grid(dequant_f16_rne_kernel, kThreads, 0, kThreads * 2, (n >> 4) + 1);
    return launch_status(launch(dequant_f16_rne_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale,
                                static_cast<__half*>(out), n, mismatches),
                         "dequantize_int8_rne");
  }
  const unsigned grid = persistent_grid(dequant_f16_rne_generic_kernel, kThreads, 0, kThreads * 4, n);
  return launch_status(launch(dequant_f16_rne_generic_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale,
                              static_cast<unsigned short*>(out), n, mismatches),
                       "dequantize_int8_rne");
}

int dequantize_int8_batched(const int8_t* const* data, const float* const* scales, void* const* outs,
                            const int64_t* counts, int n_tensors, int out_dtype, const LaunchOpts& o) {
  if (n_tensors < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_batched: negative tensor count");
  if (n_tensors == 0) return KLLM_B200_OK;
  if (!data || !scales || !outs || !counts) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_batched: null array");
  }
  if (!is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "dequantize_int8_batched: output dtype %d not supported (F32/F16)", out_dtype);
  }
  for (int i = 0; i < n_tensors; ++i) {
    if (counts[i] < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_batched: tensor %d has negative size", i);
    if (counts[i] > 0 && (!data[i] || !scales[i] || !outs[i])) {
      return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_batched: tensor %d has a null pointer", i);
    }
  }
  DequantBatch batch;
  int i = 0;
  while (i < n_tensors) {
    batch.n_tasks = 0;
    batch.n_chunks = 0;
    // fill one launch with up to kMaxTasks aligned tensors; unaligned ones
    // go through the single-tensor entry point
    for (; i < n_tensors && batch.n_tasks < kMaxTasks; ++i) {
      if (counts[i] == 0) continue;
      if (!aligned16(data[i]) || !aligned16(outs[i])) {
        const int rc = dequantize_int8(data[i], scales[i], outs[i], counts[i], out_dtype, o);
        if (rc != KLLM_B200_OK) return rc;
        continue;
      }
      DequantTask& t = batch.task[batch.n_tasks++];
      t.q = data[i];
      t.scale = scales[i];
      t.out = outs[i];
      t.n = counts[i];
      t.first_chunk = batch.n_chunks;
      batch.n_chunks += (counts[i] + kChunk - 1) / kChunk;
    }
    if (batch.n_tasks == 0) continue;
    auto k = out_dtype == KLLM_B200_F16 ? dequant_batched_kernel<true> : dequant_batched_kernel<false>;
    const unsigned grid = persistent_grid(k, kThreads, 0, 1, batch.n_chunks);
    const int rc = launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, batch), "dequantize_int8_batched");
    if (rc != KLLM_B200_OK) return rc;
  }
  return KLLM_B200_OK;
}

}  // namespace kb

extern "C" int kllm_b200_dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n,
                                         int out_dtype, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::dequantize_int8(data, scale, out, n, out_dtype, o);
}

extern "C" int kllm_b200_dequantize_int8_rne(const int8_t* data, const float* scale, void* out, int64_t n,
                                             unsigned long long* mismatches, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::dequantize_int8_rne(data, scale, out, n, mismatches, o);
}

extern "C" int kllm_b200_dequantize_int8_batched(const int8_t* const* data, const float* const* scales,
                                                 void* const* outs, const int64_t* counts, int n_tensors,
                                                 int out_dtype, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::dequantize_int8_batched(data, scales, outs, counts, n_tensors, out_dtype, o);
}
