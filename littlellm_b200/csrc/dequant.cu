// dequant.cu — INT8 per-tensor weight dequantisation.
//
// out_dtype F32: out = float(q) * scale, the reference GPU op
//   (src/op/cuda/quantize.cu:47-52,110-121) and cpu::dequantize_int8
//   (src/op/cpu/quantize.cpp:37-48).
// out_dtype F16: the reference weight loader's result
//   (src/model/weights.cpp:139-148): the fp32 product rounded by the
//   project's own float_to_half (src/base/half.cpp:38-61), bit for bit.
//
// With one scale per tensor the fp16 result is a function of the int8 byte
// alone, so each CTA evaluates the reference rounding for all 256 byte
// values once and the streaming loop becomes a table lookup. The table is
// replicated per lane (lut[byte][lane], 32 KB) so the 32 lanes of a warp
// always read 32 different banks: no bank conflicts whatever the data. The
// stream itself moves 16 int8 in (one 16-byte load) and 16 fp16 out (two
// 16-byte stores) per vector.
#include "common.cuh"

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

__global__ void __launch_bounds__(kThreads) dequant_f16_kernel(const int8_t* __restrict__ q,
                                                               const float* __restrict__ scale,
                                                               __half* __restrict__ out, int64_t n) {
  __shared__ uint32_t lut[256 * 32];
  grid_dep_wait();
  grid_dep_launch();
  const float s = __ldg(scale);
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
  for (; i + stride < nvec; i += 2 * stride) {
    const uint4 w0 = ld_stream(src + i);
    const uint4 w1 = ld_stream(src + i + stride);
    uint4 a0, a1, b0, b1;
    lut16(my, w0, a0, a1);
    lut16(my, w1, b0, b1);
    st_plain(dst + 2 * i, a0);
    st_plain(dst + 2 * i + 1, a1);
    st_plain(dst + 2 * (i + stride), b0);
    st_plain(dst + 2 * (i + stride) + 1, b1);
  }
  for (; i < nvec; i += stride) {
    uint4 a0, a1;
    lut16(my, ld_stream(src + i), a0, a1);
    st_plain(dst + 2 * i, a0);
    st_plain(dst + 2 * i + 1, a1);
  }
  if (blockIdx.x == 0) {
    unsigned short* o16 = reinterpret_cast<unsigned short*>(out);
    for (int64_t j = (nvec << 4) + threadIdx.x; j < n; j += blockDim.x) {
      o16[j] = static_cast<unsigned short>(my[(static_cast<uint32_t>(static_cast<uint8_t>(q[j]))) << 5]);
    }
  }
}

__global__ void __launch_bounds__(kThreads) dequant_f32_kernel(const int8_t* __restrict__ q,
                                                               const float* __restrict__ scale,
                                                               float* __restrict__ out, int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const float s = __ldg(scale);
  const int64_t nvec = n >> 4;
  const uint4* src = reinterpret_cast<const uint4*>(q);
  float4* dst = reinterpret_cast<float4*>(out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 w = ld_stream(src + i);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t x = words[k];
      dst[4 * i + k] = make_float4(dequant_value(x & 0xffu, s), dequant_value((x >> 8) & 0xffu, s),
                                   dequant_value((x >> 16) & 0xffu, s), dequant_value(x >> 24, s));
    }
  }
  if (blockIdx.x == 0) {
    for (int64_t j = (nvec << 4) + threadIdx.x; j < n; j += blockDim.x) {
      out[j] = __fmul_rn(static_cast<float>(q[j]), s);
    }
  }
}

// Unaligned buffers: element per thread, same arithmetic.
template <bool F16>
__global__ void __launch_bounds__(kThreads) dequant_generic_kernel(const int8_t* q, const float* scale, void* out,
                                                                   int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const float s = __ldg(scale);
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

}  // namespace

int dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n, int out_dtype,
                    const LaunchOpts& o) {
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8: negative size");
  if (n == 0) return KLLM_B200_OK;
  if (!data || !scale || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8: null pointer");
  if (!is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "dequantize_int8: output dtype %d not supported (F32/F16)", out_dtype);
  }
  const bool vec = aligned16(data) && aligned16(out);
  if (out_dtype == KLLM_B200_F16 && vec) {
    const unsigned grid = persistent_grid(dequant_f16_kernel, kThreads, 0, kThreads * 2, (n >> 4) + 1);
    return launch_status(launch(dequant_f16_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale,
                                static_cast<__half*>(out), n),
                         "dequantize_int8");
  }
  if (out_dtype == KLLM_B200_F32 && vec) {
    const unsigned grid = persistent_grid(dequant_f32_kernel, kThreads, 0, kThreads, (n >> 4) + 1);
    return launch_status(launch(dequant_f32_kernel, grid, kThreads, 0, o.stream, o.pdl, data, scale,
                                static_cast<float*>(out), n),
                         "dequantize_int8");
  }
  auto k = out_dtype == KLLM_B200_F16 ? dequant_generic_kernel<true> : dequant_generic_kernel<false>;
  const unsigned grid = persistent_grid(k, kThreads, 0, kThreads * 4, n);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, data, scale, out, n), "dequantize_int8");
}

}  // namespace kb

extern "C" int kllm_b200_dequantize_int8(const int8_t* data, const float* scale, void* out, int64_t n,
                                         int out_dtype, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::dequantize_int8(data, scale, out, n, out_dtype, o);
}
