// common.cuh — shared host/device helpers of the kllm_b200 CUDA library.
//
// Host side: status reporting (thread-local message behind the C ABI's
// negative return codes), a per-device SM-count cache, occupancy-sized grids
// and a launcher that can attach programmatic dependent launch (PDL).
// Device side: 16-byte global loads/stores with cache hints, fp16 packing,
// warp reductions and the PDL grid-dependency controls.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kllm_b200.h"

namespace kb {

// ---------------------------------------------------------------------------
// Host: errors and launch helpers
// ---------------------------------------------------------------------------

// Records `message` (printf-style) as the calling thread's last error and
// returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Maps the launch status of the kernel just enqueued to a C-ABI code.
int launch_status(cudaError_t err, const char* what);

inline bool is_float_dtype(int dt) { return dt == KLLM_B200_F32 || dt == KLLM_B200_F16; }
inline int dtype_size(int dt) { return dt == KLLM_B200_F32 || dt == KLLM_B200_I32 ? 4 : dt == KLLM_B200_F16 ? 2 : 1; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

// Resident CTAs per SM for `kernel` at `threads` threads and `smem` bytes of
// dynamic shared memory (cached per (kernel, threads, smem); all devices of
// one box are the same part).
int resident_ctas_raw(const void* kernel, int threads, size_t smem);

template <typename Kernel>
int resident_ctas(Kernel kernel, int threads, size_t smem) {
  return resident_ctas_raw(reinterpret_cast<const void*>(kernel), threads, smem);
}

// Clusters of `cluster` CTAs of `kernel` that can be resident on the device at
// once (0 when none can be scheduled).
int active_clusters_raw(const void* kernel, int threads, size_t smem, int cluster);

// Opt `kernel` in to `smem` bytes of dynamic shared memory when that exceeds
// the 48 KB default (once per kernel and size).
cudaError_t allow_smem(const void* kernel, size_t smem);

// Grid for a grid-stride kernel: one full wave of resident CTAs, never more
// CTAs than work items.
template <typename Kernel>
unsigned persistent_grid(Kernel kernel, int threads, size_t smem, int64_t work_items_per_cta_unit,
                         int64_t work_items) {
  const int64_t wave = static_cast<int64_t>(sm_count()) * resident_ctas(kernel, threads, smem);
  int64_t need = (work_items + work_items_per_cta_unit - 1) / work_items_per_cta_unit;
  if (need < 1) need = 1;
  return static_cast<unsigned>(need < wave ? need : wave);
}

// Launches `kernel` on `stream`; with `pdl` the launch carries the
// programmatic-stream-serialization attribute, so it may begin while the
// previous kernel on the stream drains (kernels call grid_dep_wait() before
// touching memory the predecessor writes).
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch() with the grid divided into clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_clustered(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             bool pdl, int cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Whether the calling thread asked the individual entry points to launch
// with programmatic dependent launch (kllm_b200_set_pdl).
bool default_pdl();

// Launch options shared by the individual entry points and the chain runner.
struct LaunchOpts {
  cudaStream_t stream = nullptr;
  bool pdl = default_pdl();
  // Under PDL, read before the grid-dependency wait the inputs that no launch
  // of the chain writes (norm weights, q/k/v biases, positions, cache slots,
  // the embedding table and ids). Valid only when the launch directly before
  // on the stream does not write them; the chain executor sets it for every
  // launch after its first, since it knows what each of its launches writes.
  // An individual entry point cannot know what the caller launched before it,
  // so without this flag a kernel reads nothing before its wait.
  bool early_inputs = false;
  // add_rms_norm under PDL: the residual was last written two or more
  // launches back on this stream (the previous launch leaves it alone), so
  // its rows may be read before the grid-dependency wait. Every kernel of
  // this library triggers its dependents only after its own wait, so when a
  // launch starts, all launches two or more back have completed.
  bool early_residual = false;
};

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Wait until the grid this launch depends on (PDL) has completed and its
// writes are visible; a no-op for launches without the PDL attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next PDL launch on the stream to start scheduling its CTAs.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// 16-byte load through the non-coherent path, not allocated in L1: for
// inputs read exactly once.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte coherent load (for buffers the same kernel also writes).
__device__ __forceinline__ uint4 ld_cg(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte read-only load kept in L1 (small tensors reused by many rows).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// 16-byte store, streaming (evict-first): outputs not re-read by this kernel.
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Asks L2 to fetch [p, p + bytes) from memory (p 16-byte aligned, bytes a
// multiple of 16). A cache hint that returns no data: it may be issued before
// the grid-dependency wait for memory the previous kernel is still writing,
// since the loads after the wait read the coherent values either way.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Asks L2 for the line holding `p` (a hint, as above).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Pull the line holding `p` into L1 ahead of a later load.
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// 16-byte plain store.
__device__ __forceinline__ void st_plain(void* p, uint4 v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// 32-byte store of two 16-byte vectors (sm_100; `p` 32-byte aligned).
__device__ __forceinline__ void st_plain32(void* p, uint4 lo, uint4 hi) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(lo.x), "r"(lo.y), "r"(lo.z),
               "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}

inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

__device__ __forceinline__ float2 h2_to_f2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

__device__ __forceinline__ uint32_t f2_to_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// Eight fp16 values of a 16-byte vector as floats, and back (round to nearest even).
__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(f2_to_h2(f[0], f[1]), f2_to_h2(f[2], f[3]), f2_to_h2(f[4], f[5]), f2_to_h2(f[6], f[7]));
}

// fp16(x + b) for 8 packed fp16 lanes (four HADD2). This equals rounding the
// fp32 sum of the two values to fp16: that sum is itself a rounding of the
// exact sum, and fp32 carries 24 >= 2 * 11 + 2 significand bits, so the
// double rounding is innocuous for addition.
__device__ __forceinline__ uint4 hadd8(uint4 x, uint4 b) {
  auto add = [](uint32_t u, uint32_t v) {
    __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&u), *reinterpret_cast<const __half2*>(&v));
    return *reinterpret_cast<uint32_t*>(&r);
  };
  return make_uint4(add(x.x, b.x), add(x.y, b.y), add(x.z, b.z), add(x.w, b.w));
}

// RoPE pair rotation shared by every RoPE path (the fused bias+RoPE+KV
// kernel, rope_inplace, the QKV GEMM epilogue) so that they agree bit for bit:
// y1 = x1*c - x2*s, y2 = x2*c + x1*s, each as one fp32 product and one FMA.
__device__ __forceinline__ void rope_rotate(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = __fmaf_rn(x1, c, -__fmul_rn(x2, s));
  y2 = __fmaf_rn(x2, c, __fmul_rn(x1, s));
}

// Eight rotations (pairs i = 0..7) with the packed fp32x2 multiply / FMA of
// sm_100 (two pairs per instruction). Element by element the arithmetic is
// rope_rotate's: y1 = fma(x1, c, x2 * (-s)) where x2 * (-s) equals -(x2 * s)
// exactly in round-to-nearest, and y2 = fma(x2, c, x1 * s); `ns` holds -s.
__device__ __forceinline__ unsigned long long f32x2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f32x2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// Two fp32 products (round to nearest) in one packed multiply.
__device__ __forceinline__ unsigned long long f32x2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ void rope_rotate8_x2(const float (&x1)[8], const float (&x2)[8], const float (&c)[8],
                                                const float (&s)[8], const float (&ns)[8], float (&y1)[8],
                                                float (&y2)[8]) {
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const unsigned long long a1 = f32x2_pack(x1[i], x1[i + 1]), a2 = f32x2_pack(x2[i], x2[i + 1]);
    const unsigned long long cc = f32x2_pack(c[i], c[i + 1]);
    const unsigned long long ss = f32x2_pack(s[i], s[i + 1]), nss = f32x2_pack(ns[i], ns[i + 1]);
    unsigned long long p, q, r1, r2;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(a2), "l"(nss));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r1) : "l"(a1), "l"(cc), "l"(p));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(a1), "l"(ss));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r2) : "l"(a2), "l"(cc), "l"(q));
    f32x2_unpack(r1, y1[i], y1[i + 1]);
    f32x2_unpack(r2, y2[i], y2[i + 1]);
  }
}

// (cos, sin) of the RoPE angle pos * inv_freq, the angle as one fp32 product
// and the accurate sincosf.
__device__ __forceinline__ float2 rope_angle_cs(int32_t pos, float inv_freq) {
  float s, c;
  sincosf(__fmul_rn(static_cast<float>(pos), inv_freq), &s, &c);
  return make_float2(c, s);
}

// silu(g) = g * sigmoid(g) = g / (1 + e^-g). The exponent argument is capped
// at 80 so 1 + e^-g stays finite; below g = -80 the result is ~1e-33, zero
// in fp16 either way.
__device__ __forceinline__ float silu(float g) {
  const float e = __expf(fminf(-g, 80.0f));
  return __fdividef(g, 1.0f + e);
}

template <int WIDTH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int m = WIDTH / 2; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Element load/store as float for the generic (any dtype / any shape) paths.
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ void set_flag(int32_t* flags, int32_t bit) {
  if (flags != nullptr) atomicOr(flags, bit);
}

}  // namespace kb
