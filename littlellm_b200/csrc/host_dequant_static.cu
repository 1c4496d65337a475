// host_dequant_static.cu — INT8 -> fp16/fp32 dequant of a tensor held in host
// memory, without allocating any device memory.
//
// kllm_b200_kllm_load stages INT8 records in device memory the caller
// allocates before the dequant kernel reads them. Some callers cannot
// allocate device memory: a plugin that only receives device output buffers
// from the application hosting it, or a weight-refresh path running inside a
// serving process whose GPU memory is owned by another allocator that forbids
// cudaMalloc while requests are in flight. For them this entry point stages
// the int8 bytes in a fixed device array compiled into this file instead.
//
// The array is kStaticStagingBytes (32 MiB) and every GPU that loads the
// library holds it until the process exits. Host code cannot use the array's
// name as a device address (it names a host-side stand-in), so the device
// address comes from cudaGetSymbolAddress with the caller's device current.
// That address belongs to the CUDA context current at the call: a plugin
// host that runs its own (non-primary) context, or a cudaDeviceReset between
// calls, gives the array a different address. So the lookup is done on every
// call; once the library's module is loaded in that context it is a
// host-side table lookup; the first call in a context loads the module.
// Every call uses the same array: the
// copy of a call's int8 bytes overwrites the previous contents entirely
// (nothing needs to start at zero), and calls that overlap on the GPU
// (different streams, or different host threads on the same device) race
// on it.
#include "ops.cuh"

namespace kb {
namespace {

constexpr int64_t kStaticStagingBytes = int64_t{32} << 20;  // the largest tensor one call accepts

// One int8 value per byte; file scope, so every device holds one copy.
__device__ __align__(256) int8_t g_int8_staging[kStaticStagingBytes];

// The array's device address in the context current on this thread.
int staging_address(int8_t** out) {
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_int8_staging);
  if (err != cudaSuccess || p == nullptr) {
    return launch_status(err != cudaSuccess ? err : cudaErrorInvalidSymbol,
                         "dequantize_int8_host_static: cudaGetSymbolAddress");
  }
  *out = static_cast<int8_t*>(p);
  return KLLM_B200_OK;
}

}  // namespace
}  // namespace kb

extern "C" int kllm_b200_dequantize_int8_host_static(const int8_t* host_data, float scale, void* out,
                                                     int64_t n, int out_dtype, void* stream) {
  using namespace kb;
  if (n < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_host_static: negative size");
  if (n == 0) return KLLM_B200_OK;
  if (!host_data || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "dequantize_int8_host_static: null pointer");
  if (!is_float_dtype(out_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "dequantize_int8_host_static: output dtype %d not supported (F32/F16)",
                out_dtype);
  }
  if (n > kStaticStagingBytes) {
    return fail(KLLM_B200_ERR_CAPACITY,
                "dequantize_int8_host_static: %lld values exceed the %lld-byte static staging area; "
                "use kllm_b200_kllm_load or kllm_b200_dequantize_int8 with caller-allocated memory",
                (long long)n, (long long)kStaticStagingBytes);
  }
  int8_t* staging = nullptr;
  int rc = staging_address(&staging);
  if (rc != KLLM_B200_OK) return rc;
  LaunchOpts o;
  o.pdl = false;  // the kernels follow host-to-device copies on the stream
  o.stream = static_cast<cudaStream_t>(stream);
  const cudaError_t err = cudaMemcpyAsync(staging, host_data, static_cast<size_t>(n), cudaMemcpyHostToDevice, o.stream);
  if (err != cudaSuccess) return launch_status(err, "dequantize_int8_host_static: copy to the staging area");
  return dequantize_int8_value(staging, scale, out, n, out_dtype, o);
}
