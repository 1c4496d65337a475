// status.cu — error reporting and device queries for the C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace kb {
namespace {
thread_local std::string t_last_error;
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];  // 0 = not yet queried; benign racy cache of a constant
}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int launch_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(KLLM_B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return KLLM_B200_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return 148;
  }
  int v = __atomic_load_n(&g_sm_count[dev], __ATOMIC_RELAXED);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v < 1) {
      (void)cudaGetLastError();
      v = 148;
    }
    __atomic_store_n(&g_sm_count[dev], v, __ATOMIC_RELAXED);
  }
  return v;
}

namespace {
struct OccEntry {
  const void* kernel;
  int threads;
  size_t smem;
  int cluster;  // 0: resident CTAs per SM; else co-resident clusters of this size on the device
  int ctas;
};
std::mutex g_occ_mutex;
OccEntry g_occ[256];
int g_occ_n = 0;

struct SmemEntry {
  const void* kernel;
  size_t smem;
};
SmemEntry g_smem[64];
int g_smem_n = 0;
}  // namespace

int resident_ctas_raw(const void* kernel, int threads, size_t smem) {
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  for (int i = 0; i < g_occ_n; ++i) {
    if (g_occ[i].kernel == kernel && g_occ[i].threads == threads && g_occ[i].smem == smem && g_occ[i].cluster == 0) {
      return g_occ[i].ctas;
    }
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = 1;
  }
  if (g_occ_n < 256) g_occ[g_occ_n++] = {kernel, threads, smem, 0, n};
  return n;
}

int active_clusters_raw(const void* kernel, int threads, size_t smem, int cluster) {
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  for (int i = 0; i < g_occ_n; ++i) {
    if (g_occ[i].kernel == kernel && g_occ[i].threads == threads && g_occ[i].smem == smem &&
        g_occ[i].cluster == cluster) {
      return g_occ[i].ctas;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster * sm_count()));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = 0;  // not schedulable (or unknown): the caller does not split
  }
  if (g_occ_n < 256) g_occ[g_occ_n++] = {kernel, threads, smem, cluster, n};
  return n;
}

cudaError_t allow_smem(const void* kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  for (int i = 0; i < g_smem_n; ++i) {
    if (g_smem[i].kernel == kernel && g_smem[i].smem >= smem) return cudaSuccess;
  }
  const cudaError_t err =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err == cudaSuccess && g_smem_n < 64) g_smem[g_smem_n++] = {kernel, smem};
  return err;
}

}  // namespace kb

extern "C" size_t kllm_b200_last_error(char* buf, size_t len) {
  const std::string& m = kb::t_last_error;
  if (buf != nullptr && len > 0) {
    const size_t n = m.size() < len - 1 ? m.size() : len - 1;
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return m.size();
}

extern "C" const char* kllm_b200_status_string(int status) {
  switch (status) {
    case KLLM_B200_OK: return "ok";
    case KLLM_B200_ERR_INVALID_ARG: return "invalid argument";
    case KLLM_B200_ERR_SHAPE: return "shape mismatch";
    case KLLM_B200_ERR_DTYPE: return "unsupported dtype";
    case KLLM_B200_ERR_ALIGN: return "misaligned pointer";
    case KLLM_B200_ERR_RANGE: return "value out of range";
    case KLLM_B200_ERR_CAPACITY: return "KV cache capacity exceeded";
    case KLLM_B200_ERR_CUDA: return "CUDA error";
    case KLLM_B200_ERR_IO: return "I/O error";
    case KLLM_B200_ERR_FORMAT: return "malformed model file";
    default: return "unknown status";
  }
}

extern "C" int kllm_b200_version(void) { return 100; }

namespace kb {
namespace {
thread_local bool g_default_pdl = false;  // see kllm_b200_set_pdl
}  // namespace
bool default_pdl() { return g_default_pdl; }
}  // namespace kb

extern "C" int kllm_b200_set_pdl(int enable) {
  const int previous = kb::g_default_pdl ? 1 : 0;
  kb::g_default_pdl = enable != 0;
  return previous;
}
