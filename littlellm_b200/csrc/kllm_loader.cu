// kllm_loader.cu — .kllm weight files: index and streaming load.
//
// The reference loader (ModelWeights::load, src/model/weights.cpp:47-163)
// reads each record into a host vector and, for INT8 records, dequantises it
// on the host element by element (float(q) * scale, then float_to_half),
// keeps two more host copies and uploads with a blocking cudaMemcpy. Here the
// file is streamed through two pinned staging halves (file reads overlap the
// H2D copies) and INT8 records are dequantised on the device by the dequant
// kernel, bit-identical to the host loop.
#include <fcntl.h>
#include <unistd.h>

#include <cstring>
#include <string>

#include "ops.cuh"

namespace kb {
namespace {

constexpr size_t kMinStaging = 64 * 1024;
constexpr int kMaxDims = 8;

int dtype_bytes_or_neg(int32_t dt) {
  switch (dt) {
    case KLLM_B200_F32: return 4;
    case KLLM_B200_F16: return 2;
    case KLLM_B200_I32: return 4;
    case KLLM_B200_I8: return 1;
    default: return -1;
  }
}

class File {
 public:
  explicit File(const char* path) : fd_(::open(path, O_RDONLY | O_CLOEXEC)) {}
  ~File() {
    if (fd_ >= 0) ::close(fd_);
  }
  bool ok() const { return fd_ >= 0; }
  // Reads exactly n bytes at offset; false on error or short file.
  bool read_at(void* dst, size_t n, uint64_t offset) const {
    char* p = static_cast<char*>(dst);
    while (n > 0) {
      const ssize_t r = ::pread(fd_, p, n, static_cast<off_t>(offset));
      if (r <= 0) return false;
      p += r;
      n -= static_cast<size_t>(r);
      offset += static_cast<uint64_t>(r);
    }
    return true;
  }

 private:
  int fd_;
};

// Sequential reader over the header / record table.
struct Cursor {
  const File& f;
  uint64_t pos = 0;
  bool ok = true;
  template <typename T>
  T pod() {
    T v{};
    if (ok) ok = f.read_at(&v, sizeof v, pos);
    pos += sizeof v;
    return v;
  }
};

}  // namespace
}  // namespace kb

extern "C" int kllm_b200_kllm_read_index(const char* path, kllm_b200_kllm_config* config,
                                         kllm_b200_kllm_record* records, int max_records, int* n_records) {
  using namespace kb;
  if (!path || !n_records || max_records < 0 || (max_records > 0 && !records)) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "kllm_read_index: bad arguments");
  }
  *n_records = 0;
  File f(path);
  if (!f.ok()) return fail(KLLM_B200_ERR_IO, "failed to open model file: %s", path);
  Cursor c{f};
  char magic[8];
  if (!f.read_at(magic, 8, 0)) return fail(KLLM_B200_ERR_FORMAT, "%s: file too short", path);
  if (std::memcmp(magic, "KLLM0001", 8) != 0) {
    return fail(KLLM_B200_ERR_FORMAT, "invalid model file magic, expected KLLM0001");
  }
  c.pos = 8;
  if (c.pod<uint32_t>() != 1 || !c.ok) return fail(KLLM_B200_ERR_FORMAT, "unsupported model file version");
  kllm_b200_kllm_config cfg{};
  cfg.model_type = c.pod<uint32_t>();
  cfg.vocab_size = c.pod<int32_t>();
  cfg.hidden_size = c.pod<int32_t>();
  cfg.intermediate_size = c.pod<int32_t>();
  cfg.num_layers = c.pod<int32_t>();
  cfg.num_heads = c.pod<int32_t>();
  cfg.num_kv_heads = c.pod<int32_t>();
  cfg.head_dim = c.pod<int32_t>();
  cfg.max_seq_len = c.pod<int32_t>();
  cfg.rms_norm_eps = c.pod<float>();
  cfg.rope_theta = c.pod<float>();
  cfg.tie_word_embeddings = c.pod<uint8_t>();
  cfg.qkv_bias = c.pod<uint8_t>();
  cfg.o_bias = c.pod<uint8_t>();
  cfg.mlp_bias = c.pod<uint8_t>();
  const uint32_t count = c.pod<uint32_t>();
  if (!c.ok) return fail(KLLM_B200_ERR_FORMAT, "%s: truncated header", path);
  if (config) *config = cfg;
  for (uint32_t i = 0; i < count; ++i) {
    kllm_b200_kllm_record r{};
    const uint32_t name_len = c.pod<uint32_t>();
    if (!c.ok || name_len >= sizeof r.name) return fail(KLLM_B200_ERR_FORMAT, "record %u: bad name length", i);
    if (!f.read_at(r.name, name_len, c.pos)) return fail(KLLM_B200_ERR_FORMAT, "record %u: truncated name", i);
    c.pos += name_len;
    r.dtype = static_cast<int32_t>(c.pod<uint32_t>());
    const uint32_t ndim = c.pod<uint32_t>();
    if (!c.ok || ndim > static_cast<uint32_t>(kMaxDims)) {
      return fail(KLLM_B200_ERR_FORMAT, "record %s: bad rank", r.name);
    }
    r.ndim = static_cast<int32_t>(ndim);
    int64_t numel = 1;
    for (uint32_t d = 0; d < ndim; ++d) {
      r.dims[d] = c.pod<int64_t>();
      if (r.dims[d] < 0) return fail(KLLM_B200_ERR_FORMAT, "record %s: negative dimension", r.name);
      numel *= r.dims[d];
    }
    r.numel = numel;
    r.nbytes = c.pod<uint64_t>();
    if (!c.ok) return fail(KLLM_B200_ERR_FORMAT, "record %s: truncated", r.name);
    const int esz = dtype_bytes_or_neg(r.dtype);
    if (esz < 0) return fail(KLLM_B200_ERR_FORMAT, "record %s: unknown dtype %d", r.name, r.dtype);
    // src/model/weights.cpp:96-117: I8 records carry numel int8 + one fp32 scale
    const uint64_t expected = r.dtype == KLLM_B200_I8 ? static_cast<uint64_t>(numel) + sizeof(float)
                                                      : static_cast<uint64_t>(numel) * esz;
    if (r.nbytes != expected) {
      return fail(KLLM_B200_ERR_FORMAT, "tensor byte size mismatch: %s (expected %llu, got %llu)", r.name,
                  (unsigned long long)expected, (unsigned long long)r.nbytes);
    }
    r.data_offset = c.pos;
    c.pos += r.nbytes;
    r.load_dtype = r.dtype == KLLM_B200_I8 ? KLLM_B200_F16 : r.dtype;
    r.load_bytes = numel * dtype_bytes_or_neg(r.load_dtype);
    if (static_cast<int>(i) < max_records) records[i] = r;
  }
  // the last record must end inside the file
  char probe;
  if (count > 0 && c.pos > 0 && !f.read_at(&probe, 1, c.pos - 1)) {
    return fail(KLLM_B200_ERR_FORMAT, "%s: truncated tensor data", path);
  }
  *n_records = static_cast<int>(count);
  return KLLM_B200_OK;
}

extern "C" int kllm_b200_kllm_load(const char* path, const kllm_b200_kllm_record* records, int n_records,
                                   void* const* dst, void* host_staging, size_t host_staging_bytes,
                                   void* dev_staging, size_t dev_staging_bytes, void* stream) {
  using namespace kb;
  if (!path || n_records < 0 || (n_records > 0 && (!records || !dst))) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "kllm_load: bad arguments");
  }
  bool any_i8 = false;
  for (int i = 0; i < n_records; ++i) {
    if (records[i].numel > 0 && !dst[i]) return fail(KLLM_B200_ERR_INVALID_ARG, "kllm_load: null destination %d", i);
    any_i8 |= records[i].dtype == KLLM_B200_I8 && records[i].numel > 0;
  }
  if (!host_staging || host_staging_bytes < kMinStaging) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "kllm_load: host staging must be at least %zu bytes", kMinStaging);
  }
  if (any_i8 && (!dev_staging || dev_staging_bytes < kMinStaging)) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "kllm_load: INT8 records need at least %zu bytes of device staging",
                kMinStaging);
  }
  File f(path);
  if (!f.ok()) return fail(KLLM_B200_ERR_IO, "failed to open model file: %s", path);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // chunk: half of each staging area, a multiple of 256 bytes (keeps every
  // int8 chunk start 16-byte aligned and its fp16 output 32-byte aligned)
  size_t chunk = host_staging_bytes / 2;
  if (any_i8 && dev_staging_bytes / 2 < chunk) chunk = dev_staging_bytes / 2;
  chunk &= ~static_cast<size_t>(255);
  char* host_half[2] = {static_cast<char*>(host_staging), static_cast<char*>(host_staging) + chunk};
  char* dev_half[2] = {static_cast<char*>(dev_staging), any_i8 ? static_cast<char*>(dev_staging) + chunk : nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  for (auto& e : done) {
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      (void)cudaGetLastError();
      for (auto& e2 : done) if (e2) cudaEventDestroy(e2);
      return fail(KLLM_B200_ERR_CUDA, "kllm_load: cudaEventCreate failed");
    }
  }
  LaunchOpts o;
  o.pdl = false;  // the kernels follow host-to-device copies on the stream
  o.stream = s;
  int rc = KLLM_B200_OK;
  int k = 0;  // chunk counter selects the staging half
  for (int i = 0; i < n_records && rc == KLLM_B200_OK; ++i) {
    const kllm_b200_kllm_record& r = records[i];
    if (r.numel == 0) continue;
    const bool i8 = r.dtype == KLLM_B200_I8;
    float scale = 0.0f;
    if (i8 && !f.read_at(&scale, sizeof scale, r.data_offset + static_cast<uint64_t>(r.numel))) {
      rc = fail(KLLM_B200_ERR_IO, "%s: reading the scale of %s failed", path, r.name);
      break;
    }
    const uint64_t data_bytes = i8 ? static_cast<uint64_t>(r.numel) : r.nbytes;
    for (uint64_t off = 0; off < data_bytes && rc == KLLM_B200_OK; off += chunk, ++k) {
      const size_t len = static_cast<size_t>(data_bytes - off < chunk ? data_bytes - off : chunk);
      const int h = k & 1;
      // the previous copy out of this host half must have finished
      cudaError_t err = cudaEventSynchronize(done[h]);
      if (err != cudaSuccess) {
        rc = launch_status(err, "kllm_load");
        break;
      }
      if (!f.read_at(host_half[h], len, r.data_offset + off)) {
        rc = fail(KLLM_B200_ERR_IO, "%s: reading %s failed", path, r.name);
        break;
      }
      if (!i8) {
        err = cudaMemcpyAsync(static_cast<char*>(dst[i]) + off, host_half[h], len, cudaMemcpyHostToDevice, s);
      } else {
        err = cudaMemcpyAsync(dev_half[h], host_half[h], len, cudaMemcpyHostToDevice, s);
        if (err == cudaSuccess) {
          // the next H2D into this device half is queued after this kernel on the same stream
          rc = dequantize_int8_value(reinterpret_cast<const int8_t*>(dev_half[h]), scale,
                                     static_cast<char*>(dst[i]) + off * 2, static_cast<int64_t>(len),
                                     KLLM_B200_F16, o);
        }
      }
      if (err == cudaSuccess) err = cudaEventRecord(done[h], s);
      if (err != cudaSuccess) rc = launch_status(err, "kllm_load");
    }
  }
  const cudaError_t serr = cudaStreamSynchronize(s);
  if (rc == KLLM_B200_OK && serr != cudaSuccess) rc = launch_status(serr, "kllm_load");
  for (auto& e : done) cudaEventDestroy(e);
  return rc;
}
