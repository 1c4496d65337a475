// rms_norm.cu — residual add fused with RMSNorm, and plain RMSNorm.
//
// Replaces add_inplace (src/op/cuda/add.cu:71-76) + rms_norm
// (src/op/cuda/rms_norm.cu:177-188) at src/model/llama.cpp:135-143/166/176.
//
// fp16 fast path (hidden % 8 == 0, 16-byte aligned rows, hidden <= 16384):
// a group of G threads (8..256) owns a row; each thread holds VPT 16-byte
// vectors of the row in registers, so the row is read from HBM once, the
// residual written once and the output written once (4*H*2 bytes per row
// with a delta, 2*H*2 without). G and VPT are picked per hidden size (H=896:
// one warp per row, VPT=4; H=4096: G=128, VPT=4) so registers stay at 64 and
// small CTAs (128 threads) spread the rows evenly over the SMs. Sub-warp
// groups reduce with shuffles; multi-warp groups add one shared-memory
// exchange. CTAs stride over row groups (one wave of CTAs).
//
// Arithmetic: r = fp16_rn(a + d) (what the reference's fp16 add_inplace
// stores), sum of r^2 in fp32, scale = rsqrt(sum / H + eps), y = (r * scale)
// * w rounded to fp16.
//
// The same kernel also gathers its rows from an embedding table
// (embedding_rms_norm): r = table[ids[t]] is stored as the residual and its
// norm written, one launch for the embedding and layer 0's input norm
// (src/model/llama.cpp:84 then :83-87 of the next layer loop). The gathered
// row is never re-read from HBM, and the result is bit-identical to the
// embedding followed by rms_norm. The table and the ids are never written by
// a kernel of the chain, so a launch with EARLY (a chain launch after the
// chain's first) issues the row loads before the grid-dependency wait; the
// chain's first launch and the individual entry point load them after it.
//
// Before the wait (any launch), thread 0 of a CTA asks L2 for the delta rows
// (or the ids) of its first row group: a hint that returns no data, so it is
// correct whatever the previous kernel is still writing.
#include "ops.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;      // largest CTA (generic path, widest rows)
constexpr int kFastThreads = 128;  // CTA of the fast path unless a row needs more

// Where a row comes from and what is stored besides the normed output.
enum NormMode : int {
  kPlain = 0,     // r = residual row (read only)
  kAddDelta = 1,  // r = fp16(residual + delta), stored back as the residual
  kGather = 2,    // r = table[ids[row]] (`src` is the table), stored as the residual
  kAddSelect = 3, // kAddDelta, and each sequence's last row also written to last_rows
};

// Stages weight vector i (16 bytes: 8 fp16 or 4 fp32 values) as fp32 into
// two planes of float4: plane 0 holds values 0-3 and plane 1 values 4-7 of
// every 8-value group, so the output phase's two 16-byte reads per group are
// both consecutive across the lanes of a warp (no bank conflicts).
template <typename TW>
__device__ __forceinline__ void stage_weight_vec(float4* planes, int ngroups, int i, uint4 v);

template <>
__device__ __forceinline__ void stage_weight_vec<__half>(float4* planes, int ngroups, int i, uint4 v) {
  float f[8];
  unpack8(v, f);
  planes[i] = make_float4(f[0], f[1], f[2], f[3]);
  planes[ngroups + i] = make_float4(f[4], f[5], f[6], f[7]);
}

template <>
__device__ __forceinline__ void stage_weight_vec<float>(float4* planes, int ngroups, int i, uint4 v) {
  planes[(i & 1) * ngroups + (i >> 1)] = *reinterpret_cast<const float4*>(&v);
}

// GROUP and NVEC are the row group's threads and the row's 16-byte vectors
// when they are compile-time constants (the served hidden sizes: the
// per-vector bounds checks and the reduction loop then resolve at compile
// time), 0 when they come from the arguments.
template <int VPT, int GROUP, int NVEC, typename TW, int MODE, bool EARLY>
__global__ void __launch_bounds__(kThreads) add_rms_norm_f16_kernel(__half* __restrict__ residual,
                                                                    const __half* __restrict__ src,
                                                                    const TW* __restrict__ weight,
                                                                    __half* __restrict__ out, int64_t rows,
                                                                    int hidden, int group_arg, float eps,
                                                                    const int32_t* __restrict__ ids, int64_t vocab,
                                                                    int32_t* err_flags, int early_residual,
                                                                    __half* __restrict__ last_rows, int64_t seq_len) {
  constexpr bool HAS_DELTA = MODE == kAddDelta || MODE == kAddSelect;
  constexpr bool GATHER = MODE == kGather;
  constexpr bool SELECT = MODE == kAddSelect;
  constexpr int kWv = 16 / static_cast<int>(sizeof(TW));  // weight values per 16-byte vector
  extern __shared__ __align__(16) float4 s_w4[];          // the norm weight as fp32, two planes
  __shared__ float partial[2][kThreads / 32];
  // The delta rows (or the ids) of this CTA's first row group into L2 while
  // the previous kernel drains (a hint that returns no data).
  if (threadIdx.x == 0 && (HAS_DELTA || GATHER)) {
    const int rpc = blockDim.x / (GROUP != 0 ? GROUP : group_arg);
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
    if (r0 < rows) {
      const int64_t nr = rows - r0 < rpc ? rows - r0 : rpc;
      if (HAS_DELTA) prefetch_l2_bulk(src + r0 * hidden, static_cast<uint32_t>(nr * hidden * 2));
      if (GATHER) prefetch_l2(ids + r0);
    }
  }
  // The norm weight is staged into shared memory as fp32 once per CTA and
  // the output phase reads it from there. With EARLY (a PDL launch of the
  // chain executor after its first, whose predecessor writes no weight, table
  // or ids) the staging runs before the grid-dependency wait, overlapping the
  // previous kernel's tail. Without EARLY the kernel waits before its first
  // global read (a no-op for a launch without PDL).
  if (!EARLY) {
    grid_dep_wait();
    grid_dep_launch();
  }
  const int wvec = hidden / kWv;
  const int wgroups = hidden >> 3;
  auto stage_weight = [&]() {
    const uint4* wsrc = reinterpret_cast<const uint4*>(weight);
    for (int i = threadIdx.x; i < wvec; i += blockDim.x) stage_weight_vec<TW>(s_w4, wgroups, i, ld_keep(wsrc + i));
    __syncthreads();
  };
  // Without EARLY, a weight that fits one 16-byte vector per thread is loaded
  // into a register first and parked in shared memory after the first row
  // loads are issued, so the two round trips overlap; wider weights are
  // staged up front.
  const bool park = !EARLY && wvec <= static_cast<int>(blockDim.x);
  uint4 wreg = make_uint4(0, 0, 0, 0);
  if (park && static_cast<int>(threadIdx.x) < wvec) wreg = ld_keep(reinterpret_cast<const uint4*>(weight) + threadIdx.x);
  if (!park) stage_weight();
  // With EARLY a gathering launch issues its first rows' loads (table and
  // ids, which no kernel of the chain writes) before the wait, and so does an
  // add launch for its residual rows when early_residual says the previous
  // launch did not write them; the delta always waits.
  bool waited = !(EARLY && (GATHER || (HAS_DELTA && early_residual != 0)));
  if (EARLY && waited) {
    grid_dep_wait();
    grid_dep_launch();
  }
  bool staged = !park;

  const int nvec = NVEC != 0 ? NVEC : hidden >> 3;
  const int group = GROUP != 0 ? GROUP : group_arg;
  const int rows_per_cta = blockDim.x / group;
  const int lane_g = threadIdx.x % group;          // position inside the row group
  const int row_in_cta = threadIdx.x / group;
  const int warp = threadIdx.x >> 5;
  const int warps_per_group = group >> 5;          // 0 for sub-warp groups
  const float inv_h = 1.0f / static_cast<float>(hidden);
  const int64_t n_groups = (rows + rows_per_cta - 1) / rows_per_cta;

  int parity = 0;
  for (int64_t g = blockIdx.x; g < n_groups; g += gridDim.x, parity ^= 1) {
    const int64_t row = g * rows_per_cta + row_in_cta;
    const bool live = row < rows;
    __half* rrow = residual + row * hidden;
    uint4 r[VPT], d[VPT];
    bool id_ok = true;
    if (live) {
      const __half* rsrc = rrow;
      if (GATHER) {
        const int32_t id = __ldg(ids + row);
        id_ok = id >= 0 && id < vocab;
        rsrc = src + static_cast<int64_t>(id_ok ? id : 0) * hidden;
      }
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = j * group + lane_g;
        if (v < nvec) {
          if (GATHER) {
            // table rows are read once (random ids): no L1 allocation
            r[j] = id_ok ? ld_stream(rsrc + v * 8) : make_uint4(0, 0, 0, 0);
          } else {
            r[j] = HAS_DELTA ? ld_cg(rsrc + v * 8) : ld_stream(rsrc + v * 8);
            if (HAS_DELTA && waited) d[j] = ld_stream(src + row * hidden + v * 8);
          }
        }
      }
    }
    if (!waited) {  // uniform over the grid: every thread passes here in its first iteration
      grid_dep_wait();
      grid_dep_launch();
      waited = true;
      if (HAS_DELTA && live) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int v = j * group + lane_g;
          if (v < nvec) d[j] = ld_stream(src + row * hidden + v * 8);
        }
      }
    }
    if (GATHER && live && !id_ok && lane_g == 0) set_flag(err_flags, KLLM_B200_FLAG_BAD_TOKEN);
    // `staged` and the loop trip count are uniform over the CTA, so every
    // thread reaches this barrier.
    if (!staged) {
      if (static_cast<int>(threadIdx.x) < wvec) stage_weight_vec<TW>(s_w4, wgroups, threadIdx.x, wreg);
      __syncthreads();
      staged = true;
    }
    // the rounded row stays packed in r (four registers per 16-byte vector);
    // it is unpacked for the sum of squares and again for the output
    float ss = 0.0f;
    if (live) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = j * group + lane_g;
        if (v < nvec) {
          // r = fp16(residual + delta): the rounded sum the reference's fp16
          // add_inplace stores (HADD2 equals the fp32 sum rounded to fp16)
          if (HAS_DELTA) r[j] = hadd8(r[j], d[j]);
          if (HAS_DELTA || GATHER) st_plain(rrow + v * 8, r[j]);
          float f[8];
          unpack8(r[j], f);
          float sj = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) sj = fmaf(f[i], f[i], sj);
          ss += sj;
        }
      }
    }
    // Reduce over the row group: shuffles inside the warp, then (groups
    // wider than a warp) one exchange of per-warp partials in shared memory.
    const int sub = group < 32 ? group : 32;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      if (m < sub) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    }
    if (warps_per_group > 1) {
      if ((threadIdx.x & 31) == 0) partial[parity][warp] = ss;
      __syncthreads();
      const int first = (threadIdx.x / group) * warps_per_group;
      ss = 0.0f;
      for (int w = 0; w < warps_per_group; ++w) ss += partial[parity][first + w];
    }
    if (live) {
      const float scale = rsqrtf(ss * inv_h + eps);
      const unsigned long long scale2 = f32x2_pack(scale, scale);
      __half* orow = out + row * hidden;
      // the last row of each sequence of seq_len rows also goes to last_rows
      // (select_last_rows fused into the final norm)
      __half* lrow = nullptr;
      if (SELECT) {  // rows < 2^31 and seq_len >= 1 (checked on the host)
        const int r32 = static_cast<int>(row), sl = static_cast<int>(seq_len);
        if ((r32 + 1) % sl == 0) lrow = last_rows + static_cast<int64_t>(r32 / sl) * hidden;
      }
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = j * group + lane_g;
        if (v < nvec) {
          const float4 w0 = s_w4[v], w1 = s_w4[wgroups + v];
          const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          float x[8];
          unpack8(r[j], x);
          // y = (x * scale) * w, two roundings per element as the reference
          // evaluates it, two elements per packed multiply
          uint32_t h[4];
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const unsigned long long xs = f32x2_mul(f32x2_pack(x[i], x[i + 1]), scale2);
            float y0, y1;
            f32x2_unpack(f32x2_mul(xs, f32x2_pack(w[i], w[i + 1])), y0, y1);
            h[i / 2] = f2_to_h2(y0, y1);
          }
          const uint4 y = make_uint4(h[0], h[1], h[2], h[3]);
          st_plain(orow + v * 8, y);
          if (SELECT && lrow != nullptr) st_plain(lrow + v * 8, y);
        }
      }
    }
  }
}

// Any dtype / hidden size: one CTA per row, element per thread, two passes
// (the second re-reads the row from L1/L2).
template <typename TA, typename TW>
__global__ void __launch_bounds__(kThreads) add_rms_norm_generic_kernel(TA* residual, const TA* delta,
                                                                        const TW* weight, TA* out,
                                                                        int64_t rows, int64_t hidden,
                                                                        float eps) {
  __shared__ float partial[kThreads / 32];
  grid_dep_wait();
  grid_dep_launch();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    TA* x = residual + row * hidden;
    float ss = 0.0f;
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      float v = to_f(x[c]);
      if (delta != nullptr) {
        const TA r = from_f<TA>(v + to_f(delta[row * hidden + c]));
        x[c] = r;
        v = to_f(r);
      }
      ss += v * v;
    }
    ss = group_sum<32>(ss);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) ss += partial[w];
    __syncthreads();
    const float scale = rsqrtf(ss / static_cast<float>(hidden) + eps);
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      out[row * hidden + c] = from_f<TA>(to_f(x[c]) * scale * to_f(weight[c]));
    }
  }
}

struct FastConfig {
  int group = 0;
  int vpt = 0;
};

// Row-group width G and 16-byte vectors per thread VPT for a row of nvec
// vectors: rows of up to 128 vectors (H <= 1024) get one warp each (or a
// quarter/half warp when tiny), wider rows the smallest multi-warp group that
// keeps VPT <= 4 (VPT <= 8 above 1024 vectors). Small VPT keeps registers at
// or below 64 so enough rows are resident per SM to cover DRAM latency.
FastConfig pick_config(int nvec) {
  if (nvec <= 8) return {8, 1};
  if (nvec <= 16) return {16, 1};
  if (nvec <= 128) return {32, (nvec + 31) / 32};
  for (int g = 64; g <= kThreads; g <<= 1) {
    if (nvec <= 4 * g) return {g, (nvec + g - 1) / g};
  }
  if (nvec <= 8 * kThreads) return {kThreads, (nvec + kThreads - 1) / kThreads};
  return {};
}

// Extra arguments: the ids and vocabulary of a gathering launch, and the
// last-rows output of a final norm that also selects each sequence's last
// row (unused otherwise).
struct GatherArgs {
  const int32_t* ids = nullptr;
  int64_t vocab = 0;
  int32_t* err_flags = nullptr;
  void* last_rows = nullptr;
  int64_t seq_len = 1;
};

template <int VPT, int GROUP, int NVEC, typename TW, int MODE>
int launch_fast(void* residual, const void* src, const void* weight, void* out, int64_t rows, int hidden,
                int group, float eps, const GatherArgs& ga, const LaunchOpts& o, const char* what) {
  auto k = o.pdl && o.early_inputs ? add_rms_norm_f16_kernel<VPT, GROUP, NVEC, TW, MODE, true>
                                   : add_rms_norm_f16_kernel<VPT, GROUP, NVEC, TW, MODE, false>;
  const int threads = group > kFastThreads ? group : kFastThreads;
  const int rows_per_cta = threads / group;
  const size_t smem = static_cast<size_t>(hidden) * sizeof(float);  // the weight staged as fp32
  const cudaError_t attr = allow_smem(reinterpret_cast<const void*>(k), smem);
  if (attr != cudaSuccess) return launch_status(attr, what);
  const unsigned grid = persistent_grid(k, threads, smem, rows_per_cta, rows);
  return launch_status(launch(k, grid, threads, smem, o.stream, o.pdl, static_cast<__half*>(residual),
                              static_cast<const __half*>(src), static_cast<const TW*>(weight),
                              static_cast<__half*>(out), rows, hidden, group, eps, ga.ids, ga.vocab, ga.err_flags,
                              static_cast<int>(o.early_residual), static_cast<__half*>(ga.last_rows), ga.seq_len),
                       what);
}

template <int VPT, int GROUP, int NVEC, typename TW>
int launch_fast_m(int mode, void* residual, const void* src, const void* weight, void* out, int64_t rows,
                  int hidden, int group, float eps, const GatherArgs& ga, const LaunchOpts& o) {
  switch (mode) {
    case kAddDelta:
      return launch_fast<VPT, GROUP, NVEC, TW, kAddDelta>(residual, src, weight, out, rows, hidden, group, eps, ga,
                                                          o, "add_rms_norm");
    case kGather:
      return launch_fast<VPT, GROUP, NVEC, TW, kGather>(residual, src, weight, out, rows, hidden, group, eps, ga,
                                                        o, "embedding_rms_norm");
    case kAddSelect:
      return launch_fast<VPT, GROUP, NVEC, TW, kAddSelect>(residual, src, weight, out, rows, hidden, group, eps,
                                                           ga, o, "add_rms_norm_last_rows");
    default:
      return launch_fast<VPT, GROUP, NVEC, TW, kPlain>(residual, src, weight, out, rows, hidden, group, eps, ga, o,
                                                       "add_rms_norm");
  }
}

// Runtime geometry, or the compile-time one of a served hidden size:
// 896 (Qwen2.5-0.5B: one warp per row, 4 vectors per lane, 112 in the row)
// and 4096 (Llama-2-7B: 128 threads per row, 4 vectors per lane).
template <int VPT, typename TW>
int launch_fast_d(int mode, void* residual, const void* src, const void* weight, void* out, int64_t rows,
                  int hidden, int group, float eps, const GatherArgs& ga, const LaunchOpts& o) {
  if (VPT == 4 && group == 32 && hidden == 896) {
    return launch_fast_m<4, 32, 112, TW>(mode, residual, src, weight, out, rows, hidden, group, eps, ga, o);
  }
  if (VPT == 4 && group == 128 && hidden == 4096) {
    return launch_fast_m<4, 128, 512, TW>(mode, residual, src, weight, out, rows, hidden, group, eps, ga, o);
  }
  return launch_fast_m<VPT, 0, 0, TW>(mode, residual, src, weight, out, rows, hidden, group, eps, ga, o);
}

template <typename TW>
int dispatch_fast(const FastConfig& c, int mode, void* residual, const void* src, const void* weight, void* out,
                  int64_t rows, int hidden, float eps, const GatherArgs& ga, const LaunchOpts& o) {
  switch (c.vpt) {
    case 1: return launch_fast_d<1, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 2: return launch_fast_d<2, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 3: return launch_fast_d<3, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 4: return launch_fast_d<4, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 5: return launch_fast_d<5, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 6: return launch_fast_d<6, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    case 7: return launch_fast_d<7, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
    default: return launch_fast_d<8, TW>(mode, residual, src, weight, out, rows, hidden, c.group, eps, ga, o);
  }
}

template <typename TA, typename TW>
int launch_generic(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                   int64_t hidden, float eps, const LaunchOpts& o) {
  auto k = add_rms_norm_generic_kernel<TA, TW>;
  const unsigned grid = persistent_grid(k, kThreads, 0, 1, rows);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, static_cast<TA*>(residual),
                              static_cast<const TA*>(delta), static_cast<const TW*>(weight), static_cast<TA*>(out),
                              rows, hidden, eps),
                       "add_rms_norm");
}

}  // namespace

int add_rms_norm(void* residual, const void* delta, const void* weight, void* out, int64_t rows, int64_t hidden,
                 float eps, int act_dtype, int weight_dtype, const LaunchOpts& o) {
  if (rows < 0 || hidden < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "rms_norm: negative size");
  if (rows == 0) return KLLM_B200_OK;
  if (hidden == 0) return fail(KLLM_B200_ERR_SHAPE, "rms_norm: hidden must be positive");
  if (!residual || !weight || !out) return fail(KLLM_B200_ERR_INVALID_ARG, "rms_norm: null pointer");
  if (!is_float_dtype(act_dtype) || !is_float_dtype(weight_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "rms_norm: dtypes %d/%d not supported", act_dtype, weight_dtype);
  }
  if (act_dtype == KLLM_B200_F16) {
    const bool fast = hidden % 8 == 0 && hidden <= 8 * 8 * kThreads && aligned16(residual) && aligned16(out) &&
                      aligned16(weight) && (delta == nullptr || aligned16(delta));
    if (fast) {
      const FastConfig c = pick_config(static_cast<int>(hidden / 8));
      if (c.vpt > 0) {
        const int mode = delta ? kAddDelta : kPlain;
        const GatherArgs ga;
        return weight_dtype == KLLM_B200_F16
                   ? dispatch_fast<__half>(c, mode, residual, delta, weight, out, rows, (int)hidden, eps, ga, o)
                   : dispatch_fast<float>(c, mode, residual, delta, weight, out, rows, (int)hidden, eps, ga, o);
      }
    }
    return weight_dtype == KLLM_B200_F16
               ? launch_generic<__half, __half>(residual, delta, weight, out, rows, hidden, eps, o)
               : launch_generic<__half, float>(residual, delta, weight, out, rows, hidden, eps, o);
  }
  return weight_dtype == KLLM_B200_F16
             ? launch_generic<float, __half>(residual, delta, weight, out, rows, hidden, eps, o)
             : launch_generic<float, float>(residual, delta, weight, out, rows, hidden, eps, o);
}

int add_rms_norm_last_rows(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                           int64_t hidden, float eps, int weight_dtype, void* last_rows, int64_t seq_len,
                           int64_t n_seqs, int32_t* err_flags, const LaunchOpts& o, int* n_launched) {
  *n_launched = 0;
  const bool fast = rows > 0 && hidden % 8 == 0 && hidden <= 8 * 8 * kThreads && aligned16(residual) &&
                    aligned16(out) && aligned16(weight) && (delta == nullptr || aligned16(delta)) &&
                    delta != nullptr && last_rows != nullptr && aligned16(last_rows) && seq_len >= 1 &&
                    n_seqs * seq_len == rows && rows < (int64_t{1} << 31) && is_float_dtype(weight_dtype);
  if (fast) {
    const FastConfig c = pick_config(static_cast<int>(hidden / 8));
    if (c.vpt > 0) {
      GatherArgs ga;
      ga.last_rows = last_rows;
      ga.seq_len = seq_len;
      const int mode = kAddSelect;
      const int rc = weight_dtype == KLLM_B200_F16
                         ? dispatch_fast<__half>(c, mode, residual, delta, weight, out, rows, (int)hidden, eps, ga, o)
                         : dispatch_fast<float>(c, mode, residual, delta, weight, out, rows, (int)hidden, eps, ga, o);
      if (rc == KLLM_B200_OK) *n_launched = 1;
      return rc;
    }
  }
  int rc = add_rms_norm(residual, delta, weight, out, rows, hidden, eps, KLLM_B200_F16, weight_dtype, o);
  if (rc != KLLM_B200_OK) return rc;
  *n_launched = 1;
  LaunchOpts plain = o;
  plain.early_residual = false;
  rc = select_last_rows(out, rows, hidden, nullptr, seq_len, n_seqs, last_rows, KLLM_B200_F16, err_flags, plain);
  if (rc == KLLM_B200_OK) *n_launched = 2;
  return rc;
}

int embedding_rms_norm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n_tokens,
                       const void* weight, int weight_dtype, float eps, void* residual, void* out,
                       int32_t* err_flags, const LaunchOpts& o) {
  if (n_tokens < 0 || hidden < 0 || vocab < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "embedding_rms_norm: negative size");
  if (n_tokens == 0) return KLLM_B200_OK;
  if (hidden == 0) return fail(KLLM_B200_ERR_SHAPE, "embedding_rms_norm: hidden must be positive");
  if (!table || !ids || !weight || !residual || !out) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "embedding_rms_norm: null pointer");
  }
  if (!is_float_dtype(weight_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "embedding_rms_norm: weight dtype %d not supported", weight_dtype);
  }
  const bool fast = hidden % 8 == 0 && hidden <= 8 * 8 * kThreads && aligned16(table) && aligned16(residual) &&
                    aligned16(out) && aligned16(weight);
  if (fast) {
    const FastConfig c = pick_config(static_cast<int>(hidden / 8));
    if (c.vpt > 0) {
      GatherArgs ga;
      ga.ids = ids;
      ga.vocab = vocab;
      ga.err_flags = err_flags;
      return weight_dtype == KLLM_B200_F16
                 ? dispatch_fast<__half>(c, kGather, residual, table, weight, out, n_tokens, (int)hidden, eps, ga, o)
                 : dispatch_fast<float>(c, kGather, residual, table, weight, out, n_tokens, (int)hidden, eps, ga, o);
    }
  }
  // other shapes and alignments: the gather, then the norm of the gathered rows
  const int rc = embedding(table, vocab, hidden, KLLM_B200_F16, ids, n_tokens, residual, KLLM_B200_F16, err_flags, o);
  if (rc != KLLM_B200_OK) return rc;
  return add_rms_norm(residual, nullptr, weight, out, n_tokens, hidden, eps, KLLM_B200_F16, weight_dtype, o);
}

}  // namespace kb

extern "C" int kllm_b200_embedding_rms_norm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids,
                                            int64_t n_tokens, const void* weight, int weight_dtype, float eps,
                                            void* residual_out, void* norm_out, int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::embedding_rms_norm(table, vocab, hidden, ids, n_tokens, weight, weight_dtype, eps, residual_out,
                                norm_out, err_flags, o);
}

extern "C" int kllm_b200_add_rms_norm(void* residual, const void* delta, const void* weight, void* out,
                                      int64_t rows, int64_t hidden, float eps, int act_dtype, int weight_dtype,
                                      void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::add_rms_norm(residual, delta, weight, out, rows, hidden, eps, act_dtype, weight_dtype, o);
}

extern "C" int kllm_b200_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t hidden,
                                  float eps, int act_dtype, int weight_dtype, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  // With no delta the kernel only reads `x`.
  return kb::add_rms_norm(const_cast<void*>(x), nullptr, weight, out, rows, hidden, eps, act_dtype, weight_dtype,
                          o);
}
