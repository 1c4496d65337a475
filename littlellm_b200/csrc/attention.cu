// attention.cu — causal attention of new tokens over the head-major KV cache
// [n_slots, kv_heads, max_seq, head_dim] (one layer) that
// qkv_bias_rope_kv_append fills.
//
// Semantics follow cpu_attention (src/op/cpu/attention.cpp:12-67): for token
// t and query head h, scores q·k * 1/sqrt(head_dim) over the cached positions
// 0..positions[t] of sequence slot slots[t] and kv head h / (Hq / Hkv), a
// softmax, and the probability-weighted sum of the cached values. The
// reference reads a per-sequence cache [max_seq, kv_heads, head_dim] with a
// scalar past_len (src/op/cuda/attention.cu:30-149); here every token carries
// its own position and slot, so one launch serves a whole batch of sequences.
//
// Decode kernel (one token per sequence, or any token set): a CTA takes one
// (token, kv head, chunk of positions) item. Its four warps stream 32-position
// K/V tiles of the chunk through a per-warp cp.async ring and run both
// products on mma.sync m16n8k16 (fp16 in, fp32 accumulate) with the
// kv head's query heads as the M rows, keeping an online softmax per row.
// The warps merge in shared memory; a sequence whose positions span several
// chunks writes normalised partials (o, max, sum) to the caller's workspace
// and a combine kernel merges them. The kernel is bound by HBM reads of
// K and V: 2 * (positions[t] + 1) * head_dim * 2 bytes per (token, kv head).
//
// Prefill kernels (runs of seq_len >= 16 tokens of one sequence), bound by
// the tensor pipe: 4 * head_dim FLOPs per (token, head, attended position).
// head_dim 128 runs on tcgen05 (attn_prefill_tc_kernel, below). head_dim 64
// runs on mma.sync (attn_prefill_kernel): a CTA takes 64 consecutive tokens
// of a run and one query head; each warp owns 16 of the tokens as mma rows.
// 64-position K/V tiles of the run's slot are double-buffered in shared
// memory (cp.async, one barrier per tile) and shared by the four warps; each
// row masks positions beyond its own.
#include <math.h>

#include "ops.cuh"
#include "tcgen05.cuh"

namespace kb {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kTile = 32;                       // positions per warp tile
constexpr int kStages = 3;                      // cp.async ring depth per warp
constexpr int kChunkUnit = kAttnWarps * kTile;  // chunk sizes are multiples of this
constexpr int kMaxGroups = 16;                  // query heads per kv head (the mma M rows)
constexpr int kCombineWarps = 4;

struct AttnArgs {
  const __half* q;        // [T, Hq, D]
  const __half* k_cache;  // [n_slots, Hkv, max_seq, D]
  const __half* v_cache;
  __half* out;            // [T, Hq, D]
  const int32_t* positions;
  const int32_t* slots;
  float* part_o;          // [T, Hq, n_chunks, D] chunk outputs, normalised by their own sum
  float* part_ml;         // [T, Hq, n_chunks, 2] chunk (max, sum), max in log2 units
  int32_t* err_flags;
  int64_t n_tokens;
  int n_heads, n_kv_heads, groups;
  int max_seq, n_slots;
  int chunk;              // positions per CTA, a multiple of kChunkUnit
  int n_chunks;           // ceil(max_seq / chunk)
  float scale_log2;       // log2(e) / sqrt(D)
  int64_t seq_len;        // prefill: tokens per run of one sequence
};

// 16-byte global -> shared copy; src_bytes 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// c += a * b for one m16n8k16 tile (row-major A, column-major B).
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t ld_u32(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Byte offset of 16-byte chunk `chunk` of row `row` in a [rows][D] fp16 tile;
// the chunk index is XOR-ed with row % 8 so that the eight rows one
// ldmatrix phase reads fall in eight different bank groups.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * (D * 2) + ((chunk ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int kRowChunks = D / 8;        // 16-byte chunks per cached row
  constexpr int kTileBytes = kTile * D * 2;
  constexpr int kKS = D / 16;              // k-steps of q·k over head_dim
  constexpr int kND = D / 8;               // n8 tiles of the output over head_dim
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int64_t t = blockIdx.x / a.n_chunks;
  const int c = static_cast<int>(blockIdx.x - t * a.n_chunks);
  const int g = blockIdx.y;
  const int G = a.groups;

  grid_dep_wait();
  grid_dep_launch();  // the next kernel's CTAs may take idle SMs and wait there
  const int pos = a.positions[t];
  const int slot = a.slots[t];
  __half* out_t = a.out + (t * a.n_heads + static_cast<int64_t>(g) * G) * D;
  if (pos < 0 || pos >= a.max_seq || slot < 0 || slot >= a.n_slots) {
    if (c == 0) {
      if (threadIdx.x == 0 && g == 0) {
        if (pos < 0 || pos >= a.max_seq) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
        if (slot < 0 || slot >= a.n_slots) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
      }
      for (int i = threadIdx.x; i < G * kRowChunks; i += kAttnThreads) {
        reinterpret_cast<uint4*>(out_t)[i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    return;
  }
  const int c0 = c * a.chunk;
  if (c0 > pos) return;  // this chunk lies past the token's position
  const int c1 = min(c0 + a.chunk, pos + 1);
  const int n_tiles = (c1 - c0 + kTile - 1) / kTile;
  const int my_tiles = n_tiles > warp ? (n_tiles - warp + kAttnWarps - 1) / kAttnWarps : 0;

  const size_t head_off = (static_cast<size_t>(slot) * a.n_kv_heads + g) * static_cast<size_t>(a.max_seq) * D;
  const __half* kbase = a.k_cache + head_off;
  const __half* vbase = a.v_cache + head_off;
  unsigned char* ring = smem + warp * (kStages * 2 * kTileBytes);

  // Warp tile i covers positions c0 + (warp + 4 i) * 32 ... (+31); rows past
  // c1 are zero-filled so that no stale bits reach the products.
  auto issue = [&](int i) {
    if (i < my_tiles) {
      const int j0 = c0 + (warp + i * kAttnWarps) * kTile;
      unsigned char* sk = ring + (i % kStages) * 2 * kTileBytes;
      unsigned char* sv = sk + kTileBytes;
#pragma unroll
      for (int it = 0; it < kTile * kRowChunks / 32; ++it) {
        const int idx = lane + it * 32;
        const int r = idx / kRowChunks, ch = idx % kRowChunks;
        const int j = j0 + r;
        const bool ok = j < c1;
        const size_t off = static_cast<size_t>(ok ? j : c0) * D + ch * 8;
        cp_async16(smem_u32(sk + swz<D>(r, ch)), kbase + off, ok ? 16 : 0);
        cp_async16(smem_u32(sv + swz<D>(r, ch)), vbase + off, ok ? 16 : 0);
      }
    }
    cp_async_commit();  // empty groups keep the group count uniform
  };

#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) issue(i);

  // A fragments of the query rows (rows >= G are zero).
  uint32_t qa[kKS][4];
  const __half* qg = a.q + (t * a.n_heads + static_cast<int64_t>(g) * G) * D;
#pragma unroll
  for (int ks = 0; ks < kKS; ++ks) {
    const int d0 = ks * 16 + 2 * tig;
    qa[ks][0] = gid < G ? ld_u32(qg + gid * D + d0) : 0u;
    qa[ks][1] = gid + 8 < G ? ld_u32(qg + (gid + 8) * D + d0) : 0u;
    qa[ks][2] = gid < G ? ld_u32(qg + gid * D + d0 + 8) : 0u;
    qa[ks][3] = gid + 8 < G ? ld_u32(qg + (gid + 8) * D + d0 + 8) : 0u;
  }

  float o[kND][4];
#pragma unroll
  for (int nd = 0; nd < kND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = a.scale_log2;

  for (int i = 0; i < my_tiles; ++i) {
    issue(i + kStages - 1);
    cp_async_wait<kStages - 1>();
    __syncwarp();
    const int j0 = c0 + (warp + i * kAttnWarps) * kTile;
    const unsigned char* sk = ring + (i % kStages) * 2 * kTileBytes;
    const unsigned char* sv = sk + kTileBytes;

    // scores of 16 rows x 32 positions
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 32; ++kk) {
        uint32_t b[4];
        ldsm_x4(b, smem_u32(sk + swz<D>(nt * 8 + (lane & 7), 4 * kk + (lane >> 3))));
        mma16816(s[nt], qa[2 * kk], b[0], b[1]);
        mma16816(s[nt], qa[2 * kk + 1], b[2], b[3]);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = j0 + nt * 8 + 2 * tig + (e & 1);
        const float v = col < c1 ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: every tile has a valid column
    const float cr0 = exp2f(m0 - mn0), cr1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - mn0);
      s[nt][1] = exp2f(s[nt][1] - mn0);
      s[nt][2] = exp2f(s[nt][2] - mn1);
      s[nt][3] = exp2f(s[nt][3] - mn1);
      ps0 += s[nt][0] + s[nt][1];
      ps1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * cr0 + ps0;
    l1 = l1 * cr1 + ps1;
#pragma unroll
    for (int nd = 0; nd < kND; ++nd) {
      o[nd][0] *= cr0;
      o[nd][1] *= cr0;
      o[nd][2] *= cr1;
      o[nd][3] *= cr1;
    }
    // o += p v: the score accumulators of n-tiles 2kv, 2kv+1 are the A fragment
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const uint32_t pa[4] = {pack_h2(s[2 * kv][0], s[2 * kv][1]), pack_h2(s[2 * kv][2], s[2 * kv][3]),
                              pack_h2(s[2 * kv + 1][0], s[2 * kv + 1][1]),
                              pack_h2(s[2 * kv + 1][2], s[2 * kv + 1][3])};
      const int mtx = lane >> 3;
#pragma unroll
      for (int nd2 = 0; nd2 < D / 16; ++nd2) {
        uint32_t b[4];
        ldsm_x4_trans(b, smem_u32(sv + swz<D>(16 * kv + 8 * (mtx & 1) + (lane & 7), 2 * nd2 + (mtx >> 1))));
        mma16816(o[2 * nd2], pa, b[0], b[1]);
        mma16816(o[2 * nd2 + 1], pa, b[2], b[3]);
      }
    }
    __syncwarp();  // the stage is refilled by the next iteration's issue
  }
  cp_async_wait<0>();

  // merge the four warps (each row's sum is spread over its quad)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();  // all rings idle: reuse them for the merge
  constexpr int kRedRow = D + 8;  // padded rows: the float2 stores of 8 rows spread over the banks
  float* red_o = reinterpret_cast<float*>(smem);       // [warps][16][kRedRow]
  float* red_ml = red_o + kAttnWarps * 16 * kRedRow;   // [warps][16][2]
#pragma unroll
  for (int nd = 0; nd < kND; ++nd) {
    *reinterpret_cast<float2*>(red_o + (warp * 16 + gid) * kRedRow + nd * 8 + 2 * tig) =
        make_float2(o[nd][0], o[nd][1]);
    *reinterpret_cast<float2*>(red_o + (warp * 16 + gid + 8) * kRedRow + nd * 8 + 2 * tig) =
        make_float2(o[nd][2], o[nd][3]);
  }
  if (tig == 0) {
    red_ml[(warp * 16 + gid) * 2] = m0;
    red_ml[(warp * 16 + gid) * 2 + 1] = l0;
    red_ml[(warp * 16 + gid + 8) * 2] = m1;
    red_ml[(warp * 16 + gid + 8) * 2 + 1] = l1;
  }
  __syncthreads();
  const int n_used = pos / a.chunk + 1;  // chunks holding positions 0..pos
  for (int idx = threadIdx.x; idx < G * D; idx += kAttnThreads) {
    const int row = idx / D, d = idx - row * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, red_ml[(w * 16 + row) * 2]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = exp2f(red_ml[(w * 16 + row) * 2] - M);  // 0 for a warp without tiles
      L += red_ml[(w * 16 + row) * 2 + 1] * f;
      acc += red_o[(w * 16 + row) * kRedRow + d] * f;
    }
    if (n_used == 1) {
      out_t[row * D + d] = __float2half_rn(acc / L);
    } else {
      const int64_t prow = (t * a.n_heads + static_cast<int64_t>(g) * G + row) * a.n_chunks + c;
      a.part_o[prow * D + d] = acc / L;
      if (d == 0) {
        a.part_ml[prow * 2] = M;
        a.part_ml[prow * 2 + 1] = L;
      }
    }
  }
}

// One warp per (token, query head) row whose positions span several chunks.
template <int D>
__global__ void __launch_bounds__(kCombineWarps * 32) attn_combine_kernel(const AttnArgs a) {
  constexpr int kPer = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kCombineWarps + (threadIdx.x >> 5);
  grid_dep_wait();
  grid_dep_launch();  // the next kernel's CTAs may take idle SMs and wait there
  if (row >= a.n_tokens * a.n_heads) return;
  const int64_t t = row / a.n_heads;
  const int pos = a.positions[t], slot = a.slots[t];
  if (pos < 0 || pos >= a.max_seq || slot < 0 || slot >= a.n_slots) return;
  const int n_used = pos / a.chunk + 1;
  if (n_used <= 1) return;
  const float* ml = a.part_ml + row * a.n_chunks * 2;
  const float* po = a.part_o + row * a.n_chunks * D;
  float M = -INFINITY;
  for (int c = lane; c < n_used; c += 32) M = fmaxf(M, ml[2 * c]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float L = 0.f;
  for (int c = lane; c < n_used; c += 32) L += ml[2 * c + 1] * exp2f(ml[2 * c] - M);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  float acc[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) acc[k] = 0.f;
  for (int c = 0; c < n_used; ++c) {
    const float w = ml[2 * c + 1] * exp2f(ml[2 * c] - M);
#pragma unroll
    for (int k = 0; k < kPer; ++k) acc[k] += w * po[c * D + lane * kPer + k];
  }
  const float inv = 1.f / L;
  __half* dst = a.out + row * D + lane * kPer;
#pragma unroll
  for (int k = 0; k < kPer; ++k) dst[k] = __float2half_rn(acc[k] * inv);
}

constexpr int kPfRows = kAttnWarps * 16;  // query tokens per prefill CTA
constexpr int kPfKeys = 64;               // positions per prefill K/V tile

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int kRowChunks = D / 8;
  constexpr int kTileBytes = kPfKeys * D * 2;
  constexpr int kKS = D / 16;
  constexpr int kND = D / 8;
  __shared__ int s_max_pos;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int h = blockIdx.y;
  const int g = h / a.groups;
  const int tiles_per_run = static_cast<int>((a.seq_len + kPfRows - 1) / kPfRows);
  const int64_t run = blockIdx.x / tiles_per_run;
  // the tiles late in a run attend to the most positions: schedule them first
  const int qt = tiles_per_run - 1 - static_cast<int>(blockIdx.x - run * tiles_per_run);
  const int64_t run_start = run * a.seq_len;
  const int64_t run_end = min(run_start + a.seq_len, a.n_tokens);
  const int64_t tok0 = run_start + static_cast<int64_t>(qt) * kPfRows;
  if (tok0 >= run_end) return;  // the short last run has fewer tiles
  const int rows = static_cast<int>(min(static_cast<int64_t>(kPfRows), run_end - tok0));

  grid_dep_wait();
  grid_dep_launch();  // the next kernel's CTAs may take idle SMs and wait there
  const int run_slot = a.slots[run_start];
  const bool run_slot_ok = run_slot >= 0 && run_slot < a.n_slots;
  if (threadIdx.x == 0) s_max_pos = -1;
  __syncthreads();
  if (threadIdx.x < rows) {
    const int p = a.positions[tok0 + threadIdx.x];
    const int sl = a.slots[tok0 + threadIdx.x];
    const bool pos_ok = p >= 0 && p < a.max_seq;
    const bool slot_ok = run_slot_ok && sl == run_slot;
    if (pos_ok && slot_ok) atomicMax(&s_max_pos, p);
    if (h == 0) {
      if (!pos_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
      if (!slot_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
    }
  }
  __syncthreads();
  const int max_pos = s_max_pos;

  // this thread's two rows (r0, r0 + 8 of the warp's 16); -1 = not computed
  const int r0 = warp * 16 + gid, r1 = r0 + 8;
  auto row_pos = [&](int r) -> int {
    if (r >= rows) return -1;
    const int p = a.positions[tok0 + r];
    const int sl = a.slots[tok0 + r];
    return (p >= 0 && p < a.max_seq && run_slot_ok && sl == run_slot) ? p : -1;
  };
  const int p0 = row_pos(r0), p1 = row_pos(r1);
  __half* out0 = a.out + ((tok0 + r0) * a.n_heads + h) * D;
  __half* out1 = a.out + ((tok0 + r1) * a.n_heads + h) * D;
  if (max_pos < 0) {  // no valid row in the tile: zero the rows that exist
#pragma unroll
    for (int nd = 0; nd < kND; ++nd) {
      if (r0 < rows) *reinterpret_cast<uint32_t*>(out0 + nd * 8 + 2 * tig) = 0u;
      if (r1 < rows) *reinterpret_cast<uint32_t*>(out1 + nd * 8 + 2 * tig) = 0u;
    }
    return;
  }

  const size_t head_off = (static_cast<size_t>(run_slot) * a.n_kv_heads + g) * static_cast<size_t>(a.max_seq) * D;
  const __half* kbase = a.k_cache + head_off;
  const __half* vbase = a.v_cache + head_off;
  const int n_kt = max_pos / kPfKeys + 1;

  auto issue = [&](int kt) {
    unsigned char* sk = smem + (kt & 1) * 2 * kTileBytes;
    unsigned char* sv = sk + kTileBytes;
    const int j0 = kt * kPfKeys;
#pragma unroll
    for (int it = 0; it < kPfKeys * kRowChunks / kAttnThreads; ++it) {
      const int idx = threadIdx.x + it * kAttnThreads;
      const int r = idx / kRowChunks, ch = idx % kRowChunks;
      const int j = j0 + r;
      const bool ok = j <= max_pos;
      const size_t off = static_cast<size_t>(ok ? j : 0) * D + ch * 8;
      cp_async16(smem_u32(sk + swz<D>(r, ch)), kbase + off, ok ? 16 : 0);
      cp_async16(smem_u32(sv + swz<D>(r, ch)), vbase + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  issue(0);

  uint32_t qa[kKS][4];
  const __half* q0 = a.q + ((tok0 + r0) * a.n_heads + h) * D;
  const __half* q1 = a.q + ((tok0 + r1) * a.n_heads + h) * D;
#pragma unroll
  for (int ks = 0; ks < kKS; ++ks) {
    const int d0 = ks * 16 + 2 * tig;
    qa[ks][0] = r0 < rows ? ld_u32(q0 + d0) : 0u;
    qa[ks][1] = r1 < rows ? ld_u32(q1 + d0) : 0u;
    qa[ks][2] = r0 < rows ? ld_u32(q0 + d0 + 8) : 0u;
    qa[ks][3] = r1 < rows ? ld_u32(q1 + d0 + 8) : 0u;
  }

  float o[kND][4];
#pragma unroll
  for (int nd = 0; nd < kND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = a.scale_log2;

  for (int kt = 0; kt < n_kt; ++kt) {
    cp_async_wait<0>();
    __syncthreads();  // tile kt landed; every warp is done with tile kt - 1
    if (kt + 1 < n_kt) issue(kt + 1);  // into the buffer tile kt - 1 used
    const unsigned char* sk = smem + (kt & 1) * 2 * kTileBytes;
    const unsigned char* sv = sk + kTileBytes;
    const int j0 = kt * kPfKeys;

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 32; ++kk) {
        uint32_t b[4];
        ldsm_x4(b, smem_u32(sk + swz<D>(nt * 8 + (lane & 7), 4 * kk + (lane >> 3))));
        mma16816(s[nt], qa[2 * kk], b[0], b[1]);
        mma16816(s[nt], qa[2 * kk + 1], b[2], b[3]);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = j0 + nt * 8 + 2 * tig + (e & 1);
        const bool keep = col <= (e < 2 ? p0 : p1);
        const float v = keep ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    // a row with nothing unmasked yet (a row not computed) keeps exponent base 0
    const float b0 = mn0 == -INFINITY ? 0.f : mn0, b1 = mn1 == -INFINITY ? 0.f : mn1;
    const float cr0 = exp2f(m0 - b0), cr1 = exp2f(m1 - b1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - b0);
      s[nt][1] = exp2f(s[nt][1] - b0);
      s[nt][2] = exp2f(s[nt][2] - b1);
      s[nt][3] = exp2f(s[nt][3] - b1);
      ps0 += s[nt][0] + s[nt][1];
      ps1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * cr0 + ps0;
    l1 = l1 * cr1 + ps1;
#pragma unroll
    for (int nd = 0; nd < kND; ++nd) {
      o[nd][0] *= cr0;
      o[nd][1] *= cr0;
      o[nd][2] *= cr1;
      o[nd][3] *= cr1;
    }
    const int mtx = lane >> 3;
#pragma unroll
    for (int kv = 0; kv < 4; ++kv) {
      const uint32_t pa[4] = {pack_h2(s[2 * kv][0], s[2 * kv][1]), pack_h2(s[2 * kv][2], s[2 * kv][3]),
                              pack_h2(s[2 * kv + 1][0], s[2 * kv + 1][1]),
                              pack_h2(s[2 * kv + 1][2], s[2 * kv + 1][3])};
#pragma unroll
      for (int nd2 = 0; nd2 < D / 16; ++nd2) {
        uint32_t b[4];
        ldsm_x4_trans(b, smem_u32(sv + swz<D>(16 * kv + 8 * (mtx & 1) + (lane & 7), 2 * nd2 + (mtx >> 1))));
        mma16816(o[2 * nd2], pa, b[0], b[1]);
        mma16816(o[2 * nd2 + 1], pa, b[2], b[3]);
      }
    }
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = p0 >= 0 ? 1.f / l0 : 0.f, inv1 = p1 >= 0 ? 1.f / l1 : 0.f;
#pragma unroll
  for (int nd = 0; nd < kND; ++nd) {
    if (r0 < rows) *reinterpret_cast<uint32_t*>(out0 + nd * 8 + 2 * tig) = pack_h2(o[nd][0] * inv0, o[nd][1] * inv0);
    if (r1 < rows) *reinterpret_cast<uint32_t*>(out1 + nd * 8 + 2 * tig) = pack_h2(o[nd][2] * inv1, o[nd][3] * inv1);
  }
}

// ---------------------------------------------------------------------------
// Prefill on tcgen05: q.k and p.v are single-thread-issued UMMAs (M = 128 query
// rows) whose fp32 accumulators live in tensor memory; one thread per row
// reads its scores back (tcgen05.ld), runs the online softmax and writes its
// row of P to shared memory for the p.v product.
//
// Shared-memory operands use the 128-byte-swizzle canonical layouts: a tile
// is stored as 64-element (128-byte) wide panels, row r of a panel at r * 128
// bytes with 16-byte chunk c at ((c ^ (r % 8)) * 16), panels and 8-row atoms
// 1024-byte aligned. Q, K and P are K-major operands (rows = M or N, the
// reduction dimension contiguous); V is the N-major B operand of p.v (rows =
// positions = the reduction dimension, head_dim contiguous).
// ---------------------------------------------------------------------------

constexpr int kTcKeys = 128;                      // positions per K/V tile: the UMMA N of q.k

// 2^x with the hardware approximation (ex2.approx, flush to zero); used for
// softmax probabilities that are rounded to fp16 right after.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk c (of D / 8) of row r in a 128-byte-swizzled
// tile of `rows` rows stored as 64-element panels.
__device__ __forceinline__ uint32_t sw128(int rows, int r, int c) {
  return static_cast<uint32_t>((c >> 3) * rows * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Arrive on `bar` once this thread's cp.async copies issued so far have landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// Warp roles of the tcgen05 prefill CTA: two softmax warpgroups (one per
// 128-row query tile; thread t of a warpgroup owns row t and tensor-memory
// lane t; they also load their query tile), one warp whose lane 0 issues
// every tcgen05.mma, two K/V load warps.
constexpr int kTcQTiles = 2;
constexpr int kMmaWarp = 4 * kTcQTiles;
constexpr int kLoadWarp = kMmaWarp + 1;
constexpr int kLoadWarps = 2;
constexpr int kTcThreads = (kLoadWarp + kLoadWarps) * 32;
constexpr float kRescaleLog2 = 8.f;  // rescale O only when a row max grows by more than 2^8
constexpr int kTcMaxStages = 4;
__host__ __device__ constexpr int tc_stages(int head_dim) { return head_dim > 64 ? 2 : 4; }  // K/V tiles in flight

// mbarriers: Q loaded; K/V stage full / empty; S_i complete; P_i written; p.v of tile i complete
enum TcBar {
  kQFull = 0,
  kKvFull = 1,
  kKvEmpty = kKvFull + kTcMaxStages,
  kSFull = kKvEmpty + kTcMaxStages,
  kPFull = kSFull + kTcQTiles,
  kODone = kPFull + kTcQTiles,
  kNumTcBars = kODone + kTcQTiles
};

// Tensor memory (512 columns): S_i (fp32, 128 columns) at i * 128, with P_i
// (fp16 pairs, 64 columns) written over its first half; O_i (fp32, D
// columns) at 256 + i * D.
template <int D>
__global__ void __launch_bounds__(kTcThreads, 1) attn_prefill_tc_kernel(const AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  constexpr int kStages = tc_stages(D);
  constexpr int kChunks = D / 8;
  constexpr int kRowsCta = 128 * kTcQTiles;
  constexpr int kQBytes = 128 * D * 2;        // one query tile
  constexpr int kKVBytes = kTcKeys * D * 2;   // one K or V tile
  constexpr uint32_t kOCol = kTcQTiles * kTcKeys;
  constexpr uint32_t kCols = 512;
  constexpr uint32_t kIdescS = umma_idesc(128, kTcKeys, false);
  constexpr uint32_t kIdescO = umma_idesc(128, D, true);
  static_assert(kOCol + kTcQTiles * D <= kCols, "tensor memory overflow");
  __shared__ __align__(8) uint64_t s_bar[kNumTcBars];
  __shared__ uint32_t s_tmem;
  __shared__ int s_max_pos[kTcQTiles];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  const int g = h / a.groups;
  const int tiles_per_run = static_cast<int>((a.seq_len + kRowsCta - 1) / kRowsCta);
  const int64_t run = blockIdx.x / tiles_per_run;
  const int qt = tiles_per_run - 1 - static_cast<int>(blockIdx.x - run * tiles_per_run);
  const int64_t run_start = run * a.seq_len;
  const int64_t run_end = min(run_start + a.seq_len, a.n_tokens);
  const int64_t tok0 = run_start + static_cast<int64_t>(qt) * kRowsCta;
  if (tok0 >= run_end) return;
  const int rows = static_cast<int>(min(static_cast<int64_t>(kRowsCta), run_end - tok0));

  grid_dep_wait();
  grid_dep_launch();  // the next kernel's CTAs may take idle SMs and wait there
  const int run_slot = a.slots[run_start];
  const bool run_slot_ok = run_slot >= 0 && run_slot < a.n_slots;
  if (tid < kTcQTiles) s_max_pos[tid] = -1;
  __syncthreads();
  int my_pos = -1;  // softmax threads: row tid of the CTA's 256
  if (tid < rows) {
    const int p = a.positions[tok0 + tid];
    const int sl = a.slots[tok0 + tid];
    const bool pos_ok = p >= 0 && p < a.max_seq;
    const bool slot_ok = run_slot_ok && sl == run_slot;
    if (pos_ok && slot_ok) {
      my_pos = p;
      atomicMax(&s_max_pos[tid >> 7], p);
    }
    if (h == 0) {
      if (!pos_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
      if (!slot_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
    }
  }
  __syncthreads();
  // K/V tiles each query tile needs (0: no valid row), and the CTA's maximum
  int n_kt_q[kTcQTiles];
  int max_pos = -1;
#pragma unroll
  for (int i = 0; i < kTcQTiles; ++i) {
    n_kt_q[i] = s_max_pos[i] < 0 ? 0 : s_max_pos[i] / kTcKeys + 1;
    max_pos = max(max_pos, s_max_pos[i]);
  }
  __half* out_row = a.out + ((tok0 + tid) * a.n_heads + h) * D;
  if (max_pos < 0) {
    if (tid < rows) {
#pragma unroll
      for (int c = 0; c < kChunks; ++c) reinterpret_cast<uint4*>(out_row)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  const int n_kt = max_pos / kTcKeys + 1;

  // 1024-byte aligned carve-out: Q_0 Q_1 | (K V) x stages
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = base;
  const uint32_t kv_s = q_s + kTcQTiles * kQBytes;
  auto bar = [&](int i) { return smem_u32(&s_bar[i]); };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar(kQFull), 128 * kTcQTiles);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(kKvFull + i), 32 * kLoadWarps);
      mbar_init(bar(kKvEmpty + i), 1);
    }
    for (int i = 0; i < kTcQTiles; ++i) {
      mbar_init(bar(kSFull + i), 1);
      mbar_init(bar(kPFull + i), 128);
      mbar_init(bar(kODone + i), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  bool ok = true;

  if (warp < kMmaWarp) {
    // ---------------- softmax warpgroup i: row tid of the CTA ----------------
    const int wg = warp >> 2;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_base + wg * kTcKeys;  // S_i, then P_i over its first 64 columns
    const uint32_t t_o = tmem + lane_base + kOCol + wg * D;
    {  // this warpgroup's query tile (rows past `rows` zero-filled)
      const __half* qrow0 = a.q + (tok0 * a.n_heads + h) * D;
      const int64_t q_stride = static_cast<int64_t>(a.n_heads) * D;
      const int r0 = tid & 127;
#pragma unroll 4
      for (int idx = r0; idx < 128 * kChunks; idx += 128) {
        const int r = idx / kChunks, c = idx % kChunks;
        const int row = wg * 128 + r;
        const bool in = row < rows;
        cp_async16(q_s + wg * kQBytes + sw128(128, r, c), qrow0 + (in ? row : 0) * q_stride + c * 8, in ? 16 : 0);
      }
      cp_async_mbar_arrive(bar(kQFull));
    }
    float m_used = -INFINITY, l = 0.f;
    const float sl2 = a.scale_log2;
    const int my_n_kt = n_kt_q[wg];
    for (int kt = 0; kt < my_n_kt && ok; ++kt) {
      // waits and tensor-memory accesses stay warp-uniform (tcgen05.ld/st are .sync.aligned)
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kSFull + wg), kt & 1));
      if (!ok) break;
      tc_fence_after();
      // pass 1 over the row's 128 scores in tensor memory: the max of the raw
      // scores (the scale is positive, so it is applied to the max alone);
      // masks only where the tile crosses a row's position
      const int j0 = kt * kTcKeys;
      const bool warp_full = __all_sync(0xffffffffu, j0 + kTcKeys - 1 <= my_pos);
      float mxp[8];  // eight independent chains instead of one 128-long one
#pragma unroll
      for (int q = 0; q < 8; ++q) mxp[q] = -INFINITY;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float t[2][32];
        tmem_ld32(t_s + hh * 64, t[0]);
        tmem_ld32(t_s + hh * 64 + 32, t[1]);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float v = (warp_full || j0 + hh * 64 + i <= my_pos) ? t[i >> 5][i & 31] : -INFINITY;
          mxp[i & 7] = fmaxf(mxp[i & 7], v);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                             fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7]))) * sl2;
      if (kt > 0) {  // p.v of the previous tile done: P_i is read and O_i stable
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kODone + wg), (kt - 1) & 1));
        if (!ok) break;
        tc_fence_after();
      }
      // lazy rescale: the exponent base m_used moves only when the row max
      // grows by more than 2^8, so P stays <= 256 and O is rarely rewritten
      const bool grow = mx > m_used + kRescaleLog2;
      const float f = !grow ? 1.f : (m_used == -INFINITY ? 0.f : exp2f(m_used - mx));
      if (kt > 0 && __any_sync(0xffffffffu, f != 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float t[32];
          tmem_ld32(t_o + c * 32, t);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] *= f;
          tmem_st32(t_o + c * 32, t);
        }
        tc_wait_st();
      }
      l *= f;
      if (grow) m_used = mx;
      // pass 2: p = 2^(s * scale - base), one FMA and one ex2 per score,
      // written back as P (fp16 pairs) over score columns already read
      const float nb = m_used == -INFINITY ? 0.f : -m_used;
      float psp[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) psp[q] = 0.f;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float t[2][32];
        tmem_ld32(t_s + hh * 64, t[0]);
        tmem_ld32(t_s + hh * 64 + 32, t[1]);
        tc_wait_ld();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int j = j0 + hh * 64 + c2 * 32 + 2 * i;
            float e0 = ex2_approx(__fmaf_rn(t[c2][2 * i], sl2, nb));
            float e1 = ex2_approx(__fmaf_rn(t[c2][2 * i + 1], sl2, nb));
            if (!warp_full) {
              e0 = j <= my_pos ? e0 : 0.f;
              e1 = j + 1 <= my_pos ? e1 : 0.f;
            }
            psp[(2 * i) & 7] += e0;
            psp[(2 * i + 1) & 7] += e1;
            pk[i] = pack_h2(e0, e1);
          }
          tmem_st16(t_s + hh * 32 + c2 * 16, pk);  // P columns for positions 64 hh + 32 c2 ...
        }
      }
      l += ((psp[0] + psp[1]) + (psp[2] + psp[3])) + ((psp[4] + psp[5]) + (psp[6] + psp[7]));
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kPFull + wg));
    }
    if (ok && my_n_kt > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(kODone + wg), (my_n_kt - 1) & 1));
    if (ok && my_n_kt == 0) {  // no valid row in this query tile
      if (tid < rows) {
#pragma unroll
        for (int c = 0; c < kChunks; ++c) reinterpret_cast<uint4*>(out_row)[c] = make_uint4(0u, 0u, 0u, 0u);
      }
    } else if (ok) {
      tc_fence_after();
      const float inv = my_pos >= 0 ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float t[32];
        tmem_ld32(t_o + c * 32, t);
        tc_wait_ld();
        if (tid < rows) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_h2(t[q * 8 + 0] * inv, t[q * 8 + 1] * inv);
            w.y = pack_h2(t[q * 8 + 2] * inv, t[q * 8 + 3] * inv);
            w.z = pack_h2(t[q * 8 + 4] * inv, t[q * 8 + 5] * inv);
            w.w = pack_h2(t[q * 8 + 6] * inv, t[q * 8 + 7] * inv);
            reinterpret_cast<uint4*>(out_row)[c * 4 + q] = w;
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue: lane 0 ----------------
    if (lane == 0) {
      // descriptors of stage 0 / query tile 0; other stages and tiles add a
      // byte offset / 16 to the start-address field
      const uint64_t q_desc = umma_desc(q_s, 16, 1024);
      const uint64_t k_desc = umma_desc(kv_s, 16, 1024);
      const uint64_t v_desc = umma_desc(kv_s + kKVBytes, kTcKeys * 128, 1024);
      auto issue_s = [&](int i, int kt) {
        const uint64_t qd = q_desc + static_cast<uint64_t>((i * kQBytes) >> 4);
        const uint64_t kd = k_desc + static_cast<uint64_t>(((kt % kStages) * 2 * kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t qo = ((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4;
          const uint32_t ko = ((k >> 2) * (kTcKeys * 128) + (k & 3) * 32) >> 4;
          umma_f16(tmem + i * kTcKeys, qd + qo, kd + ko, kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(bar(kSFull + i));
      };
      auto issue_pv = [&](int i, int kt) {
        const uint64_t vd = v_desc + static_cast<uint64_t>(((kt % kStages) * 2 * kKVBytes) >> 4);
#pragma unroll
        for (int k = 0; k < kTcKeys / 16; ++k) {
          umma_f16_ts(tmem + kOCol + i * D, tmem + i * kTcKeys + k * 8, vd + static_cast<uint64_t>((k * 2048) >> 4),
                      kIdescO, (kt > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(bar(kODone + i));
      };
      // step kt: p.v of tile kt - 1 and q.k of tile kt for each query tile that
      // reaches them, then release the stage of tile kt - 1
      ok = mbar_wait(bar(kQFull), 0);
      for (int kt = 0; kt <= n_kt && ok; ++kt) {
        bool kv_ready = false;
        for (int i = 0; i < kTcQTiles && ok; ++i) {
          if (kt > 0 && kt - 1 < n_kt_q[i]) {  // softmax i wrote P_i of tile kt - 1
            ok = mbar_wait(bar(kPFull + i), (kt - 1) & 1);
            if (!ok) break;
            tc_fence_after();
            issue_pv(i, kt - 1);
          }
          if (kt < n_kt_q[i]) {  // S_i is free: p.v above was issued before it
            if (!kv_ready) {
              ok = mbar_wait(bar(kKvFull + kt % kStages), (kt / kStages) & 1);
              if (!ok) break;
              fence_async_smem();
              tc_fence_after();
              kv_ready = true;
            }
            issue_s(i, kt);
          }
        }
        if (ok && kt > 0) umma_commit(bar(kKvEmpty + (kt - 1) % kStages));
      }
    }
  } else {
    // ---------------- K/V loads: the load warps, cp.async with zero fill ----------------
    const int lt = (warp - kLoadWarp) * 32 + lane;  // 0 .. 32 * kLoadWarps - 1
    const size_t head_off =
        (static_cast<size_t>(run_slot) * a.n_kv_heads + g) * static_cast<size_t>(a.max_seq) * D;
    const __half* kbase = a.k_cache + head_off;
    const __half* vbase = a.v_cache + head_off;
    for (int kt = 0; kt < n_kt; ++kt) {
      if (kt >= kStages) {  // the stage's previous tile (kt - stages) has been consumed
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kKvEmpty + kt % kStages), ((kt / kStages) - 1) & 1));
        if (!ok) break;
      }
      const uint32_t ks = kv_s + (kt % kStages) * 2 * kKVBytes, vs = ks + kKVBytes;
#pragma unroll 4
      for (int idx = lt; idx < kTcKeys * kChunks; idx += 32 * kLoadWarps) {
        const int r = idx / kChunks, c = idx % kChunks;
        const int j = kt * kTcKeys + r;
        const bool in = j <= max_pos;
        const size_t off = static_cast<size_t>(in ? j : 0) * D + c * 8;
        cp_async16(ks + sw128(kTcKeys, r, c), kbase + off, in ? 16 : 0);
        cp_async16(vs + sw128(kTcKeys, r, c), vbase + off, in ? 16 : 0);
      }
      cp_async_mbar_arrive(bar(kKvFull + kt % kStages));
    }
    cp_async_wait<0>();
  }

  if (!ok) set_flag(a.err_flags, KLLM_B200_FLAG_TIMEOUT);
  cp_async_wait<0>();  // no copy of this thread is still in flight
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

constexpr size_t prefill_tc_smem(int head_dim) {
  return static_cast<size_t>(kTcQTiles) * 128 * head_dim * 2 +
         2 * static_cast<size_t>(tc_stages(head_dim)) * kTcKeys * head_dim * 2 + 1024;
}

constexpr size_t prefill_smem(int head_dim) { return static_cast<size_t>(2) * 2 * kPfKeys * head_dim * 2; }

constexpr size_t decode_smem(int head_dim) { return static_cast<size_t>(kAttnWarps) * kStages * 2 * kTile * head_dim * 2; }

// Positions per decode CTA. Splitting a (token, kv head) item costs partial
// writes, a combine pass and per-CTA prologues, so items are split only as far
// as needed for load balance: a chunk is about an eighth of one resident CTA
// slot's share of the work, counting half of max_seq per item (positions are
// on the device), in multiples of 128, at most max_seq (no split).
int64_t preferred_chunk(int64_t n_tokens, int64_t n_kv_heads, int64_t max_seq) {
  const int64_t cap = (max_seq + kChunkUnit - 1) / kChunkUnit * kChunkUnit;
  const int64_t slots = 2LL * sm_count();  // decode CTAs resident per SM at head_dim 64
  const int64_t share = n_tokens * n_kv_heads * ((max_seq + 1) / 2) / (8 * slots);
  const int64_t chunk = (share + kChunkUnit - 1) / kChunkUnit * kChunkUnit;
  return chunk < kChunkUnit ? kChunkUnit : (chunk < cap ? chunk : cap);
}

// Split workspace: chunk partials (o, then max/sum); none when every
// sequence fits one chunk.
int64_t workspace_for(int64_t n_tokens, int64_t n_heads, int64_t head_dim, int64_t max_seq, int64_t chunk) {
  const int64_t n_chunks = (max_seq + chunk - 1) / chunk;
  if (n_chunks <= 1) return 0;
  return n_tokens * n_heads * n_chunks * (head_dim + 2) * static_cast<int64_t>(sizeof(float));
}

int check_attention_args(const void* q, const void* k_cache, const void* v_cache, const void* out,
                         const int32_t* positions, const int32_t* slots, int64_t n_tokens, int64_t n_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t n_slots, int64_t max_seq, int dtype) {
  if (n_tokens < 0 || n_heads < 0 || n_kv_heads < 0 || head_dim < 0 || n_slots < 0 || max_seq < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "attention: negative size");
  }
  if (dtype != KLLM_B200_F16) return fail(KLLM_B200_ERR_DTYPE, "attention: dtype %d not supported (F16)", dtype);
  if (head_dim != 64 && head_dim != 128) {
    return fail(KLLM_B200_ERR_SHAPE, "attention: head_dim %lld not supported (64, 128)", (long long)head_dim);
  }
  if (n_kv_heads == 0 || n_heads % n_kv_heads != 0) {
    return fail(KLLM_B200_ERR_SHAPE, "attention: %lld query heads not a multiple of %lld kv heads",
                (long long)n_heads, (long long)n_kv_heads);
  }
  if (n_heads / n_kv_heads > kMaxGroups) {
    return fail(KLLM_B200_ERR_SHAPE, "attention: more than %d query heads per kv head", kMaxGroups);
  }
  if (n_tokens == 0 || n_heads == 0) return KLLM_B200_OK;
  if (max_seq == 0 || n_slots == 0) return fail(KLLM_B200_ERR_SHAPE, "attention: empty cache");
  if (max_seq > (1LL << 30) || n_kv_heads > 65535) return fail(KLLM_B200_ERR_SHAPE, "attention: cache too large");
  if (!q || !k_cache || !v_cache || !out || !positions || !slots) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "attention: null pointer");
  }
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) {
    return fail(KLLM_B200_ERR_ALIGN, "attention: q, caches and out must be 16-byte aligned");
  }
  return KLLM_B200_OK;
}

constexpr int64_t kPrefillMinRun = 16;  // runs this long take the prefill kernel

template <int D>
int launch_prefill_tc(AttnArgs& a, const LaunchOpts& o) {
  const size_t smem = prefill_tc_smem(D);
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(attn_prefill_tc_kernel<D>), smem);
  if (err != cudaSuccess) return launch_status(err, "attention: shared memory opt-in");
  const int64_t tiles_per_run = (a.seq_len + 128 * kTcQTiles - 1) / (128 * kTcQTiles);
  const int64_t runs = (a.n_tokens + a.seq_len - 1) / a.seq_len;
  if (runs * tiles_per_run > 0x7fffffffLL) return fail(KLLM_B200_ERR_SHAPE, "attention: too many tokens");
  const dim3 grid(static_cast<unsigned>(runs * tiles_per_run), static_cast<unsigned>(a.n_heads));
  err = launch(attn_prefill_tc_kernel<D>, grid, dim3(kTcThreads), smem, o.stream, o.pdl, a);
  if (err != cudaSuccess) return launch_status(err, "attention: prefill kernel");
  return KLLM_B200_OK;
}

template <int D>
int launch_prefill(AttnArgs& a, const LaunchOpts& o) {
  const size_t smem = prefill_smem(D);
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(attn_prefill_kernel<D>), smem);
  if (err != cudaSuccess) return launch_status(err, "attention: shared memory opt-in");
  const int64_t tiles_per_run = (a.seq_len + kPfRows - 1) / kPfRows;
  const int64_t runs = (a.n_tokens + a.seq_len - 1) / a.seq_len;
  if (runs * tiles_per_run > 0x7fffffffLL) return fail(KLLM_B200_ERR_SHAPE, "attention: too many tokens");
  const dim3 grid(static_cast<unsigned>(runs * tiles_per_run), static_cast<unsigned>(a.n_heads));
  err = launch(attn_prefill_kernel<D>, grid, dim3(kAttnThreads), smem, o.stream, o.pdl, a);
  if (err != cudaSuccess) return launch_status(err, "attention: prefill kernel");
  return KLLM_B200_OK;
}

template <int D>
int launch_attention(AttnArgs& a, const LaunchOpts& o) {
  // prefill: tcgen05 at head_dim 128; at head_dim 64 the mma.sync kernel is
  // faster (half the tensor work per score, and 64-row tiles give 4x the CTAs)
  if (a.seq_len >= kPrefillMinRun) {
    if constexpr (D == 128) {
      return launch_prefill_tc<D>(a, o);
    } else {
      return launch_prefill<D>(a, o);
    }
  }
  const size_t smem = decode_smem(D);
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(attn_decode_kernel<D>), smem);
  if (err != cudaSuccess) return launch_status(err, "attention: shared memory opt-in");
  const dim3 grid(static_cast<unsigned>(a.n_tokens * a.n_chunks), static_cast<unsigned>(a.n_kv_heads));
  err = launch(attn_decode_kernel<D>, grid, dim3(kAttnThreads), smem, o.stream, o.pdl, a);
  if (err != cudaSuccess) return launch_status(err, "attention: decode kernel");
  if (a.n_chunks > 1) {
    const int64_t rows = a.n_tokens * a.n_heads;
    const dim3 cgrid(static_cast<unsigned>((rows + kCombineWarps - 1) / kCombineWarps));
    err = launch(attn_combine_kernel<D>, cgrid, dim3(kCombineWarps * 32), 0, o.stream, true, a);
    if (err != cudaSuccess) return launch_status(err, "attention: combine kernel");
  }
  return KLLM_B200_OK;
}

}  // namespace

int attention_workspace_bytes(int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                              int64_t max_seq, int64_t* bytes) {
  if (!bytes) return fail(KLLM_B200_ERR_INVALID_ARG, "attention_workspace_bytes: null pointer");
  *bytes = 0;
  if (n_tokens < 0 || n_heads < 0 || n_kv_heads < 0 || head_dim < 0 || max_seq < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "attention_workspace_bytes: negative size");
  }
  if (n_tokens == 0 || n_heads == 0 || n_kv_heads == 0 || max_seq == 0) return KLLM_B200_OK;
  *bytes = workspace_for(n_tokens, n_heads, head_dim, max_seq, preferred_chunk(n_tokens, n_kv_heads, max_seq));
  return KLLM_B200_OK;
}

int attention_head_major(const void* q, const void* k_cache, const void* v_cache, void* out,
                         const int32_t* positions, const int32_t* slots, int64_t n_tokens, int64_t seq_len,
                         int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t n_slots, int64_t max_seq,
                         int dtype, void* workspace, int64_t workspace_bytes, int32_t* err_flags,
                         const LaunchOpts& o, int* n_launched) {
  if (n_launched) *n_launched = 0;
  int rc = check_attention_args(q, k_cache, v_cache, out, positions, slots, n_tokens, n_heads, n_kv_heads,
                                head_dim, n_slots, max_seq, dtype);
  if (rc != KLLM_B200_OK || n_tokens == 0 || n_heads == 0) return rc;
  if (seq_len < 1) return fail(KLLM_B200_ERR_SHAPE, "attention: seq_len must be >= 1");
  if (workspace_bytes < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "attention: negative workspace size");
  if (workspace_bytes > 0 && (!workspace || !aligned16(workspace))) {
    return fail(KLLM_B200_ERR_ALIGN, "attention: workspace must be non-null and 16-byte aligned");
  }
  if (n_heads > 65535) return fail(KLLM_B200_ERR_SHAPE, "attention: too many heads");
  // the preferred chunk, doubled until its partials fit the workspace (one
  // chunk per sequence needs none); the prefill kernel does not split
  int64_t chunk = seq_len >= kPrefillMinRun ? max_seq : preferred_chunk(n_tokens, n_kv_heads, max_seq);
  while (workspace_for(n_tokens, n_heads, head_dim, max_seq, chunk) > (workspace ? workspace_bytes : 0)) chunk *= 2;
  const int64_t n_chunks = (max_seq + chunk - 1) / chunk;
  if (n_tokens * n_chunks > 0x7fffffffLL) return fail(KLLM_B200_ERR_SHAPE, "attention: too many tokens");

  AttnArgs a = {};
  a.q = static_cast<const __half*>(q);
  a.k_cache = static_cast<const __half*>(k_cache);
  a.v_cache = static_cast<const __half*>(v_cache);
  a.out = static_cast<__half*>(out);
  a.positions = positions;
  a.slots = slots;
  a.err_flags = err_flags;
  a.n_tokens = n_tokens;
  a.n_heads = static_cast<int>(n_heads);
  a.n_kv_heads = static_cast<int>(n_kv_heads);
  a.groups = static_cast<int>(n_heads / n_kv_heads);
  a.max_seq = static_cast<int>(max_seq);
  a.n_slots = static_cast<int>(n_slots > 0x7fffffffLL ? 0x7fffffffLL : n_slots);
  a.chunk = static_cast<int>(chunk);
  a.n_chunks = static_cast<int>(n_chunks);
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
  a.seq_len = seq_len;
  if (n_chunks > 1) {
    a.part_o = static_cast<float*>(workspace);
    a.part_ml = a.part_o + n_tokens * n_heads * n_chunks * head_dim;
  }
  rc = head_dim == 64 ? launch_attention<64>(a, o) : launch_attention<128>(a, o);
  if (rc == KLLM_B200_OK && n_launched) *n_launched = (seq_len < kPrefillMinRun && n_chunks > 1) ? 2 : 1;
  return rc;
}

}  // namespace kb

extern "C" int kllm_b200_attention_workspace_bytes(int64_t n_tokens, int64_t n_heads, int64_t n_kv_heads,
                                                   int64_t head_dim, int64_t max_seq, int64_t* bytes) {
  return kb::attention_workspace_bytes(n_tokens, n_heads, n_kv_heads, head_dim, max_seq, bytes);
}

extern "C" int kllm_b200_attention_head_major(const void* q, const void* k_cache, const void* v_cache, void* out,
                                              const int32_t* positions, const int32_t* slots, int64_t n_tokens,
                                              int64_t seq_len, int64_t n_heads, int64_t n_kv_heads,
                                              int64_t head_dim, int64_t n_slots, int64_t max_seq, int dtype,
                                              void* workspace, int64_t workspace_bytes, int32_t* err_flags,
                                              void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::attention_head_major(q, k_cache, v_cache, out, positions, slots, n_tokens, seq_len, n_heads,
                                  n_kv_heads, head_dim, n_slots, max_seq, dtype, workspace, workspace_bytes,
                                  err_flags, o);
}
