// gemm.cu — fp16 GEMM on the Blackwell tensor cores (tcgen05, TMA) with the
// epilogues that follow it in a decoder layer fused in:
//
//   linear        out = fp16(fp16(x . w^T) + bias)   replaces linear() =
//                 matmul + add_bias_inplace (src/model/llama.cpp:12-24;
//                 cuda_matmul src/op/cuda/matmul.cu:130-160 and
//                 cuda_add_bias_inplace src/op/cuda/add.cu:59-69)
//   linear_swiglu out = silu_mul(linear(x, w_gate, b_gate), linear(x, w_up, b_up))
//                 replaces the MLP's gate and up linears and silu_mul
//                 (src/model/llama.cpp:145-158); gate and up never reach HBM.
//
// Layout: x [m, k] and w [n, k] row-major, both contiguous along k (the
// reference's out[m, n] = a[m, k] * b[n, k]^T, src/op/cpu/matmul.cpp:9-33).
// The epilogue rounds the fp32 accumulator to fp16 (round to nearest even,
// as cuBLAS's fp16 output does), then adds the bias and rounds again, the
// two roundings of matmul followed by add_bias_inplace; silu_mul then runs on
// those fp16 values with the same arithmetic as kllm_b200_silu_mul, so the
// fused op equals linear + linear + silu_mul of this library bit for bit.
//
// Kernel: persistent, one CTA per SM, 128 x BN accumulator tiles with BN in
// {256, 224, 192, 128} chosen per problem (pick_tile_width: tiles that fit n,
// a last wave that is not mostly idle); a SwiGLU tile is BN / 2 output
// columns: BN / 2 gate rows and BN / 2 up rows of the weights stacked as the
// UMMA's N. Warp 0 issues TMA loads of 64-wide k slices (128-byte swizzle)
// into a ring of 4 to 6 stages (up to 16 for a few rows of x); warp 1
// issues tcgen05.mma (M 128, N BN, K 16) into one of two fp32 accumulators
// in tensor memory; warps 2-5 read
// the other accumulator back (tcgen05.ld, one row per thread), apply the
// epilogue and write each warp's 32 x 32 output chunks through shared memory
// with TMA stores, so the epilogue of tile i overlaps the main loop of tile
// i + 1. Tiles are visited in groups of 4096 rows (all column tiles of a
// group before the next group) so the CTAs in flight share x and w in L2.
// Every mbarrier wait is bounded; a wait that runs out sets
// KLLM_B200_FLAG_TIMEOUT and the CTA drains its copies and MMAs and returns.
//
// Decode-sized GEMMs (one row tile, m <= 128) load an x box of m rows
// (rounded up to 8) into a deeper ring, and those with a long k and few
// columns split each tile's k range over a thread-block cluster (split-K,
// pick_split): every peer CTA stores the fp32 sums of its live rows into its
// slot in the leader CTA's shared memory, and the leader adds them to its
// accumulator in rank order before the epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <type_traits>

#include "ops.cuh"
#include "tcgen05.cuh"

namespace kb {
namespace {

constexpr int kBM = 128;                      // tile rows: the UMMA M
constexpr int kBK = 64;                       // k per stage: one 128-byte swizzle panel of fp16
constexpr int kABytes = kBM * kBK * 2;        // 16 KB
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kGroupRows = 4096;              // rows of x per raster group (x slab resident in L2)
constexpr int kMaxStages = 16;                // ring depth with a compact x region (one row tile)

// Tile width BN (the UMMA N, accumulator columns per tile): 256, 224, 192 or
// 128, chosen per problem by the host (pick_tile_width) so that the column
// tiles fit n and the last wave of SMs is not left mostly idle. The ring
// holds as many stages as fit beside the epilogue's staging buffers.
// The ring's shared memory, in stages of full-height x tiles: 4 for a
// split-K launch (kSplit), beside the 64 KB of fp32 partial sums its peer
// CTAs hand to the cluster's leader CTA. With one row tile the x region of a
// stage shrinks and the same memory holds more stages (GemmArgs::stages).
__host__ __device__ constexpr int gemm_stages(int bn, bool split = false) {
  return split ? 4 : (bn >= 224 ? 4 : (bn == 192 ? 5 : 6));
}
__host__ __device__ constexpr int gemm_stage_bytes(int bn) { return kABytes + bn * kBK * 2; }
// Output staging of the epilogue: per epilogue warp two 2 KB buffers, each
// one 32-row x 32-column fp16 chunk on its way to a TMA store.
constexpr int kEpiChunkBytes = 32 * 32 * 2;
constexpr int kEpiStageBytes = kEpiWarps * 2 * kEpiChunkBytes;
constexpr int kSplitBN = 128;                         // the tile width of split-K launches
constexpr int kPartBytes = 64 * 1024;                 // the leader's partial-sum slots
constexpr int kMaxSplit = 8;                          // CTAs per cluster (portable cluster size)
constexpr size_t gemm_smem(int bn, bool split = false) {
  return static_cast<size_t>(gemm_stages(bn, split)) * gemm_stage_bytes(bn) + kEpiStageBytes +
         (split ? kPartBytes : 0) + 1024;  // + alignment
}

// mbarriers: stage full (TMA bytes landed) / empty (MMAs that read it done);
// accumulator full (tile's MMAs done) / empty (epilogue read it); final drain
enum GemmBar {
  kFull = 0,
  kEmpty = kFull + kMaxStages,
  kAccFull = kEmpty + kMaxStages,
  kAccEmpty = kAccFull + 2,
  kMmaDone = kAccEmpty + 2,
  kPartFull = kMmaDone + 1,  // split-K, leader CTA, per accumulator: every peer's partial sums are in place
  kPartFree = kPartFull + 2, // split-K, peer CTA, per accumulator: the leader has read this CTA's sums
  kNumBars = kPartFree + 2
};

// Epilogue kinds: linear (bias), SwiGLU over stacked gate/up rows, and the
// q/k/v projections with bias + RoPE + KV-cache append.
enum GemmEpi { kEpiLinear = 0, kEpiSwiGLU = 1, kEpiQkvRope = 2 };

constexpr int kMaxHalfDim = 64;  // RoPE frequencies: head_dim <= 128

struct alignas(64) GemmArgs {
  CUtensorMap map_a;   // x [m, k], box 64 x 128
  CUtensorMap map_b;   // w [n, k] (SwiGLU: w_gate; QKV: wq), box 64 x BN (SwiGLU: 64 x BN / 2)
  CUtensorMap map_b2;  // SwiGLU: w_up, box 64 x BN / 2; QKV: wk
  CUtensorMap map_b3;  // QKV: wv
  CUtensorMap map_out; // out [m, n], box 32 x 32, 64-byte swizzle (when tma_out)
  __half* out;         // [m, n] (QKV: q out, [m, n_heads * head_dim])
  const void* bias;    // [n] or NULL (SwiGLU: gate bias; QKV: q bias)
  const void* bias2;   // SwiGLU: up bias; QKV: k bias; or NULL
  const void* bias3;   // QKV: v bias or NULL
  int32_t* err_flags;
  int64_t m, n;        // output rows and columns
  int m_tiles, n_tiles, k_blocks;
  int group;           // row tiles per raster group
  int split;           // CTAs per cluster sharing each tile's k range (1: no split)
  int part_rows;       // rows of the x box: m rounded up to 8 for one row tile, else 128
  uint32_t stage_tx;   // bytes one stage's TMA loads deliver
  uint32_t a_region;   // bytes of a stage's x region (part_rows x 128 bytes, rounded up to 1 KB)
  int stages;          // ring depth: as many stages as the ring's shared memory holds, <= kMaxStages
  int vec_out;         // n % 8 == 0: 16-byte stores
  int tma_out;         // linear / SwiGLU output written by TMA stores from shared memory
  // QKV + RoPE epilogue: the column tiles are q_tiles of wq, k_tiles of wk,
  // then those of wv; k and v go to the head-major caches
  // [n_slots, n_kv_heads, max_seq, head_dim] at (slots[row], positions[row])
  int q_tiles, k_tiles;
  int head_dim, n_heads, n_kv_heads;
  __half* k_cache;
  __half* v_cache;
  const int32_t* positions;
  const int32_t* slots;
  int64_t n_slots, max_seq;
  float inv_freq[kMaxHalfDim];
};

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 2-D tiled TMA load of the box at (x = k element, y = row) into shared
// memory, completing `bytes` of the transaction count of `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 2-D tiled TMA store of the box at (x = column, y = row) from shared memory,
// tracked in this thread's bulk async-group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups still read their shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until this thread's bulk groups have completed (writes performed).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void st_shared16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Row tile and column tile of persistent tile index `tile`: groups of
// `group` row tiles (kGroupRows rows of x), column-major inside a group, so
// the CTAs in flight share one slab of x and a few column tiles of w in L2
// and w is read from HBM once per group.
__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int group, int& mt, int& nt) {
  const int per_group = group * n_tiles;
  const int g = tile / per_group;
  const int first = g * group;
  const int rows = min(group, m_tiles - first);
  const int local = tile - g * per_group;
  mt = first + local % rows;
  nt = local / rows;
}

// Bias value of column c as float (fp16 or fp32 bias vector).
template <typename TB>
__device__ __forceinline__ float bias_at(const void* b, int64_t c) {
  return to_f<TB>(static_cast<const TB*>(b)[c]);
}

// fp16(acc) and, with a bias, fp16(float(fp16(acc)) + bias): matmul's output
// rounding followed by add_bias_inplace's.
template <typename TB>
__device__ __forceinline__ __half2 round_bias2(float lo, float hi, const void* bias, int64_t c) {
  __half2 h = __floats2half2_rn(lo, hi);
  if (bias != nullptr) {
    if constexpr (std::is_same<TB, __half>::value) {
      // fp16 + fp16 summed in fp32 and rounded once to fp16 equals the packed
      // fp16 add (fp32 carries >= 2 * 11 + 2 significand bits)
      h = __hadd2(h, *reinterpret_cast<const __half2*>(static_cast<const __half*>(bias) + c));
    } else {
      const float2 f = __half22float2(h);
      h = __floats2half2_rn(f.x + bias_at<TB>(bias, c), f.y + bias_at<TB>(bias, c + 1));
    }
  }
  return h;
}

template <typename TB>
__device__ __forceinline__ __half round_bias1(float v, const void* bias, int64_t c) {
  __half h = __float2half_rn(v);
  if (bias != nullptr) h = __float2half_rn(__half2float(h) + bias_at<TB>(bias, c));
  return h;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// The 32 fp16 outputs of one row's 32 accumulator columns starting at output
// column c0 (bias added when given), as four 16-byte vectors (linear).
template <typename TB>
__device__ __forceinline__ void linear_chunk(const GemmArgs& a, int64_t c0, const float (&v)[32], uint4 (&w)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    w[q].x = h2_bits(round_bias2<TB>(v[q * 8 + 0], v[q * 8 + 1], a.bias, c0 + q * 8 + 0));
    w[q].y = h2_bits(round_bias2<TB>(v[q * 8 + 2], v[q * 8 + 3], a.bias, c0 + q * 8 + 2));
    w[q].z = h2_bits(round_bias2<TB>(v[q * 8 + 4], v[q * 8 + 5], a.bias, c0 + q * 8 + 4));
    w[q].w = h2_bits(round_bias2<TB>(v[q * 8 + 6], v[q * 8 + 7], a.bias, c0 + q * 8 + 6));
  }
}

// 32 accumulator columns of one row -> out[row, c0 .. c0 + 31] (linear).
template <typename TB>
__device__ __forceinline__ void store_linear(const GemmArgs& a, int64_t row, int64_t c0, const float (&v)[32]) {
  __half* orow = a.out + row * a.n;
  if (a.vec_out && c0 + 32 <= a.n) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = h2_bits(round_bias2<TB>(v[q * 8 + 0], v[q * 8 + 1], a.bias, c0 + q * 8 + 0));
      w.y = h2_bits(round_bias2<TB>(v[q * 8 + 2], v[q * 8 + 3], a.bias, c0 + q * 8 + 2));
      w.z = h2_bits(round_bias2<TB>(v[q * 8 + 4], v[q * 8 + 5], a.bias, c0 + q * 8 + 4));
      w.w = h2_bits(round_bias2<TB>(v[q * 8 + 6], v[q * 8 + 7], a.bias, c0 + q * 8 + 6));
      st_plain(orow + c0 + q * 8, w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (c0 + j < a.n) orow[c0 + j] = round_bias1<TB>(v[j], a.bias, c0 + j);
    }
  }
}

// silu(fp16 gate) * fp16 up, rounded to fp16: the arithmetic of silu_mul.
__device__ __forceinline__ __half2 swiglu2(__half2 g, __half2 u) {
  const float2 gf = __half22float2(g), uf = __half22float2(u);
  return __floats2half2_rn(silu(gf.x) * uf.x, silu(gf.y) * uf.y);
}

// SwiGLU outputs of 32 gate and 32 up accumulator columns, as four 16-byte vectors.
template <typename TB>
__device__ __forceinline__ void swiglu_chunk(const GemmArgs& a, int64_t c0, const float (&g)[32],
                                             const float (&u)[32], uint4 (&w)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = q * 8 + e * 2;
      p[e] = h2_bits(swiglu2(round_bias2<TB>(g[j], g[j + 1], a.bias, c0 + j),
                             round_bias2<TB>(u[j], u[j + 1], a.bias2, c0 + j)));
    }
    w[q] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

// One warp's 32 rows x 32 columns of output through shared memory and a TMA
// store: lane r writes its row's four 16-byte vectors into the 2 KB buffer
// `sbuf` in the 64-byte-swizzled layout the output tensor map reads (16-byte
// chunk q of row r at r * 64 + (q ^ ((r >> 1) & 3)) * 16), then lane 0 stores
// the box at (column c0, row r0). The buffer alternates per chunk; a buffer is
// rewritten only after the store issued from it two chunks earlier has read it.
__device__ __forceinline__ void stage_and_store(const GemmArgs& a, uint32_t sbuf, int lane, int64_t c0, int64_t r0,
                                                const uint4 (&w)[4]) {
  if (lane == 0) tma_store_wait_read<1>();
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q) st_shared16(sbuf + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4), w[q]);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(&a.map_out, static_cast<int>(c0), static_cast<int>(r0), sbuf);
    tma_store_commit();
  }
}

// 32 gate and 32 up accumulator columns of one row -> out[row, c0 .. c0 + 31].
template <typename TB>
__device__ __forceinline__ void store_swiglu(const GemmArgs& a, int64_t row, int64_t c0, const float (&g)[32],
                                             const float (&u)[32]) {
  __half* orow = a.out + row * a.n;
  if (a.vec_out && c0 + 32 <= a.n) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int j = q * 8 + p * 2;
        w[p] = h2_bits(swiglu2(round_bias2<TB>(g[j], g[j + 1], a.bias, c0 + j),
                               round_bias2<TB>(u[j], u[j + 1], a.bias2, c0 + j)));
      }
      st_plain(orow + c0 + q * 8, make_uint4(w[0], w[1], w[2], w[3]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (c0 + j < a.n) {
        const float gh = __half2float(round_bias1<TB>(g[j], a.bias, c0 + j));
        const float uh = __half2float(round_bias1<TB>(u[j], a.bias2, c0 + j));
        orow[c0 + j] = __float2half_rn(silu(gh) * uh);
      }
    }
  }
}

// Split-K partial sums in the leader CTA's shared memory: for each of the two
// accumulators and each peer CTA (rank 1 .. split - 1) a slot of
// kSplitBN / 4 four-column groups x part_rows rows x 16 bytes, so the rows of
// one group a warp writes or reads are contiguous (no bank conflicts). Byte
// offset of (accumulator b, peer, group, row).
__device__ __forceinline__ uint32_t part_off(const GemmArgs& a, int b, int peer, int col4, int r) {
  return static_cast<uint32_t>((((b * (a.split - 1) + peer - 1) * (kSplitBN / 4)) + col4) * a.part_rows + r) << 4;
}

// Split-K leader, one warp: the rows of this warp (tile rows 32 * quad ..,
// all live) in the slots of peers 2 .. split - 1 are added into peer 1's
// slot, in rank order. The warp's lanes cover (four-column group, row)
// items: the live rows padded to a power of two on the low lane bits (no
// divisions), consecutive rows on consecutive lanes (contiguous 16-byte
// loads), and the loads of all peers of an item in flight together.
__device__ __forceinline__ void prereduce_peers(const GemmArgs& a, uint32_t part, int b, int quad, int lane) {
  const int64_t left = a.m - quad * 32;
  const int nr = static_cast<int>(left < 32 ? left : 32);
  int lg = 0;
  while ((1 << lg) < nr) ++lg;
  const int rr = lane & ((1 << lg) - 1);
  if (rr >= nr) return;  // a padding lane (no __syncwarp follows: the caller syncs the warp)
  const int r = quad * 32 + rr;
  const uint32_t slot = static_cast<uint32_t>(kSplitBN / 4 * a.part_rows * 16);  // bytes of one peer's slot
  for (int c4 = lane >> lg; c4 < kSplitBN / 4; c4 += 32 >> lg) {
    const uint32_t dst = part + part_off(a, b, 1, c4, r);
    float4 sum = ld_shared_f4(dst);
    float4 f[kMaxSplit - 2];
#pragma unroll
    for (int p = 2; p < kMaxSplit; ++p) {
      if (p < a.split) f[p - 2] = ld_shared_f4(dst + (p - 1) * slot);
    }
#pragma unroll
    for (int p = 2; p < kMaxSplit; ++p) {
      if (p < a.split) {
        sum.x += f[p - 2].x;
        sum.y += f[p - 2].y;
        sum.z += f[p - 2].z;
        sum.w += f[p - 2].w;
      }
    }
    st_shared_f4(dst, sum);
  }
}

// Split-K leader: add to the 32 accumulator columns col .. col + 31 of tile
// row r the peers' partial sums (peer 1's slot, into which prereduce_peers
// gathered the others), so the sum is acc + (p1 + p2 + ...) in a fixed order.
template <bool kSplit>
__device__ __forceinline__ void add_peer_partials(const GemmArgs& a, uint32_t part, int b, int r, bool live, int col,
                                                  float (&v)[32]) {
  if constexpr (kSplit) {
    if (!live) return;
    float4 f[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) f[q] = ld_shared_f4(part + part_off(a, b, 1, (col >> 2) + q, r));
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[q * 4 + 0] += f[q].x;
      v[q * 4 + 1] += f[q].y;
      v[q * 4 + 2] += f[q].z;
      v[q * 4 + 3] += f[q].w;
    }
  }
}

// The q/k/v tile's epilogue (kEpiQkvRope; a tile of kBN columns holds whole
// heads of 64 or 128 columns, all of one segment). Bias and rounding as linear() + add_bias_inplace store
// them, then for q and k the rotate-half RoPE of pairs (d, d + D/2) at the
// row's position with the same arithmetic as the fused RoPE kernel; q to its
// buffer, k and v into the caches (rows whose position or slot is out of
// range write no cache row and set the error flag).
template <int kBN, typename TB, bool kSplit>
__device__ __forceinline__ void qkv_rope_epilogue(const GemmArgs& a, uint32_t t, int64_t row, int nt, uint32_t part,
                                                  int b, int r) {
  const int D = a.head_dim;
  int seg, ct;
  if (nt < a.q_tiles) {
    seg = 0;
    ct = nt;
  } else if (nt < a.q_tiles + a.k_tiles) {
    seg = 1;
    ct = nt - a.q_tiles;
  } else {
    seg = 2;
    ct = nt - a.q_tiles - a.k_tiles;
  }
  const int col0 = ct * kBN;  // first column of the tile within its segment
  const int seg_cols = (seg == 0 ? a.n_heads : a.n_kv_heads) * D;
  const void* bias = seg == 0 ? a.bias : (seg == 1 ? a.bias2 : a.bias3);
  const bool live = row < a.m;
  int32_t pos = 0, slot = 0;
  bool cache_ok = false;
  if (live) {
    pos = a.positions[row];
    slot = a.slots[row];
    cache_ok = pos >= 0 && pos < a.max_seq && slot >= 0 && slot < a.n_slots;
    if (seg == 1 && ct == 0) {  // one tile per row reports a bad position or slot
      if (pos < 0 || pos >= a.max_seq) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
      if (slot < 0 || slot >= a.n_slots) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
    }
  }
  auto cache_row = [&](__half* cache, int head) {
    return cache + ((static_cast<int64_t>(slot) * a.n_kv_heads + head) * a.max_seq + pos) * D;
  };
  if (seg == 2) {  // v: bias only, straight into the cache
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
      float v[32];
      tmem_ld32(t + c * 32, v);
      tc_wait_ld();
      const int col = col0 + c * 32;
      if (col >= seg_cols) break;  // a segment that ends inside the tile (uniform)
      add_peer_partials<kSplit>(a, part, b, r, live, c * 32, v);
      if (live && cache_ok) {
        __half* dst = cache_row(a.v_cache, col / D) + col % D;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = h2_bits(round_bias2<TB>(v[q * 8 + 0], v[q * 8 + 1], bias, col + q * 8 + 0));
          w.y = h2_bits(round_bias2<TB>(v[q * 8 + 2], v[q * 8 + 3], bias, col + q * 8 + 2));
          w.z = h2_bits(round_bias2<TB>(v[q * 8 + 4], v[q * 8 + 5], bias, col + q * 8 + 4));
          w.w = h2_bits(round_bias2<TB>(v[q * 8 + 6], v[q * 8 + 7], bias, col + q * 8 + 6));
          st_plain(dst + q * 8, w);
        }
      }
    }
    return;
  }
  const int half = D / 2;
  // 32 frequencies at a time (d = j*32 .. j*32+31), shared by the tile's heads
#pragma unroll 1
  for (int j = 0; j < half / 32; ++j) {
    float cs[32], sn[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float2 e = rope_angle_cs(pos, a.inv_freq[j * 32 + i]);
      cs[i] = e.x;
      sn[i] = e.y;
    }
#pragma unroll 1
    for (int hc = 0; hc < kBN; hc += D) {  // heads of this tile
      const int col = col0 + hc;
      if (col >= seg_cols) break;  // a segment that ends inside the tile (uniform)
      float x1[32], x2[32];
      tmem_ld32(t + hc + j * 32, x1);
      tmem_ld32(t + hc + half + j * 32, x2);
      tc_wait_ld();
      if (!live || (seg == 1 && !cache_ok)) continue;
      add_peer_partials<kSplit>(a, part, b, r, live, hc + j * 32, x1);
      add_peer_partials<kSplit>(a, part, b, r, live, hc + half + j * 32, x2);
      uint32_t p1[16], p2[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        // fp16 rounding of the linear, the bias add, then the rotation in fp32
        const float2 a1 = __half22float2(round_bias2<TB>(x1[i], x1[i + 1], bias, col + j * 32 + i));
        const float2 a2 = __half22float2(round_bias2<TB>(x2[i], x2[i + 1], bias, col + half + j * 32 + i));
        float y1a, y2a, y1b, y2b;
        rope_rotate(a1.x, a2.x, cs[i], sn[i], y1a, y2a);
        rope_rotate(a1.y, a2.y, cs[i + 1], sn[i + 1], y1b, y2b);
        p1[i / 2] = h2_bits(__floats2half2_rn(y1a, y1b));
        p2[i / 2] = h2_bits(__floats2half2_rn(y2a, y2b));
      }
      __half* dst = seg == 0 ? a.out + row * a.n + col : cache_row(a.k_cache, col / D);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        st_plain(dst + j * 32 + q * 8, make_uint4(p1[q * 4], p1[q * 4 + 1], p1[q * 4 + 2], p1[q * 4 + 3]));
        st_plain(dst + half + j * 32 + q * 8, make_uint4(p2[q * 4], p2[q * 4 + 1], p2[q * 4 + 2], p2[q * 4 + 3]));
      }
    }
  }
}

template <int kBN, int kEpi, typename TB, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs a) {
  static_assert(!kSplit || kBN == kSplitBN, "split-K tiles are kSplitBN wide");
  constexpr bool kSwiGLU = kEpi == kEpiSwiGLU;
  // The ring's shared memory is fixed per kernel; its depth is a runtime
  // value: with one row tile the x region of a stage shrinks to the rows
  // loaded (the UMMA's reads of rows past them land in the same stage's
  // weight region and only feed accumulator rows that are never stored), so
  // more stages fit.
  constexpr uint32_t kRingBytes = gemm_stages(kBN, kSplit) * gemm_stage_bytes(kBN);
  const int stages = a.stages;
  const uint32_t stage_bytes = a.a_region + kBN * kBK * 2;
  constexpr int kBBytes = kBN * kBK * 2;
  constexpr uint32_t kTmemCols = kBN <= 128 ? 256 : 512;  // two accumulators, a power-of-two allocation
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t s_bar[kNumBars];
  __shared__ uint32_t s_tmem;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;  // stage s: A at base + s * stage_bytes, then B
  const int n_tiles_total = a.m_tiles * a.n_tiles;
  constexpr int kOutCols = kSwiGLU ? kBN / 2 : kBN;  // output columns per tile
  auto bar = [&](int i) { return smem_u32(&s_bar[i]); };
  // Tiles are dealt to clusters (without split-K a CTA is a cluster of one);
  // the `split` CTAs of a cluster take consecutive k ranges of each tile.
  const int rank = kSplit ? static_cast<int>(cluster_rank()) : 0;
  const int first_tile = kSplit ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tile_step = kSplit ? static_cast<int>(cluster_count_x()) : static_cast<int>(gridDim.x);
  const int kb0 = kSplit ? rank * a.k_blocks / a.split : 0;
  const int kb1 = kSplit ? (rank + 1) * a.k_blocks / a.split : a.k_blocks;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kAccFull + b), 1);
      mbar_init(bar(kAccEmpty + b), kEpiWarps);
      if (kSplit) {
        mbar_init(bar(kPartFull + b), 1);          // the leader's arming; the peers' stores complete its bytes
        mbar_init(bar(kPartFree + b), kEpiWarps);  // every epilogue warp of the leader
      }
    }
    mbar_init(bar(kMmaDone), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_map(&a.map_a);
    tma_prefetch_map(&a.map_b);
    if (kEpi != kEpiLinear) tma_prefetch_map(&a.map_b2);
    if (kEpi == kEpiQkvRope) tma_prefetch_map(&a.map_b3);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (kSplit) cluster_sync();  // every CTA's barriers are initialised before a peer arrives on them
  const uint32_t tmem = s_tmem;
  // x may come from the previous kernel on the stream and out may be read by it
  grid_dep_wait();
  grid_dep_launch();  // the next kernel's CTAs may take the SMs this grid leaves idle and wait there
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer: lane 0 ----------------
    if (lane == 0) {
      int it = 0;          // k slices issued by this CTA
      int s = 0, round = 0;  // the stage of slice `it` and how often the ring wrapped before it
      for (int tile = first_tile; tile < n_tiles_total && ok; tile += tile_step) {
        int mt, nt;
        tile_coords(tile, a.m_tiles, a.n_tiles, a.group, mt, nt);
        const int m0 = mt * kBM;
        int n0 = nt * kOutCols;
        const CUtensorMap* bmap = &a.map_b;
        if (kEpi == kEpiQkvRope) {  // the tile's weight: wq, wk or wv
          if (nt >= a.q_tiles + a.k_tiles) {
            bmap = &a.map_b3;
            n0 = (nt - a.q_tiles - a.k_tiles) * kOutCols;
          } else if (nt >= a.q_tiles) {
            bmap = &a.map_b2;
            n0 = (nt - a.q_tiles) * kOutCols;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          if (round > 0) {  // the slice issued one round ago into this stage has been consumed
            ok = mbar_wait(bar(kEmpty + s), (round - 1) & 1);
            if (!ok) break;
          }
          const uint32_t sa = base + s * stage_bytes, sb = sa + a.a_region;
          mbar_expect_tx(bar(kFull + s), a.stage_tx);
          tma_load_2d(sa, &a.map_a, kb * kBK, m0, bar(kFull + s));
          if (kSwiGLU) {
            tma_load_2d(sb, &a.map_b, kb * kBK, n0, bar(kFull + s));
            tma_load_2d(sb + kBBytes / 2, &a.map_b2, kb * kBK, n0, bar(kFull + s));
          } else {
            tma_load_2d(sb, bmap, kb * kBK, n0, bar(kFull + s));
          }
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
      }
      // every copy issued has landed before the CTA may exit (on the normal
      // path these phases completed long ago)
      for (int j = it > stages ? it - stages : 0; j < it; ++j) {
        if (!mbar_wait(bar(kFull + j % stages), (j / stages) & 1)) ok = false;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: lane 0 ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc(kBM, kBN, false);
      const uint64_t adesc = umma_desc(base, 16, 1024);
      const uint64_t bdesc = umma_desc(base + a.a_region, 16, 1024);
      int i = 0, s = 0, round = 0;
      for (int tile = first_tile; tile < n_tiles_total && ok; tile += tile_step, ++i) {
        const int b = i & 1;
        if (i >= 2) {  // the epilogue has read this accumulator's previous tile
          ok = mbar_wait(bar(kAccEmpty + b), ((i >> 1) - 1) & 1);
          if (!ok) break;
          tc_fence_after();
        }
        const uint32_t d = tmem + b * kBN;
        for (int kb = kb0; kb < kb1; ++kb) {
          ok = mbar_wait(bar(kFull + s), round & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>((s * stage_bytes) >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // k step: 16 elements = 32 bytes along the swizzled 128-byte row
            umma_f16(d, adesc + so + 2 * k, bdesc + so + 2 * k, kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(bar(kEmpty + s));
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
        if (!ok) break;
        umma_commit(bar(kAccFull + b));
      }
      // no MMA is in flight when tensor memory is released
      umma_commit(bar(kMmaDone));
      if (!mbar_wait(bar(kMmaDone), 0)) ok = false;
    }
  } else {
    // ---------------- epilogue: warps 2-5, one accumulator row per thread ----------------
    const int quad = warp & 3;  // tensor-memory lanes 32 * quad .. + 31 are this warp's
    const int r = quad * 32 + lane;
    const uint32_t ebuf0 = base + kRingBytes + quad * 2 * kEpiChunkBytes;  // this warp's buffers
    const uint32_t part = base + kRingBytes + kEpiStageBytes;  // split-K: the peers' partial sums
    int ebuf = 0;
    int i = 0;
    for (int tile = first_tile; tile < n_tiles_total; tile += tile_step, ++i) {
      int mt, nt;
      tile_coords(tile, a.m_tiles, a.n_tiles, a.group, mt, nt);
      const int b = i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kAccFull + b), (i >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(mt) * kBM + r;
      const bool live = row < a.m;
      const bool warp_live = static_cast<int64_t>(mt) * kBM + quad * 32 < a.m;  // any output row in this warp
      const int64_t n0 = static_cast<int64_t>(nt) * kOutCols;
      const uint32_t t = tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * kBN;
      if (kSplit && rank > 0) {
        // peer: this CTA's k range of the tile -> its slot in the leader's shared memory
        if (i >= 2) {  // the leader has read the sums this slot held two tiles ago
          ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar(kPartFree + b), ((i >> 1) - 1) & 1));
          if (!ok) break;
        }
        if (warp_live) {
          // asynchronous stores that complete their bytes on the leader's barrier
          const uint32_t dst = cluster_map(part, 0);
          const uint32_t full = cluster_map(bar(kPartFull + b), 0);
#pragma unroll 1
          for (int c = 0; c < kBN / 32; ++c) {
            float v[32];
            tmem_ld32(t + c * 32, v);
            tc_wait_ld();
            if (live) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                st_async_f4(dst + part_off(a, b, rank, c * 8 + q, r), v[q * 4], v[q * 4 + 1], v[q * 4 + 2],
                            v[q * 4 + 3], full);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kAccEmpty + b));
        continue;
      }
      if (kSplit) {  // leader: every peer's sums of this tile are in place
        if (quad == 0 && lane == 0) {  // the bytes the peers' live rows send (one tile is all of m)
          mbar_expect_tx(bar(kPartFull + b), static_cast<uint32_t>((a.split - 1) * a.m * kSplitBN * 4));
        }
        ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar(kPartFull + b), (i >> 1) & 1));
        if (!ok) break;
        if (a.split > 2 && warp_live) {
          prereduce_peers(a, part, b, quad, lane);
          __syncwarp();  // the lanes read each other's sums below
        }
      }
      if (!warp_live) {
        // no output row in this warp: nothing to store
      } else if constexpr (kEpi == kEpiQkvRope) {
        qkv_rope_epilogue<kBN, TB, kSplit>(a, t, row, nt, part, b, r);
      } else if constexpr (!kSwiGLU) {
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          tmem_ld32(t + c * 32, v);
          tc_wait_ld();
          add_peer_partials<kSplit>(a, part, b, r, live, c * 32, v);
          if (a.tma_out) {
            uint4 w[4];
            linear_chunk<TB>(a, n0 + c * 32, v, w);
            stage_and_store(a, ebuf0 + ebuf * kEpiChunkBytes, lane, n0 + c * 32, row - lane, w);
            ebuf ^= 1;
          } else if (live) {
            store_linear<TB>(a, row, n0 + c * 32, v);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kBN / 64; ++c) {
          float g[32], u[32];
          tmem_ld32(t + c * 32, g);
          tmem_ld32(t + kBN / 2 + c * 32, u);
          tc_wait_ld();
          add_peer_partials<kSplit>(a, part, b, r, live, c * 32, g);
          add_peer_partials<kSplit>(a, part, b, r, live, kBN / 2 + c * 32, u);
          if (a.tma_out) {
            uint4 w[4];
            swiglu_chunk<TB>(a, n0 + c * 32, g, u, w);
            stage_and_store(a, ebuf0 + ebuf * kEpiChunkBytes, lane, n0 + c * 32, row - lane, w);
            ebuf ^= 1;
          } else if (live) {
            store_swiglu<TB>(a, row, n0 + c * 32, g, u);
          }
        }
      }
      tc_fence_before();
      __syncwarp();  // the warp's reads of the peers' slots are done
      if (lane == 0) mbar_arrive(bar(kAccEmpty + b));
      // lane p frees peer p's slot (a release arrive at cluster scope)
      if (kSplit && lane >= 1 && lane < a.split) mbar_arrive_cluster(bar(kPartFree + b), lane);
    }
    if (lane == 0) tma_store_wait_all();  // the TMA stores have read their buffers and written the output
  }

  if (!ok) set_flag(a.err_flags, KLLM_B200_FLAG_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  // split-K: no CTA leaves while a peer may still write its shared memory or arrive on its barriers
  if (kSplit) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// cuTensorMapEncodeTiled from the driver, through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor map of a row-major fp16 [rows, k] matrix read in boxes of 64 (k) x
// box_rows, 128-byte swizzled; reads past the edges return zeros.
// Tensor map of a row-major fp16 [rows, cols] matrix moved in boxes of
// box_cols x box_rows with the given swizzle; loads past the edges read
// zeros, stores past them are dropped.
int make_map2d(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows,
               CUtensorMapSwizzle swizzle, const char* what) {
  auto fn = encode_tiled();
  if (fn == nullptr) return fail(KLLM_B200_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KLLM_B200_ERR_INVALID_ARG, "%s: tensor map rejected (CUresult %d)", what, (int)r);
  return KLLM_B200_OK;
}

// Operand map: [rows, k] read in 64 (k) x box_rows boxes, 128-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int box_rows, const char* what) {
  return make_map2d(map, ptr, rows, k, kBK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B, what);
}

int check_gemm_args(const char* what, const void* x, const void* w, const void* w2, const void* bias,
                    const void* bias2, int bias_dtype, const void* out, int64_t m, int64_t n, int64_t k,
                    bool swiglu) {
  if (m < 0 || n < 0 || k < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "%s: negative size", what);
  if ((bias || bias2) && bias_dtype != KLLM_B200_F16 && bias_dtype != KLLM_B200_F32) {
    return fail(KLLM_B200_ERR_DTYPE, "%s: bias dtype %d not supported (F32, F16)", what, bias_dtype);
  }
  if (m == 0 || n == 0) return KLLM_B200_OK;
  if (k == 0) return fail(KLLM_B200_ERR_SHAPE, "%s: k must be positive", what);
  if (k % 8 != 0) return fail(KLLM_B200_ERR_SHAPE, "%s: k = %lld is not a multiple of 8", what, (long long)k);
  if (k > (1LL << 31) || m > (1LL << 31) || n > (1LL << 31)) {
    return fail(KLLM_B200_ERR_SHAPE, "%s: dimension too large", what);
  }
  if (!x || !w || !out || (swiglu && !w2)) return fail(KLLM_B200_ERR_INVALID_ARG, "%s: null pointer", what);
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || (swiglu && !aligned16(w2))) {
    return fail(KLLM_B200_ERR_ALIGN, "%s: x, weights and out must be 16-byte aligned", what);
  }
  if ((bias && (reinterpret_cast<uintptr_t>(bias) & 3u)) || (bias2 && (reinterpret_cast<uintptr_t>(bias2) & 3u))) {
    return fail(KLLM_B200_ERR_ALIGN, "%s: biases must be 4-byte aligned", what);
  }
  return KLLM_B200_OK;
}

template <int kBN, int kEpi, typename TB, bool kSplit>
int launch_gemm(GemmArgs& a, const LaunchOpts& o, const char* what) {
  auto kernel = gemm_tc_kernel<kBN, kEpi, TB, kSplit>;
  constexpr size_t smem = gemm_smem(kBN, kSplit);
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(kernel), smem);
  if (err != cudaSuccess) return launch_status(err, what);
  const int64_t tiles = static_cast<int64_t>(a.m_tiles) * a.n_tiles;
  if (kSplit) {
    const int clusters = active_clusters_raw(reinterpret_cast<const void*>(kernel), kThreads, smem, a.split);
    if (clusters < 1) return fail(KLLM_B200_ERR_CUDA, "%s: no cluster of %d CTAs fits the device", what, a.split);
    const int n = static_cast<int>(tiles < clusters ? tiles : clusters);
    err = launch_clustered(kernel, dim3(n * a.split), dim3(kThreads), smem, o.stream, o.pdl, a.split, a);
  } else {
    const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
    err = launch(kernel, dim3(grid), dim3(kThreads), smem, o.stream, o.pdl, a);
  }
  return launch_status(err, what);
}

// Split-K: CTAs per cluster sharing each tile's k range. Only for GEMMs of
// one row tile (m <= 128: decode batches) with few column tiles (n <= 2048),
// whose handful of CTAs would otherwise each stream a strip of weights alone.
// Half as many CTAs as k slices of 64, at most kMaxSplit, and two tiles'
// partial sums of the peers within kPartBytes; a long k (>= 32 slices) splits
// from 2 CTAs, a shorter one only from 4 (measured on B200 at m = 8: the
// 896 x 4864 down projection 26.7 -> 10.5 us with 8 CTAs, the 896 x 896 o
// projection 8.4 -> 7.9 us with 7; at m = 64, where the slots allow 2, only
// the long k gains; splits of wide n lose: per-tile hand-offs cost more than
// the extra CTAs gain). `n` is the output columns of one weight: a fused op
// passes the width its separate linear would have, so both split alike and
// stay bit-identical.
int pick_split(int64_t m, int64_t n, int64_t k) {
  if (m > kBM || m <= 0 || n > 2048) return 1;
  const int64_t k_blocks = (k + kBK - 1) / kBK;
  const int64_t rows = (m + 7) / 8 * 8;
  int64_t s = k_blocks / 2;
  if (s > kMaxSplit) s = kMaxSplit;
  const int64_t by_smem = 1 + kPartBytes / (2 * rows * kSplitBN * 4);
  if (s > by_smem) s = by_smem;
  if (s < (k_blocks >= 32 ? 2 : 4)) return 1;
  // clusters of s CTAs must fit the device (every split kernel has the same
  // shared memory and threads)
  auto probe = gemm_tc_kernel<kSplitBN, kEpiLinear, __half, true>;
  const size_t smem = gemm_smem(kSplitBN, true);
  if (allow_smem(reinterpret_cast<const void*>(probe), smem) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  while (s >= 2 && active_clusters_raw(reinterpret_cast<const void*>(probe), kThreads, smem, (int)s) < 1) --s;
  return s >= 2 ? static_cast<int>(s) : 1;
}

// The x operand's box and the ring: with one row tile the x box is m
// rounded up to 8 rows and a stage's x region only that many rows (rounded
// up to 1 KB, the swizzle atom), so the ring of the kernel's fixed shared
// memory holds more stages. `bn` is the tile width, `split` the CTAs per
// cluster.
int setup_a(GemmArgs& a, const void* x, int64_t m, int64_t k, int bn, int split, const char* what) {
  const int rows = m <= kBM ? static_cast<int>((m + 7) / 8 * 8) : kBM;
  a.split = split;
  a.part_rows = rows;
  a.a_region = static_cast<uint32_t>((rows * kBK * 2 + 1023) / 1024 * 1024);
  const uint32_t ring = static_cast<uint32_t>(gemm_stages(bn, split > 1) * gemm_stage_bytes(bn));
  const uint32_t stage = a.a_region + static_cast<uint32_t>(bn * kBK * 2);
  a.stages = static_cast<int>(ring / stage < kMaxStages ? ring / stage : kMaxStages);
  a.stage_tx = static_cast<uint32_t>(rows * kBK * 2 + bn * kBK * 2);
  return make_map(&a.map_a, x, m, k, rows, what);
}

// Tile width for an m x n problem: the candidate with the fewest accumulator
// columns swept by the busiest CTA (tiles per CTA x width; a narrower tile
// that fits n exactly, e.g. 224 for n = 896, wins over a half-empty last
// 256-wide tile), with
// 128-wide tiles charged 45% extra per column (measured on B200: an N = 128
// UMMA reads 4/3 the shared-memory bytes per FLOP and each x tile is fetched
// twice as often; 832 against 1190 TFLOP/s on the Qwen2.5-0.5B MLP).
// `only_128_256` restricts the choice to the two widths the q/k/v epilogue
// has (whole heads of one segment per tile).
int pick_tile_width(int64_t m, int64_t n, bool swiglu, bool only_128_256 = false) {
  const int64_t sms = sm_count();
  const int64_t m_tiles = (m + kBM - 1) / kBM;
  int64_t best_cost = -1;
  int best = 256;
  for (int bn : {256, 224, 192, 128}) {
    if (swiglu && bn == 224) continue;  // a SwiGLU tile's gate and up halves are whole 32-column chunks
    if (only_128_256 && bn != 256 && bn != 128) continue;
    const int64_t cols = swiglu ? bn / 2 : bn;
    const int64_t tiles = m_tiles * ((n + cols - 1) / cols);
    const int64_t cost = (tiles + sms - 1) / sms * bn * (bn >= 192 ? 20 : 29);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <int kBN, bool kSplit = false>
int dispatch_linear(GemmArgs& a, bool f32_bias, const LaunchOpts& o, const char* what) {
  return f32_bias ? launch_gemm<kBN, kEpiLinear, float, kSplit>(a, o, what)
                  : launch_gemm<kBN, kEpiLinear, __half, kSplit>(a, o, what);
}

template <int kBN, bool kSplit = false>
int dispatch_gemm(GemmArgs& a, bool swiglu, bool f32_bias, const LaunchOpts& o, const char* what) {
  if (swiglu) {
    return f32_bias ? launch_gemm<kBN, kEpiSwiGLU, float, kSplit>(a, o, what)
                    : launch_gemm<kBN, kEpiSwiGLU, __half, kSplit>(a, o, what);
  }
  return dispatch_linear<kBN, kSplit>(a, f32_bias, o, what);
}

int run_gemm(const void* x, const void* w, const void* w2, const void* bias, const void* bias2, int bias_dtype,
             void* out, int64_t m, int64_t n, int64_t k, int32_t* err_flags, bool swiglu, const LaunchOpts& o) {
  const char* what = swiglu ? "linear_swiglu" : "linear";
  int rc = check_gemm_args(what, x, w, w2, bias, bias2, bias_dtype, out, m, n, k, swiglu);
  if (rc != KLLM_B200_OK || m == 0 || n == 0) return rc;
  const int split = pick_split(m, n, k);
  const int bn = split > 1 ? kSplitBN : pick_tile_width(m, n, swiglu);
  const int out_cols = swiglu ? bn / 2 : bn;  // output columns per tile
  const int64_t m_tiles = (m + kBM - 1) / kBM, n_tiles = (n + out_cols - 1) / out_cols;
  if (m_tiles * n_tiles > 0x7fffffffLL) return fail(KLLM_B200_ERR_SHAPE, "%s: too many tiles", what);
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  if ((rc = setup_a(a, x, m, k, bn, split, what)) != KLLM_B200_OK) return rc;
  if ((rc = make_map(&a.map_b, w, n, k, out_cols, what)) != KLLM_B200_OK) return rc;
  if (swiglu && (rc = make_map(&a.map_b2, w2, n, k, out_cols, what)) != KLLM_B200_OK) return rc;
  a.out = static_cast<__half*>(out);
  a.bias = bias;
  a.bias2 = bias2;
  a.err_flags = err_flags;
  a.m = m;
  a.n = n;
  a.m_tiles = static_cast<int>(m_tiles);
  a.n_tiles = static_cast<int>(n_tiles);
  a.k_blocks = static_cast<int>((k + kBK - 1) / kBK);
  a.group = kGroupRows / kBM;
  a.vec_out = n % 8 == 0;
  if (a.vec_out) {  // TMA stores: the output row pitch (n * 2 bytes) is a multiple of 16
    if ((rc = make_map2d(&a.map_out, out, m, n, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B, what)) != KLLM_B200_OK) return rc;
    a.tma_out = 1;
  }
  const bool f32_bias = (bias || bias2) && bias_dtype == KLLM_B200_F32;
  if (split > 1) return dispatch_gemm<kSplitBN, true>(a, swiglu, f32_bias, o, what);
  switch (bn) {
    case 256: return dispatch_gemm<256>(a, swiglu, f32_bias, o, what);
    case 192: return dispatch_gemm<192>(a, swiglu, f32_bias, o, what);
    case 128: return dispatch_gemm<128>(a, swiglu, f32_bias, o, what);
    default: return dispatch_linear<224>(a, f32_bias, o, what);  // linear only
  }
}

template <typename TB>
int launch_qkv(GemmArgs& a, int bn, const LaunchOpts& o, const char* what) {
  if (bn != 256 && bn != 128) return fail(KLLM_B200_ERR_SHAPE, "%s: tile width %d has no q/k/v epilogue", what, bn);
  if (a.split > 1) return launch_gemm<kSplitBN, kEpiQkvRope, TB, true>(a, o, what);
  return bn == 256 ? launch_gemm<256, kEpiQkvRope, TB, false>(a, o, what)
                   : launch_gemm<128, kEpiQkvRope, TB, false>(a, o, what);
}

}  // namespace

int qkv_linear_rope_kv_append(const void* x, const void* wq, const void* wk, const void* wv, const void* bq,
                              const void* bk, const void* bv, int bias_dtype, const int32_t* positions,
                              const int32_t* slots, int64_t n_tokens, int64_t hidden, int64_t n_heads,
                              int64_t n_kv_heads, int64_t head_dim, float theta, void* q_out, void* k_cache,
                              void* v_cache, int64_t n_slots, int64_t max_seq, int32_t* err_flags,
                              const LaunchOpts& o) {
  const char* what = "qkv_linear_rope_kv_append";
  if (n_tokens < 0 || hidden < 0 || n_heads < 0 || n_kv_heads < 0 || n_slots < 0 || max_seq < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "%s: negative size", what);
  }
  if (head_dim != 64 && head_dim != 128) {
    return fail(KLLM_B200_ERR_SHAPE, "%s: head_dim %lld not supported (64, 128)", what, (long long)head_dim);
  }
  if ((bq || bk || bv) && bias_dtype != KLLM_B200_F16 && bias_dtype != KLLM_B200_F32) {
    return fail(KLLM_B200_ERR_DTYPE, "%s: bias dtype %d not supported (F32, F16)", what, bias_dtype);
  }
  if (n_tokens == 0) return KLLM_B200_OK;
  if (n_heads == 0 || n_kv_heads == 0) return fail(KLLM_B200_ERR_SHAPE, "%s: no heads", what);
  if (hidden == 0 || hidden % 8 != 0) {
    return fail(KLLM_B200_ERR_SHAPE, "%s: hidden = %lld is not a positive multiple of 8", what, (long long)hidden);
  }
  if (n_slots == 0 || max_seq == 0) return fail(KLLM_B200_ERR_SHAPE, "%s: empty cache", what);
  if (n_tokens > (1LL << 31) || hidden > (1LL << 31) || n_heads * head_dim > (1LL << 24) ||
      n_kv_heads * head_dim > (1LL << 24)) {
    return fail(KLLM_B200_ERR_SHAPE, "%s: dimension too large", what);
  }
  if (!x || !wq || !wk || !wv || !positions || !slots || !q_out || !k_cache || !v_cache) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "%s: null pointer", what);
  }
  if (!aligned16(x) || !aligned16(wq) || !aligned16(wk) || !aligned16(wv) || !aligned16(q_out) ||
      !aligned16(k_cache) || !aligned16(v_cache)) {
    return fail(KLLM_B200_ERR_ALIGN, "%s: x, weights, q and the caches must be 16-byte aligned", what);
  }
  for (const void* b : {bq, bk, bv}) {
    if (b && (reinterpret_cast<uintptr_t>(b) & 3u)) return fail(KLLM_B200_ERR_ALIGN, "%s: biases must be 4-byte aligned", what);
  }
  const int64_t qd = n_heads * head_dim, kvd = n_kv_heads * head_dim;
  // a tile never spans two segments: 256-wide tiles only when both segment
  // widths are multiples of 256, and then only where the tile model prefers them
  // split as the q linear would (the k and v linears split alike whenever they
  // are on the same side of pick_split's column limit as q)
  const int split = pick_split(n_tokens, n_heads * head_dim, hidden);
  const int bn = split > 1 ? kSplitBN
                           : ((qd % 256 == 0 && kvd % 256 == 0) ? pick_tile_width(n_tokens, qd + 2 * kvd, false, true)
                                                                 : 128);
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  int rc;
  if ((rc = setup_a(a, x, n_tokens, hidden, bn, split, what)) != KLLM_B200_OK) return rc;
  if ((rc = make_map(&a.map_b, wq, qd, hidden, bn, what)) != KLLM_B200_OK) return rc;
  if ((rc = make_map(&a.map_b2, wk, kvd, hidden, bn, what)) != KLLM_B200_OK) return rc;
  if ((rc = make_map(&a.map_b3, wv, kvd, hidden, bn, what)) != KLLM_B200_OK) return rc;
  a.out = static_cast<__half*>(q_out);
  a.bias = bq;
  a.bias2 = bk;
  a.bias3 = bv;
  a.err_flags = err_flags;
  a.m = n_tokens;
  a.n = qd;
  a.q_tiles = static_cast<int>((qd + bn - 1) / bn);
  a.k_tiles = static_cast<int>((kvd + bn - 1) / bn);
  a.m_tiles = static_cast<int>((n_tokens + kBM - 1) / kBM);
  a.n_tiles = a.q_tiles + 2 * a.k_tiles;
  a.k_blocks = static_cast<int>((hidden + kBK - 1) / kBK);
  a.group = kGroupRows / kBM;
  a.vec_out = 1;
  a.head_dim = static_cast<int>(head_dim);
  a.n_heads = static_cast<int>(n_heads);
  a.n_kv_heads = static_cast<int>(n_kv_heads);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.positions = positions;
  a.slots = slots;
  a.n_slots = n_slots;
  a.max_seq = max_seq;
  rope_inv_freq(a.inv_freq, static_cast<int>(head_dim), theta);
  const bool f32_bias = (bq || bk || bv) && bias_dtype == KLLM_B200_F32;
  return f32_bias ? launch_qkv<float>(a, bn, o, what) : launch_qkv<__half>(a, bn, o, what);
}

int linear(const void* x, const void* w, const void* bias, int bias_dtype, void* out, int64_t m, int64_t n,
           int64_t k, int32_t* err_flags, const LaunchOpts& o) {
  return run_gemm(x, w, nullptr, bias, nullptr, bias_dtype, out, m, n, k, err_flags, false, o);
}

int linear_swiglu(const void* x, const void* w_gate, const void* w_up, const void* b_gate, const void* b_up,
                  int bias_dtype, void* out, int64_t m, int64_t n, int64_t k, int32_t* err_flags,
                  const LaunchOpts& o) {
  return run_gemm(x, w_gate, w_up, b_gate, b_up, bias_dtype, out, m, n, k, err_flags, true, o);
}

}  // namespace kb

extern "C" int kllm_b200_linear(const void* x, const void* w, const void* bias, int bias_dtype, void* out,
                                int64_t m, int64_t n, int64_t k, int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::linear(x, w, bias, bias_dtype, out, m, n, k, err_flags, o);
}

extern "C" int kllm_b200_linear_swiglu(const void* x, const void* w_gate, const void* w_up, const void* b_gate,
                                       const void* b_up, int bias_dtype, void* out, int64_t m, int64_t n,
                                       int64_t k, int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::linear_swiglu(x, w_gate, w_up, b_gate, b_up, bias_dtype, out, m, n, k, err_flags, o);
}

extern "C" int kllm_b200_qkv_linear_rope_kv_append(
    const void* x, const void* wq, const void* wk, const void* wv, const void* bq, const void* bk, const void* bv,
    int bias_dtype, const int32_t* positions, const int32_t* slots, int64_t n_tokens, int64_t hidden,
    int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float theta, void* q_out, void* k_cache, void* v_cache,
    int64_t n_slots, int64_t max_seq, int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::qkv_linear_rope_kv_append(x, wq, wk, wv, bq, bk, bv, bias_dtype, positions, slots, n_tokens, hidden,
                                       n_heads, n_kv_heads, head_dim, theta, q_out, k_cache, v_cache, n_slots,
                                       max_seq, err_flags, o);
}
