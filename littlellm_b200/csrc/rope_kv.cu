// rope_kv.cu — q/k/v bias add + rotate-half RoPE + KV-cache append (fused),
// plus the reference-compatible rope_inplace and copy_kv_to_cache.
//
// Fused op (replaces, per layer, 3x add_bias_inplace src/op/cuda/add.cu:59-69,
// 2x rope_inplace src/op/cuda/rope.cu:188-201 and copy_kv_to_cache
// src/op/cuda/kv_cache.cu:32-41, as called at src/model/llama.cpp:89-114).
//
// Work unit = 8 consecutive rotation pairs of one q or k head (d0..d0+7 with
// d0+half..: two 16-byte loads, two 16-byte stores) or 16 bytes of one v
// head. Each token is owned by one or more warps (enough that a lane holds at
// most 4 units); a warp issues all its loads first, computes the cos/sin of
// the token's frequencies into its slice of shared memory while they are in
// flight, then rotates and stores. The angle depends only on position and d,
// so all q and k heads of the token share one sincos per frequency. q is
// rotated in place; k (rotated) and v (biased) go straight to the head-major
// cache [slot, kv_head, pos, d], so neither is written back.
//
// Frequencies: inv_freq[d] = powf(theta, (-2 * d) / head_dim) evaluated on
// the host in fp32 (the expression of src/op/cpu/rope.cpp:24, which is also
// how the reference CUDA path builds its table, src/op/cuda/rope.cu:51-55)
// and passed by value. Angles use the accurate sincosf (the reference CUDA
// kernel's __sincosf loses accuracy at the large angles positions up to
// 4095 produce).
#include <cmath>

#include "ops.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxHalf = 128;   // head_dim <= 256
constexpr int kWarpsPerCta = 4;
constexpr int kWarpThreads = 32 * kWarpsPerCta;

struct RopeArgs {
  __half* q;
  const __half* k;
  const __half* v;
  const void* bq;
  const void* bk;
  const void* bv;
  const int32_t* positions;  // NULL: position = past_len + t
  const int32_t* slots;      // NULL: slot 0
  int32_t past_len;
  int64_t n_tokens;
  int n_heads, n_kv_heads, head_dim;
  __half* k_cache;
  __half* v_cache;
  int64_t n_slots, max_seq;
  int32_t* err_flags;
  int warps_per_token;
  int prefetch;  // launched with PDL: ask L2 for the token rows before the dependency wait
  float inv_freq[kMaxHalf];
};

// Eight fp32 bias values at element `off`.
__device__ __forceinline__ void load_bias8(const float* p, int64_t off, float (&b)[8]) {
  const float4 x = *reinterpret_cast<const float4*>(p + off);
  const float4 y = *reinterpret_cast<const float4*>(p + off + 4);
  b[0] = x.x; b[1] = x.y; b[2] = x.z; b[3] = x.w; b[4] = y.x; b[5] = y.y; b[6] = y.z; b[7] = y.w;
}


// fp16(x + b) for 8 lanes, b at element `off` of a bias vector (shared or
// global memory): the fp32 sum rounded to nearest even, which is what the
// reference's bias add stores. For an fp16 bias this is one packed fp16 add
// per pair: rounding the fp32 sum of two fp16 values to fp16 equals rounding
// the exact sum once, because fp32 carries 24 >= 2*11 + 2 significand bits
// (double rounding through such a format is innocuous for addition).
template <typename TB>
__device__ __forceinline__ uint4 add_bias8(uint4 x, const TB* bias, int off);

template <>
__device__ __forceinline__ uint4 add_bias8<__half>(uint4 x, const __half* bias, int off) {
  return hadd8(x, *reinterpret_cast<const uint4*>(bias + off));
}

template <>
__device__ __forceinline__ uint4 add_bias8<float>(uint4 x, const float* bias, int off) {
  float b[8];
  load_bias8(bias, off, b);
  const float2 a0 = h2_to_f2(x.x), a1 = h2_to_f2(x.y), a2 = h2_to_f2(x.z), a3 = h2_to_f2(x.w);
  return make_uint4(f2_to_h2(a0.x + b[0], a0.y + b[1]), f2_to_h2(a1.x + b[2], a1.y + b[3]),
                    f2_to_h2(a2.x + b[4], a2.y + b[5]), f2_to_h2(a3.x + b[6], a3.y + b[7]));
}


// One token is owned by `warps_per_token` warps; the token's work units are
// dealt to its warps' lanes round-robin (consecutive units on consecutive
// lanes, so loads and stores coalesce), UPL units per lane. The cos/sin of
// the token's frequencies go into the warp's slice of shared memory (one or
// a few sincosf per lane). The q/k/v biases are read through L1 (every token
// reads the same few KB); staging them in shared memory measured slower in
// the chain (an L2 round trip and a CTA barrier ahead of the loads).
//
// DT is the head_dim when it is a compile-time constant (64, 128: unit
// geometry becomes shifts), 0 for a runtime head_dim.
//
// Positions, slots and the frequency table are never written by a kernel of
// the chain, so with EARLY (a PDL launch of the chain executor after its
// first) the position load and sincos run before the grid-dependency wait,
// overlapping the previous kernel's tail, and only the activation loads wait.
// Without EARLY the kernel waits before its first global read (a no-op for a
// launch without PDL), issues the activation loads and runs the sincos while
// they are in flight.
template <int DT, int UPL, typename TB, bool EARLY>
__global__ void __launch_bounds__(kWarpThreads) qkv_rope_warp_kernel(const __grid_constant__ RopeArgs a) {
  __shared__ float s_freq[kMaxHalf];
  __shared__ __align__(16) float s_cos[kWarpsPerCta][kMaxHalf];
  __shared__ __align__(16) float s_sin[kWarpsPerCta][kMaxHalf];

  if (!EARLY) {
    grid_dep_wait();
    grid_dep_launch();
  }
  const int D = DT != 0 ? DT : a.head_dim;
  const int half = D >> 1;
  const int chunks = D >> 4;   // rotation units per head (8 pairs each)
  const int vchunks = D >> 3;  // copy units per v head (16 bytes each)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + warp;
  const int64_t t = gw / a.warps_per_token;
  const int part = static_cast<int>(gw - t * a.warps_per_token);
  const bool live = t < a.n_tokens;  // uniform per warp

  const int rot_q = a.n_heads * chunks;
  const int rot_k = a.k ? a.n_kv_heads * chunks : 0;
  const int n_rot = rot_q + rot_k;
  const int n_units = n_rot + (a.v ? a.n_kv_heads * vchunks : 0);

  // The position feeds the sincos: load it before any other global access.
  int32_t pos = 0, slot = 0;
  if (live) {
    pos = a.positions ? __ldg(a.positions + t) : a.past_len + static_cast<int32_t>(t);
    slot = a.slots ? __ldg(a.slots + t) : 0;
  }

  // unit j of this lane: kind 0 = q rotation, 1 = k rotation, 2 = v copy, -1 none;
  // `off` = element offset of the unit inside its token row (head * D + d0)
  int kind[UPL], off[UPL];
#pragma unroll
  for (int j = 0; j < UPL; ++j) {
    const int u = (part * UPL + j) * 32 + lane;
    int h = 0, d0 = 0;
    if (!live || u >= n_units) {
      kind[j] = -1;
    } else if (u < n_rot) {
      const bool is_q = u < rot_q;
      const int w = is_q ? u : u - rot_q;
      kind[j] = is_q ? 0 : 1;
      h = w / chunks;
      d0 = (w - h * chunks) << 3;
    } else {
      const int w = u - n_rot;
      kind[j] = 2;
      h = w / vchunks;
      d0 = (w - h * vchunks) << 3;
    }
    off[j] = h * D + d0;
  }

  const __half* q_tok = a.q + t * a.n_heads * D;
  const __half* k_tok = a.k + t * a.n_kv_heads * D;
  const __half* v_tok = a.v + t * a.n_kv_heads * D;
  uint4 x1[UPL], x2[UPL];
  auto issue_loads = [&]() {
#pragma unroll
    for (int j = 0; j < UPL; ++j) {
      if (kind[j] == 0) {
        x1[j] = ld_cg(q_tok + off[j]);
        x2[j] = ld_cg(q_tok + off[j] + half);
      } else if (kind[j] == 1) {
        x1[j] = ld_stream(k_tok + off[j]);
        x2[j] = ld_stream(k_tok + off[j] + half);
      } else if (kind[j] == 2) {
        x1[j] = ld_stream(v_tok + off[j]);
      }
    }
  };
  if (!EARLY) issue_loads();

  for (int i = threadIdx.x; i < half; i += blockDim.x) s_freq[i] = a.inv_freq[i];
  const TB* bq = static_cast<const TB*>(a.bq);
  const TB* bk = static_cast<const TB*>(a.bk);
  const TB* bv = static_cast<const TB*>(a.bv);
  __syncthreads();  // s_freq visible; every thread reaches this point

  if (live) {
    for (int d = lane; d < half; d += 32) {
      float sn, cs;
      sincosf(__fmul_rn(static_cast<float>(pos), s_freq[d]), &sn, &cs);
      s_cos[warp][d] = cs;
      s_sin[warp][d] = sn;
    }
  }
  if (EARLY) {
    grid_dep_wait();
    grid_dep_launch();
    issue_loads();
  }
  if (!live) return;
  __syncwarp();

  bool cache_ok = true;
  if (a.k_cache != nullptr || a.v_cache != nullptr) {
    const bool pos_ok = pos >= 0 && pos < a.max_seq;
    const bool slot_ok = slot >= 0 && slot < a.n_slots;
    if (part == 0 && lane == 0) {
      if (!pos_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
      if (!slot_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
    }
    cache_ok = pos_ok && slot_ok;
  }
  // With a compile-time head_dim, 32 is a multiple of the rotation units per
  // head, so every rotation unit of this lane covers the same 8 frequencies
  // (lane % chunks): read their cos/sin once. At 4 units per lane the 16
  // extra live registers would cost occupancy, so there they are re-read per
  // unit.
  constexpr bool kHoistCs = DT != 0 && UPL <= 3;
  float cc[8], ss[8];
  if (kHoistCs) {
    const int rd0 = (lane % chunks) << 3;
    const float4* cp = reinterpret_cast<const float4*>(&s_cos[warp][rd0]);
    const float4* sp = reinterpret_cast<const float4*>(&s_sin[warp][rd0]);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    cc[0] = c0.x; cc[1] = c0.y; cc[2] = c0.z; cc[3] = c0.w; cc[4] = c1.x; cc[5] = c1.y; cc[6] = c1.z; cc[7] = c1.w;
    ss[0] = s0.x; ss[1] = s0.y; ss[2] = s0.z; ss[3] = s0.w; ss[4] = s1.x; ss[5] = s1.y; ss[6] = s1.z; ss[7] = s1.w;
  }
  // [slot, head, pos, :] of a [n_slots, n_kv_heads, max_seq, D] plane: head h
  // of this token starts at cache_tok + h * max_seq * D
  const int64_t cache_tok = (static_cast<int64_t>(slot) * a.n_kv_heads * a.max_seq + pos) * D;
  const int64_t head_stride = a.max_seq * D;
  __half* q_out = a.q + t * a.n_heads * D;

#pragma unroll
  for (int j = 0; j < UPL; ++j) {
    if (kind[j] < 0) continue;
    if (kind[j] < 2) {
      const bool is_q = kind[j] == 0;
      float f1[8], f2[8];
      const TB* bias = is_q ? bq : bk;
      if (bias != nullptr) {
        // the biased values rounded to fp16, as the reference's separate
        // bias add stores them
        const int bo = off[j];
        unpack8(add_bias8<TB>(x1[j], bias, bo), f1);
        unpack8(add_bias8<TB>(x2[j], bias, bo + half), f2);
      } else {
        unpack8(x1[j], f1);
        unpack8(x2[j], f2);
      }
      float y1[8], y2[8];
      if (kHoistCs) {
#pragma unroll
        for (int i = 0; i < 8; ++i) rope_rotate(f1[i], f2[i], cc[i], ss[i], y1[i], y2[i]);
      } else {
        const int d0 = off[j] % D;
        const float4* cp = reinterpret_cast<const float4*>(&s_cos[warp][d0]);
        const float4* sp = reinterpret_cast<const float4*>(&s_sin[warp][d0]);
        const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
        const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) rope_rotate(f1[i], f2[i], c[i], sn[i], y1[i], y2[i]);
      }
      __half* dst;
      if (is_q) {
        dst = q_out + off[j];
      } else {
        if (a.k_cache == nullptr || !cache_ok) continue;
        const int h = off[j] / D;
        dst = a.k_cache + cache_tok + h * head_stride + (off[j] - h * D);
      }
      st_plain(dst, pack8(y1));
      st_plain(dst + half, pack8(y2));
    } else {
      if (a.v_cache == nullptr || !cache_ok) continue;
      uint4 x = x1[j];
      if (bv != nullptr) x = add_bias8<TB>(x, bv, off[j]);
      const int h = off[j] / D;
      st_plain(a.v_cache + cache_tok + h * head_stride + (off[j] - h * D), x);
    }
  }
}

// Token kernel: the fused op's fast path for the head layouts of the served
// models (head_dim, q heads, kv heads as template constants; see
// kTokenShapes). One token per W warps. A token's rotation units (8 pairs of
// one q or k head: two 16-byte loads and two 16-byte stores) are numbered
// head-major, chunk-minor and dealt to the token's warps in rows of 32: unit
// u = (j * W + part) * 32 + lane. With C = D / 16 units per head dividing
// 32, every unit of a lane has chunk lane % C, i.e. the same 8 frequencies,
// so the lane reads its 8 cos/sin from shared memory once into registers.
// The v units (16 bytes of one v head) are dealt the same way. All index
// arithmetic is on template constants, positions and slots are loaded once
// per token (one broadcast load), and a unit picks its source, bias and
// destination (q in place, or the head-major K cache) by selection, so a row
// holding both q and k heads runs one instruction stream.
//
// Qwen2.5-0.5B (64, 14, 2): one warp per token, 2 rotation units per lane and
// half a v unit. Llama-2-7B (128, 32, 32): 8 warps per token, 2 + 2.
template <int D, int HQ, int HKV, int W, typename TB, bool EARLY>
__global__ void __launch_bounds__(kWarpThreads) qkv_rope_token_kernel(const __grid_constant__ RopeArgs a) {
  constexpr int C = D / 16;              // rotation units per head
  constexpr int HALF = D / 2;
  constexpr int VC = D / 8;              // v units per head
  constexpr int R = (HQ + HKV) * C;      // rotation units per token
  constexpr int V = HKV * VC;            // v units per token
  constexpr int UR = (R + 32 * W - 1) / (32 * W);  // rotation units per lane
  constexpr int UV = (V + 32 * W - 1) / (32 * W);  // v units per lane
  static_assert(32 % C == 0, "chunks per head must divide 32");
  static_assert((W & (W - 1)) == 0, "warps per token must be a power of two");
  __shared__ __align__(16) float s_cs[kWarpsPerCta][2][HALF];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWarpsPerCta + warp;
  const int t = gw / W;
  const int part = gw % W;
  const bool live = t < a.n_tokens;  // uniform per warp
  // under PDL, the token's q, k and v rows into L2 while the previous kernel
  // drains (a hint that returns no data; the rows are read after the wait).
  // Without PDL the loads follow at once and the hint would only duplicate them.
  if (a.prefetch != 0 && live && part == 0 && lane == 0) {
    prefetch_l2_bulk(a.q + static_cast<int64_t>(t) * HQ * D, HQ * D * 2);
    prefetch_l2_bulk(a.k + static_cast<int64_t>(t) * HKV * D, HKV * D * 2);
    prefetch_l2_bulk(a.v + static_cast<int64_t>(t) * HKV * D, HKV * D * 2);
  }
  if (!EARLY) {  // nothing is read before the wait (a no-op for a launch without PDL)
    grid_dep_wait();
    grid_dep_launch();
  }

  // position and slot (never written by a kernel of the chain: loaded before
  // the dependency wait with EARLY)
  int32_t pos = 0, slot = 0;
  if (live) {
    pos = __ldg(a.positions + t);
    slot = __ldg(a.slots + t);
  }
  const bool pos_ok = pos >= 0 && pos < a.max_seq;
  const bool slot_ok = slot >= 0 && slot < a.n_slots;
  const bool cache_ok = pos_ok && slot_ok;
  if (live && part == 0 && lane == 0) {
    if (!pos_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
    if (!slot_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
  }

  const int chunk8 = (lane % C) * 8;
  uint4 x1[UR], x2[UR], xv[UV];
  auto unit_head = [&](int j) { return (j * W + part) * (32 / C) + lane / C; };

  const TB* bq = static_cast<const TB*>(a.bq);
  const TB* bk = static_cast<const TB*>(a.bk);
  const TB* bv = static_cast<const TB*>(a.bv);
  // fp16 biases of a layout with few units per lane: this lane's slices (16 bytes
  // per 8 values) are loaded into registers with the position, before the
  // dependency wait, so no bias round trip sits behind the activation loads
  // of this latency-bound case. Wider layouts (bandwidth-bound, more units
  // per lane) and fp32 biases read them through L1 when used: there the
  // extra registers cost more occupancy than the round trip.
  constexpr bool kRegBias = sizeof(TB) == 2 && 2 * UR + UV <= 5;
  uint4 b1[kRegBias ? UR : 1], b2[kRegBias ? UR : 1], bvr[kRegBias ? UV : 1];
  if (kRegBias && live) {
#pragma unroll
    for (int j = 0; j < UR; ++j) {
      const int head = unit_head(j);
      const TB* bias = head < HQ ? bq : bk;
      if (head < HQ + HKV && bias != nullptr) {
        const int bo = (head < HQ ? head : head - HQ) * D + chunk8;
        b1[j] = ld_keep(bias + bo);
        b2[j] = ld_keep(bias + bo + HALF);
      }
    }
#pragma unroll
    for (int j = 0; j < UV; ++j) {
      const int u = (j * W + part) * 32 + lane;
      if (u < V && bv != nullptr) bvr[j] = ld_keep(bv + (u / VC) * D + (u % VC) * 8);
    }
  }
  auto issue_loads = [&]() {
    if (!live) return;
#pragma unroll
    for (int j = 0; j < UR; ++j) {
      const int head = unit_head(j);
      if (head < HQ + HKV) {
        const __half* src = head < HQ ? a.q + (t * HQ + head) * D + chunk8
                                      : a.k + (t * HKV + (head - HQ)) * D + chunk8;
        x1[j] = ld_cg(src);
        x2[j] = ld_cg(src + HALF);
      }
    }
#pragma unroll
    for (int j = 0; j < UV; ++j) {
      const int u = (j * W + part) * 32 + lane;
      if (u < V) xv[j] = ld_stream(a.v + (t * HKV + u / VC) * D + (u % VC) * 8);
    }
  };
  if (!EARLY) issue_loads();
  // cos/sin of the token's HALF frequencies, HALF / 32 per lane
#pragma unroll
  for (int d = lane; d < HALF; d += 32) {
    float sn, cs;
    sincosf(__fmul_rn(static_cast<float>(pos), a.inv_freq[d]), &sn, &cs);
    s_cs[warp][0][d] = cs;
    s_cs[warp][1][d] = sn;
  }
  if (EARLY) {
    grid_dep_wait();
    grid_dep_launch();
    issue_loads();
  }
  __syncwarp();
  float c[8], sn[8], nsn[8];
  {
    const float4* cp = reinterpret_cast<const float4*>(&s_cs[warp][0][chunk8]);
    const float4* sp = reinterpret_cast<const float4*>(&s_cs[warp][1][chunk8]);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
    sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
#pragma unroll
    for (int i = 0; i < 8; ++i) nsn[i] = -sn[i];
  }
  if (!live) return;

  // head h of this token in a [n_slots, HKV, max_seq, D] plane (the host
  // checks max_seq * D < 2^31)
  const int64_t cache_tok = (static_cast<int64_t>(slot) * HKV * a.max_seq + pos) * D + chunk8;
  const int head_stride = static_cast<int>(a.max_seq) * D;
#pragma unroll
  for (int j = 0; j < UR; ++j) {
    const int head = unit_head(j);
    if (head >= HQ + HKV) continue;
    const bool is_q = head < HQ;
    const int kh = head - HQ;
    const TB* bias = is_q ? bq : bk;
    float f1[8], f2[8];
    if (bias != nullptr) {
      if constexpr (kRegBias) {
        unpack8(hadd8(x1[j], b1[j]), f1);
        unpack8(hadd8(x2[j], b2[j]), f2);
      } else {
        const int bo = (is_q ? head : kh) * D + chunk8;
        unpack8(add_bias8<TB>(x1[j], bias, bo), f1);
        unpack8(add_bias8<TB>(x2[j], bias, bo + HALF), f2);
      }
    } else {
      unpack8(x1[j], f1);
      unpack8(x2[j], f2);
    }
    float y1[8], y2[8];
    rope_rotate8_x2(f1, f2, c, sn, nsn, y1, y2);
    __half* dst = is_q ? a.q + (t * HQ + head) * D + chunk8
                       : a.k_cache + cache_tok + static_cast<int64_t>(kh) * head_stride;
    if (is_q || cache_ok) {
      st_plain(dst, pack8(y1));
      st_plain(dst + HALF, pack8(y2));
    }
  }
  if (!cache_ok) return;
#pragma unroll
  for (int j = 0; j < UV; ++j) {
    const int u = (j * W + part) * 32 + lane;
    if (u >= V) continue;
    const int vh = u / VC;
    const int vd = (u % VC) * 8;
    uint4 x = xv[j];
    if (bv != nullptr) {
      if constexpr (kRegBias) {
        x = hadd8(x, bvr[j]);
      } else {
        x = add_bias8<TB>(x, bv, vh * D + vd);
      }
    }
    st_plain(a.v_cache + cache_tok - chunk8 + static_cast<int64_t>(vh) * head_stride + vd, x);
  }
}

// Any even head_dim, fp16 or fp32 activations: one thread per rotation pair
// or per v element; no shared tables.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kThreads) qkv_rope_generic_kernel(const __grid_constant__ RopeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  TA* q = reinterpret_cast<TA*>(a.q);
  const TA* k = reinterpret_cast<const TA*>(a.k);
  const TA* v = reinterpret_cast<const TA*>(a.v);
  TA* kc = reinterpret_cast<TA*>(a.k_cache);
  TA* vc = reinterpret_cast<TA*>(a.v_cache);
  const TB* bq = static_cast<const TB*>(a.bq);
  const TB* bk = static_cast<const TB*>(a.bk);
  const TB* bv = static_cast<const TB*>(a.bv);
  const int D = a.head_dim, half = D >> 1;
  const int rot_q = a.n_heads * half;
  const int rot_k = k ? a.n_kv_heads * half : 0;
  const int cp_v = v ? a.n_kv_heads * D : 0;
  const int per_tok = rot_q + rot_k + cp_v;
  const int64_t total = a.n_tokens * per_tok;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total; u += stride) {
    const int64_t t = u / per_tok;
    const int w = static_cast<int>(u - t * per_tok);
    const int32_t pos = a.positions ? a.positions[t] : a.past_len + static_cast<int32_t>(t);
    const int32_t slot = a.slots ? a.slots[t] : 0;
    bool ok = true;
    if (kc != nullptr || vc != nullptr) {
      const bool pos_ok = pos >= 0 && pos < a.max_seq;
      const bool slot_ok = slot >= 0 && slot < a.n_slots;
      if (w == 0) {
        if (!pos_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_POSITION);
        if (!slot_ok) set_flag(a.err_flags, KLLM_B200_FLAG_BAD_SLOT);
      }
      ok = pos_ok && slot_ok;
    }
    if (w < rot_q + rot_k) {
      const bool is_q = w < rot_q;
      const int ww = is_q ? w : w - rot_q;
      const int h = ww / half;
      const int d = ww - h * half;
      const int heads = is_q ? a.n_heads : a.n_kv_heads;
      const TA* src = (is_q ? q : k) + (t * heads + h) * D;
      float x1 = to_f(src[d]), x2 = to_f(src[d + half]);
      const TB* b = is_q ? bq : bk;
      if (b != nullptr) {
        x1 = to_f(from_f<TA>(x1 + to_f(b[h * D + d])));
        x2 = to_f(from_f<TA>(x2 + to_f(b[h * D + d + half])));
      }
      const float2 c = rope_angle_cs(pos, a.inv_freq[d]);
      float y1, y2;
      rope_rotate(x1, x2, c.x, c.y, y1, y2);
      if (is_q) {
        q[(t * a.n_heads + h) * D + d] = from_f<TA>(y1);
        q[(t * a.n_heads + h) * D + d + half] = from_f<TA>(y2);
      } else if (kc != nullptr && ok) {
        const int64_t dst = ((static_cast<int64_t>(slot) * a.n_kv_heads + h) * a.max_seq + pos) * D;
        kc[dst + d] = from_f<TA>(y1);
        kc[dst + d + half] = from_f<TA>(y2);
      }
    } else {
      const int ww = w - rot_q - rot_k;
      const int h = ww / D;
      const int d = ww - h * D;
      float x = to_f(v[(t * a.n_kv_heads + h) * D + d]);
      if (bv != nullptr) x = x + to_f(bv[h * D + d]);
      if (vc != nullptr && ok) {
        vc[((static_cast<int64_t>(slot) * a.n_kv_heads + h) * a.max_seq + pos) * D + d] = from_f<TA>(x);
      }
    }
  }
}

void fill_inv_freq(RopeArgs& a, float theta) { rope_inv_freq(a.inv_freq, a.head_dim, theta); }

template <int DT, int UPL>
void (*pick_tb(bool bias16, bool early))(RopeArgs) {
  if (early) return bias16 ? qkv_rope_warp_kernel<DT, UPL, __half, true> : qkv_rope_warp_kernel<DT, UPL, float, true>;
  return bias16 ? qkv_rope_warp_kernel<DT, UPL, __half, false> : qkv_rope_warp_kernel<DT, UPL, float, false>;
}

template <int D, int HQ, int HKV, int W>
void (*pick_token_tb(bool bias16, bool early))(RopeArgs) {
  if (early) {
    return bias16 ? qkv_rope_token_kernel<D, HQ, HKV, W, __half, true> : qkv_rope_token_kernel<D, HQ, HKV, W, float, true>;
  }
  return bias16 ? qkv_rope_token_kernel<D, HQ, HKV, W, __half, false> : qkv_rope_token_kernel<D, HQ, HKV, W, float, false>;
}

struct TokenKernel {
  void (*kernel)(RopeArgs) = nullptr;
  int warps_per_token = 0;
};

// Head layouts (head_dim, q heads, kv heads) with a token kernel: Qwen2.5-0.5B,
// Llama-2-7B, Qwen2.5-7B and Llama-3-8B. W (warps per token) keeps two to
// three rotation units per lane. Other layouts take qkv_rope_warp_kernel.
TokenKernel pick_token_kernel(int D, int hq, int hkv, bool bias16, bool early) {
  if (D == 64 && hq == 14 && hkv == 2) return {pick_token_tb<64, 14, 2, 1>(bias16, early), 1};
  if (D == 128 && hq == 32 && hkv == 32) return {pick_token_tb<128, 32, 32, 8>(bias16, early), 8};
  if (D == 128 && hq == 28 && hkv == 4) return {pick_token_tb<128, 28, 4, 4>(bias16, early), 4};
  if (D == 128 && hq == 32 && hkv == 8) return {pick_token_tb<128, 32, 8, 4>(bias16, early), 4};
  return {};
}

template <int DT>
void (*pick_upl(int upl, bool bias16, bool early))(RopeArgs) {
  switch (upl) {
    case 1: return pick_tb<DT, 1>(bias16, early);
    case 2: return pick_tb<DT, 2>(bias16, early);
    case 3: return pick_tb<DT, 3>(bias16, early);
    default: return pick_tb<DT, 4>(bias16, early);
  }
}

// head_dim 64 and 128 get compile-time unit geometry; others the runtime form.
void (*pick_warp_kernel(int head_dim, int upl, bool bias16, bool early))(RopeArgs) {
  if (head_dim == 64) return pick_upl<64>(upl, bias16, early);
  if (head_dim == 128) return pick_upl<128>(upl, bias16, early);
  return pick_upl<0>(upl, bias16, early);
}

int run_rope(RopeArgs& a, int act_dtype, int bias_dtype, const LaunchOpts& o, const char* what) {
  const int D = a.head_dim;
  const bool bias16 = bias_dtype == KLLM_B200_F16;
  auto al = [](const void* p) { return p == nullptr || aligned16(p); };
  const bool fast = act_dtype == KLLM_B200_F16 && D % 16 == 0 && al(a.q) && al(a.k) && al(a.v) && al(a.bq) &&
                    al(a.bk) && al(a.bv) && al(a.k_cache) && al(a.v_cache);
  if (fast && a.k != nullptr && a.v != nullptr && a.k_cache != nullptr && a.v_cache != nullptr &&
      a.positions != nullptr && a.slots != nullptr) {
    const bool early = o.pdl && o.early_inputs;
    a.prefetch = o.pdl ? 1 : 0;
    const TokenKernel tk = pick_token_kernel(D, a.n_heads, a.n_kv_heads, bias16, early);
    const int64_t widest = a.n_heads > a.n_kv_heads ? a.n_heads : a.n_kv_heads;
    // token-row offsets are 32-bit in the kernel
    if (tk.kernel != nullptr && a.n_tokens * tk.warps_per_token < (int64_t{1} << 30) &&
        a.n_tokens * widest * D < (int64_t{1} << 31) && a.max_seq * D < (int64_t{1} << 31)) {
      const int64_t warps = a.n_tokens * tk.warps_per_token;
      const unsigned grid = static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta);
      return launch_status(launch(tk.kernel, grid, kWarpThreads, 0, o.stream, o.pdl, a), what);
    }
  }
  if (fast) {
    const int chunks = D / 16;
    const int units = a.n_heads * chunks + (a.k ? a.n_kv_heads * chunks : 0) + (a.v ? a.n_kv_heads * D / 8 : 0);
    // spread a token over enough warps that each lane holds at most 4 units
    const int wpt = units > 0 ? (units + 32 * 4 - 1) / (32 * 4) : 1;
    const int upl = units > 0 ? (units + 32 * wpt - 1) / (32 * wpt) : 1;
    a.warps_per_token = wpt;
    const int64_t warps = a.n_tokens * wpt;
    const unsigned grid = static_cast<unsigned>((warps + kWarpsPerCta - 1) / kWarpsPerCta);
    void (*k)(RopeArgs) = pick_warp_kernel(D, upl, bias16, o.pdl && o.early_inputs);
    return launch_status(launch(k, grid, kWarpThreads, 0, o.stream, o.pdl, a), what);
  }
  const int per_tok = a.n_heads * (D / 2) + (a.k ? a.n_kv_heads * (D / 2) : 0) + (a.v ? a.n_kv_heads * D : 0);
  const int64_t total = a.n_tokens * per_tok;
  if (act_dtype == KLLM_B200_F16) {
    auto k = bias16 ? qkv_rope_generic_kernel<__half, __half> : qkv_rope_generic_kernel<__half, float>;
    const unsigned grid = persistent_grid(k, kThreads, 0, kThreads, total);
    return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, a), what);
  }
  auto k = bias16 ? qkv_rope_generic_kernel<float, __half> : qkv_rope_generic_kernel<float, float>;
  const unsigned grid = persistent_grid(k, kThreads, 0, kThreads, total);
  return launch_status(launch(k, grid, kThreads, 0, o.stream, o.pdl, a), what);
}

// ---- reference copy_kv_to_cache: contiguous block copy of K and V --------

__global__ void __launch_bounds__(kThreads) copy_kv_vec_kernel(const uint4* __restrict__ k,
                                                               const uint4* __restrict__ v, uint4* __restrict__ kc,
                                                               uint4* __restrict__ vc, int64_t nvec) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < 2 * nvec; i += stride) {
    if (i < nvec) {
      st_plain(kc + i, ld_stream(k + i));
    } else {
      st_plain(vc + (i - nvec), ld_stream(v + (i - nvec)));
    }
  }
}

template <typename TS, typename TC>
__global__ void __launch_bounds__(kThreads) copy_kv_generic_kernel(const TS* k, const TS* v, TC* kc, TC* vc,
                                                                   int64_t n) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < 2 * n; i += stride) {
    if (i < n) {
      kc[i] = from_f<TC>(to_f(k[i]));
    } else {
      vc[i - n] = from_f<TC>(to_f(v[i - n]));
    }
  }
}

template <typename TS, typename TC>
int run_copy_kv_generic(const void* k, const void* v, void* kc, void* vc, int64_t n, const LaunchOpts& o) {
  auto kern = copy_kv_generic_kernel<TS, TC>;
  const unsigned grid = persistent_grid(kern, kThreads, 0, kThreads * 4, 2 * n);
  return launch_status(launch(kern, grid, kThreads, 0, o.stream, o.pdl, static_cast<const TS*>(k),
                              static_cast<const TS*>(v), static_cast<TC*>(kc), static_cast<TC*>(vc), n),
                       "copy_kv_to_cache");
}

}  // namespace

int qkv_bias_rope_kv_append(void* q, const void* k, const void* v, const void* bq, const void* bk, const void* bv,
                            int bias_dtype, const int32_t* positions, const int32_t* slots, int64_t n_tokens,
                            int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float theta, void* k_cache,
                            void* v_cache, int64_t n_slots, int64_t max_seq, int32_t* err_flags,
                            const LaunchOpts& o) {
  if (n_tokens < 0 || n_heads < 0 || n_kv_heads < 0 || head_dim < 0 || n_slots < 0 || max_seq < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "qkv_bias_rope_kv_append: negative size");
  }
  if (n_tokens == 0) return KLLM_B200_OK;
  if (head_dim == 0 || head_dim % 2 != 0 || head_dim > 2 * kMaxHalf) {
    return fail(KLLM_B200_ERR_SHAPE, "qkv_bias_rope_kv_append: head_dim %lld must be even and <= %d",
                (long long)head_dim, 2 * kMaxHalf);
  }
  if (!q || !k || !v || !positions || !slots || !k_cache || !v_cache) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "qkv_bias_rope_kv_append: null pointer");
  }
  if (n_slots < 1 || max_seq < 1) return fail(KLLM_B200_ERR_SHAPE, "qkv_bias_rope_kv_append: empty cache");
  if ((bq || bk || bv) && !is_float_dtype(bias_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "qkv_bias_rope_kv_append: bias dtype %d not supported", bias_dtype);
  }
  if (n_heads * head_dim > (1 << 24) || n_kv_heads * head_dim > (1 << 24)) {
    return fail(KLLM_B200_ERR_SHAPE, "qkv_bias_rope_kv_append: rows too wide");
  }
  RopeArgs a = {};
  a.q = static_cast<__half*>(q);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.bq = bq;
  a.bk = bk;
  a.bv = bv;
  a.positions = positions;
  a.slots = slots;
  a.n_tokens = n_tokens;
  a.n_heads = static_cast<int>(n_heads);
  a.n_kv_heads = static_cast<int>(n_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.n_slots = n_slots;
  a.max_seq = max_seq;
  a.err_flags = err_flags;
  fill_inv_freq(a, theta);
  return run_rope(a, KLLM_B200_F16, bias_dtype, o, "qkv_bias_rope_kv_append");
}

// inv_freq[d] = theta^((-2d) / head_dim) for d < head_dim / 2, in fp32 on the
// host: the expression of src/op/cpu/rope.cpp:24 (also how the reference CUDA
// path builds its table, src/op/cuda/rope.cu:51-55).
void rope_inv_freq(float* inv_freq, int head_dim, float theta) {
  for (int d = 0; d < head_dim / 2; ++d) {
    inv_freq[d] = std::pow(theta, -2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
  }
}

}  // namespace kb

extern "C" int kllm_b200_qkv_bias_rope_kv_append(void* q, const void* k, const void* v, const void* bq,
                                                 const void* bk, const void* bv, int bias_dtype,
                                                 const int32_t* positions, const int32_t* slots, int64_t n_tokens,
                                                 int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                                                 float theta, void* k_cache, void* v_cache, int64_t n_slots,
                                                 int64_t max_seq, int32_t* err_flags, void* stream) {
  kb::LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return kb::qkv_bias_rope_kv_append(q, k, v, bq, bk, bv, bias_dtype, positions, slots, n_tokens, n_heads,
                                     n_kv_heads, head_dim, theta, k_cache, v_cache, n_slots, max_seq, err_flags, o);
}

extern "C" int kllm_b200_rope_inplace(void* x, int64_t seq, int64_t heads, int64_t head_dim, int32_t past_len,
                                      float theta, int dtype, void* stream) {
  using namespace kb;
  if (seq < 0 || heads < 0 || head_dim < 0) return fail(KLLM_B200_ERR_INVALID_ARG, "rope_inplace: negative size");
  if (head_dim % 2 != 0) return fail(KLLM_B200_ERR_SHAPE, "rope requires an even head_dim");
  if (seq == 0 || heads == 0 || head_dim == 0) return KLLM_B200_OK;
  if (head_dim > 2 * kMaxHalf) return fail(KLLM_B200_ERR_SHAPE, "rope_inplace: head_dim > %d", 2 * kMaxHalf);
  if (!x) return fail(KLLM_B200_ERR_INVALID_ARG, "rope_inplace: null pointer");
  if (!is_float_dtype(dtype)) return fail(KLLM_B200_ERR_DTYPE, "rope_inplace: dtype %d not supported", dtype);
  if (heads * head_dim > (1 << 24)) return fail(KLLM_B200_ERR_SHAPE, "rope_inplace: rows too wide");
  RopeArgs a = {};
  a.q = static_cast<__half*>(x);
  a.past_len = past_len;
  a.n_tokens = seq;
  a.n_heads = static_cast<int>(heads);
  a.head_dim = static_cast<int>(head_dim);
  fill_inv_freq(a, theta);
  LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  return run_rope(a, dtype, KLLM_B200_F16, o, "rope_inplace");
}

extern "C" int kllm_b200_copy_kv_to_cache(const void* k, const void* v, int64_t seq, int64_t kv_heads,
                                          int64_t head_dim, void* k_cache, void* v_cache, int64_t max_seq,
                                          int32_t past_len, int src_dtype, int cache_dtype, void* stream) {
  using namespace kb;
  if (seq < 0 || kv_heads < 0 || head_dim < 0 || max_seq < 0) {
    return fail(KLLM_B200_ERR_INVALID_ARG, "copy_kv_to_cache: negative size");
  }
  if (past_len < 0) return fail(KLLM_B200_ERR_RANGE, "copy_kv_to_cache: negative past_len %d", past_len);
  if (static_cast<int64_t>(past_len) + seq > max_seq) return fail(KLLM_B200_ERR_CAPACITY, "KV cache capacity exceeded");
  if (!is_float_dtype(src_dtype) || !is_float_dtype(cache_dtype)) {
    return fail(KLLM_B200_ERR_DTYPE, "copy_kv_to_cache: dtypes %d/%d not supported", src_dtype, cache_dtype);
  }
  const int64_t row = kv_heads * head_dim;
  const int64_t n = seq * row;
  if (n == 0) return KLLM_B200_OK;
  if (!k || !v || !k_cache || !v_cache) return fail(KLLM_B200_ERR_INVALID_ARG, "copy_kv_to_cache: null pointer");
  LaunchOpts o;
  o.stream = static_cast<cudaStream_t>(stream);
  const int esz = dtype_size(cache_dtype);
  char* kc = static_cast<char*>(k_cache) + static_cast<int64_t>(past_len) * row * esz;
  char* vc = static_cast<char*>(v_cache) + static_cast<int64_t>(past_len) * row * esz;
  if (src_dtype == cache_dtype && (n * esz) % 16 == 0 && aligned16(k) && aligned16(v) && aligned16(kc) &&
      aligned16(vc)) {
    const int64_t nvec = n * esz / 16;
    const unsigned grid = persistent_grid(copy_kv_vec_kernel, kThreads, 0, kThreads, 2 * nvec);
    return launch_status(launch(copy_kv_vec_kernel, grid, kThreads, 0, o.stream, o.pdl,
                                static_cast<const uint4*>(k), static_cast<const uint4*>(v),
                                reinterpret_cast<uint4*>(kc), reinterpret_cast<uint4*>(vc), nvec),
                         "copy_kv_to_cache");
  }
  if (src_dtype == KLLM_B200_F16) {
    return cache_dtype == KLLM_B200_F16 ? run_copy_kv_generic<__half, __half>(k, v, kc, vc, n, o)
                                        : run_copy_kv_generic<__half, float>(k, v, kc, vc, n, o);
  }
  return cache_dtype == KLLM_B200_F16 ? run_copy_kv_generic<float, __half>(k, v, kc, vc, n, o)
                                      : run_copy_kv_generic<float, float>(k, v, kc, vc, n, o);
}
