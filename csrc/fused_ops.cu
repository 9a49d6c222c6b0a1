// Memory-bound fused ops of the decoder step:
//   * qkv_rope_store: per-head QK RMSNorm + (M-)RoPE on q and k in place, and
//     the paged KV-cache write of k and v (one warp per token-head);
//   * moe_topk / moe_scatter / moe_combine: router top-k (softmax or sigmoid
//     group-limited), expert histogram + offsets, permutation + row gather,
//     and the top-k weighted combine (+ optional gated shared expert);
//   * embed: token-embedding gather with multimodal row overwrite;
//   * sample: greedy / temperature / top-k / top-p / min-p sampling with
//     repetition penalty, one CTA per row.
//
// Reference counterparts: sgl_kernel fused_qk_norm_rope and SGLang
// MRotaryEmbedding (sglang_omni/models/qwen3_omni/thinker.py:262-323), TopK +
// FusedMoE routing (thinker.py:395-412, ming_omni/thinker.py:370-462), the
// omni embedding injection (engines/omni/runtime/sglang_ar.py:548-701) and the
// sampling path (engines/omni/runtime/sglang_ar.py:882-1032).
#include <algorithm>

#include <cuda_bf16.h>
#include <float.h>
#include <stdint.h>

#include "omni_kernels.h"
#include "pdl.cuh"
#include "sampling.cuh"

namespace omni {
namespace {

__device__ __forceinline__ void unpack8(const uint4& p, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 p;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&p);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return p;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ unsigned long long omni_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// QK norm + RoPE + KV store
// ---------------------------------------------------------------------------
__device__ __forceinline__ int mrope_section(int j, const int* sec, int interleaved) {
  if (interleaved) {
    if ((j % 3) == 1 && j < 3 * sec[1]) return 1;
    if ((j % 3) == 2 && j < 3 * sec[2]) return 2;
    return 0;
  }
  if (j < sec[0]) return 0;
  if (j < sec[0] + sec[1]) return 1;
  return 2;
}

template <int D>
__global__ void __launch_bounds__(256) qkv_rope_store_kernel(RopeStoreArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  constexpr int PER = D / 32;  // elements per lane
  __shared__ float rope_row[8 * D];  // one row per warp (neox with half % 32 != 0)
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + 2 * a.hkv;
  const int tok = warp_global / heads;
  const int head = warp_global - tok * heads;
  if (tok >= a.tokens) return;
  __nv_bfloat16* row = static_cast<__nv_bfloat16*>(a.qkv) + static_cast<int64_t>(tok) * a.qkv_stride + head * D;
  const bool is_q = head < a.hq;
  const bool is_k = !is_q && head < a.hq + a.hkv;
  const bool is_v = !is_q && !is_k;
  // Lane owns elements e = lane + 32 * i (i < PER).  For neox rotation the
  // partner of e is e +- rot/2; we load the whole row into registers via
  // shared-free shuffles by owning both halves: element index mapping below.
  // Every load this warp needs is issued before the first use (two dependent round trips:
  // row / norm weights / positions, then the cos / sin table entries).
  float x[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) x[i] = __bfloat162float(row[lane + 32 * i]);
  const __nv_bfloat16* nw = is_v ? nullptr
                                 : (is_q ? static_cast<const __nv_bfloat16*>(a.q_norm)
                                         : static_cast<const __nv_bfloat16*>(a.k_norm));
  float wn[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) wn[i] = nw != nullptr ? __bfloat162float(nw[lane + 32 * i]) : 1.f;
  int pos3[3] = {0, 0, 0};
  if (!is_v && a.rot_dim > 0) {
    if (a.pos_rows == 3) {
      pos3[0] = a.positions[tok];
      pos3[1] = a.positions[a.tokens + tok];
      pos3[2] = a.positions[2 * a.tokens + tok];
    } else {
      pos3[0] = pos3[1] = pos3[2] = a.positions[tok];
    }
  }
  if (!is_v) {
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / D + a.eps);
#pragma unroll
      for (int i = 0; i < PER; ++i) x[i] = bf16r(bf16r(x[i] * rstd) * wn[i]);
    }
    if (a.rot_dim > 0) {
      const int half = a.rot_dim / 2;
      float y[PER];
      // Partner of element e = lane + 32 i: neox with half % 32 == 0 -> same
      // lane, register i +- half/32; neox otherwise -> through this warp's
      // shared-memory copy of the row; interleaved pairs -> lane ^ 1.
      const int hs = half >> 5;
      const bool neox_smem = a.neox && (half & 31) != 0;
      float* srow = rope_row + (threadIdx.x >> 5) * D;
      if (neox_smem) {
#pragma unroll
        for (int i = 0; i < PER; ++i) srow[lane + 32 * i] = x[i];
        __syncwarp();
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        float pv;
        if (neox_smem) {
          pv = e < a.rot_dim ? srow[e < half ? e + half : e - half] : 0.f;
        } else if (a.neox) {
          const int pi = e < half ? i + hs : i - hs;
          pv = 0.f;
#pragma unroll
          for (int ii = 0; ii < PER; ++ii)
            if (ii == pi) pv = x[ii];
        } else {
          pv = __shfl_xor_sync(0xffffffffu, x[i], 1);
        }
        y[i] = x[i];
        if (e < a.rot_dim) {
          const int j = a.neox ? (e < half ? e : e - half) : (e >> 1);
          const float sign = a.neox ? (e < half ? -1.f : 1.f) : ((e & 1) ? 1.f : -1.f);
          const int s = a.pos_rows == 3 ? mrope_section(j, a.section, a.interleaved) : 0;
          const int pos = pos3[s];
          const float c = a.cos_tab[static_cast<int64_t>(pos) * half + j];
          const float sn = a.sin_tab[static_cast<int64_t>(pos) * half + j];
          y[i] = x[i] * c + sign * pv * sn;
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) x[i] = y[i];
    }
  }
  // write back q / k in place, k / v into the cache
  if (!is_v) {
#pragma unroll
    for (int i = 0; i < PER; ++i) row[lane + 32 * i] = __float2bfloat16(x[i]);
  }
  if (!is_q && a.slot_mapping != nullptr) {
    const int slot = a.slot_mapping[tok];
    if (slot >= 0 && (a.num_slots == 0 || slot < a.num_slots)) {
      const int h = is_k ? head - a.hq : head - a.hq - a.hkv;
      const int page = slot >> 6, off = slot & 63;
      __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache);
      __nv_bfloat16* dst = cache + ((static_cast<int64_t>(page) * a.hkv + h) * 64 + off) * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = __float2bfloat16(x[i]);
    }
  }
}

// head_dim 128 fast path: one warp = one token x up to kHeadsPerWarp consecutive heads.  Lane l
// owns elements 4l .. 4l+3 (8-byte loads and stores, a head row is one coalesced 256-byte
// access).  The token's cos / sin entries (one per rotated element of the lane, M-RoPE section
// by element) are loaded once and serve every q / k head of the warp; the neox partner element
// e +- rot/2 sits in the same register of lane l +- rot/8 (a shuffle), the interleaved partner
// e ^ 1 in the lane's own registers.  Every head's row load of the warp is issued before the
// first use.
constexpr int kRopeHeadsPerWarp = 8;

__device__ __forceinline__ void load4_bf16(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

__device__ __forceinline__ void store4_bf16(__nv_bfloat16* p, const float (&v)[4]) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__global__ void __launch_bounds__(128) qkv_rope_store_d128_kernel(RopeStoreArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  constexpr int D = 128;
  const int heads = a.hq + 2 * a.hkv;
  const int chunks = (heads + kRopeHeadsPerWarp - 1) / kRopeHeadsPerWarp;
  const long wg = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int tok = static_cast<int>(wg / chunks);
  if (tok >= a.tokens) return;
  const int h0 = static_cast<int>(wg - static_cast<long>(tok) * chunks) * kRopeHeadsPerWarp;
  const int e0 = 4 * lane;
  __nv_bfloat16* base = static_cast<__nv_bfloat16*>(a.qkv) + static_cast<int64_t>(tok) * a.qkv_stride;
  // every row of the warp in flight first
  float x[kRopeHeadsPerWarp][4];
#pragma unroll
  for (int u = 0; u < kRopeHeadsPerWarp; ++u) {
    const int head = h0 + u;
    if (head < heads) load4_bf16(base + head * D + e0, x[u]);
  }
  const bool any_qk = h0 < a.hq + a.hkv;
  float wq[4] = {1.f, 1.f, 1.f, 1.f}, wk[4] = {1.f, 1.f, 1.f, 1.f};
  if (any_qk && a.q_norm != nullptr) load4_bf16(static_cast<const __nv_bfloat16*>(a.q_norm) + e0, wq);
  if (any_qk && a.k_norm != nullptr) load4_bf16(static_cast<const __nv_bfloat16*>(a.k_norm) + e0, wk);
  // this lane's cos / sin, shared by the warp's q / k heads
  const int rot = a.rot_dim, half = rot >> 1;
  float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
  if (any_qk && rot > 0) {
    const int p0 = a.positions[tok];
    const int p1 = a.pos_rows == 3 ? a.positions[a.tokens + tok] : p0;
    const int p2 = a.pos_rows == 3 ? a.positions[2 * a.tokens + tok] : p0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = e0 + k;
      if (e < rot) {
        const int j = a.neox ? (e < half ? e : e - half) : (e >> 1);
        const int sec = a.pos_rows == 3 ? mrope_section(j, a.section, a.interleaved) : 0;
        const int pos = sec == 0 ? p0 : (sec == 1 ? p1 : p2);
        const int64_t idx = static_cast<int64_t>(pos) * half + j;
        const float sgn = a.neox ? (e < half ? -1.f : 1.f) : ((e & 1) ? 1.f : -1.f);
        cs[k] = a.cos_tab[idx];
        sn[k] = sgn * a.sin_tab[idx];
      }
    }
  }
  const int shift = half >> 2;                       // neox partner lane distance
  const int src_lane = e0 < half ? lane + shift : lane - shift;
  int slot = -1;
  if (a.slot_mapping != nullptr && h0 + kRopeHeadsPerWarp > a.hq) {
    slot = a.slot_mapping[tok];
    if (a.num_slots != 0 && slot >= a.num_slots) slot = -1;
  }
#pragma unroll
  for (int u = 0; u < kRopeHeadsPerWarp; ++u) {
    const int head = h0 + u;
    if (head >= heads) break;                         // warp-uniform
    const bool is_q = head < a.hq;
    const bool is_v = head >= a.hq + a.hkv;
    float (&v)[4] = x[u];
    if (!is_v) {
      if (is_q ? a.q_norm != nullptr : a.k_norm != nullptr) {
        float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
        ss = warp_sum(ss);
        const float rstd = rsqrtf(ss / D + a.eps);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = bf16r(bf16r(v[k] * rstd) * (is_q ? wq[k] : wk[k]));
      }
      if (rot > 0) {
        float pv[4];
        if (a.neox) {
#pragma unroll
          for (int k = 0; k < 4; ++k) pv[k] = __shfl_sync(0xffffffffu, v[k], src_lane);
        } else {
          pv[0] = v[1]; pv[1] = v[0]; pv[2] = v[3]; pv[3] = v[2];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (e0 + k < rot) v[k] = v[k] * cs[k] + pv[k] * sn[k];
      }
      store4_bf16(base + head * D + e0, v);
    }
    if (!is_q && slot >= 0) {
      const int h = is_v ? head - a.hq - a.hkv : head - a.hq;
      const int page = slot >> 6, off = slot & 63;
      __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_v ? a.v_cache : a.k_cache);
      store4_bf16(cache + ((static_cast<int64_t>(page) * a.hkv + h) * 64 + off) * D + e0, v);
    }
  }
}

// ---------------------------------------------------------------------------
// MoE routing
// ---------------------------------------------------------------------------
// One warp per token.  E <= 512 (E/32 values per lane).
template <int PER>
__global__ void moe_topk_kernel(MoeRouteArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tok >= a.tokens) return;
  const float* lg = a.logits + static_cast<int64_t>(tok) * a.logits_stride;
  float sc[PER];    // selection score
  float wt[PER];    // weight score
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    const float v = e < a.experts ? lg[e] : -INFINITY;
    sc[i] = v == v ? v : -INFINITY;  // a NaN logit never wins a selection
  }
  if (a.mode == 0) {
    // softmax over experts
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) m = fmaxf(m, sc[i]);
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      wt[i] = (lane + 32 * i) < a.experts ? __expf(sc[i] - m) : 0.f;
      s += wt[i];
    }
    s = warp_sum(s);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      wt[i] /= s;
      sc[i] = (lane + 32 * i) < a.experts ? wt[i] : -INFINITY;
    }
  } else {
    // sigmoid scores; selection adds the expert bias; group-limited choice
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < a.experts) {
        wt[i] = 1.f / (1.f + __expf(-sc[i]));
        sc[i] = wt[i] + (a.bias ? a.bias[e] : 0.f);
      } else {
        wt[i] = 0.f;
      }
    }
    if (a.n_group > 1) {
      // experts of group gi are e in [gi*gs, (gi+1)*gs); with gs == 32 a group is
      // one register index across the warp.
      const int gs = a.experts / a.n_group;
      float gscore[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) gscore[i] = -INFINITY;
      for (int gi = 0; gi < a.n_group; ++gi) {
        // top-2 sum inside group gi
        float best1 = -INFINITY, best2 = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int e = lane + 32 * i;
          if (e / gs == gi) {
            const float v = sc[i];
            if (v > best1) { best2 = best1; best1 = v; } else if (v > best2) { best2 = v; }
          }
        }
        // warp-level top-2 merge
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
          const float o1 = __shfl_xor_sync(0xffffffffu, best1, d);
          const float o2 = __shfl_xor_sync(0xffffffffu, best2, d);
          const float n1 = fmaxf(best1, o1);
          const float n2 = fmaxf(fminf(best1, o1), fmaxf(best2, o2));
          best1 = n1;
          best2 = n2;
        }
        const float gsc = best1 + best2;
#pragma unroll
        for (int i = 0; i < PER; ++i)
          if ((lane + 32 * i) / gs == gi) gscore[i] = gsc;
      }
      // keep the topk_group best groups: a group is dropped when at least
      // topk_group groups score strictly higher (ties keep lower index first).
      for (int gi = 0; gi < a.n_group; ++gi) {
        float my = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; ++i)
          if ((lane + 32 * i) / gs == gi) my = gscore[i];
        my = warp_max(my);
        int better = 0;
        for (int gj = 0; gj < a.n_group; ++gj) {
          float other = -INFINITY;
#pragma unroll
          for (int i = 0; i < PER; ++i)
            if ((lane + 32 * i) / gs == gj) other = gscore[i];
          other = warp_max(other);
          if (other > my || (other == my && gj < gi)) ++better;
        }
        if (better >= a.topk_group) {
#pragma unroll
          for (int i = 0; i < PER; ++i)
            if ((lane + 32 * i) / gs == gi) sc[i] = -INFINITY;
        }
      }
    }
  }
  // top-k by repeated warp argmax (lowest index wins ties)
  float wsum = 0.f;
  int my_ids[16];
  float my_w[16];
  for (int k = 0; k < a.topk; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < a.experts && (sc[i] > best || (sc[i] == best && e < bi))) {
        best = sc[i];
        bi = e;
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (bi >= a.experts) bi = 0;  // no finite score left: route to expert 0 (ids stay in range)
    // owner lane fetches the weight and removes the expert
    float w = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (lane + 32 * i == bi) {
        w = wt[i];
        sc[i] = -INFINITY;
      }
    }
    w = warp_sum(w);  // only the owner contributed
    my_ids[k] = bi;
    my_w[k] = w;
    wsum += w;
  }
  const float scale = (a.renormalize ? 1.f / wsum : 1.f) * a.scaling;
  if (lane < a.topk) {
    float w = 0.f;
    int id = 0;
    for (int k = 0; k < a.topk; ++k)
      if (k == lane) {
        w = my_w[k];
        id = my_ids[k];
      }
    a.topk_ids[tok * a.topk + lane] = id;
    a.topk_w[tok * a.topk + lane] = w * scale;
    if (a.counts) atomicAdd(&a.counts[id], 1);
  }
}

// Offsets (exclusive scan of counts, computed by every CTA) + permutation + row gather.
__global__ void moe_scatter_kernel(MoeRouteArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  extern __shared__ int s_off[];
  // exclusive scan of the expert histogram by warp 0 (32 experts per round)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    // all counts in flight at once (experts <= 512: 16 per lane), then the rounds of the scan
    constexpr int kRounds = 16;
    int cnt[kRounds];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int e = 32 * r + lane;
      cnt[r] = e < a.experts ? a.counts[e] : 0;
    }
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int base = 32 * r;
      if (base >= a.experts) break;
      const int e = base + lane;
      const int c = cnt[r];
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (e < a.experts) s_off[e] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_off[a.experts] = carry;
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e <= a.experts; e += blockDim.x) a.offsets[e] = s_off[e];
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = a.tokens * a.topk;
  // one warp per (token, k) pair
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += gridDim.x * warps) {
    int pos = 0;
    if (lane == 0) {
      const int e = a.topk_ids[i];
      pos = s_off[e] + atomicAdd(&a.cursor[e], 1);
      a.inv_perm[i] = pos;
    }
    pos = __shfl_sync(0xffffffffu, pos, 0);
    bool copy = a.x != nullptr;
    if (copy && a.local_el > 0) {  // tensor-parallel MoE: only this rank's experts are computed
      const int e = a.topk_ids[i];
      copy = e >= a.local_e0 && e < a.local_e0 + a.local_el;
    }
    if (copy) {
      const uint4* __restrict__ src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) +
                                                                     static_cast<int64_t>(i / a.topk) * a.hidden);
      uint4* __restrict__ dst =
          reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.x_perm) + static_cast<int64_t>(pos) * a.hidden);
      const int nv = a.hidden / 8;
      // the whole row in flight (8 vectors per lane per round) before any store
      for (int v0 = lane; v0 < nv; v0 += 32 * 8) {
        uint4 buf[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + 32 * u;
          if (v < nv) buf[u] = __ldg(src + v);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + 32 * u;
          if (v < nv) dst[v] = buf[u];
        }
      }
    }
  }
  if (a.self_clean) {
    // the last CTA to finish leaves counts / cursor zeroed for the next call (no memset launches)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(&a.cursor[a.experts], 1) + 1 == static_cast<int>(gridDim.x)) {
        for (int e = 0; e < a.experts; ++e) {
          a.counts[e] = 0;
          a.cursor[e] = 0;
        }
        a.cursor[a.experts] = 0;
        __threadfence();
      }
    }
  }
}

// out[t] = sum_k w[t,k] * y[inv[t,k]] (+ sigmoid(gate[t]) * shared[t]), rounded to bf16.
// With a residual: residual[t] = bf16(residual[t] + out[t]) and normed[t] = w * rmsnorm(residual[t])
// (the next block's fused add + RMSNorm, same rounding points as rmsnorm_kernel).
// One CTA of 256 threads per token, VPT 16-byte vectors per thread.
template <int VPT>
__global__ void __launch_bounds__(256) moe_combine_kernel(MoeCombineArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  __shared__ int s_pos[16];
  __shared__ float s_w[16];
  __shared__ float red[8];
  const int tok = blockIdx.x;
  if (a.wait_count > 0) {
    // expert-parallel: the expert outputs of this rank's rows are stored by their owners; wait
    // (bounded, wrap-safe compare) until every owner has raised its flag for this layer
    if (threadIdx.x < 32) {
      const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(a.wait_seq);
      const unsigned long long t0 = omni_globaltimer();
      for (int i = threadIdx.x; i < a.wait_count; i += 32) {
        uint32_t v;
        while (true) {
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.wait_flags + i) : "memory");
          if (static_cast<int>(v - target) >= 0) break;
          if (omni_globaltimer() - t0 > static_cast<unsigned long long>(a.wait_timeout_ns)) {
            if (a.status != nullptr) atomicCAS(a.status, 0, 2);  // peer timeout
            break;
          }
        }
      }
    }
    __syncthreads();
    __threadfence_system();
  }
  if (threadIdx.x < a.topk) {
    int pos = a.inv_perm[tok * a.topk + threadIdx.x];
    if (a.local_offsets != nullptr && (pos < a.local_offsets[0] || pos >= a.local_offsets[a.local_experts])) pos = -1;
    s_pos[threadIdx.x] = pos;
    s_w[threadIdx.x] = a.topk_w[tok * a.topk + threadIdx.x];
  }
  __syncthreads();
  const int nvec = a.hidden >> 3;
  const uint4* y = static_cast<const uint4*>(a.y_perm);
  float sg = 0.f;
  if (a.shared != nullptr) sg = a.shared_gate ? 1.f / (1.f + __expf(-a.shared_gate[tok * a.shared_gate_stride])) : 1.f;
  float vals[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + 256 * i;
    if (v >= nvec) continue;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    // the first 8 expert rows are loaded together (8 loads in flight), then summed in k order
    constexpr int kBatch = 8;
    uint4 rows[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      rows[k] = make_uint4(0u, 0u, 0u, 0u);
      if (k < a.topk && s_pos[k] >= 0)  // < 0: another rank's expert (tensor-parallel MoE)
        rows[k] = __ldg(y + static_cast<int64_t>(s_pos[k]) * nvec + v);
    }
    uint4 res_v = make_uint4(0u, 0u, 0u, 0u);
    if (a.residual != nullptr) res_v = static_cast<const uint4*>(a.residual)[static_cast<int64_t>(tok) * nvec + v];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (k < a.topk && s_pos[k] >= 0) {
        float f[8];
        unpack8(rows[k], f);
        const float w = s_w[k];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += w * f[j];
      }
    }
    for (int k = kBatch; k < a.topk; ++k) {
      if (s_pos[k] < 0) continue;
      float f[8];
      unpack8(__ldg(y + static_cast<int64_t>(s_pos[k]) * nvec + v), f);
      const float w = s_w[k];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += w * f[j];
    }
    if (a.shared != nullptr) {
      float f[8];
      unpack8(static_cast<const uint4*>(a.shared)[static_cast<int64_t>(tok) * nvec + v], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += sg * f[j];
    }
    uint4 h = pack8(acc);
    if (a.peer_out != nullptr)
      reinterpret_cast<uint4*>(a.peer_out[tok / a.rows_per])[static_cast<int64_t>(tok) * nvec + v] = h;
    else if (a.out != nullptr)
      static_cast<uint4*>(a.out)[static_cast<int64_t>(tok) * nvec + v] = h;
    if (a.residual != nullptr) {
      uint4* rr = static_cast<uint4*>(a.residual) + static_cast<int64_t>(tok) * nvec + v;
      float r[8];
      unpack8(h, acc);
      unpack8(res_v, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += r[j];
      const uint4 s = pack8(acc);
      *rr = s;
      unpack8(s, vals[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
    }
  }
  if (a.residual == nullptr) return;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float rstd = rsqrtf(tot / static_cast<float>(a.hidden) + a.eps);
  const uint4* wr = static_cast<const uint4*>(a.norm_w);
  uint4* yr = static_cast<uint4*>(a.normed) + static_cast<int64_t>(tok) * nvec;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + 256 * i;
    if (v >= nvec) continue;
    float wf[8], o[8];
    unpack8(wr[v], wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __bfloat162float(__float2bfloat16(vals[i][j] * rstd)) * wf[j];
    yr[v] = pack8(o);
  }
}

// ---------------------------------------------------------------------------
// Embedding gather with multimodal overwrite
// ---------------------------------------------------------------------------
__global__ void embed_kernel(EmbedArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  const int tok = blockIdx.x;
  const int mm = a.mm_index ? a.mm_index[tok] : -1;
  const uint4* src;
  if (mm >= 0) {
    src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.mm_embeds) + static_cast<int64_t>(mm) * a.hidden);
  } else {
    int id = a.ids[tok];
    if (a.vocab > 0) id = id < 0 ? 0 : (id >= a.vocab ? a.vocab - 1 : id);
    src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.table) + static_cast<int64_t>(id) * a.hidden);
  }
  uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + static_cast<int64_t>(tok) * a.hidden);
  for (int v = threadIdx.x; v < a.hidden / 8; v += blockDim.x) dst[v] = src[v];
}

// ---------------------------------------------------------------------------
// Dual-AR input embedding with the VQ codebook sum (one CTA per token)
// ---------------------------------------------------------------------------
__global__ void vq_embed_kernel(VqEmbedArgs a) {
  const int t = blockIdx.x;
  const int s = a.slot ? a.slot[t] : -1;
  int id = a.slot ? a.slot_tokens[s] : a.ids[t];
  if (a.vocab > 0) id = id < 0 ? 0 : (id >= a.vocab ? a.vocab - 1 : id);
  int r;
  bool vq;
  if (a.code_row) {
    r = a.code_row[t];
    vq = r >= 0;
  } else {
    r = a.slot ? s : t;
    vq = id >= a.sem_lo && id <= a.sem_hi;
  }
  const __nv_bfloat16* e = static_cast<const __nv_bfloat16*>(a.table) + static_cast<int64_t>(id) * a.hidden;
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + static_cast<int64_t>(t) * a.hidden;
  const int nvec = a.hidden >> 3;
  if (!vq) {
    for (int v = threadIdx.x; v < nvec; v += blockDim.x)
      reinterpret_cast<uint4*>(o)[v] = reinterpret_cast<const uint4*>(e)[v];
    return;
  }
  __shared__ int rows[32];
  if (threadIdx.x < a.ncb) {
    int c = a.codes[static_cast<int64_t>(r) * a.codes_stride + threadIdx.x];
    c = c < 0 ? 0 : (c >= a.cb_size ? a.cb_size - 1 : c);
    rows[threadIdx.x] = threadIdx.x * a.cb_size + c;
  }
  __syncthreads();
  const __nv_bfloat16* cb = static_cast<const __nv_bfloat16*>(a.codebooks);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < a.ncb; ++c) {
      const uint4 u = reinterpret_cast<const uint4*>(cb + static_cast<int64_t>(rows[c]) * a.hidden)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    const uint4 ue = reinterpret_cast<const uint4*>(e)[v];
    const __nv_bfloat162* he = reinterpret_cast<const __nv_bfloat162*>(&ue);
    uint4 uo;
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&uo);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(he[j]);
      const float x0 = bf16r(bf16r(f.x + bf16r(acc[2 * j])) * a.scale);
      const float x1 = bf16r(bf16r(f.y + bf16r(acc[2 * j + 1])) * a.scale);
      ho[j] = __floats2bfloat162_rn(x0, x1);
    }
    reinterpret_cast<uint4*>(o)[v] = uo;
  }
}

// ---------------------------------------------------------------------------
// Sampling: one CTA (1024 threads) per row (helpers in sampling.cuh).
// ---------------------------------------------------------------------------
using namespace samp;

constexpr int kSampleCand = 4096;   // candidates (value, index) kept in shared memory

// One CTA (1024 threads) per row.  Full-row passes: (1) logits processing fused with
// the row max / greedy argmax, (2) top-k threshold by a 4-pass radix select, (3) the
// surviving candidates (>= the top-k / min-p threshold, or within 40 nats of the max
// when only top-p is set) are compacted into shared memory; top-p's threshold search
// and the Gumbel-max draw then run on the candidates only.  When more candidates than
// fit survive, top-p and the draw sweep the full row instead.  The Gumbel noise of
// token i depends only on (seed, step, i), so both routes draw the same token.
__global__ void __launch_bounds__(1024) sample_kernel(SampleArgs a) {
  __shared__ float sred[33];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_kleft;
  __shared__ unsigned long long s_best;
  __shared__ int s_ncand;
  __shared__ float cand_x[kSampleCand];
  __shared__ int cand_i[kSampleCand];
  const int row = blockIdx.x;
  const int sr = a.row_slot ? a.row_slot[row] : row;  // state row
  float* lg = a.logits + static_cast<int64_t>(row) * a.logits_stride;
  const int V = a.vocab;
  const float temp = a.temperature ? a.temperature[sr] : 0.f;
  const float rep = a.rep_penalty ? a.rep_penalty[sr] : 1.f;
  const uint8_t* seen = a.seen ? a.seen + static_cast<int64_t>(sr) * a.seen_stride : nullptr;
  const bool greedy = !(temp > 0.f);
  const bool suppress = a.suppress_lo >= 0;
  const bool penal = seen != nullptr && rep != 1.f;
  const float inv_t = greedy ? 1.f : 1.f / temp;
  auto process = [&](int i, float x) {
    if (suppress && i >= a.suppress_lo && i < a.suppress_hi && i != a.suppress_keep) x = -INFINITY;
    if (penal && seen[i]) x = x > 0.f ? x / rep : x * rep;
    return greedy ? x : x * inv_t;
  };
  if (threadIdx.x == 0) s_best = 0ull;
  __syncthreads();

  // 1) processing (written back only when it changes the row) + max / argmax
  unsigned long long best = 0ull;
  float m = -INFINITY;
  if (suppress || penal || !greedy) {
    row_transform(lg, V, [&](int i, float x) {
      const float y = process(i, x);
      m = fmaxf(m, y);
      const unsigned long long k = argmax_key(y, i);
      best = k > best ? k : best;
      return y;
    });
  } else {
    row_for_each(lg, V, [&](int i, float x) {
      const unsigned long long k = argmax_key(x, i);
      best = k > best ? k : best;
    });
  }
  if (greedy) {
    atomicMax(&s_best, best);
    __syncthreads();
  } else {
    m = block_reduce(m, sred, MaxOp(), -INFINITY);
  }
  if (!greedy) {
    // 2) top-k threshold by 4-pass radix select on order-preserving keys
    float thr = -INFINITY;
    const int topk = a.top_k ? a.top_k[sr] : 0;
    if (topk > 0 && topk < V) {
      if (threadIdx.x == 0) {
        s_prefix = 0u;
        s_kleft = topk;
      }
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        const uint32_t mask_hi = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
        __syncthreads();
        const uint32_t pref = s_prefix;
        row_for_each(lg, V, [&](int, float x) {
          const uint32_t k = f2key(x);
          if ((k & mask_hi) == pref) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        });
        __syncthreads();
        if (threadIdx.x == 0) {
          int left = s_kleft;
          int bin = 255;
          for (; bin > 0; --bin) {
            const int c = static_cast<int>(hist[bin]);
            if (c >= left) break;
            left -= c;
          }
          s_kleft = left;
          s_prefix = pref | (static_cast<uint32_t>(bin) << shift);
        }
        __syncthreads();
      }
      thr = key2f(s_prefix);
    }
    const float minp = a.min_p ? a.min_p[sr] : 0.f;
    if (minp > 0.f) thr = fmaxf(thr, m + logf(minp));
    const float topp = a.top_p ? a.top_p[sr] : 1.f;
    // 3) candidates into shared memory (beyond 40 nats below the max a token's mass is < 5e-18
    //    of the max's: negligible for top-p, never drawn in fp32 Gumbel-max either)
    const float cthr = fmaxf(thr, m - 40.f);
    if (threadIdx.x == 0) s_ncand = 0;
    __syncthreads();
    row_for_each(lg, V, [&](int i, float x) {
      // warp-aggregated append: one shared-memory atomic per warp and element slot
      const bool keep = x >= cthr && x > -INFINITY;
      const unsigned act = __activemask();
      const unsigned bal = __ballot_sync(act, keep);
      if (bal == 0u) return;
      const int leader = __ffs(act) - 1;
      const int lane = threadIdx.x & 31;
      int base = 0;
      if (lane == leader) base = atomicAdd(&s_ncand, __popc(bal));
      base = __shfl_sync(act, base, leader);
      if (keep) {
        const int slot = base + __popc(bal & ((1u << lane) - 1u));
        if (slot < kSampleCand) {
          cand_x[slot] = x;
          cand_i[slot] = i;
        }
      }
    });
    __syncthreads();
    const int nc = s_ncand;
    const bool in_smem = nc <= kSampleCand;
    auto for_kept = [&](auto f) {   // every kept token (>= thr), from shared memory or the row
      if (in_smem) {
        for (int j = threadIdx.x; j < nc; j += blockDim.x)
          if (cand_x[j] >= thr) f(cand_i[j], cand_x[j]);
      } else {
        row_for_each(lg, V, [&](int i, float x) {
          if (x >= thr && x > -INFINITY) f(i, x);
        });
      }
    };
    // 4) top-p threshold: largest v with sum_{x >= v} e^(x-m) >= p * Z (bisection)
    if (topp < 1.f) {
      float z = 0.f;
      for_kept([&](int, float x) { z += __expf(x - m); });
      z = block_reduce(z, sred, SumOp(), 0.f);
      float lo = thr == -INFINITY ? m - 80.f : thr, hi = m;
      for (int it = 0; it < 24; ++it) {
        const float mid = 0.5f * (lo + hi);
        float sm = 0.f;
        for_kept([&](int, float x) {
          if (x >= mid) sm += __expf(x - m);
        });
        sm = block_reduce(sm, sred, SumOp(), 0.f);
        if (sm >= topp * z) lo = mid; else hi = mid;
      }
      thr = fmaxf(thr, lo);
    }
    // 5) Gumbel-max over the kept set
    const uint64_t seed = a.seeds ? static_cast<uint64_t>(a.seeds[sr]) : 0x1234ull;
    const uint64_t step = a.step ? static_cast<uint64_t>(a.step[sr]) : 0ull;
    best = 0ull;
    for_kept([&](int i, float x) {
      const float u = uniform01(seed + 0x9E37ull * step, static_cast<uint64_t>(i));
      const float gmb = -logf(-logf(u));
      const unsigned long long k = argmax_key(x + gmb, i);
      best = k > best ? k : best;
    });
    __syncthreads();
    if (threadIdx.x == 0) s_best = 0ull;
    __syncthreads();
    atomicMax(&s_best, best);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int tok = static_cast<int>(0xffffffffu - static_cast<uint32_t>(s_best & 0xffffffffull));
    if (s_best == 0ull) tok = 0;
    a.out_tokens[row] = tok;
    if (a.slot_tokens) a.slot_tokens[sr] = tok;
    if (a.step) a.step[sr] += 1;
    if (a.seen) a.seen[static_cast<int64_t>(sr) * a.seen_stride + tok] = 1;
  }
}

}  // namespace

cudaError_t qkv_rope_store(const RopeStoreArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  const int threads = 256;
  const bool vec_ok = (a.qkv_stride % 4) == 0 && (reinterpret_cast<uintptr_t>(a.qkv) & 7) == 0 &&
                      (a.k_cache == nullptr || (reinterpret_cast<uintptr_t>(a.k_cache) & 7) == 0) &&
                      (a.v_cache == nullptr || (reinterpret_cast<uintptr_t>(a.v_cache) & 7) == 0);
  if (a.head_dim == 128 && a.rot_dim % 8 == 0 && a.rot_dim <= 128 && vec_ok) {
    const int chunks = (a.hq + 2 * a.hkv + kRopeHeadsPerWarp - 1) / kRopeHeadsPerWarp;
    const long warps = static_cast<long>(a.tokens) * chunks;
    // 128-thread blocks: at 90 registers a thread, five resident blocks keep more rows in flight
    // per SM than two 256-thread blocks would
    qkv_rope_store_d128_kernel<<<(warps + 3) / 4, 128, 0, stream>>>(a);
    return cudaGetLastError();
  }
  const long warps = static_cast<long>(a.tokens) * (a.hq + 2 * a.hkv);
  const long grid = (warps + 7) / 8;
  switch (a.head_dim) {
    case 32: qkv_rope_store_kernel<32><<<grid, threads, 0, stream>>>(a); break;
    case 64: qkv_rope_store_kernel<64><<<grid, threads, 0, stream>>>(a); break;
    case 96: qkv_rope_store_kernel<96><<<grid, threads, 0, stream>>>(a); break;
    case 128: qkv_rope_store_kernel<128><<<grid, threads, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t moe_route(const MoeRouteArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  if (a.experts > 512 || a.topk > 16 || a.topk < 1) return cudaErrorInvalidValue;
  if (a.counts && !a.self_clean) {
    cudaMemsetAsync(a.counts, 0, sizeof(int) * a.experts, stream);
    cudaMemsetAsync(a.cursor, 0, sizeof(int) * a.experts, stream);
  }
  const int grid = (a.tokens + 7) / 8;
  const int per = (a.experts + 31) / 32;
  if (per <= 4) moe_topk_kernel<4><<<grid, 256, 0, stream>>>(a);
  else if (per <= 8) moe_topk_kernel<8><<<grid, 256, 0, stream>>>(a);
  else moe_topk_kernel<16><<<grid, 256, 0, stream>>>(a);
  if (a.counts) {
    int sgrid = (a.tokens * a.topk + 7) / 8;   // one warp per (token, k)
    if (sgrid > 148 * 8) sgrid = 148 * 8;
    moe_scatter_kernel<<<sgrid, 256, sizeof(int) * (a.experts + 1), stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t moe_combine(const MoeCombineArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  const int nvec = a.hidden / 8;
  if (a.hidden % 8 != 0 || a.topk > 16 || nvec > 256 * 4) return cudaErrorInvalidValue;
  if (a.residual != nullptr && (a.norm_w == nullptr || a.normed == nullptr)) return cudaErrorInvalidValue;
  if (nvec <= 256) moe_combine_kernel<1><<<a.tokens, 256, 0, stream>>>(a);
  else if (nvec <= 512) moe_combine_kernel<2><<<a.tokens, 256, 0, stream>>>(a);
  else moe_combine_kernel<4><<<a.tokens, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t vq_embed(const VqEmbedArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  if (a.hidden % 8 != 0 || a.ncb > 32 || a.ncb < 1) return cudaErrorInvalidValue;
  vq_embed_kernel<<<a.tokens, 128, 0, stream>>>(a);
  return cudaGetLastError();
}

namespace {
// One thread per (row, head, pair i): x_i, x_{i+half} -> rotated in fp32, stored as bf16.
__global__ void __launch_bounds__(256) rope_half_inplace_kernel(__nv_bfloat16* __restrict__ x, int64_t row_stride,
                                                                int rows, int heads, int head_stride, int half,
                                                                const float* __restrict__ cs,
                                                                const float* __restrict__ sn, int64_t cs_stride) {
  const int64_t total = static_cast<int64_t>(rows) * heads * half;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % half);
    const int64_t th = idx / half;
    const int h = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    __nv_bfloat16* p = x + t * row_stride + static_cast<int64_t>(h) * head_stride;
    const float a = __bfloat162float(p[i]), b = __bfloat162float(p[i + half]);
    const float* c = cs + t * cs_stride;
    const float* s = sn + t * cs_stride;
    p[i] = __float2bfloat16(a * c[i] - b * s[i]);
    p[i + half] = __float2bfloat16(b * c[i + half] + a * s[i + half]);
  }
}
// Two adjacent pairs per thread with 4-byte bf16x2 accesses (half, strides even, 4-byte base).
__global__ void __launch_bounds__(256) rope_half_inplace_x2_kernel(__nv_bfloat16* __restrict__ x, int64_t row_stride,
                                                                   int rows, int heads, int head_stride, int half,
                                                                   const float* __restrict__ cs,
                                                                   const float* __restrict__ sn, int64_t cs_stride) {
  const int q = half >> 1;   // pairs of pairs per head
  const int64_t total = static_cast<int64_t>(rows) * heads * q;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = 2 * static_cast<int>(idx % q);
    const int64_t th = idx / q;
    const int h = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    __nv_bfloat16* p = x + t * row_stride + static_cast<int64_t>(h) * head_stride;
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p + i));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p + i + half));
    const float2 c0 = *reinterpret_cast<const float2*>(cs + t * cs_stride + i);
    const float2 s0 = *reinterpret_cast<const float2*>(sn + t * cs_stride + i);
    const float2 c1 = *reinterpret_cast<const float2*>(cs + t * cs_stride + i + half);
    const float2 s1 = *reinterpret_cast<const float2*>(sn + t * cs_stride + i + half);
    *reinterpret_cast<__nv_bfloat162*>(p + i) = __floats2bfloat162_rn(a.x * c0.x - b.x * s0.x, a.y * c0.y - b.y * s0.y);
    *reinterpret_cast<__nv_bfloat162*>(p + i + half) =
        __floats2bfloat162_rn(b.x * c1.x + a.x * s1.x, b.y * c1.y + a.y * s1.y);
  }
}
}  // namespace

cudaError_t rope_half_inplace(void* x, int64_t row_stride, int rows, int heads, int head_stride, int rot,
                              const float* cos, const float* sin, int64_t cs_stride, cudaStream_t stream) {
  if (rows == 0 || heads == 0) return cudaSuccess;
  if (rot <= 0 || rot % 2 != 0 || rot > head_stride) return cudaErrorInvalidValue;
  const int half = rot / 2;
  if (half % 2 == 0 && row_stride % 2 == 0 && head_stride % 2 == 0 && cs_stride % 2 == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 3) == 0 && (reinterpret_cast<uintptr_t>(cos) & 7) == 0 &&
      (reinterpret_cast<uintptr_t>(sin) & 7) == 0) {
    const int64_t total = static_cast<int64_t>(rows) * heads * (half / 2);
    const int64_t grid = std::min<int64_t>((total + 255) / 256, 148 * 16);
    rope_half_inplace_x2_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<__nv_bfloat16*>(x), row_stride, rows, heads, head_stride, half, cos, sin, cs_stride);
    return cudaGetLastError();
  }
  const int64_t total = static_cast<int64_t>(rows) * heads * (rot / 2);
  const int64_t grid = std::min<int64_t>((total + 255) / 256, 148 * 16);
  rope_half_inplace_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(x), row_stride, rows, heads, head_stride, rot / 2, cos, sin, cs_stride);
  return cudaGetLastError();
}

cudaError_t embed(const EmbedArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  if (a.hidden % 8 != 0) return cudaErrorInvalidValue;
  embed_kernel<<<a.tokens, 128, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t sample(const SampleArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  sample_kernel<<<a.rows, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace omni
