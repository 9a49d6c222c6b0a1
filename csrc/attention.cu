// Paged GQA attention: prefill (causal or not, ragged, paged or contiguous
// K/V) and split-KV decode, plus the split combine.
//
// Grouped-query packing: the G = Hq / Hkv query heads that share one KV head
// are laid out as consecutive rows of the query tile, so a K/V tile staged in
// shared memory once serves all G heads (decode: one token x G heads per warp;
// prefill: 64 rows = (64 / G) tokens x G heads per CTA).
//
// KV cache layout (one layer): [pages, Hkv, 64, D] bf16, page size 64, so a
// 64-key tile of one KV head is a single contiguous block.
//
// Reference counterparts: RadixAttention backends used by
// sglang_omni/models/qwen3_omni/thinker.py:236-243 (FlashInfer / FA3) and the
// HF encoders' SDPA (audio / vision, non-causal varlen).
#include <cuda_bf16.h>
#include <stdint.h>

#include "host_util.h"
#include "omni_kernels.h"
#include "pdl.cuh"

namespace omni {
namespace {

constexpr int kPage = 64;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t ld_u32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Shared-memory K/V tile: 64 rows of D bf16, padded to D + 8 elements so that
// ldmatrix row groups fall in distinct banks.
template <int D>
struct Tile {
  static constexpr int kStride = D + 8;
  static constexpr int kElems = kPage * kStride;
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
};

// Loads a 64 x D tile (rows valid < nvalid are copied, the rest zero-filled)
// with all 128 threads.  `src_row(r)` returns the global address of row r.
template <int D, class RowFn>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, RowFn src_row, int nvalid) {
  using T = Tile<D>;
  for (int i = threadIdx.x; i < kPage * T::kChunks; i += blockDim.x) {
    const int r = i / T::kChunks;
    const int c = i - r * T::kChunks;
    const bool valid = r < nvalid;
    const __nv_bfloat16* src = src_row(valid ? r : 0) + c * 8;
    cp_async16(smem_addr(dst + r * T::kStride + c * 8), src, valid);
  }
}

// ---------------------------------------------------------------------------
// Prefill / varlen attention.  One CTA = 64 packed rows of one KV head.
// ---------------------------------------------------------------------------
// A block-table entry outside the cache reads the reserved padding page 0.
__device__ __forceinline__ int checked_page(int page, int num_pages) {
  return (num_pages > 0 && static_cast<unsigned>(page) >= static_cast<unsigned>(num_pages)) ? 0 : page;
}

// A decode request sees at most the keys its block-table row can name
// (bt_stride pages of 64): a longer kv_len would read past the row.
__device__ __forceinline__ int decode_kv_len(const int* kv_lens, int b, int bt_stride) {
  const int n = kv_lens[b];
  const int cap = bt_stride > 0 ? bt_stride * 64 : n;
  return n < cap ? n : cap;
}

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_stride;  // elements between tokens
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t kv_stride;  // contiguous mode: elements between tokens
  const int* block_table;  // paged mode (nullptr => contiguous)
  int bt_stride;
  const int* cu_q;     // [B+1]
  const int* kv_lens;  // [B] keys visible to the request (incl. this chunk)
  const int* cu_kv;    // contiguous mode: [B+1] key row offsets
  const int* tile_req;
  const int* tile_tok0;
  int hq, hkv;
  float scale_log2;
  int causal;
  __nv_bfloat16* out;
  int64_t out_stride;
  int window;
  int num_pages;
};

template <int D>
__global__ void __launch_bounds__(128) prefill_kernel(const PrefillParams p) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  using T = Tile<D>;
  constexpr int KS = D / 16;  // k-steps over head dim
  constexpr int NJ = D / 8;   // output n-tiles
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [2][64][stride]
  __nv_bfloat16* sv = sk + 2 * T::kElems;

  const int tile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = p.tile_req[tile];
  const int tok0 = p.tile_tok0[tile];
  const int G = p.hq / p.hkv;
  const int q_begin = p.cu_q[b];
  const int q_len = p.cu_q[b + 1] - q_begin;
  const int kv_len = p.kv_lens[b];
  const int pos_base = kv_len - q_len;  // absolute position of query token 0
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tokens_per_tile = 64 / G;

  // rows handled by this thread: r0 = 16*warp + g, r1 = r0 + 8
  const int r0 = 16 * warp + g, r1 = r0 + 8;
  const int tokA = tok0 + r0 / G, tokB = tok0 + r1 / G;
  const int headA = h * G + r0 % G, headB = h * G + r1 % G;
  const bool validA = tokA < q_len, validB = tokB < q_len;
  const int posA = pos_base + tokA, posB = pos_base + tokB;

  // Q fragments
  uint32_t qa[KS][4];
  {
    const __nv_bfloat16* qA = p.q + static_cast<int64_t>(q_begin + (validA ? tokA : 0)) * p.q_stride + headA * D;
    const __nv_bfloat16* qB = p.q + static_cast<int64_t>(q_begin + (validB ? tokB : 0)) * p.q_stride + headB * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = validA ? ld_u32(qA + 16 * ks + 2 * t) : 0u;
      qa[ks][1] = validB ? ld_u32(qB + 16 * ks + 2 * t) : 0u;
      qa[ks][2] = validA ? ld_u32(qA + 16 * ks + 2 * t + 8) : 0u;
      qa[ks][3] = validB ? ld_u32(qB + 16 * ks + 2 * t + 8) : 0u;
    }
  }

  // Key range of the tile.
  const int last_tok = min(q_len, tok0 + tokens_per_tile) - 1;
  const int key_end = p.causal ? min(kv_len, pos_base + last_tok + 1) : kv_len;
  const int ntiles = (key_end + kPage - 1) / kPage;
  // sliding window: keys below (first query pos - window + 1) are never visible
  const int first_tile = p.window > 0 ? max(0, pos_base + tok0 - p.window + 1) / kPage : 0;

  float o[NJ][4];
#pragma unroll
  for (int j = 0; j < NJ; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  const int64_t kv_base = p.block_table ? 0 : static_cast<int64_t>(p.cu_kv[b]);
  auto issue = [&](int it, int buf) {
    const int k0 = it * kPage;
    const int nvalid = min(kPage, kv_len - k0);
    if (p.block_table) {
      const int page = checked_page(p.block_table[static_cast<int64_t>(b) * p.bt_stride + it], p.num_pages);
      const int64_t base = (static_cast<int64_t>(page) * p.hkv + h) * kPage * D;
      load_tile<D>(sk + buf * T::kElems, [&](int r) { return p.k + base + static_cast<int64_t>(r) * D; }, nvalid);
      load_tile<D>(sv + buf * T::kElems, [&](int r) { return p.v + base + static_cast<int64_t>(r) * D; }, nvalid);
    } else {
      load_tile<D>(sk + buf * T::kElems,
                   [&](int r) { return p.k + (kv_base + k0 + r) * p.kv_stride + static_cast<int64_t>(h) * D; },
                   nvalid);
      load_tile<D>(sv + buf * T::kElems,
                   [&](int r) { return p.v + (kv_base + k0 + r) * p.kv_stride + static_cast<int64_t>(h) * D; },
                   nvalid);
    }
    cp_async_commit();
  };

  if (ntiles > first_tile) issue(first_tile, first_tile & 1);
  for (int it = first_tile; it < ntiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < ntiles) {
      issue(it + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* kt = sk + buf * T::kElems;
    const __nv_bfloat16* vt = sv + buf * T::kElems;
    const int k0 = it * kPage;

    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int row = np * 16 + (mi >> 1) * 8 + rr;
        const int col = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_addr(kt + row * T::kStride + col), b0, b1, b2, b3);
        mma16816(s[2 * np], qa[ks], b0, b1);
        mma16816(s[2 * np + 1], qa[ks], b2, b3);
      }
    }
    // scale + mask + online softmax
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + n * 8 + 2 * t + e;
        const bool okA = validA && key < kv_len && (!p.causal || key <= posA) &&
                         (p.window <= 0 || key > posA - p.window);
        const bool okB = validB && key < kv_len && (!p.causal || key <= posB) &&
                         (p.window <= 0 || key > posB - p.window);
        s[n][e] = okA ? s[n][e] * p.scale_log2 : -INFINITY;
        s[n][2 + e] = okB ? s[n][2 + e] * p.scale_log2 : -INFINITY;
        mxA = fmaxf(mxA, s[n][e]);
        mxB = fmaxf(mxB, s[n][2 + e]);
      }
    }
#pragma unroll
    for (int d = 1; d < 4; d <<= 1) {
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, d));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, d));
    }
    const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
    const float subA = mnA == -INFINITY ? 0.f : mnA;
    const float subB = mnB == -INFINITY ? 0.f : mnB;
    const float corrA = exp2f(mA - subA), corrB = exp2f(mB - subB);
    mA = mnA;
    mB = mnB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = exp2f(s[n][e] - subA);
        s[n][2 + e] = exp2f(s[n][2 + e] - subB);
        sumA += s[n][e];
        sumB += s[n][2 + e];
      }
    }
    lA = lA * corrA + sumA;
    lB = lB * corrB + sumB;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      o[j][0] *= corrA;
      o[j][1] *= corrA;
      o[j][2] *= corrB;
      o[j][3] *= corrB;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dj = 0; dj < NJ / 2; ++dj) {
        const int row = kk * 16 + (mi & 1) * 8 + rr;
        const int col = dj * 16 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_addr(vt + row * T::kStride + col), b0, b1, b2, b3);
        mma16816(o[2 * dj], pa, b0, b1);
        mma16816(o[2 * dj + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  // finalise: quad-sum of l, normalise, store
#pragma unroll
  for (int d = 1; d < 4; d <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, d);
    lB += __shfl_xor_sync(0xffffffffu, lB, d);
  }
  const float invA = lA > 0.f ? 1.f / lA : 0.f;
  const float invB = lB > 0.f ? 1.f / lB : 0.f;
  __nv_bfloat16* oA = p.out + static_cast<int64_t>(q_begin + tokA) * p.out_stride + headA * D;
  __nv_bfloat16* oB = p.out + static_cast<int64_t>(q_begin + tokB) * p.out_stride + headB * D;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    if (validA) *reinterpret_cast<uint32_t*>(oA + 8 * j + 2 * t) = pack_bf16(o[j][0] * invA, o[j][1] * invA);
    if (validB) *reinterpret_cast<uint32_t*>(oB + 8 * j + 2 * t) = pack_bf16(o[j][2] * invB, o[j][3] * invB);
  }
}

// ---------------------------------------------------------------------------
// Split-KV decode: grid (splits, Hkv, B); the G heads of a KV head are the rows
// of one 16-row MMA tile; each warp takes 16 keys of every 64-key tile.
// ---------------------------------------------------------------------------
// Keys per split for one request: the configured split size, widened (in
// whole pages) when the context would need more than max_splits splits, so a
// request never writes or reads partials past its max_splits slots.
__device__ __forceinline__ int split_keys(int kv_len, int keys_per_split, int max_splits) {
  const int need = (kv_len + max_splits - 1) / max_splits;
  const int need_pages = (need + kPage - 1) / kPage * kPage;
  return need_pages > keys_per_split ? need_pages : keys_per_split;
}

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const int* block_table;
  int bt_stride;
  const int* kv_lens;
  int hq, hkv;
  float scale_log2;
  int keys_per_split;
  int max_splits;
  __nv_bfloat16* out;
  int64_t out_stride;
  float* part_o;    // [B, Hq, max_splits, D]
  float* part_lse;  // [B, Hq, max_splits]
  int num_pages;
  int* counters;    // [B, Hkv] zeros: split arrivals (nullptr: separate combine launch)
};


template <int D>
__global__ void __launch_bounds__(128) decode_kernel(const DecodeParams p) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  using T = Tile<D>;
  constexpr int KS = D / 16;
  constexpr int NJ = D / 8;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sv = sk + 2 * T::kElems;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = p.hq / p.hkv;
  const int kv_len = decode_kv_len(p.kv_lens, b, p.bt_stride);
  const int kps = split_keys(kv_len, p.keys_per_split, p.max_splits);
  const int k_begin = split * kps;
  if (kv_len <= 0) {
    // empty context (a padding row of a batch bucket): defined zero output, so
    // later layers never see uninitialised memory
    if (split == 0) {
      for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        p.out[static_cast<int64_t>(b) * p.out_stride + (h * G) * D + i] = __float2bfloat16(0.f);
    }
    return;
  }
  if (k_begin >= kv_len) return;
  const int k_end = min(kv_len, k_begin + kps);
  const int nsplit = (kv_len + kps - 1) / kps;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool validA = g < G, validB = g + 8 < G;

  uint32_t qa[KS][4];
  {
    const __nv_bfloat16* qA = p.q + static_cast<int64_t>(b) * p.q_stride + (h * G + (validA ? g : 0)) * D;
    const __nv_bfloat16* qB = p.q + static_cast<int64_t>(b) * p.q_stride + (h * G + (validB ? g + 8 : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = validA ? ld_u32(qA + 16 * ks + 2 * t) : 0u;
      qa[ks][1] = validB ? ld_u32(qB + 16 * ks + 2 * t) : 0u;
      qa[ks][2] = validA ? ld_u32(qA + 16 * ks + 2 * t + 8) : 0u;
      qa[ks][3] = validB ? ld_u32(qB + 16 * ks + 2 * t + 8) : 0u;
    }
  }
  float o[NJ][4];
#pragma unroll
  for (int j = 0; j < NJ; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  const int first_tile = k_begin / kPage;
  const int ntiles = (k_end - k_begin + kPage - 1) / kPage;
  auto issue = [&](int i, int buf) {
    const int it = first_tile + i;
    const int nvalid = min(kPage, k_end - it * kPage);
    const int page = checked_page(p.block_table[static_cast<int64_t>(b) * p.bt_stride + it], p.num_pages);
    const int64_t base = (static_cast<int64_t>(page) * p.hkv + h) * kPage * D;
    load_tile<D>(sk + buf * T::kElems, [&](int r) { return p.k + base + static_cast<int64_t>(r) * D; }, nvalid);
    load_tile<D>(sv + buf * T::kElems, [&](int r) { return p.v + base + static_cast<int64_t>(r) * D; }, nvalid);
    cp_async_commit();
  };
  issue(0, 0);
  const int mi = lane >> 3, rr = lane & 7;
  for (int i = 0; i < ntiles; ++i) {
    const int buf = i & 1;
    if (i + 1 < ntiles) {
      issue(i + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* kt = sk + buf * T::kElems + warp * 16 * T::kStride;
    const __nv_bfloat16* vt = sv + buf * T::kElems + warp * 16 * T::kStride;
    const int kw = (first_tile + i) * kPage + warp * 16;  // first key of this warp
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int row = (mi >> 1) * 8 + rr;
      const int col = ks * 16 + (mi & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_addr(kt + row * T::kStride + col), b0, b1, b2, b3);
      mma16816(s[0], qa[ks], b0, b1);
      mma16816(s[1], qa[ks], b2, b3);
    }
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kw + n * 8 + 2 * t + e;
        const bool ok = key < k_end;
        s[n][e] = (ok && validA) ? s[n][e] * p.scale_log2 : -INFINITY;
        s[n][2 + e] = (ok && validB) ? s[n][2 + e] * p.scale_log2 : -INFINITY;
        mxA = fmaxf(mxA, s[n][e]);
        mxB = fmaxf(mxB, s[n][2 + e]);
      }
    }
#pragma unroll
    for (int d = 1; d < 4; d <<= 1) {
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, d));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, d));
    }
    const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
    const float subA = mnA == -INFINITY ? 0.f : mnA;
    const float subB = mnB == -INFINITY ? 0.f : mnB;
    const float corrA = exp2f(mA - subA), corrB = exp2f(mB - subB);
    mA = mnA;
    mB = mnB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = exp2f(s[n][e] - subA);
        s[n][2 + e] = exp2f(s[n][2 + e] - subB);
        sumA += s[n][e];
        sumB += s[n][2 + e];
      }
    }
    lA = lA * corrA + sumA;
    lB = lB * corrB + sumB;
    uint32_t pa[4];
    pa[0] = pack_bf16(s[0][0], s[0][1]);
    pa[1] = pack_bf16(s[0][2], s[0][3]);
    pa[2] = pack_bf16(s[1][0], s[1][1]);
    pa[3] = pack_bf16(s[1][2], s[1][3]);
#pragma unroll
    for (int dj = 0; dj < NJ / 2; ++dj) {
      o[2 * dj][0] *= corrA;
      o[2 * dj][1] *= corrA;
      o[2 * dj][2] *= corrB;
      o[2 * dj][3] *= corrB;
      o[2 * dj + 1][0] *= corrA;
      o[2 * dj + 1][1] *= corrA;
      o[2 * dj + 1][2] *= corrB;
      o[2 * dj + 1][3] *= corrB;
      const int row = (mi & 1) * 8 + rr;
      const int col = dj * 16 + (mi >> 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_addr(vt + row * T::kStride + col), b0, b1, b2, b3);
      mma16816(o[2 * dj], pa, b0, b1);
      mma16816(o[2 * dj + 1], pa, b2, b3);
    }
    __syncthreads();
  }
#pragma unroll
  for (int d = 1; d < 4; d <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, d);
    lB += __shfl_xor_sync(0xffffffffu, lB, d);
  }
  // Cross-warp merge through shared memory (reuses the K/V buffers).
  float* red_o = reinterpret_cast<float*>(smem_raw);            // [4][16][D]
  float* red_ml = red_o + 4 * 16 * D;                           // [4][16][2]
  if (t == 0) {
    red_ml[(warp * 16 + g) * 2 + 0] = mA;
    red_ml[(warp * 16 + g) * 2 + 1] = lA;
    red_ml[(warp * 16 + g + 8) * 2 + 0] = mB;
    red_ml[(warp * 16 + g + 8) * 2 + 1] = lB;
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    red_o[(warp * 16 + g) * D + 8 * j + 2 * t] = o[j][0];
    red_o[(warp * 16 + g) * D + 8 * j + 2 * t + 1] = o[j][1];
    red_o[(warp * 16 + g + 8) * D + 8 * j + 2 * t] = o[j][2];
    red_o[(warp * 16 + g + 8) * D + 8 * j + 2 * t + 1] = o[j][3];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int r = idx / D, d = idx - r * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_ml[(w * 16 + r) * 2]);
    const float sub = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(red_ml[(w * 16 + r) * 2] - sub);
      L += red_ml[(w * 16 + r) * 2 + 1] * f;
      acc += red_o[(w * 16 + r) * D + d] * f;
    }
    const float val = L > 0.f ? acc / L : 0.f;
    const int head = h * G + r;
    if (nsplit == 1) {
      p.out[static_cast<int64_t>(b) * p.out_stride + head * D + d] = __float2bfloat16(val);
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * p.hq + head) * p.max_splits + split;
      p.part_o[slot * D + d] = val;
      if (d == 0) p.part_lse[slot] = L > 0.f ? sub + log2f(L) : -INFINITY;
    }
  }
  if (nsplit == 1 || p.counters == nullptr) return;
  // The last split of (request, KV head) to finish merges all splits: no second launch.
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* c = p.counters + static_cast<int64_t>(b) * p.hkv + h;
    const int done = atomicAdd(c, 1) + 1;
    s_last = done == nsplit;
    if (s_last) *c = 0;  // ready for the next launch (graph replays reuse the counters)
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Merge weights per (head, split) in shared memory (the K/V buffers are free now):
  // w[r][sp] = 2^(lse - max) / sum, so the output is a plain weighted sum of partials.
  float* wsm = reinterpret_cast<float*>(smem_raw);  // [G][nsplit]
  const int64_t slot_h = (static_cast<int64_t>(b) * p.hq + h * G) * p.max_splits;
  for (int i = threadIdx.x; i < G * nsplit; i += blockDim.x) {
    const int r = i / nsplit, sp = i - r * nsplit;
    wsm[i] = __ldcg(p.part_lse + slot_h + static_cast<int64_t>(r) * p.max_splits + sp);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float* w = wsm + threadIdx.x * nsplit;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, w[sp]);
    const float sub = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      w[sp] = exp2f(w[sp] - sub);
      L += w[sp];
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int sp = 0; sp < nsplit; ++sp) w[sp] *= inv;
  }
  __syncthreads();
  // 16-byte partial loads, four splits per round per item
  constexpr int V = D / 4;
  for (int it = threadIdx.x; it < G * V; it += blockDim.x) {
    const int r = it / V, d4 = it - r * V;
    const float4* src = reinterpret_cast<const float4*>(p.part_o + (slot_h + static_cast<int64_t>(r) * p.max_splits) * D) + d4;
    const float* w = wsm + r * nsplit;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int sp = 0;
    for (; sp + 4 <= nsplit; sp += 4) {
      float4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = __ldcg(src + static_cast<int64_t>(sp + u) * V);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float wu = w[sp + u];
        acc.x += wu * x[u].x;
        acc.y += wu * x[u].y;
        acc.z += wu * x[u].z;
        acc.w += wu * x[u].w;
      }
    }
    for (; sp < nsplit; ++sp) {
      const float4 x = __ldcg(src + static_cast<int64_t>(sp) * V);
      const float wu = w[sp];
      acc.x += wu * x.x;
      acc.y += wu * x.y;
      acc.z += wu * x.z;
      acc.w += wu * x.w;
    }
    __nv_bfloat16* o = p.out + static_cast<int64_t>(b) * p.out_stride + (h * G + r) * D + 4 * d4;
    *reinterpret_cast<uint32_t*>(o) = pack_bf16(acc.x, acc.y);
    *reinterpret_cast<uint32_t*>(o + 2) = pack_bf16(acc.z, acc.w);
  }
}

template <int D>
__global__ void decode_combine_kernel(const DecodeParams p) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  const int head = blockIdx.x, b = blockIdx.y;
  const int kv_len = decode_kv_len(p.kv_lens, b, p.bt_stride);
  const int kps = split_keys(kv_len, p.keys_per_split, p.max_splits);
  const int nsplit = (kv_len + kps - 1) / kps;
  if (nsplit <= 1) return;
  const int64_t slot0 = (static_cast<int64_t>(b) * p.hq + head) * p.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, p.part_lse[slot0 + s]);
  const float sub = M == -INFINITY ? 0.f : M;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float f = exp2f(p.part_lse[slot0 + s] - sub);
      L += f;
      acc += f * p.part_o[(slot0 + s) * D + d];
    }
    p.out[static_cast<int64_t>(b) * p.out_stride + head * D + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

template <int D>
cudaError_t launch_prefill(const PrefillParams& p, int num_tiles, cudaStream_t stream) {
  const int smem = 4 * Tile<D>::kElems * 2;
  cudaError_t e = ensure_smem_attr<prefill_kernel<D>>(smem);
  if (e != cudaSuccess) return e;
  dim3 grid(num_tiles, p.hkv);
  prefill_kernel<D><<<grid, 128, smem, stream>>>(p);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_decode(const DecodeParams& p, int batch, cudaStream_t stream) {
  const int tiles = 4 * Tile<D>::kElems * 2;
  const int red = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;
  const int smem = tiles > red ? tiles : red;
  cudaError_t e = ensure_smem_attr<decode_kernel<D>>(smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.max_splits, p.hkv, batch);
  decode_kernel<D><<<grid, 128, smem, stream>>>(p);
  if (p.max_splits > 1 && p.counters == nullptr) {
    dim3 g2(p.hq, batch);
    decode_combine_kernel<D><<<g2, D, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_prefill(const AttnPrefillArgs& a, cudaStream_t stream) {
  if (a.num_tiles == 0) return cudaSuccess;
  if (a.tile_rows == 128 || a.tile_rows == 256) return attention_prefill_sm100(a, stream);
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0 || 64 % (a.hq / a.hkv) != 0) return cudaErrorInvalidValue;
  PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_stride = a.q_stride;
  p.k = static_cast<const __nv_bfloat16*>(a.k);
  p.v = static_cast<const __nv_bfloat16*>(a.v);
  p.kv_stride = a.kv_stride;
  p.block_table = a.block_table;
  p.bt_stride = a.bt_stride;
  p.cu_q = a.cu_q;
  p.kv_lens = a.kv_lens;
  p.cu_kv = a.cu_kv;
  p.tile_req = a.tile_req;
  p.tile_tok0 = a.tile_tok0;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.scale_log2 = a.scale * kLog2e;
  p.causal = a.causal;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.window = a.window;
  p.num_pages = a.num_pages;
  switch (a.head_dim) {
    case 64: return launch_prefill<64>(p, a.num_tiles, stream);
    case 80: return launch_prefill<80>(p, a.num_tiles, stream);
    case 96: return launch_prefill<96>(p, a.num_tiles, stream);
    case 128: return launch_prefill<128>(p, a.num_tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream) {
  if (a.batch == 0) return cudaSuccess;
  if (a.batch < 0 || a.hq <= 0 || a.hkv <= 0 || a.max_splits < 1) return cudaErrorInvalidValue;
  if (a.hq % a.hkv != 0 || a.hq / a.hkv > 16 || a.keys_per_split <= 0 || a.keys_per_split % kPage != 0)
    return cudaErrorInvalidValue;
  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_stride = a.q_stride;
  p.k = static_cast<const __nv_bfloat16*>(a.k);
  p.v = static_cast<const __nv_bfloat16*>(a.v);
  p.block_table = a.block_table;
  p.bt_stride = a.bt_stride;
  p.kv_lens = a.kv_lens;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.scale_log2 = a.scale * kLog2e;
  p.keys_per_split = a.keys_per_split;
  p.max_splits = a.max_splits;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.part_o = a.part_o;
  p.part_lse = a.part_lse;
  p.num_pages = a.num_pages;
  p.counters = a.counters;
  switch (a.head_dim) {
    case 64: return launch_decode<64>(p, a.batch, stream);
    case 128: return launch_decode<128>(p, a.batch, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace omni

// ===========================================================================
// Allocation-free decode attention (C ABI).  See omni_noalloc.h.
// ===========================================================================
#include <cstdio>
#include <mutex>

#include "omni_noalloc.h"

namespace {

// Split-KV scratch of the allocation-free entry point: partial outputs
// followed by partial log-sum-exps.  It lives in the module's static device
// memory, so every GPU that loads this library holds these 16.25 MiB until the
// process exits.  In host code `g_noalloc_decode_scratch` names a host-side
// stand-in, not the device array: its device address comes from
// cudaGetSymbolAddress below.
constexpr long long kNoAllocPartFloats = OMNI_NOALLOC_DECODE_PART_FLOATS;
constexpr long long kNoAllocLseFloats = OMNI_NOALLOC_DECODE_LSE_FLOATS;
static __device__ __align__(256) float g_noalloc_decode_scratch[kNoAllocPartFloats + kNoAllocLseFloats];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of the scratch array on the current device.  It is resolved
// with that device current and kept only once the lookup succeeded: a lookup
// that failed (for example because another library was capturing a stream at
// that moment) is retried on the next call instead of being remembered.
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_decode_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();  // the failed lookup must not be reported by the caller's next CUDA call
      return e;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int omni_attention_decode_noalloc(
    const void* q, long long q_stride, const void* k_cache, const void* v_cache, const int* block_table,
    int bt_stride, const int* kv_lens, int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
    int keys_per_split, int max_splits, int num_pages, void* out, long long out_stride, void* stream) {
  // Shapes first, before any division by them.
  const bool bad = batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 ||
                   num_heads / num_kv_heads > 16 || (head_dim != 64 && head_dim != 128) || keys_per_split <= 0 ||
                   keys_per_split % 64 != 0 || max_splits < 1 || num_pages < 1 || bt_stride < 0 ||
                   q_stride < static_cast<long long>(num_heads) * head_dim ||
                   out_stride < static_cast<long long>(num_heads) * head_dim;
  if (bad) {
    std::fprintf(stderr,
                 "omni_attention_decode_noalloc: invalid arguments (batch %d, heads %d / %d, head_dim %d, "
                 "keys_per_split %d, max_splits %d, num_pages %d, strides q %lld out %lld block table %d)\n",
                 batch, num_heads, num_kv_heads, head_dim, keys_per_split, max_splits, num_pages, q_stride, out_stride,
                 bt_stride);
    return OMNI_NOALLOC_ERR_INVALID;
  }
  if (batch > 0 && (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
                    kv_lens == nullptr || out == nullptr)) {
    std::fprintf(stderr, "omni_attention_decode_noalloc: null input or output pointer\n");
    return OMNI_NOALLOC_ERR_INVALID;
  }
  const long long slots = static_cast<long long>(batch) * num_heads * max_splits;
  if (slots * head_dim > kNoAllocPartFloats || slots > kNoAllocLseFloats) {
    std::fprintf(stderr,
                 "omni_attention_decode_noalloc: batch %d x heads %d x splits %d x head_dim %d needs %lld partial "
                 "floats and %lld LSE floats; the static scratch holds %lld and %lld\n",
                 batch, num_heads, max_splits, head_dim, slots * head_dim, slots, kNoAllocPartFloats,
                 kNoAllocLseFloats);
    return OMNI_NOALLOC_ERR_TOO_LARGE;
  }
  if (batch == 0) return 0;
  float* scratch = nullptr;
  cudaError_t e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  omni::AttnDecodeArgs a{};
  a.q = q;
  a.q_stride = q_stride;
  a.k = k_cache;
  a.v = v_cache;
  a.block_table = block_table;
  a.bt_stride = bt_stride;
  a.kv_lens = kv_lens;
  a.batch = batch;
  a.hq = num_heads;
  a.hkv = num_kv_heads;
  a.head_dim = head_dim;
  a.scale = scale;
  a.keys_per_split = keys_per_split;
  a.max_splits = max_splits;
  a.out = out;
  a.out_stride = out_stride;
  a.part_o = scratch;
  a.part_lse = scratch + kNoAllocPartFloats;
  a.num_pages = num_pages;  // block-table entries outside [0, num_pages) read page 0
  return static_cast<int>(omni::attention_decode(a, static_cast<cudaStream_t>(stream)));
}
