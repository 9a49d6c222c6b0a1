// Persistent tcgen05 GEMM for every projection of the serving path: dense
// linear layers, the MoE grouped expert GEMMs (w13 with SiLU*up fused, w2),
// the LM head (fp32 logits) and the encoders' linear layers (bias + GELU).
//
// Layout choice ("weights as A"): the weight matrix feeds the M=128 side of the
// UMMA and the token rows feed N (16..256).  Decode batches therefore keep the
// tensor core's M dimension full, and one kernel covers decode (few tokens per
// expert) and prefill (thousands of tokens) by picking the token tile BN.
//
// Warp roles (6 warps, one CTA per SM, persistent over tiles):
//   warp 0     TMA producer (one elected lane), 128B-swizzled K-major tiles
//   warp 1     TMEM allocator + MMA issuer (one elected lane)
//   warps 2-5  epilogue: tcgen05.ld -> activation/bias/residual -> global store
// Accumulators are double buffered in TMEM so the epilogue of tile i overlaps
// the MMAs of tile i+1.
//
// Launched as a programmatic dependent launch: the prologue (barriers, TMEM,
// tensor-map prefetch) and, for dense GEMMs, the first stages' weight tiles run
// while the previous kernel of the stream finishes; every read of activations,
// group offsets or residuals and every store comes after grid_dep_wait().
//
// Reference counterparts: SGLang QKVParallelLinear / RowParallelLinear /
// FusedMoE as used by sglang_omni/models/qwen3_omni/thinker.py:192-213,402-412
// and the talker's native MoE (sglang_omni/models/qwen3_omni/talker.py:242-247).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "host_util.h"
#include "omni_kernels.h"
#include "sm100.cuh"

namespace omni {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 512;

struct DevParams {
  void* out;
  int64_t ldo;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int64_t ldr;
  const int* offsets;
  int rows;
  int m_out;
  int a_rows;
  int k;
  int groups;
  int m_tiles;           // weight tiles of the output (dense GEMMs)
  int mt_fast;           // 1: tile order walks the weight tiles fastest (large token operand)
  int out_f32;
  int act;
  int* status;
  int k_splits;          // > 1: split-K over K blocks with an fp32 workspace
  float* ws;             // [splits][tiles][BN][128] fp32 partial sums (each split owns its plane;
                         // token-major inside a tile, so stores and the finaliser's reads coalesce)
  int vec4;              // outputs / bias / residual allow 4-wide vector access (split-K finaliser)
  int pdl_prefetch_a;    // programmatic dependent launch with static weights: prefetch them before the wait
  int cluster_splitk;    // split-K over a thread-block cluster: partials stay in shared memory (DSMEM reduce)
  int vec8;              // outputs / residual rows allow 16-byte vectors of 8 (staged epilogue)
  int* counters;         // [tiles] arrival counters, zero between calls
  const unsigned long long* peer_out;  // owner scatter: row r -> peer_out[r / rows_per] + r * ldo
  int rows_per;
  const unsigned int* wait_flags;      // wait before the first load: wait_flags[i] == *wait_seq
  const unsigned int* wait_seq;
  int wait_count;
  long long wait_timeout_ns;
  // expert-parallel fused modes (see GemmArgs)
  int seg_cap;                         // > 0: group g = rows [g * seg_cap, + seg_counts[g])
  const int* seg_counts;
  int* seg_counts_copy;
  int setup_wait;                      // the flags are awaited before the counts are read
  const int* row_tag;                  // combine epilogue: row r -> peer_rows[tag.x] + tag.y * ldo
  const unsigned long long* peer_rows;
  int tag_ranks, tag_slots;
  const unsigned long long* signal_flags;  // completion: last CTA release-stores *signal_seq there
  const unsigned int* signal_seq;
  int signal_count;
  int* arrive_counter;
  int* zero_ptr;
  int zero_n;
};

// Bounded wait until every flags[i] (i < count) has reached *seq (wrap-safe compare); lane i
// of the calling warp waits on flags i, i + 32, ...  Returns false after a timeout (status 2).
__device__ __forceinline__ bool wait_flags_warp(const unsigned int* flags, const unsigned int* seq, int count,
                                                long long timeout_ns, int* status, int lane) {
  const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(seq);
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  for (int i = lane; i < count && ok; i += 32) {
    uint32_t v;
    while (true) {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if (static_cast<int>(v - target) >= 0) break;
      if (globaltimer_ns() - t0 > static_cast<uint64_t>(timeout_ns)) {
        record_status(status, kStatusPeerTimeout);
        ok = false;
        break;
      }
    }
  }
  __syncwarp();
  __threadfence_system();  // the other lanes' later reads follow every lane's acquire
  return __all_sync(0xffffffffu, ok);
}

// Destination of bf16 output row `row`, or nullptr when a combine tag drops it.
__device__ __forceinline__ __nv_bfloat16* out_row_bf16(const DevParams& p, int row) {
  if (p.row_tag != nullptr) {
    const int2 t = reinterpret_cast<const int2*>(p.row_tag)[row];
    if (static_cast<unsigned>(t.x) >= static_cast<unsigned>(p.tag_ranks) ||
        static_cast<unsigned>(t.y) >= static_cast<unsigned>(p.tag_slots))
      return nullptr;
    return reinterpret_cast<__nv_bfloat16*>(p.peer_rows[t.x]) + static_cast<int64_t>(t.y) * p.ldo;
  }
  if (p.peer_out != nullptr)
    return reinterpret_cast<__nv_bfloat16*>(p.peer_out[row / p.rows_per]) + static_cast<int64_t>(row) * p.ldo;
  return static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo;
}

// The activations live out of line: inlined into every unrolled epilogue store
// they made the kernel's code large enough that instruction fetch, not memory,
// bounded the small decode GEMMs.
__device__ __noinline__ float act_apply(float v, int act) {
  if (act == kActGeluTanh) return gelu_tanh_f(v);
  if (act == kActGeluErf) return gelu_erf_f(v);
  if (act == kActSilu) return silu_f(v);
  return v;
}

__device__ __forceinline__ float epilogue_act(float v, int act) { return act == kActNone ? v : act_apply(v, act); }

// Split-K finaliser store of four consecutive outputs (m .. m+3) of one token row:
// bias, activation, residual, bf16 / fp32 store (8 / 16-byte vectors when p.vec4).
__device__ __noinline__ void store_out4(const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ residual,
                                        int64_t ldr, void* out_row, int out_f32, int act, int m, int m_out, int vec4,
                                        int64_t row, float4 v4) {
  float v[4] = {v4.x, v4.y, v4.z, v4.w};
  if (vec4 && m + 3 < m_out) {
    if (bias != nullptr) {
      const uint2 b = *reinterpret_cast<const uint2*>(bias + m);
      const __nv_bfloat162 b01 = *reinterpret_cast<const __nv_bfloat162*>(&b.x);
      const __nv_bfloat162 b23 = *reinterpret_cast<const __nv_bfloat162*>(&b.y);
      v[0] += __low2float(b01); v[1] += __high2float(b01); v[2] += __low2float(b23); v[3] += __high2float(b23);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = epilogue_act(v[j], act);
    if (residual != nullptr) {
      const uint2 r = *reinterpret_cast<const uint2*>(residual + row * ldr + m);
      const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
      const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
      v[0] += __low2float(r01); v[1] += __high2float(r01); v[2] += __low2float(r23); v[3] += __high2float(r23);
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(out_row) + m) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      const __nv_bfloat162 o01 = __floats2bfloat162_rn(v[0], v[1]);
      const __nv_bfloat162 o23 = __floats2bfloat162_rn(v[2], v[3]);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&o01);
      o.y = *reinterpret_cast<const uint32_t*>(&o23);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out_row) + m) = o;
    }
    return;
  }
  for (int j = 0; j < 4; ++j) {
    if (m + j >= m_out) break;
    float x = v[j];
    if (bias != nullptr) x += __bfloat162float(bias[m + j]);
    x = epilogue_act(x, act);
    if (residual != nullptr) x += __bfloat162float(residual[row * ldr + m + j]);
    if (out_f32) static_cast<float*>(out_row)[m + j] = x;
    else static_cast<__nv_bfloat16*>(out_row)[m + j] = __float2bfloat16(x);
  }
}

template <int BN, bool GATED>
struct Cfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes * (GATED ? 2 : 1) + kBBytes;
  static constexpr int kAccCols = BN * (GATED ? 2 : 1);
  static constexpr int kTmemCols = (2 * kAccCols) <= 32    ? 32
                                   : (2 * kAccCols) <= 64  ? 64
                                   : (2 * kAccCols) <= 128 ? 128
                                   : (2 * kAccCols) <= 256 ? 256
                                                           : 512;
  static constexpr int kStagesRaw = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  // tiles + 1 KB alignment slack + barriers and the group tables (starts, ends, tile prefix sums:
  // 3 * (kMaxGroups + 1) ints after 512 bytes of barriers)
  static constexpr int kAuxBytes = (1024 + 12 * (kMaxGroups + 1) + 512 + 15) / 16 * 16;
  // wide token tiles stage each 16-token chunk of the epilogue through shared memory (two
  // [16][128] fp32 buffers) so that outputs leave as 16-byte vectors along the feature axis
  static constexpr bool kStagedEpi = BN >= 64;
  static constexpr int kEpiBytes = kStagedEpi ? 2 * 16 * kBM * 4 : 0;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kAuxBytes + kEpiBytes;
  static_assert(2 * kAccCols <= 512, "accumulators exceed TMEM");
  static_assert(kSmemBytes <= 232448, "shared memory exceeds 227 KB");
  static_assert(kBBytes % 1024 == 0, "B tile must keep 1024-byte alignment");
};

// Tile t -> group g, weight tile mt, token tile nt.  Group g's rows are [offs[g], ends[g]).
// Order: token tiles fastest (a weight tile stays hot while the CTAs of a wave walk the token
// tiles: decode and MoE, where the weights are the big operand), or with `mt_fast` weight tiles
// fastest (a dense GEMM whose token operand is larger than L2: the CTAs of a wave share a few
// token tiles, each read from DRAM once, while the weights stay in L2).
template <int BN>
__device__ __forceinline__ void decode_tile(int t, const int* prefix, const int* offs, const int* ends, int groups,
                                            int& g, int& mt, int& nt, int mtiles = 0, int mt_fast = 0) {
  int lo = 0, hi = groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  g = lo;
  const int local = t - prefix[g];
  if (mt_fast) {
    nt = local / mtiles;
    mt = local - nt * mtiles;
    return;
  }
  const int rows = ends[g] - offs[g];
  const int ntiles = (rows + BN - 1) / BN;
  mt = local / ntiles;
  nt = local - mt * ntiles;
}

// ACT = false: the epilogue has no activation code at all (the common case; a
// smaller kernel is fetched faster, which the few-tile decode GEMMs feel).
// CL = true: the split-K-over-a-cluster variant (only the cluster epilogue is compiled in, so
// the few-tile decode GEMMs run a smaller kernel); CL = false: every other mode.
template <int BN, bool GATED, bool ACT, bool CL>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const DevParams p) {
  using C = Cfg<BN, GATED>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base for the swizzled tiles.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* aux = smem + C::kStages * C::kStageBytes;
  float* epi = reinterpret_cast<float*>(aux + C::kAuxBytes);   // staged-epilogue buffers
  __shared__ int s_last;  // split-K: this CTA finalises the tile
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(aux);
  uint64_t* empty_bar = full_bar + C::kStages;
  uint64_t* tfull_bar = empty_bar + C::kStages;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2]
  uint64_t* drain_bar = tempty_bar + 2;           // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* total_tiles_s = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));
  int* offs_s = reinterpret_cast<int*>(aux + 512);
  int* prefix_s = offs_s + (kMaxGroups + 1);
  int* ends_s = prefix_s + (kMaxGroups + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = p.groups;
  const int m_tiles = (p.m_out + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  // Group row offsets and tile prefix sums (warp 2); device offsets come from a
  // previous kernel, dense GEMMs need none.
  if (warp == 2) {
    if (p.offsets != nullptr || p.seg_counts != nullptr) grid_dep_wait();
    // expert-parallel: every source has dispatched its rows (and its counter updates); after a
    // timeout (status 2) the groups are taken as empty, so the CTA does no work
    const bool counts_ok = !(p.setup_wait && p.wait_count > 0) ||
                           wait_flags_warp(p.wait_flags, p.wait_seq, p.wait_count, p.wait_timeout_ns, p.status, lane);
    int carry = 0;
    for (int base = 0; base < groups; base += 32) {
      const int g = base + lane;
      int rows = 0;
      if (g < groups) {
        int o0, o1;
        if (p.seg_counts != nullptr) {
          int c = counts_ok ? p.seg_counts[g] : 0;
          c = c < 0 ? 0 : (c > p.seg_cap ? p.seg_cap : c);
          if (blockIdx.x == 0 && p.seg_counts_copy != nullptr) p.seg_counts_copy[g] = c;
          o0 = g * p.seg_cap;
          o1 = o0 + c;
        } else {
          o0 = p.offsets ? p.offsets[g] : 0;
          o1 = p.offsets ? p.offsets[g + 1] : p.rows;
        }
        offs_s[g] = o0;
        ends_s[g] = o1;
        if (g == groups - 1) offs_s[groups] = o1;
        rows = o1 - o0;
      }
      const int tiles = (g < groups) ? m_tiles * ((rows + BN - 1) / BN) : 0;
      int incl = tiles;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
      }
      if (g < groups) prefix_s[g] = carry + incl - tiles;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      prefix_s[groups] = carry;
      *total_tiles_s = carry;
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();

  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = *total_tiles_s;
  const int num_kb = (p.k + kBK - 1) / kBK;
  const int ks = p.k_splits > 1 ? p.k_splits : 1;
  const int kb_per = (num_kb + ks - 1) / ks;
  const int total_work = total_tiles * ks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // Dense GEMMs: issue the weight tiles of the first work item's first stages before
      // waiting for the previous kernel (weights never depend on it); their activation tiles
      // follow the wait on the same stage barriers.
      int pre = 0;
      if (p.pdl_prefetch_a && p.offsets == nullptr && p.seg_counts == nullptr && p.wait_count == 0 &&
          static_cast<int>(blockIdx.x) < total_work) {
        const int w = blockIdx.x;
        const int t = w / ks, split = w - t * ks;
        int g, mt, nt;
        decode_tile<BN>(t, prefix_s, offs_s, ends_s, groups, g, mt, nt, p.m_tiles, p.mt_fast);
        const int a_row = g * p.a_rows + mt * kBM;
        const int kb0 = split * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        pre = min(C::kStages, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          uint8_t* sa = smem + i * C::kStageBytes;
          mbar_arrive_expect_tx(&full_bar[i], C::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full_bar[i], (kb0 + i) * kBK, a_row);
          if (GATED) tma_load_2d(sa + C::kABytes, &tmap_a, &full_bar[i], (kb0 + i) * kBK, a_row + p.m_out);
        }
      }
      grid_dep_wait();
      if (p.wait_count > 0 && !p.setup_wait) {
        // the activations are gathered from the other ranks: wait (bounded) until all have landed
        const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(p.wait_seq);
        const uint64_t t0 = globaltimer_ns();
        for (int i = 0; i < p.wait_count; ++i) {
          uint32_t v;
          do {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.wait_flags + i) : "memory");
            if (v == target) break;
            if (globaltimer_ns() - t0 > static_cast<uint64_t>(p.wait_timeout_ns)) {
              if (p.status) atomicExch(p.status, kStatusPeerTimeout);
              break;
            }
          } while (true);
        }
      }
      // Rows that peers stored with generic-proxy writes are read below by TMA (async proxy).
      if (p.wait_count > 0) asm volatile("fence.proxy.async.global;" ::: "memory");
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x) {
        const int t = w / ks, split = w - t * ks;
        int g, mt, nt;
        decode_tile<BN>(t, prefix_s, offs_s, ends_s, groups, g, mt, nt, p.m_tiles, p.mt_fast);
        const int a_row = g * p.a_rows + mt * kBM;
        const int b_row = offs_s[g] + nt * BN;
        const int kb0 = split * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pre > 0 && w == static_cast<int>(blockIdx.x) && kb - kb0 < pre) {
            // weight tile already in flight on this (fresh) stage: add the activation tile
            tma_load_2d(smem + stage * C::kStageBytes + C::kABytes * (GATED ? 2 : 1), &tmap_b, &full_bar[stage],
                        kb * kBK, b_row);
            ++issued;
            if (++stage == C::kStages) { stage = 0; phase ^= 1; }
            continue;
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes * (GATED ? 2 : 1);
          mbar_arrive_expect_tx(&full_bar[stage], C::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * kBK, a_row);
          if (GATED) tma_load_2d(sa + C::kABytes, &tmap_a, &full_bar[stage], kb * kBK, a_row + p.m_out);
          tma_load_2d(sb, &tmap_b, &full_bar[stage], kb * kBK, b_row);
          ++issued;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: wait (bounded) for the loads this thread issued last on every stage.
      const long first = issued > C::kStages ? issued - C::kStages : 0;
      for (long i = first; i < issued; ++i) {
        const int s = static_cast<int>(i % C::kStages);
        const uint32_t ph = static_cast<uint32_t>((i / C::kStages) & 1);
        mbar_wait(&full_bar[s], ph, nullptr, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    grid_dep_wait();  // nothing to do before the activations arrive; keeps the bounded waits short
    constexpr uint32_t idesc = umma_idesc_bf16_f32(kBM, BN);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x, ++local) {
      const int split = w % ks;
      const int kb0 = split * kb_per, kb1 = min(num_kb, kb0 + kb_per);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * C::kAccCols;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes * (GATED ? 2 : 1);
          const uint64_t adesc = umma_desc_sw128(sa);
          const uint64_t bdesc = umma_desc_sw128(sb);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle atom (>>4 => +2).
            const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
            umma_f16_ss(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, accum);
            if (GATED) {
              const uint64_t adesc_up = umma_desc_sw128(sa + C::kABytes);
              umma_f16_ss(d_tmem + BN, adesc_up + 2 * kk, bdesc + 2 * kk, idesc, accum);
            }
          }
          umma_commit(&empty_bar[stage]);
        }
        __syncwarp();
        if (++stage == C::kStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull_bar[acc]);
      __syncwarp();
    }
    // Drain every MMA this thread issued before TMEM is released.
    if (lane == 0) {
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, nullptr, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // residual / output buffers belong to the stream's earlier kernels
    const int lane_base = 32 * (warp & 3);
    int local = 0;
    int epi_ctr = 0;   // staged chunks so far (alternates the two buffers)
    for (int w = blockIdx.x; w < total_work; w += gridDim.x, ++local) {
      const int t = w / ks;
      int g, mt, nt;
      decode_tile<BN>(t, prefix_s, offs_s, ends_s, groups, g, mt, nt, p.m_tiles, p.mt_fast);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // warp-uniform outcome: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.status))) break;
      tc_fence_after();
      const int m = mt * kBM + lane_base + lane;
      const int row0 = offs_s[g] + nt * BN;
      const int row_end = ends_s[g];
      const bool m_ok = m < p.m_out;
      float bias_v = 0.f;
      if (p.bias != nullptr && m_ok) bias_v = __bfloat162float(p.bias[static_cast<int64_t>(g) * p.m_out + m]);
      const uint32_t t_base = tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * C::kAccCols;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        uint32_t u[16];
        tmem_ld_32x32b_x16(t_base + c, r);
        if (GATED) tmem_ld_32x32b_x16(t_base + BN + c, u);
        tmem_ld_wait();
        if (CL) {
          // split-K partial into this CTA's shared memory as a [BN][128] fp32 tile (the stage
          // ring is idle: this CTA's only work item has finished its MMAs)
          float* sp = reinterpret_cast<float*>(smem) + c * kBM + lane_base + lane;
#pragma unroll
          for (int j = 0; j < 16; ++j) sp[j * kBM] = __uint_as_float(r[j]);
        } else if (!CL && ks > 1) {
          // split-K partial into this split's plane [split][t][BN][128] (thread = one A row; for
          // each token a warp stores 32 consecutive floats); summed in split order by the
          // finaliser, so the result does not depend on which split arrives first
          float* wsp = p.ws + ((static_cast<int64_t>(w - t * ks) * total_tiles + t) * BN + c) * kBM + lane_base + lane;
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(wsp + j * kBM, __uint_as_float(r[j]));
        } else if (!CL && C::kStagedEpi && p.vec8) {
          // activations per thread (one feature m, 16 tokens), the chunk through shared memory,
          // then each thread stores two vectors of 8 consecutive features of one token (and adds
          // the matching 16-byte residual vectors).  One named barrier per chunk: a buffer is
          // rewritten two chunks later, after every thread has passed the barrier in between.
          float* stg = epi + (epi_ctr & 1) * (16 * kBM);
          ++epi_ctr;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v = __uint_as_float(r[j]);
            if (GATED) {
              v = silu_f(v) * __uint_as_float(u[j]);
            } else {
              v += bias_v;
              if (ACT) {
                if (p.act == kActGeluTanh) v = gelu_tanh_f(v);
                else if (p.act == kActGeluErf) v = gelu_erf_f(v);
                else if (p.act == kActSilu) v = silu_f(v);
              }
            }
            stg[j * kBM + lane_base + lane] = v;
          }
          asm volatile("bar.sync 2, 128;" ::: "memory");
          const int tid = static_cast<int>(threadIdx.x) - 64;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int idx = tid + 128 * q;          // 16 tokens x 16 groups of 8 features
            const int tok = idx >> 4, cg = (idx & 15) * 8;
            const int row = row0 + c + tok;
            const int mm = mt * kBM + cg;
            if (row < row_end && mm < p.m_out) {
              const float4 a0 = *reinterpret_cast<const float4*>(stg + tok * kBM + cg);
              const float4 a1 = *reinterpret_cast<const float4*>(stg + tok * kBM + cg + 4);
              float o[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
              if (p.residual != nullptr) {
                const uint4 rv = *reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(row) * p.ldr + mm);
                const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  o[2 * j] += __low2float(rh[j]);
                  o[2 * j + 1] += __high2float(rh[j]);
                }
              }
              if (p.out_f32) {
                float* dst = static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo + mm;
                reinterpret_cast<float4*>(dst)[0] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4*>(dst)[1] = make_float4(o[4], o[5], o[6], o[7]);
              } else {
                uint4 ov;
                __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
                for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
                __nv_bfloat16* orow = out_row_bf16(p, row);
                if (orow != nullptr) *reinterpret_cast<uint4*>(orow + mm) = ov;
              }
            }
          }
        } else if (!CL && m_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = row0 + c + j;
            if (row < row_end) {
              float v = __uint_as_float(r[j]);
              if (GATED) {
                v = silu_f(v) * __uint_as_float(u[j]);
              } else {
                v += bias_v;
                if (ACT) {
                  if (p.act == kActGeluTanh) v = gelu_tanh_f(v);
                  else if (p.act == kActGeluErf) v = gelu_erf_f(v);
                  else if (p.act == kActSilu) v = silu_f(v);
                }
              }
              if (p.residual != nullptr) v += __bfloat162float(p.residual[static_cast<int64_t>(row) * p.ldr + m]);
              if (p.out_f32) {
                static_cast<float*>(p.out)[static_cast<int64_t>(row) * p.ldo + m] = v;
              } else {
                __nv_bfloat16* orow = out_row_bf16(p, row);
                if (orow != nullptr) orow[m] = __float2bfloat16(v);
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      if (!CL && ks > 1 && p.counters != nullptr) {
        // The last split of this tile to arrive sums the partials and runs the epilogue:
        // no second launch.  Counters reset themselves for the next call / graph replay.
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(&p.counters[t], 1);
          s_last = prev == ks - 1;
          if (s_last) p.counters[t] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (s_last) {
          __threadfence();
          // Sum the split planes of tile t in split order: the 128 epilogue threads sweep the
          // [BN][128] tile as float4s (coalesced), 8 per thread per round, every split's loads
          // of a round in flight together; the epilogue stores four outputs per float4.
          constexpr int kU = 8;
          constexpr int kN4 = BN * kBM / 4;
          const int tid = threadIdx.x - 64;
          const int64_t plane4 = static_cast<int64_t>(total_tiles) * BN * kBM / 4;
          const float4* base4 = reinterpret_cast<const float4*>(p.ws + static_cast<int64_t>(t) * BN * kBM);
#pragma unroll 1
          for (int e0 = tid; e0 < kN4; e0 += 128 * kU) {
            float4 acc[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
              const int e = e0 + u * 128;
              acc[u] = e < kN4 ? __ldcg(base4 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll 1
            for (int sp = 1; sp < ks; ++sp) {
              float4 x[kU];
#pragma unroll
              for (int u = 0; u < kU; ++u) {
                const int e = e0 + u * 128;
                x[u] = e < kN4 ? __ldcg(base4 + sp * plane4 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < kU; ++u) {
                acc[u].x += x[u].x;
                acc[u].y += x[u].y;
                acc[u].z += x[u].z;
                acc[u].w += x[u].w;
              }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
              const int e = e0 + u * 128;
              if (e >= kN4) break;
              const int tok = e / (kBM / 4);
              const int mm = mt * kBM + (e - tok * (kBM / 4)) * 4;
              const int row = row0 + tok;
              if (row < row_end && mm < p.m_out) {
                void* orow = p.out_f32 ? static_cast<void*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo)
                                       : static_cast<void*>(out_row_bf16(p, row));
                if (orow != nullptr)
                store_out4(p.bias == nullptr ? nullptr : p.bias + static_cast<int64_t>(g) * p.m_out, p.residual, p.ldr,
                           orow, p.out_f32, p.act, mm, p.m_out, p.vec4, row, acc[u]);
              }
            }
          }
        }
      }
    }
  }

  if (!CL && warp >= 2 && p.signal_count > 0) {
    // Completion signal (expert-parallel combine): each epilogue thread fences its stores at
    // system scope, the CTA arrives once, and the last CTA to arrive release-stores the layer's
    // sequence number into every peer's flag.  CTA 0 clears the per-expert counters first.
    __threadfence_system();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (threadIdx.x == 64) {
      if (blockIdx.x == 0 && p.zero_ptr != nullptr) {
        for (int i = 0; i < p.zero_n; ++i) p.zero_ptr[i] = 0;
        __threadfence_system();
      }
      const int prev = atomicAdd(p.arrive_counter, 1);
      if (prev == static_cast<int>(gridDim.x) - 1) {
        *p.arrive_counter = 0;
        __threadfence_system();
        const uint32_t seq = *reinterpret_cast<const volatile uint32_t*>(p.signal_seq);
        for (int d = 0; d < p.signal_count; ++d)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.signal_flags[d]), "r"(seq) : "memory");
      }
    }
  }

  if (CL) {
    // Cluster split-K: CTA r of the cluster holds split r's partial tile in shared memory.
    // After the cluster barrier each CTA sums one slice of the tile's token rows over every
    // CTA's copy (distributed shared memory, in rank order, so the result does not depend
    // on timing) and runs the epilogue; the second barrier keeps every CTA's shared memory
    // alive until the others have read it.  Every thread of the CTA takes both barriers.
    cluster_sync();
    if (warp >= 2 && total_work > 0) {
      const int t = static_cast<int>(blockIdx.x) / ks;
      const uint32_t rank = cluster_ctarank();
      int g, mt, nt;
      decode_tile<BN>(t, prefix_s, offs_s, ends_s, groups, g, mt, nt, p.m_tiles, p.mt_fast);
      const int row0 = offs_s[g] + nt * BN;
      const int row_end = ends_s[g];
      const int per = (BN + ks - 1) / ks;
      const int tok_lo = static_cast<int>(rank) * per, tok_hi = min(BN, tok_lo + per);
      const int n4 = max(0, tok_hi - tok_lo) * (kBM / 4);
      const uint32_t base = smem_u32(smem) + static_cast<uint32_t>(tok_lo * kBM * 4);
      const int tid = threadIdx.x - 64;
#pragma unroll 1
      for (int e = tid; e < n4; e += 128) {
        const uint32_t off = static_cast<uint32_t>(e) * 16u;
        float4 x[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          x[q] = q < ks ? ld_dsmem_f4(dsmem_addr(base + off, static_cast<uint32_t>(q))) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 acc = x[0];
#pragma unroll
        for (int q = 1; q < 8; ++q) {
          if (q < ks) {
            acc.x += x[q].x;
            acc.y += x[q].y;
            acc.z += x[q].z;
            acc.w += x[q].w;
          }
        }
        const int tok = tok_lo + e / (kBM / 4);
        const int mm = mt * kBM + (e % (kBM / 4)) * 4;
        const int row = row0 + tok;
        if (row < row_end && mm < p.m_out) {
          void* orow = p.out_f32 ? static_cast<void*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo)
                                 : static_cast<void*>(out_row_bf16(p, row));
          if (orow != nullptr)
          store_out4(p.bias == nullptr ? nullptr : p.bias + static_cast<int64_t>(g) * p.m_out, p.residual, p.ldr, orow,
                     p.out_f32, p.act, mm, p.m_out, p.vec4, row, acc);
        }
      }
    }
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Fallback finaliser (more tiles than arrival counters): sums the split planes
// [splits][tiles][BN][128] in split order and applies the epilogue.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int ks, int bn, int n_tiles, int total_tiles,
                                     int rows, int m_out, void* out, int64_t ldo, int out_f32,
                                     const __nv_bfloat16* __restrict__ bias,
                                     const __nv_bfloat16* __restrict__ residual, int64_t ldr, int act) {
  const int64_t n = static_cast<int64_t>(rows) * m_out;
  const int64_t plane = static_cast<int64_t>(total_tiles) * kBM * bn;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / m_out);
    const int m = static_cast<int>(i - static_cast<int64_t>(row) * m_out);
    const int t = (m / kBM) * n_tiles + row / bn;
    const float* src = ws + (static_cast<int64_t>(t) * bn + row % bn) * kBM + m % kBM;
    float v = 0.f;
    for (int s = 0; s < ks; ++s) v += __ldcg(src + s * plane);
    if (bias != nullptr) v += __bfloat162float(bias[m]);
    v = epilogue_act(v, act);
    if (residual != nullptr) v += __bfloat162float(residual[static_cast<int64_t>(row) * ldr + m]);
    if (out_f32) static_cast<float*>(out)[static_cast<int64_t>(row) * ldo + m] = v;
    else static_cast<__nv_bfloat16*>(out)[static_cast<int64_t>(row) * ldo + m] = __float2bfloat16(v);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

// 2-D bf16 tensor map [rows, cols] (cols contiguous), box [box_rows, 64], 128-byte swizzle.
bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                  uint32_t box_rows) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  });
  return n;
}

// Largest split count of the split-K modes (OMNI_SPLITK_MAX, 2..8; default 8 = the portable
// cluster size limit).
int splitk_max() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("OMNI_SPLITK_MAX");
    const int x = e ? std::atoi(e) : 8;
    v = x < 2 ? 2 : (x > 8 ? 8 : x);
  }
  return v;
}

bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("OMNI_PDL");
    on = (e == nullptr || std::strcmp(e, "0") != 0) ? 1 : 0;
  }
  return on == 1;
}

template <int BN, bool GATED, bool ACT>
cudaError_t launch(const GemmArgs& a, cudaStream_t stream) {
  using C = Cfg<BN, GATED>;
  {
    cudaError_t e = ensure_smem_attr<gemm_bf16_kernel<BN, GATED, ACT, false>>(C::kSmemBytes);
    if (e != cudaSuccess) return e;
    if constexpr (!GATED) {
      e = ensure_smem_attr<gemm_bf16_kernel<BN, GATED, ACT, true>>(C::kSmemBytes);
      if (e != cudaSuccess) return e;
    }
  }
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, a.a, static_cast<uint64_t>(a.groups) * a.a_rows, a.k, a.k, kBM)) return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tb, a.b, a.rows > 0 ? a.rows : 1, a.k, a.k, BN)) return cudaErrorInvalidValue;
  DevParams p;
  p.out = a.out;
  p.ldo = a.ldo;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.ldr = a.ldr;
  p.offsets = a.offsets;
  p.rows = a.rows;
  p.m_out = a.m_out;
  p.a_rows = a.a_rows;
  p.k = a.k;
  p.groups = a.groups;
  p.out_f32 = a.out_f32;
  p.act = a.act;
  p.status = a.status;
  p.k_splits = 1;
  p.ws = nullptr;
  {
    auto al = [](const void* q, int bytes) { return (reinterpret_cast<uintptr_t>(q) % bytes) == 0; };
    const int ob = a.out_f32 ? 16 : 8;
    p.vec4 = (a.m_out % 4 == 0) && (a.ldo % 4 == 0) && al(a.out, ob) && (a.bias == nullptr || al(a.bias, 8)) &&
             (a.residual == nullptr || (a.ldr % 4 == 0 && al(a.residual, 8))) ? 1 : 0;
    p.vec8 = (a.m_out % 8 == 0) && (a.ldo % 8 == 0) && al(a.out, 16) &&
             (a.residual == nullptr || (a.ldr % 8 == 0 && al(a.residual, 16))) ? 1 : 0;
  }
  p.counters = nullptr;
  p.peer_out = a.peer_out;
  p.rows_per = a.rows_per > 0 ? a.rows_per : 1;
  p.wait_flags = a.wait_flags;
  p.wait_seq = a.wait_seq;
  p.wait_count = a.wait_flags != nullptr && a.wait_seq != nullptr ? a.wait_count : 0;
  p.wait_timeout_ns = a.wait_timeout_ns;
  p.seg_cap = a.seg_cap;
  p.seg_counts = a.seg_cap > 0 ? a.seg_counts : nullptr;
  p.seg_counts_copy = a.seg_counts_copy;
  p.setup_wait = a.setup_wait;
  p.row_tag = a.row_tag;
  p.peer_rows = a.peer_rows;
  p.tag_ranks = a.tag_ranks;
  p.tag_slots = a.tag_slots;
  p.signal_flags = a.signal_flags;
  p.signal_seq = a.signal_seq;
  p.signal_count = a.signal_flags != nullptr && a.signal_seq != nullptr && a.arrive_counter != nullptr
                       ? a.signal_count : 0;
  p.arrive_counter = a.arrive_counter;
  p.zero_ptr = a.zero_ptr;
  p.zero_n = a.zero_n;
  const int m_tiles = (a.m_out + kBM - 1) / kBM;
  const int num_kb = (a.k + kBK - 1) / kBK;
  p.m_tiles = m_tiles;
  {
    // a dense GEMM whose token operand exceeds L2 while its weights fit: weight tiles fastest
    const double w_bytes = static_cast<double>(a.m_out) * (GATED ? 2 : 1) * a.k * 2.0;
    const double x_bytes = static_cast<double>(a.rows) * a.k * 2.0;
    p.mt_fast = (a.groups == 1 && a.offsets == nullptr && a.seg_cap <= 0 && x_bytes > 64e6 && w_bytes <= 64e6) ? 1 : 0;
  }
  // Split-K for dense GEMMs that would leave most SMs idle (decode projections).
  p.cluster_splitk = 0;
  if (!GATED && a.offsets == nullptr && a.seg_cap <= 0 && (a.splitk_ws != nullptr || a.splitk_cluster)) {
    const long tiles = static_cast<long>(m_tiles) * ((a.rows + BN - 1) / BN);
    const int sms = num_sms();
    if (tiles * 2 <= sms && num_kb >= 4) {
      // one wave: tiles * splits <= SMs (a partial second wave doubles the time)
      int ksp = static_cast<int>(sms / tiles);
      if (ksp > num_kb / 2) ksp = num_kb / 2;
      const int kmax = splitk_max();
      if (ksp > kmax) ksp = kmax;   // the finaliser reads every split: keep its rounds few
      // Clusters of 8 are placed inside one GPC two at a time; more than a couple of them do
      // not all fit at once and a second wave doubles the time (o_proj at 64 tokens: 16 tiles x 8
      // splits 22.8 us, x 4 splits 17.3 us), so several tiles take clusters of at most 4.
      if (a.splitk_cluster && tiles > 2 && ksp > 4) ksp = 4;
      if (ksp > 1) {
        const int per = (num_kb + ksp - 1) / ksp;
        ksp = (num_kb + per - 1) / per;  // no empty splits
        const long long plane = static_cast<long long>(m_tiles) * kBM * ((a.rows + BN - 1) / BN) * BN;
        if (a.splitk_cluster && tiles * ksp <= sms) {
          // one cluster of ksp CTAs per output tile: no global scratch, no arrival counters
          p.k_splits = ksp;
          p.cluster_splitk = 1;
        } else if (plane * ksp <= a.splitk_ws_floats) {
          p.k_splits = ksp;
          p.ws = a.splitk_ws;
          // tiles within the counter slots: the last split finalises in-kernel (no reduce launch)
          if (a.splitk_counters != nullptr && tiles <= a.splitk_counter_slots) p.counters = a.splitk_counters;
          if (p.counters == nullptr && a.peer_out != nullptr) {  // the fallback reduce writes locally only
            p.k_splits = 1;
            p.ws = nullptr;
          }
        }
      }
    }
  }
  // Upper bound of the tile count: every group may add one partial token tile.
  const bool grouped = a.offsets != nullptr || a.seg_cap > 0;
  const long row_tiles = (grouped ? (static_cast<long>(a.rows) + BN - 1) / BN + a.groups : (a.rows + BN - 1) / BN);
  const long bound = static_cast<long>(m_tiles) * (row_tiles > 0 ? row_tiles : 1) * p.k_splits;
  int grid = a.max_ctas > 0 ? a.max_ctas : num_sms();
  if (bound < grid) grid = static_cast<int>(bound);
  if (grid < 1) grid = 1;
  const bool pdl = pdl_enabled();
  p.pdl_prefetch_a = pdl && a.static_a ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.cluster_splitk) {
    grid = static_cast<int>((static_cast<long>(m_tiles) * ((a.rows + BN - 1) / BN)) * p.k_splits);
    cfg.gridDim = dim3(grid);
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.k_splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t le;
  if constexpr (!GATED) {
    le = p.cluster_splitk ? cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<BN, GATED, ACT, true>, ta, tb, p)
                          : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<BN, GATED, ACT, false>, ta, tb, p);
  } else {
    le = cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<BN, GATED, ACT, false>, ta, tb, p);
  }
  if (le != cudaSuccess) return le;
  if (p.k_splits > 1 && p.counters == nullptr && !p.cluster_splitk) {
    const long long n = static_cast<long long>(a.rows) * a.m_out;
    int rgrid = static_cast<int>((n + 255) / 256);
    if (rgrid > 4 * num_sms()) rgrid = 4 * num_sms();
    const int n_tiles = (a.rows + BN - 1) / BN;
    splitk_reduce_kernel<<<rgrid, 256, 0, stream>>>(p.ws, p.k_splits, BN, n_tiles, m_tiles * n_tiles, a.rows, a.m_out,
                                                    a.out, a.ldo, a.out_f32, p.bias, p.residual, a.ldr, a.act);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  if (a.groups < 1 || a.groups > kMaxGroups || a.k <= 0 || a.m_out <= 0) return cudaErrorInvalidValue;
  if (a.k % 8 != 0) return cudaErrorInvalidValue;  // 16-byte row stride for TMA
  if (a.seg_cap > 0 && (a.seg_counts == nullptr || static_cast<long long>(a.seg_cap) * a.groups > a.rows))
    return cudaErrorInvalidValue;
  if (a.row_tag != nullptr && (a.peer_rows == nullptr || a.out_f32 || a.tag_ranks < 1)) return cudaErrorInvalidValue;
  // a GEMM that signals completion must run even without rows: its peers wait for the flags
  if (a.rows == 0 && a.signal_count == 0) return cudaSuccess;
  int hint = a.expected_rows_per_group > 0 ? a.expected_rows_per_group : a.rows;
  if (a.gated) {
    if (hint <= 16) return launch<16, true, false>(a, stream);
    if (hint <= 32) return launch<32, true, false>(a, stream);
    if (hint <= 64) return launch<64, true, false>(a, stream);
    return launch<128, true, false>(a, stream);
  }
  if (a.act != kActNone) {
    if (hint <= 16) return launch<16, false, true>(a, stream);
    if (hint <= 32) return launch<32, false, true>(a, stream);
    if (hint <= 64) return launch<64, false, true>(a, stream);
    if (hint <= 128) return launch<128, false, true>(a, stream);
    return launch<256, false, true>(a, stream);
  }
  if (hint <= 16) return launch<16, false, false>(a, stream);
  if (hint <= 32) return launch<32, false, false>(a, stream);
  if (hint <= 64) return launch<64, false, false>(a, stream);
  if (hint <= 128) return launch<128, false, false>(a, stream);
  return launch<256, false, false>(a, stream);
}

}  // namespace omni
