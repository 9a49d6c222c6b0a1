// Paged GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes one 128-row query tile of one (request, KV head): the rows
// are GQA-packed, row r = (token tok0 + r / G, query head h * G + r % G), so a
// K/V block staged once serves all G heads.  Per 128-key block j:
//
//   S_j = Q K_j^T          tcgen05.mma (A = Q, B = K, both K-major in shared
//                          memory), fp32 accumulator in TMEM (two buffers)
//   P_j = exp2(S_j - m)    softmax warps: one thread per row reads its S row
//                          with tcgen05.ld, masks (causal / context length),
//                          keeps the running max m and sum l in registers,
//                          writes P (bf16) into shared memory in the 128-byte
//                          swizzled K-major layout (two buffers)
//   O += P_j V_j           tcgen05.mma (A = P, B = V as an MN-major operand:
//                          V rows are keys, 64 contiguous dims per 128-byte
//                          row), accumulator in TMEM
//
// The running max is only raised when a block's max exceeds it by more than 8
// (log2 units, i.e. P values stay below 2^8); the O row in TMEM is then
// rescaled by its thread (tcgen05.ld / st) after the previous PV product has
// completed.  The final O row is divided by l and stored as bf16.
//
// Warp roles (6 warps): warp 0 TMA producer (Q once, then K/V pages through the
// block table into a two-stage ring, local memory only, no multicast), warp 1
// TMEM allocator + MMA issuer (one elected lane), warps 2-5 softmax +
// epilogue (warp w owns TMEM lanes 32 * (w % 4) .. + 31 = those query rows).
// The MMA issue order S_0, S_1, PV_0, S_2, PV_1, ... lets the softmax of block
// j overlap the PV product of block j-1.  Every wait is bounded (%globaltimer);
// a wait that runs out records status 1, drains and frees TMEM.
//
// Tensor maps: Q as [tokens, Hq, D] (box 128 / G tokens x G heads x 64 dims),
// the K / V cache of one layer as [pages * Hkv * 64, D] rows (box 64 x 64).
//
// Reference counterpart: the FlashInfer / TRT-LLM prefill attention behind
// RadixAttention (sglang_omni/models/qwen3_omni/thinker.py:236-243).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "host_util.h"
#include "omni_kernels.h"
#include "sm100.cuh"

namespace omni {
namespace {

constexpr int kRows = 128;          // packed query rows per tile
constexpr int kBN = 128;            // keys per block (two pages)
constexpr int kD = 128;             // head dim
constexpr int kKvStages = 2;
constexpr int kThreads = 192;
constexpr int kRegion = kRows * 128;        // one 64-column region of a 128-row tile: 16 KB
constexpr int kTileBytes = 2 * kRegion;     // 128 rows x 128 columns bf16: 32 KB
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units
constexpr int kTmemCols = 512;              // S0 | S1 | O (128 columns each)

struct FaSmem {
  // every tile 1024-byte aligned (128-byte swizzle atoms)
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTileBytes;
  static constexpr int kV = kK + kKvStages * kTileBytes;
  static constexpr int kP = kV + kKvStages * kTileBytes;
  static constexpr int kBars = kP + 2 * kTileBytes;
  static constexpr int kBytes = kBars + 256 + 1024;   // barriers + alignment slack
};
static_assert(FaSmem::kBytes <= 232448, "shared memory exceeds 227 KB");

struct FaParams {
  const int* block_table;
  int bt_stride;
  const int* cu_q;
  const int* kv_lens;
  const int* tile_req;
  const int* tile_tok0;
  int hq, hkv, G;
  float scale_log2;
  int causal;
  __nv_bfloat16* out;
  int64_t out_stride;
  int num_pages;
  int* status;
  const int* cu_kv;   // contiguous mode: first key row of each request (nullptr: paged)
  int d_head;         // head dim of q / k / v / out rows (<= 128; columns past it load as zeros)
};

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Generic-proxy writes of shared memory (P) become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// UMMA shared-memory descriptor of an MN-major operand in the 128-byte swizzled layout:
// rows of 64 bf16 along MN (128 bytes), 8-row atoms along K (1024 bytes apart, SBO), MN
// blocks of 64 columns `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// kind::f16 instruction descriptor, bf16 x bf16 -> f32, A K-major, B MN-major (bit 16).
constexpr uint32_t umma_idesc_bf16_f32_bmn(int m, int n) { return umma_idesc_bf16_f32(m, n) | (1u << 16); }

__device__ __forceinline__ int fa_page(const FaParams& p, int req, int idx) {
  const int page = p.block_table[static_cast<int64_t>(req) * p.bt_stride + idx];
  return (p.num_pages > 0 && static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_pages)) ? 0 : page;
}

// Issues the TMA loads of one 64-key half block: paged (one page of the block table) or
// contiguous (64 consecutive key rows of head h starting at the request's first key + key0).
__device__ __forceinline__ void load_kv_half(const FaParams& p, const CUtensorMap* tmap_k, const CUtensorMap* tmap_v,
                                             uint64_t* bar, uint8_t* dk, uint8_t* dv, int region_bytes, int req,
                                             int h, int key0, int pages) {
  if (p.cu_kv == nullptr) {
    const int idx = key0 >> 6;
    // a page past the context reads page 0 (masked): constant byte count
    const int page = idx < pages ? fa_page(p, req, idx) : 0;
    const int row = (page * p.hkv + h) * 64;
    for (int r = 0; r < 2; ++r) {
      tma_load_2d(dk + r * region_bytes, tmap_k, bar, r * 64, row);
      tma_load_2d(dv + r * region_bytes, tmap_v, bar, r * 64, row);
    }
  } else {
    const int row = p.cu_kv[req] + key0;   // rows past the tensor read zeros, other requests' are masked
    for (int r = 0; r < 2; ++r) {
      tma_load_3d(dk + r * region_bytes, tmap_k, bar, r * 64, h, row);
      tma_load_3d(dv + r * region_bytes, tmap_v, bar, r * 64, h, row);
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 2^x by the SFU's approximate base-2 exponential (denormal results flush to zero: the
// probabilities are rounded to bf16 anyway).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A bounded wait whose outcome is the same in every lane of the warp (the warp-collective
// tcgen05 loads / stores that follow must never run with part of the warp gone after a
// timeout); `site` names the wait in the status code (16 + site).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int site) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status, kWaitTimeoutNs, kStatusWaitSite + site);
  return __all_sync(0xffffffffu, ok);
}

// Row max of n raw scores with 8 independent partial maxima (no 64-long dependency chain).
template <int N>
__device__ __forceinline__ float row_max(const float (&s)[N]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = s[i];
#pragma unroll
  for (int i = 8; i < N; ++i) m[i & 7] = fmaxf(m[i & 7], s[i]);
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const FaParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* sQ = smem + FaSmem::kQ;
  uint8_t* sK = smem + FaSmem::kK;
  uint8_t* sV = smem + FaSmem::kV;
  uint8_t* sP = smem + FaSmem::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FaSmem::kBars);
  uint64_t* q_full = bars;                 // [1]
  uint64_t* kv_full = bars + 1;            // [2]
  uint64_t* kv_empty = bars + 3;           // [2]
  uint64_t* s_full = bars + 5;             // [2]
  uint64_t* p_full = bars + 7;             // [2]
  uint64_t* pv_done = bars + 9;            // [2]
  uint64_t* drain = bars + 11;             // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int req = p.tile_req[tile];
  const int tok0 = p.tile_tok0[tile];
  const int q_begin = p.cu_q[req];
  const int q_len = p.cu_q[req + 1] - q_begin;
  const int kv_len = p.kv_lens[req];
  const int tpt = kRows / p.G;                       // tokens per tile
  const int past = kv_len - q_len;                   // keys before this chunk's first query
  const int key_end = p.causal ? min(kv_len, past + min(q_len, tok0 + tpt)) : kv_len;
  const int nb = key_end > 0 ? (key_end + kBN - 1) / kBN : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && nb > 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      for (int r = 0; r < 2; ++r)
        tma_load_3d(sQ + r * kRegion, &tmap_q, q_full, r * 64, h * p.G, q_begin + tok0);
      int issued = 0;   // blocks whose loads were issued
      for (int j = 0; j < nb; ++j) {
        const int s = j & 1;
        if (j >= kKvStages && !mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.status, kWaitTimeoutNs,
                                         kStatusWaitSite + 8))
          break;
        issued = j + 1;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
        const int pages = (kv_len + 63) / 64;
        for (int pg = 0; pg < 2; ++pg)
          load_kv_half(p, &tmap_k, &tmap_v, &kv_full[s], sK + s * kTileBytes + pg * (kRegion / 2),
                       sV + s * kTileBytes + pg * (kRegion / 2), kRegion, req, h, j * kBN + pg * 64, pages);
      }
      // drain: every issued load has landed before the CTA's shared memory goes away (also
      // after an aborted wait, so no late copy writes into the next CTA on this SM)
      mbar_wait(q_full, 0, nullptr, p.status);
      for (int j = max(0, issued - kKvStages); j < issued; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, nullptr, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = umma_idesc_bf16_f32(kRows, kBN);
    constexpr uint32_t idesc_o = umma_idesc_bf16_f32_bmn(kRows, kD);
    bool ok = nb > 0 && warp_wait(q_full, 0, abort_flag, p.status, 5);
    auto issue_pv = [&](int j) -> bool {
      const int b = j & 1;
      if (!warp_wait(&p_full[b], (j >> 1) & 1, abort_flag, p.status, 6)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_u32(sP + b * kTileBytes);
        const uint32_t va = smem_u32(sV + (j & 1) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(pa + (kk >> 2) * kRegion) + 2 * (kk & 3);
          const uint64_t bdesc = umma_desc_sw128_mn(va + kk * 16 * 128, kRegion);
          umma_f16_ss(tmem + 256, adesc, bdesc, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[b]);
        umma_commit(&kv_empty[j & 1]);
      }
      __syncwarp();
      return true;
    };
    for (int j = 0; j < nb && ok; ++j) {
      const int s = j & 1;
      if (!warp_wait(&kv_full[s], (j >> 1) & 1, abort_flag, p.status, 7)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sQ);
        const uint32_t ka = smem_u32(sK + s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(qa + (kk >> 2) * kRegion) + 2 * (kk & 3);
          const uint64_t bdesc = umma_desc_sw128(ka + (kk >> 2) * kRegion) + 2 * (kk & 3);
          umma_f16_ss(tmem + s * 128, adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
      }
      __syncwarp();
      if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
    }
    if (ok && nb > 0) issue_pv(nb - 1);
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                  // query row = TMEM lane
    const int tok = tok0 + r / p.G;
    const bool row_ok = tok < q_len;
    const int qpos = past + tok;                        // absolute position of this query
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nb && ok; ++j) {
      const int b = j & 1;
      if (!warp_wait(&s_full[b], (j >> 1) & 1, abort_flag, p.status, 1)) { ok = false; break; }
      tc_fence_after();
      float s[kBN];
      {
        uint32_t v[kBN];
#pragma unroll
        for (int c = 0; c < kBN; c += 32)
          tmem_ld_32x32b_x32(tmem + lane_addr + b * 128 + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < kBN; ++i) s[i] = __uint_as_float(v[i]);
      }
      const int k0 = j * kBN;
      const int lim = p.causal ? min(kv_len, qpos + 1) : kv_len;   // keys [0, lim) are visible
      if (k0 + kBN > lim) {   // diagonal / last block: mask the invisible keys
#pragma unroll
        for (int i = 0; i < kBN; ++i) s[i] = (k0 + i < lim) ? s[i] : -INFINITY;
      }
      const float mraw = row_max(s);
      const float mb = mraw == -INFINITY ? -INFINITY : mraw * p.scale_log2;   // log2 units
      // Lazy rescale, decided per row but executed per warp: the TMEM loads / stores are
      // warp-collective, so when any row of the warp raises its max every lane takes the
      // branch (rows that keep their max scale by 1).
      const bool grow = mb > m_run + kRescaleThreshold || (m_run == -INFINITY && mb > -INFINITY);
      if (__any_sync(0xffffffffu, grow)) {
        const bool scale_o = grow && j > 0 && m_run > -INFINITY;
        if (__any_sync(0xffffffffu, scale_o)) {
          // O holds sum over earlier blocks at max m_run: rescale once the previous PV is done
          if (!warp_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.status, 2)) { ok = false; break; }
          tc_fence_after();
          const float f = scale_o ? ex2_ftz(m_run - mb) : 1.f;
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + 256 + c, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
            tmem_st_32x32b_x32(tmem + lane_addr + 256 + c, v);
          }
          tmem_st_wait();
          l_run *= f;
        }
        if (grow) m_run = mb;
      }
      const float msub = m_run == -INFINITY ? 0.f : m_run;
      // P buffer b was last read by PV_{j-2}
      if (j >= 2 && !warp_wait(&pv_done[b], ((j - 2) >> 1) & 1, abort_flag, p.status, 3)) { ok = false; break; }
      uint8_t* prow = sP + b * kTileBytes + r * 128;
      float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c8 = 0; c8 < kBN / 8; ++c8) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = ex2_ftz(fmaf(s[c8 * 8 + i], p.scale_log2, -msub));
          ls[i] += e[i];
        }
        uint4 pk;
        pk.x = pack_bf16x2(e[0], e[1]);
        pk.y = pack_bf16x2(e[2], e[3]);
        pk.z = pack_bf16x2(e[4], e[5]);
        pk.w = pack_bf16x2(e[6], e[7]);
        const int region = c8 >> 3, chunk = c8 & 7;
        *reinterpret_cast<uint4*>(prow + region * kRegion + ((chunk ^ (r & 7)) << 4)) = pk;
      }
      l_run += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
    }
    // epilogue: O / l once the last PV product is done
    if (ok && nb > 0 && warp_wait(&pv_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1, abort_flag, p.status, 4)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = p.out + static_cast<int64_t>(q_begin + tok) * p.out_stride +
                            static_cast<int64_t>(h * p.G + r % p.G) * p.d_head;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + 256 + c, v);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (c + i >= p.d_head) break;
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv);
            o.y = pack_bf16x2(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
            o.z = pack_bf16x2(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv);
            o.w = pack_bf16x2(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c + i) = o;
          }
        }
      }
    } else if (nb == 0 && row_ok) {
      __nv_bfloat16* orow = p.out + static_cast<int64_t>(q_begin + tok) * p.out_stride +
                            static_cast<int64_t>(h * p.G + r % p.G) * p.d_head;
      for (int c = 0; c < p.d_head; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0u, 0u, 0u, 0u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ two-tile (ping-pong) variant
// One CTA = two 128-row query tiles (A, B) sharing every 64-key K/V block (one page).  The MMA
// issue order  PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)  lets the softmax of tile A on block j+1
// overlap the softmax of tile B on block j and the tensor core's work for the other tile.
// TMEM: S_A | S_B (64 columns each), O_A | O_B (128 each).  Warps: 0 producer, 1 MMA,
// 2-5 softmax + epilogue of tile A, 6-9 of tile B.
namespace pp {
constexpr int kPBN = 64;              // keys per block (one page)
constexpr int kStages = 3;
constexpr int kThreads = 320;
constexpr int kQBytes = kRows * kD * 2;            // 32 KB per tile
constexpr int kKVBytes = kPBN * kD * 2;             // 16 KB (two 64-column regions of 8 KB)
constexpr int kPBytes = kRows * kPBN * 2;           // 16 KB
constexpr int kQ = 0;
constexpr int kK = kQ + 2 * kQBytes;
constexpr int kV = kK + kStages * kKVBytes;
constexpr int kP = kV + kStages * kKVBytes;
constexpr int kBars = kP + 2 * kPBytes;
constexpr int kSmem = kBars + 256 + 1024;
static_assert(kSmem <= 232448, "shared memory exceeds 227 KB");
}  // namespace pp

__global__ void __launch_bounds__(pp::kThreads, 1)
    fa_prefill_pp_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const FaParams p) {
  using namespace pp;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint64_t* q_full = bars;                   // [1]
  uint64_t* kv_full = bars + 1;              // [kStages]
  uint64_t* kv_empty = kv_full + kStages;    // [kStages]
  uint64_t* s_full = kv_empty + kStages;     // [2] tile A / B
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* pv_done = p_full + 2;            // [2]
  uint64_t* drain = pv_done + 2;             // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int req = p.tile_req[tile];
  const int tok0 = p.tile_tok0[tile];
  const int q_begin = p.cu_q[req];
  const int q_len = p.cu_q[req + 1] - q_begin;
  const int kv_len = p.kv_lens[req];
  const int tpt = kRows / p.G;                       // tokens per 128-row tile
  const int past = kv_len - q_len;
  const int key_end = p.causal ? min(kv_len, past + min(q_len, tok0 + 2 * tpt)) : kv_len;
  const int nb = key_end > 0 ? (key_end + kPBN - 1) / kPBN : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto s_col = [](int t) -> uint32_t { return static_cast<uint32_t>(t) * 64u; };           // S_A | S_B
  auto o_col = [](int t) -> uint32_t { return 128u + static_cast<uint32_t>(t) * 128u; };   // O_A | O_B

  if (warp == 0) {
    if (lane == 0 && nb > 0) {
      mbar_arrive_expect_tx(q_full, 2 * kQBytes);
      for (int t = 0; t < 2; ++t)
        for (int r = 0; r < 2; ++r)
          tma_load_3d(smem + kQ + t * kQBytes + r * (kQBytes / 2), &tmap_q, q_full, r * 64, h * p.G,
                      q_begin + tok0 + t * tpt);
      const int pages = (kv_len + 63) / 64;
      int issued = 0;   // blocks whose loads were issued
      for (int j = 0; j < nb; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) & 1) ^ 1, abort_flag, p.status, kWaitTimeoutNs,
                                       kStatusWaitSite + 17))
          break;
        issued = j + 1;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
        load_kv_half(p, &tmap_k, &tmap_v, &kv_full[s], smem + kK + s * kKVBytes, smem + kV + s * kKVBytes,
                     kKVBytes / 2, req, h, j * kPBN, pages);
      }
      mbar_wait(q_full, 0, nullptr, p.status);
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, nullptr, p.status);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = umma_idesc_bf16_f32(kRows, kPBN);
    constexpr uint32_t idesc_o = umma_idesc_bf16_f32_bmn(kRows, kD);
    bool ok = nb > 0 && warp_wait(q_full, 0, abort_flag, p.status, 14);
    auto issue_s = [&](int t, int j) -> bool {
      const int s = j % kStages;
      if (t == 0 && !warp_wait(&kv_full[s], (j / kStages) & 1, abort_flag, p.status, 15)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(smem + kQ + t * kQBytes);
        const uint32_t ka = smem_u32(smem + kK + s * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(qa + (kk >> 2) * (kQBytes / 2)) + 2 * (kk & 3);
          const uint64_t bdesc = umma_desc_sw128(ka + (kk >> 2) * (kKVBytes / 2)) + 2 * (kk & 3);
          umma_f16_ss(tmem + s_col(t), adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int t, int j) -> bool {
      if (!warp_wait(&p_full[t], j & 1, abort_flag, p.status, 16)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_u32(smem + kP + t * kPBytes);
        const uint32_t va = smem_u32(smem + kV + (j % kStages) * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < kPBN / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(pa) + 2 * kk;
          const uint64_t bdesc = umma_desc_sw128_mn(va + kk * 16 * 128, kKVBytes / 2);
          umma_f16_ss(tmem + o_col(t), adesc, bdesc, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[t]);
        if (t == 1) umma_commit(&kv_empty[j % kStages]);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
    for (int j = 0; j < nb && ok; ++j) {
      if (!issue_pv(0, j)) { ok = false; break; }
      if (j + 1 < nb && !issue_s(0, j + 1)) { ok = false; break; }
      if (!issue_pv(1, j)) { ok = false; break; }
      if (j + 1 < nb && !issue_s(1, j + 1)) { ok = false; break; }
    }
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status);
    }
    __syncwarp();
  } else {
    const int t = warp < 6 ? 0 : 1;                   // tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                  // row within the tile = TMEM lane
    const int tok = tok0 + t * tpt + r / p.G;
    const bool row_ok = tok < q_len;
    const int qpos = past + tok;
    const int lim = p.causal ? min(kv_len, qpos + 1) : kv_len;   // keys [0, lim) are visible
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint8_t* prow = smem + kP + t * kPBytes + r * 128;
    for (int j = 0; j < nb && ok; ++j) {
      if (!warp_wait(&s_full[t], j & 1, abort_flag, p.status, 11)) { ok = false; break; }
      tc_fence_after();
      float s[kPBN];
      {
        uint32_t v[kPBN];
#pragma unroll
        for (int c = 0; c < kPBN; c += 32)
          tmem_ld_32x32b_x32(tmem + lane_addr + s_col(t) + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < kPBN; ++i) s[i] = __uint_as_float(v[i]);
      }
      const int k0 = j * kPBN;
      if (k0 + kPBN > lim) {   // diagonal / last block: mask the invisible keys
#pragma unroll
        for (int i = 0; i < kPBN; ++i) s[i] = (k0 + i < lim) ? s[i] : -INFINITY;
      }
      const float mraw = row_max(s);
      const float mb = mraw == -INFINITY ? -INFINITY : mraw * p.scale_log2;   // log2 units
      // the previous PV of this tile has read P and (for a rescale) finished accumulating O
      if (j > 0 && !warp_wait(&pv_done[t], (j - 1) & 1, abort_flag, p.status, 12)) { ok = false; break; }
      // lazy rescale, warp-uniform (see the one-tile kernel)
      const bool grow = mb > m_run + kRescaleThreshold || (m_run == -INFINITY && mb > -INFINITY);
      if (__any_sync(0xffffffffu, grow)) {
        const bool scale_o = grow && j > 0 && m_run > -INFINITY;
        if (__any_sync(0xffffffffu, scale_o)) {
          tc_fence_after();
          const float f = scale_o ? ex2_ftz(m_run - mb) : 1.f;
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + o_col(t) + c, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
            tmem_st_32x32b_x32(tmem + lane_addr + o_col(t) + c, v);
          }
          tmem_st_wait();
          l_run *= f;
        }
        if (grow) m_run = mb;
      }
      const float msub = m_run == -INFINITY ? 0.f : m_run;
      float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c8 = 0; c8 < kPBN / 8; ++c8) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = ex2_ftz(fmaf(s[c8 * 8 + i], p.scale_log2, -msub));
          ls[i] += e[i];
        }
        uint4 pk;
        pk.x = pack_bf16x2(e[0], e[1]);
        pk.y = pack_bf16x2(e[2], e[3]);
        pk.z = pack_bf16x2(e[4], e[5]);
        pk.w = pack_bf16x2(e[6], e[7]);
        *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) = pk;
      }
      l_run += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    __nv_bfloat16* orow = p.out + static_cast<int64_t>(q_begin + tok) * p.out_stride +
                          static_cast<int64_t>(h * p.G + r % p.G) * p.d_head;
    if (ok && nb > 0 && warp_wait(&pv_done[t], (nb - 1) & 1, abort_flag, p.status, 13)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + o_col(t) + c, v);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (c + i >= p.d_head) break;
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv);
            o.y = pack_bf16x2(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
            o.z = pack_bf16x2(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv);
            o.w = pack_bf16x2(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c + i) = o;
          }
        }
      }
    } else if (nb == 0 && row_ok) {
      for (int c = 0; c < p.d_head; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0u, 0u, 0u, 0u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
            const cuuint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Paged mode: head_dim 128.  Contiguous mode (ragged encoder batches, K/V rows [tokens, hkv, D]):
// head_dim 64..128 in steps of 16, the columns past it loaded as zeros.  G = Hq / Hkv dividing 128,
// no sliding window.
bool attention_prefill_sm100_supported(const AttnPrefillArgs& a) {
  if (a.window > 0 || a.hkv <= 0 || a.hq % a.hkv != 0) return false;
  const bool paged = a.block_table != nullptr;
  if (paged ? a.head_dim != kD : (a.cu_kv == nullptr || a.head_dim < 64 || a.head_dim > kD || a.head_dim % 16 != 0))
    return false;
  if (!paged && ((a.kv_stride * 2) % 16 != 0 || a.kv_stride < static_cast<int64_t>(a.hkv) * a.head_dim)) return false;
  const int G = a.hq / a.hkv;
  return G >= 1 && G <= 16 && kRows % G == 0 && (a.q_stride * 2) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 && (a.out_stride % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
}

cudaError_t attention_prefill_sm100(const AttnPrefillArgs& a, cudaStream_t stream) {
  if (a.num_tiles == 0) return cudaSuccess;
  const bool paged = a.block_table != nullptr;
  if (!attention_prefill_sm100_supported(a) || (paged && a.num_pages <= 0) || (!paged && a.kv_rows <= 0))
    return cudaErrorInvalidValue;
  const int G = a.hq / a.hkv;
  const int D = a.head_dim;
  CUtensorMap tq, tk, tv;
  // Q [tokens, Hq, D]: the tensor spans every row the tile table can address (q rows are
  // never written past the last request; rows past a request's end are masked).  With D < 128
  // the second 64-column box reads zeros past column D.
  {
    const cuuint64_t rows = static_cast<cuuint64_t>(a.q_rows > 0 ? a.q_rows : 1);
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(a.hq), rows};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(a.q_stride) * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(kRows / G)};
    if (!encode(&tq, a.q, 3, dims, strides, box)) return cudaErrorInvalidValue;
  }
  if (paged) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.num_pages) * a.hkv * 64};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
    cuuint32_t box[2] = {64, 64};
    if (!encode(&tk, a.k, 2, dims, strides, box) || !encode(&tv, a.v, 2, dims, strides, box))
      return cudaErrorInvalidValue;
  } else {
    // K / V rows [kv_rows, Hkv, D] of stride kv_stride: one head's 64 consecutive key rows per box
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(a.hkv),
                          static_cast<cuuint64_t>(a.kv_rows)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(a.kv_stride) * 2};
    cuuint32_t box[3] = {64, 1, 64};
    if (!encode(&tk, a.k, 3, dims, strides, box) || !encode(&tv, a.v, 3, dims, strides, box))
      return cudaErrorInvalidValue;
  }
  FaParams p;
  p.block_table = a.block_table;
  p.bt_stride = a.bt_stride;
  p.cu_q = a.cu_q;
  p.kv_lens = a.kv_lens;
  p.tile_req = a.tile_req;
  p.tile_tok0 = a.tile_tok0;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.G = G;
  p.scale_log2 = a.scale * kLog2e;
  p.causal = a.causal;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.num_pages = a.num_pages;
  p.status = a.status;
  p.cu_kv = paged ? nullptr : a.cu_kv;
  p.d_head = D;
  dim3 grid(a.num_tiles, a.hkv);
  if (a.tile_rows == 256) {
    cudaError_t e = ensure_smem_attr<fa_prefill_pp_kernel>(pp::kSmem);
    if (e != cudaSuccess) return e;
    fa_prefill_pp_kernel<<<grid, pp::kThreads, pp::kSmem, stream>>>(tq, tk, tv, p);
  } else {
    cudaError_t e = ensure_smem_attr<fa_prefill_kernel>(FaSmem::kBytes);
    if (e != cudaSuccess) return e;
    fa_prefill_kernel<<<grid, kThreads, FaSmem::kBytes, stream>>>(tq, tk, tv, p);
  }
  return cudaGetLastError();
}

}  // namespace omni
