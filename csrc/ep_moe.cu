// Expert-parallel MoE over NVLink peer memory (sm_100a): the dispatch kernel.
//
// One MoE layer of an EP group is four kernels on each rank, joined by two
// flag waits that sit inside the kernels that need them (no barrier launches):
//
//   ep_dispatch   (this file) every (token, k) row is stored straight into the
//                 owner rank's receive segment of its expert; a CTA reserves its
//                 rows of an expert with one system-scope atomic on the owner's
//                 per-expert counter, so no count exchange precedes the stores.
//                 The last CTA to finish bumps the layer sequence number and
//                 release-stores it into flags[0][rank] of every peer.
//   w13 GEMM      (gemm_sm100.cu, segment mode) waits for flags[0][*] of every
//                 source, then reads the final per-expert counts and runs the
//                 gated grouped GEMM over the received segments.
//   w2 GEMM       (gemm_sm100.cu, segment + combine epilogue) stores every output
//                 row into comb[slot] of the rank the row came from (its tag), and
//                 its last CTA release-stores the sequence number into flags[1][rank]
//                 of every peer; CTA 0 has cleared the per-expert counters first.
//   moe_combine   (fused_ops.cu) waits for flags[1][*] of every owner, then the
//                 top-k weighted sum (+ the next block's residual add + RMSNorm).
//
// Buffer reuse is safe by construction: a source dispatches layer l+1 only after
// its combine of layer l saw every owner's flags[1], which the owners raise after
// their w13 and w2 of layer l finished reading recv_x / recv_tag and after the
// counters were cleared; an owner overwrites comb of a source only after that
// source's flags[0] of the next layer, raised after its combine read comb.
// Every wait is bounded (%globaltimer); one that runs out records status 2.
// No TMA touches peer memory: peers are reached with plain stores and atomics.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "omni_kernels.h"
#include "sm100.cuh"

namespace omni {
namespace {

constexpr int kPairsPerCta = 32;    // (token, k) rows per CTA
constexpr int kDispatchThreads = 256;
constexpr int kMaxExperts = 512;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <class T>
__device__ __forceinline__ T* region(const EpDispatchArgs& a, int rank, int64_t off) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(a.peer_base[rank]) + off);
}

// Grid: ceil(tokens * topk / kPairsPerCta) CTAs (at least one, which then only signals).
__global__ void __launch_bounds__(kDispatchThreads) ep_dispatch_kernel(EpDispatchArgs a) {
  __shared__ int s_cnt[kMaxExperts];   // rows of each expert in this CTA's chunk
  __shared__ int s_base[kMaxExperts];  // first reserved row of each expert on its owner
  __shared__ int s_e[kPairsPerCta];
  __shared__ int s_lpos[kPairsPerCta];
  const int n = a.tokens * a.topk;
  const int i0 = blockIdx.x * kPairsPerCta;
  const int np = max(0, min(kPairsPerCta, n - i0));
  for (int e = threadIdx.x; e < a.experts; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  if (threadIdx.x < np) {
    int e = a.topk_ids[i0 + threadIdx.x];
    e = e < 0 ? 0 : (e >= a.experts ? a.experts - 1 : e);
    s_e[threadIdx.x] = e;
    s_lpos[threadIdx.x] = atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  // one system-scope reservation per (CTA, expert) on the expert's owner
  for (int e = threadIdx.x; e < a.experts; e += blockDim.x) {
    const int c = s_cnt[e];
    if (c > 0) {
      const int d = e / a.local_experts;
      int* cur = region<int>(a, d, a.off_cursor) + (e - d * a.local_experts);
      s_base[e] = atomicAdd_system(cur, c);
    }
  }
  __syncthreads();
  // one warp per row: 16-byte vectors, every load of the row in flight before the stores
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = a.hidden >> 3;
  for (int j = warp; j < np; j += kDispatchThreads / 32) {
    const int e = s_e[j];
    const int d = e / a.local_experts;
    const int pos = s_base[e] + s_lpos[j];
    if (pos >= a.seg_cap) {  // cannot happen with seg_cap = world * max_tokens; never write past the segment
      if (lane == 0) record_status(a.status, kStatusBounds);
      continue;
    }
    const int64_t row = static_cast<int64_t>(e - d * a.local_experts) * a.seg_cap + pos;
    const int slot = i0 + j;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) +
                                                      static_cast<int64_t>(slot / a.topk) * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(region<__nv_bfloat16>(a, d, a.off_recv_x) + row * a.hidden);
    for (int v0 = lane; v0 < nvec; v0 += 32 * 8) {
      uint4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (v0 + 32 * u < nvec) buf[u] = __ldg(src + v0 + 32 * u);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (v0 + 32 * u < nvec) dst[v0 + 32 * u] = buf[u];
    }
    if (lane == 0) {
      int2* tag = reinterpret_cast<int2*>(region<int>(a, d, a.off_recv_tag)) + row;
      *tag = make_int2(a.rank, slot);
    }
  }
  // The last CTA to finish publishes the layer: every CTA's stores are fenced (system scope)
  // before its arrival, so they precede the release stores of the flags.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(a.arrive, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      *a.arrive = 0;
      __threadfence_system();
      const uint32_t seq = *a.seq + 1u;
      *a.seq = seq;
      for (int d = 0; d < a.world; ++d) st_release_sys(region<uint32_t>(a, d, a.off_flags) + a.rank, seq);
    }
  }
}

}  // namespace

cudaError_t ep_dispatch(const EpDispatchArgs& a, cudaStream_t stream) {
  if (a.world > 32 || a.world < 1 || a.experts > kMaxExperts || a.experts % a.world != 0 || a.hidden % 8 != 0 ||
      a.local_experts * a.world != a.experts || a.seg_cap <= 0)
    return cudaErrorInvalidValue;
  const int n = a.tokens * a.topk;
  const int grid = n > 0 ? (n + kPairsPerCta - 1) / kPairsPerCta : 1;
  ep_dispatch_kernel<<<grid, kDispatchThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace omni
