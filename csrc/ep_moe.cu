// Expert-parallel MoE exchange over NVLink peer memory (sm_100a).
//
// Every rank of an EP group owns experts [rank * El, (rank + 1) * El) and one
// symmetric buffer (same layout on every rank, peers' copies mapped through
// CUDA IPC):
//
//   counts   int32 [world, E]        row s = per-expert token counts of rank s
//   flags    uint32 [3, world]       phase (counts / dispatch / combine) x source rank
//   recv_x   bf16  [cap_rows, H]     rows routed to this rank, expert-major:
//                                    (local expert, source rank, source order)
//   recv_meta int32 [cap_rows, 2]    (source rank, source slot = token * topk + k)
//   comb     bf16  [max_slots, H]    expert outputs returned to this rank, by slot
//
// One MoE layer = four launches plus the two grouped GEMMs on recv_x:
//   ep_counts     histogram of this rank's top-k ids, written into every peer's
//                 counts row; wait for all rows; every rank derives the same
//                 offsets: where its (expert) rows start on the destination and
//                 the group offsets of its own local experts.
//   ep_dispatch   each (token, k) row is stored straight into the destination
//                 rank's recv_x at its expert-major position (the permutation
//                 of a local MoE and the all-to-all in one pass), with its
//                 (source, slot) tag.
//   ep_signal     release-store this rank's phase flag into every peer, then
//                 wait (acquire) for every peer's flag: the rows are in place.
//   ... grouped GEMMs (w13 gated, w2) over recv_x[:rows] ...
//   ep_combine    each expert-output row is stored back into its source rank's
//                 comb[slot]; ep_signal again; the source rank then does the
//                 top-k weighted sum (+ shared expert) with moe_combine.
//
// The epoch of a layer is a device counter bumped by ep_counts, so the same
// launches can be captured once in a CUDA graph and replayed.  Every wait is
// bounded (%globaltimer); a wait that runs out writes status 2 and returns.
// No TMA here: peer memory is only touched by plain vector loads and stores.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "omni_kernels.h"
#include "sm100.cuh"

namespace omni {
namespace {

constexpr int kPhaseCounts = 0, kPhaseDispatch = 1, kPhaseCombine = 2;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <class T>
__device__ __forceinline__ T* region(const EpArgs& a, int rank, int64_t off) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(a.peer_base[rank]) + off);
}

// Waits until flags[phase][s] == epoch for every source s (thread s waits on source s).
__device__ void wait_flags(const EpArgs& a, int phase, uint32_t epoch) {
  const int s = threadIdx.x;
  if (s < a.world) {
    const uint32_t* f = region<uint32_t>(a, a.rank, a.off_flags) + phase * a.world + s;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) != epoch) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        if (a.status) atomicExch(a.status, kStatusPeerTimeout);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();  // every thread's later reads of peer-written data follow the acquire
}

__device__ void signal_peers(const EpArgs& a, int phase, uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  const int d = threadIdx.x;
  if (d < a.world) st_release_sys(region<uint32_t>(a, d, a.off_flags) + phase * a.world + a.rank, epoch);
}

// One CTA.  counts -> peers, wait, derive offsets.
__global__ void __launch_bounds__(1024) ep_counts_kernel(EpArgs a) {
  extern __shared__ int sm[];
  int* hist = sm;                    // [E]
  int* tot = sm + a.experts;         // [E] totals over sources
  __shared__ uint32_t s_epoch;
  for (int e = threadIdx.x; e < a.experts; e += blockDim.x) hist[e] = 0;
  if (threadIdx.x == 0) s_epoch = ++(*a.epoch);
  __syncthreads();
  const int n = a.tokens * a.topk;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int e = a.topk_ids[i];
    e = e < 0 ? 0 : (e >= a.experts ? a.experts - 1 : e);
    atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  // my row into every peer's counts[rank]
  for (int d = 0; d < a.world; ++d) {
    int* dst = region<int>(a, d, a.off_counts) + a.rank * a.experts;
    for (int e = threadIdx.x; e < a.experts; e += blockDim.x) dst[e] = hist[e];
  }
  signal_peers(a, kPhaseCounts, epoch);
  wait_flags(a, kPhaseCounts, epoch);
  const int* cnt = region<int>(a, a.rank, a.off_counts);
  const int El = a.local_experts;
  for (int e = threadIdx.x; e < a.experts; e += blockDim.x) {
    int t = 0;
    for (int s = 0; s < a.world; ++s) t += cnt[s * a.experts + e];
    tot[e] = t;
  }
  __syncthreads();
  // start of my rows of expert e on its owner d: sum of totals of d's earlier experts + earlier sources of e
  for (int e = threadIdx.x; e < a.experts; e += blockDim.x) {
    const int d0 = (e / El) * El;
    int base = 0;
    for (int e2 = d0; e2 < e; ++e2) base += tot[e2];
    for (int s = 0; s < a.rank; ++s) base += cnt[s * a.experts + e];
    a.cursor[e] = base;
  }
  if (threadIdx.x == 0) {
    int acc = 0;
    const int e0 = a.rank * El;
    for (int j = 0; j < El; ++j) {
      a.local_offsets[j] = acc;
      acc += tot[e0 + j];
    }
    a.local_offsets[El] = acc;
    *a.total_rows = acc;
    if (acc > a.cap_rows && a.status) atomicExch(a.status, kStatusBounds);
  }
}

// One warp per (token, k): copy the row to its destination, tag it.
__global__ void ep_dispatch_kernel(EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int n = a.tokens * a.topk;
  const int nvec = a.hidden >> 3;
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += gridDim.x * warps) {
    int e = a.topk_ids[i];
    e = e < 0 ? 0 : (e >= a.experts ? a.experts - 1 : e);
    const int d = e / a.local_experts;
    int pos = 0;
    if (lane == 0) pos = atomicAdd(&a.cursor[e], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (pos >= a.cap_rows) continue;  // counted as a bounds error by ep_counts
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) +
                                                      static_cast<int64_t>(i / a.topk) * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(region<__nv_bfloat16>(a, d, a.off_recv_x) + static_cast<int64_t>(pos) * a.hidden);
    for (int v = lane; v < nvec; v += 32) dst[v] = src[v];
    if (lane == 0) {
      int* meta = region<int>(a, d, a.off_recv_meta) + 2 * static_cast<int64_t>(pos);
      meta[0] = a.rank;
      meta[1] = i;
    }
  }
  __threadfence_system();
}

// One CTA: publish this rank's flag for `phase`, wait for everyone's.
__global__ void ep_signal_kernel(EpArgs a, int phase) {
  const uint32_t epoch = *a.epoch;
  signal_peers(a, phase, epoch);
  wait_flags(a, phase, epoch);
}

// One warp per received row: expert output back to its source slot.
__global__ void ep_combine_kernel(EpArgs a, const void* y, int64_t y_stride) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int rows = *a.total_rows < a.cap_rows ? *a.total_rows : a.cap_rows;
  const int nvec = a.hidden >> 3;
  const int* meta = region<int>(a, a.rank, a.off_recv_meta);
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps) {
    const int s = meta[2 * r], slot = meta[2 * r + 1];
    if (s < 0 || s >= a.world || slot < 0 || slot >= a.max_slots) continue;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(y) + r * y_stride);
    uint4* dst = reinterpret_cast<uint4*>(region<__nv_bfloat16>(a, s, a.off_comb) + static_cast<int64_t>(slot) * a.hidden);
    for (int v = lane; v < nvec; v += 32) dst[v] = src[v];
  }
  __threadfence_system();
}

int grid_rows(int n) {
  int g = (n + 7) / 8;
  if (g > 148 * 4) g = 148 * 4;
  return g < 1 ? 1 : g;
}

}  // namespace

cudaError_t ep_counts(const EpArgs& a, cudaStream_t stream) {
  if (a.world > 32 || a.world < 1 || a.experts % a.world != 0 || a.hidden % 8 != 0) return cudaErrorInvalidValue;
  const int smem = 2 * a.experts * static_cast<int>(sizeof(int));
  ep_counts_kernel<<<1, 1024, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t ep_dispatch(const EpArgs& a, cudaStream_t stream) {
  const int n = a.tokens * a.topk;
  if (n > 0) ep_dispatch_kernel<<<grid_rows(n), 256, 0, stream>>>(a);
  ep_signal_kernel<<<1, 32, 0, stream>>>(a, kPhaseDispatch);
  return cudaGetLastError();
}

cudaError_t ep_combine(const EpArgs& a, const void* y, int64_t y_stride, cudaStream_t stream) {
  ep_combine_kernel<<<grid_rows(a.cap_rows), 256, 0, stream>>>(a, y, y_stride);
  ep_signal_kernel<<<1, 32, 0, stream>>>(a, kPhaseCombine);
  return cudaGetLastError();
}

}  // namespace omni
