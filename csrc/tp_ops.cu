// Tensor-parallel reduce point over NVLink peer memory (sm_100a):
// reduce-scatter of partial sums + residual add + RMSNorm + all-gather, one launch.
//
// Every rank of a TP group holds one symmetric buffer (same layout everywhere,
// the peers' copies mapped through CUDA IPC):
//
//   part   bf16 [world][max_tokens][H]   partial sums: slot s holds rank s's
//                                        contribution to the rows this rank owns
//   gath   bf16 [max_tokens][H]          normalised rows of every token (all-gathered)
//   gres   bf16 [max_tokens][H]          residual rows of every token (optional gather)
//   flags  u32  [2][world]               phase A (partials written) / phase B (rows
//                                        gathered) x source rank
//
// Token r is owned by rank r / rows_per.  The producer of the partials (a
// row-parallel GEMM epilogue or the tensor-parallel MoE combine) already stored
// row r into part[rank] of its owner, so the reduce-scatter's transfer happened
// inside the producing kernel, tile by tile.  This kernel then:
//   1. (CTA 0) release-stores phase A = seq + 1 into every peer: my partials are in place;
//   2. waits (acquire, bounded) for phase A from every rank;
//   3. per owned row: sum the world partials in fp32, add the residual (the bf16
//      residual stream is updated in place), RMSNorm with the next block's weight;
//   4. stores the normalised row (and optionally the residual row) into every
//      rank's gath / gres;
//   5. the last CTA to finish release-stores phase B = seq + 1 into every peer
//      and advances seq.
// Two variants serve attention TP combined with expert-parallel MoE: ``gather_local``
// keeps the normalised owned rows on this rank (they feed the EP dispatch, which
// moves each token once), and ``single_src`` takes the owned rows already reduced
// in part[rank] (the EP combine's output) instead of summing world partials.
// The consumer (the next GEMM, see GemmArgs::wait_flags, or tp_wait) waits for
// phase B == seq from every rank before it reads gath.  seq lives on the
// device, so the whole sequence is captured in a CUDA graph and replayed.
//
// Reference counterparts: the all-reduce after o_proj / MoE with the fused
// residual + RMSNorm (sglang_omni/vendor/sglang/layers.py:92-137,
// sglang_omni/models/qwen3_omni/thinker.py:447-453), never enabled there.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "omni_kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"

namespace omni {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

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

__device__ __forceinline__ uint32_t* flag_at(const TpReduceArgs& a, int rank, int phase, int src) {
  return reinterpret_cast<uint32_t*>(a.peer_flags[rank]) + phase * a.world + src;
}

// Thread s < world waits for flags[phase][s] == target on this rank.
__device__ void wait_phase(const TpReduceArgs& a, int phase, uint32_t target) {
  const int s = threadIdx.x;
  if (s < a.world) {
    const uint32_t* f = flag_at(a, a.rank, phase, s);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) != target) {
      if (globaltimer_ns() - t0 > static_cast<uint64_t>(a.timeout_ns)) {
        if (a.status) atomicExch(a.status, kStatusPeerTimeout);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();
}

template <int VPT>
__global__ void __launch_bounds__(256) tp_reduce_norm_kernel(TpReduceArgs a) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  __shared__ uint32_t s_target;
  __shared__ int s_last;
  __shared__ float red[8];
  if (threadIdx.x == 0) s_target = *reinterpret_cast<const volatile uint32_t*>(a.seq) + 1u;
  __syncthreads();
  const uint32_t target = s_target;
  if (blockIdx.x == 0) {
    __threadfence_system();
    if (threadIdx.x < a.world) st_release_sys(flag_at(a, threadIdx.x, 0, a.rank), target);
  }
  wait_phase(a, 0, target);

  const int row0 = a.rank * a.rows_per;
  const int owned = max(0, min(a.rows_per, a.tokens - row0));
  const int nvec = a.hidden >> 3;
  for (int lr = blockIdx.x; lr < owned; lr += gridDim.x) {
    const int row = row0 + lr;
    float vals[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + 256 * i;
      if (v >= nvec) continue;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      const uint4* part = reinterpret_cast<const uint4*>(a.peer_part[a.rank]);
      const int s0 = a.single_src ? a.rank : 0, s1 = a.single_src ? a.rank + 1 : a.world;
      for (int s = s0; s < s1; ++s) {
        float f[8];
        unpack8(__ldcg(part + (static_cast<int64_t>(s) * a.max_tokens + row) * nvec + v), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += f[j];
      }
      uint4* rr = reinterpret_cast<uint4*>(a.residual) + static_cast<int64_t>(row) * nvec + v;
      float r[8];
      // the summed partials are rounded to bf16 (the value an all-reduce would produce)
      // before the residual add, as the unsharded model rounds its block output
      unpack8(pack8(acc), acc);
      unpack8(*rr, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += r[j];
      const uint4 sres = pack8(acc);
      *rr = sres;
      unpack8(sres, vals[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
      if (a.peer_gres != nullptr)
        for (int d = 0; d < a.world; ++d)
          reinterpret_cast<uint4*>(a.peer_gres[d])[static_cast<int64_t>(row) * nvec + v] = sres;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    __syncthreads();  // red is reused by the next row
    const float rstd = rsqrtf(tot / static_cast<float>(a.hidden) + a.eps);
    const uint4* wr = static_cast<const uint4*>(a.norm_w);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + 256 * i;
      if (v >= nvec) continue;
      float wf[8], o[8];
      unpack8(wr[v], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __bfloat162float(__float2bfloat16(vals[i][j] * rstd)) * wf[j];
      const uint4 ov = pack8(o);
      const int d0 = a.gather_local ? a.rank : 0, d1 = a.gather_local ? a.rank + 1 : a.world;
      for (int d = d0; d < d1; ++d)
        reinterpret_cast<uint4*>(a.peer_gath[d])[static_cast<int64_t>(row) * nvec + v] = ov;
    }
  }

  // the last CTA publishes phase B once every CTA's stores are out
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(a.counter, 1) + 1;
    s_last = done == static_cast<int>(gridDim.x);
    if (s_last) *a.counter = 0;
  }
  __syncthreads();
  if (s_last) {
    __threadfence_system();
    if (threadIdx.x < a.world) st_release_sys(flag_at(a, threadIdx.x, 1, a.rank), target);
    if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(a.seq) = target;
  }
}

// One CTA: wait until phase B == seq from every rank (for consumers that are not our GEMMs).
__global__ void tp_wait_kernel(TpReduceArgs a) {
  const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(a.seq);
  wait_phase(a, 1, target);
}

}  // namespace

cudaError_t tp_reduce_norm(const TpReduceArgs& a, cudaStream_t stream) {
  if (a.world < 1 || a.world > 32 || a.hidden % 8 != 0 || a.hidden / 8 > 4 * 256 || a.rows_per < 1 ||
      a.tokens > a.max_tokens)
    return cudaErrorInvalidValue;
  const int owned = a.tokens - a.rank * a.rows_per;
  int grid = owned < 1 ? 1 : (owned > a.rows_per ? a.rows_per : owned);
  if (grid > 148 * 8) grid = 148 * 8;
  const int nvec = a.hidden / 8;
  if (nvec <= 256) tp_reduce_norm_kernel<1><<<grid, 256, 0, stream>>>(a);
  else if (nvec <= 512) tp_reduce_norm_kernel<2><<<grid, 256, 0, stream>>>(a);
  else tp_reduce_norm_kernel<4><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t tp_wait(const TpReduceArgs& a, cudaStream_t stream) {
  tp_wait_kernel<<<1, 32, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace omni
