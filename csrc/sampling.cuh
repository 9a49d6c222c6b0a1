// Device helpers of the token samplers (fused_ops.cu ``sample_kernel`` and the
// vocab-parallel pair in vocab_parallel.cu): a counter-based uniform draw, order-preserving
// float keys, block reductions and vectorised row sweeps.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace omni {
namespace samp {

// SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014) as a counter-based hash.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t ctr) {
  const uint64_t h = splitmix64(seed ^ splitmix64(ctr));
  return (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

template <class Op>
__device__ __forceinline__ float block_reduce(float v, float* sred, Op op, float init) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, d));
  __syncthreads();
  if (lane == 0) sred[warp] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? sred[threadIdx.x] : init;
  if (warp == 0) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, d));
    if (lane == 0) sred[32] = v;
  }
  __syncthreads();
  return sred[32];
}

struct MaxOp { __device__ float operator()(float a, float b) const { return fmaxf(a, b); } };
struct SumOp { __device__ float operator()(float a, float b) const { return a + b; } };

// Row sweeps: 16-byte loads (four per thread in flight) when the row is 16-byte
// aligned, scalar otherwise; f(index, value).
template <class F>
__device__ __forceinline__ void row_for_each(const float* __restrict__ lg, int V, F f) {
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(lg) & 15) == 0) {
    const int n4 = V >> 2;
    const float4* p4 = reinterpret_cast<const float4*>(lg);
#pragma unroll 4
    for (int j = threadIdx.x; j < n4; j += blockDim.x) {
      const float4 v = p4[j];
      f(4 * j, v.x);
      f(4 * j + 1, v.y);
      f(4 * j + 2, v.z);
      f(4 * j + 3, v.w);
    }
    done = n4 << 2;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) f(i, lg[i]);
}

// In-place transform x -> g(index, x) of the row, same access pattern.
template <class G>
__device__ __forceinline__ void row_transform(float* __restrict__ lg, int V, G g) {
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(lg) & 15) == 0) {
    const int n4 = V >> 2;
    float4* p4 = reinterpret_cast<float4*>(lg);
#pragma unroll 4
    for (int j = threadIdx.x; j < n4; j += blockDim.x) {
      float4 v = p4[j];
      v.x = g(4 * j, v.x);
      v.y = g(4 * j + 1, v.y);
      v.z = g(4 * j + 2, v.z);
      v.w = g(4 * j + 3, v.w);
      p4[j] = v;
    }
    done = n4 << 2;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) lg[i] = g(i, lg[i]);
}

__device__ __forceinline__ unsigned long long argmax_key(float x, int i) {
  return (static_cast<unsigned long long>(f2key(x)) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
}


}  // namespace samp
}  // namespace omni
