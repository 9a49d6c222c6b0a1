// RMSNorm (optionally fused with the residual add) and LayerNorm.
//
// One warp per row, 16-byte vector loads, fp32 statistics.  The fused form
// computes r = x + r, writes r back, then y = w * rmsnorm(r): the
// "fused_add_rmsnorm" contract used before every attention/MLP block
// (sglang_omni/vendor/sglang/layers.py:45-87).
#include <cuda_bf16.h>

#include "omni_kernels.h"
#include "pdl.cuh"

namespace omni {
namespace {

struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void unpack(const bf16x8& p, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p.v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bf16x8 pack(const float (&f)[8]) {
  bf16x8 p;
#pragma unroll
  for (int i = 0; i < 4; ++i) p.v[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return p;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

// hidden % 8 == 0; rows handled one per warp.
template <int MAXV>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ res, int rows, int hidden,
                               int64_t ld_x, int64_t ld_y, float eps) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = hidden >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + row * ld_x);
  bf16x8* rr = res ? reinterpret_cast<bf16x8*>(res + static_cast<int64_t>(row) * hidden) : nullptr;
  float vals[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      bf16x8 p = xr[v];
      unpack(p, vals[i]);
      if (rr) {
        float r[8];
        unpack(rr[v], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[i][j] += r[j];
        // the residual stream is kept in bf16, as the reference's fused add does
        bf16x8 s = pack(vals[i]);
        rr[v] = s;
        unpack(s, vals[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / static_cast<float>(hidden) + eps);
  const bf16x8* wr = reinterpret_cast<const bf16x8*>(w);
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + row * ld_y);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      float wf[8];
      unpack(wr[v], wf);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // HF order: normalise in fp32, round to bf16, then scale by the weight.
        const float n = __bfloat162float(__float2bfloat16(vals[i][j] * rstd));
        o[j] = n * wf[j];
      }
      yr[v] = pack(o);
    }
  }
}

__global__ void layernorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                 const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y, int rows,
                                 int hidden, float eps) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = hidden >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + static_cast<int64_t>(row) * hidden);
  float s = 0.f, ss = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    float f[8];
    unpack(xr[v], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s += f[j];
      ss += f[j] * f[j];
    }
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  const float mean = s / hidden;
  const float var = fmaxf(ss / hidden - mean * mean, 0.f);
  const float rstd = rsqrtf(var + eps);
  const bf16x8* wr = reinterpret_cast<const bf16x8*>(w);
  const bf16x8* br = reinterpret_cast<const bf16x8*>(b);
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + static_cast<int64_t>(row) * hidden);
  for (int v = lane; v < nvec; v += 32) {
    float f[8], wf[8], bf[8], o[8];
    unpack(xr[v], f);
    unpack(wr[v], wf);
    if (br) unpack(br[v], bf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (f[j] - mean) * rstd * wf[j] + (br ? bf[j] : 0.f);
    yr[v] = pack(o);
  }
}

}  // namespace

// One CTA per row (few rows: decode batches); each thread owns VPT 16-byte vectors.
template <int VPT>
__global__ void rmsnorm_row_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ res, int hidden,
                                   int64_t ld_x, int64_t ld_y, float eps) {
  grid_dep_launch();  // a dependent GEMM may start its prologue now
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = hidden >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + row * ld_x);
  bf16x8* rr = res ? reinterpret_cast<bf16x8*>(res + static_cast<int64_t>(row) * hidden) : nullptr;
  float vals[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + blockDim.x * i;
    if (v < nvec) {
      unpack(xr[v], vals[i]);
      if (rr) {
        float r[8];
        unpack(rr[v], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[i][j] += r[j];
        bf16x8 s = pack(vals[i]);
        rr[v] = s;
        unpack(s, vals[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / static_cast<float>(hidden) + eps);
  const bf16x8* wr = reinterpret_cast<const bf16x8*>(w);
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + row * ld_y);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + blockDim.x * i;
    if (v < nvec) {
      float wf[8], o[8];
      unpack(wr[v], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __bfloat162float(__float2bfloat16(vals[i][j] * rstd)) * wf[j];
      yr[v] = pack(o);
    }
  }
}

cudaError_t rmsnorm_bf16(const void* x, const void* w, void* y, void* residual, int rows, int hidden, int64_t ld_x,
                         int64_t ld_y, float eps, cudaStream_t stream) {
  if (hidden % 8 != 0 || hidden > 8 * 32 * 32) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (rows <= 512) {  // few rows: a CTA per row keeps many SMs busy (a warp per row would use rows / 8 SMs)
    const int nvec = hidden / 8;
    int threads = nvec <= 256 ? ((nvec + 31) / 32) * 32 : 256;
    const int vpt = (nvec + threads - 1) / threads;
    auto xp = static_cast<const __nv_bfloat16*>(x);
    auto wp = static_cast<const __nv_bfloat16*>(w);
    auto yp = static_cast<__nv_bfloat16*>(y);
    auto rp = static_cast<__nv_bfloat16*>(residual);
    if (vpt <= 1) rmsnorm_row_kernel<1><<<rows, threads, 0, stream>>>(xp, wp, yp, rp, hidden, ld_x, ld_y, eps);
    else if (vpt <= 2) rmsnorm_row_kernel<2><<<rows, threads, 0, stream>>>(xp, wp, yp, rp, hidden, ld_x, ld_y, eps);
    else if (vpt <= 4) rmsnorm_row_kernel<4><<<rows, threads, 0, stream>>>(xp, wp, yp, rp, hidden, ld_x, ld_y, eps);
    else rmsnorm_row_kernel<8><<<rows, threads, 0, stream>>>(xp, wp, yp, rp, hidden, ld_x, ld_y, eps);
    return cudaGetLastError();
  }
  const int threads = 256;
  const int grid = (rows + 7) / 8;
  auto xp = static_cast<const __nv_bfloat16*>(x);
  auto wp = static_cast<const __nv_bfloat16*>(w);
  auto yp = static_cast<__nv_bfloat16*>(y);
  auto rp = static_cast<__nv_bfloat16*>(residual);
  const int nv = (hidden / 8 + 31) / 32;
  if (nv <= 1) rmsnorm_kernel<1><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  else if (nv <= 2) rmsnorm_kernel<2><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  else if (nv <= 4) rmsnorm_kernel<4><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  else if (nv <= 8) rmsnorm_kernel<8><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  else if (nv <= 16) rmsnorm_kernel<16><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  else rmsnorm_kernel<32><<<grid, threads, 0, stream>>>(xp, wp, yp, rp, rows, hidden, ld_x, ld_y, eps);
  return cudaGetLastError();
}

cudaError_t layernorm_bf16(const void* x, const void* w, const void* b, void* y, int rows, int hidden, float eps,
                           cudaStream_t stream) {
  if (hidden % 8 != 0) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  layernorm_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                       static_cast<const __nv_bfloat16*>(w),
                                                       static_cast<const __nv_bfloat16*>(b),
                                                       static_cast<__nv_bfloat16*>(y), rows, hidden, eps);
  return cudaGetLastError();
}

}  // namespace omni
