// Memory-bound pieces of the audio front-end and the causal-conv vocoders,
// all channels-last ([rows, C] with C contiguous) so the convolutions run as
// tcgen05 GEMMs on the im2col rows:
//   * snake_beta      y = x + 1/(exp(b)+1e-9) * sin(x * exp(a))^2     (SnakeBeta)
//   * snake           y = x + 1/(a+1e-9) * sin(a x)^2                 (Snake1d, DAC)
//   * conv1d_im2col   causal / padded dilated conv1d -> [T_out, K*C] rows
//   * conv_transpose_ola  overlap-add of the [T, 2s*C] GEMM rows of a
//                     kernel-2s stride-s transposed conv, + bias, causal trim
//   * dwconv1d_causal depthwise causal conv (ConvNeXt), kernel <= 16
//   * conv2d_im2col   3x3 / stride / pad 2-D conv rows [(n, ho, wo), (kh, kw, c)]
//
// Reference counterparts: transformers Qwen3OmniMoeCode2Wav (SnakeBeta,
// CausalConvNet, CausalTransConvNet, ConvNeXtBlock) used by
// sglang_omni/models/qwen3_omni/components/code2wav_executor.py, the DAC
// decoder of sglang_omni/models/fishaudio_s2_pro/fish_speech/models/dac/modded_dac.py,
// and the Conv2d front-end of the Qwen3-Omni audio tower.
#include <cuda_bf16.h>
#include <stdint.h>

#include "omni_kernels.h"

namespace omni {
namespace {

__global__ void snake_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ alpha,
                             const float* __restrict__ beta, __nv_bfloat16* __restrict__ y, int64_t n, int C,
                             int log_scale) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const float v = __bfloat162float(x[i]);
    float a = alpha[c];
    float b = beta ? beta[c] : a;
    if (log_scale) {
      a = __expf(a);
      b = __expf(b);
    }
    const float s = sinf(v * a);
    y[i] = __float2bfloat16(v + s * s / (b + 1e-9f));
  }
}

// out[b, t, k*C + c] = x[b, t*stride + k*dil - pad_left, c] (zero outside [0, T_in))
__global__ void conv1d_im2col_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                                     int B, int T_in, int T_out, int C, int K, int dil, int stride, int pad_left,
                                     int C_out_stride) {
  const int64_t rows = static_cast<int64_t>(B) * T_out;
  const int vec = C / 8;  // 16-byte chunks per tap
  const int64_t total = rows * K * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vec);
    const int64_t rk = i / vec;
    const int k = static_cast<int>(rk % K);
    const int64_t row = rk / K;
    const int t = static_cast<int>(row % T_out);
    const int b = static_cast<int>(row / T_out);
    const int src_t = t * stride + k * dil - pad_left;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (src_t >= 0 && src_t < T_in)
      val = reinterpret_cast<const uint4*>(x + (static_cast<int64_t>(b) * T_in + src_t) * C)[v];
    reinterpret_cast<uint4*>(out + row * C_out_stride + static_cast<int64_t>(k) * C)[v] = val;
  }
}

// y: [B, T, 2s, C] rows of the GEMM x @ W(c_in -> (j, c_out)); out: [B, (T-1)*s, C]
// out[u] = y[u/s + 1, u%s] + y[u/s, u%s + s] + bias
// Output sample u is sample f = u + shift of the full transposed conv
// (length (T + 1) * s): full[f] = y[f / s][f % s] + y[f / s - 1][f % s + s].
__global__ void conv_transpose_ola_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ bias,
                                          __nv_bfloat16* __restrict__ out, int B, int T, int s, int C, int T_out,
                                          int shift) {
  const int64_t total = static_cast<int64_t>(B) * T_out * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const int64_t bu = i / C;
    const int u = static_cast<int>(bu % T_out);
    const int b = static_cast<int>(bu / T_out);
    const int f = u + shift;
    const int t = f / s, j = f - t * s;
    const int64_t base = static_cast<int64_t>(b) * T;
    float v = bias ? __bfloat162float(bias[c]) : 0.f;
    if (t < T) v += __bfloat162float(y[((base + t) * (2 * s) + j) * C + c]);
    if (t >= 1 && t - 1 < T) v += __bfloat162float(y[((base + t - 1) * (2 * s) + j + s) * C + c]);
    out[i] = __float2bfloat16(v);
  }
}

// out[b, t, c] = bias[c] + sum_k w[c, k] * x[b, t + k - (K-1), c]
__global__ void dwconv1d_causal_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                       const float* __restrict__ bias, __nv_bfloat16* __restrict__ out, int B, int T,
                                       int C, int K) {
  const int64_t total = static_cast<int64_t>(B) * T * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const int64_t bt = i / C;
    const int t = static_cast<int>(bt % T);
    const int64_t b = bt / T;
    float acc = bias ? bias[c] : 0.f;
    for (int k = 0; k < K; ++k) {
      const int st = t + k - (K - 1);
      if (st >= 0) acc += w[c * K + k] * __bfloat162float(x[(b * T + st) * C + c]);
    }
    out[i] = __float2bfloat16(acc);
  }
}

// x: [N, H, W, C] channels-last; out: [N*Ho*Wo, kh*kw*C] in (kh, kw, c) order
__global__ void conv2d_im2col_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out, int N,
                                     int H, int W, int C, int Ho, int Wo, int kh, int kw, int stride, int pad,
                                     int K_stride) {
  const int64_t rows = static_cast<int64_t>(N) * Ho * Wo;
  const int64_t total = rows * kh * kw * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    int64_t r = i / C;
    const int kx = static_cast<int>(r % kw);
    r /= kw;
    const int ky = static_cast<int>(r % kh);
    const int64_t row = r / kh;
    const int wo = static_cast<int>(row % Wo);
    const int ho = static_cast<int>((row / Wo) % Ho);
    const int n = static_cast<int>(row / (static_cast<int64_t>(Wo) * Ho));
    const int hi = ho * stride + ky - pad, wi = wo * stride + kx - pad;
    __nv_bfloat16 v = __float2bfloat16(0.f);
    if (hi >= 0 && hi < H && wi >= 0 && wi < W) v = x[((static_cast<int64_t>(n) * H + hi) * W + wi) * C + c];
    out[row * K_stride + (static_cast<int64_t>(ky) * kw + kx) * C + c] = v;
  }
}

// The same layout when C % 8 == 0 and rows are 16-byte aligned: one warp per (output row,
// tap) copies the tap's C channels as 16-byte vectors (or zeros outside the input), so reads
// and writes are contiguous 16 * C-byte runs and the index math is paid once per warp.
__global__ void __launch_bounds__(256) conv2d_im2col_vec8_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 __nv_bfloat16* __restrict__ out, int N, int H, int W,
                                                                 int C, int Ho, int Wo, int kh, int kw, int stride,
                                                                 int pad, int K_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t items = static_cast<int64_t>(N) * Ho * Wo * kh * kw;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int nv = C >> 3;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); it < items;
       it += warps) {
    const int tap = static_cast<int>(it % (kh * kw));
    const int64_t row = it / (kh * kw);
    const int ky = tap / kw, kx = tap % kw;
    const int wo = static_cast<int>(row % Wo);
    const int ho = static_cast<int>((row / Wo) % Ho);
    const int n = static_cast<int>(row / (static_cast<int64_t>(Wo) * Ho));
    const int hi = ho * stride + ky - pad, wi = wo * stride + kx - pad;
    uint4* dst = reinterpret_cast<uint4*>(out + row * K_stride + static_cast<int64_t>(tap) * C);
    if (hi >= 0 && hi < H && wi >= 0 && wi < W) {
      const uint4* src = reinterpret_cast<const uint4*>(x + ((static_cast<int64_t>(n) * H + hi) * W + wi) * C);
      for (int v = lane; v < nv; v += 32) dst[v] = __ldg(src + v);
    } else {
      for (int v = lane; v < nv; v += 32) dst[v] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

int grid_for(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t snake(const void* x, const float* alpha, const float* beta, void* y, int64_t n, int C, int log_scale,
                  cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  snake_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), alpha, beta,
                                                static_cast<__nv_bfloat16*>(y), n, C, log_scale);
  return cudaGetLastError();
}

cudaError_t conv1d_im2col(const void* x, void* out, int B, int T_in, int T_out, int C, int K, int dil, int stride,
                          int pad_left, int out_row_stride, cudaStream_t stream) {
  if (C % 8 != 0) return cudaErrorInvalidValue;
  const int64_t n = static_cast<int64_t>(B) * T_out * K * (C / 8);
  if (n == 0) return cudaSuccess;
  conv1d_im2col_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<__nv_bfloat16*>(out), B, T_in, T_out, C, K, dil,
                                                        stride, pad_left, out_row_stride);
  return cudaGetLastError();
}

cudaError_t conv_transpose_ola(const void* y, const void* bias, void* out, int B, int T, int s, int C, int T_out,
                               int shift, cudaStream_t stream) {
  if (shift < 0 || T_out + shift > (T + 1) * s) return cudaErrorInvalidValue;
  const int64_t n = static_cast<int64_t>(B) * T_out * C;
  if (n <= 0) return cudaSuccess;
  conv_transpose_ola_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(y),
                                                             static_cast<const __nv_bfloat16*>(bias),
                                                             static_cast<__nv_bfloat16*>(out), B, T, s, C, T_out, shift);
  return cudaGetLastError();
}

cudaError_t dwconv1d_causal(const void* x, const float* w, const float* bias, void* out, int B, int T, int C, int K,
                            cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(B) * T * C;
  if (n == 0) return cudaSuccess;
  dwconv1d_causal_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), w, bias,
                                                          static_cast<__nv_bfloat16*>(out), B, T, C, K);
  return cudaGetLastError();
}

cudaError_t conv2d_im2col(const void* x, void* out, int N, int H, int W, int C, int Ho, int Wo, int kh, int kw,
                          int stride, int pad, int K_stride, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(N) * Ho * Wo * kh * kw * C;
  if (n == 0) return cudaSuccess;
  if (C % 8 == 0 && K_stride % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    const int64_t warps = static_cast<int64_t>(N) * Ho * Wo * kh * kw;
    int64_t grid = (warps + 7) / 8;
    if (grid > 148 * 32) grid = 148 * 32;
    conv2d_im2col_vec8_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), N, H, W, C, Ho, Wo, kh, kw, stride,
        pad, K_stride);
    return cudaGetLastError();
  }
  conv2d_im2col_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<__nv_bfloat16*>(out), N, H, W, C, Ho, Wo, kh, kw,
                                                        stride, pad, K_stride);
  return cudaGetLastError();
}

}  // namespace omni
