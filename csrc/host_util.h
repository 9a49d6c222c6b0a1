// Host-side launch helpers shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace omni {

// Raises the dynamic shared-memory limit of `Kernel` to `bytes` once per device.
// The attribute belongs to the device context, so a process that launches on a
// second GPU must set it there too; one bit per device (per kernel: the kernel
// is a template argument, so each kernel has its own mask) records that it was
// done.  Racing threads may both set it, which is harmless (the call is
// idempotent).
template <auto Kernel>
cudaError_t ensure_smem_attr(int bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

}  // namespace omni
