// The dynamic shared memory a kernel may use above the 48 KB default, raised per device the first time a launch needs
// more. Function attributes belong to the device's primary context: after a host calls cudaDeviceReset they are gone
// (as is every other piece of module state, e.g. the address of a __device__ array) while the sizes recorded here
// stay, so a process must not call this library on a device after resetting it.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <mutex>

namespace bnn {

constexpr int kAttrDevices = 64;

struct SmemAttr {
  std::mutex mu;  // host threads of several contexts may launch the same kernel on one device at once
  size_t cur[kAttrDevices] = {};

  template <typename Kernel>
  cudaError_t ensure(Kernel *kernel, size_t smem) {
    int dev = 0;
    if (cudaGetDevice(&dev) || dev < 0 || dev >= kAttrDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (smem <= cur[dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (!e) cur[dev] = smem;
    return e;
  }
};

// The dynamic shared memory each of k resident CTAs of `kernel` may use on this device: the SM's shared memory split k
// ways, less the per-CTA reservation and the kernel's static shared memory.
template <typename Kernel>
size_t smem_budget(Kernel *kernel, int k) {
  int dev = 0, per_sm = 0, reserved = 0;
  cudaFuncAttributes fa;
  if (cudaGetDevice(&dev) || cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) ||
      cudaFuncGetAttributes(&fa, kernel))
    return 0;
  const long long b = (long long)per_sm / k - reserved - (long long)fa.sharedSizeBytes;
  return b > 0 ? (size_t)b : 0;
}

}  // namespace bnn
