// Host helpers of libxpager: version, status strings, NUMA-placed pinned memory.
#define _GNU_SOURCE 1
#include <cuda_runtime.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include "xpager.h"

namespace {
constexpr int kVersion = 1;
// mbind(2) policy; spelled out to avoid depending on libnuma headers.
constexpr int kMpolPreferred = 1;
}  // namespace

extern "C" int xp_version(void) { return kVersion; }

extern "C" const char *xp_status_string(int status) {
  switch (status) {
    case XP_OK:
      return "ok";
    case XP_EINVAL:
      return "invalid argument (size, null pointer or alignment)";
    case XP_ERANGE:
      return "size above the kernel's limits";
    case XP_EPITCH:
      return "compressed row does not fit the pitch";
    default:
      return status > 0 ? cudaGetErrorString(static_cast<cudaError_t>(status)) : "unknown status";
  }
}

// Pinned host memory for the RAM tier.  The pages are reserved with mmap,
// placed on the GPU's NUMA node with mbind (best effort: a failure leaves the
// kernel's default placement), touched, then page-locked and mapped for the
// device with cudaHostRegister.  Unlike a caching pinned allocator nothing is
// rounded up to a power of two (store.py:54-58).
extern "C" int xp_pinned_alloc(int64_t bytes, int numa_node, void **host, void **dev) {
  if (bytes <= 0 || !host || !dev) return XP_EINVAL;
  void *p = mmap(nullptr, static_cast<size_t>(bytes), PROT_READ | PROT_WRITE,
                 MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p == MAP_FAILED) return XP_EINVAL;
  if (numa_node >= 0 && numa_node < 1024) {
    unsigned long mask[1024 / (8 * sizeof(unsigned long))] = {0};
    mask[numa_node / (8 * sizeof(unsigned long))] |= 1ul << (numa_node % (8 * sizeof(unsigned long)));
    syscall(SYS_mbind, p, static_cast<unsigned long>(bytes), kMpolPreferred, mask, 1024ul, 0u);
  }
  memset(p, 0, static_cast<size_t>(bytes));  // fault the pages in on that node
  cudaError_t err = cudaHostRegister(p, static_cast<size_t>(bytes),
                                     cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (err != cudaSuccess) {
    munmap(p, static_cast<size_t>(bytes));
    return static_cast<int>(err);
  }
  err = cudaHostGetDevicePointer(dev, p, 0);
  if (err != cudaSuccess) {
    cudaHostUnregister(p);
    munmap(p, static_cast<size_t>(bytes));
    return static_cast<int>(err);
  }
  *host = p;
  return XP_OK;
}

extern "C" int xp_pinned_free(void *host, int64_t bytes) {
  if (!host || bytes <= 0) return XP_EINVAL;
  cudaError_t err = cudaHostUnregister(host);
  munmap(host, static_cast<size_t>(bytes));
  return err == cudaSuccess ? XP_OK : static_cast<int>(err);
}

extern "C" int xp_device_pointer(void *host, void **dev) {
  if (!host || !dev) return XP_EINVAL;
  cudaError_t err = cudaHostGetDevicePointer(dev, host, 0);
  return err == cudaSuccess ? XP_OK : static_cast<int>(err);
}
