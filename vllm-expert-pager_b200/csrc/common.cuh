// Shared helpers of the xpager CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "xpager.h"

namespace xp {

// Launch status: a pending launch error, or XP_OK.
inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? XP_OK : static_cast<int>(err);
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Expert id k of an int32 or int64 id array.
__device__ __forceinline__ int64_t load_id(const void *ids, int ids_bytes, int64_t k) {
  return ids_bytes == 4 ? static_cast<int64_t>(static_cast<const int32_t *>(ids)[k])
                        : static_cast<const int64_t *>(ids)[k];
}

__device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
  int64_t q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

__device__ __forceinline__ int64_t floor_mod(int64_t a, int64_t b) { return a - floor_div(a, b) * b; }

// System-scope accesses to pinned host memory (the SSD request ring).
__device__ __forceinline__ int64_t load_acquire_sys(const int64_t *p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int64_t load_relaxed_sys(const int64_t *p) {
  int64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void store_release_sys(int64_t *p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace xp
