// System-scope flag helpers for kernels that exchange data through another
// GPU's memory (peer pointers mapped with CUDA IPC).  sm_100a only.
#pragma once

#include "common.cuh"

namespace parrot {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_volatile(const int* p) {
  return *reinterpret_cast<const volatile int*>(p);
}

// Waits until *flag >= want.  Gives up when limit_ns pass or another thread
// has already recorded an error in *status; returns false then.
__device__ __forceinline__ bool wait_flag(const unsigned* flag, unsigned want, uint64_t limit_ns,
                                          const int* status) {
  if (ld_acquire_sys(flag) >= want) return true;
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_sys(flag) < want) {
    if (global_timer_ns() - t0 > limit_ns) return false;
    if (status != nullptr && ld_volatile(status) != 0) return false;
    __nanosleep(100);
  }
  return true;
}

}  // namespace parrot
