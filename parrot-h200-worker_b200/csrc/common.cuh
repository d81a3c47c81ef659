// Shared device helpers for the Parrot B200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "parrot_b200 targets sm_100a only"
#endif

namespace parrot {

// ---------------------------------------------------------------------------
// device status word: {code, site, info, unused}.  The first error wins.
// Codes are >0 so the C-ABI can return them unchanged.
// ---------------------------------------------------------------------------
enum StatusCode : int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,   // a bounded mbarrier / flag wait ran out
  kStatusBadIndex = 2,      // an expert id or row fell outside its range
  kStatusBadShape = 3,      // launch shape inconsistent with the tables
};

__device__ __forceinline__ void report_status(int* status, int code, int site, int info) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = site;
    status[2] = info;
  }
}

// ---------------------------------------------------------------------------
// bf16 <-> fp32 vector helpers (16-byte rows)
// ---------------------------------------------------------------------------
// bf16 pair (low half first) -> fp32 pair, exact
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ void bf16x8_to_float(const uint4& v, float f[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 float_to_bf16x8(const float f[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Round an fp32 value to the nearest bf16 and back: models a tensor that the
// reference materialises in bf16 between two torch ops.
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Reduce N per-lane partial values across the warp at once (N a power of two,
// N <= 32).  Halving exchanges move half of the remaining values per step, so
// N values cost N - 1 + log2(32 / N) shuffles instead of 5 N.  On return,
// lane l holds the warp-wide total of value index (l % N) in v[0].
template <int N, typename V>
__device__ __forceinline__ V warp_reduce_many(V (&v)[N], int lane) {
#pragma unroll
  for (int o = N / 2; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < o; ++j) {
      const V send = upper ? v[j] : v[j + o];
      const V keep = upper ? v[j + o] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
#pragma unroll
  for (int o = N; o < 32; o <<= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  return v[0];
}

// Arg-max over aligned groups of NP lanes (NP a power of two): every lane
// ends with its group's largest v, the lowest i among equal values.
template <int NP>
__device__ __forceinline__ void best_of_group(float& v, int& i) {
#pragma unroll
  for (int o = NP / 2; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// 16-byte global -> shared asynchronous copy (bypasses L1), and its fences.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Programmatic dependent launch.  Kernels launched with launch_pdl may start
// while the previous kernel on the stream is still running: everything before
// griddep_wait() must only read data that kernel does not write (weights,
// constants) and must write nothing that it reads.  griddep_launch() lets the
// next PDL kernel start its own independent prologue.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound for every spin-wait in these kernels (nanoseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Launch with programmatic stream serialization (see griddep_wait).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace parrot
