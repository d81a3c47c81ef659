// Projections of a decode step (at most 8 token rows): y[t, n] = sum_k x[t, k]
// w[n, k] with fp32 accumulation and one rounding of the result, the
// semantics of F.linear on these dtypes (model.py:303-328, 399-432):
//   bf16 x, bf16 w -> bf16 y    (local attention qkv / out, MLA latent down)
//   bf16 x, fp32 w -> fp32 y    (absorbed MLA query: x.float() is exact)
//   fp32 x, fp32 w -> bf16 y    (absorbed MLA output, then .to(bf16))
// Small-batch projections are weight-bound and latency-bound: each CTA takes
// 16 output rows and copies their weights into shared memory before its grid
// dependency wait (the weights are parameters; only the token rows come from
// the previous kernel), then stages the token rows as fp32.  Warp w takes rows
// 4w .. 4w + 3: its lanes stride over 16-byte weight vectors, accumulate the
// 4 x NT dots in one pass over k, and one warp_reduce_many folds them.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

namespace {
constexpr int kRowsPerCta = 16;  // 4 per warp

template <int N>
__device__ __forceinline__ void load_w_vec(const uint4& v, float (&f)[N]);
template <>
__device__ __forceinline__ void load_w_vec<8>(const uint4& v, float (&f)[8]) {
  bf16x8_to_float(v, f);
}
template <>
__device__ __forceinline__ void load_w_vec<4>(const uint4& v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}
}  // namespace

// WF: fp32 weights (else bf16); NT: token capacity of the instantiation.
template <bool WF, int NT>
__global__ void __launch_bounds__(128) linear_small_kernel(LinearSmallArgs a) {
  constexpr int EW = WF ? 4 : 8;  // weight elements per 16-byte vector
  extern __shared__ __align__(16) uint4 ls_smem[];
  const int K = a.k_in, kv = K / EW;  // 16-byte weight vectors per row
  uint4* w_s = ls_smem;                                                  // [16][kv]
  float* x_s = reinterpret_cast<float*>(w_s + (size_t)kRowsPerCta * kv);  // [NT][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kRowsPerCta;
  const uint4* wg = reinterpret_cast<const uint4*>(
      static_cast<const char*>(a.w) + (size_t)n0 * K * (WF ? 4 : 2));
  for (int i = threadIdx.x; i < kRowsPerCta * kv; i += blockDim.x) cp_async16(w_s + i, wg + i);
  griddep_wait();
  griddep_launch();
  const int B = a.rows;
  if (a.x_f32) {
    const float4* xg = static_cast<const float4*>(a.x);
    for (int i = threadIdx.x; i < B * K / 4; i += blockDim.x)
      reinterpret_cast<float4*>(x_s)[i] = xg[i];
  } else {
    const uint4* xg = static_cast<const uint4*>(a.x);
    for (int i = threadIdx.x; i < B * K / 8; i += blockDim.x) {
      float f[8];
      bf16x8_to_float(xg[i], f);
      reinterpret_cast<float4*>(x_s)[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
      reinterpret_cast<float4*>(x_s)[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  constexpr int NV = 4 * NT;  // values to fold: row r of the warp, token t at r * NT + t
  float acc[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) acc[v] = 0.f;
  const uint4* wr = w_s + (size_t)(4 * warp) * kv;
  for (int c = lane; c < kv; c += 32) {
    float xf[NT][EW];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < B) {
        const float4* xp = reinterpret_cast<const float4*>(x_s + (size_t)t * K + c * EW);
#pragma unroll
        for (int q = 0; q < EW / 4; ++q) {
          const float4 v = xp[q];
          xf[t][4 * q] = v.x;
          xf[t][4 * q + 1] = v.y;
          xf[t][4 * q + 2] = v.z;
          xf[t][4 * q + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < EW; ++e) xf[t][e] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float wf[EW];
      load_w_vec<EW>(wr[(size_t)r * kv + c], wf);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < EW; ++e) acc[r * NT + t] = fmaf(wf[e], xf[t][e], acc[r * NT + t]);
    }
  }
  const float tot = warp_reduce_many<NV>(acc, lane);  // lane v: value v % NV
  const int r = (lane % NV) / NT, t = lane % NT;
  if (lane < NV && t < B) {
    const size_t oi = (size_t)t * a.n_out + n0 + 4 * warp + r;
    if (a.y_f32)
      static_cast<float*>(a.y)[oi] = tot;
    else
      static_cast<__nv_bfloat16*>(a.y)[oi] = __float2bfloat16_rn(tot);
  }
}

template <bool WF, int NT>
static int launch_linear_small_nt(const LinearSmallArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)kRowsPerCta * a.k_in * (WF ? 4 : 2) + (size_t)NT * a.k_in * 4;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    // the largest call: k_in = kLinearSmallMaxK
    const int most = kRowsPerCta * kLinearSmallMaxK * (WF ? 4 : 2) + NT * kLinearSmallMaxK * 4;
    if (cudaFuncSetAttribute(linear_small_kernel<WF, NT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, most) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  return launch_pdl(linear_small_kernel<WF, NT>, dim3(a.n_out / kRowsPerCta), dim3(128), smem,
                    stream, a) == cudaSuccess
             ? 0
             : -2;
}

template <bool WF>
static int launch_linear_small_w(const LinearSmallArgs& a, cudaStream_t stream) {
  if (a.rows <= 1) return launch_linear_small_nt<WF, 1>(a, stream);
  if (a.rows <= 2) return launch_linear_small_nt<WF, 2>(a, stream);
  if (a.rows <= 4) return launch_linear_small_nt<WF, 4>(a, stream);
  return launch_linear_small_nt<WF, 8>(a, stream);
}

int launch_linear_small(const LinearSmallArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return 0;
  return a.w_f32 ? launch_linear_small_w<true>(a, stream) : launch_linear_small_w<false>(a, stream);
}

}  // namespace parrot
