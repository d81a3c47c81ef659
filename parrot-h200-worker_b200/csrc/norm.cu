// RMSNorm (N3) and Block AttnRes depth mixing fused with its consumer RMSNorm (N5).
//
// Both are HBM-bound row kernels: one warp per token row, 16-byte vector
// loads, fp32 statistics, warp-shuffle reductions and no shared memory.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

// ---------------------------------------------------------------------------
// RMSNorm: y = bf16((x * rsqrt(mean(x^2) + eps)) * w)     (model.py:125-127)
// ---------------------------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(128) rmsnorm_kernel(__nv_bfloat16* __restrict__ out,
                                                      const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      int rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = dim >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * dim);
  uint4 v[V];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      v[i] = __ldg(xr + c);
      float f[8];
      bf16x8_to_float(v[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)dim + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * dim);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float f[8], g[8];
      bf16x8_to_float(v[i], f);
      bf16x8_to_float(__ldg(wr + c), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = (f[j] * inv) * g[j];
      orow[c] = float_to_bf16x8(f);
    }
  }
}

int launch_rmsnorm(__nv_bfloat16* out, const __nv_bfloat16* x, const __nv_bfloat16* w,
                   int rows, int dim, float eps, cudaStream_t stream) {
  if (rows == 0) return 0;
  const int warps = 4;
  dim3 grid((rows + warps - 1) / warps), block(32 * warps);
  const int v = (dim / 8 + 31) / 32;
  switch (v) {
    case 1: rmsnorm_kernel<1><<<grid, block, 0, stream>>>(out, x, w, rows, dim, eps); break;
    case 2: rmsnorm_kernel<2><<<grid, block, 0, stream>>>(out, x, w, rows, dim, eps); break;
    case 3: rmsnorm_kernel<3><<<grid, block, 0, stream>>>(out, x, w, rows, dim, eps); break;
    case 4: rmsnorm_kernel<4><<<grid, block, 0, stream>>>(out, x, w, rows, dim, eps); break;
    case 5: case 6: case 7: case 8:
      rmsnorm_kernel<8><<<grid, block, 0, stream>>>(out, x, w, rows, dim, eps); break;
    default: return -1;
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Depth mix (model.py:149-155) with optional consumer RMSNorm (model.py:157-164)
// and optional deferred residual (model.py:702: partial = partial + delta).
//
// Per token row t and source i, all in fp32:
//   key_i  = v_i * rsqrt(mean(v_i^2) + key_eps) * key_w            (F.rms_norm)
//   s_i    = sum_d key_i[d] * q[d]
//   a      = softmax_i(s)
//   h      = bf16(sum_i a_i * v_i)                                 (the mixed tensor)
//   out    = out_w ? bf16((h * rsqrt(mean(h^2) + out_eps)) * out_w) : h
// Scores and weights stay fp32 (as the reference's fused Metal kernel keeps
// them, moe_bf16.metal:331-435): with a peaked softmax over sources, rounding
// the keys to bf16 first would move the weights by percents.
// When `pending_delta` is set, the last source is bf16(pending_base + delta)
// and is written to `pending_out` (the resolved partial block sum).
// ---------------------------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(128) depthmix_kernel(DepthMixArgs a) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int dim = a.dim;
  const int nvec = dim >> 3;
  const size_t off = (size_t)row * dim;
  const int S = a.n_sources;
  const bool pending = a.pending_delta != nullptr;

  float q[V][8], kw[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.query) + c), q[i]);
      bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.key_w) + c), kw[i]);
    }
  }

  // The pending (last) source lives in registers for both passes.
  uint4 pend[V];
  if (pending) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float b[8], d[8];
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.pending_base + off) + c), b);
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.pending_delta + off) + c), d);
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] = b[j] + d[j];
        pend[i] = float_to_bf16x8(b);
        reinterpret_cast<uint4*>(a.pending_out + off)[c] = pend[i];
      }
    }
  }

  float score[kMaxDepthSources];
  float smax = -INFINITY;
  for (int s = 0; s < S; ++s) {
    const bool is_pend = pending && s == S - 1;
    const uint4* src = reinterpret_cast<const uint4*>(a.sources[s] + off);
    uint4 v[V];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        v[i] = is_pend ? pend[i] : __ldg(src + c);
        float f[8];
        bf16x8_to_float(v[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
      }
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)dim + a.key_eps);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float f[8];
        bf16x8_to_float(v[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf((f[j] * inv) * kw[i][j], q[i][j], dot);
      }
    }
    dot = warp_sum(dot);
    score[s] = dot;
    smax = fmaxf(smax, dot);
  }
  float den = 0.f;
  for (int s = 0; s < S; ++s) {
    score[s] = expf(score[s] - smax);
    den += score[s];
  }
  for (int s = 0; s < S; ++s) score[s] = score[s] / den;

  float h[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) h[i][j] = 0.f;
  for (int s = 0; s < S; ++s) {
    const bool is_pend = pending && s == S - 1;
    const uint4* src = reinterpret_cast<const uint4*>(a.sources[s] + off);
    const float alpha = score[s];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float f[8];
        bf16x8_to_float(is_pend ? pend[i] : __ldg(src + c), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[i][j] = fmaf(alpha, f[j], h[i][j]);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[i][j] = round_bf16(h[i][j]);
      ss = fmaf(h[i][j], h[i][j], ss);
    }
  uint4* orow = reinterpret_cast<uint4*>(a.out + off);
  if (a.mix_out != nullptr) {
    uint4* mrow = reinterpret_cast<uint4*>(a.mix_out + off);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) mrow[c] = float_to_bf16x8(h[i]);
    }
  }
  if (a.out_w == nullptr) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) orow[c] = float_to_bf16x8(h[i]);
    }
    return;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)dim + a.out_eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float g[8];
      bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.out_w) + c), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = (h[i][j] * inv) * g[j];
      orow[c] = float_to_bf16x8(g);
    }
  }
}

int launch_depthmix(const DepthMixArgs& args, cudaStream_t stream) {
  if (args.rows == 0) return 0;
  const int warps = 4;
  dim3 grid((args.rows + warps - 1) / warps), block(32 * warps);
  const int v = (args.dim / 8 + 31) / 32;
  switch (v) {
    case 1: depthmix_kernel<1><<<grid, block, 0, stream>>>(args); break;
    case 2: depthmix_kernel<2><<<grid, block, 0, stream>>>(args); break;
    case 3: depthmix_kernel<3><<<grid, block, 0, stream>>>(args); break;
    case 4: depthmix_kernel<4><<<grid, block, 0, stream>>>(args); break;
    default: return -1;
  }
  return 0;
}

}  // namespace parrot
