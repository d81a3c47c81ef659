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
  griddep_wait();
  griddep_launch();
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
    case 1: launch_pdl(rmsnorm_kernel<1>, grid, block, 0, stream, out, x, w, rows, dim, eps); break;
    case 2: launch_pdl(rmsnorm_kernel<2>, grid, block, 0, stream, out, x, w, rows, dim, eps); break;
    case 3: launch_pdl(rmsnorm_kernel<3>, grid, block, 0, stream, out, x, w, rows, dim, eps); break;
    case 4: launch_pdl(rmsnorm_kernel<4>, grid, block, 0, stream, out, x, w, rows, dim, eps); break;
    case 5: case 6: case 7: case 8:
      launch_pdl(rmsnorm_kernel<8>, grid, block, 0, stream, out, x, w, rows, dim, eps); break;
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
//
// One warp per row.  The warp first issues 16-byte async copies of every
// source row into its shared-memory slab (all loads in flight at once: one
// memory round trip), then makes one pass for the S sums of squares and the S
// raw key.query dots (s_i = rsqrt(...) * sum_d v kw q), reduced together with
// warp_reduce_many, a lane-parallel softmax, and a second pass for the mix.
// ---------------------------------------------------------------------------
constexpr int kDepthWarps = 4;

template <int V>
__global__ void __launch_bounds__(32 * kDepthWarps) depthmix_kernel(DepthMixArgs a) {
  extern __shared__ __align__(16) unsigned char depth_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = blockIdx.x * kDepthWarps + warp;
  griddep_wait();
  griddep_launch();
  if (row >= a.rows) return;
  const int dim = a.dim, nvec = dim >> 3, S = a.n_sources;
  const size_t off = (size_t)row * dim;
  const bool pending = a.pending_delta != nullptr;
  uint4* slab = reinterpret_cast<uint4*>(depth_smem) + (size_t)warp * S * nvec;

  // 1. every source slice of this row in flight at once
  for (int s = 0; s < S; ++s) {
    if (pending && s == S - 1) continue;
    const uint4* src = reinterpret_cast<const uint4*>(a.sources[s] + off);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) cp_async16(slab + s * nvec + c, src + c);
    }
  }
  // every small vector this warp needs, requested together
  uint4 qv[V], kwv[V], owv[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      qv[i] = __ldg(reinterpret_cast<const uint4*>(a.query) + c);
      kwv[i] = __ldg(reinterpret_cast<const uint4*>(a.key_w) + c);
      if (a.out_w != nullptr) owv[i] = __ldg(reinterpret_cast<const uint4*>(a.out_w) + c);
    }
  }
  float q[V][8], kw[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      bf16x8_to_float(qv[i], q[i]);
      bf16x8_to_float(kwv[i], kw[i]);
    }
  }
  if (pending) {  // the deferred residual add, resolved in registers
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float b[8], dl[8];
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.pending_base + off) + c), b);
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.pending_delta + off) + c), dl);
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] = b[j] + dl[j];
        const uint4 r = float_to_bf16x8(b);
        reinterpret_cast<uint4*>(a.pending_out + off)[c] = r;
        slab[(S - 1) * nvec + c] = r;
      }
    }
  }
  cp_async_wait_all();  // each lane reads back only the slices it copied

  // 2. sums of squares and raw key.query dots of all sources, reduced together
  float ss[kMaxDepthSources], raw[kMaxDepthSources];
#pragma unroll
  for (int s = 0; s < kMaxDepthSources; ++s) {
    ss[s] = 0.f;
    raw[s] = 0.f;
    if (s < S) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) {
          float f[8];
          bf16x8_to_float(slab[s * nvec + c], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            ss[s] = fmaf(f[j], f[j], ss[s]);
            raw[s] = fmaf(f[j] * kw[i][j], q[i][j], raw[s]);
          }
        }
      }
    }
  }
  const float ss_l = warp_reduce_many<kMaxDepthSources>(ss, lane);
  const float raw_l = warp_reduce_many<kMaxDepthSources>(raw, lane);
  // lane l now owns source l % 16
  const int src_l = lane & (kMaxDepthSources - 1);
  const bool valid = src_l < S;
  const float score = valid ? rsqrtf(ss_l / (float)dim + a.key_eps) * raw_l : -INFINITY;
  const float m = warp_max(score);
  const float e = valid ? expf(score - m) : 0.f;
  const float den = warp_sum(lane < kMaxDepthSources ? e : 0.f);
  const float alpha_l = e / den;

  // 3. mix, then the consumer RMSNorm
  float h[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) h[i][j] = 0.f;
  for (int s = 0; s < S; ++s) {
    const float alpha = __shfl_sync(0xffffffffu, alpha_l, s);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float f[8];
        bf16x8_to_float(slab[s * nvec + c], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[i][j] = fmaf(alpha, f[j], h[i][j]);
      }
    }
  }
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[i][j] = round_bf16(h[i][j]);
      sq = fmaf(h[i][j], h[i][j], sq);
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
  sq = warp_sum(sq);
  const float inv = rsqrtf(sq / (float)dim + a.out_eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float g[8];
      bf16x8_to_float(owv[i], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = (h[i][j] * inv) * g[j];
      orow[c] = float_to_bf16x8(g);
    }
  }
}

template <int V>
static int launch_depthmix_v(const DepthMixArgs& args, cudaStream_t stream) {
  const size_t smem = (size_t)kDepthWarps * args.n_sources * (args.dim / 8) * sizeof(uint4);
  static unsigned long long configured = 0;  // per device: the attribute lives in its context
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    const int max_smem = kDepthWarps * kMaxDepthSources * (1024 / 8) * (int)sizeof(uint4);
    if (cudaFuncSetAttribute(depthmix_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_smem) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  dim3 grid((args.rows + kDepthWarps - 1) / kDepthWarps), block(32 * kDepthWarps);
  return launch_pdl(depthmix_kernel<V>, grid, block, smem, stream, args) == cudaSuccess ? 0 : -2;
}

int launch_depthmix(const DepthMixArgs& args, cudaStream_t stream) {
  if (args.rows == 0) return 0;
  const int v = (args.dim / 8 + 31) / 32;
  switch (v) {
    case 1: return launch_depthmix_v<1>(args, stream);
    case 2: return launch_depthmix_v<2>(args, stream);
    case 3: return launch_depthmix_v<3>(args, stream);
    case 4: return launch_depthmix_v<4>(args, stream);
    default: return -1;
  }
}

// ---------------------------------------------------------------------------
// Rotary embedding in place (model.py:206-216), for the packed projection
// output of local attention: the first n_heads * head_dim columns of each row
// hold the q and k heads; pair (x[2j], x[2j+1]) of a head at position p becomes
//   (bf16(bf16(x0 c) - bf16(x1 s)), bf16(bf16(x0 s) + bf16(x1 c))),
// c = cos[p][j], s = sin[p][j] (bf16 tables): every product and sum rounded
// like the reference's bf16 tensor expression.  One thread per 8 columns.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rope_kernel(__nv_bfloat16* __restrict__ x,
                                                   const __nv_bfloat16* __restrict__ cos_t,
                                                   const __nv_bfloat16* __restrict__ sin_t,
                                                   int rows, int row_stride, int rot_cols,
                                                   int head_dim, int seq_len, int start) {
  griddep_wait();
  griddep_launch();
  const int vec_per_row = rot_cols >> 3;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * vec_per_row) return;
  const int r = (int)(i / vec_per_row), v = (int)(i % vec_per_row);
  const int col = v * 8;
  const int pos = start + r % seq_len;
  const int j0 = (col % head_dim) >> 1;
  uint4* px = reinterpret_cast<uint4*>(x + (size_t)r * row_stride + col);
  float f[8];
  bf16x8_to_float(*px, f);
  const uint2 cv = *reinterpret_cast<const uint2*>(cos_t + (size_t)pos * (head_dim >> 1) + j0);
  const uint2 sv = *reinterpret_cast<const uint2*>(sin_t + (size_t)pos * (head_dim >> 1) + j0);
  const __nv_bfloat16* cb = reinterpret_cast<const __nv_bfloat16*>(&cv);
  const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(&sv);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float c = __bfloat162float(cb[k]), s = __bfloat162float(sb[k]);
    const float e = f[2 * k], o = f[2 * k + 1];
    f[2 * k] = round_bf16(e * c) - round_bf16(o * s);
    f[2 * k + 1] = round_bf16(e * s) + round_bf16(o * c);
  }
  *px = float_to_bf16x8(f);
}

int launch_rope(__nv_bfloat16* x, const __nv_bfloat16* cos_t, const __nv_bfloat16* sin_t,
                int rows, int row_stride, int rot_cols, int head_dim, int seq_len, int start,
                cudaStream_t stream) {
  const long long total = (long long)rows * (rot_cols / 8);
  if (total == 0) return 0;
  const int threads = 256;
  return launch_pdl(rope_kernel, dim3((unsigned)((total + threads - 1) / threads)),
                    dim3(threads), 0, stream, x, cos_t, sin_t, rows, row_stride, rot_cols,
                    head_dim, seq_len, start) == cudaSuccess ? 0 : -2;
}

}  // namespace parrot
