// Greedy next token of a decode step: the tied LM-head projection fused with
// the argmax over the vocabulary, so the [B, V] logits are never written.
//   out[t] = argmax_v bf16( sum_k h[t, k] * W[v, k] )
// with fp32 accumulation and the logit rounded to bf16 before the comparison
// (F.linear on bf16 tensors rounds its fp32 result once), the lowest v among
// equal values (torch.argmax returns the first maximal index).  Replaces
// parrot/model.py:927-931 (decode_next: F.linear(normalized,
// embedding.weight).argmax(-1)) and the Metal vocab_argmax_partials_bf16 /
// vocab_argmax_reduce_bf16 pair (parrot/kernels/moe_bf16.metal:1541-1621,
// bound in parrot/metal_moe.py:329-353).
//
// The projection streams the whole embedding (V x d bf16, 50 MB for Parrot XL)
// once: it is HBM-bound.  Each warp takes groups of four vocabulary rows in a
// grid-stride loop; a lane holds ceil(d / 256) 16-byte vectors of each row and the
// next group's vectors are loaded while the current group is folded.  The
// first group's weights are loaded before the grid-dependency wait (the
// embedding is a parameter; only h comes from the previous kernel).  A warp's
// 4 x NT dots are folded by one warp_reduce_many; the per-CTA best (value,
// row) per token goes to a partial table and the last CTA to finish reduces
// the table to the token ids (the lowest row among equal values, whatever the
// order of the reduction).
#include "common.cuh"
#include "kernels.h"

namespace parrot {

namespace {

constexpr int kVocabWarps = 4;

struct Best {
  float v;
  int i;
};

// a better than b: larger value, or the same value at a lower index
__device__ __forceinline__ bool better(float av, int ai, float bv, int bi) {
  return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ Best shfl_best(Best b, int mask) {
  Best o;
  o.v = __shfl_xor_sync(0xffffffffu, b.v, mask);
  o.i = __shfl_xor_sync(0xffffffffu, b.i, mask);
  return better(o.v, o.i, b.v, b.i) ? o : b;
}

template <int NV>
__device__ __forceinline__ void load_rows(uint4 (&w)[4][NV], const uint4* __restrict__ W,
                                          int row0, int kv, int lane, int V) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = min(row0 + r, V - 1);  // a short last group re-reads a valid row
#pragma unroll
    for (int c = 0; c < NV; ++c)
      w[r][c] = lane + 32 * c < kv ? __ldcs(W + (size_t)row * kv + lane + 32 * c)
                                   : make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace

// NT: token capacity of the instantiation (1, 2, 4, 8); NV: 16-byte vectors
// per lane per row (ceil(d / 256); lanes past the row's end hold zeros).
template <int NT, int NV>
__global__ void __launch_bounds__(32 * kVocabWarps) vocab_argmax_kernel(VocabArgmaxArgs a) {
  extern __shared__ __align__(16) float va_x[];  // [NT][d] fp32 token rows
  __shared__ Best warp_best[kVocabWarps][NT];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.dim, kv = K >> 3, V = a.vocab;
  const uint4* W = static_cast<const uint4*>(a.weight);
  const int groups = (V + 3) >> 2;
  const int stride = gridDim.x * kVocabWarps;
  int g = blockIdx.x * kVocabWarps + warp;
  uint4 cur[4][NV], nxt[4][NV];
  if (g < groups) load_rows<NV>(cur, W, 4 * g, kv, lane, V);
  griddep_wait();
  griddep_launch();
  const int B = a.rows;
  const uint4* hg = static_cast<const uint4*>(a.hidden);
  for (int i = threadIdx.x; i < B * kv; i += blockDim.x) {
    float f[8];
    bf16x8_to_float(hg[i], f);
    reinterpret_cast<float4*>(va_x)[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(va_x)[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  __syncthreads();

  Best best{-INFINITY, 0x7fffffff};  // lane t < NT: this warp's best for token t
  for (; g < groups; g += stride) {
    const int gn = g + stride;
    if (gn < groups) load_rows<NV>(nxt, W, 4 * gn, kv, lane, V);
    float2 acc[4 * NT];
#pragma unroll
    for (int v = 0; v < 4 * NT; ++v) acc[v] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const int col = 8 * (lane + 32 * c);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < B && col < K) {
          const float4* xp = reinterpret_cast<const float4*>(va_x + (size_t)t * K + col);
          const float4 x0 = xp[0], x1 = xp[1];
          const float2 xa = make_float2(x0.x, x0.y), xb = make_float2(x0.z, x0.w);
          const float2 xc = make_float2(x1.x, x1.y), xd = make_float2(x1.z, x1.w);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint4 w = cur[r][c];
            float2 s = acc[r * NT + t];
            s = __ffma2_rn(bf16x2_to_float2(w.x), xa, s);
            s = __ffma2_rn(bf16x2_to_float2(w.y), xb, s);
            s = __ffma2_rn(bf16x2_to_float2(w.z), xc, s);
            s = __ffma2_rn(bf16x2_to_float2(w.w), xd, s);
            acc[r * NT + t] = s;
          }
        }
      }
    }
    float dots[4 * NT];
#pragma unroll
    for (int v = 0; v < 4 * NT; ++v) dots[v] = acc[v].x + acc[v].y;
    // lane l: the dot of row (l % 4NT) / NT, token l % NT
    const float total = warp_reduce_many<4 * NT>(dots, lane);
    const int k = lane % (4 * NT);
    const int row = 4 * g + k / NT;
    Best cand{row < V ? round_bf16(total) : -INFINITY, row};
    // the four rows of each token: lanes t, t + NT, t + 2NT, t + 3NT
    cand = shfl_best(cand, NT);
    cand = shfl_best(cand, 2 * NT);
    if (better(cand.v, cand.i, best.v, best.i)) best = cand;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < NV; ++c) cur[r][c] = nxt[r][c];
  }
  if (lane < NT) warp_best[warp][lane] = best;
  __syncthreads();
  if (threadIdx.x < NT) {
    const int t = threadIdx.x;
    Best b = warp_best[0][t];
    for (int w = 1; w < kVocabWarps; ++w)
      if (better(warp_best[w][t].v, warp_best[w][t].i, b.v, b.i)) b = warp_best[w][t];
    a.partial_value[(size_t)blockIdx.x * NT + t] = b.v;
    a.partial_index[(size_t)blockIdx.x * NT + t] = b.i;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    if (last) *a.counter = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The last CTA reduces the partials token by token: each thread loads its
  // share of the CTAs' entries at once (a chain of dependent L2 loads per lane
  // was this kernel's tail), then shuffles and one shared-memory join.
  constexpr int kPer = kVocabMaxGrid / (32 * kVocabWarps);
  for (int t = 0; t < B; ++t) {
    float v[kPer];
    int ix[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = threadIdx.x + k * (32 * kVocabWarps);
      const bool in = c < (int)gridDim.x;
      v[k] = in ? __ldcg(a.partial_value + (size_t)c * NT + t) : -INFINITY;
      ix[k] = in ? __ldcg(a.partial_index + (size_t)c * NT + t) : 0x7fffffff;
    }
    Best b{v[0], ix[0]};
#pragma unroll
    for (int k = 1; k < kPer; ++k)
      if (better(v[k], ix[k], b.v, b.i)) b = Best{v[k], ix[k]};
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) b = shfl_best(b, m);
    if (lane == 0) warp_best[warp][0] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
      Best r = warp_best[0][0];
      for (int w = 1; w < kVocabWarps; ++w)
        if (better(warp_best[w][0].v, warp_best[w][0].i, r.v, r.i)) r = warp_best[w][0];
      a.out[t] = r.i;
    }
    __syncthreads();
  }
}

// Row-wise argmax of bf16 logits [rows, cols] (one CTA per row), the
// torch.argmax(-1) of decode_next when the projection runs as a GEMM
// (more than 8 token rows).  Lowest column among equal maxima.
__global__ void __launch_bounds__(512) argmax_rows_kernel(ArgmaxRowsArgs a) {
  __shared__ Best warp_best[16];
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = a.cols >> 3;
  const uint4* src = static_cast<const uint4*>(a.logits) + (size_t)row * nvec;
  Best b{-INFINITY, 0x7fffffff};
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float f[8];
    bf16x8_to_float(__ldcs(src + c), f);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (f[j] > b.v) b = Best{f[j], 8 * c + j};  // ascending within a thread: strict >
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) b = shfl_best(b, m);
  if (lane == 0) warp_best[warp] = b;
  __syncthreads();
  if (warp == 0) {
    b = lane < (int)(blockDim.x >> 5) ? warp_best[lane] : Best{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) b = shfl_best(b, m);
    if (lane == 0) a.out[row] = b.i;
  }
}

// Grid: as many CTAs as fit on every SM at once (register-bound: 4 per SM at
// one token row, fewer at eight), up to kVocabMaxGrid; a grid of two CTAs per
// SM kept a third of the HBM bandwidth busy at one row (ncu: 12% of warp
// slots active).
template <int NT, int NV>
static int launch_vocab_nt(const VocabArgmaxArgs& a, int sms, cudaStream_t stream) {
  const size_t smem = (size_t)NT * a.dim * sizeof(float);
  static int cached[64] = {};  // CTAs per SM, per device (smem is at most 8 x 1024 floats)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  int per_sm = cached[dev];
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, vocab_argmax_kernel<NT, NV>, 32 * kVocabWarps,
            (size_t)NT * 1024 * sizeof(float)) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cached[dev] = per_sm;
  }
  int grid = sms * per_sm;
  if (grid > kVocabMaxGrid) grid = kVocabMaxGrid;
  return launch_pdl(vocab_argmax_kernel<NT, NV>, dim3(grid), dim3(32 * kVocabWarps), smem, stream,
                    a) == cudaSuccess
             ? 0
             : -1;
}

int launch_vocab_argmax(const VocabArgmaxArgs& a, int sms, cudaStream_t stream) {
  const int nt = a.rows <= 1 ? 1 : a.rows <= 2 ? 2 : a.rows <= 4 ? 4 : 8;
  const int nv = (a.dim + 255) / 256;
#define PARROT_VOCAB_CASE(NT, NV) \
  if (nt == NT && nv == NV) return launch_vocab_nt<NT, NV>(a, sms, stream);
#define PARROT_VOCAB_NV(NV) \
  PARROT_VOCAB_CASE(1, NV) PARROT_VOCAB_CASE(2, NV) PARROT_VOCAB_CASE(4, NV) PARROT_VOCAB_CASE(8, NV)
  PARROT_VOCAB_NV(1)
  PARROT_VOCAB_NV(2)
  PARROT_VOCAB_NV(3)
  PARROT_VOCAB_NV(4)
#undef PARROT_VOCAB_NV
#undef PARROT_VOCAB_CASE
  return -1;
}

int launch_argmax_rows(const ArgmaxRowsArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return 0;
  return launch_pdl(argmax_rows_kernel, dim3(a.rows), dim3(512), 0, stream, a) == cudaSuccess
             ? 0
             : -1;
}

}  // namespace parrot
