// RMSNorm (N3) and Block AttnRes depth mixing fused with its consumer RMSNorm (N5).
//
// Both are row kernels with 16-byte vector loads and fp32 statistics: RMSNorm
// takes one warp per token row; the depth mix one CTA per row (a warp per 256
// columns), so each thread's chain of dependent work stays short.
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
// and an optional deferred last source, computed while the sources are read
// and also written out:
//   residual add (model.py:702):  bf16(base + delta)
//   MoE combine (model.py:546-551, then :702):
//                 bf16(base + bf16(bf16(shared + c_lo) + c_hi)), c_lo / c_hi the
//                 token's routed contributions of the lower / higher expert id
//                 (the combine kernel's arithmetic; without base, no add).
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
// One CTA of W warps per row (W = ceil(d / 256): 3 at d = 768); thread t owns
// the row's 16-byte vector t.  A row at a time keeps the per-thread chain
// short: every source vector is one register load (all S in flight at once),
// each thread reduces its 8 columns, warp_reduce_many folds the S sums of
// squares and S raw key.query dots (s_i = rsqrt(mean(v_i^2) + eps) *
// sum_d v kw q) across the warp, and one shared-memory exchange joins the
// warps.  Every thread then computes the S scores and the softmax itself (the
// same order everywhere, so all threads agree bit for bit) and mixes its own
// vector; a second exchange gives the consumer norm's sum of squares.
// ---------------------------------------------------------------------------
// NS: the source capacity of this instantiation (2, 4, 8 or 16 >= n_sources),
// so the per-source arrays and loops are sized to the call.
// Up to 8 sources the kernel fits 80 registers without spilling, so 768
// threads (8 CTAs at d = 768) stay resident per SM; 16 sources need more.
//
// With a router (NP = E padded to 16 or 32; NP = 0: none) the mixed,
// normalised rows are an MoE block's input and the kernel routes them too,
// the router kernel's job (route.cu) folded in: a CTA takes R =
// kRouteSmallTile (4) rows (blockDim.y), the router weight is copied into shared
// memory before the grid-dependency wait, each thread dots its 8 columns of
// the bf16 output with the E weight rows, and after one warp_reduce_many and
// a shared-memory join warp 0 of each row does the softmax, top-2 and
// renormalisation (the router kernel's formulas); the CTA writes its tile's
// histogram and probability sums.
template <int W, int NS, int R, int NP>
__global__ void __launch_bounds__(32 * W * R, (NS <= 8 && R == 1) ? 768 / (32 * W) : 1)
    depthmix_kernel(DepthMixArgs a, DepthRouteArgs ra) {
  static_assert(NP == 0 || R == kRouteSmallTile, "a routing CTA covers one router tile");
  __shared__ float red_sr[R][W][2 * NS], red_sq[R][W];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = threadIdx.x;
  const int ty = R > 1 ? (int)threadIdx.y : 0;
  const int row = blockIdx.x * R + ty;
  const int dim = a.dim, nvec = dim >> 3, S = a.n_sources;
  const bool active = c < nvec && row < a.rows;
  const size_t off = (size_t)row * dim;
  if constexpr (NP > 0) {
    // the router weight is a parameter: staged before the dependency wait
    extern __shared__ __align__(16) uint4 dm_rw[];  // [E][nvec]
    const int tid = ty * blockDim.x + c, nthreads = blockDim.x * R;
    const uint4* wg = reinterpret_cast<const uint4*>(ra.router_w);
    for (int i = tid; i < ra.r.n_experts * nvec; i += nthreads) cp_async16(dm_rw + i, wg + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const bool pend_moe = a.pending_contrib != nullptr;
  const bool pending = a.pending_delta != nullptr || pend_moe;

  // the query and norm weights are parameters: read before the grid dependency
  float q[8], kw[8];
  uint4 owv = make_uint4(0, 0, 0, 0);
  if (active) {
    bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.query) + c), q);
    bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.key_w) + c), kw);
    if (a.out_w != nullptr) owv = __ldg(reinterpret_cast<const uint4*>(a.out_w) + c);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = kw[j] = 0.f;
  }
  griddep_wait();
  griddep_launch();

  // 1. every source vector of this thread in flight at once
  uint4 v[NS];
  uint4 pb = make_uint4(0, 0, 0, 0), pd = make_uint4(0, 0, 0, 0);
  uint4 pc0 = make_uint4(0, 0, 0, 0), pc1 = make_uint4(0, 0, 0, 0);
  if (pending && active) {
    if (a.pending_base != nullptr) pb = __ldg(reinterpret_cast<const uint4*>(a.pending_base + off) + c);
    if (pend_moe) {
      pd = __ldg(reinterpret_cast<const uint4*>(a.pending_shared + off) + c);
      pc0 = __ldg(reinterpret_cast<const uint4*>(a.pending_contrib + 2 * off) + c);
      pc1 = __ldg(reinterpret_cast<const uint4*>(a.pending_contrib + 2 * off + dim) + c);
    } else {
      pd = __ldg(reinterpret_cast<const uint4*>(a.pending_delta + off) + c);
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    v[s] = make_uint4(0, 0, 0, 0);
    if (s < S && active && !(pending && s == S - 1))
      v[s] = __ldg(reinterpret_cast<const uint4*>(a.sources[s] + off) + c);
  }
  uint4 r = make_uint4(0, 0, 0, 0);
  if (pending && active) {
    // the deferred last source
    float b[8], dl[8];
    bf16x8_to_float(pb, b);
    bf16x8_to_float(pd, dl);
    if (pend_moe) {
      float p0[8], p1[8];
      bf16x8_to_float(pc0, p0);
      bf16x8_to_float(pc1, p1);
#pragma unroll
      for (int j = 0; j < 8; ++j) dl[j] = round_bf16(round_bf16(dl[j] + p0[j]) + p1[j]);
    }
    if (a.pending_base != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = b[j] + dl[j];
      r = float_to_bf16x8(b);
    } else {
      r = float_to_bf16x8(dl);
    }
    reinterpret_cast<uint4*>(a.pending_out + off)[c] = r;
  }
  // source s as this thread sees it.  Up to 8 sources the deferred one takes
  // its register slot once (a select per slot); with 16 the compiler turns
  // those selects into a run-time indexed store (local memory), so there each
  // read selects instead.
  if constexpr (NS <= 8) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const bool take = pending && s == S - 1;
      v[s].x = take ? r.x : v[s].x;
      v[s].y = take ? r.y : v[s].y;
      v[s].z = take ? r.z : v[s].z;
      v[s].w = take ? r.w : v[s].w;
    }
  }
  auto source = [&](int s) {
    if constexpr (NS <= 8) return v[s];
    else return (pending && s == S - 1) ? r : v[s];
  };

  // key.query weight per column pair (the score needs sum_d v kw q, not the
  // key itself); the per-column sums below run on packed fp32 pairs
  float2 kq[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) kq[p] = make_float2(kw[2 * p] * q[2 * p], kw[2 * p + 1] * q[2 * p + 1]);
  // 2. per-source sums of squares and raw key.query dots, folded across the
  // warp together: lane s holds source s's sum of squares, lane NS + s its dot
  float sr[2 * NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    sr[s] = 0.f;
    sr[NS + s] = 0.f;
    if (s < S) {
      const uint4 sv = source(s);
      const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
      float2 ss2 = make_float2(0.f, 0.f), raw2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 f2 = bf16x2_to_float2(w[p]);
        ss2 = __ffma2_rn(f2, f2, ss2);
        raw2 = __ffma2_rn(f2, kq[p], raw2);
      }
      sr[s] = ss2.x + ss2.y;
      sr[NS + s] = raw2.x + raw2.y;
    }
  }
  const float sr_l = warp_reduce_many<2 * NS>(sr, lane);
  if (lane < 2 * NS) red_sr[ty][warp][lane] = sr_l;
  if constexpr (NP > 0) cp_async_wait_all();  // the router weight, visible after the barrier
  __syncthreads();

  // 3. scores and softmax: lane s of every warp scores source s (the warps'
  // partials added in warp order), the max over lanes, its exponential; each
  // thread gathers the S exponentials and sums them in source order, so all
  // threads agree bit for bit.  Short dependent chains matter here (a few
  // warps per SM): one reciprocal for the mean, one for the denominator, the
  // fast exp.
  const float inv_dim = 1.0f / (float)dim;
  float score = -INFINITY;
  if (lane < S) {
    float tss = 0.f, traw = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      tss += red_sr[ty][w][lane];
      traw += red_sr[ty][w][NS + lane];
    }
    score = rsqrtf(tss * inv_dim + a.key_eps) * traw;
  }
  const float m = warp_max(score);
  const float e_l = lane < S ? __expf(score - m) : 0.f;
  float alpha[NS];
  float den = 0.f;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    alpha[s] = __shfl_sync(0xffffffffu, e_l, s);
    den += alpha[s];
  }
  const float rden = 1.0f / den;
  float2 h2[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) h2[p] = make_float2(0.f, 0.f);
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    if (s < S) {
      const float al = alpha[s] * rden;
      const float2 al2 = make_float2(al, al);
      const uint4 sv = source(s);
      const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) h2[p] = __ffma2_rn(al2, bf16x2_to_float2(w[p]), h2[p]);
    }
  }
  float h[8];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    h[2 * p] = h2[p].x;
    h[2 * p + 1] = h2[p].y;
  }
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    h[j] = round_bf16(h[j]);
    sq = fmaf(h[j], h[j], sq);
  }
  if (active && a.mix_out != nullptr) reinterpret_cast<uint4*>(a.mix_out + off)[c] = float_to_bf16x8(h);
  if (a.out_w == nullptr) {
    if (active) reinterpret_cast<uint4*>(a.out + off)[c] = float_to_bf16x8(h);
    return;
  }
  // 4. the consumer RMSNorm
  sq = warp_sum(sq);
  if (lane == 0) red_sq[ty][warp] = sq;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) total += red_sq[ty][w];
  const float inv = rsqrtf(total / (float)dim + a.out_eps);
  float gb[8];  // the output as the bf16 tensor it is
  uint4 ov = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int j = 0; j < 8; ++j) gb[j] = 0.f;
  if (active) {
    float g[8];
    bf16x8_to_float(owv, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = (h[j] * inv) * g[j];
    ov = float_to_bf16x8(g);
    reinterpret_cast<uint4*>(a.out + off)[c] = ov;
    bf16x8_to_float(ov, gb);
  }
  if constexpr (NP > 0) {
    // 5. the router (MoE.forward's logits / softmax / top-2, model.py:521-527)
    extern __shared__ __align__(16) uint4 dm_rw[];
    __shared__ float red_r[R][W][NP];
    __shared__ float psum[R][NP];
    __shared__ int hist[NP];
    __shared__ int slot_row[R][2];  // slot mode: the grouped rows of this row's two assignments
    const int E = ra.r.n_experts;
    if (ty == 0 && c < NP) hist[c] = 0;
    float pr[NP];
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      pr[e] = 0.f;
      if (active && e < E) {
        const uint4 w = dm_rw[e * nvec + c];
        float2 t2 = make_float2(0.f, 0.f);
        t2 = __ffma2_rn(bf16x2_to_float2(w.x), make_float2(gb[0], gb[1]), t2);
        t2 = __ffma2_rn(bf16x2_to_float2(w.y), make_float2(gb[2], gb[3]), t2);
        t2 = __ffma2_rn(bf16x2_to_float2(w.z), make_float2(gb[4], gb[5]), t2);
        t2 = __ffma2_rn(bf16x2_to_float2(w.w), make_float2(gb[6], gb[7]), t2);
        pr[e] = t2.x + t2.y;
      }
    }
    const float wsum = warp_reduce_many<NP>(pr, lane);
    if (lane < NP) red_r[ty][warp][lane] = wsum;
    __syncthreads();
    if (warp == 0) {
      const int ex = lane % NP;
      const bool valid_e = ex < E, valid_t = row < a.rows;
      float logit = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) logit += red_r[ty][w][ex];
      if (ra.r.bias != nullptr && valid_e) logit += __ldg(ra.r.bias + ex);
      float m = valid_e ? logit : -INFINITY;
#pragma unroll
      for (int o = NP / 2; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float p = valid_e ? __expf(logit - m) : 0.f;
      float den = p;
#pragma unroll
      for (int o = NP / 2; o >= 1; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
      p = valid_t ? p * (1.0f / den) : 0.f;
      float v1 = valid_e ? p : -1.f;
      int i1 = ex;
      best_of_group<NP>(v1, i1);
      float v2 = (valid_e && ex != i1) ? p : -1.f;
      int i2 = ex;
      best_of_group<NP>(v2, i2);
      if (valid_t && lane == 0) {
        const float sel = v1 + v2;
        const float w1 = v1 / sel, w2 = v2 / sel;
        reinterpret_cast<int2*>(ra.r.indices)[row] = make_int2(i1, i2);
        reinterpret_cast<float2*>(ra.r.weights)[row] = make_float2(w1, w2);
        if (ra.r.weights_out != nullptr)
          reinterpret_cast<float2*>(ra.r.weights_out)[row] = make_float2(w1, w2);
        if (ra.r.indices64 != nullptr) {
          ra.r.indices64[2 * row] = i1;
          ra.r.indices64[2 * row + 1] = i2;
        }
        atomicAdd(&hist[i1], 1);
        atomicAdd(&hist[i2], 1);
        if (ra.r.slot_counts != nullptr) {
          // the grouping: the next free slot of each expert, then the row's
          // position, contribution slot (the lower expert id first) and weight
          const int s1 = atomicAdd(ra.r.slot_counts + i1, 1);
          const int s2 = atomicAdd(ra.r.slot_counts + i2, 1);
          int r1 = i1 * ra.r.slot_stride + s1, r2 = i2 * ra.r.slot_stride + s2;
          if (s1 >= ra.r.slot_stride || s2 >= ra.r.slot_stride) {
            // counters left over from a routing call whose block never ran:
            // nothing is written past the expert's region
            report_status(ra.r.status, kStatusBadIndex, 50, max(s1, s2));
            r1 = r2 = -1;
          } else {
            reinterpret_cast<int2*>(ra.r.positions)[row] = make_int2(r1, r2);
            ra.r.row_dst[r1] = 2 * row + (i1 < i2 ? 0 : 1);
            ra.r.row_dst[r2] = 2 * row + (i2 < i1 ? 0 : 1);
            ra.r.row_w[r1] = w1;
            ra.r.row_w[r2] = w2;
          }
          slot_row[ty][0] = r1;
          slot_row[ty][1] = r2;
        }
      }
      if (valid_t && valid_e && lane < NP && ra.r.probs != nullptr)
        ra.r.probs[(size_t)row * E + ex] = p;
      if (lane < NP) psum[ty][lane] = p;
    }
    __syncthreads();
    if (ra.r.slot_counts != nullptr && active && row < a.rows && slot_row[ty][0] >= 0) {
      // this thread's 16 bytes of the row, into both grouped rows
      const size_t nv = (size_t)nvec;
      reinterpret_cast<uint4*>(ra.r.grouped)[(size_t)slot_row[ty][0] * nv + c] = ov;
      reinterpret_cast<uint4*>(ra.r.grouped)[(size_t)slot_row[ty][1] * nv + c] = ov;
    }
    if (ty == 0 && c < E) {
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < R; ++k) sum += psum[k][c];
      ra.r.tab.tile_hist[(size_t)blockIdx.x * E + c] = hist[c];
      ra.r.tab.tile_probsum[(size_t)blockIdx.x * E + c] = sum;
    }
  }
}

// The plain depth mix at large row counts (no deferred source, no router):
// each thread takes its 16-byte vector of two rows, so the per-CTA work that
// does not depend on the row (the query and norm weights, their products,
// the launch and the block barriers) is shared by two rows and the two rows'
// chains interleave.  Every row's arithmetic is the one-row kernel's, in the
// same order (bit-identical outputs).
template <int W, int NS>
__global__ void __launch_bounds__(32 * W, 4)
    depthmix2_kernel(DepthMixArgs a) {
  __shared__ float red_sr[2][W][2 * NS], red_sq[2][W];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = threadIdx.x;
  const int dim = a.dim, nvec = dim >> 3, S = a.n_sources;
  const int row0 = 2 * blockIdx.x;
  bool active[2];
  size_t off[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    active[u] = c < nvec && row0 + u < a.rows;
    off[u] = (size_t)(row0 + u) * dim;
  }
  float q[8], kw[8];
  uint4 owv = make_uint4(0, 0, 0, 0);
  if (c < nvec) {
    bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.query) + c), q);
    bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.key_w) + c), kw);
    if (a.out_w != nullptr) owv = __ldg(reinterpret_cast<const uint4*>(a.out_w) + c);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = kw[j] = 0.f;
  }
  griddep_wait();
  griddep_launch();

  uint4 v[2][NS];
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      v[u][s] = make_uint4(0, 0, 0, 0);
      if (s < S && active[u]) v[u][s] = __ldg(reinterpret_cast<const uint4*>(a.sources[s] + off[u]) + c);
    }
  float2 kq[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) kq[p] = make_float2(kw[2 * p] * q[2 * p], kw[2 * p + 1] * q[2 * p + 1]);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    float sr[2 * NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      sr[s] = 0.f;
      sr[NS + s] = 0.f;
      if (s < S) {
        const uint32_t w[4] = {v[u][s].x, v[u][s].y, v[u][s].z, v[u][s].w};
        float2 ss2 = make_float2(0.f, 0.f), raw2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 f2 = bf16x2_to_float2(w[p]);
          ss2 = __ffma2_rn(f2, f2, ss2);
          raw2 = __ffma2_rn(f2, kq[p], raw2);
        }
        sr[s] = ss2.x + ss2.y;
        sr[NS + s] = raw2.x + raw2.y;
      }
    }
    const float sr_l = warp_reduce_many<2 * NS>(sr, lane);
    if (lane < 2 * NS) red_sr[u][warp][lane] = sr_l;
  }
  __syncthreads();
  const float inv_dim = 1.0f / (float)dim;
  float h[2][8], sq[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    float score = -INFINITY;
    if (lane < S) {
      float tss = 0.f, traw = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        tss += red_sr[u][w][lane];
        traw += red_sr[u][w][NS + lane];
      }
      score = rsqrtf(tss * inv_dim + a.key_eps) * traw;
    }
    const float m = warp_max(score);
    const float e_l = lane < S ? __expf(score - m) : 0.f;
    float alpha[NS];
    float den = 0.f;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      alpha[s] = __shfl_sync(0xffffffffu, e_l, s);
      den += alpha[s];
    }
    const float rden = 1.0f / den;
    float2 h2[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) h2[p] = make_float2(0.f, 0.f);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      if (s < S) {
        const float al = alpha[s] * rden;
        const float2 al2 = make_float2(al, al);
        const uint32_t w[4] = {v[u][s].x, v[u][s].y, v[u][s].z, v[u][s].w};
#pragma unroll
        for (int p = 0; p < 4; ++p) h2[p] = __ffma2_rn(al2, bf16x2_to_float2(w[p]), h2[p]);
      }
    }
    sq[u] = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      h[u][2 * p] = round_bf16(h2[p].x);
      h[u][2 * p + 1] = round_bf16(h2[p].y);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sq[u] = fmaf(h[u][j], h[u][j], sq[u]);
    if (active[u] && a.mix_out != nullptr)
      reinterpret_cast<uint4*>(a.mix_out + off[u])[c] = float_to_bf16x8(h[u]);
    if (a.out_w == nullptr) {
      if (active[u]) reinterpret_cast<uint4*>(a.out + off[u])[c] = float_to_bf16x8(h[u]);
    } else {
      sq[u] = warp_sum(sq[u]);
      if (lane == 0) red_sq[u][warp] = sq[u];
    }
  }
  if (a.out_w == nullptr) return;
  __syncthreads();
  float g[8];
  bf16x8_to_float(owv, g);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) total += red_sq[u][w];
    const float inv = rsqrtf(total / (float)dim + a.out_eps);
    if (active[u]) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (h[u][j] * inv) * g[j];
      reinterpret_cast<uint4*>(a.out + off[u])[c] = float_to_bf16x8(o);
    }
  }
}

// rows from which the two-row kernel takes the plain mix, up to 4 sources (at
// 32768 rows: 4 sources 69.2 -> 61.8 us; 8 sources measured 109.0 against
// 102.9 us, its 118 registers leaving too few warps per SM)
constexpr int kDepthMixTwoRowsFrom = 8192;

template <int W>
static int launch_depthmix_w(const DepthMixArgs& args, cudaStream_t stream) {
  const dim3 grid(args.rows), block(32 * W);
  const int S = args.n_sources;
  const DepthRouteArgs none{};
  cudaError_t e;
  const bool plain = args.pending_delta == nullptr && args.pending_contrib == nullptr;
  if (plain && args.rows >= kDepthMixTwoRowsFrom && S <= 4) {
    const dim3 grid2((args.rows + 1) / 2);
    if (S <= 2) e = launch_pdl(depthmix2_kernel<W, 2>, grid2, block, 0, stream, args);
    else e = launch_pdl(depthmix2_kernel<W, 4>, grid2, block, 0, stream, args);
    return e == cudaSuccess ? 0 : -2;
  }
  if (S <= 2) e = launch_pdl(depthmix_kernel<W, 2, 1, 0>, grid, block, 0, stream, args, none);
  else if (S <= 4) e = launch_pdl(depthmix_kernel<W, 4, 1, 0>, grid, block, 0, stream, args, none);
  else if (S <= 8) e = launch_pdl(depthmix_kernel<W, 8, 1, 0>, grid, block, 0, stream, args, none);
  else
    e = launch_pdl(depthmix_kernel<W, kMaxDepthSources, 1, 0>, grid, block, 0, stream, args, none);
  return e == cudaSuccess ? 0 : -2;
}

template <int W, int NS, int NP>
static cudaError_t launch_depthmix_route_k(const DepthMixArgs& args, const DepthRouteArgs& route,
                                           cudaStream_t stream) {
  constexpr int R = kRouteSmallTile;
  static unsigned long long configured = 0;  // per device: the router weight may exceed 48 KB
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!(configured & (1ull << dev))) {
    const cudaError_t e = cudaFuncSetAttribute(
        depthmix_kernel<W, NS, R, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (e != cudaSuccess) return e;
    configured |= 1ull << dev;
  }
  const size_t smem = (size_t)route.r.n_experts * args.dim * 2;
  return launch_pdl(depthmix_kernel<W, NS, R, NP>, dim3((args.rows + R - 1) / R),
                    dim3(32 * W, R), smem, stream, args, route);
}

template <int W, int NP>
static int launch_depthmix_route_w(const DepthMixArgs& args, const DepthRouteArgs& route,
                                   cudaStream_t stream) {
  const int S = args.n_sources;
  cudaError_t e;
  if (S <= 2) e = launch_depthmix_route_k<W, 2, NP>(args, route, stream);
  else if (S <= 4) e = launch_depthmix_route_k<W, 4, NP>(args, route, stream);
  else if (S <= 8) e = launch_depthmix_route_k<W, 8, NP>(args, route, stream);
  else e = launch_depthmix_route_k<W, kMaxDepthSources, NP>(args, route, stream);
  return e == cudaSuccess ? 0 : -2;
}

template <int NP>
static int launch_depthmix_route_np(const DepthMixArgs& args, const DepthRouteArgs& route,
                                    cudaStream_t stream) {
  switch ((args.dim / 8 + 31) / 32) {
    case 1: return launch_depthmix_route_w<1, NP>(args, route, stream);
    case 2: return launch_depthmix_route_w<2, NP>(args, route, stream);
    case 3: return launch_depthmix_route_w<3, NP>(args, route, stream);
    case 4: return launch_depthmix_route_w<4, NP>(args, route, stream);
    default: return -1;
  }
}

int launch_depthmix_route(const DepthMixArgs& args, const DepthRouteArgs& route,
                          cudaStream_t stream) {
  if (args.rows == 0) return 0;
  if (args.n_sources < 1 || args.n_sources > kMaxDepthSources || args.out_w == nullptr ||
      route.r.tokens != args.rows || route_tile(args.rows) != kRouteSmallTile)
    return -1;
  return route_experts_padded(route.r.n_experts) == 16
             ? launch_depthmix_route_np<16>(args, route, stream)
             : launch_depthmix_route_np<32>(args, route, stream);
}

int launch_depthmix(const DepthMixArgs& args, cudaStream_t stream) {
  if (args.rows == 0) return 0;
  if (args.n_sources < 1 || args.n_sources > kMaxDepthSources) return -1;
  switch ((args.dim / 8 + 31) / 32) {
    case 1: return launch_depthmix_w<1>(args, stream);
    case 2: return launch_depthmix_w<2>(args, stream);
    case 3: return launch_depthmix_w<3>(args, stream);
    case 4: return launch_depthmix_w<4>(args, stream);
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
// start_dev (optional) holds the first position in device memory (decode
// steps replayed from a graph); a position past the tables is reported and
// the row left unrotated.
__global__ void __launch_bounds__(256) rope_kernel(__nv_bfloat16* __restrict__ x,
                                                   const __nv_bfloat16* __restrict__ cos_t,
                                                   const __nv_bfloat16* __restrict__ sin_t,
                                                   int rows, int row_stride, int rot_cols,
                                                   int head_dim, int seq_len, int start,
                                                   const int* start_dev, int max_positions,
                                                   int* status) {
  griddep_wait();
  griddep_launch();
  const int vec_per_row = rot_cols >> 3;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * vec_per_row) return;
  const int r = (int)(i / vec_per_row), v = (int)(i % vec_per_row);
  const int col = v * 8;
  const int pos = (start_dev != nullptr ? __ldg(start_dev) : start) + r % seq_len;
  if (pos < 0 || pos >= max_positions) {
    report_status(status, kStatusBadIndex, 41, pos);
    return;
  }
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
                const int* start_dev, int max_positions, int* status, cudaStream_t stream) {
  const long long total = (long long)rows * (rot_cols / 8);
  if (total == 0) return 0;
  const int threads = 256;
  return launch_pdl(rope_kernel, dim3((unsigned)((total + threads - 1) / threads)),
                    dim3(threads), 0, stream, x, cos_t, sin_t, rows, row_stride, rot_cols,
                    head_dim, seq_len, start, start_dev, max_positions, status) == cudaSuccess
             ? 0
             : -2;
}

}  // namespace parrot
