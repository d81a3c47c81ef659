// Router (N1) and deterministic capacity grouping (N2).
//
// route_kernel:  fp32 router logits + softmax + top-2 + renormalised weights,
//                one warp per token, router weight staged in shared memory.
//                Each block also counts its assignments per expert and sums
//                its probabilities per expert; the last block to finish (a
//                ticket counter, no spinning) turns those into exclusive
//                per-block prefixes, segment tables and router statistics.
// group_kernel:  ranks each assignment inside its block with warp match,
//                adds the block prefix -> a stable slot (ascending token order
//                within each expert, the reference's torch.where order), maps
//                slot -> grouped row (capacity region, else the overflow
//                region), and copies the token rows with 16-byte vectors.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

constexpr int kRouteWarps = 8;
constexpr int kTokensPerWarp = kRouteTokensPerBlock / kRouteWarps;

template <int V>
__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* w_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __shared__ int hist_s[kMaxExperts];
  __shared__ float psum_s[kRouteWarps][kMaxExperts];
  __shared__ int last_s;

  const int E = a.n_experts, d = a.dim, T = a.tokens;
  const int nvec = d >> 3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;

  // stage the router weight [E, d]
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.w);
    uint4* dst = reinterpret_cast<uint4*>(w_s);
    for (int i = threadIdx.x; i < E * nvec; i += blockDim.x) dst[i] = __ldg(src + i);
    if (threadIdx.x < kMaxExperts) hist_s[threadIdx.x] = 0;
  }
  __syncthreads();

  float psum_lane = 0.f;  // lane e accumulates p[e] over this warp's tokens
  for (int j = 0; j < kTokensPerWarp; ++j) {
    const int t = blk * kRouteTokensPerBlock + warp * kTokensPerWarp + j;
    if (t >= T) break;
    float xf[V][8];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.x + (size_t)t * d) + c), xf[i]);
    }
    float logit[kMaxExperts];
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) {
      if (e < E) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int c = lane + 32 * i;
          if (c < nvec) {
            float wf[8];
            bf16x8_to_float(reinterpret_cast<const uint4*>(w_s + (size_t)e * d)[c], wf);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc = fmaf(xf[i][k], wf[k], acc);
          }
        }
        acc = warp_sum(acc);
        if (a.bias != nullptr) acc += __ldg(a.bias + e);
        logit[e] = acc;
      } else {
        logit[e] = -INFINITY;
      }
    }
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) m = fmaxf(m, logit[e]);
    float den = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) {
      logit[e] = (e < E) ? expf(logit[e] - m) : 0.f;
      den += logit[e];
    }
    // probabilities, top-2 on them (strict '>' so the lower expert id wins ties)
    int first = 0, second = -1;
    float pf = -1.f, ps = -1.f, mine = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) {
      if (e < E) {
        const float p = logit[e] / den;
        if (lane == e) mine = p;
        if (p > pf) {
          second = first; ps = pf; first = e; pf = p;
        } else if (p > ps) {
          second = e; ps = p;
        }
      }
    }
    if (lane < E) {
      psum_lane += mine;
      if (a.probs != nullptr) a.probs[(size_t)t * E + lane] = mine;
    }
    if (lane == 0) {
      const float sel = pf + ps;
      a.indices[2 * t] = first;
      a.indices[2 * t + 1] = second;
      a.weights[2 * t] = pf / sel;
      a.weights[2 * t + 1] = ps / sel;
      if (a.indices64 != nullptr) {
        a.indices64[2 * t] = first;
        a.indices64[2 * t + 1] = second;
      }
      atomicAdd(&hist_s[first], 1);
      atomicAdd(&hist_s[second], 1);
    }
  }
  if (lane < kMaxExperts) psum_s[warp][lane] = psum_lane;
  __syncthreads();
  if (threadIdx.x < E) {
    float s = 0.f;
    for (int w = 0; w < kRouteWarps; ++w) s += psum_s[w][threadIdx.x];
    a.tab.block_hist[blk * E + threadIdx.x] = hist_s[threadIdx.x];
    a.tab.block_probsum[blk * E + threadIdx.x] = s;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(a.tab.done_counter, 1);
    last_s = (ticket == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();

  // ---- last block: one warp per expert builds the exclusive prefix over
  // blocks (warp scan, 32 blocks per step) and the probability column sum
  // (lane partials in block order, then a fixed-order tree: deterministic).
  const int nb = gridDim.x;
  __shared__ int count_s[kMaxExperts];
  __shared__ float psum_e[kMaxExperts];
  for (int e = warp; e < E; e += kRouteWarps) {
    int carry = 0;
    float ps = 0.f;
    for (int base = 0; base < nb; base += 32) {
      const int b = base + lane;
      const int v = (b < nb) ? __ldcg(a.tab.block_hist + b * E + e) : 0;
      if (b < nb) ps += __ldcg(a.tab.block_probsum + b * E + e);
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (b < nb) a.tab.block_prefix[b * E + e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    ps = warp_sum(ps);
    if (lane == 0) {
      count_s[e] = carry;
      psum_e[e] = ps;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int C = a.capacity;
    const int A = 2 * T;
    int overflow_base = E * C;
    float aux = 0.f;
    for (int e = 0; e < E; ++e) {
      const int c = count_s[e];
      a.tab.counts[e] = c;
      a.tab.seg_rows[e] = c < C ? c : C;
      a.tab.seg_base[e] = e * C;
      const int ov = c > C ? c - C : 0;
      a.tab.seg_rows[E + e] = ov;
      a.tab.seg_base[E + e] = overflow_base;
      overflow_base += ov;
      const float util = (float)c / (float)A;
      a.tab.stats[e] = util;
      aux += util * (psum_e[e] / (float)T);
    }
    a.tab.stats[E] = (float)E * aux;
    *a.tab.done_counter = 0;  // ready for the next launch
  }
}

int launch_route(const RouteArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  const int nb = route_blocks(args.tokens);
  const size_t smem = (size_t)args.n_experts * args.dim * sizeof(__nv_bfloat16);
  const int v = (args.dim / 8 + 31) / 32;
  switch (v) {
#define PARROT_ROUTE_CASE(VV)                                                             \
  case VV: {                                                                              \
    if (smem > 48 * 1024)                                                                 \
      cudaFuncSetAttribute(route_kernel<VV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)smem);                                                    \
    route_kernel<VV><<<nb, 256, smem, stream>>>(args);                                    \
    break;                                                                                \
  }
    PARROT_ROUTE_CASE(1)
    PARROT_ROUTE_CASE(2)
    PARROT_ROUTE_CASE(3)
    PARROT_ROUTE_CASE(4)
#undef PARROT_ROUTE_CASE
    default: return -1;
  }
  return 0;
}

// ---------------------------------------------------------------------------
// grouping: stable slots and the 16-byte row scatter
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) group_kernel(GroupArgs a) {
  constexpr int kAssign = 2 * kRouteTokensPerBlock;  // 64 per block
  __shared__ int warp_cnt[2][kMaxExperts];
  __shared__ int row_s[kAssign];
  const int E = a.n_experts, C = a.capacity, T = a.tokens, d = a.dim;
  const int blk = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid < 2 * kMaxExperts) (&warp_cnt[0][0])[tid] = 0;
  __syncthreads();

  int e = -1, rank = 0;
  const int a_idx = blk * kAssign + tid;
  if (warp < 2) {
    if (a_idx < 2 * T) {
      e = __ldg(a.indices + a_idx);
      if (e < 0 || e >= E) {
        report_status(a.status, kStatusBadIndex, 1, a_idx);
        e = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(peers) - 1) warp_cnt[warp][e] = __popc(peers);
  }
  __syncthreads();
  if (warp < 2) {
    int row = -1;
    if (e >= 0) {
      const int slot = a.tab.block_prefix[blk * E + e] + (warp == 1 ? warp_cnt[0][e] : 0) + rank;
      row = slot < C ? e * C + slot : a.tab.seg_base[E + e] + (slot - C);
      if (split == 0) a.positions[a_idx] = row;
    }
    row_s[tid] = row;
  }
  __syncthreads();

  // copy this split's share of the block's rows
  const int per = (kAssign + a.copy_split - 1) / a.copy_split;
  const int lo = split * per, hi = min(kAssign, lo + per);
  const int nvec = d >> 3;
  for (int j = lo + warp; j < hi; j += 4) {
    const int row = row_s[j];
    if (row < 0) continue;
    const int t = (blk * kAssign + j) >> 1;
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)t * d);
    uint4* dst = reinterpret_cast<uint4*>(a.grouped + (size_t)row * d);
    for (int c = lane; c < nvec; c += 32) dst[c] = __ldg(src + c);
  }
}

int launch_group(const GroupArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  dim3 grid(route_blocks(args.tokens), args.copy_split);
  group_kernel<<<grid, 128, 0, stream>>>(args);
  return 0;
}

// ---------------------------------------------------------------------------
// combine (N6): out = [residual +] (shared + sum_k bf16(y_k * bf16(w_k)))
// Contributions are added in ascending expert id, each sum rounded to bf16:
// the reference's index_add sequence (model.py:546-551), then the residual
// add of model.py:702 / :585.
// ---------------------------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(128) combine_kernel(CombineArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= a.tokens) return;
  const int d = a.dim, nvec = d >> 3;
  int e0 = __ldg(a.indices + 2 * t), e1 = __ldg(a.indices + 2 * t + 1);
  int r0 = __ldg(a.positions + 2 * t), r1 = __ldg(a.positions + 2 * t + 1);
  float w0 = round_bf16(__ldg(a.weights + 2 * t)), w1 = round_bf16(__ldg(a.weights + 2 * t + 1));
  if (e1 < e0) {  // lower expert id is added first
    int ti = r0; r0 = r1; r1 = ti;
    float tf = w0; w0 = w1; w1 = tf;
  }
  const uint4* ya = reinterpret_cast<const uint4*>(a.y + (size_t)r0 * d);
  const uint4* yb = reinterpret_cast<const uint4*>(a.y + (size_t)r1 * d);
  const uint4* sh = reinterpret_cast<const uint4*>(a.shared_y + (size_t)t * d);
  const uint4* rs = a.residual ? reinterpret_cast<const uint4*>(a.residual + (size_t)t * d) : nullptr;
  uint4* o = reinterpret_cast<uint4*>(a.out + (size_t)t * d);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float s[8], p[8], q[8];
      bf16x8_to_float(__ldg(sh + c), s);
      bf16x8_to_float(__ldg(ya + c), p);
      bf16x8_to_float(__ldg(yb + c), q);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float r = round_bf16(s[k] + round_bf16(p[k] * w0));
        s[k] = round_bf16(r + round_bf16(q[k] * w1));
      }
      if (rs != nullptr) {
        float b[8];
        bf16x8_to_float(__ldg(rs + c), b);
#pragma unroll
        for (int k = 0; k < 8; ++k) s[k] = b[k] + s[k];
      }
      o[c] = float_to_bf16x8(s);
    }
  }
}

int launch_combine(const CombineArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  const int warps = 4;
  dim3 grid((args.tokens + warps - 1) / warps), block(32 * warps);
  const int v = (args.dim / 8 + 31) / 32;
  switch (v) {
    case 1: combine_kernel<1><<<grid, block, 0, stream>>>(args); break;
    case 2: combine_kernel<2><<<grid, block, 0, stream>>>(args); break;
    case 3: combine_kernel<3><<<grid, block, 0, stream>>>(args); break;
    case 4: combine_kernel<4><<<grid, block, 0, stream>>>(args); break;
    default: return -1;
  }
  return 0;
}

}  // namespace parrot
