// Router (N1) and deterministic capacity grouping (N2).
//
// route_kernel:  fp32 router logits + softmax + top-2 + renormalised weights,
//                one warp per two tokens from shared-memory staged inputs,
//                lane-parallel over experts.
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

constexpr int kRouteWarps = 4;
constexpr int kTokensPerWarp = kRouteTokensPerBlock / kRouteWarps;  // 2
constexpr int kRouteBlocksPerGroup = kGroupTokensPerBlock / kRouteTokensPerBlock;  // 4

// One warp routes kTokensPerWarp tokens.  The block first stages the router
// weight [E, d] and its 32 token rows in shared memory with 16-byte async
// copies (every load in flight at once), then lanes split d and accumulate
// all E partial dot products, reduced together (warp_reduce_many); after that
// lane l owns expert l % EP for the softmax and the top-2 search.
template <int V, int EP>
__global__ void __launch_bounds__(32 * kRouteWarps) route_kernel(RouteArgs a) {
  extern __shared__ __align__(16) unsigned char route_smem[];
  __shared__ int hist_s[kMaxExperts];
  __shared__ float psum_s[kRouteWarps][kMaxExperts];
  __shared__ int last_s;

  const int E = a.n_experts, d = a.dim, T = a.tokens;
  const int nvec = d >> 3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  uint4* w_s = reinterpret_cast<uint4*>(route_smem);            // [E][nvec]
  uint4* x_s = w_s + (size_t)E * nvec;                          // [32][nvec]
  {
    // the router weight is a parameter: fetch it before the upstream kernel ends
    const uint4* wg = reinterpret_cast<const uint4*>(a.w);
    for (int i = threadIdx.x; i < E * nvec; i += blockDim.x) cp_async16(w_s + i, wg + i);
    griddep_wait();
    griddep_launch();
    const int first = blk * kRouteTokensPerBlock;
    const int rows = min(kRouteTokensPerBlock, T - first);
    const uint4* xg = reinterpret_cast<const uint4*>(a.x + (size_t)first * d);
    for (int i = threadIdx.x; i < rows * nvec; i += blockDim.x) cp_async16(x_s + i, xg + i);
    if (threadIdx.x < kMaxExperts) hist_s[threadIdx.x] = 0;
    cp_async_wait_all();
  }
  __syncthreads();

  const int t0 = blk * kRouteTokensPerBlock + warp * kTokensPerWarp;
  float xf[kTokensPerWarp][V][8];
#pragma unroll
  for (int j = 0; j < kTokensPerWarp; ++j)
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = lane + 32 * i;
      if (t0 + j < T && c < nvec)
        bf16x8_to_float(x_s[(warp * kTokensPerWarp + j) * nvec + c], xf[j][i]);
      else
#pragma unroll
        for (int k = 0; k < 8; ++k) xf[j][i][k] = 0.f;
    }
  float part[kTokensPerWarp][EP];
#pragma unroll
  for (int j = 0; j < kTokensPerWarp; ++j)
#pragma unroll
    for (int e = 0; e < EP; ++e) part[j][e] = 0.f;
#pragma unroll
  for (int e = 0; e < EP; ++e) {
    if (e < E) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) {
          float wf[8];
          bf16x8_to_float(w_s[e * nvec + c], wf);
#pragma unroll
          for (int j = 0; j < kTokensPerWarp; ++j)
#pragma unroll
            for (int k = 0; k < 8; ++k) part[j][e] = fmaf(xf[j][i][k], wf[k], part[j][e]);
        }
      }
    }
  }

  const int my_e = lane & (EP - 1);
  const bool valid = my_e < E;
  float psum_lane = 0.f;
#pragma unroll
  for (int j = 0; j < kTokensPerWarp; ++j) {
    const int t = t0 + j;
    float logit = warp_reduce_many<EP>(part[j], lane);
    if (t >= T) continue;  // warp-uniform
    if (a.bias != nullptr && valid) logit += __ldg(a.bias + my_e);
    const float m = warp_max(valid ? logit : -INFINITY);
    const float ex = valid ? expf(logit - m) : 0.f;
    const float den = warp_sum(lane < EP ? ex : 0.f);
    const float p = ex / den;
    // top-2 on the probabilities; equal values resolve to the lower expert id
    float v1 = valid ? p : -1.f;
    int i1 = my_e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v1, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i1, o);
      if (ov > v1 || (ov == v1 && oi < i1)) { v1 = ov; i1 = oi; }
    }
    float v2 = (valid && my_e != i1) ? p : -1.f;
    int i2 = my_e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v2, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i2, o);
      if (ov > v2 || (ov == v2 && oi < i2)) { v2 = ov; i2 = oi; }
    }
    if (lane < E) {
      psum_lane += p;
      if (a.probs != nullptr) a.probs[(size_t)t * E + lane] = p;
    }
    if (lane == 0) {
      const float sel = v1 + v2;
      a.indices[2 * t] = i1;
      a.indices[2 * t + 1] = i2;
      a.weights[2 * t] = v1 / sel;
      a.weights[2 * t + 1] = v2 / sel;
      if (a.weights_out != nullptr) {
        a.weights_out[2 * t] = v1 / sel;
        a.weights_out[2 * t + 1] = v2 / sel;
      }
      if (a.indices64 != nullptr) {
        a.indices64[2 * t] = i1;
        a.indices64[2 * t + 1] = i2;
      }
      atomicAdd(&hist_s[i1], 1);
      atomicAdd(&hist_s[i2], 1);
    }
  }
  psum_s[warp][lane] = psum_lane;
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
  // grouping blocks (each the sum of 4 router blocks; warp scan, 32 grouping
  // blocks per step) and the probability column sum (lane partials in block
  // order, then a fixed-order tree: deterministic).
  const int nb = gridDim.x;
  const int ng = (nb + kRouteBlocksPerGroup - 1) / kRouteBlocksPerGroup;
  __shared__ int count_s[kMaxExperts];
  __shared__ float psum_e[kMaxExperts];
  for (int e = warp; e < E; e += kRouteWarps) {
    int carry = 0;
    float ps = 0.f;
    for (int base = 0; base < ng; base += 32) {
      const int gb = base + lane;
      int v = 0;
#pragma unroll
      for (int r = 0; r < kRouteBlocksPerGroup; ++r) {
        const int b = gb * kRouteBlocksPerGroup + r;
        if (gb < ng && b < nb) {
          v += __ldcg(a.tab.block_hist + b * E + e);
          ps += __ldcg(a.tab.block_probsum + b * E + e);
        }
      }
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (gb < ng) a.tab.block_prefix[gb * E + e] = carry + incl - v;
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
    const int G = a.ep_ranks, El = E / G;
    int overflow_base = E * C;
    for (int q = 0; q < E; ++q) {
      const int e = (q % El) * G + q / El;  // rank q / El, local expert q % El
      const int ov = count_s[e] > C ? count_s[e] - C : 0;
      a.tab.seg_rows[E + e] = ov;
      a.tab.seg_base[E + e] = overflow_base;
      overflow_base += ov;
    }
    float aux = 0.f;
    for (int e = 0; e < E; ++e) {
      const int c = count_s[e];
      a.tab.counts[e] = c;
      if (a.counts_out != nullptr) a.counts_out[e] = c;
      a.tab.seg_rows[e] = c < C ? c : C;
      a.tab.seg_base[e] = e * C;
      const float util = (float)c / (float)A;
      a.tab.stats[e] = util;
      if (a.stats_out != nullptr) a.stats_out[e] = util;
      aux += util * (psum_e[e] / (float)T);
    }
    a.tab.stats[E] = (float)E * aux;
    if (a.stats_out != nullptr) a.stats_out[E] = (float)E * aux;
    *a.tab.done_counter = 0;  // ready for the next launch
  }
}

template <int V, int EP>
static int launch_route_ve(const RouteArgs& args, int nb, cudaStream_t stream) {
  const size_t smem = (size_t)(args.n_experts + kRouteTokensPerBlock) * (args.dim / 8) * 16;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    const int max_smem = (kMaxExperts + kRouteTokensPerBlock) * (1024 / 8) * 16;
    if (cudaFuncSetAttribute(route_kernel<V, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_smem) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  return launch_pdl(route_kernel<V, EP>, dim3(nb), dim3(32 * kRouteWarps), smem, stream, args) ==
                 cudaSuccess ? 0 : -2;
}

template <int V>
static int launch_route_v(const RouteArgs& args, int nb, cudaStream_t stream) {
  return args.n_experts <= 16 ? launch_route_ve<V, 16>(args, nb, stream)
                              : launch_route_ve<V, 32>(args, nb, stream);
}

int launch_route(const RouteArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  const int nb = route_blocks(args.tokens);
  switch ((args.dim / 8 + 31) / 32) {
    case 1: return launch_route_v<1>(args, nb, stream);
    case 2: return launch_route_v<2>(args, nb, stream);
    case 3: return launch_route_v<3>(args, nb, stream);
    case 4: return launch_route_v<4>(args, nb, stream);
    default: return -1;
  }
}

// ---------------------------------------------------------------------------
// grouping: stable slots and the 16-byte row scatter
//
// Block b owns assignments [64 b, 64 b + 64) (tokens [32 b, 32 b + 32)); its
// exclusive per-expert prefix comes from the router's last block.
// Everything independent is requested up front: the assignment expert ids,
// this block's exclusive prefix and the overflow bases, and (async copies)
// the token rows this split copies.  Then ranks come from warp match, and
// every assignment's grouped row is written along with where its expert
// output goes (token-major slot 2 t + j, j = 0 for the lower expert id of
// the token's pair, the order the reference adds them) and its route weight.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) group_kernel(GroupArgs a) {
  constexpr int kAssign = 2 * kGroupTokensPerBlock;  // 64 per block
  extern __shared__ __align__(16) unsigned char group_smem[];
  __shared__ int warp_cnt[2][kMaxExperts];
  __shared__ int prefix_s[kMaxExperts];
  __shared__ int obase_s[kMaxExperts];
  __shared__ int row_s[kAssign];
  const int E = a.n_experts, C = a.capacity, T = a.tokens, d = a.dim;
  const int blk = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = d >> 3;
  griddep_wait();
  griddep_launch();

  // this split's assignments [lo, hi) cover tokens [lo/2, hi/2) of the block
  const int per = (kAssign + a.copy_split - 1) / a.copy_split;
  const int lo = min(kAssign, split * per) & ~1, hi = min(kAssign, lo + per + (per & 1));
  const int tok_lo = blk * kGroupTokensPerBlock + lo / 2;
  const int n_tok = max(0, min(T - tok_lo, (hi - lo) / 2));
  uint4* x_s = reinterpret_cast<uint4*>(group_smem);
  {
    const uint4* xg = reinterpret_cast<const uint4*>(a.x + (size_t)tok_lo * d);
    for (int i = tid; i < n_tok * nvec; i += blockDim.x) cp_async16(x_s + i, xg + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int a_idx = blk * kAssign + tid;
  int e = -1;
  if (warp < 2 && a_idx < 2 * T) e = __ldg(a.indices + a_idx);
  if (tid >= 64 && tid < 64 + E) prefix_s[tid - 64] = __ldg(a.tab.block_prefix + blk * E + tid - 64);
  if (tid >= 96 && tid < 96 + E) obase_s[tid - 96] = __ldg(a.tab.seg_base + E + tid - 96);
  if (tid < 2 * kMaxExperts) (&warp_cnt[0][0])[tid] = 0;
  __syncthreads();

  int rank = 0;
  if (warp < 2) {
    if (e >= E || (e < 0 && a_idx < 2 * T)) {
      report_status(a.status, kStatusBadIndex, 1, a_idx);
      e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(peers) - 1) warp_cnt[warp][e] = __popc(peers);
  }
  __syncthreads();
  if (warp < 2) {
    const int partner = __shfl_xor_sync(0xffffffffu, e, 1);  // the token's other expert
    int row = -1;
    if (e >= 0) {
      const int slot = prefix_s[e] + (warp == 1 ? warp_cnt[0][e] : 0) + rank;
      row = slot < C ? e * C + slot : obase_s[e] + (slot - C);
      if (split == 0) {
        a.positions[a_idx] = row;
        if (a.positions_out != nullptr) a.positions_out[a_idx] = row;
        a.row_dst[row] = (a_idx & ~1) + (e < partner ? 0 : 1);
        a.row_w[row] = __ldg(a.weights + a_idx);
      }
    }
    row_s[tid] = row;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  // scatter this split's rows from shared memory
  for (int j = lo + warp; j < hi; j += 4) {
    const int row = row_s[j];
    const int lt = (j - lo) >> 1;
    if (row < 0 || lt >= n_tok) continue;
    uint4* dst = reinterpret_cast<uint4*>(a.grouped + (size_t)row * d);
    for (int c = lane; c < nvec; c += 32) dst[c] = x_s[lt * nvec + c];
  }
}

int launch_group(const GroupArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  dim3 grid(group_blocks(args.tokens), args.copy_split);
  const int per = (2 * kGroupTokensPerBlock + args.copy_split - 1) / args.copy_split;
  const size_t smem = (size_t)((per + (per & 1)) / 2) * (args.dim / 8) * 16;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kGroupTokensPerBlock * (1024 / 8) * 16) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  return launch_pdl(group_kernel, grid, dim3(128), smem, stream, args) == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------------------
// combine (N6): out = [residual +] bf16(bf16(shared + c_lo) + c_hi)
// The down-projection epilogue already wrote each routed contribution
// c = bf16(bf16(y) * bf16(w)) at token-major slot 2 t + j, j = 0 for the lower
// expert id: the reference's index_add sequence (model.py:546-551) adds the
// experts in ascending id, each sum rounded to bf16; then the residual add
// of model.py:702 / :585.  Pure streaming: no index loads.
// ---------------------------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(128) combine_kernel(CombineArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  griddep_wait();
  griddep_launch();
  if (t >= a.tokens) return;
  const int d = a.dim, nvec = d >> 3;
  const uint4* c0 = reinterpret_cast<const uint4*>(a.contrib + (size_t)(2 * t) * d);
  const uint4* c1 = reinterpret_cast<const uint4*>(a.contrib + (size_t)(2 * t + 1) * d);
  const uint4* sh = reinterpret_cast<const uint4*>(a.shared_y + (size_t)t * d);
  const uint4* rs = a.residual ? reinterpret_cast<const uint4*>(a.residual + (size_t)t * d) : nullptr;
  uint4* o = reinterpret_cast<uint4*>(a.out + (size_t)t * d);
  uint4 vs[V], v0[V], v1[V], vr[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      vs[i] = __ldg(sh + c);
      v0[i] = __ldg(c0 + c);
      v1[i] = __ldg(c1 + c);
      if (rs != nullptr) vr[i] = __ldg(rs + c);
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float s[8], p[8], q[8];
      bf16x8_to_float(vs[i], s);
      bf16x8_to_float(v0[i], p);
      bf16x8_to_float(v1[i], q);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] = round_bf16(round_bf16(s[k] + p[k]) + q[k]);
      if (rs != nullptr) {
        float b[8];
        bf16x8_to_float(vr[i], b);
#pragma unroll
        for (int k = 0; k < 8; ++k) s[k] = b[k] + s[k];
      }
      o[c] = float_to_bf16x8(s);
    }
  }
}

// One warp per token: gathers the token's two expert rows through positions,
// weights them exactly as the down GEMM's scatter epilogue does
// (bf16(bf16(y) * bf16(w))) and adds them to the shared output in ascending
// expert order, so the result is bit-identical to the single-GPU block.
template <int V>
__global__ void __launch_bounds__(128) ep_combine_kernel(EpCombineArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  griddep_wait();
  griddep_launch();
  if (t >= a.tokens) return;
  const int d = a.dim, nvec = d >> 3;
  const int e0 = __ldg(a.indices + 2 * t), e1 = __ldg(a.indices + 2 * t + 1);
  int p0 = __ldg(a.positions + 2 * t), p1 = __ldg(a.positions + 2 * t + 1);
  if (p0 < 0 || p0 >= a.rows || p1 < 0 || p1 >= a.rows) {
    if (lane == 0) report_status(a.status, kStatusBadIndex, 4, t);
    return;
  }
  float w0 = round_bf16(__ldg(a.weights + 2 * t)), w1 = round_bf16(__ldg(a.weights + 2 * t + 1));
  if (e1 < e0) {  // lower expert id first
    const int tp = p0; p0 = p1; p1 = tp;
    const float tw = w0; w0 = w1; w1 = tw;
  }
  const uint4* y0 = reinterpret_cast<const uint4*>(a.y + (size_t)p0 * d);
  const uint4* y1 = reinterpret_cast<const uint4*>(a.y + (size_t)p1 * d);
  const uint4* sh = reinterpret_cast<const uint4*>(a.shared_y + (size_t)t * d);
  const uint4* rs = a.residual ? reinterpret_cast<const uint4*>(a.residual + (size_t)t * d) : nullptr;
  uint4* o = reinterpret_cast<uint4*>(a.out + (size_t)t * d);
  uint4 vs[V], v0[V], v1[V], vr[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      vs[i] = __ldg(sh + c);
      v0[i] = __ldg(y0 + c);
      v1[i] = __ldg(y1 + c);
      if (rs != nullptr) vr[i] = __ldg(rs + c);
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      float s[8], p[8], q[8];
      bf16x8_to_float(vs[i], s);
      bf16x8_to_float(v0[i], p);
      bf16x8_to_float(v1[i], q);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        s[k] = round_bf16(round_bf16(s[k] + round_bf16(p[k] * w0)) + round_bf16(q[k] * w1));
      if (rs != nullptr) {
        float b[8];
        bf16x8_to_float(vr[i], b);
#pragma unroll
        for (int k = 0; k < 8; ++k) s[k] = b[k] + s[k];
      }
      o[c] = float_to_bf16x8(s);
    }
  }
}

int launch_ep_combine(const EpCombineArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  const dim3 grid((args.tokens + 3) / 4), block(128);
  switch ((args.dim / 8 + 31) / 32) {
    case 1: launch_pdl(ep_combine_kernel<1>, grid, block, 0, stream, args); break;
    case 2: launch_pdl(ep_combine_kernel<2>, grid, block, 0, stream, args); break;
    case 3: launch_pdl(ep_combine_kernel<3>, grid, block, 0, stream, args); break;
    case 4: launch_pdl(ep_combine_kernel<4>, grid, block, 0, stream, args); break;
    default: return -1;
  }
  return 0;
}

int launch_combine(const CombineArgs& args, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  const int warps = 4;
  dim3 grid((args.tokens + warps - 1) / warps), block(32 * warps);
  const int v = (args.dim / 8 + 31) / 32;
  switch (v) {
    case 1: launch_pdl(combine_kernel<1>, grid, block, 0, stream, args); break;
    case 2: launch_pdl(combine_kernel<2>, grid, block, 0, stream, args); break;
    case 3: launch_pdl(combine_kernel<3>, grid, block, 0, stream, args); break;
    case 4: launch_pdl(combine_kernel<4>, grid, block, 0, stream, args); break;
    default: return -1;
  }
  return 0;
}

}  // namespace parrot
