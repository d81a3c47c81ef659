// The MoE block at decode batch sizes (a few tokens): three kernels instead
// of router + grouping + two grouped GEMMs + combine.
//
// moe_decode_route_kernel: one warp per token: fp32 logits of the bf16 row,
//                          softmax, top-2 with the lower id on ties,
//                          renormalised weights (model.py:521-527).  Up to 4
//                          tokens it is not launched: every routed gate/up CTA
//                          computes the same routing itself (route_small) and
//                          CTA 0 publishes it.
// moe_decode_up_kernel:    work item = 16 SwiGLU features of one chosen
//                          expert (ascending id; at most min(E, 2T) of them)
//                          or of the shared expert: the CTA stages the
//                          features' packed gate/up rows and the tokens routed
//                          to that expert in shared memory with one round of
//                          async copies, then one warp per feature dots both
//                          rows with every such token,
//                          h = bf16(silu(bf16 gate) * bf16 up).
// moe_decode_down_kernel:  one CTA per (token, 16 output columns) stages the
//                          token's two routed down rows, the shared one and its
//                          hidden rows, computes y = bf16(down . h) and combines
//                          them exactly as the reference's index_add sequence
//                          does: out = [residual +] bf16(bf16(shared + c_lo) +
//                          c_hi), c = bf16(y * bf16(w)), lower expert id first
//                          (model.py:545-551).
// The weights are the tiled packs the grouped GEMM streams (128 x 64 tiles).
// All dot products accumulate in fp32; only their order differs from the
// tensor-core path.  SiLU is computed as x / (1 + expf(-x)) in fp32, the
// expression the reference evaluates for a bf16 tensor.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

namespace {
constexpr int kTileRows = 128, kTileCols = 64;
constexpr int kFeatPerCta = 16;   // SwiGLU features per up CTA (4 per warp)
constexpr int kColsPerCta = 16;   // output columns per down CTA (4 per warp)

// element (row, col) of matrix m in the tiled layout of a [rows, cols] matrix
__device__ __forceinline__ size_t tiled_index(int m, int row, int col, int rows, int cols) {
  const int rt = row / kTileRows, kb = col / kTileCols;
  const size_t tile = ((size_t)m * (rows / kTileRows) + rt) * (cols / kTileCols) + kb;
  return tile * (kTileRows * kTileCols) + (size_t)(row % kTileRows) * kTileCols + col % kTileCols;
}
}  // namespace

// Softmax, top-2 with the lower id on ties and renormalised weights of token
// t, from its fp32 logit in lane e (expert e; lanes >= E hold anything).  All
// lanes get the chosen ids; with `publish` the route outputs are written.
__device__ __forceinline__ void finish_route(const MoeDecodeArgs& a, int t, float logit, int lane,
                                             bool publish, int* i1_out, int* i2_out) {
  const int E = a.n_experts;
  const bool valid = lane < E;
  if (valid && a.router_bias != nullptr) logit += __ldg(a.router_bias + lane);
  const float m = warp_max(valid ? logit : -INFINITY);
  const float ev = valid ? expf(logit - m) : 0.f;
  const float p = ev / warp_sum(ev);
  float v1 = valid ? p : -1.f;
  int i1 = lane;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v1, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i1, o);
    if (ov > v1 || (ov == v1 && oi < i1)) { v1 = ov; i1 = oi; }
  }
  float v2 = (valid && lane != i1) ? p : -1.f;
  int i2 = lane;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v2, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i2, o);
    if (ov > v2 || (ov == v2 && oi < i2)) { v2 = ov; i2 = oi; }
  }
  *i1_out = i1;
  *i2_out = i2;
  if (!publish) return;
  if (valid && a.probs != nullptr) a.probs[(size_t)t * E + lane] = p;
  if (lane == 0) {
    const float sel = v1 + v2;
    const float w1 = v1 / sel, w2 = v2 / sel;
    a.indices[2 * t] = i1;
    a.indices[2 * t + 1] = i2;
    a.weights[2 * t] = w1;
    a.weights[2 * t + 1] = w2;
    if (a.indices64 != nullptr) {
      a.indices64[2 * t] = i1;
      a.indices64[2 * t + 1] = i2;
    }
    if (a.weights_out != nullptr) {
      a.weights_out[2 * t] = w1;
      a.weights_out[2 * t + 1] = w2;
    }
  }
}

// Router for up to 4 tokens inside a gate/up CTA: all 128 threads split d
// (thread c: 16-byte vector c of every token row against every expert row),
// one warp_reduce_many per token and warp, the four warps' partials added in
// shared memory; warp t finishes token t.  x_s: [T][d / 8] token rows, r_s:
// [E][d / 8] router rows; the chosen ids land in ids_s.
__device__ __forceinline__ void route_small(const MoeDecodeArgs& a, const uint4* r_s,
                                            const uint4* x_s, int* ids_s, float* red_s,
                                            bool publish) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.tokens, E = a.n_experts, nvec = a.dim >> 3;
  for (int t = 0; t < T; ++t) {
    float part[kMaxExperts];
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) part[e] = 0.f;
    for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
      float xf[8];
      bf16x8_to_float(x_s[(size_t)t * nvec + c], xf);
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) {
        if (e < E) {
          float wf[8];
          bf16x8_to_float(r_s[(size_t)e * nvec + c], wf);
#pragma unroll
          for (int j = 0; j < 8; ++j) part[e] = fmaf(xf[j], wf[j], part[e]);
        }
      }
    }
    red_s[(t * 4 + warp) * 32 + lane] = warp_reduce_many<kMaxExperts>(part, lane);
  }
  __syncthreads();
  if (warp < T) {
    const float* r = red_s + warp * 4 * 32 + lane;
    const float logit = (r[0] + r[32]) + (r[64] + r[96]);
    int i1, i2;
    finish_route(a, warp, logit, lane, publish, &i1, &i2);
    if (lane == 0) {
      ids_s[2 * warp] = i1;
      ids_s[2 * warp + 1] = i2;
    }
  }
}

// Router: one warp per token (lanes over d, every expert's dot reduced
// together), softmax, top-2 with the lower id on ties, renormalised weights.
__global__ void __launch_bounds__(128) moe_decode_route_kernel(MoeDecodeArgs a) {
  extern __shared__ __align__(16) uint4 rw_s[];  // router weight [E][d / 8], then 4 token rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  const int d = a.dim, E = a.n_experts, nvec = d >> 3;
  uint4* x_s = rw_s + (size_t)E * nvec;
  // the router weight is a parameter: all of it in flight before the wait
  for (int i = threadIdx.x; i < E * nvec; i += blockDim.x)
    cp_async16(rw_s + i, reinterpret_cast<const uint4*>(a.router) + i);
  griddep_wait();
  griddep_launch();
  const int t0 = blockIdx.x * 4, rows = min(4, a.tokens - t0);
  for (int i = threadIdx.x; i < rows * nvec; i += blockDim.x)
    cp_async16(x_s + i, reinterpret_cast<const uint4*>(a.x) + (size_t)t0 * nvec + i);
  cp_async_wait_all();
  __syncthreads();
  if (t >= a.tokens) return;
  float part[kMaxExperts];
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) part[e] = 0.f;
  for (int c = lane; c < nvec; c += 32) {
    float xf[8];
    bf16x8_to_float(x_s[warp * nvec + c], xf);
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) {
      if (e < E) {
        float wf[8];
        bf16x8_to_float(rw_s[e * nvec + c], wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) part[e] = fmaf(xf[j], wf[j], part[e]);
      }
    }
  }
  const float logit = warp_reduce_many<kMaxExperts>(part, lane);  // lane e: expert e
  int i1, i2;
  finish_route(a, t, logit, lane, true, &i1, &i2);
}

// Gate/up + SwiGLU.  Work item c: feature block c % blocks of the
// (c / blocks)-th chosen expert in ascending id, or of the shared expert after
// the routed items; a CTA past the chosen experts' items returns at once.
// NT: the token capacity of this instantiation (4 or kDecodeMoeMaxTokens).
template <int NT>
__global__ void __launch_bounds__(128) moe_decode_up_kernel(MoeDecodeArgs a) {
  // [2 * kFeatPerCta rows][d / 8] gate/up rows, then [tokens][d / 8] token rows
  extern __shared__ __align__(16) uint4 wrows_s[];
  __shared__ int list_s[kDecodeMoeMaxTokens];   // tokens this CTA serves
  __shared__ int slot_s[kDecodeMoeMaxTokens];   // their hidden slot (0, 1: routed k; 2: shared)
  __shared__ int n_list, expert_s;
  const int T = a.tokens, d = a.dim, E = a.n_experts, H = a.expert_dim, Hs = a.shared_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = d >> 3;
  // NT <= 4: every token row [T][d / 8], then the router rows [E][d / 8];
  // otherwise the listed tokens' rows
  uint4* x_s = wrows_s + (size_t)2 * kFeatPerCta * nvec;
  uint4* r_s = x_s + (size_t)NT * nvec;
  const int routed_blocks = H / kFeatPerCta;
  const int max_chosen = min(E, 2 * T);
  const bool shared = (int)blockIdx.x >= max_chosen * routed_blocks;
  const int f0 = (shared ? (int)blockIdx.x - max_chosen * routed_blocks
                         : (int)blockIdx.x % routed_blocks) * kFeatPerCta;
  if (shared) {
    // the shared expert's rows depend on nothing upstream: fetch them now
    for (int i = threadIdx.x; i < 2 * kFeatPerCta * nvec; i += blockDim.x) {
      const int r = i / nvec, c = i - r * nvec;
      const int f = f0 + (r >> 1);
      const int row = packed_gate_up_row(f, r & 1);
      cp_async16(wrows_s + i, a.shared_gate_up + tiled_index(0, row, c * 8, 2 * Hs, d));
    }
  }
  __shared__ int ids_s[2 * kDecodeMoeMaxTokens];
  if constexpr (NT <= 4) {
    // routed CTAs route the (at most 4) tokens themselves, unless the depth
    // mix before did: the router weight is a parameter, so it is in flight
    // before the wait
    if (!shared && !a.routed)
      for (int i = threadIdx.x; i < E * nvec; i += blockDim.x)
        cp_async16(r_s + i, reinterpret_cast<const uint4*>(a.router) + i);
    griddep_wait();
    griddep_launch();
    for (int i = threadIdx.x; i < T * nvec; i += blockDim.x)
      cp_async16(x_s + i, reinterpret_cast<const uint4*>(a.x) + i);
    if (a.routed) {
      if (threadIdx.x < 2 * T) ids_s[threadIdx.x] = a.indices[threadIdx.x];
    } else if (!shared) {
      __shared__ float red_s[4 * 4 * 32];
      cp_async_wait_all();
      __syncthreads();
      route_small(a, r_s, x_s, ids_s, red_s, blockIdx.x == 0);  // CTA 0 publishes
    }
  } else {
    griddep_wait();
    griddep_launch();
    if (threadIdx.x < 2 * T) ids_s[threadIdx.x] = a.indices[threadIdx.x];  // one parallel load
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int e = -1;
    if (!shared) {
      // the (blockIdx / blocks)-th distinct chosen expert, ascending id
      unsigned mask = 0;
      for (int i = 0; i < 2 * T; ++i) mask |= 1u << ids_s[i];
      const int want = (int)blockIdx.x / routed_blocks;
      for (int x = 0, seen = 0; x < E; ++x)
        if (mask & (1u << x)) {
          if (seen == want) e = x;
          ++seen;
        }
    }
    int n = 0;
    if (shared || e >= 0)
      for (int t = 0; t < T; ++t) {
        const int k = shared ? 2 : (ids_s[2 * t] == e ? 0 : (ids_s[2 * t + 1] == e ? 1 : -1));
        if (k >= 0) {
          list_s[n] = t;
          slot_s[n] = k;
          ++n;
        }
      }
    n_list = n;
    expert_s = e;
  }
  __syncthreads();
  const int n = n_list;
  if (n == 0) {
    cp_async_wait_all();  // nothing may be in flight when the CTA exits
    return;
  }
  if (!shared) {
    const int e = expert_s;
    for (int i = threadIdx.x; i < 2 * kFeatPerCta * nvec; i += blockDim.x) {
      const int r = i / nvec, c = i - r * nvec;
      const int f = f0 + (r >> 1);
      const int row = packed_gate_up_row(f, r & 1);
      cp_async16(wrows_s + i, a.gate_up + tiled_index(e, row, c * 8, 2 * H, d));
    }
  }
  if constexpr (NT > 4) {
    for (int i = threadIdx.x; i < n * nvec; i += blockDim.x) {
      const int li = i / nvec, c = i - li * nvec;
      cp_async16(x_s + i, reinterpret_cast<const uint4*>(a.x) + (size_t)list_s[li] * nvec + c);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  if constexpr (NT <= 4) {
    // up to 4 tokens: warp w takes features 4w .. 4w + 3 together — one pass
    // over d accumulates all 2 x 4 x NT dots (gate and up of each feature for
    // each token), one warp_reduce_many folds them, and lane 2 NT q + i
    // finishes feature q's token i with the gate total and the up total NT
    // lanes above it
    constexpr int FW = kFeatPerCta / 4;
    constexpr int NV = 2 * FW * NT;  // values to reduce (32 at NT = 4)
    static_assert(NV <= 32 && (NV & (NV - 1)) == 0, "one value per lane");
    const int fb = warp * FW;
    float acc[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[v] = 0.f;
    for (int c = lane; c < nvec; c += 32) {
      float xf[NT][8];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        if (i < n) {
          bf16x8_to_float(x_s[(size_t)list_s[i] * nvec + c], xf[i]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xf[i][j] = 0.f;
        }
      }
#pragma unroll
      for (int q = 0; q < 2 * FW; ++q) {  // row 2 (fb + q / 2) + q % 2: gate / up of a feature
        float wf[8];
        bf16x8_to_float(wrows_s[(size_t)(2 * fb + q) * nvec + c], wf);
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[q * NT + i] = fmaf(wf[j], xf[i][j], acc[q * NT + i]);
      }
    }
    const float tot = warp_reduce_many<NV>(acc, lane);  // lane v: total of value v % NV
    const float up_tot = __shfl_down_sync(0xffffffffu, tot, NT);
    const int q = (lane % NV) / NT, i = lane % NT;
    if (lane < NV && (q & 1) == 0 && i < n) {
      const int f = f0 + fb + q / 2;
      const float g = round_bf16(tot);
      const float u = round_bf16(up_tot);
      const float silu = round_bf16(g / (1.0f + expf(-g)));
      a.hidden[((size_t)list_s[i] * 3 + slot_s[i]) * H + f] = __float2bfloat16_rn(silu * u);
    }
  } else {
    // each feature's gate and up rows, dotted with every listed token
    // (a warp per feature, the features of a warp one after the other)
    for (int fi = warp; fi < kFeatPerCta; fi += 4) {
      const int f = f0 + fi;
      const uint4* g_row = wrows_s + (size_t)(2 * fi) * nvec;
      const uint4* u_row = g_row + nvec;
      float acc_g[kDecodeMoeMaxTokens], acc_u[kDecodeMoeMaxTokens];
#pragma unroll
      for (int i = 0; i < kDecodeMoeMaxTokens; ++i) acc_g[i] = acc_u[i] = 0.f;
      for (int c = lane; c < nvec; c += 32) {
        float gf[8], uf[8];
        bf16x8_to_float(g_row[c], gf);
        bf16x8_to_float(u_row[c], uf);
#pragma unroll
        for (int i = 0; i < kDecodeMoeMaxTokens; ++i) {
          if (i < n) {
            float xf[8];
            bf16x8_to_float(x_s[(size_t)i * nvec + c], xf);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acc_g[i] = fmaf(gf[j], xf[j], acc_g[i]);
              acc_u[i] = fmaf(uf[j], xf[j], acc_u[i]);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kDecodeMoeMaxTokens; ++i) {
        if (i < n) {
          const float g = round_bf16(warp_sum(acc_g[i]));
          const float u = round_bf16(warp_sum(acc_u[i]));
          if (lane == 0) {
            const float silu = round_bf16(g / (1.0f + expf(-g)));
            a.hidden[((size_t)list_s[i] * 3 + slot_s[i]) * H + f] = __float2bfloat16_rn(silu * u);
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(128) moe_decode_down_kernel(MoeDecodeArgs a) {
  // [3][kColsPerCta rows][hid / 8]: routed k = 0, 1 (H wide), shared (Hs wide)
  extern __shared__ __align__(16) uint4 drows_s[];
  __shared__ __align__(16) __nv_bfloat16 h_s[3][1024];
  const int d = a.dim, H = a.expert_dim, Hs = a.shared_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col_blocks = d / kColsPerCta;
  const int t = blockIdx.x / col_blocks, o0 = (blockIdx.x % col_blocks) * kColsPerCta;
  const int hv = H / 8, hsv = Hs / 8;
  uint4* rows[3] = {drows_s, drows_s + kColsPerCta * hv, drows_s + 2 * kColsPerCta * hv};
  // the shared expert's rows do not depend on the routing: fetch them first
  for (int i = threadIdx.x; i < kColsPerCta * hsv; i += blockDim.x) {
    const int r = i / hsv, c = i - r * hsv;
    cp_async16(rows[2] + i, a.shared_down + tiled_index(0, o0 + r, c * 8, d, Hs));
  }
  auto fetch_routed = [&](int e0, int e1) {
    for (int i = threadIdx.x; i < 2 * kColsPerCta * hv; i += blockDim.x) {
      const int k = i / (kColsPerCta * hv), rem = i - k * (kColsPerCta * hv);
      const int r = rem / hv, c = rem - r * hv;
      cp_async16(rows[k] + rem, a.down + tiled_index(k == 0 ? e0 : e1, o0 + r, c * 8, d, H));
    }
  };
  // routed by the depth mix two launches back: its ids are complete before
  // the gate/up kernel this one follows could start, so the expert rows come
  // before the wait too
  int e0 = 0, e1 = 0;
  if (a.routed) {
    e0 = a.indices[2 * t];
    e1 = a.indices[2 * t + 1];
    fetch_routed(e0, e1);
  }
  griddep_wait();
  griddep_launch();
  if (!a.routed) {
    e0 = a.indices[2 * t];
    e1 = a.indices[2 * t + 1];
    fetch_routed(e0, e1);
  }
  const float w0 = round_bf16(a.weights[2 * t]), w1 = round_bf16(a.weights[2 * t + 1]);
  for (int i = threadIdx.x; i < (2 * H + Hs) / 8; i += blockDim.x) {
    const int k = i < H / 4 ? i / (H / 8) : 2;
    const int c = k < 2 ? i - k * (H / 8) : i - H / 4;
    cp_async16(reinterpret_cast<uint4*>(&h_s[k][0]) + c,
               reinterpret_cast<const uint4*>(a.hidden + ((size_t)t * 3 + k) * H) + c);
  }
  cp_async_wait_all();
  __syncthreads();
  // warp w takes output columns 4w .. 4w + 3 together: its lanes hold their
  // slices of the three hidden vectors once, accumulate the 4 x 3 dots in one
  // pass, one warp_reduce_many folds them (lane 4 c + k: column c, source k)
  // and lane 4 c combines column c exactly as the block's combine does
  static_assert(kColsPerCta == 16, "four columns per warp");
  const int cb = warp * 4;
  float acc[16];
#pragma unroll
  for (int v = 0; v < 16; ++v) acc[v] = 0.f;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int nv = k < 2 ? hv : hsv;
    for (int c = lane; c < nv; c += 32) {
      float hf[8];
      bf16x8_to_float(reinterpret_cast<const uint4*>(&h_s[k][0])[c], hf);
#pragma unroll
      for (int ci = 0; ci < 4; ++ci) {
        float wf[8];
        bf16x8_to_float(rows[k][(size_t)(cb + ci) * nv + c], wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[4 * ci + k] = fmaf(wf[j], hf[j], acc[4 * ci + k]);
      }
    }
  }
  const float tot = warp_reduce_many<16>(acc, lane);
  const float y1 = __shfl_down_sync(0xffffffffu, tot, 1);
  const float y2 = __shfl_down_sync(0xffffffffu, tot, 2);
  if (lane < 16 && (lane & 3) == 0) {
    const int o = o0 + cb + (lane >> 2);
    const float c0 = round_bf16(round_bf16(tot) * w0), c1 = round_bf16(round_bf16(y1) * w1);
    const float lo = e0 < e1 ? c0 : c1, hi = e0 < e1 ? c1 : c0;
    float r = round_bf16(round_bf16(round_bf16(y2) + lo) + hi);
    if (a.residual != nullptr) r = __bfloat162float(a.residual[(size_t)t * d + o]) + r;
    a.out[(size_t)t * d + o] = __float2bfloat16_rn(r);
  }
}

int launch_moe_decode(const MoeDecodeArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return 0;
  const size_t up_smem = (size_t)(2 * kFeatPerCta + (a.tokens <= 4 ? 4 + a.n_experts : a.tokens)) *
                         a.dim * 2;
  const size_t down_smem = (size_t)kColsPerCta * (2 * a.expert_dim + a.shared_dim) * 2;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(moe_decode_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (kMaxExperts + 4) * 1024 * 2) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_up_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (2 * kFeatPerCta + 4 + kMaxExperts) * 1024 * 2) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_up_kernel<4>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_up_kernel<kDecodeMoeMaxTokens>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (2 * kFeatPerCta + kDecodeMoeMaxTokens) * 1024 * 2) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_up_kernel<kDecodeMoeMaxTokens>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_down_kernel,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
        cudaFuncSetAttribute(moe_decode_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kColsPerCta * 3 * 1024 * 2) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  const int max_chosen = a.n_experts < 2 * a.tokens ? a.n_experts : 2 * a.tokens;
  const int up_ctas = max_chosen * (a.expert_dim / kFeatPerCta) + a.shared_dim / kFeatPerCta;
  const size_t route_smem = (size_t)(a.n_experts + 4) * a.dim * 2;
  // up to 4 tokens the gate/up CTAs route the tokens themselves (or read the
  // routing the depth mix did)
  if ((a.tokens > 4 && !a.routed && launch_pdl(moe_decode_route_kernel, dim3((a.tokens + 3) / 4), dim3(128),
                                  route_smem, stream, a) != cudaSuccess) ||
      (a.tokens <= 4
           ? launch_pdl(moe_decode_up_kernel<4>, dim3(up_ctas), dim3(128), up_smem, stream, a)
           : launch_pdl(moe_decode_up_kernel<kDecodeMoeMaxTokens>, dim3(up_ctas), dim3(128),
                        up_smem, stream, a)) != cudaSuccess)
    return -2;
  return launch_pdl(moe_decode_down_kernel, dim3(a.tokens * (a.dim / kColsPerCta)), dim3(128),
                    down_smem, stream, a) == cudaSuccess
             ? 0
             : -2;
}

}  // namespace parrot
