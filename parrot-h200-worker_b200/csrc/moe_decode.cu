// The MoE block at decode batch sizes (a few tokens): two kernels instead of
// router + grouping + two grouped GEMMs + combine.
//
// moe_decode_up_kernel:   every CTA routes all the tokens (fp32 logits of the
//                         bf16 rows, softmax, top-2 with the lower id on ties,
//                         renormalised weights; model.py:521-527) — the same
//                         arithmetic in every CTA, so they agree — then takes 32
//                         SwiGLU features of one expert (or of the shared
//                         expert) for the tokens routed to it: one warp per
//                         feature pair of rows streams the packed gate/up rows
//                         once and dots them with every such token,
//                         h = bf16(silu(bf16 gate) * bf16 up).  CTAs of experts
//                         no token chose return after routing.
// moe_decode_down_kernel: one CTA per (token, 16 output columns) computes the
//                         token's two routed rows and the shared row,
//                         y = bf16(down . h), and combines them exactly as the
//                         reference's index_add sequence does:
//                         out = [residual +] bf16(bf16(shared + c_lo) + c_hi),
//                         c = bf16(y * bf16(w)), lower expert id first
//                         (model.py:545-551).
// The weights are the tiled packs the grouped GEMM streams (128 x 64 tiles).
// All dot products accumulate in fp32; only their order differs from the
// tensor-core path.  SiLU is computed as x / (1 + expf(-x)) in fp32, the
// expression the reference evaluates for a bf16 tensor.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

namespace {
constexpr int kTileRows = 128, kTileCols = 64;
constexpr int kFeatPerCta = 32;   // SwiGLU features per up CTA (8 per warp)
constexpr int kColsPerCta = 16;   // output columns per down CTA (4 per warp)

// element (row, col) of matrix m in the tiled layout of a [rows, cols] matrix
__device__ __forceinline__ size_t tiled_index(int m, int row, int col, int rows, int cols) {
  const int rt = row / kTileRows, kb = col / kTileCols;
  const size_t tile = ((size_t)m * (rows / kTileRows) + rt) * (cols / kTileCols) + kb;
  return tile * (kTileRows * kTileCols) + (size_t)(row % kTileRows) * kTileCols + col % kTileCols;
}
}  // namespace

__global__ void __launch_bounds__(128) moe_decode_up_kernel(MoeDecodeArgs a) {
  __shared__ __align__(16) __nv_bfloat16 x_s[kDecodeMoeMaxTokens][1024];
  __shared__ int idx_s[kDecodeMoeMaxTokens][2];
  __shared__ float w_s[kDecodeMoeMaxTokens][2];
  __shared__ int list_s[kDecodeMoeMaxTokens];   // tokens this CTA serves
  __shared__ int slot_s[kDecodeMoeMaxTokens];   // their hidden slot (0, 1: routed k; 2: shared)
  __shared__ int n_list;
  const int T = a.tokens, d = a.dim, E = a.n_experts, H = a.expert_dim, Hs = a.shared_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = d >> 3;
  griddep_wait();
  griddep_launch();
  for (int i = threadIdx.x; i < T * nvec; i += blockDim.x) {
    const int t = i / nvec, c = i - t * nvec;
    reinterpret_cast<uint4*>(&x_s[t][0])[c] = __ldg(reinterpret_cast<const uint4*>(a.x) + (size_t)t * nvec + c);
  }
  __syncthreads();

  // 1. routing, one warp per token (lanes over d, all experts reduced together)
  for (int t = warp; t < T; t += 4) {
    float part[kMaxExperts];
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) part[e] = 0.f;
    for (int c = lane; c < nvec; c += 32) {
      float xf[8];
      bf16x8_to_float(reinterpret_cast<const uint4*>(&x_s[t][0])[c], xf);
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) {
        if (e < E) {
          float wf[8];
          bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(a.router + (size_t)e * d) + c), wf);
#pragma unroll
          for (int j = 0; j < 8; ++j) part[e] = fmaf(xf[j], wf[j], part[e]);
        }
      }
    }
    float logit = warp_reduce_many<kMaxExperts>(part, lane);  // lane e: expert e
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
    if (lane == 0) {
      const float sel = v1 + v2;
      idx_s[t][0] = i1;
      idx_s[t][1] = i2;
      w_s[t][0] = v1 / sel;
      w_s[t][1] = v2 / sel;
    }
    if (blockIdx.x == 0) {  // one CTA publishes the decisions
      if (valid && a.probs != nullptr) a.probs[(size_t)t * E + lane] = p;
      if (lane == 0) {
        const float sel = v1 + v2;
        a.indices[2 * t] = i1;
        a.indices[2 * t + 1] = i2;
        a.weights[2 * t] = v1 / sel;
        a.weights[2 * t + 1] = v2 / sel;
        if (a.indices64 != nullptr) {
          a.indices64[2 * t] = i1;
          a.indices64[2 * t + 1] = i2;
        }
        if (a.weights_out != nullptr) {
          a.weights_out[2 * t] = v1 / sel;
          a.weights_out[2 * t + 1] = v2 / sel;
        }
      }
    }
  }
  __syncthreads();

  // 2. this CTA's expert and features, and the tokens that need them
  const int routed_ctas = E * (H / kFeatPerCta);
  const bool shared = (int)blockIdx.x >= routed_ctas;
  const int e = shared ? -1 : (int)blockIdx.x / (H / kFeatPerCta);
  const int f0 = (shared ? (int)blockIdx.x - routed_ctas : (int)blockIdx.x % (H / kFeatPerCta)) *
                 kFeatPerCta;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int t = 0; t < T; ++t) {
      const int k = shared ? 2 : (idx_s[t][0] == e ? 0 : (idx_s[t][1] == e ? 1 : -1));
      if (k >= 0) {
        list_s[n] = t;
        slot_s[n] = k;
        ++n;
      }
    }
    n_list = n;
  }
  __syncthreads();
  const int n = n_list;
  if (n == 0) return;
  const int hid = shared ? Hs : H;
  const __nv_bfloat16* gu = shared ? a.shared_gate_up : a.gate_up;
  const int m = shared ? 0 : e;

  // 3. gate and up rows of each feature, dotted with every listed token
  for (int fi = warp; fi < kFeatPerCta; fi += 4) {
    const int f = f0 + fi;
    const int row_g = (f / 64) * kTileRows + 2 * (f % 64), row_u = row_g + 1;
    float acc_g[kDecodeMoeMaxTokens], acc_u[kDecodeMoeMaxTokens];
#pragma unroll
    for (int i = 0; i < kDecodeMoeMaxTokens; ++i) acc_g[i] = acc_u[i] = 0.f;
    for (int c = lane; c < nvec; c += 32) {
      float gf[8], uf[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(gu + tiled_index(m, row_g, c * 8, 2 * hid, d)), gf);
      bf16x8_to_float(*reinterpret_cast<const uint4*>(gu + tiled_index(m, row_u, c * 8, 2 * hid, d)), uf);
#pragma unroll
      for (int i = 0; i < kDecodeMoeMaxTokens; ++i) {
        if (i < n) {
          float xf[8];
          bf16x8_to_float(reinterpret_cast<const uint4*>(&x_s[list_s[i]][0])[c], xf);
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

__global__ void __launch_bounds__(128) moe_decode_down_kernel(MoeDecodeArgs a) {
  __shared__ __align__(16) __nv_bfloat16 h_s[3][1024];
  const int d = a.dim, H = a.expert_dim, Hs = a.shared_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col_blocks = d / kColsPerCta;
  const int t = blockIdx.x / col_blocks, o0 = (blockIdx.x % col_blocks) * kColsPerCta;
  griddep_wait();
  griddep_launch();
  const int e0 = a.indices[2 * t], e1 = a.indices[2 * t + 1];
  const float w0 = round_bf16(a.weights[2 * t]), w1 = round_bf16(a.weights[2 * t + 1]);
  for (int i = threadIdx.x; i < (2 * H + Hs) / 8; i += blockDim.x) {
    const int k = i < H / 4 ? i / (H / 8) : 2;
    const int c = k < 2 ? i - k * (H / 8) : i - H / 4;
    reinterpret_cast<uint4*>(&h_s[k][0])[c] =
        reinterpret_cast<const uint4*>(a.hidden + ((size_t)t * 3 + k) * H)[c];
  }
  __syncthreads();
  for (int oi = warp; oi < kColsPerCta; oi += 4) {
    const int o = o0 + oi;
    float y[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < 3; ++k) {
      const int hid = k < 2 ? H : Hs;
      const __nv_bfloat16* dn = k < 2 ? a.down : a.shared_down;
      const int mat = k == 0 ? e0 : (k == 1 ? e1 : 0);
      for (int c = lane; c < hid / 8; c += 32) {
        float wf[8], hf[8];
        bf16x8_to_float(*reinterpret_cast<const uint4*>(dn + tiled_index(mat, o, c * 8, d, hid)), wf);
        bf16x8_to_float(reinterpret_cast<const uint4*>(&h_s[k][0])[c], hf);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[k] = fmaf(wf[j], hf[j], y[k]);
      }
      y[k] = warp_sum(y[k]);
    }
    if (lane == 0) {
      const float c0 = round_bf16(round_bf16(y[0]) * w0), c1 = round_bf16(round_bf16(y[1]) * w1);
      const float lo = e0 < e1 ? c0 : c1, hi = e0 < e1 ? c1 : c0;
      float r = round_bf16(round_bf16(round_bf16(y[2]) + lo) + hi);
      if (a.residual != nullptr) r = __bfloat162float(a.residual[(size_t)t * d + o]) + r;
      a.out[(size_t)t * d + o] = __float2bfloat16_rn(r);
    }
  }
}

int launch_moe_decode(const MoeDecodeArgs& a, cudaStream_t stream) {
  if (a.tokens == 0) return 0;
  const int up_ctas = a.n_experts * (a.expert_dim / kFeatPerCta) + a.shared_dim / kFeatPerCta;
  if (launch_pdl(moe_decode_up_kernel, dim3(up_ctas), dim3(128), 0, stream, a) != cudaSuccess)
    return -2;
  return launch_pdl(moe_decode_down_kernel, dim3(a.tokens * (a.dim / kColsPerCta)), dim3(128), 0,
                    stream, a) == cudaSuccess
             ? 0
             : -2;
}

}  // namespace parrot
