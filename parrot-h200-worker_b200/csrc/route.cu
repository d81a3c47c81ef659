// Router (N1) and deterministic capacity grouping (N2).
//
// route_small_kernel (up to 4096 tokens): one CTA per 4 tokens on CUDA
//                cores; the router weight is staged in shared memory before
//                the grid-dependency wait, each warp folds its tokens' E dots
//                with one warp_reduce_many, softmax and top-2 are shuffle
//                reductions (see the kernel).
// route_kernel (above 4096 tokens): one CTA per 128 tokens.  The router
//                logits are a skinny GEMM [128 x d] x [d x E]: TMA streams
//                64-column slabs of the token tile and of the router weight
//                through a shared-memory ring, one thread issues tcgen05.mma
//                (M = 128 tokens, N = E rounded up to 16/32, fp32 accumulator
//                in TMEM).  Each of the 128 threads then reads its token's E
//                logits from TMEM with one tcgen05.ld and does the softmax,
//                top-2 and renormalisation in registers (no cross-lane
//                reductions).  Each warp (32 tokens) records its expert
//                histogram; the CTA records its tile histogram and
//                probability sums.
// group_kernel:  every block derives its exclusive per-expert prefix from the
//                tile and chunk histograms (no serial pass, no spinning),
//                ranks each assignment inside its block with warp match -> a
//                stable slot (ascending token order within each expert, the
//                reference's torch.where order), maps slot -> grouped row
//                (capacity region, else the overflow region), and copies the
//                token rows with 16-byte vectors.  Block 0 also writes the
//                segment tables, counts and router statistics.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"
#include "tc.cuh"

namespace parrot {

using namespace tc;

constexpr int kRouteM = 128;                   // MMA rows (tokens of a tile, padded)
constexpr int kRouteXTile = kRouteM * 64 * 2;  // 16 KB slab: 128 token rows x 64 columns
constexpr int kRouteMaxStages = 12;

struct __align__(8) RouteSmem {
  uint64_t full[kRouteMaxStages];
  uint64_t empty[kRouteMaxStages];
  uint64_t done;
  uint32_t tmem;
  int abort;
  int hist[4][kMaxExperts];
  float psum[4][kMaxExperts];
  int slot_cur[kMaxExperts];  // slot mode: this tile's next grouped row per expert
};

// The 128-token tiles stream through a 4-slot ring: about
// 75 KB per CTA, so three CTAs share an SM and one's loads overlap another's
// MMAs and epilogue (a whole row block per CTA left one CTA per SM, idle
// between its load and its epilogue).
constexpr int kRouteLargeStages = 4;

template <int NP, int ST>
constexpr size_t route_smem_bytes() {
  return 1024 + (size_t)ST * (kRouteXTile + NP * 128) + sizeof(RouteSmem);
}

// ST: slab slots in the shared-memory ring.
template <int NP, int ST>
__global__ void __launch_bounds__(128) route_kernel(const __grid_constant__ CUtensorMap x_map,
                                                    const __grid_constant__ CUtensorMap w_map,
                                                    RouteArgs a) {
  constexpr int kWTile = NP * 128;  // NP experts x 64 columns
  constexpr int kRouteStages = ST;
  static_assert(ST >= 2 && ST <= kRouteMaxStages, "ring slots");
  extern __shared__ unsigned char route_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(route_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* x_tiles = base;
  unsigned char* w_tiles = base + kRouteStages * kRouteXTile;
  RouteSmem& sm = *reinterpret_cast<RouteSmem*>(w_tiles + kRouteStages * kWTile);

  const int E = a.n_experts, T = a.tokens;
  const int kb_count = a.dim / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int rows = route_tile(T);                  // token rows this CTA loads (32 or 128)
  const uint32_t x_bytes = (uint32_t)rows * 128u;  // of each 64-column slab

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRouteStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  (&sm.hist[0][0])[threadIdx.x] = 0;
  if (warp == 1) tmem_alloc(&sm.tmem, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  volatile int* abort_flag = &sm.abort;

  // the harness logit offset is a parameter too
  float bias[NP];
#pragma unroll
  for (int e = 0; e < NP; ++e) bias[e] = (a.bias != nullptr && e < E) ? __ldg(a.bias + e) : 0.f;

  // the router weight is a parameter: its slabs stream in before the
  // upstream kernel (which writes x) has finished
  const int pre = min(kRouteStages, kb_count);
  // When every slab has its own slot (d <= 64 * stages), all of them land on
  // one barrier and the MMAs run as one straight chain: a wait and a commit
  // per 4-MMA slab cost more than the MMAs themselves.
  const bool whole = kb_count <= kRouteStages;
  if (threadIdx.x == 0) {
    if (whole) mbar_arrive_expect_tx(&sm.full[0], (uint32_t)kb_count * (x_bytes + kWTile));
    for (int kb = 0; kb < pre; ++kb) {
      uint64_t* bar = whole ? &sm.full[0] : &sm.full[kb];
      if (!whole) mbar_arrive_expect_tx(bar, x_bytes + kWTile);
      tma_load_2d(w_tiles + kb * kWTile, &w_map, kb * 64, 0, bar);
    }
  }
  griddep_wait();
  griddep_launch();

  if (whole) {
    if (warp == 0 && lane == 0) {
      for (int kb = 0; kb < kb_count; ++kb)
        tma_load_2d(x_tiles + kb * kRouteXTile, &x_map, kb * 64, tile * rows, &sm.full[0]);
    } else if (warp == 1 && lane == 0) {
      const uint32_t idesc = make_idesc(kRouteM, NP);
      if (mbar_wait(&sm.full[0], 0, abort_flag, a.status, 21)) {
        tc_fence_after();
        for (int kb = 0; kb < kb_count; ++kb)
          mma_slab(sm.tmem, sw128_desc(x_tiles + kb * kRouteXTile),
                   sw128_desc(w_tiles + kb * kWTile), idesc, kb != 0);
      }
      mma_commit(&sm.done);
    }
    if (warp == 0 && lane == 0) mbar_drain(&sm.full[0], 0);  // every copy has landed
    __syncwarp();
  } else if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      static_assert(kRouteStages <= 32, "per-stage bit masks");
      uint32_t issued = 0, issued_phase = 0;  // per-stage bits
      for (int kb = 0; kb < pre; ++kb) {
        tma_load_2d(x_tiles + kb * kRouteXTile, &x_map, kb * 64, tile * rows, &sm.full[kb]);
        issued |= 1u << kb;
      }
      int stage = pre % kRouteStages;
      uint32_t phase = (uint32_t)(pre / kRouteStages) & 1u;
      for (int kb = pre; kb < kb_count; ++kb) {
        if (!mbar_wait_fast(&sm.empty[stage], phase ^ 1u, abort_flag, a.status, 20)) break;
        mbar_arrive_expect_tx(&sm.full[stage], x_bytes + kWTile);
        tma_load_2d(w_tiles + stage * kWTile, &w_map, kb * 64, 0, &sm.full[stage]);
        tma_load_2d(x_tiles + stage * kRouteXTile, &x_map, kb * 64, tile * rows,
                    &sm.full[stage]);
        issued |= 1u << stage;
        issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
        stage = stage + 1 == kRouteStages ? 0 : stage + 1;
        phase ^= stage == 0 ? 1u : 0u;
      }
      // every issued copy has landed before the CTA can exit
      for (int st = 0; st < kRouteStages; ++st)
        if (issued & (1u << st)) mbar_drain(&sm.full[st], (issued_phase >> st) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(kRouteM, NP);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = 0; kb < kb_count; ++kb) {
        if (!mbar_wait_fast(&sm.full[stage], phase, abort_flag, a.status, 21)) break;
        tc_fence_after();
        mma_slab(sm.tmem, sw128_desc(x_tiles + stage * kRouteXTile),
                 sw128_desc(w_tiles + stage * kWTile), idesc, kb != 0);
        mma_commit(&sm.empty[stage]);
        stage = stage + 1 == kRouteStages ? 0 : stage + 1;
        phase ^= stage == 0 ? 1u : 0u;
      }
      mma_commit(&sm.done);  // also fires when the loop stopped early: in-flight MMAs drain
    }
    __syncwarp();
  }

  // ---------------- epilogue: one thread per token ----------------
  mbar_wait(&sm.done, 0, abort_flag, a.status, 22);
  __syncwarp();
  tc_fence_after();
  const bool ok = *abort_flag == 0;
  float p[NP];
  const int t = tile * rows + (int)threadIdx.x;
  const bool valid_tok = ok && (int)threadIdx.x < rows && t < T;
  {
    uint32_t r[NP];
    const uint32_t addr = sm.tmem + ((uint32_t)(warp * 32) << 16);
    if constexpr (NP == 16) {
      tmem_ld16(addr, r);
    } else {
      uint32_t (&r32)[32] = reinterpret_cast<uint32_t (&)[32]>(r);
      tmem_ld32(addr, r32);
    }
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      const float l = __uint_as_float(r[e]) + bias[e];
      p[e] = e < E ? l : -INFINITY;
      m = fmaxf(m, p[e]);
    }
    float den = 0.f;
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      p[e] = e < E ? __expf(p[e] - m) : 0.f;
      den += p[e];
    }
    // one reciprocal and the fast exp: the per-thread chain is the cost here
    const float rden = 1.0f / den;
#pragma unroll
    for (int e = 0; e < NP; ++e) p[e] = valid_tok ? p[e] * rden : 0.f;
  }
  int i1 = 0, i2 = -1;
  float w1 = 0.f, w2 = 0.f;
  if (valid_tok) {
    // top-2; equal probabilities resolve to the lower expert id
    float v1 = p[0];
#pragma unroll
    for (int e = 1; e < NP; ++e)
      if (e < E && p[e] > v1) {
        v1 = p[e];
        i1 = e;
      }
    float v2 = -1.f;  // every probability is >= 0
#pragma unroll
    for (int e = 0; e < NP; ++e)
      if (e < E && e != i1 && p[e] > v2) {
        v2 = p[e];
        i2 = e;
      }
    const float sel = v1 + v2;
    w1 = v1 / sel;
    w2 = v2 / sel;
    reinterpret_cast<int2*>(a.indices)[t] = make_int2(i1, i2);
    reinterpret_cast<float2*>(a.weights)[t] = make_float2(w1, w2);
    if (a.weights_out != nullptr) reinterpret_cast<float2*>(a.weights_out)[t] = make_float2(w1, w2);
    if (a.indices64 != nullptr) {
      a.indices64[2 * t] = i1;
      a.indices64[2 * t + 1] = i2;
    }
    if (a.probs != nullptr) {
#pragma unroll
      for (int e = 0; e < NP; ++e)
        if (e < E) a.probs[(size_t)t * E + e] = p[e];
    }
    atomicAdd(&sm.hist[warp][i1], 1);
    atomicAdd(&sm.hist[warp][i2], 1);
  }
  // per-warp probability sums in a fixed shuffle order (deterministic)
  const float ps = warp_reduce_many<NP>(p, lane);
  if (lane < E) sm.psum[warp][lane] = ps;
  __syncthreads();
  if (ok) {
    const int chunk0 = tile * (rows / kGroupTokensPerBlock);
    const int n_chunks = (T + kGroupTokensPerBlock - 1) / kGroupTokensPerBlock;
    if (lane < E && warp < rows / kGroupTokensPerBlock && chunk0 + warp < n_chunks)
      a.tab.chunk_hist[(size_t)(chunk0 + warp) * E + lane] = sm.hist[warp][lane];
    if (threadIdx.x < E) {
      const int e = threadIdx.x;
      a.tab.tile_hist[(size_t)tile * E + e] =
          sm.hist[0][e] + sm.hist[1][e] + sm.hist[2][e] + sm.hist[3][e];
      a.tab.tile_probsum[(size_t)tile * E + e] =
          ((sm.psum[0][e] + sm.psum[1][e]) + sm.psum[2][e]) + sm.psum[3][e];
    }
  }
  if (a.slot_counts != nullptr && ok) {
    // slot mode: the grouping too.  One atomic per expert reserves this
    // tile's block of its region, shared-memory atomics hand out the rows in
    // it; each assignment's position, contribution slot (the lower expert id
    // first) and weight are written, then each warp copies its 32 token rows
    // (x, read again) to their two grouped rows.
    if (threadIdx.x < E) {
      const int e = threadIdx.x;
      const int cnt = sm.hist[0][e] + sm.hist[1][e] + sm.hist[2][e] + sm.hist[3][e];
      const int base = atomicAdd(a.slot_counts + e, cnt);
      if (base + cnt > a.slot_stride) {
        // counters left over from a call whose block never ran: nothing is
        // written past the expert's region (negative rows are skipped)
        report_status(a.status, kStatusBadIndex, 52, base + cnt);
        sm.slot_cur[e] = -(1 << 30);
      } else {
        sm.slot_cur[e] = e * a.slot_stride + base;
      }
    }
    __syncthreads();
    int r1 = -1, r2 = -1;
    if (valid_tok) {
      r1 = atomicAdd(&sm.slot_cur[i1], 1);
      r2 = atomicAdd(&sm.slot_cur[i2], 1);
      if (r1 < 0 || r2 < 0) {
        r1 = r2 = -1;
      } else {
        reinterpret_cast<int2*>(a.positions)[t] = make_int2(r1, r2);
        a.row_dst[r1] = 2 * t + (i1 < i2 ? 0 : 1);
        a.row_dst[r2] = 2 * t + (i2 < i1 ? 0 : 1);
        a.row_w[r1] = w1;
        a.row_w[r2] = w2;
      }
    }
    // four tokens' loads in flight before their stores (a load after a store
    // through another pointer waits for it: one memory round trip per token)
    const int nvec = a.dim >> 3;
    const uint4* __restrict__ xs = reinterpret_cast<const uint4*>(a.slot_x);
    uint4* __restrict__ grouped = reinterpret_cast<uint4*>(a.grouped);
    constexpr int kU = 4, kV = 4;  // tokens per batch; vectors per lane (d <= 1024)
    for (int u0 = 0; u0 < 32; u0 += kU) {
      uint4 v[kU][kV];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int tu = tile * rows + warp * 32 + u0 + u;
        const bool in = warp * 32 + u0 + u < rows && tu < T;
#pragma unroll
        for (int k = 0; k < kV; ++k) {
          const int c = lane + 32 * k;
          v[u][k] = in && c < nvec ? __ldg(xs + (size_t)tu * nvec + c) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int g1 = __shfl_sync(0xffffffffu, r1, u0 + u);
        const int g2 = __shfl_sync(0xffffffffu, r2, u0 + u);
        const int tu = tile * rows + warp * 32 + u0 + u;
        if (warp * 32 + u0 + u >= rows || tu >= T || g1 < 0) continue;  // uniform over the warp
#pragma unroll
        for (int k = 0; k < kV; ++k) {
          const int c = lane + 32 * k;
          if (c < nvec) {
            grouped[(size_t)g1 * nvec + c] = v[u][k];
            grouped[(size_t)g2 * nvec + c] = v[u][k];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sm.tmem, 32);
  }
}

// ---------------------------------------------------------------------------
// Router up to 4096 tokens, on CUDA cores: one CTA per 4-token tile (128
// CTAs at 512 tokens, where 32-token tensor-core tiles gave 16 CTAs, each MMA
// row block three-quarters padding; 2 warps with 16 experts, 4 with 32).  The router weight [E, d] is a parameter:
// every CTA copies it into shared memory before its grid-dependency wait, so
// the copy overlaps the kernel that writes x.  Each warp takes 32 / NP tokens
// (NP = E padded to 16 or 32): its lanes hold 16-byte vectors of the token
// rows in registers, accumulate the NP x (32 / NP) dots in packed fp32 pairs
// in one pass over d, and one warp_reduce_many leaves lane l with the logit
// of token l / NP, expert l % NP.  Softmax, top-2 (lower id on equal
// probabilities) and renormalisation are shuffle reductions over each
// token's NP lanes, with the tensor-core router's formulas.  The CTA writes
// its tile histogram and (in token order) its probability sums.
// ---------------------------------------------------------------------------
template <int NP>
__global__ void __launch_bounds__(32 * kRouteSmallTile)
    route_small_kernel(RouteArgs a, const __nv_bfloat16* __restrict__ x,
                       const __nv_bfloat16* __restrict__ router_w) {
  constexpr int TW = 32 / NP;               // tokens per warp
  constexpr int kTile = kRouteSmallTile;    // tokens per CTA: kTile / TW warps
  extern __shared__ __align__(16) uint4 rw_s[];    // [E][d / 8] router weight rows
  __shared__ int hist[NP];
  __shared__ float psum[kTile][NP];
  const int E = a.n_experts, T = a.tokens, nvec = a.dim >> 3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  {
    const uint4* wg = reinterpret_cast<const uint4*>(router_w);
    for (int i = threadIdx.x; i < E * nvec; i += blockDim.x) cp_async16(rw_s + i, wg + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  if (threadIdx.x < NP) hist[threadIdx.x] = 0;
  const int ex = lane % NP, tw = lane / NP;
  const float bias = (a.bias != nullptr && ex < E) ? __ldg(a.bias + ex) : 0.f;
  griddep_wait();
  griddep_launch();

  // this warp's token rows, 16-byte vectors c = lane + 32 k (d <= 1024)
  const int t_first = tile * kTile + warp * TW;
  float2 xf[TW][4][4];
#pragma unroll
  for (int t = 0; t < TW; ++t) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = lane + 32 * k;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (c < nvec && t_first + t < T)
        v = __ldg(reinterpret_cast<const uint4*>(x) + (size_t)(t_first + t) * nvec + c);
      xf[t][k][0] = bf16x2_to_float2(v.x);
      xf[t][k][1] = bf16x2_to_float2(v.y);
      xf[t][k][2] = bf16x2_to_float2(v.z);
      xf[t][k][3] = bf16x2_to_float2(v.w);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  float2 acc[TW * NP];
#pragma unroll
  for (int v = 0; v < TW * NP; ++v) acc[v] = make_float2(0.f, 0.f);
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    if (e < E) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = lane + 32 * k;
        if (c < nvec) {
          const uint4 w = rw_s[e * nvec + c];
          const float2 w0 = bf16x2_to_float2(w.x), w1 = bf16x2_to_float2(w.y);
          const float2 w2 = bf16x2_to_float2(w.z), w3 = bf16x2_to_float2(w.w);
#pragma unroll
          for (int t = 0; t < TW; ++t) {
            float2 s = acc[t * NP + e];
            s = __ffma2_rn(w0, xf[t][k][0], s);
            s = __ffma2_rn(w1, xf[t][k][1], s);
            s = __ffma2_rn(w2, xf[t][k][2], s);
            s = __ffma2_rn(w3, xf[t][k][3], s);
            acc[t * NP + e] = s;
          }
        }
      }
    }
  }
  float dots[TW * NP];
#pragma unroll
  for (int v = 0; v < TW * NP; ++v) dots[v] = acc[v].x + acc[v].y;
  // lane l: logit of token l / NP, expert l % NP
  const float logit = warp_reduce_many<TW * NP>(dots, lane) + bias;
  const bool valid_e = ex < E;
  const int t = t_first + tw;
  const bool valid_t = t < T;
  float m = valid_e ? logit : -INFINITY;
#pragma unroll
  for (int o = NP / 2; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float p = valid_e ? __expf(logit - m) : 0.f;
  float den = p;
#pragma unroll
  for (int o = NP / 2; o >= 1; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  p = valid_t ? p * (1.0f / den) : 0.f;
  // top-2; equal probabilities resolve to the lower expert id (every p >= 0)
  float v1 = valid_e ? p : -1.f;
  int i1 = ex;
  best_of_group<NP>(v1, i1);
  float v2 = (valid_e && ex != i1) ? p : -1.f;
  int i2 = ex;
  best_of_group<NP>(v2, i2);
  if (valid_t && ex == 0) {
    const float sel = v1 + v2;
    const float w1 = v1 / sel, w2 = v2 / sel;
    reinterpret_cast<int2*>(a.indices)[t] = make_int2(i1, i2);
    reinterpret_cast<float2*>(a.weights)[t] = make_float2(w1, w2);
    if (a.weights_out != nullptr) reinterpret_cast<float2*>(a.weights_out)[t] = make_float2(w1, w2);
    if (a.indices64 != nullptr) {
      a.indices64[2 * t] = i1;
      a.indices64[2 * t + 1] = i2;
    }
    atomicAdd(&hist[i1], 1);
    atomicAdd(&hist[i2], 1);
  }
  if (valid_t && valid_e && a.probs != nullptr) a.probs[(size_t)t * E + ex] = p;
  psum[warp * TW + tw][ex] = p;
  if (a.slot_counts != nullptr) {
    // slot mode: the grouping too.  Lane 0 of each token's group takes the
    // next slot of both experts and writes the position, contribution slot
    // (the lower expert id first) and weight; then the warp writes its
    // tokens' rows to their two grouped rows from the registers that hold
    // them (exact bf16 values, packed again).
    int r1 = -1, r2 = -1;
    if (valid_t && ex == 0) {
      const float sel = v1 + v2;
      const int s1 = atomicAdd(a.slot_counts + i1, 1), s2 = atomicAdd(a.slot_counts + i2, 1);
      if (s1 >= a.slot_stride || s2 >= a.slot_stride) {
        // counters left over from a call whose block never ran: nothing is
        // written past the expert's region
        report_status(a.status, kStatusBadIndex, 51, max(s1, s2));
      } else {
        r1 = i1 * a.slot_stride + s1;
        r2 = i2 * a.slot_stride + s2;
        reinterpret_cast<int2*>(a.positions)[t] = make_int2(r1, r2);
        a.row_dst[r1] = 2 * t + (i1 < i2 ? 0 : 1);
        a.row_dst[r2] = 2 * t + (i2 < i1 ? 0 : 1);
        a.row_w[r1] = v1 / sel;
        a.row_w[r2] = v2 / sel;
      }
    }
    uint4* grouped = reinterpret_cast<uint4*>(a.grouped);
#pragma unroll
    for (int u = 0; u < TW; ++u) {
      const int g1 = __shfl_sync(0xffffffffu, r1, u * NP);
      const int g2 = __shfl_sync(0xffffffffu, r2, u * NP);
      if (t_first + u >= T || g1 < 0) continue;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = lane + 32 * k;
        if (c < nvec) {
          uint4 v;
          v.x = pack_bf16x2(xf[u][k][0].x, xf[u][k][0].y);
          v.y = pack_bf16x2(xf[u][k][1].x, xf[u][k][1].y);
          v.z = pack_bf16x2(xf[u][k][2].x, xf[u][k][2].y);
          v.w = pack_bf16x2(xf[u][k][3].x, xf[u][k][3].y);
          grouped[(size_t)g1 * nvec + c] = v;
          grouped[(size_t)g2 * nvec + c] = v;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < E) {
    const int e = threadIdx.x;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kTile; ++k) s += psum[k][e];
    a.tab.tile_hist[(size_t)tile * E + e] = hist[e];
    a.tab.tile_probsum[(size_t)tile * E + e] = s;
  }
}

template <int NP>
static int launch_route_small(const RouteArgs& args, const void* x, const void* router_w,
                              cudaStream_t stream) {
  const size_t smem = (size_t)args.n_experts * args.dim * 2;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(route_small_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             64 * 1024) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  return launch_pdl(route_small_kernel<NP>, dim3(route_blocks(args.tokens)),
                    dim3(32 * kRouteSmallTile * NP / 32), smem, stream, args,
                    static_cast<const __nv_bfloat16*>(x),
                    static_cast<const __nv_bfloat16*>(router_w)) == cudaSuccess
             ? 0
             : -2;
}

template <int NP, int ST>
static int launch_route_st(const RouteArgs& args, const CUtensorMap* x_map,
                           const CUtensorMap* w_map, cudaStream_t stream) {
  constexpr size_t smem = route_smem_bytes<NP, ST>();
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(route_kernel<NP, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  return launch_pdl(route_kernel<NP, ST>, dim3(route_blocks(args.tokens)), dim3(128), smem,
                    stream, *x_map, *w_map, args) == cudaSuccess
             ? 0
             : -2;
}

int launch_route(const RouteArgs& args, const void* x, const void* router_w,
                 const CUtensorMap* x_map, const CUtensorMap* w_map, cudaStream_t stream) {
  if (args.tokens == 0) return 0;
  if (args.dim % 64 || args.dim > 1024) return -1;
  const bool e16 = route_experts_padded(args.n_experts) == 16;
  if (route_tile(args.tokens) == kRouteSmallTile)
    return e16 ? launch_route_small<16>(args, x, router_w, stream)
               : launch_route_small<32>(args, x, router_w, stream);
  return e16 ? launch_route_st<16, kRouteLargeStages>(args, x_map, w_map, stream)
             : launch_route_st<32, kRouteLargeStages>(args, x_map, w_map, stream);
}

// ---------------------------------------------------------------------------
// grouping: stable slots and the 16-byte row scatter
//
// Block b owns assignments [64 b, 64 b + 64) (tokens [32 b, 32 b + 32), the
// router's chunk b).  Its exclusive per-expert prefix is the sum of the tile
// histograms before its router tile plus the chunk histograms before it in
// that tile; the per-expert totals (for the overflow bases) are the sum of all
// tile histograms.  Every block computes both itself from a few KB in L2, so
// no block waits for another.  Everything independent is requested up front:
// the assignment expert ids and (async copies) the token rows this split
// copies.  Then ranks come from warp match, and every assignment's grouped row
// is written along with where its expert output goes (token-major slot
// 2 t + j, j = 0 for the lower expert id of the token's pair, the order the
// reference adds them) and its route weight.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) group_kernel(GroupArgs a) {
  constexpr int kAssign = 2 * kGroupTokensPerBlock;  // 64 per block
  extern __shared__ __align__(16) unsigned char group_smem[];
  __shared__ int warp_cnt[2][kMaxExperts];
  __shared__ int prefix_s[kMaxExperts];
  __shared__ int count_s[kMaxExperts];
  __shared__ int obase_s[kMaxExperts];
  __shared__ uint4* dst_s[kAssign];  // where each assignment's row goes
  __shared__ int dbase_s[kEpMaxRanks];
  __shared__ int red_before[128], red_total[128];
  __shared__ float red_psum[128];
  const int E = a.n_experts, C = a.capacity, T = a.tokens, d = a.dim;
  const int blk = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = d >> 3;
  const bool writer = blk == 0 && split == 0;  // writes tables, counts and statistics

  // this split's assignments [lo, hi) cover tokens [lo/2, hi/2) of the block
  const int per = (kAssign + a.copy_split - 1) / a.copy_split;
  const int lo = min(kAssign, split * per) & ~1, hi = min(kAssign, lo + per + (per & 1));
  const int tok_lo = blk * kGroupTokensPerBlock + lo / 2;
  const int n_tok = max(0, min(T - tok_lo, (hi - lo) / 2));
  uint4* x_s = reinterpret_cast<uint4*>(group_smem);
  auto stage_rows = [&] {
    const uint4* xg = reinterpret_cast<const uint4*>(a.x + (size_t)tok_lo * d);
    for (int i = tid; i < n_tok * nvec; i += blockDim.x) cp_async16(x_s + i, xg + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // The token rows are the router's input: complete before the router kernel
  // that precedes this one began, so they are read before the dependency
  // wait.  When the router was folded into the kernel that writes them
  // (x_from_upstream), that kernel is the one being waited for.
  if (!a.x_from_upstream) stage_rows();
  griddep_wait();
  griddep_launch();
  if (a.x_from_upstream) stage_rows();

  const int a_idx = blk * kAssign + tid;
  int e = -1;
  if (warp < 2 && a_idx < 2 * T) e = __ldg(a.indices + a_idx);
  {
    // prefix and totals: thread (phase, expert) sums every P-th tile row
    const int P = blockDim.x / E;
    // whole router tiles before this block's first token; with tiles larger
    // than a block, the 32-token chunks of its own tile before it come after
    const int tile_tok = route_tile(T), n_tiles = route_blocks(T);
    const int tiles_before = blk * kGroupTokensPerBlock / tile_tok;
    const int chunk_from = tiles_before * tile_tok / kGroupTokensPerBlock;
    int before = 0, total = 0;
    float ps = 0.f;
    if (tid < P * E) {
      // eight rows' loads in flight before their sums (a load-add loop would
      // wait on each L2 round trip in turn: 64 of them per thread at 512
      // router tiles); the sums keep the row order
      constexpr int U = 8;
      const int ex = tid % E;
      for (int r0 = tid / E; r0 < n_tiles; r0 += U * P) {
        int v[U];
        float pv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int r = r0 + u * P;
          v[u] = r < n_tiles ? __ldcg(a.tab.tile_hist + (size_t)r * E + ex) : 0;
          pv[u] = (writer && r < n_tiles) ? __ldcg(a.tab.tile_probsum + (size_t)r * E + ex) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int r = r0 + u * P;
          total += v[u];
          if (r < tiles_before) before += v[u];
          if (writer && r < n_tiles) ps += pv[u];
        }
      }
    }
    red_before[tid] = before;
    red_total[tid] = total;
    red_psum[tid] = ps;
    if (tid < 2 * kMaxExperts) (&warp_cnt[0][0])[tid] = 0;
    __syncthreads();
    if (tid < E) {
      int b = 0, c = 0;
      float s = 0.f;
      for (int ph = 0; ph < P; ++ph) {
        b += red_before[ph * E + tid];
        c += red_total[ph * E + tid];
        s += red_psum[ph * E + tid];
      }
      for (int ch = chunk_from; ch < blk; ++ch)
        b += __ldcg(a.tab.chunk_hist + (size_t)ch * E + tid);
      prefix_s[tid] = b;
      count_s[tid] = c;
      red_psum[tid] = s;  // slot tid is only read by this thread from here on
    }
    __syncthreads();
  }
  if (!a.ep_packed) {
    // overflow bases in expert id order: an exclusive warp scan of the overflow counts
    if (warp == 0) {
      const int over = lane < E ? max(count_s[lane] - C, 0) : 0;
      int incl = over;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (lane < E) obase_s[lane] = E * C + incl - over;
    }
  } else if (tid == 0) {
    // destination-major for expert parallelism: experts in the send order
    // (and each destination's first grouped row, for rows sent from here)
    int base = E * C;
    for (int q = 0; q < kEpMaxRanks; ++q) dbase_s[q] = 0;
    for (int q = 0; q < E; ++q) {
      const int ex = a.ep_order[q];
      if (q == 0 || a.ep_dest[ex] != a.ep_dest[a.ep_order[q - 1]]) dbase_s[a.ep_dest[ex]] = base;
      obase_s[ex] = base;
      base += max(count_s[ex] - C, 0);
    }
  }
  __syncthreads();
  if (writer && tid < E) {
    const int c = count_s[tid];
    a.tab.counts[tid] = c;
    if (a.counts_out != nullptr) a.counts_out[tid] = c;
    if (C > 0) {
      a.tab.seg_rows[tid] = min(c, C);
      a.tab.seg_base[tid] = tid * C;
      a.tab.seg_rows[E + tid] = max(c - C, 0);
      a.tab.seg_base[E + tid] = obase_s[tid];
    } else {
      // packed rows: the expert's one segment comes first, like a capacity segment
      a.tab.seg_rows[tid] = c;
      a.tab.seg_base[tid] = obase_s[tid];
      a.tab.seg_rows[E + tid] = 0;
      a.tab.seg_base[E + tid] = obase_s[tid] + c;
    }
    const float util = (float)c / (float)(2 * T);
    a.tab.stats[tid] = util;
    if (a.stats_out != nullptr) a.stats_out[tid] = util;
    // aux = E * sum_e util_e * mean_t p_te: the terms in parallel (two
    // divisions each), summed in expert order by one lane below
    red_total[tid] = __float_as_int(util * (red_psum[tid] / (float)T));
  }
  if (writer) {
    __syncwarp();
    if (tid == 0) {
      float aux = 0.f;
      for (int x = 0; x < E; ++x) aux += __int_as_float(red_total[x]);
      a.tab.stats[E] = (float)E * aux;
      if (a.stats_out != nullptr) a.stats_out[E] = (float)E * aux;
    }
  }

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
    uint4* dst = nullptr;
    if (e >= 0) {
      const int slot = prefix_s[e] + (warp == 1 ? warp_cnt[0][e] : 0) + rank;
      row = slot < C ? e * C + slot : obase_s[e] + (slot - C);
      if (split == 0) {
        a.positions[a_idx] = row;
        if (a.positions_out != nullptr) a.positions_out[a_idx] = row;
        a.row_dst[row] = (a_idx & ~1) + (e < partner ? 0 : 1);
        a.row_w[row] = __ldg(a.weights + a_idx);
      }
      if (a.ep_recv[0] == nullptr) {
        dst = reinterpret_cast<uint4*>(a.grouped + (size_t)row * d);
      } else {
        // straight into the destination's receive region (peer memory)
        const int q = a.ep_dest[e], k = row - dbase_s[q];
        if (k >= 0 && k < a.ep_region)
          dst = reinterpret_cast<uint4*>(a.ep_recv[q] + (size_t)k * d);
        else if (split == 0)
          report_status(a.status, kStatusBadIndex, 2, row);
      }
    }
    dst_s[tid] = dst;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  // scatter this split's rows from shared memory
  for (int j = lo + warp; j < hi; j += 4) {
    uint4* dst = dst_s[j];
    const int lt = (j - lo) >> 1;
    if (dst == nullptr || lt >= n_tok) continue;
    for (int c = lane; c < nvec; c += 32) dst[c] = x_s[lt * nvec + c];
  }
  // rows stored into another GPU's memory are visible there before this
  // kernel completes, so the send kernel after it may raise the arrival flags
  if (a.ep_recv[0] != nullptr) __threadfence_system();
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
//
// With the peer exchange (wait_flags set), the expert outputs arrive from the
// other ranks: the CTA first waits (bounded) until every expert rank has
// raised its return flag for this call.
template <int V>
__global__ void __launch_bounds__(128) ep_combine_kernel(EpCombineArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  griddep_wait();
  griddep_launch();
  if (a.wait_flags != nullptr) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    if (threadIdx.x < a.wait_ranks) {
      const unsigned e = *reinterpret_cast<const volatile unsigned*>(a.wait_epoch);
      if (!wait_flag(a.wait_flags + threadIdx.x, e, a.wait_ns, a.wait_status)) {
        report_status(a.wait_status, kStatusWaitTimeout, 23, threadIdx.x);
        failed = 1;
      }
    }
    __syncthreads();
    if (failed) return;
  }
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
