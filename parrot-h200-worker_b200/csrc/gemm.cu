// Grouped expert GEMMs on the 5th-generation tensor cores (N4).
//
// One persistent kernel computes, for every (segment, 128-row weight tile,
// token tile) work unit,  D[128 x N] = W_tile[128 x K] * X_tile[N x K]^T
// with tcgen05.mma (A and B from shared memory, fp32 accumulator in TMEM).
// Weights are the MMA M side ("swap-AB"): a routed expert sees a few dozen
// to a few thousand token rows, and putting tokens on N keeps every MMA
// at M = 128 while N shrinks to the rows actually present (multiple of 16).
// Token tiles are up to 256 rows, loaded as 64-row boxes so a tile with few
// rows moves few bytes; a weight tile is streamed once per 256 tokens of its
// expert, which matters because routing is often skewed (an expert can take
// most of a batch while others are empty).
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: 128-byte-swizzled K slabs of W and X into a
//               4- or 6-stage shared-memory ring (no multicast anywhere).
//   warp 1      TMEM allocator + single-thread MMA issuer; tcgen05.commit
//               frees ring stages and publishes finished accumulators.
//   warps 2..9  epilogue: warps w and w + 4 read TMEM lane quarter w % 4 and
//               take alternate 32-column (token) chunks; the loads of the next
//               chunk are in flight while the current one is converted.  A
//               chunk is read as two 16-lane fragments (tcgen05.ld .16x256b),
//               so each thread holds two adjacent tokens of a feature:
//               SwiGLU mode:  each 16-row group of the weight tile is 8 gate
//                             rows then the same 8 features' up rows, so a
//                             thread holds gate and up of one feature:
//                             h = bf16(silu(bf16 g) * bf16 u)
//               plain mode:   y = bf16(acc) (routed: bf16(bf16(y) * bf16(w)))
//               packed two per register, written transposed (token-major) into
//               the warp's own shared-memory tile by stmatrix, and copied out
//               as 16-byte vectors (scattered rows: one destination per token).
// Two TMEM accumulators (2 x 256 columns) let the epilogue of one unit run
// under the MMAs of the next.
//
// CTA pairs (PAIR, the gate/up GEMM at 256-token tiles): a 2-CTA cluster
// runs M = 256 tcgen05.mma.cta_group::2 over its two CTAs' shared memory —
// each CTA's TMA loads its own 128 weight rows and half of the token tile
// (N / 2 rows) and signals the leader's barrier; the leader issues the MMAs
// and multicasts their completions to both CTAs' ring and accumulator
// barriers; each CTA's epilogue reads its own TMEM rows and arrives on the
// leader's accumulator-free barrier.  No multicast load.
//
// Scheduling.  With primary units enabled, CTA b < E * MT owns the first
// token tile of expert b / MT, M tile b % MT (its "primary" unit) and, before
// its grid-dependency wait, pulls that unit's weights into L2 — they depend
// on nothing the upstream kernel writes.  Every other unit (further token
// tiles, the shared expert, everything when primaries are off) is dealt
// round-robin over the CTAs, CTAs without a primary unit (empty experts,
// b >= E * MT) first.  Launched with programmatic dependent launch.  Every
// mbarrier wait is bounded; a timeout records a status code, drains in-flight
// copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace parrot {
namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int BK = kGemmBlockK;
constexpr int kSubRows = kGemmSubRows;        // 64-row activation boxes
constexpr int kTileA = BM * BK * 2;           // 16 KB
constexpr int kSubBytes = kSubRows * BK * 2;  // 8 KB
constexpr int kChunk = 32;                    // TMEM columns per epilogue step
constexpr int kEpiWarps = 8;                  // two per TMEM lane quarter
constexpr int kEpiTile = 32 * 64;             // per-warp staging: 32 tokens x 32 features bf16
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSegMax = 2 * kMaxExperts;

// Token tile BN (128 or 256 rows).  PAIR: the tile runs on a CTA pair
// (cta_group::2, M = 256 weight rows), each CTA holding BN / 2 token rows of B.
// The ring holds as many stages as shared memory allows (at small batches a
// unit's loads are bound by the bytes in flight per SM over the L2 latency):
// 6 of 16 + 16 KB (BN = 128, or a pair's 256-token tile), 4 of 16 + 32 KB
// (BN = 256 on one CTA); the two TMEM accumulators take 2 * BN columns.
template <int BN, bool PAIR>
struct GemmCfg {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;  // token rows of B in this CTA
  static constexpr int kTileB = kBRows * BK * 2;
  static constexpr int kStages = (PAIR || BN == 128) ? 6 : 4;
  static constexpr int kMPerUnit = PAIR ? 2 : 1;      // 128-row weight tiles per unit
};

template <int BN, bool PAIR>
struct __align__(16) SmemTail {
  uint64_t full[GemmCfg<BN, PAIR>::kStages];
  uint64_t empty[GemmCfg<BN, PAIR>::kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int scan_carry;
  int has_primary;      // this CTA's schedule: primary unit present,
  int rank;             // its position in the round-robin over other units
  int stride;           // (CTAs, or CTA pairs, sharing that round-robin)
  int n_secondary;      // and how many such units exist
  alignas(16) int unit_dst[BN];  // plain-mode scatter: destination row of each token row
  alignas(16) uint16_t unit_wb[BN];  // and its route weight in bf16 (read as pairs)
  int prefix[kSegMax + 2];
  int seg_rows[kSegMax];
  int seg_base[kSegMax];
  int seg_expert[kSegMax];
  int seg_shift[kSegMax];  // output row - input row (rows sent back to their source)
};

template <int BN, bool PAIR>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)GemmCfg<BN, PAIR>::kStages * (kTileA + GemmCfg<BN, PAIR>::kTileB) +
         kEpiWarps * kEpiTile + sizeof(SmemTail<BN, PAIR>);
}

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
}

struct Unit {
  bool routed;
  int w_row;      // row of the unit's first weight tile in the tiled weight view
  int x_row;      // first token row of the tile
  int valid;      // token rows present (<= BN)
  int k_blocks;
  int out_col;    // first output feature
  int out_row;    // output row of the tile's first token row
  __nv_bfloat16* out;
  int ld;
};

template <bool PAIR>
__device__ __forceinline__ bool primaries_on(const GemmArgs& g) {
  return !PAIR && g.static_routed && g.n_experts * g.m_tiles_routed <= (int)gridDim.x;
}

// token tiles of segment s handed out round-robin (the primary tile excluded)
template <int BN>
__device__ __forceinline__ int secondary_tiles(int s, int rows, bool primary, int n_experts) {
  const int tiles = (rows + BN - 1) / BN;
  return (primary && s < n_experts) ? max(tiles - 1, 0) : tiles;
}

template <int BN, bool PAIR>
__device__ __forceinline__ Unit routed_unit(const GemmArgs& g, const SmemTail<BN, PAIR>& t, int s,
                                            int mt, int nt) {
  Unit r;
  const int e = t.seg_expert[s];
  r.routed = true;
  r.w_row = (e * g.m_tiles_routed + mt) * g.k_blocks_routed * BM;
  r.x_row = t.seg_base[s] + nt * BN;
  r.valid = max(0, min(BN, t.seg_rows[s] - nt * BN));
  r.k_blocks = g.k_blocks_routed;
  if (g.out_peer_segs > 0) {
    r.out = g.out_peer[s / g.out_peer_segs];
    r.out_row = r.x_row + t.seg_shift[s];
  } else {
    r.out = g.out_routed;
    r.out_row = r.x_row;
  }
  r.ld = g.ld_out_routed;
  r.out_col = mt * (g.mode == kGemmSwiGLU ? BM / 2 : BM);
  return r;
}

// The k-th unit of this CTA; false when it has no more.
//   primary (k == 0, when present): segment e = b / MT, M tile b % MT, token tile 0
//   secondary j = rank + i * stride:  routed tiles segment by segment (M unit
//                                     major), then the shared expert's tiles
// A unit covers kMPerUnit weight tiles: on a CTA pair, M unit u is tiles
// 2u (rank 0) and 2u + 1 (rank 1), and this CTA loads and stores its own.
// seg: the caller's segment cursor (0 before its first call, k increasing):
// j grows with k, so the segment search resumes where the last one stopped
// (from segment 0 each time it was up to 32 dependent shared-memory loads
// per unit, on the critical path of the producer, the MMA issuer and the
// epilogue alike).
template <int BN, bool PAIR>
__device__ __forceinline__ bool cta_unit(int k, const GemmArgs& g, const SmemTail<BN, PAIR>& t,
                                         Unit& r, int crank, int& seg) {
  constexpr int MD = GemmCfg<BN, PAIR>::kMPerUnit;
  const int MT = g.m_tiles_routed;
  if (t.has_primary) {
    if (k == 0) {
      const int e = blockIdx.x / MT;
      r = routed_unit<BN, PAIR>(g, t, e, blockIdx.x - e * MT, 0);
      return true;
    }
    --k;
  }
  const int j = t.rank + k * t.stride;
  if (j >= t.n_secondary) return false;
  const int n_routed = t.prefix[g.n_seg];
  if (j < n_routed) {
    const bool prim = primaries_on<PAIR>(g);
    int s = seg;
    while (t.prefix[s + 1] <= j) ++s;
    seg = s;
    const int local = j - t.prefix[s];
    const int n_tiles = secondary_tiles<BN>(s, t.seg_rows[s], prim, g.n_experts);
    const int mu = local / n_tiles;
    const int nt = local - mu * n_tiles + ((prim && s < g.n_experts) ? 1 : 0);
    r = routed_unit<BN, PAIR>(g, t, s, MD * mu + crank, nt);
    return true;
  }
  const int shared_tiles = (g.shared_rows + BN - 1) / BN;
  const int local = j - n_routed;
  const int mu = local / shared_tiles, nt = local - mu * shared_tiles;
  const int mt = MD * mu + crank;
  r.routed = false;
  r.w_row = mt * g.k_blocks_shared * BM;
  r.x_row = nt * BN;
  r.out_row = r.x_row;
  r.valid = min(BN, g.shared_rows - nt * BN);
  r.k_blocks = g.k_blocks_shared;
  r.out = g.out_shared;
  r.ld = g.ld_out_shared;
  r.out_col = mt * (g.mode == kGemmSwiGLU ? BM / 2 : BM);
  return true;
}

// SiLU of every bf16 value, rounded to bf16: silu_lut[bits(x)] =
// bf16(x / (1 + expf(-x))), the expression PyTorch evaluates in fp32 for a
// bf16 tensor.  The gate projection is rounded to bf16 before SiLU (the
// reference materialises it as a bf16 tensor), so the epilogue looks its
// SiLU up instead of spending an exp and an IEEE divide per element.
__device__ __nv_bfloat16 silu_lut[1 << 16];

__global__ void build_silu_lut_kernel() {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (1 << 16)) return;
  const float x = __uint_as_float((uint32_t)i << 16);
  silu_lut[i] = __float2bfloat16_rn(x / (1.0f + expf(-x)));
}

// The same bf16 SiLU without a table read for almost every input.  A table
// lookup per element is a 32-lane gather over 128 KB: nearly one L1
// wavefront per lane, which made the SwiGLU epilogue L1-bound.  Instead
//   y = x * rcp.approx(1 + ex2.approx(-x * log2 e))
// is within 2^-17 (relative) of the exactly evaluated x / (1 + expf(-x)) for
// 2^-20 <= |x| <= 64 (the ex2 argument carries |x| * 2^-24 of rounding error,
// ex2 and rcp a few ulps each), i.e. within about 100 float ulps; when y is
// more than 256 ulps away from the bf16 rounding midpoint both round to the
// same bf16.  Inputs outside the range, and the ~1% of results near a
// midpoint, read the table.  silu_bf16_fast() is checked against PyTorch's
// bf16 SiLU for all 65,536 inputs.
struct SiluFast {
  uint16_t bits;
  bool exact;  // false: read silu_lut instead
};

__device__ __forceinline__ SiluFast silu_bf16_fast(uint16_t xb) {
  const float x = __uint_as_float((uint32_t)xb << 16);
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  const uint32_t yb = __float_as_uint(x * r);
  const float ax = fabsf(x);
  const bool near_mid = ((yb & 0xFFFFu) - (0x8000u - 256u)) < 512u;
  SiluFast out;
  out.bits = (uint16_t)((yb + 0x8000u) >> 16);
  out.exact = ax >= 0x1p-20f && ax <= 64.0f && !near_mid;
  return out;
}

__global__ void silu_bf16_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint16_t xb = x[i];
  const SiluFast f = silu_bf16_fast(xb);
  y[i] = f.exact ? f.bits : __bfloat16_as_ushort(silu_lut[xb]);
}



// Slot mode: the counts, router statistics and positions copy that the
// grouping kernel writes otherwise, by the epilogue warps of the last CTA
// before its first unit (the segment table in shared memory holds the
// counts).  Utilisation = count / 2T; aux = E * sum_e util_e * (probability
// sum_e / T) with the probability sums added in the grouping kernel's order:
// per (phase, expert) over every P-th router tile, P = 128 / E, then over the
// phases.  scratch: 128 floats of the epilogue staging tiles, unused yet.
template <int BN, bool PAIR>
__device__ __forceinline__ void slot_stats(const GemmArgs& g, const SmemTail<BN, PAIR>& t,
                                        float* scratch, int tid) {
  const GemmArgs::SlotStats& st = g.st;
  const int E = g.n_experts, P = 128 / E, A2 = 2 * st.tokens;
  float ps = 0.f;
  if (tid < P * E) {
    constexpr int U = 16;  // sixteen tiles' loads in flight before their in-order sum
    const int ex = tid % E;
    for (int r0 = tid / E; r0 < st.route_tiles; r0 += U * P) {
      float pv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int r = r0 + u * P;
        pv[u] = r < st.route_tiles ? __ldcg(st.tile_probsum + (size_t)r * E + ex) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (r0 + u * P < st.route_tiles) ps += pv[u];
    }
  }
  if (tid < 128) scratch[tid] = ps;
  epi_bar();
  float term = 0.f;
  if (tid < E) {
    float sum = 0.f;
    for (int ph = 0; ph < P; ++ph) sum += scratch[ph * E + tid];
    const int cnt = t.seg_rows[tid];
    st.counts[tid] = cnt;
    if (st.counts_out != nullptr) st.counts_out[tid] = cnt;
    const float util = (float)cnt / (float)A2;
    st.stats[tid] = util;
    if (st.stats_out != nullptr) st.stats_out[tid] = util;
    term = util * (sum / (float)st.tokens);
  }
  epi_bar();
  if (tid < E) scratch[tid] = term;
  epi_bar();
  if (tid == 0) {
    float aux = 0.f;
    for (int x = 0; x < E; ++x) aux += scratch[x];
    st.stats[E] = (float)E * aux;
    if (st.stats_out != nullptr) st.stats_out[E] = (float)E * aux;
  }
  if (st.positions_out != nullptr)
    for (int i = tid; i < A2; i += 32 * kEpiWarps) st.positions_out[i] = st.positions[i];
  epi_bar();  // the staging tiles are the epilogue's again
}

template <int BN, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w_routed,
                        const __grid_constant__ CUtensorMap tm_x_routed,
                        const __grid_constant__ CUtensorMap tm_w_shared,
                        const __grid_constant__ CUtensorMap tm_x_shared, const GemmArgs g) {
  using Cfg = GemmCfg<BN, PAIR>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kTileB = Cfg::kTileB;
  constexpr int kTmemCols = 2 * BN;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles_a = base;
  unsigned char* tiles_b = base + kStages * kTileA;
  unsigned char* epi_tiles = tiles_b + kStages * kTileB;
  SmemTail<BN, PAIR>& t =
      *reinterpret_cast<SmemTail<BN, PAIR>*>(epi_tiles + kEpiWarps * kEpiTile);
  const int crank = PAIR ? (int)cluster_ctarank() : 0;  // rank in the CTA pair

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_seg = g.n_seg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&t.full[s], 1);
      mbar_init(&t.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&t.tfull[a], 1);
      mbar_init(&t.tempty[a], PAIR ? 2 * kEpiWarps : kEpiWarps);  // both CTAs' epilogues
    }
    mbar_init(&t.drain, 1);
    t.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrival
  if (warp == 1) {
    if constexpr (PAIR) {
      // both CTAs' warp 1, same shared-memory destination
      asm volatile(
          "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
              smem_u32(&t.tmem_base)),
          "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile(
          "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
              smem_u32(&t.tmem_base)),
          "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // The weights of this CTA's likely primary unit go to L2 before the
  // upstream kernel has finished (they depend on nothing it writes) — only
  // when most experts are likely to have rows (at least eight assignments per
  // expert on average): at decode sizes it would stream every expert's weights
  // for the two that are used.
  if (warp == 0 && lane == 0 && primaries_on<PAIR>(g) &&
      (int)blockIdx.x < g.n_experts * g.m_tiles_routed && g.w_routed != nullptr &&
      2 * g.shared_rows >= 8 * g.n_experts) {
    const char* w = static_cast<const char*>(g.w_routed) +
                    (size_t)blockIdx.x * g.k_blocks_routed * kTileA;
    for (int kb = 0; kb < g.k_blocks_routed; kb += 2) {
      const unsigned bytes = (unsigned)min(2, g.k_blocks_routed - kb) * kTileA;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w + (size_t)kb * kTileA),
                   "r"(bytes)
                   : "memory");
    }
  }
  griddep_wait();

  if (warp == 2 || warp == 3) {
    // segment tables and the prefix of the round-robin (secondary) units:
    // one thread per segment, then a two-warp inclusive scan
    const int s = threadIdx.x - 64;
    const bool prim = primaries_on<PAIR>(g);
    constexpr int MD = Cfg::kMPerUnit;
    int rows = 0;
    if (s < n_seg) {
      rows = g.seg_rows[s];
      if (g.seg_stride > 0 && rows > g.seg_stride) {
        // slot mode: a counter beyond its region (left over from a routing
        // call whose block never ran) is reported and read no further
        report_status(g.status, kStatusBadIndex, 53, rows);
        rows = g.seg_stride;
      }
      t.seg_rows[s] = rows;
      t.seg_base[s] = g.seg_stride > 0 ? s * g.seg_stride : g.seg_base[s];
      t.seg_expert[s] = g.seg_expert != nullptr ? g.seg_expert[s] : s % g.n_experts;
      if (g.out_peer_segs > 0) {
        // the receive kernel checked that base + rows stays in the return region
        const int q = s / g.out_peer_segs;
        t.seg_shift[s] = __ldg(g.out_peer_base + q) - q * g.out_peer_region;
      }
    }
    int incl =
        s < n_seg ? secondary_tiles<BN>(s, rows, prim, g.n_experts) * (g.m_tiles_routed / MD) : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (warp == 2 && lane == 31) t.scan_carry = incl;
    asm volatile("bar.sync 2, 64;" ::: "memory");
    if (warp == 3) incl += t.scan_carry;
    if (s < n_seg) t.prefix[s + 1] = incl;
    if (s == 0) t.prefix[0] = 0;
    if (warp == 2) {
      // this CTA's place in the schedule (lane e looks at expert e)
      const int E = g.n_experts, MT = g.m_tiles_routed, b = blockIdx.x;
      const unsigned empty = __ballot_sync(0xffffffffu, lane < E && rows == 0);
      if (lane == 0) {
        // a CTA pair shares one place in the round-robin
        int has = 0, rank = PAIR ? b / 2 : b;
        if (prim) {
          const int n_empty = __popc(empty);
          const int n_free = n_empty * MT + ((int)gridDim.x - E * MT);
          if (b < E * MT) {
            const int e = b / MT;
            const unsigned below = (1u << e) - 1u;
            if (empty & (1u << e)) {
              rank = __popc(empty & below) * MT + b % MT;
            } else {
              has = 1;
              rank = n_free + __popc(~empty & below) * MT + b % MT;
            }
          } else {
            rank = n_empty * MT + (b - E * MT);
          }
        }
        t.has_primary = has;
        t.rank = rank;
        t.stride = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    t.n_secondary = t.prefix[n_seg] +
                    ((g.shared_rows + BN - 1) / BN) * (g.m_tiles_shared / Cfg::kMPerUnit);
    griddep_launch();
  }
  __syncthreads();

  const uint32_t tmem = t.tmem_base;
  volatile int* abort_flag = &t.abort;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_phase = 0;  // per-stage bits
      bool ok = true;
      Unit un;
      int seg = 0;
      for (int k = 0; ok && cta_unit<BN, PAIR>(k, g, t, un, crank, seg); ++k) {
        const CUtensorMap* mw = un.routed ? &tm_w_routed : &tm_w_shared;
        const CUtensorMap* mx = un.routed ? &tm_x_routed : &tm_x_shared;
        // this CTA's token rows of the tile: all of them, or on a pair its
        // half of the MMA's N (a multiple of 16) starting at rank * N / 2
        const int n_mma = max(16, (un.valid + 15) & ~15);
        const int rows_b = PAIR ? n_mma / 2 : un.valid;
        const int b0 = PAIR ? crank * (n_mma / 2) : 0;
        const int subs = max(1, (rows_b + kSubRows - 1) / kSubRows);
        const uint32_t bytes = kTileA + subs * kSubBytes;
        for (int kb = 0; kb < un.k_blocks; ++kb) {
          if (!mbar_wait_fast(&t.empty[stage], phase ^ 1, abort_flag, g.status, 10)) {
            ok = false;
            break;
          }
          if constexpr (PAIR) {
            // both CTAs' bytes land on the leader's barrier, which the leader arms
            if (crank == 0) mbar_arrive_expect_tx(&t.full[stage], 2 * bytes);
            const uint32_t bar0 = mapa_shared(&t.full[stage], 0);
            tma_load_2d_pair(tiles_a + stage * kTileA, mw, 0, un.w_row + kb * BM, bar0);
            for (int sb = 0; sb < subs; ++sb)
              tma_load_2d_pair(tiles_b + stage * kTileB + sb * kSubBytes, mx, kb * BK,
                               un.x_row + b0 + sb * kSubRows, bar0);
          } else {
            mbar_arrive_expect_tx(&t.full[stage], bytes);
            tma_load_2d(tiles_a + stage * kTileA, mw, 0, un.w_row + kb * BM, &t.full[stage]);
            for (int sb = 0; sb < subs; ++sb)
              tma_load_2d(tiles_b + stage * kTileB + sb * kSubBytes, mx, kb * BK,
                          un.x_row + sb * kSubRows, &t.full[stage]);
          }
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // every issued copy has landed before the CTA can exit (on a pair the
      // leader's barriers count both CTAs' copies; the closing cluster
      // barrier keeps the peer alive until then)
      if (!PAIR || crank == 0)
        for (int s = 0; s < kStages; ++s)
          if (issued & (1u << s)) mbar_drain(&t.full[s], (issued_phase >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // (on a CTA pair only the leader issues: M = 256 over both CTAs' tiles,
    // completions multicast to the same barriers in both CTAs)
    if (lane == 0 && (!PAIR || crank == 0)) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      Unit un;
      int seg = 0;
      for (int k = 0; ok && cta_unit<BN, PAIR>(k, g, t, un, crank, seg); ++k) {
        if (!mbar_wait(&t.tempty[acc], acc_phase ^ 1, abort_flag, g.status, 20)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        const int n = max(16, (un.valid + 15) & ~15);  // an empty expert still drains its slabs
        const uint32_t idesc = make_idesc(PAIR ? 2 * BM : BM, n);
        static_assert(BK == 64, "one slab = four K = 16 MMAs");
        for (int kb = 0; kb < un.k_blocks; ++kb) {
          if (!mbar_wait_fast(&t.full[stage], phase, abort_flag, g.status, 21)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (PAIR) {
            mma_slab_pair(d_tmem, sw128_desc(tiles_a + stage * kTileA),
                          sw128_desc(tiles_b + stage * kTileB), idesc, kb != 0);
            mma_commit_pair_mc(&t.empty[stage], 3);
          } else {
            mma_slab(d_tmem, sw128_desc(tiles_a + stage * kTileA),
                     sw128_desc(tiles_b + stage * kTileB), idesc, kb != 0);
            mma_commit(&t.empty[stage]);
          }
          stage = stage + 1 == kStages ? 0 : stage + 1;
          phase ^= stage == 0 ? 1u : 0u;
        }
        if (!ok) break;
        if constexpr (PAIR)
          mma_commit_pair_mc(&t.tfull[acc], 3);
        else
          mma_commit(&t.tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // all MMAs issued by this thread have finished before TMEM is freed
      if constexpr (PAIR)
        mma_commit_pair(&t.drain);
      else
        mma_commit(&t.drain);
      mbar_drain(&t.drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // slot mode: this CTA has copied the counters (the barrier above); the
    // last CTA to get here zeroes them for the next block (the kernels after
    // this one start once it has completed).  Taken by an epilogue warp,
    // idle until its first accumulator, so the round trip delays no load.
    if (g.slot_ticket != nullptr && warp == 2 && lane == 0 &&
        atomicAdd(g.slot_ticket, 1) == (int)gridDim.x - 1) {
      for (int e = 0; e < g.n_experts; ++e) g.slot_counts[e] = 0;
      *g.slot_ticket = 0;
    }
    if (g.st.stats != nullptr && blockIdx.x == gridDim.x - 1)
      slot_stats(g, t, reinterpret_cast<float*>(epi_tiles), threadIdx.x - 64);
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;       // which alternate chunks it takes
    const int et = threadIdx.x - 64;        // 0..255
    const uint32_t tile_s = smem_u32(epi_tiles + (warp - 2) * kEpiTile);
    const unsigned char* tile_p = epi_tiles + (warp - 2) * kEpiTile;
    const int tq = lane & 3;                // this thread's token pair within 8 columns
    int acc = 0;
    uint32_t acc_phase = 0;
    Unit un;
    int seg = 0;
    for (int k = 0; cta_unit<BN, PAIR>(k, g, t, un, crank, seg); ++k) {
      const bool scatter = g.mode == kGemmPlain && un.routed && g.row_dst != nullptr;
      if (scatter) {
        // per-row destination and weight, fetched while the MMAs run
        epi_bar();  // the previous unit's stores are done with these arrays
        for (int i = et; i < un.valid; i += 32 * kEpiWarps) {
          t.unit_dst[i] = __ldg(g.row_dst + un.x_row + i);
          t.unit_wb[i] = __bfloat16_as_ushort(__float2bfloat16_rn(__ldg(g.row_w + un.x_row + i)));
        }
        epi_bar();
      }
      if (!mbar_wait(&t.tfull[acc], acc_phase, abort_flag, g.status, 30)) break;
      tc_fence_after();
      const int chunks = (un.valid + kChunk - 1) / kChunk;
      const uint32_t taddr = tmem + acc * BN + ((uint32_t)(q * 32) << 16);
      // one chunk: 32 token columns of this warp's 32 weight rows, as two
      // 16-lane fragments (registers 0-15: rows +0..15, 16-31: rows +16..31)
      auto load_chunk = [&](int c, uint32_t (&r)[32]) {
        tmem_ld_frag16_async<0>(taddr + c * kChunk, r);
        tmem_ld_frag16_async<16>(taddr + (16u << 16) + c * kChunk, r);
      };
      auto store_chunk = [&](const uint32_t (&r)[32], int c) {
        const int rows_here = min(kChunk, un.valid - c * kChunk);
        if (g.mode == kGemmSwiGLU) {
          // fragment (h, i): gate / up of feature 16q + 8h + lane / 4 for
          // tokens 8i + 2 tq, + 1  ->  hp[4h + i] = h of those two tokens
          uint32_t hp[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t gb = pack_bf16x2(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]));
            const uint32_t ub = pack_bf16x2(__uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            SiluFast s0 = silu_bf16_fast((uint16_t)(gb & 0xFFFFu));
            SiluFast s1 = silu_bf16_fast((uint16_t)(gb >> 16));
            if (!s0.exact) s0.bits = __bfloat16_as_ushort(silu_lut[gb & 0xFFFFu]);
            if (!s1.exact) s1.bits = __bfloat16_as_ushort(silu_lut[gb >> 16]);
            // bf16(silu * up): both factors are bf16, their product is exact
            // in fp32, so one bf16x2 multiply rounds it the same way
            hp[j] = mul_bf16x2((uint32_t)s0.bits | ((uint32_t)s1.bits << 16), ub);
          }
          // tile: 32 tokens x 16 features (32-byte rows, the 16-byte half
          // swizzled by bit 2 of the token so the 8 rows of a matrix hit
          // distinct banks); thread = token of the row it addresses
#pragma unroll
          for (int h = 0; h < 2; ++h)
            stmatrix_x4_trans(tile_s + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4), hp[4 * h],
                              hp[4 * h + 1], hp[4 * h + 2], hp[4 * h + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int v = lane + 32 * i, tok = v >> 1, cc = v & 1;
            if (tok < rows_here)
              *reinterpret_cast<uint4*>(un.out + (size_t)(un.out_row + c * kChunk + tok) * un.ld +
                                        un.out_col + q * 16 + cc * 8) =
                  *reinterpret_cast<const uint4*>(tile_p + tok * 32 +
                                                  ((cc ^ ((tok >> 2) & 1)) << 4));
          }
        } else {
          // fragment (h, i), rows +0..7 (ab = 0) / +8..15 (ab = 1):
          // yp[(4h + i) * 2 + ab] = bf16 of feature 32q + 16h + 8ab + lane / 4,
          // tokens 8i + 2 tq, + 1
          uint32_t yp[16];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            yp[2 * j] = pack_bf16x2(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]));
            yp[2 * j + 1] =
                pack_bf16x2(__uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (scatter) {
              // routed contribution bf16(bf16(y) * bf16(w)) of each token: the
              // product of two bf16 values is exact in fp32, so one bf16x2
              // multiply (rounded once) equals the fp32 multiply then rounding
              const int tok = c * kChunk + 8 * (j & 3) + 2 * tq;
              const uint32_t w = *reinterpret_cast<const uint32_t*>(t.unit_wb + tok);
              yp[2 * j] = mul_bf16x2(yp[2 * j], w);
              yp[2 * j + 1] = mul_bf16x2(yp[2 * j + 1], w);
            }
          }
          // tile: 32 tokens x 32 features (64-byte rows, 16-byte quarters
          // swizzled by bits 1-2 of the token); quarter 2h + ab
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int ab = 0; ab < 2; ++ab)
              stmatrix_x4_trans(tile_s + lane * 64 + (((2 * h + ab) ^ ((lane >> 1) & 3)) << 4),
                                yp[8 * h + ab], yp[8 * h + 2 + ab], yp[8 * h + 4 + ab],
                                yp[8 * h + 6 + ab]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int v = lane + 32 * i, tok = v >> 2, cc = v & 3;
            if (tok < rows_here) {
              const size_t row = scatter ? (size_t)t.unit_dst[c * kChunk + tok]
                                         : (size_t)(un.out_row + c * kChunk + tok);
              *reinterpret_cast<uint4*>(un.out + row * un.ld + un.out_col + q * 32 + cc * 8) =
                  *reinterpret_cast<const uint4*>(tile_p + tok * 64 +
                                                  ((cc ^ ((tok >> 1) & 3)) << 4));
            }
          }
        }
        __syncwarp();  // the tile is read out before the next chunk overwrites it
      };
      // chunks half, half + 2, ...: the loads of the next one are in flight
      // while the current one is converted and stored
      uint32_t ra[32], rb[32];
      int c = half;
      if (c < chunks) {
        load_chunk(c, ra);
        tmem_wait_ld(ra);
      }
      while (c < chunks) {
        if (c + 2 < chunks) load_chunk(c + 2, rb);
        store_chunk(ra, c);
        c += 2;
        if (c >= chunks) break;
        tmem_wait_ld(rb);
        if (c + 2 < chunks) load_chunk(c + 2, ra);
        store_chunk(rb, c);
        c += 2;
        if (c >= chunks) break;
        tmem_wait_ld(ra);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && crank != 0)
          mbar_arrive_cluster(mapa_shared(&t.tempty[acc], 0));  // the leader's MMA waits on it
        else
          mbar_arrive(&t.tempty[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // rows stored into another GPU's memory are visible there before this
    // kernel completes, so the kernel after it may raise the return flags
    if (g.out_peer_segs > 0) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  // a pair finishes together: no remote arrival or copy is still on its way
  // into either CTA, and both have stopped reading TMEM before it is freed
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(kTmemCols));
  }
}

// Weight tiles are stored in the order the GEMM streams them: tile (m, rt, kb)
// is rows [rt*128, rt*128 + 128) x columns [kb*64, kb*64 + 64) of matrix m,
// 128 rows of 64 bf16 (16 KB) back to back, so every TMA box is one
// contiguous 16 KB block of HBM.
constexpr int kTileVecs = BM * BK / 8;   // 16-byte vectors per tile

// gate/up: packed row p of tile rt holds gate (p % 16 < 8) or up of feature
// rt*64 + (p / 16) * 8 + p % 8 (packed_gate_up_row), so an M tile carries 64
// features' gate and up rows and a 16-lane TMEM fragment pairs them.
__global__ void pack_gate_up_kernel(__nv_bfloat16* __restrict__ dst,
                                    const __nv_bfloat16* __restrict__ gate,
                                    const __nv_bfloat16* __restrict__ up, int n_mats, int hidden,
                                    int dim) {
  const int kb_count = dim / BK, rt_count = 2 * hidden / BM;
  const size_t total = (size_t)n_mats * rt_count * kb_count * kTileVecs;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t tile = i / kTileVecs;
    const int w = (int)(i % kTileVecs), r = w >> 3, cv = w & 7;
    const int kb = (int)(tile % kb_count);
    const int rt = (int)((tile / kb_count) % rt_count);
    const int m = (int)(tile / ((size_t)kb_count * rt_count));
    const int feat = rt * (BM / 2) + (r >> 4) * 8 + (r & 7);
    const __nv_bfloat16* src = (r & 8) ? up : gate;
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(
        src + ((size_t)m * hidden + feat) * dim + kb * BK)[cv];
  }
}

// plain [n_mats, rows, cols] -> tiles
__global__ void pack_tiles_kernel(__nv_bfloat16* __restrict__ dst,
                                  const __nv_bfloat16* __restrict__ src, int n_mats, int rows,
                                  int cols) {
  const int kb_count = cols / BK, rt_count = rows / BM;
  const size_t total = (size_t)n_mats * rt_count * kb_count * kTileVecs;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t tile = i / kTileVecs;
    const int w = (int)(i % kTileVecs), r = w >> 3, cv = w & 7;
    const int kb = (int)(tile % kb_count);
    const int rt = (int)((tile / kb_count) % rt_count);
    const int m = (int)(tile / ((size_t)kb_count * rt_count));
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(
        src + ((size_t)m * rows + rt * BM + r) * cols + kb * BK)[cv];
  }
}

}  // namespace

// The SiLU table of the current device, built once on the caller's stream
// ahead of its first use (which is why that first call should not be captured).
static int ensure_silu_lut(cudaStream_t stream) {
  static unsigned long long lut_built = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(lut_built & (1ull << dev))) {
    build_silu_lut_kernel<<<(1 << 16) / 256, 256, 0, stream>>>();
    if (cudaGetLastError() != cudaSuccess) return -2;
    lut_built |= 1ull << dev;
  }
  return 0;
}

template <int BN, bool PAIR>
static int launch_gemm_bn(const GemmArgs& args, const CUtensorMap* tm_w_routed,
                          const CUtensorMap* tm_x_routed, const CUtensorMap* tm_w_shared,
                          const CUtensorMap* tm_x_shared, int grid, cudaStream_t stream) {
  constexpr size_t smem = smem_bytes<BN, PAIR>();
  static_assert(smem <= 227 * 1024, "grouped GEMM shared memory");
  // the attribute belongs to each device's context: set it once per device
  static unsigned long long configured = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(grouped_gemm_kernel<BN, PAIR>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // CTA pairs (1 x 1 x 1 otherwise)
  attr[1].val.clusterDim.x = PAIR ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<BN, PAIR>, *tm_w_routed, *tm_x_routed,
                            *tm_w_shared, *tm_x_shared, args) == cudaSuccess
             ? 0
             : -2;
}

int launch_grouped_gemm(const GemmArgs& args, const CUtensorMap* tm_w_routed,
                        const CUtensorMap* tm_x_routed, const CUtensorMap* tm_w_shared,
                        const CUtensorMap* tm_x_shared, int grid, int token_tile,
                        cudaStream_t stream) {
  if (ensure_silu_lut(stream) != 0) return -2;
  if (token_tile == 256) {
    // large batches: the gate/up GEMM (whose K loop, not its epilogue, bounds
    // it) on CTA pairs: M = 256 weight rows per MMA, each SM loading half the
    // token tile, a third fewer bytes per FLOP (measured at T = 16384: 59
    // instead of 63 us).  The down GEMM is bound by its epilogue, which runs
    // slower beside pair MMAs (51 instead of 45 us), so it stays on single CTAs.
    if (args.mode == kGemmSwiGLU && args.m_tiles_routed % 2 == 0 &&
        args.m_tiles_shared % 2 == 0 && grid >= 2)
      return launch_gemm_bn<256, true>(args, tm_w_routed, tm_x_routed, tm_w_shared, tm_x_shared,
                                       grid & ~1, stream);
    return launch_gemm_bn<256, false>(args, tm_w_routed, tm_x_routed, tm_w_shared, tm_x_shared,
                                      grid, stream);
  }
  if (token_tile == 128)
    return launch_gemm_bn<128, false>(args, tm_w_routed, tm_x_routed, tm_w_shared, tm_x_shared,
                                      grid, stream);
  return -1;
}

int launch_silu_bf16(const uint16_t* x, uint16_t* y, int n, cudaStream_t stream) {
  if (ensure_silu_lut(stream) != 0) return -2;
  if (n > 0) silu_bf16_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, y, n);
  return 0;  // the caller reads the launch status
}

static int pack_blocks(size_t vecs) {
  const size_t b = (vecs + 255) / 256;
  return (int)(b < 4096 ? b : 4096);
}

int launch_pack_gate_up(__nv_bfloat16* dst, const __nv_bfloat16* gate, const __nv_bfloat16* up,
                        int n_mats, int hidden, int dim, cudaStream_t stream) {
  const size_t vecs = (size_t)n_mats * 2 * hidden * (dim / 8);
  pack_gate_up_kernel<<<pack_blocks(vecs), 256, 0, stream>>>(dst, gate, up, n_mats, hidden, dim);
  return 0;
}

int launch_pack_tiles(__nv_bfloat16* dst, const __nv_bfloat16* src, int n_mats, int rows,
                      int cols, cudaStream_t stream) {
  const size_t vecs = (size_t)n_mats * rows * (cols / 8);
  pack_tiles_kernel<<<pack_blocks(vecs), 256, 0, stream>>>(dst, src, n_mats, rows, cols);
  return 0;
}

}  // namespace parrot
