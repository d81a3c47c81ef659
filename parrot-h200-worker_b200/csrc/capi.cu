// extern "C" entry points of libparrot_b200.so (declared in include/parrot_b200.h).
//
// This layer validates arguments, carves the caller's workspace, builds the
// TMA tensor maps (host-side encode, cached per buffer) and enqueues the
// kernels on the caller's stream.  It never allocates device memory and
// never synchronises (except parrot_moe_read_status, a debugging read).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "kernels.h"
#include "parrot_b200.h"

using parrot::kGemmBlockK;
using parrot::kGemmSubRows;

namespace {

thread_local std::string g_last_error;
std::atomic<unsigned long long> g_launches{0};

int fail(int code, const char* fmt, const char* detail = "") {
  char buf[512];
  std::snprintf(buf, sizeof(buf), fmt, detail);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(err);
    return PARROT_ECUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return PARROT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- TMA tensor maps ------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  long long rows, cols;
  int box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (size_t)(k.rows * 1315423911ll) ^
           (size_t)(k.cols * 2654435761ll) ^ (size_t)k.box_rows;
  }
};

std::mutex g_map_mutex;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// Row-major bf16 [rows, cols] matrix, box = 64 columns x box_rows rows, 128-B swizzle.
bool tensor_map(CUtensorMap* out, const void* ptr, long long rows, long long cols, int box_rows) {
  const MapKey key{ptr, rows, cols, box_rows};
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmBlockK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(g_map_mutex);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, map);
  *out = map;
  return true;
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  return n;
}

// ---- MoE workspace ----------------------------------------------------------
int validate_dims(const parrot_moe_dims* d) {
  if (d == nullptr) return fail(PARROT_EINVAL, "dims is NULL%s");
  if (d->tokens < 0) return fail(PARROT_EINVAL, "tokens must be >= 0%s");
  if (d->top_k != 2) return fail(PARROT_EINVAL, "top_k must be 2%s");
  if (d->n_experts < 2 || d->n_experts > parrot::kMaxExperts)
    return fail(PARROT_EINVAL, "n_experts must be in [2, 32]%s");
  if (d->dim <= 0 || d->dim % 128 || d->dim > 1024)
    return fail(PARROT_EINVAL, "dim must be a positive multiple of 128, <= 1024%s");
  if (d->expert_dim <= 0 || d->expert_dim % 64)
    return fail(PARROT_EINVAL, "expert_dim must be a positive multiple of 64%s");
  if (d->shared_dim <= 0 || d->shared_dim % 64)
    return fail(PARROT_EINVAL, "shared_dim must be a positive multiple of 64%s");
  if (d->capacity < -2) return fail(PARROT_EINVAL, "capacity must be >= -2%s");
  return PARROT_OK;
}

int layout_of(const parrot_moe_dims* d, parrot_moe_layout* L) {
  const int rc = validate_dims(d);
  if (rc) return rc;
  std::memset(L, 0, sizeof(*L));
  const size_t T = d->tokens, D = d->dim, E = d->n_experts, H = d->expert_dim,
               Hs = d->shared_dim;
  // capacity 0 selects the default; -1 packs every row per expert (no capacity
  // region); -2 (slot mode) gives every expert a region of 2T rows
  const int C = d->capacity > 0     ? d->capacity
                : d->capacity == 0  ? parrot_moe_capacity(d->tokens, d->n_experts)
                : d->capacity == -1 ? 0
                                    : 2 * d->tokens;
  const size_t A = 2 * T;
  const size_t n_tiles = (size_t)parrot::route_blocks(d->tokens);
  const size_t n_chunks = (size_t)parrot::group_blocks(d->tokens);
  const size_t R = E * (size_t)C + A;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  // the status word first, then the slot-mode counters [E] and ticket: the
  // region parrot_moe_workspace_init zeroes
  L->status = take(16 + 4 * (E + 1));
  L->indices = take(A * 4);
  L->weights = take(A * 4);
  L->positions = take(A * 4);
  L->chunk_hist = take(n_chunks * E * 4);
  L->tile_hist = take(n_tiles * E * 4);
  L->tile_probsum = take(n_tiles * E * 4);
  L->counts = take(E * 4);
  L->seg_rows = take(2 * E * 4);
  L->seg_base = take(2 * E * 4);
  L->stats = take((E + 1) * 4);
  L->row_dst = take(R * 4);
  L->row_w = take(R * 4);
  L->grouped = take(R * D * 2);
  L->hidden = take(R * H * 2);
  L->contrib = take(A * D * 2);
  L->shared_hidden = take(T * Hs * 2);
  L->shared_y = take(T * D * 2);
  L->total = off;
  L->capacity = C;
  L->grouped_rows = (int)R;
  L->route_blocks = (int)n_tiles;
  return PARROT_OK;
}

template <typename T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

int check_weights(const parrot_moe_weights* w) {
  if (w == nullptr || w->router == nullptr || w->gate_up == nullptr || w->down == nullptr ||
      w->shared_gate_up == nullptr || w->shared_down == nullptr)
    return fail(PARROT_EINVAL, "missing weight pointer%s");
  if (!aligned16(w->router) || !aligned16(w->gate_up) || !aligned16(w->down) ||
      !aligned16(w->shared_gate_up) || !aligned16(w->shared_down))
    return fail(PARROT_EINVAL, "weights must be 16-byte aligned%s");
  return PARROT_OK;
}

parrot::MoeTables tables(void* ws, const parrot_moe_layout& L) {
  parrot::MoeTables t;
  t.chunk_hist = at<int>(ws, L.chunk_hist);
  t.tile_hist = at<int>(ws, L.tile_hist);
  t.tile_probsum = at<float>(ws, L.tile_probsum);
  t.counts = at<int>(ws, L.counts);
  t.seg_rows = at<int>(ws, L.seg_rows);
  t.seg_base = at<int>(ws, L.seg_base);
  t.stats = at<float>(ws, L.stats);
  return t;
}

int prepare(const parrot_moe_dims* dims, const parrot_moe_weights* w, const void* x,
            const parrot_moe_outputs* o, void* ws, size_t ws_bytes, parrot_moe_layout* L,
            bool need_out = true) {
  int rc = layout_of(dims, L);
  if (rc) return rc;
  if ((rc = check_weights(w))) return rc;
  if (o == nullptr || (need_out && dims->tokens > 0 && o->out == nullptr))
    return fail(PARROT_EINVAL, "outputs->out is required%s");
  if (ws == nullptr || ws_bytes < L->total || !aligned16(ws))
    return fail(PARROT_EINVAL, "workspace missing, misaligned or smaller than the layout total%s");
  if (dims->tokens > 0 && (x == nullptr || !aligned16(x) || (need_out && !aligned16(o->out)) ||
                           (o->residual && !aligned16(o->residual))))
    return fail(PARROT_EINVAL, "x/out/residual must be non-null and 16-byte aligned%s");
  return PARROT_OK;
}

// The router's arguments: its outputs in the workspace (and the caller's
// optional copies).
parrot::RouteArgs route_args(const parrot_moe_dims* dims, const parrot_moe_weights* w,
                             const parrot_moe_outputs* o, void* ws, const parrot_moe_layout& L) {
  parrot::RouteArgs ra{};
  ra.bias = w->router_bias;
  ra.probs = o->probs;
  ra.indices = at<int>(ws, L.indices);
  ra.weights = at<float>(ws, L.weights);
  ra.indices64 = o->indices;
  ra.weights_out = o->weights;
  ra.tab = tables(ws, L);
  ra.tokens = dims->tokens;
  ra.dim = dims->dim;
  ra.n_experts = dims->n_experts;
  ra.status = at<int>(ws, L.status);
  return ra;
}

// Grouping (capacity slots, overflow, the 16-byte row scatter) after the
// router's outputs are in the workspace.  ep_order (expert parallelism): the
// packing order of the experts' rows, destination rank major; nullptr:
// expert id order.
// x_from_upstream: x was written by the kernel just before this one on the
// stream (the depth mix with the router folded in), so the grouping may only
// read it after its dependency wait.
// Expert parallelism: the dispatched rows go straight into each destination's
// receive region for this source (peer memory) instead of the workspace.
struct EpRowsTo {
  __nv_bfloat16* recv[parrot::kEpMaxRanks];
  signed char dest[parrot::kMaxExperts];  // destination rank of each expert
  int region;                             // rows of one receive region
};

int run_group(const parrot_moe_dims* dims, const void* x, const parrot_moe_outputs* o, void* ws,
              const parrot_moe_layout& L, cudaStream_t s, const signed char* ep_order = nullptr,
              bool x_from_upstream = false, const EpRowsTo* to = nullptr) {
  const int T = dims->tokens, E = dims->n_experts;
  parrot::GroupArgs ga{};
  ga.x = static_cast<const __nv_bfloat16*>(x);
  ga.indices = at<int>(ws, L.indices);
  ga.tab = tables(ws, L);
  ga.weights = at<float>(ws, L.weights);
  ga.positions = at<int>(ws, L.positions);
  ga.positions_out = o->positions;
  ga.row_dst = at<int>(ws, L.row_dst);
  ga.row_w = at<float>(ws, L.row_w);
  ga.grouped = at<__nv_bfloat16>(ws, L.grouped);
  ga.counts_out = o->counts;
  ga.stats_out = o->stats;
  ga.tokens = T;
  ga.dim = dims->dim;
  ga.n_experts = E;
  ga.capacity = L.capacity;
  ga.ep_packed = ep_order != nullptr;
  if (ep_order != nullptr)
    for (int q = 0; q < E; ++q) ga.ep_order[q] = ep_order[q];
  if (to != nullptr) {
    for (int q = 0; q < parrot::kEpMaxRanks; ++q) ga.ep_recv[q] = to->recv[q];
    for (int e = 0; e < parrot::kMaxExperts; ++e) ga.ep_dest[e] = to->dest[e];
    ga.ep_region = to->region;
  }
  const int ng = parrot::group_blocks(T);
  const int want = (2 * sm_count() + ng - 1) / ng;  // about two blocks per SM
  int split = 1;
  while (split * 2 <= want && split < 8) split *= 2;
  ga.copy_split = split;
  ga.status = at<int>(ws, L.status);
  ga.x_from_upstream = x_from_upstream ? 1 : 0;
  if (parrot::launch_group(ga, s)) return fail(PARROT_ECUDA, "group: shared-memory setup failed%s");
  return check_launch("group_kernel");
}

// Slot mode (dims->capacity == -2): the router (kernel, or folded into the
// depth mix) does the grouping too (an atomic slot per assignment in a 2T-row
// region of its expert, the rows written straight to their grouped rows), and
// the block's GEMMs read the per-expert counters as their segments; the down
// GEMM leaves them zero.
bool slot_mode(const parrot_moe_dims* d, const parrot_moe_layout& L) {
  return d->capacity == -2 && L.capacity == 2 * d->tokens;
}
int* slot_counters(void* ws, const parrot_moe_layout& L) {
  return reinterpret_cast<int*>(static_cast<char*>(ws) + L.status + 16);  // [E], then the ticket
}

void set_slots(parrot::RouteArgs* ra, void* ws, const parrot_moe_layout& L, const void* x) {
  ra->slot_counts = slot_counters(ws, L);
  ra->slot_x = static_cast<const __nv_bfloat16*>(x);
  ra->slot_stride = L.capacity;
  ra->grouped = at<__nv_bfloat16>(ws, L.grouped);
  ra->positions = at<int>(ws, L.positions);
  ra->row_dst = at<int>(ws, L.row_dst);
  ra->row_w = at<float>(ws, L.row_w);
}

// Router + grouping (slots: the router groups the rows itself, slot mode).
int run_route(const parrot_moe_dims* dims, const parrot_moe_weights* w, const void* x,
              const parrot_moe_outputs* o, void* ws, const parrot_moe_layout& L, cudaStream_t s,
              const signed char* ep_order = nullptr, bool slots = false,
              const EpRowsTo* to = nullptr) {
  const int T = dims->tokens, E = dims->n_experts;
  parrot::RouteArgs ra = route_args(dims, w, o, ws, L);
  if (slots) set_slots(&ra, ws, L, x);
  CUtensorMap mx, mw;
  if (parrot::route_tile(T) != parrot::kRouteSmallTile &&
      (!tensor_map(&mx, x, T, dims->dim, parrot::route_tile(T)) ||
       !tensor_map(&mw, w->router, E, dims->dim, parrot::route_experts_padded(E))))
    return fail(PARROT_ECUDA, "route: cuTensorMapEncodeTiled failed%s");
  if (parrot::launch_route(ra, x, w->router, &mx, &mw, s))
    return fail(PARROT_ECUDA, "route: unsupported dim or shared-memory setup failed%s");
  int rc = check_launch("route_kernel");
  if (rc || slots) return rc;
  return run_group(dims, x, o, ws, L, s, ep_order, false, to);
}

int run_gemm(bool swiglu, const parrot_moe_dims* dims, const parrot_moe_weights* w,
             const void* x, void* ws, const parrot_moe_layout& L, cudaStream_t s,
             bool shared_only = false, const parrot_moe_outputs* slots = nullptr) {
  const int T = dims->tokens, D = dims->dim, E = dims->n_experts, H = dims->expert_dim,
            Hs = dims->shared_dim, R = L.grouped_rows;
  parrot::GemmArgs g{};
  g.seg_rows = at<int>(ws, L.seg_rows);
  g.seg_base = at<int>(ws, L.seg_base);
  g.seg_expert = nullptr;
  g.n_seg = shared_only ? 0 : 2 * E;
  if (slots != nullptr && !shared_only) {
    // slot mode: one segment per expert, its rows counted by the depth mix
    int* counters = slot_counters(ws, L);
    g.seg_rows = counters;
    g.seg_stride = L.capacity;
    g.n_seg = E;
    if (!swiglu) {  // the last reader zeroes them; CTA grid - 1 writes the statistics
      g.slot_counts = counters;
      g.slot_ticket = counters + E;
      const parrot::MoeTables tab = tables(ws, L);
      g.st.tile_probsum = tab.tile_probsum;
      g.st.route_tiles = parrot::route_blocks(T);
      g.st.tokens = T;
      g.st.counts = tab.counts;
      g.st.counts_out = slots->counts;
      g.st.stats = tab.stats;
      g.st.stats_out = slots->stats;
      g.st.positions = at<int>(ws, L.positions);
      g.st.positions_out = slots->positions;
    }
  }
  g.static_routed = shared_only ? 0 : 1;
  g.n_experts = E;
  g.shared_rows = T;
  g.status = at<int>(ws, L.status);
  CUtensorMap mw, mx, msw, msx;
  bool ok;
  if (swiglu) {
    g.m_tiles_routed = 2 * H / 128;
    g.k_blocks_routed = D / kGemmBlockK;
    g.out_routed = at<__nv_bfloat16>(ws, L.hidden);
    g.ld_out_routed = H;
    g.m_tiles_shared = 2 * Hs / 128;
    g.k_blocks_shared = D / kGemmBlockK;
    g.out_shared = at<__nv_bfloat16>(ws, L.shared_hidden);
    g.ld_out_shared = Hs;
    g.mode = parrot::kGemmSwiGLU;
    g.w_routed = shared_only ? nullptr : w->gate_up;
    // weights are tiled (parrot_pack_*): a [tiles * 128, 64] view, one box per tile
    ok = tensor_map(&msw, w->shared_gate_up, 2LL * Hs * D / kGemmBlockK, kGemmBlockK, 128) &&
         tensor_map(&msx, x, T, D, kGemmSubRows);
    if (shared_only) {  // no routed units: the routed maps are never read
      mw = msw;
      mx = msx;
    } else {
      ok = ok &&
           tensor_map(&mw, w->gate_up, (long long)E * 2 * H * D / kGemmBlockK, kGemmBlockK, 128) &&
           tensor_map(&mx, at<void>(ws, L.grouped), R, D, kGemmSubRows);
    }
  } else {
    g.m_tiles_routed = D / 128;
    g.k_blocks_routed = H / kGemmBlockK;
    g.out_routed = at<__nv_bfloat16>(ws, L.contrib);
    g.ld_out_routed = D;
    g.row_dst = at<int>(ws, L.row_dst);
    g.row_w = at<float>(ws, L.row_w);
    g.m_tiles_shared = D / 128;
    g.k_blocks_shared = Hs / kGemmBlockK;
    g.out_shared = at<__nv_bfloat16>(ws, L.shared_y);
    g.ld_out_shared = D;
    g.mode = parrot::kGemmPlain;
    g.w_routed = shared_only ? nullptr : w->down;
    ok = tensor_map(&msw, w->shared_down, (long long)D * Hs / kGemmBlockK, kGemmBlockK, 128) &&
         tensor_map(&msx, at<void>(ws, L.shared_hidden), T, Hs, kGemmSubRows);
    if (shared_only) {
      mw = msw;
      mx = msx;
    } else {
      ok = ok &&
           tensor_map(&mw, w->down, (long long)E * D * H / kGemmBlockK, kGemmBlockK, 128) &&
           tensor_map(&mx, at<void>(ws, L.hidden), R, H, kGemmSubRows);
    }
  }
  if (!ok) return fail(PARROT_ECUDA, "cuTensorMapEncodeTiled failed%s");
  const int A = 2 * T;
  const int bn = parrot::gemm_token_tile(A);
  const long long routed_units =
      shared_only ? 0 : (long long)((A + bn - 1) / bn + 2 * E) * g.m_tiles_routed;
  const long long shared_units = (long long)((T + bn - 1) / bn) * g.m_tiles_shared;
  long long grid = routed_units + shared_units;
  const int sms = sm_count();
  if (grid > sms) grid = sms;
  if (grid < 1) grid = 1;
  if (parrot::launch_grouped_gemm(g, &mw, &mx, &msw, &msx, (int)grid, bn, s))
    return fail(PARROT_ECUDA, "grouped GEMM: could not set shared-memory size%s");
  return check_launch(swiglu ? "grouped_gemm(gate_up)" : "grouped_gemm(down)");
}

int run_experts(const parrot_moe_dims* dims, const parrot_moe_weights* w, const void* x,
                const parrot_moe_outputs* o, void* ws, const parrot_moe_layout& L,
                cudaStream_t s, bool combine = true, bool slots = false) {
  int rc = run_gemm(true, dims, w, x, ws, L, s, false, slots ? o : nullptr);
  if (rc) return rc;
  if ((rc = run_gemm(false, dims, w, x, ws, L, s, false, slots ? o : nullptr))) return rc;
  if (!combine) return PARROT_OK;
  parrot::CombineArgs c{};
  c.contrib = at<__nv_bfloat16>(ws, L.contrib);
  c.shared_y = at<__nv_bfloat16>(ws, L.shared_y);
  c.residual = static_cast<const __nv_bfloat16*>(o->residual);
  c.out = static_cast<__nv_bfloat16*>(o->out);
  c.tokens = dims->tokens;
  c.dim = dims->dim;
  if (parrot::launch_combine(c, s)) return fail(PARROT_EINVAL, "combine: unsupported dim%s");
  return check_launch("combine_kernel");
}

// ---- expert-parallel pieces -------------------------------------------------
int check_router(const parrot_moe_weights* w) {
  if (w == nullptr || w->router == nullptr || !aligned16(w->router))
    return fail(PARROT_EINVAL, "router weight missing or not 16-byte aligned%s");
  return PARROT_OK;
}

int check_shared(const parrot_moe_weights* w) {
  if (w == nullptr || w->shared_gate_up == nullptr || w->shared_down == nullptr ||
      !aligned16(w->shared_gate_up) || !aligned16(w->shared_down))
    return fail(PARROT_EINVAL, "shared expert weights missing or not 16-byte aligned%s");
  return PARROT_OK;
}

int ws_ok(const void* ws, size_t ws_bytes, const parrot_moe_layout& L) {
  if (ws == nullptr || ws_bytes < L.total || !aligned16(ws))
    return fail(PARROT_EINVAL, "workspace missing, misaligned or smaller than the layout total%s");
  return PARROT_OK;
}

// Grouped SwiGLU FFN over caller-described row segments: hidden = SwiGLU
// halves of x @ gate_up, y = hidden @ down, rows in the order of x.
// Expert parallelism: the down GEMM stores source q's rows straight into q's
// return region (peer memory), at the row base q sent, instead of into y.
struct EpRowsBack {
  __nv_bfloat16* back[parrot::kEpMaxRanks];  // each source's return region
  const int* base;                           // [ranks] device table: each source's row base
  int segs_per_source;                       // segment s belongs to source s / segs_per_source
  int region;                                // rows of one receive region
};

int run_ffn(int rows, int dim, int expert_dim, int n_mats, int n_seg, const int* seg_rows,
            const int* seg_base, const int* seg_expert, const void* gate_up, const void* down,
            const void* x, void* hidden, void* y, int* status, cudaStream_t s,
            const EpRowsBack* back = nullptr) {
  CUtensorMap mw, mx;
  const int sms = sm_count();
  for (int stage = 0; stage < 2; ++stage) {
    const bool swiglu = stage == 0;
    parrot::GemmArgs g{};
    g.seg_rows = seg_rows;
    g.seg_base = seg_base;
    g.seg_expert = seg_expert;
    g.n_seg = n_seg;
    g.static_routed = 0;
    g.n_experts = n_mats;
    g.shared_rows = 0;
    g.status = status;
    bool ok;
    if (swiglu) {
      g.m_tiles_routed = 2 * expert_dim / 128;
      g.k_blocks_routed = dim / kGemmBlockK;
      g.out_routed = static_cast<__nv_bfloat16*>(hidden);
      g.ld_out_routed = expert_dim;
      g.mode = parrot::kGemmSwiGLU;
      ok = tensor_map(&mw, gate_up, (long long)n_mats * 2 * expert_dim * dim / kGemmBlockK,
                      kGemmBlockK, 128) &&
           tensor_map(&mx, x, rows, dim, kGemmSubRows);
    } else {
      g.m_tiles_routed = dim / 128;
      g.k_blocks_routed = expert_dim / kGemmBlockK;
      g.out_routed = static_cast<__nv_bfloat16*>(y);
      g.ld_out_routed = dim;
      g.mode = parrot::kGemmPlain;
      if (back != nullptr) {
        g.out_peer_segs = back->segs_per_source;
        g.out_peer_region = back->region;
        g.out_peer_base = back->base;
        for (int q = 0; q < parrot::kEpMaxRanks; ++q) g.out_peer[q] = back->back[q];
      }
      ok = tensor_map(&mw, down, (long long)n_mats * dim * expert_dim / kGemmBlockK, kGemmBlockK,
                      128) &&
           tensor_map(&mx, hidden, rows, expert_dim, kGemmSubRows);
    }
    if (!ok) return fail(PARROT_ECUDA, "cuTensorMapEncodeTiled failed%s");
    // the shared maps are never read (shared_rows == 0)
    const int bn = parrot::gemm_token_tile(rows);
    long long grid = (long long)((rows + bn - 1) / bn + n_seg) * g.m_tiles_routed;
    if (grid > sms) grid = sms;
    if (grid < 1) grid = 1;
    if (parrot::launch_grouped_gemm(g, &mw, &mx, &mw, &mx, (int)grid, bn, s))
      return fail(PARROT_ECUDA, "grouped GEMM: could not set shared-memory size%s");
    const int rc = check_launch(swiglu ? "grouped_gemm(ffn gate_up)" : "grouped_gemm(ffn down)");
    if (rc) return rc;
  }
  return PARROT_OK;
}

// ---- expert-parallel exchange over peer memory -----------------------------
int ep_layout_of(const parrot_ep_dims* e, parrot_ep_layout* L) {
  if (e == nullptr || L == nullptr) return fail(PARROT_EINVAL, "ep: null dims or layout%s");
  if (e->ranks < 1 || e->ranks > parrot::kEpMaxRanks || e->rank < 0 || e->rank >= e->ranks)
    return fail(PARROT_EINVAL, "ep: 1 <= ranks <= 8 and 0 <= rank < ranks required%s");
  if (e->n_experts < 2 || e->n_experts > parrot::kMaxExperts)
    return fail(PARROT_EINVAL, "ep: 2 <= n_experts <= 32 required%s");
  if (e->slots == 0 && e->n_experts % e->ranks)
    return fail(PARROT_EINVAL, "ep: round-robin placement needs ranks dividing n_experts%s");
  if (e->slots < 0 || e->slots > parrot::kMaxExperts || e->ranks * e->slots > 2 * parrot::kMaxExperts)
    return fail(PARROT_EINVAL, "ep: 0 <= slots <= 32 and ranks * slots <= 64 required%s");
  if (e->dim <= 0 || e->dim % 128 || e->dim > 1024 || e->expert_dim <= 0 || e->expert_dim % 64)
    return fail(PARROT_EINVAL, "ep: dim % 128 == 0 (<= 1024), expert_dim % 64 == 0 required%s");
  if (e->max_tokens < 1 || (long long)e->ranks * 2 * e->max_tokens > (1ll << 30))
    return fail(PARROT_EINVAL, "ep: max_tokens out of range%s");
  std::memset(L, 0, sizeof(*L));
  const size_t G = e->ranks, R = 2 * (size_t)e->max_tokens, D = e->dim;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  L->flags_in = take(parrot::kEpMaxRanks * 4);
  L->flags_back = take(parrot::kEpMaxRanks * 4);
  L->meta = take(parrot::kEpMaxRanks * parrot::kEpMetaStride * 4);
  L->recv_rows = take(G * R * D * 2);
  L->back_rows = take(R * D * 2);
  L->epoch = take(4);
  L->counters = take(2 * 4);
  L->status = take(16);
  L->seg_rows = take(2 * parrot::kMaxExperts * 4);
  L->seg_base = take(2 * parrot::kMaxExperts * 4);
  L->seg_expert = take(2 * parrot::kMaxExperts * 4);
  L->back_n = take(parrot::kEpMaxRanks * 4);
  L->back_base = take(parrot::kEpMaxRanks * 4);
  L->hidden = take(G * R * e->expert_dim * 2);
  L->y = take(G * R * D * 2);
  L->total = off;
  L->region_rows = (int)R;
  return PARROT_OK;
}

int ep_slots(const parrot_ep_dims* e) { return e->slots ? e->slots : e->n_experts / e->ranks; }

// This rank's send plan (round-robin when e->slots == 0); every expert must
// appear exactly once.
int ep_plan(const parrot_ep_dims* e, signed char plan[parrot::kEpMaxRanks][parrot::kMaxExperts]) {
  const int G = e->ranks, E = e->n_experts;
  for (int q = 0; q < parrot::kEpMaxRanks; ++q)
    for (int j = 0; j < parrot::kMaxExperts; ++j) {
      int x = -1;
      if (q < G) {
        if (e->slots == 0) x = j < E / G ? q + j * G : -1;
        else x = e->plan[q][j];
      }
      plan[q][j] = (signed char)x;
    }
  int seen[parrot::kMaxExperts] = {};
  for (int q = 0; q < G; ++q)
    for (int j = 0; j < parrot::kMaxExperts; ++j) {
      const int x = plan[q][j];
      if (x < -1 || x >= E) return fail(PARROT_EINVAL, "ep: plan entry out of range%s");
      if (x >= 0) ++seen[x];
    }
  for (int x = 0; x < E; ++x)
    if (seen[x] != 1) return fail(PARROT_EINVAL, "ep: every expert must appear once in the plan%s");
  return PARROT_OK;
}

// The packing order of the dispatched rows: destination major, slot order.
void ep_order(const signed char plan[parrot::kEpMaxRanks][parrot::kMaxExperts], int G,
              signed char* order) {
  int n = 0;
  for (int q = 0; q < G; ++q)
    for (int j = 0; j < parrot::kMaxExperts; ++j)
      if (plan[q][j] >= 0) order[n++] = plan[q][j];
}

unsigned long long ep_wait_ns(const parrot_ep_dims* e) {
  return e->wait_ns ? e->wait_ns : 2000000000ull;  // 2 s, as the kernels' mbarrier waits
}

int ep_peers_ok(const parrot_ep_dims* e, const parrot_ep_peers* p) {
  if (p == nullptr) return fail(PARROT_EINVAL, "ep: peers is NULL%s");
  for (int r = 0; r < e->ranks; ++r)
    if (p->buffers[r] == nullptr || (reinterpret_cast<uintptr_t>(p->buffers[r]) & 255))
      return fail(PARROT_EINVAL, "ep: every rank's buffer must be mapped and 256-byte aligned%s");
  return PARROT_OK;
}

typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<MemGetAddressRangeFn>(p);
  });
  return fn;
}

// ---- allocation-free MoE entry point --------------------------------------
// Some callers cannot allocate device memory when they call the MoE block: a
// runtime that hands out all device memory up front and forbids allocation on
// its hot path, or code running where the allocator must not be entered.
// parrot_moe_forward_static_bf16 serves them from a fixed workspace compiled
// into this library instead of one the caller passes in.
constexpr size_t kStaticWorkspaceBytes = size_t(4) << 20;  // 4 MiB per device

// Device-side workspace.  In host code this name is only a stand-in for the
// symbol, never a device address: its address on a device comes from
// cudaGetSymbolAddress with that device current.
static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

// The array's device address belongs to the CUDA context that loaded this
// library's module on the device.  A context that is destroyed and created
// again (cudaDeviceReset, or a caller's own driver-API context) loads the
// module afresh and the array can move, so the looked-up address is cached
// per device together with the process-unique id of the context it was
// looked up in (cuCtxGetId), and looked up again when the current context's
// id differs.  Where the id cannot be read, it is looked up on every call.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct CtxFns {
  CtxGetCurrentFn current = nullptr;
  CtxGetIdFn id = nullptr;
};

const CtxFns& ctx_fns() {
  static CtxFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.id = reinterpret_cast<CtxGetIdFn>(p);
  });
  return fns;
}

// Id of the calling thread's current context; false when there is none.
bool current_context_id(unsigned long long* id) {
  const CtxFns& f = ctx_fns();
  if (f.current == nullptr || f.id == nullptr) return false;
  CUcontext c = nullptr;
  if (f.current(&c) != CUDA_SUCCESS || c == nullptr) return false;
  return f.id(c, id) == CUDA_SUCCESS;
}

struct StaticAddress {
  unsigned long long context_id;
  void* ptr;  // nullptr: not looked up in any live context yet
};
std::mutex g_static_mutex;
StaticAddress g_static_address[64] = {};

// Address of g_static_workspace on the current device, in the current context.
int static_workspace_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(PARROT_ECUDA, "static workspace: no current CUDA device%s");
  unsigned long long id = 0;
  const bool have_id = current_context_id(&id);
  std::lock_guard<std::mutex> lock(g_static_mutex);
  StaticAddress& slot = g_static_address[dev];
  if (have_id && slot.ptr != nullptr && slot.context_id == id) {
    *out = slot.ptr;
    return PARROT_OK;
  }
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_static_workspace);
  if (err != cudaSuccess || p == nullptr)
    return fail(PARROT_ECUDA, "static workspace: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(err));
  // the lookup makes the device's primary context current if none was
  unsigned long long now = 0;
  slot = current_context_id(&now) ? StaticAddress{now, p} : StaticAddress{0, nullptr};
  *out = p;
  return PARROT_OK;
}

}  // namespace

extern "C" {

int parrot_b200_version(void) { return 100; }

const char* parrot_b200_last_error(void) { return g_last_error.c_str(); }

int parrot_b200_device_supported(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
  return prop.major == 10 ? 1 : 0;
}

int parrot_rmsnorm_bf16(void* out, const void* x, const void* weight, int rows, int dim,
                        float eps, void* stream) {
  if (rows < 0 || dim <= 0 || dim % 8 || dim > 2048)
    return fail(PARROT_EINVAL, "rmsnorm: rows >= 0 and dim % 8 == 0, dim <= 2048 required%s");
  if (rows == 0) return PARROT_OK;
  if (!out || !x || !weight || !aligned16(out) || !aligned16(x) || !aligned16(weight))
    return fail(PARROT_EINVAL, "rmsnorm: pointers must be non-null and 16-byte aligned%s");
  parrot::launch_rmsnorm(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(x),
                         static_cast<const __nv_bfloat16*>(weight), rows, dim, eps,
                         static_cast<cudaStream_t>(stream));
  return check_launch("rmsnorm_kernel");
}

namespace {
// Shared by the two depth-mix entries: the last source is replaced by the
// deferred value (pending_out) when one is given.
// route (optional): the router folded in (the output is an MoE block's input)
int depthmix_launch(void* out, const void* const* sources, int n_sources, const void* query,
                    const void* key_norm_weight, float key_eps, const void* out_norm_weight,
                    float out_eps, void* mix_out, parrot::DepthMixArgs a, int rows, int dim,
                    void* stream, const parrot::DepthRouteArgs* route = nullptr) {
  if (n_sources < 1 || n_sources > parrot::kMaxDepthSources)
    return fail(PARROT_EINVAL, "depthmix: n_sources must be in [1, 16]%s");
  if (rows < 0 || dim <= 0 || dim % 8 || dim > 1024)
    return fail(PARROT_EINVAL, "depthmix: dim % 8 == 0 and dim <= 1024 required%s");
  if (rows == 0) return PARROT_OK;
  if (!out || !query || !key_norm_weight || !sources)
    return fail(PARROT_EINVAL, "depthmix: null pointer%s");
  const bool deferred = a.pending_out != nullptr;
  for (int i = 0; i < n_sources; ++i) {
    const void* p = deferred && i == n_sources - 1 ? a.pending_out : sources[i];
    if (p == nullptr || !aligned16(p))
      return fail(PARROT_EINVAL, "depthmix: sources must be non-null and 16-byte aligned%s");
    a.sources[i] = static_cast<const __nv_bfloat16*>(p);
  }
  a.n_sources = n_sources;
  a.query = static_cast<const __nv_bfloat16*>(query);
  a.key_w = static_cast<const __nv_bfloat16*>(key_norm_weight);
  a.key_eps = key_eps;
  a.out_w = static_cast<const __nv_bfloat16*>(out_norm_weight);
  a.out_eps = out_eps;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.mix_out = static_cast<__nv_bfloat16*>(mix_out);
  a.rows = rows;
  a.dim = dim;
  if (route != nullptr) {
    if (parrot::launch_depthmix_route(a, *route, static_cast<cudaStream_t>(stream)))
      return fail(PARROT_ECUDA, "depthmix (router): unsupported shape or shared-memory setup%s");
    return check_launch("depthmix_kernel (router)");
  }
  if (parrot::launch_depthmix(a, static_cast<cudaStream_t>(stream)))
    return fail(PARROT_ECUDA, "depthmix: could not configure shared memory%s");
  return check_launch("depthmix_kernel");
}
}  // namespace

int parrot_depthmix_bf16(void* out, const void* const* sources, int n_sources,
                         const void* query, const void* key_norm_weight, float key_eps,
                         const void* out_norm_weight, float out_eps, void* mix_out,
                         const void* pending_base, const void* pending_delta,
                         void* pending_out, int rows, int dim, void* stream) {
  if ((pending_delta == nullptr) != (pending_base == nullptr) ||
      (pending_delta != nullptr) != (pending_out != nullptr))
    return fail(PARROT_EINVAL, "depthmix: pending_base, pending_delta and pending_out go together%s");
  if ((pending_base && !aligned16(pending_base)) || (pending_delta && !aligned16(pending_delta)) ||
      (pending_out && !aligned16(pending_out)))
    return fail(PARROT_EINVAL, "depthmix: pending buffers must be 16-byte aligned%s");
  parrot::DepthMixArgs a{};
  a.pending_base = static_cast<const __nv_bfloat16*>(pending_base);
  a.pending_delta = static_cast<const __nv_bfloat16*>(pending_delta);
  a.pending_out = static_cast<__nv_bfloat16*>(pending_out);
  return depthmix_launch(out, sources, n_sources, query, key_norm_weight, key_eps,
                         out_norm_weight, out_eps, mix_out, a, rows, dim, stream);
}

int parrot_depthmix_moe_bf16(void* out, const void* const* sources, int n_sources,
                             const void* query, const void* key_norm_weight, float key_eps,
                             const void* out_norm_weight, float out_eps, void* mix_out,
                             const void* pending_base, const void* pending_shared,
                             const void* pending_contrib, void* pending_out, int rows, int dim,
                             void* stream) {
  if (!pending_shared || !pending_contrib || !pending_out)
    return fail(PARROT_EINVAL, "depthmix_moe: pending_shared, pending_contrib and pending_out are required%s");
  if (!aligned16(pending_shared) || !aligned16(pending_contrib) || !aligned16(pending_out) ||
      (pending_base && !aligned16(pending_base)))
    return fail(PARROT_EINVAL, "depthmix_moe: pending buffers must be 16-byte aligned%s");
  parrot::DepthMixArgs a{};
  a.pending_base = static_cast<const __nv_bfloat16*>(pending_base);
  a.pending_shared = static_cast<const __nv_bfloat16*>(pending_shared);
  a.pending_contrib = static_cast<const __nv_bfloat16*>(pending_contrib);
  a.pending_out = static_cast<__nv_bfloat16*>(pending_out);
  return depthmix_launch(out, sources, n_sources, query, key_norm_weight, key_eps,
                         out_norm_weight, out_eps, mix_out, a, rows, dim, stream);
}

int parrot_rope_inplace_bf16(void* x, const void* cos_table, const void* sin_table, int rows,
                             int row_stride, int rot_cols, int head_dim, int seq_len, int start,
                             int max_positions, void* stream) {
  if (rows < 0 || head_dim <= 0 || head_dim % 8 || rot_cols < 0 || rot_cols % head_dim ||
      row_stride < rot_cols || row_stride % 8 || seq_len <= 0 || start < 0)
    return fail(PARROT_EINVAL, "rope: need head_dim %% 8 == 0, rot_cols a multiple of head_dim, "
                               "row_stride %% 8 == 0 and >= rot_cols%s");
  if (start + seq_len > max_positions)
    return fail(PARROT_EINVAL, "rope: position exceeds the cos/sin tables%s");
  if (rows == 0 || rot_cols == 0) return PARROT_OK;
  if (!x || !cos_table || !sin_table || !aligned16(x))
    return fail(PARROT_EINVAL, "rope: null or misaligned pointer%s");
  if (parrot::launch_rope(static_cast<__nv_bfloat16*>(x),
                          static_cast<const __nv_bfloat16*>(cos_table),
                          static_cast<const __nv_bfloat16*>(sin_table), rows, row_stride,
                          rot_cols, head_dim, seq_len, start, nullptr, max_positions, nullptr,
                          static_cast<cudaStream_t>(stream)))
    return fail(PARROT_ECUDA, "rope: launch failed%s");
  return check_launch("rope_kernel");
}

int parrot_rope_inplace_at_bf16(void* x, const void* cos_table, const void* sin_table, int rows,
                                int row_stride, int rot_cols, int head_dim, int seq_len,
                                const int* start_dev, int max_positions, int* status,
                                void* stream) {
  if (rows < 0 || head_dim <= 0 || head_dim % 8 || rot_cols < 0 || rot_cols % head_dim ||
      row_stride < rot_cols || row_stride % 8 || seq_len <= 0 || max_positions <= 0)
    return fail(PARROT_EINVAL, "rope_at: need head_dim %% 8 == 0, rot_cols a multiple of "
                               "head_dim, row_stride %% 8 == 0 and >= rot_cols%s");
  if (rows == 0 || rot_cols == 0) return PARROT_OK;
  if (!x || !cos_table || !sin_table || !start_dev || !aligned16(x))
    return fail(PARROT_EINVAL, "rope_at: null or misaligned pointer%s");
  if (parrot::launch_rope(static_cast<__nv_bfloat16*>(x),
                          static_cast<const __nv_bfloat16*>(cos_table),
                          static_cast<const __nv_bfloat16*>(sin_table), rows, row_stride,
                          rot_cols, head_dim, seq_len, 0, start_dev, max_positions, status,
                          static_cast<cudaStream_t>(stream)))
    return fail(PARROT_ECUDA, "rope_at: launch failed%s");
  return check_launch("rope_kernel(device position)");
}

static int decode_attention(void* out, int out_f32, const void* q, int q_f32,
                            long long q_row_stride, const void* k_new, const void* v_new,
                            long long kv_row_stride, void* k_cache, void* v_cache,
                            const int* pos_dev, int batch, int n_heads, int n_kv_heads,
                            int max_positions, int head_dim, int window, float scale,
                            const void* cos_table, const void* sin_table, void* partials,
                            size_t partial_bytes, int* status, void* stream) {
  if (batch < 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads ||
      max_positions <= 0 || window < 0)
    return fail(PARROT_EINVAL, "decode_attention: bad sizes%s");
  if (partial_bytes < parrot_decode_attention_scratch_bytes(batch, n_heads, max_positions, head_dim))
    return fail(PARROT_EINVAL, "decode_attention: partials smaller than the scratch size%s");
  if (batch == 0) return PARROT_OK;
  if (!out || !q || !k_new || !k_cache || !pos_dev || !partials || (v_new == nullptr) != (v_cache == nullptr))
    return fail(PARROT_EINVAL, "decode_attention: null pointer (v_new and v_cache go together)%s");
  if (!aligned16(k_new) || !aligned16(k_cache) || (v_new && (!aligned16(v_new) || !aligned16(v_cache))))
    return fail(PARROT_EINVAL, "decode_attention: K/V must be 16-byte aligned%s");
  parrot::DecodeAttnArgs a{};
  a.q = q;
  a.q_f32 = q_f32;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.pos = pos_dev;
  a.slots = parrot::decode_attn_slots(batch, max_positions);
  a.part = static_cast<float*>(partials);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(partials) +
                                      (size_t)batch * n_heads * a.slots * (head_dim + 2) * sizeof(float));
  a.out = out;
  a.out_f32 = out_f32;
  a.B = batch;
  a.H = n_heads;
  a.KVH = n_kv_heads;
  a.S = max_positions;
  a.D = head_dim;
  a.window = window;
  a.q_row = q_row_stride > 0 ? q_row_stride : (long long)n_heads * head_dim;
  a.kv_row = kv_row_stride > 0 ? kv_row_stride : (long long)n_kv_heads * head_dim;
  if (a.kv_row % 8 || (long long)n_kv_heads * head_dim > a.kv_row || (long long)n_heads * head_dim > a.q_row)
    return fail(PARROT_EINVAL, "decode_attention: row strides too small or not 16-byte multiples%s");
  a.scale = scale;
  a.status = status;
  a.cos_t = static_cast<const __nv_bfloat16*>(cos_table);
  a.sin_t = static_cast<const __nv_bfloat16*>(sin_table);
  const int rc = parrot::launch_decode_attention(a, static_cast<cudaStream_t>(stream));
  if (rc == -1)
    return fail(PARROT_EUNSUPPORTED, "decode_attention: unsupported head width / group size%s");
  if (rc) return fail(PARROT_ECUDA, "decode_attention: launch failed%s");
  return check_launch("decode_attn_kernels");
}

int parrot_decode_attention_bf16(void* out, int out_f32, const void* q, int q_f32,
                                 long long q_row_stride, const void* k_new, const void* v_new,
                                 long long kv_row_stride, void* k_cache, void* v_cache,
                                 const int* pos_dev, int batch, int n_heads, int n_kv_heads,
                                 int max_positions, int head_dim, int window, float scale,
                                 void* partials, size_t partial_bytes, int* status,
                                 void* stream) {
  return decode_attention(out, out_f32, q, q_f32, q_row_stride, k_new, v_new, kv_row_stride,
                          k_cache, v_cache, pos_dev, batch, n_heads, n_kv_heads, max_positions,
                          head_dim, window, scale, nullptr, nullptr, partials, partial_bytes,
                          status, stream);
}

int parrot_decode_attention_rope_bf16(void* out, int out_f32, const void* q,
                                      long long q_row_stride, const void* k_new,
                                      const void* v_new, long long kv_row_stride, void* k_cache,
                                      void* v_cache, const int* pos_dev, int batch, int n_heads,
                                      int n_kv_heads, int max_positions, int head_dim,
                                      int window, float scale, const void* cos_table,
                                      const void* sin_table, int rope_positions,
                                      void* partials, size_t partial_bytes, int* status,
                                      void* stream) {
  if (!cos_table || !sin_table || rope_positions < max_positions || head_dim % 8)
    return fail(PARROT_EINVAL, "decode_attention_rope: need cos/sin tables of at least "
                               "max_positions rows and head_dim %% 8 == 0%s");
  if (((uintptr_t)q & 3) || q_row_stride % 2)
    return fail(PARROT_EINVAL, "decode_attention_rope: q rows must be 4-byte aligned%s");
  return decode_attention(out, out_f32, q, 0, q_row_stride, k_new, v_new, kv_row_stride,
                          k_cache, v_cache, pos_dev, batch, n_heads, n_kv_heads, max_positions,
                          head_dim, window, scale, cos_table, sin_table, partials,
                          partial_bytes, status, stream);
}

int parrot_linear_small(void* y, int y_f32, const void* x, int x_f32, const void* w, int w_f32,
                        int rows, int n_out, int k_in, void* stream) {
  if (rows < 0 || rows > 8 || n_out <= 0 || n_out % 16 || k_in <= 0 || k_in % 8 ||
      k_in > parrot::kLinearSmallMaxK)
    return fail(PARROT_EINVAL, "linear_small: need 0 <= rows <= 8, n_out %% 16 == 0 and "
                               "k_in %% 8 == 0, k_in <= 1024%s");
  if (rows == 0) return PARROT_OK;
  if (!y || !x || !w || !aligned16(x) || !aligned16(w) || ((uintptr_t)y & 3))
    return fail(PARROT_EINVAL, "linear_small: x and w must be 16-byte aligned, y 4-byte%s");
  parrot::LinearSmallArgs a{x, x_f32, w, w_f32, y, y_f32, rows, n_out, k_in};
  if (parrot::launch_linear_small(a, static_cast<cudaStream_t>(stream)))
    return fail(PARROT_ECUDA, "linear_small: launch failed%s");
  return check_launch("linear_small_kernel");
}

size_t parrot_decode_attention_scratch_bytes(int batch, int n_heads, int max_positions,
                                             int head_dim) {
  // partials [B, H, slots, D + 2] fp32, then one arrival counter per (batch row, head)
  return (size_t)batch * n_heads * parrot::decode_attn_slots(batch, max_positions) *
             (head_dim + 2) * sizeof(float) +
         (size_t)batch * n_heads * sizeof(int);
}

int parrot_moe_capacity(int tokens, int n_experts) {
  if (n_experts <= 0 || tokens < 0) return 0;
  const long long assignments = 2LL * tokens;
  const long long balanced = (2 * assignments + n_experts - 1) / n_experts;
  const long long c = (balanced + 7) / 8 * 8;
  return (int)(c < 8 ? 8 : c);
}

int parrot_moe_workspace_layout(const parrot_moe_dims* dims, parrot_moe_layout* layout) {
  if (layout == nullptr) return fail(PARROT_EINVAL, "layout is NULL%s");
  return layout_of(dims, layout);
}

int parrot_moe_workspace_init(void* workspace, const parrot_moe_dims* dims, void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if (workspace == nullptr) return fail(PARROT_EINVAL, "workspace is NULL%s");
  if (cudaMemsetAsync(workspace, 0, L.indices, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return check_launch("workspace init");
  return PARROT_OK;
}

int parrot_pack_gate_up_bf16(void* dst, const void* gate, const void* up, int n_mats, int hidden,
                             int dim, void* stream) {
  if (!dst || !gate || !up || n_mats <= 0 || hidden <= 0 || hidden % 64 || dim <= 0 || dim % 64)
    return fail(PARROT_EINVAL, "pack_gate_up: bad arguments (hidden % 64, dim % 64)%s");
  parrot::launch_pack_gate_up(static_cast<__nv_bfloat16*>(dst),
                              static_cast<const __nv_bfloat16*>(gate),
                              static_cast<const __nv_bfloat16*>(up), n_mats, hidden, dim,
                              static_cast<cudaStream_t>(stream));
  return check_launch("pack_gate_up_kernel");
}

int parrot_silu_bf16(const void* x, void* y, int64_t n, void* stream) {
  if (n < 0 || n > INT32_MAX || (n > 0 && (!x || !y)))
    return fail(PARROT_EINVAL, "silu: bad arguments (n out of range or NULL buffer)%s");
  if (parrot::launch_silu_bf16(static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), (int)n,
                               static_cast<cudaStream_t>(stream)) != 0)
    return fail(PARROT_ECUDA, "silu: building the SiLU table failed%s");
  return check_launch("silu_bf16_kernel");
}

int parrot_pack_down_bf16(void* dst, const void* src, int n_mats, int rows, int cols,
                          void* stream) {
  if (!dst || !src || n_mats <= 0 || rows <= 0 || rows % 128 || cols <= 0 || cols % 64)
    return fail(PARROT_EINVAL, "pack_down: bad arguments (rows % 128, cols % 64)%s");
  parrot::launch_pack_tiles(static_cast<__nv_bfloat16*>(dst), static_cast<const __nv_bfloat16*>(src),
                            n_mats, rows, cols, static_cast<cudaStream_t>(stream));
  return check_launch("pack_tiles_kernel");
}

int parrot_moe_route_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                          const void* x, const parrot_moe_outputs* outputs, void* workspace,
                          size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L);
  if (rc) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  return run_route(dims, weights, x, outputs, workspace, L, static_cast<cudaStream_t>(stream));
}

int parrot_moe_experts_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                            const void* x, const parrot_moe_outputs* outputs, void* workspace,
                            size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L);
  if (rc) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  return run_experts(dims, weights, x, outputs, workspace, L, static_cast<cudaStream_t>(stream));
}

int parrot_moe_forward_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                            const void* x, const parrot_moe_outputs* outputs, void* workspace,
                            size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L);
  if (rc) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool slots = slot_mode(dims, L);
  if ((rc = run_route(dims, weights, x, outputs, workspace, L, s, nullptr, slots))) return rc;
  return run_experts(dims, weights, x, outputs, workspace, L, s, true, slots);
}

int parrot_moe_forward_deferred_bf16(const parrot_moe_dims* dims,
                                     const parrot_moe_weights* weights, const void* x,
                                     const parrot_moe_outputs* outputs, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L, false);
  if (rc) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool slots = slot_mode(dims, L);
  if ((rc = run_route(dims, weights, x, outputs, workspace, L, s, nullptr, slots))) return rc;
  return run_experts(dims, weights, x, outputs, workspace, L, s, false, slots);
}

int parrot_depthmix_route_bf16(void* out, const void* const* sources, int n_sources,
                               const void* query, const void* key_norm_weight, float key_eps,
                               const void* out_norm_weight, float out_eps, void* mix_out,
                               const void* pending_base, const void* pending_delta,
                               void* pending_out, int rows, int dim,
                               const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                               const parrot_moe_outputs* outputs, void* workspace,
                               size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if (dims->tokens != rows || dims->dim != dim || rows > 4096 || out_norm_weight == nullptr)
    return fail(PARROT_EINVAL, "depthmix_route: rows == dims->tokens <= 4096, dims->dim == dim "
                               "and the consumer norm weight required%s");
  if ((rc = check_router(weights)) || (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (outputs == nullptr) return fail(PARROT_EINVAL, "depthmix_route: outputs is NULL%s");
  if ((pending_delta == nullptr) != (pending_base == nullptr) ||
      (pending_delta != nullptr) != (pending_out != nullptr))
    return fail(PARROT_EINVAL, "depthmix_route: pending base, delta and out go together%s");
  if ((pending_base && !aligned16(pending_base)) || (pending_delta && !aligned16(pending_delta)) ||
      (pending_out && !aligned16(pending_out)))
    return fail(PARROT_EINVAL, "depthmix_route: pending buffers must be 16-byte aligned%s");
  parrot::DepthMixArgs a{};
  a.pending_base = static_cast<const __nv_bfloat16*>(pending_base);
  a.pending_delta = static_cast<const __nv_bfloat16*>(pending_delta);
  a.pending_out = static_cast<__nv_bfloat16*>(pending_out);
  parrot::DepthRouteArgs r{};
  r.router_w = static_cast<const __nv_bfloat16*>(weights->router);
  r.r = route_args(dims, weights, outputs, workspace, L);
  if (slot_mode(dims, L)) set_slots(&r.r, workspace, L, nullptr);  // the mix has the rows
  return depthmix_launch(out, sources, n_sources, query, key_norm_weight, key_eps,
                         out_norm_weight, out_eps, mix_out, a, rows, dim, stream, &r);
}

int parrot_moe_forward_routed_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                   const void* x, const parrot_moe_outputs* outputs, int deferred,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L, !deferred);
  if (rc) return rc;
  if (outputs->probs != nullptr || outputs->indices != nullptr || outputs->weights != nullptr)
    return fail(PARROT_EINVAL, "moe_forward_routed: probs, indices and weights come from the "
                               "routing call%s");
  if (dims->tokens == 0) return PARROT_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool slots = slot_mode(dims, L);  // the routing depth mix grouped the rows
  if (!slots && (rc = run_group(dims, x, outputs, workspace, L, s, nullptr, true))) return rc;
  return run_experts(dims, weights, x, outputs, workspace, L, s, !deferred, slots);
}

static int moe_decode(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                      const void* x, const parrot_moe_outputs* outputs, void* workspace,
                      size_t workspace_bytes, void* stream, bool routed) {
  parrot_moe_layout L;
  int rc = prepare(dims, weights, x, outputs, workspace, workspace_bytes, &L);
  if (rc) return rc;
  if (dims->tokens > parrot::kDecodeMoeMaxTokens || dims->expert_dim > 1024 ||
      dims->shared_dim > dims->expert_dim || dims->expert_dim % 32 || dims->shared_dim % 32)
    return fail(PARROT_EINVAL, "moe_decode: tokens <= 16, shared_dim <= expert_dim <= 1024, "
                               "both multiples of 32%s");
  if (outputs->counts != nullptr || outputs->stats != nullptr || outputs->positions != nullptr)
    return fail(PARROT_EINVAL, "moe_decode: no grouping, counts or statistics on this path%s");
  if (routed && (outputs->probs != nullptr || outputs->indices != nullptr ||
                 outputs->weights != nullptr))
    return fail(PARROT_EINVAL, "moe_decode_routed: probs, indices and weights come from the "
                               "routing call%s");
  if (dims->tokens == 0) return PARROT_OK;
  parrot::MoeDecodeArgs a{};
  a.routed = routed ? 1 : 0;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.router = static_cast<const __nv_bfloat16*>(weights->router);
  a.router_bias = weights->router_bias;
  a.gate_up = static_cast<const __nv_bfloat16*>(weights->gate_up);
  a.down = static_cast<const __nv_bfloat16*>(weights->down);
  a.shared_gate_up = static_cast<const __nv_bfloat16*>(weights->shared_gate_up);
  a.shared_down = static_cast<const __nv_bfloat16*>(weights->shared_down);
  a.hidden = at<__nv_bfloat16>(workspace, L.hidden);
  a.indices = at<int>(workspace, L.indices);
  a.weights = at<float>(workspace, L.weights);
  a.probs = outputs->probs;
  a.indices64 = outputs->indices;
  a.weights_out = outputs->weights;
  a.residual = static_cast<const __nv_bfloat16*>(outputs->residual);
  a.out = static_cast<__nv_bfloat16*>(outputs->out);
  a.tokens = dims->tokens;
  a.dim = dims->dim;
  a.n_experts = dims->n_experts;
  a.expert_dim = dims->expert_dim;
  a.shared_dim = dims->shared_dim;
  if (parrot::launch_moe_decode(a, static_cast<cudaStream_t>(stream)))
    return fail(PARROT_ECUDA, "moe_decode: launch failed%s");
  return check_launch("moe_decode kernels");
}

int parrot_moe_decode_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                           const void* x, const parrot_moe_outputs* outputs, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return moe_decode(dims, weights, x, outputs, workspace, workspace_bytes, stream, false);
}

int parrot_moe_decode_routed_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                  const void* x, const parrot_moe_outputs* outputs,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  return moe_decode(dims, weights, x, outputs, workspace, workspace_bytes, stream, true);
}

int parrot_moe_gemm_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                         const void* x, void* workspace, size_t workspace_bytes, int stage,
                         void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if ((rc = check_weights(weights))) return rc;
  if (stage != 0 && stage != 1) return fail(PARROT_EINVAL, "stage must be 0 or 1%s");
  if (workspace == nullptr || workspace_bytes < L.total || !aligned16(workspace))
    return fail(PARROT_EINVAL, "workspace missing, misaligned or too small%s");
  if (dims->tokens == 0) return PARROT_OK;
  if (x == nullptr || !aligned16(x)) return fail(PARROT_EINVAL, "x must be 16-byte aligned%s");
  return run_gemm(stage == 0, dims, weights, x, workspace, L, static_cast<cudaStream_t>(stream));
}

unsigned long long parrot_b200_launch_count(void) {
  return g_launches.load(std::memory_order_relaxed);
}

int parrot_moe_forward_static_bf16(const parrot_moe_dims* dims,
                                   const parrot_moe_weights* weights, const void* x,
                                   const parrot_moe_outputs* outputs, void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if (L.total > kStaticWorkspaceBytes) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "%zu bytes, more than the %zu-byte static workspace",
                  L.total, kStaticWorkspaceBytes);
    return fail(PARROT_EINVAL, "moe_forward_static: these dims need a workspace of %s", msg);
  }
  void* ws = nullptr;
  if ((rc = static_workspace_address(&ws))) return rc;
  if ((rc = prepare(dims, weights, x, outputs, ws, kStaticWorkspaceBytes, &L))) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps whatever the previous call left: the status word must
  // start at zero, so clear it first.
  if (cudaMemsetAsync(ws, 0, L.indices, s) != cudaSuccess)
    return check_launch("static workspace clear");
  const bool slots = slot_mode(dims, L);
  if ((rc = run_route(dims, weights, x, outputs, ws, L, s, nullptr, slots))) return rc;
  return run_experts(dims, weights, x, outputs, ws, L, s, true, slots);
}

int parrot_moe_ep_dispatch_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                const void* x, const parrot_moe_outputs* outputs, int ep_ranks,
                                void* workspace, size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if (dims->capacity != -1)
    return fail(PARROT_EINVAL, "ep_dispatch: dims->capacity must be -1 (packed rows)%s");
  if (ep_ranks < 1 || dims->n_experts % ep_ranks)
    return fail(PARROT_EINVAL, "ep_dispatch: ep_ranks must divide n_experts%s");
  if ((rc = check_router(weights)) || (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (outputs == nullptr) return fail(PARROT_EINVAL, "ep_dispatch: outputs is NULL%s");
  if (dims->tokens == 0) return PARROT_OK;
  if (x == nullptr || !aligned16(x)) return fail(PARROT_EINVAL, "x must be 16-byte aligned%s");
  signed char order[parrot::kMaxExperts];
  const int G = ep_ranks, El = dims->n_experts / G;
  for (int q = 0; q < dims->n_experts; ++q) order[q] = (signed char)((q % El) * G + q / El);
  return run_route(dims, weights, x, outputs, workspace, L, static_cast<cudaStream_t>(stream),
                   order);
}

int parrot_moe_ep_dispatch_planned_bf16(const parrot_moe_dims* dims,
                                        const parrot_moe_weights* weights, const void* x,
                                        const parrot_moe_outputs* outputs,
                                        const parrot_ep_dims* ep, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  parrot_ep_layout P;
  int rc = layout_of(dims, &L);
  if (rc || (rc = ep_layout_of(ep, &P))) return rc;
  if (dims->capacity != -1 || dims->n_experts != ep->n_experts || dims->dim != ep->dim)
    return fail(PARROT_EINVAL, "ep_dispatch: dims must be packed (capacity -1) and match ep%s");
  signed char plan[parrot::kEpMaxRanks][parrot::kMaxExperts];
  if ((rc = ep_plan(ep, plan))) return rc;
  if ((rc = check_router(weights)) || (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (outputs == nullptr) return fail(PARROT_EINVAL, "ep_dispatch: outputs is NULL%s");
  if (dims->tokens == 0) return PARROT_OK;
  if (x == nullptr || !aligned16(x)) return fail(PARROT_EINVAL, "x must be 16-byte aligned%s");
  signed char order[parrot::kMaxExperts];
  ep_order(plan, ep->ranks, order);
  return run_route(dims, weights, x, outputs, workspace, L, static_cast<cudaStream_t>(stream),
                   order);
}

int parrot_moe_shared_ffn_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                               const void* x, void* workspace, size_t workspace_bytes,
                               void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if ((rc = check_shared(weights)) || (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  if (x == nullptr || !aligned16(x)) return fail(PARROT_EINVAL, "x must be 16-byte aligned%s");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = run_gemm(true, dims, weights, x, workspace, L, s, true))) return rc;
  return run_gemm(false, dims, weights, x, workspace, L, s, true);
}

int parrot_moe_expert_ffn_bf16(int rows, int dim, int expert_dim, int n_mats, int n_segments,
                               const int* seg_rows, const int* seg_base, const int* seg_expert,
                               const void* gate_up, const void* down, const void* x,
                               void* hidden, void* y, int* status, void* stream) {
  if (rows < 0 || n_segments < 0 || n_segments > 2 * parrot::kMaxExperts)
    return fail(PARROT_EINVAL, "expert_ffn: rows >= 0 and 0 <= n_segments <= 64 required%s");
  if (dim <= 0 || dim % 128 || dim > 1024 || expert_dim <= 0 || expert_dim % 64 || n_mats < 1)
    return fail(PARROT_EINVAL, "expert_ffn: dim % 128 == 0 (<= 1024), expert_dim % 64 == 0%s");
  if (rows == 0 || n_segments == 0) return PARROT_OK;
  if (!seg_rows || !seg_base || !seg_expert || !gate_up || !down || !x || !hidden || !y)
    return fail(PARROT_EINVAL, "expert_ffn: null pointer%s");
  if (!aligned16(gate_up) || !aligned16(down) || !aligned16(x) || !aligned16(hidden) ||
      !aligned16(y))
    return fail(PARROT_EINVAL, "expert_ffn: buffers must be 16-byte aligned%s");
  return run_ffn(rows, dim, expert_dim, n_mats, n_segments, seg_rows, seg_base, seg_expert,
                 gate_up, down, x, hidden, y, status, static_cast<cudaStream_t>(stream));
}

int parrot_moe_ep_combine_bf16(const parrot_moe_dims* dims, const void* y, const void* workspace,
                               size_t workspace_bytes, const void* residual, void* out,
                               void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if ((rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  if (!y || !out || !aligned16(y) || !aligned16(out) || (residual && !aligned16(residual)))
    return fail(PARROT_EINVAL, "ep_combine: y/out/residual must be 16-byte aligned%s");
  void* ws = const_cast<void*>(workspace);
  parrot::EpCombineArgs c{};
  c.y = static_cast<const __nv_bfloat16*>(y);
  c.indices = at<int>(ws, L.indices);
  c.weights = at<float>(ws, L.weights);
  c.positions = at<int>(ws, L.positions);
  c.shared_y = at<__nv_bfloat16>(ws, L.shared_y);
  c.residual = static_cast<const __nv_bfloat16*>(residual);
  c.out = static_cast<__nv_bfloat16*>(out);
  c.tokens = dims->tokens;
  c.dim = dims->dim;
  c.rows = L.grouped_rows;
  c.status = at<int>(ws, L.status);
  if (parrot::launch_ep_combine(c, static_cast<cudaStream_t>(stream)))
    return fail(PARROT_EINVAL, "ep_combine: unsupported dim%s");
  return check_launch("ep_combine_kernel");
}

size_t parrot_vocab_argmax_scratch_bytes(void) {
  return 256 + (size_t)parrot::kVocabMaxGrid * 8 * (sizeof(float) + sizeof(int));
}

int parrot_vocab_argmax_bf16(long long* out, const void* hidden, const void* weight, int rows,
                             int dim, int vocab, void* scratch, size_t scratch_bytes,
                             void* stream) {
  if (rows < 0 || rows > 8)
    return fail(PARROT_EINVAL, "vocab_argmax: 0 <= rows <= 8 required%s");
  if (dim <= 0 || dim % 8 || dim > 1024 || vocab < 1)
    return fail(PARROT_EINVAL, "vocab_argmax: dim % 8 == 0 (<= 1024) and vocab >= 1 required%s");
  if (rows == 0) return PARROT_OK;
  if (!out || !hidden || !weight || !aligned16(hidden) || !aligned16(weight))
    return fail(PARROT_EINVAL, "vocab_argmax: out and 16-byte aligned hidden/weight required%s");
  if (!scratch || (reinterpret_cast<uintptr_t>(scratch) & 255) ||
      scratch_bytes < parrot_vocab_argmax_scratch_bytes())
    return fail(PARROT_EINVAL, "vocab_argmax: scratch missing, misaligned or too small%s");
  char* sc = static_cast<char*>(scratch);
  parrot::VocabArgmaxArgs a{};
  a.hidden = hidden;
  a.weight = weight;
  a.rows = rows;
  a.dim = dim;
  a.vocab = vocab;
  a.counter = reinterpret_cast<unsigned*>(sc);
  a.partial_value = reinterpret_cast<float*>(sc + 256);
  a.partial_index = reinterpret_cast<int*>(sc + 256 + (size_t)parrot::kVocabMaxGrid * 8 * 4);
  a.out = out;
  if (parrot::launch_vocab_argmax(a, sm_count(), static_cast<cudaStream_t>(stream)))
    return fail(PARROT_EINVAL, "vocab_argmax: unsupported dim%s");
  return check_launch("vocab_argmax_kernel");
}

int parrot_argmax_rows_bf16(long long* out, const void* logits, int rows, int cols, void* stream) {
  if (rows < 0 || cols < 8 || cols % 8)
    return fail(PARROT_EINVAL, "argmax_rows: rows >= 0 and cols % 8 == 0 required%s");
  if (rows == 0) return PARROT_OK;
  if (!out || !logits || !aligned16(logits))
    return fail(PARROT_EINVAL, "argmax_rows: out and 16-byte aligned logits required%s");
  parrot::ArgmaxRowsArgs a{logits, rows, cols, out};
  parrot::launch_argmax_rows(a, static_cast<cudaStream_t>(stream));
  return check_launch("argmax_rows_kernel");
}

int parrot_ep_buffer_layout(const parrot_ep_dims* ep, parrot_ep_layout* layout) {
  return ep_layout_of(ep, layout);
}

int parrot_ipc_export(const void* ptr, void* handle, unsigned long long* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(PARROT_EINVAL, "ipc_export: null argument%s");
  MemGetAddressRangeFn range = address_range_fn();
  if (range == nullptr) return fail(PARROT_ECUDA, "ipc_export: cuMemGetAddressRange unavailable%s");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(PARROT_EINVAL, "ipc_export: not a device allocation%s");
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess)
    return fail(PARROT_ECUDA, "ipc_export: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(err));
  std::memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<CUdeviceptr>(ptr) - base;
  return PARROT_OK;
}

int parrot_ipc_import(const void* handle, unsigned long long offset, void** ptr, void** base) {
  if (handle == nullptr || ptr == nullptr || base == nullptr)
    return fail(PARROT_EINVAL, "ipc_import: null argument%s");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess)
    return fail(PARROT_ECUDA, "ipc_import: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(err));
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return PARROT_OK;
}

int parrot_ipc_close(void* base) {
  if (base == nullptr) return PARROT_OK;
  const cudaError_t err = cudaIpcCloseMemHandle(base);
  if (err != cudaSuccess)
    return fail(PARROT_ECUDA, "ipc_close: cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(err));
  return PARROT_OK;
}

// The send kernel over a checked dispatch (rows_sent: the grouping kernel
// already stored the rows; counts, row base and arrival flags only).
static int ep_send(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                   const parrot_ep_peers* peers, const void* workspace,
                   const parrot_moe_layout& L, const parrot_ep_layout& P, bool rows_sent,
                   cudaStream_t stream) {
  char* own = static_cast<char*>(peers->buffers[ep->rank]);
  parrot::EpSendArgs a{};
  int rc = ep_plan(ep, a.plan);
  if (rc) return rc;
  if (dims->tokens > 0) {
    void* ws = const_cast<void*>(workspace);
    a.rows = at<__nv_bfloat16>(ws, L.grouped);
    a.counts = at<int>(ws, L.counts);
  }
  a.rows_sent = rows_sent ? 1 : 0;
  a.tokens = dims->tokens;
  a.dim = ep->dim;
  a.n_experts = ep->n_experts;
  a.ranks = ep->ranks;
  a.rank = ep->rank;
  a.max_tokens = ep->max_tokens;
  for (int r = 0; r < ep->ranks; ++r) a.peers[r] = static_cast<char*>(peers->buffers[r]);
  a.off_recv = P.recv_rows;
  a.off_meta = P.meta;
  a.off_flags_in = P.flags_in;
  a.epoch = reinterpret_cast<unsigned*>(own + P.epoch);
  a.counter = reinterpret_cast<unsigned*>(own + P.counters);
  a.status = reinterpret_cast<int*>(own + P.status);
  parrot::launch_ep_send(a, sm_count(), stream);
  return check_launch("ep_send_kernel");
}

static int ep_send_checks(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                          const parrot_ep_peers* peers, parrot_moe_layout* L,
                          parrot_ep_layout* P) {
  int rc = layout_of(dims, L);
  if (rc || (rc = ep_layout_of(ep, P)) || (rc = ep_peers_ok(ep, peers))) return rc;
  if (dims->capacity != -1 || dims->dim != ep->dim || dims->n_experts != ep->n_experts)
    return fail(PARROT_EINVAL, "ep_send: dims must be the packed dispatch dims of this EP set%s");
  if (dims->tokens > ep->max_tokens)
    return fail(PARROT_EINVAL, "ep_send: more tokens than ep->max_tokens%s");
  return PARROT_OK;
}

int parrot_moe_ep_send_bf16(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                            const parrot_ep_peers* peers, const void* workspace,
                            size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  parrot_ep_layout P;
  int rc = ep_send_checks(dims, ep, peers, &L, &P);
  if (rc) return rc;
  if (dims->tokens > 0 && (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  return ep_send(dims, ep, peers, workspace, L, P, false, static_cast<cudaStream_t>(stream));
}

int parrot_moe_ep_dispatch_send_bf16(const parrot_moe_dims* dims,
                                     const parrot_moe_weights* weights, const void* x,
                                     const parrot_moe_outputs* outputs, const parrot_ep_dims* ep,
                                     const parrot_ep_peers* peers, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  parrot_moe_layout L;
  parrot_ep_layout P;
  int rc = ep_send_checks(dims, ep, peers, &L, &P);
  if (rc) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dims->tokens == 0) return ep_send(dims, ep, peers, workspace, L, P, true, s);
  signed char plan[parrot::kEpMaxRanks][parrot::kMaxExperts];
  if ((rc = ep_plan(ep, plan))) return rc;
  if ((rc = check_router(weights)) || (rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (outputs == nullptr) return fail(PARROT_EINVAL, "ep_dispatch_send: outputs is NULL%s");
  if (x == nullptr || !aligned16(x)) return fail(PARROT_EINVAL, "x must be 16-byte aligned%s");
  signed char order[parrot::kMaxExperts];
  ep_order(plan, ep->ranks, order);
  EpRowsTo to{};
  for (int q = 0; q < ep->ranks; ++q) {
    to.recv[q] = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(peers->buffers[q]) +
                                                   P.recv_rows) +
                 (size_t)ep->rank * P.region_rows * ep->dim;
    for (int j = 0; j < parrot::kMaxExperts; ++j)
      if (plan[q][j] >= 0) to.dest[plan[q][j]] = (signed char)q;
  }
  to.region = P.region_rows;
  if ((rc = run_route(dims, weights, x, outputs, workspace, L, s, order, false, &to))) return rc;
  return ep_send(dims, ep, peers, workspace, L, P, true, s);
}

int parrot_moe_ep_receive(const parrot_ep_dims* ep, void* buffer, void* stream) {
  parrot_ep_layout P;
  int rc = ep_layout_of(ep, &P);
  if (rc) return rc;
  if (buffer == nullptr) return fail(PARROT_EINVAL, "ep_receive: buffer is NULL%s");
  char* b = static_cast<char*>(buffer);
  parrot::EpReceiveArgs a{};
  a.flags_in = reinterpret_cast<const unsigned*>(b + P.flags_in);
  a.meta = reinterpret_cast<const int*>(b + P.meta);
  a.epoch = reinterpret_cast<const unsigned*>(b + P.epoch);
  a.ranks = ep->ranks;
  a.slots = ep_slots(ep);
  a.max_tokens = ep->max_tokens;
  a.seg_rows = reinterpret_cast<int*>(b + P.seg_rows);
  a.seg_base = reinterpret_cast<int*>(b + P.seg_base);
  a.seg_expert = reinterpret_cast<int*>(b + P.seg_expert);
  a.back_n = reinterpret_cast<int*>(b + P.back_n);
  a.back_base = reinterpret_cast<int*>(b + P.back_base);
  a.wait_ns = ep_wait_ns(ep);
  a.status = reinterpret_cast<int*>(b + P.status);
  parrot::launch_ep_receive(a, static_cast<cudaStream_t>(stream));
  return check_launch("ep_receive_kernel");
}

int parrot_moe_ep_experts_bf16(const parrot_ep_dims* ep, void* buffer, const void* gate_up,
                               const void* down, void* stream) {
  parrot_ep_layout P;
  int rc = ep_layout_of(ep, &P);
  if (rc) return rc;
  if (buffer == nullptr || gate_up == nullptr || down == nullptr || !aligned16(gate_up) ||
      !aligned16(down))
    return fail(PARROT_EINVAL, "ep_experts: buffer and 16-byte aligned weights required%s");
  char* b = static_cast<char*>(buffer);
  const int slots = ep_slots(ep);
  return run_ffn(ep->ranks * P.region_rows, ep->dim, ep->expert_dim, slots, ep->ranks * slots,
                 reinterpret_cast<const int*>(b + P.seg_rows),
                 reinterpret_cast<const int*>(b + P.seg_base),
                 reinterpret_cast<const int*>(b + P.seg_expert), gate_up, down, b + P.recv_rows,
                 b + P.hidden, b + P.y, reinterpret_cast<int*>(b + P.status),
                 static_cast<cudaStream_t>(stream));
}

// The return kernel (rows_sent: the down GEMM already stored the outputs;
// the return flags only).
static int ep_return(const parrot_ep_dims* ep, const parrot_ep_peers* peers,
                     const parrot_ep_layout& P, bool rows_sent, void* stream) {
  char* own = static_cast<char*>(peers->buffers[ep->rank]);
  parrot::EpReturnArgs a{};
  a.rows_sent = rows_sent ? 1 : 0;
  a.y = reinterpret_cast<const __nv_bfloat16*>(own + P.y);
  a.back_n = reinterpret_cast<const int*>(own + P.back_n);
  a.back_base = reinterpret_cast<const int*>(own + P.back_base);
  for (int r = 0; r < ep->ranks; ++r) a.peers[r] = static_cast<char*>(peers->buffers[r]);
  a.off_back = P.back_rows;
  a.off_flags_back = P.flags_back;
  a.ranks = ep->ranks;
  a.rank = ep->rank;
  a.dim = ep->dim;
  a.max_tokens = ep->max_tokens;
  a.epoch = reinterpret_cast<const unsigned*>(own + P.epoch);
  a.counter = reinterpret_cast<unsigned*>(own + P.counters) + 1;
  parrot::launch_ep_return(a, sm_count(), static_cast<cudaStream_t>(stream));
  return check_launch("ep_return_kernel");
}

int parrot_moe_ep_return_bf16(const parrot_ep_dims* ep, const parrot_ep_peers* peers,
                              void* stream) {
  parrot_ep_layout P;
  int rc = ep_layout_of(ep, &P);
  if (rc || (rc = ep_peers_ok(ep, peers))) return rc;
  return ep_return(ep, peers, P, false, stream);
}

int parrot_moe_ep_experts_return_bf16(const parrot_ep_dims* ep, const parrot_ep_peers* peers,
                                      const void* gate_up, const void* down, void* stream) {
  parrot_ep_layout P;
  int rc = ep_layout_of(ep, &P);
  if (rc || (rc = ep_peers_ok(ep, peers))) return rc;
  if (gate_up == nullptr || down == nullptr || !aligned16(gate_up) || !aligned16(down))
    return fail(PARROT_EINVAL, "ep_experts_return: 16-byte aligned weights required%s");
  char* b = static_cast<char*>(peers->buffers[ep->rank]);
  const int slots = ep_slots(ep);
  EpRowsBack back{};
  for (int q = 0; q < ep->ranks; ++q)
    back.back[q] = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(peers->buffers[q]) +
                                                    P.back_rows);
  back.base = reinterpret_cast<const int*>(b + P.back_base);
  back.segs_per_source = slots;
  back.region = P.region_rows;
  rc = run_ffn(ep->ranks * P.region_rows, ep->dim, ep->expert_dim, slots, ep->ranks * slots,
               reinterpret_cast<const int*>(b + P.seg_rows),
               reinterpret_cast<const int*>(b + P.seg_base),
               reinterpret_cast<const int*>(b + P.seg_expert), gate_up, down, b + P.recv_rows,
               b + P.hidden, b + P.y, reinterpret_cast<int*>(b + P.status),
               static_cast<cudaStream_t>(stream), &back);
  if (rc) return rc;
  return ep_return(ep, peers, P, true, stream);
}

int parrot_moe_ep_combine_peer_bf16(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                                    const void* buffer, const void* workspace,
                                    size_t workspace_bytes, const void* residual, void* out,
                                    void* stream) {
  parrot_moe_layout L;
  parrot_ep_layout P;
  int rc = layout_of(dims, &L);
  if (rc || (rc = ep_layout_of(ep, &P))) return rc;
  if (dims->tokens > ep->max_tokens || dims->dim != ep->dim)
    return fail(PARROT_EINVAL, "ep_combine_peer: dims do not match the EP set%s");
  if (buffer == nullptr) return fail(PARROT_EINVAL, "ep_combine_peer: buffer is NULL%s");
  if ((rc = ws_ok(workspace, workspace_bytes, L))) return rc;
  if (dims->tokens == 0) return PARROT_OK;
  if (!out || !aligned16(out) || (residual && !aligned16(residual)))
    return fail(PARROT_EINVAL, "ep_combine_peer: out/residual must be 16-byte aligned%s");
  void* ws = const_cast<void*>(workspace);
  char* b = static_cast<char*>(const_cast<void*>(buffer));
  parrot::EpCombineArgs c{};
  c.y = reinterpret_cast<const __nv_bfloat16*>(b + P.back_rows);
  c.indices = at<int>(ws, L.indices);
  c.weights = at<float>(ws, L.weights);
  c.positions = at<int>(ws, L.positions);
  c.shared_y = at<__nv_bfloat16>(ws, L.shared_y);
  c.residual = static_cast<const __nv_bfloat16*>(residual);
  c.out = static_cast<__nv_bfloat16*>(out);
  c.tokens = dims->tokens;
  c.dim = dims->dim;
  c.rows = 2 * dims->tokens;
  c.status = at<int>(ws, L.status);
  c.wait_flags = reinterpret_cast<const unsigned*>(b + P.flags_back);
  c.wait_epoch = reinterpret_cast<const unsigned*>(b + P.epoch);
  c.wait_status = reinterpret_cast<int*>(b + P.status);
  c.wait_ranks = ep->ranks;
  c.wait_ns = ep_wait_ns(ep);
  if (parrot::launch_ep_combine(c, static_cast<cudaStream_t>(stream)))
    return fail(PARROT_EINVAL, "ep_combine_peer: unsupported dim%s");
  return check_launch("ep_combine_kernel");
}

int parrot_ep_read_status(const parrot_ep_dims* ep, const void* buffer, int* host_status4,
                          void* stream) {
  parrot_ep_layout P;
  int rc = ep_layout_of(ep, &P);
  if (rc) return rc;
  if (!buffer || !host_status4) return fail(PARROT_EINVAL, "null pointer%s");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_status4, static_cast<const char*>(buffer) + P.status, 16,
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("read EP status");
  return PARROT_OK;
}

int parrot_moe_read_status(const void* workspace, const parrot_moe_dims* dims, int* host_status4,
                           void* stream) {
  parrot_moe_layout L;
  int rc = layout_of(dims, &L);
  if (rc) return rc;
  if (!workspace || !host_status4) return fail(PARROT_EINVAL, "null pointer%s");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_status4, static_cast<const char*>(workspace) + L.status, 16,
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("read status");
  return PARROT_OK;
}

int parrot_selftest_wait_timeout(unsigned long long limit_ns, int* device_out8, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000ull)
    return fail(PARROT_EINVAL, "selftest_wait_timeout: 1 us <= limit_ns <= 1 s required%s");
  if (device_out8 == nullptr || (reinterpret_cast<uintptr_t>(device_out8) & 15))
    return fail(PARROT_EINVAL, "selftest_wait_timeout: 16-byte aligned output required%s");
  if (cudaMemsetAsync(device_out8, 0, 8 * sizeof(int), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return check_launch("selftest clear");
  parrot::launch_mbar_timeout_selftest(limit_ns, device_out8, static_cast<cudaStream_t>(stream));
  return check_launch("mbar_timeout_selftest_kernel");
}

}  // extern "C"
