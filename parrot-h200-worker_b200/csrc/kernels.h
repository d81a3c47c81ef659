// Internal launcher declarations shared by the .cu files and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace parrot {

constexpr int kMaxDepthSources = 16;
constexpr int kMaxExperts = 32;
constexpr int kEpMaxRanks = 8;             // expert-parallel ranks (ep_peer.cu)
constexpr int kGroupTokensPerBlock = 32;   // grouping block / histogram chunk: 64 assignments
constexpr int kGemmSubRows = 64;           // token rows per activation TMA box
constexpr int kGemmBlockK = 64;            // 128-byte swizzled K slab
// Token rows per grouped-GEMM tile: 256 once the rows are many (each weight
// tile is streamed once per tile of its expert), else 128 (a deeper ring).
inline int gemm_token_tile(long long rows) { return rows >= 4096 ? 256 : 128; }

struct DepthMixArgs {
  const __nv_bfloat16* sources[kMaxDepthSources];
  int n_sources;
  const __nv_bfloat16* query;
  const __nv_bfloat16* key_w;
  float key_eps;
  const __nv_bfloat16* out_w;     // consumer RMSNorm weight, or null
  float out_eps;
  __nv_bfloat16* out;
  __nv_bfloat16* mix_out;         // optional un-normalised mix
  const __nv_bfloat16* pending_base;   // optional deferred residual
  const __nv_bfloat16* pending_delta;
  const __nv_bfloat16* pending_shared;   // optional deferred MoE combine: shared output
  const __nv_bfloat16* pending_contrib;  // and [2 rows, dim] routed contributions
  __nv_bfloat16* pending_out;
  int rows;
  int dim;
};

// Device-side MoE bookkeeping.  The router writes per-chunk (32 tokens) and
// per-tile (128 tokens) expert histograms and per-tile probability sums; the
// grouping kernel turns them into slots and writes the segment tables, counts
// and statistics that the GEMMs and the caller read.
struct MoeTables {
  int* chunk_hist;     // [chunks, E]  assignments per expert in each 32-token chunk
                       //              (written by the 128-token tensor-core router)
  int* tile_hist;      // [tiles, E]   the same per router tile (8 or 128 tokens)
  float* tile_probsum;  // [tiles, E]  sum of router probabilities per expert
  int* counts;         // [E]
  int* seg_rows;       // [2E] rows in capacity segment e, overflow segment e
  int* seg_base;       // [2E] first grouped row of each segment
  float* stats;        // [E + 1]: utilisation[E], aux
};

struct RouteArgs {
  const float* bias;          // [E] or null (harness-only logit offset)
  float* probs;               // [T, E] or null
  int* indices;               // [T, 2]
  float* weights;             // [T, 2]
  long long* indices64;       // [T, 2] or null (reference dtype)
  float* weights_out;         // [T, 2] or null: caller's copy of weights
  MoeTables tab;
  int tokens, dim, n_experts;
  int* status;
  // Slot mode (slot_counts != null; the routers up to 4096 tokens): the
  // grouping done by the router too.  Each assignment takes the next slot of
  // its expert from a per-expert counter (zero before the call), its row goes
  // to grouped row e * slot_stride + slot with the position, contribution
  // slot and route weight; the GEMMs read the counters as segment sizes.
  // Rows keep no order within an expert (the products do not depend on it).
  int* slot_counts;           // [E]
  int slot_stride;            // rows per expert region (>= 2T: no overflow)
  const __nv_bfloat16* slot_x;  // the token rows the router reads (its copy source)
  __nv_bfloat16* grouped;
  int* positions;             // [2T]
  int* row_dst;               // [E * slot_stride]
  float* row_w;
};

// The router folded into a depth mix whose normalised output is the MoE
// block's input (norm.cu): the router weight and the router's outputs.
struct DepthRouteArgs {
  const __nv_bfloat16* router_w;  // [E, d]
  RouteArgs r;                    // tokens == the depth mix's rows (slot mode included)
};

struct GroupArgs {
  const __nv_bfloat16* x;     // [T, d]
  const int* indices;         // [T, 2]
  const float* weights;       // [T, 2] route weights
  MoeTables tab;
  int* positions;             // [2T] grouped row of each assignment
  int* positions_out;         // [2T] or null: caller's copy
  int* row_dst;               // [R] token-major contribution slot of each grouped row
  float* row_w;               // [R] route weight of each grouped row
  __nv_bfloat16* grouped;     // [E*C + 2T, d]
  int* counts_out;            // [E] or null
  float* stats_out;           // [E + 1] or null
  int tokens, dim, n_experts, capacity;
  // ep_packed (expert parallelism): the overflow segments are packed in the
  // order ep_order lists the experts (destination rank major, then the
  // destination's slot order), so each destination's rows form one
  // contiguous block; 0: expert id order
  int ep_packed;
  signed char ep_order[kMaxExperts];
  int x_from_upstream;  // x is written by the kernel this one waits for (router fused into it)
  int copy_split;
  int* status;
  // ep_packed, rows sent from here: a row of an expert whose destination is
  // rank q is stored at row (grouped row - q's first grouped row) of
  // ep_recv[q] (q's receive region for this source, in q's memory) instead
  // of into `grouped`; ep_dest[e] is expert e's destination rank, and no row
  // may land at or past ep_region.  Off when ep_recv[0] is null.
  __nv_bfloat16* ep_recv[kEpMaxRanks];
  signed char ep_dest[kMaxExperts];
  int ep_region;
};

struct CombineArgs {
  const __nv_bfloat16* contrib;   // [2T, d] weighted routed outputs, token-major
  const __nv_bfloat16* shared_y;  // [T, d]
  const __nv_bfloat16* residual;  // [T, d] or null
  __nv_bfloat16* out;             // [T, d]
  int tokens, dim;
};

// Expert-parallel combine: the routed outputs come back in grouped-row order
// (unweighted, bf16); each token gathers its two rows through positions.
struct EpCombineArgs {
  const __nv_bfloat16* y;         // [rows, d] expert outputs in grouped-row order
  const int* indices;             // [T, 2]
  const float* weights;           // [T, 2]
  const int* positions;           // [2T] grouped row of each assignment
  const __nv_bfloat16* shared_y;  // [T, d]
  const __nv_bfloat16* residual;  // [T, d] or null
  __nv_bfloat16* out;             // [T, d]
  int tokens, dim, rows;
  int* status;
  // peer exchange only (else null / 0): wait for return flags [wait_ranks]
  // to reach *wait_epoch first, at most wait_ns, errors into wait_status
  const unsigned* wait_flags;
  const unsigned* wait_epoch;
  int* wait_status;
  int wait_ranks;
  unsigned long long wait_ns;
};

// ---- greedy next token (vocab.cu) -------------------------------------------
constexpr int kVocabMaxGrid = 1024;

struct VocabArgmaxArgs {
  const void* hidden;     // [rows, dim] bf16
  const void* weight;     // [vocab, dim] bf16 (tied embedding)
  int rows, dim, vocab;
  float* partial_value;   // [grid, 8] per-CTA best logit per token
  int* partial_index;     // [grid, 8] and its vocabulary row
  unsigned* counter;      // last-CTA counter, zero between calls
  long long* out;         // [rows] token ids
};

struct ArgmaxRowsArgs {
  const void* logits;     // [rows, cols] bf16
  int rows, cols;
  long long* out;
};

// ---- expert-parallel exchange over peer memory (ep_peer.cu) ----------------
constexpr int kEpMetaStride = kMaxExperts + 1;  // per source: counts [El], then its row base

struct EpSendArgs {
  const __nv_bfloat16* rows;  // [2T, d] dispatched rows, packed destination-major
  const int* counts;          // [E] rows per global expert
  // plan[q][j]: the global expert of rank q's slot j whose rows this rank
  // sends there, -1 for none; the packing order of `rows` follows it
  signed char plan[kEpMaxRanks][kMaxExperts];
  int tokens, dim, n_experts, ranks, rank, max_tokens;
  char* peers[kEpMaxRanks];   // every rank's EP buffer, mapped in this process
  size_t off_recv, off_meta, off_flags_in;
  unsigned* epoch;            // this rank's send count (own buffer)
  unsigned* counter;          // last-CTA counter (own buffer)
  int* status;                // own buffer's status word
  int rows_sent;              // 1: the grouping kernel stored the rows; counts and flags only
};

struct EpReceiveArgs {
  const unsigned* flags_in;   // [G] arrival flag of each source (own buffer)
  const int* meta;            // [G, kEpMetaStride] counts + row base of each source
  const unsigned* epoch;
  int ranks, slots, max_tokens;  // slots: this rank's local experts
  int* seg_rows;              // [ranks * slots] one segment per (source, slot)
  int* seg_base;
  int* seg_expert;
  int* back_n;                // [G] rows received from each source
  int* back_base;             // [G] where they go back in the source's order
  unsigned long long wait_ns;
  int* status;
};

struct EpReturnArgs {
  const __nv_bfloat16* y;     // [G * 2 * max_tokens, d] expert outputs
  const int* back_n;
  const int* back_base;
  char* peers[kEpMaxRanks];
  size_t off_back, off_flags_back;
  int ranks, rank, dim, max_tokens;
  const unsigned* epoch;
  unsigned* counter;
  int rows_sent;              // 1: the expert GEMM stored the outputs; flags only
};

enum GemmMode : int { kGemmSwiGLU = 0, kGemmPlain = 1 };

struct GemmArgs {
  // routed part: n_seg segments of contiguous rows, each multiplied by one
  // expert's weights (capacity layout: 2E segments, capacity then overflow)
  const int* seg_rows;
  const int* seg_base;
  const int* seg_expert;  // [n_seg] expert of each segment, or null: segment s is expert s % E
  int n_seg;
  int static_routed;      // 1: segment e < E is expert e's first segment; its first token
                          // tile is a "primary" unit pinned to CTA e * MT + mt, whose
                          // weights are pulled into L2 before the grid dependency
  const void* w_routed;   // the routed weights (tiled), for that L2 prefetch, or null
  int n_experts;
  int m_tiles_routed;     // output features / 128
  int k_blocks_routed;    // K / 64
  __nv_bfloat16* out_routed;
  int ld_out_routed;      // elements per output row
  // plain mode, routed units: when set, grouped row r is written scaled by
  // bf16(row_w[r]) to out_routed row row_dst[r] instead of row r
  const int* row_dst;
  const float* row_w;
  // shared part
  int shared_rows;        // tokens (0 disables)
  int m_tiles_shared;
  int k_blocks_shared;
  __nv_bfloat16* out_shared;
  int ld_out_shared;
  int mode;
  int* status;
  // slot mode (the depth mix did the grouping): segment s has g.seg_rows[s]
  // rows from row s * seg_stride (0: g.seg_base)
  int seg_stride;
  // slot mode, down GEMM: every CTA takes a ticket once it has read the
  // counters; the last zeroes them for the next block (null: off)
  int* slot_counts;
  int* slot_ticket;
  // slot mode, down GEMM, CTA grid - 1: the counts, statistics and
  // positions copy the grouping kernel would have written (null: off)
  struct SlotStats {
    const float* tile_probsum;  // [route_tiles, E]
    int route_tiles, tokens;
    int* counts;                // [E] workspace copy
    int* counts_out;            // or null
    float* stats;               // [E + 1]
    float* stats_out;           // or null
    const int* positions;       // [2T]
    int* positions_out;         // or null
  } st;
  // expert parallelism, plain mode, rows sent back from here: segment s
  // holds rows of source q = s / out_peer_segs (rows [q * out_peer_region,
  // ...) of the receive regions); its row r is stored to row
  // r - q * out_peer_region + out_peer_base[q] of out_peer[q] (the source's
  // return region, in its memory) instead of out_routed.  Off when 0.
  int out_peer_segs;
  int out_peer_region;
  const int* out_peer_base;   // [ranks] device table (the receive kernel's back_base)
  __nv_bfloat16* out_peer[kEpMaxRanks];
};

// The MoE block at decode batch sizes (moe_decode.cu).
constexpr int kDecodeMoeMaxTokens = 16;
struct MoeDecodeArgs {
  const __nv_bfloat16* x;            // [T, d]
  const __nv_bfloat16* router;       // [E, d]
  const float* router_bias;          // [E] or null
  const __nv_bfloat16* gate_up;      // tiled packs (the grouped GEMM's)
  const __nv_bfloat16* down;
  const __nv_bfloat16* shared_gate_up;
  const __nv_bfloat16* shared_down;
  __nv_bfloat16* hidden;             // [T, 3, H] scratch: routed k = 0, 1, shared
  int* indices;                      // [T, 2]
  float* weights;                    // [T, 2]
  float* probs;                      // [T, E] or null
  long long* indices64;              // [T, 2] or null
  float* weights_out;                // [T, 2] or null
  const __nv_bfloat16* residual;     // [T, d] or null
  __nv_bfloat16* out;                // [T, d]
  int tokens, dim, n_experts, expert_dim, shared_dim;
  // 1: the routing depth mix (two launches before the down projection) wrote
  // indices and weights; the gate/up CTAs read them instead of routing, and
  // the down CTAs fetch their expert rows before their dependency wait
  int routed;
};
int launch_moe_decode(const MoeDecodeArgs& args, cudaStream_t stream);

// Single-token decode attention (decode.cu).
struct DecodeAttnArgs {
  const void* q;                 // [B, H, D] bf16, or fp32 when q_f32
  int q_f32;
  const __nv_bfloat16* k_new;    // [B, KVH, D] this step's key (RoPE applied)
  const __nv_bfloat16* v_new;    // [B, KVH, D], or null when the values are the keys
  __nv_bfloat16* k_cache;        // [B, KVH, S, D]
  __nv_bfloat16* v_cache;        // [B, KVH, S, D], or null (values = keys)
  const int* pos;                // device: position of this step's token
  float* part;                   // [B, H, slots, D + 2] partials (scratch)
  int* counters;                 // [B, KVH] arrivals per group, zero between launches
  const __nv_bfloat16* cos_t;    // [>= S, D / 2] RoPE tables, or null: q and k_new are
  const __nv_bfloat16* sin_t;    // then rotated in the kernel (bf16 q only)
  void* out;                     // [B, H, D] bf16, or fp32 when out_f32
  int out_f32;
  int B, H, KVH, S, D, window, slots;
  long long q_row, kv_row;       // elements between batch rows of q / of k_new and v_new
  float scale;
  int* status;
};
int launch_decode_attention(const DecodeAttnArgs& args, cudaStream_t stream);
int decode_attn_chunks(int max_positions);
int decode_attn_slots(int batch, int max_positions);

// Decode-step projections, at most 8 token rows (linear_small.cu).
constexpr int kLinearSmallMaxK = 1024;
struct LinearSmallArgs {
  const void* x;   // [rows, k_in] bf16, or fp32 when x_f32
  int x_f32;
  const void* w;   // [n_out, k_in] bf16, or fp32 when w_f32
  int w_f32;
  void* y;         // [rows, n_out] bf16, or fp32 when y_f32
  int y_f32;
  int rows, n_out, k_in;
};
int launch_linear_small(const LinearSmallArgs& args, cudaStream_t stream);

int launch_rmsnorm(__nv_bfloat16* out, const __nv_bfloat16* x, const __nv_bfloat16* w,
                   int rows, int dim, float eps, cudaStream_t stream);
int launch_depthmix(const DepthMixArgs& args, cudaStream_t stream);
int launch_rope(__nv_bfloat16* x, const __nv_bfloat16* cos_t, const __nv_bfloat16* sin_t,
                int rows, int row_stride, int rot_cols, int head_dim, int seq_len, int start,
                const int* start_dev, int max_positions, int* status, cudaStream_t stream);
// x_map: [T, d] bf16, box 128 rows x 64; w_map: [E, d] bf16, box
// route_experts_padded(E) rows x 64 (rows past E read as zero).
// Up to 4096 tokens the router reads x [T, d] and the router weight [E, d]
// directly (x_map / w_map unused); above, through the tensor maps.
int launch_depthmix_route(const DepthMixArgs& args, const DepthRouteArgs& route,
                          cudaStream_t stream);
int launch_route(const RouteArgs& args, const void* x, const void* router_w,
                 const CUtensorMap* x_map, const CUtensorMap* w_map, cudaStream_t stream);
int launch_group(const GroupArgs& args, cudaStream_t stream);
int launch_combine(const CombineArgs& args, cudaStream_t stream);
int launch_ep_combine(const EpCombineArgs& args, cudaStream_t stream);
int launch_ep_send(const EpSendArgs& args, int sms, cudaStream_t stream);
int launch_vocab_argmax(const VocabArgmaxArgs& args, int sms, cudaStream_t stream);
int launch_argmax_rows(const ArgmaxRowsArgs& args, cudaStream_t stream);
int launch_ep_receive(const EpReceiveArgs& args, cudaStream_t stream);
int launch_ep_return(const EpReturnArgs& args, int sms, cudaStream_t stream);

// selftest.cu: a bounded mbarrier wait on a barrier nobody arrives at.
// out[0..3] = the status word it writes, out[4] = the wait's result (0: gave
// up), out[5] = the abort flag, out[6] = microseconds waited.
constexpr int kSelftestSite = 90;
int launch_mbar_timeout_selftest(unsigned long long limit_ns, int* out, cudaStream_t stream);
int launch_grouped_gemm(const GemmArgs& args, const CUtensorMap* tm_w_routed,
                        const CUtensorMap* tm_x_routed, const CUtensorMap* tm_w_shared,
                        const CUtensorMap* tm_x_shared, int grid, int token_tile,
                        cudaStream_t stream);
// Row of the packed gate/up matrix holding gate (is_up = 0) or up (is_up = 1)
// of feature f: each 128-row tile carries 64 features as 8 groups of 16 rows,
// the group's 8 gate rows followed by the same 8 features' up rows, so one
// 16-lane TMEM fragment holds gate and up of a feature in the same thread.
__host__ __device__ constexpr int packed_gate_up_row(int f, int is_up) {
  return (f >> 6) * 128 + ((f & 63) >> 3) * 16 + (f & 7) + 8 * is_up;
}

int launch_pack_gate_up(__nv_bfloat16* dst, const __nv_bfloat16* gate, const __nv_bfloat16* up,
                        int n_mats, int hidden, int dim, cudaStream_t stream);
int launch_pack_tiles(__nv_bfloat16* dst, const __nv_bfloat16* src, int n_mats, int rows,
                      int cols, cudaStream_t stream);
int launch_silu_bf16(const uint16_t* x, uint16_t* y, int n, cudaStream_t stream);


// Tokens per router CTA: 32 while the batch is small (more CTAs share the
// load of x), 128 (the MMA's M) once it is large (fewer histogram rows for
// the grouping kernel to sum).  The MMA always has M = 128; a 32-token tile
// leaves the other accumulator lanes unused.
// Tokens per router CTA: 4 up to 4096 tokens (CUDA-core router, or the
// router folded into the depth mix), else 128 (tensor-core router).
constexpr int kRouteSmallTile = 4;
__host__ __device__ inline int route_tile(int tokens) {
  return tokens <= 4096 ? kRouteSmallTile : 128;
}
__host__ __device__ inline int route_blocks(int tokens) {
  const int r = route_tile(tokens);
  return (tokens + r - 1) / r;
}
__host__ __device__ inline int route_experts_padded(int n_experts) {
  return n_experts <= 16 ? 16 : 32;
}
__host__ __device__ inline int group_blocks(int tokens) {
  return (tokens + kGroupTokensPerBlock - 1) / kGroupTokensPerBlock;
}

}  // namespace parrot
