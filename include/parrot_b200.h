/*
 * parrot_b200.h — C ABI of libparrot_b200.so, the B200 (sm_100a) kernels for
 * Parrot XL's MoE block and its companions (bf16 inference forward).
 *
 * Conventions
 *   - Every tensor argument is a DEVICE pointer to a contiguous row-major
 *     array, 16-byte aligned; bf16 unless the type says otherwise.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls only
 *     enqueue work: they never synchronise and never allocate device memory.
 *   - Return value: 0 on success, PARROT_EINVAL for a bad argument (nothing
 *     launched), PARROT_ECUDA when a launch failed.  parrot_b200_last_error()
 *     gives a message for the calling thread.  Device-side errors (a bounded
 *     wait that ran out, an out-of-range expert id) are recorded in the
 *     workspace status word; parrot_moe_read_status() reads it.
 *
 * Each entry point names the reference code it replaces
 * (jkpdino/parrot-h200-worker, paths relative to the repository root).
 */
#ifndef PARROT_B200_H
#define PARROT_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PARROT_OK 0
#define PARROT_EINVAL (-1)
#define PARROT_ECUDA (-2)
#define PARROT_EUNSUPPORTED (-3)

/* Version of this ABI (major * 100 + minor). */
int parrot_b200_version(void);

/* Message describing the last failed call on this thread ("" if none). */
const char* parrot_b200_last_error(void);

/* 1 if `device` is an sm_100 GPU these kernels run on, else 0. */
int parrot_b200_device_supported(int device);

/* ------------------------------------------------------------------------
 * RMSNorm, y = bf16((x * rsqrt(mean(x^2) + eps)) * weight) over the last dim.
 * Replaces parrot/model.py:116-127 (RMSNorm.forward) and the Metal kernels
 * parrot/kernels/moe_bf16.metal:4-65 (rms_norm_bf16, rms_norm_decode_bf16)
 * bound in parrot/metal_moe.py:37-55 (metal_rms_norm).
 * x, out: [rows, dim]; weight: [dim].  dim % 8 == 0, dim <= 2048.
 * ---------------------------------------------------------------------- */
int parrot_rmsnorm_bf16(void* out, const void* x, const void* weight, int rows, int dim,
                        float eps, void* stream);

/* ------------------------------------------------------------------------
 * Block AttnRes depth mix over `n_sources` [rows, dim] tensors (1..16):
 *   key_i = rms_norm(src_i; key_norm_weight, key_eps), s_i = <key_i, query>,
 *   a = softmax_i(s), h = sum_i a_i * src_i,
 * then, when out_norm_weight != NULL, the consumer RMSNorm of h.
 * Replaces parrot/model.py:141-155 (DepthMix.forward) and :157-164
 * (DepthMix.normalized -> output_norm(depth_mix(...))), and the Metal kernels
 * moe_bf16.metal:249-435, 563-645 bound in metal_moe.py:419-477.
 * mix_out (optional) receives h when a norm is fused.
 * pending_base/pending_delta (optional, both or neither): the last source is
 * bf16(pending_base + pending_delta) — the residual add of model.py:702 —
 * and is also written to pending_out (cf. metal_moe.py:480-500).
 * dim % 8 == 0, dim <= 1024.
 * ---------------------------------------------------------------------- */
int parrot_depthmix_bf16(void* out, const void* const* sources, int n_sources,
                         const void* query, const void* key_norm_weight, float key_eps,
                         const void* out_norm_weight, float out_eps, void* mix_out,
                         const void* pending_base, const void* pending_delta,
                         void* pending_out, int rows, int dim, void* stream);

/* parrot_depthmix_bf16 whose last source is a deferred MoE block output:
 *   bf16(pending_base + bf16(bf16(shared + contrib[2t]) + contrib[2t + 1]))
 * (pending_base optional: without it, no residual add), the combine and
 * residual add of model.py:546-551 / :702 with the same roundings as
 * parrot_moe_forward_bf16, also written to pending_out.  pending_shared:
 * [rows, dim]; pending_contrib: [2 rows, dim] (parrot_moe_forward_deferred_bf16's
 * workspace regions); sources[n_sources - 1] is not read. */
int parrot_depthmix_moe_bf16(void* out, const void* const* sources, int n_sources,
                             const void* query, const void* key_norm_weight, float key_eps,
                             const void* out_norm_weight, float out_eps, void* mix_out,
                             const void* pending_base, const void* pending_shared,
                             const void* pending_contrib, void* pending_out, int rows, int dim,
                             void* stream);

/* ------------------------------------------------------------------------
 * Rotary position embedding, in place, for the packed q/k/v projection of
 * local attention.  Replaces parrot/model.py:206-216 (LocalGQA._rope) applied
 * to q and k in :218-230 / :232-262.  x: [rows, row_stride] bf16, rows in
 * (batch, position) order with seq_len positions per batch row, position of
 * row r = start + r % seq_len.  The first rot_cols columns (the q and k heads,
 * rot_cols = (n_heads + n_kv_heads) * head_dim) are rotated as heads of
 * head_dim interleaved (even, odd) pairs; the bf16 products and sums are
 * rounded exactly as the reference's bf16 expression.  cos/sin tables:
 * [max_positions, head_dim / 2] bf16.  head_dim % 8 == 0.
 * Outside the MoE block: part of the forward this library accelerates.
 * ---------------------------------------------------------------------- */
int parrot_rope_inplace_bf16(void* x, const void* cos_table, const void* sin_table, int rows,
                             int row_stride, int rot_cols, int head_dim, int seq_len, int start,
                             int max_positions, void* stream);

/* As parrot_rope_inplace_bf16 with the first position read from device
 * memory (*start_dev), so a decode step captured in a CUDA graph can be
 * replayed at successive positions.  A position at or past max_positions is
 * recorded in status (device int[4], may be NULL) and that row left as is.
 * Replaces the position-dependent RoPE of parrot/model.py:218-230 in decode. */
int parrot_rope_inplace_at_bf16(void* x, const void* cos_table, const void* sin_table, int rows,
                                int row_stride, int rot_cols, int head_dim, int seq_len,
                                const int* start_dev, int max_positions, int* status,
                                void* stream);

/* ------------------------------------------------------------------------
 * Single-token decode attention with the position in device memory.
 * Appends this step's key/value at *pos_dev to the cache, then attends each
 * query head over the keys [max(0, pos - window + 1), pos] of its KV head
 * (window 0 = no window): softmax(scale * q.k) weighted sum of the values,
 * fp32 math.
 *   local GQA (parrot/model.py:303-328, window 2048): q [B, H, D] bf16
 *     (q_f32 = 0), k_new/v_new [B, KVH, D] bf16, k_cache/v_cache
 *     [B, KVH, max_positions, D] bf16, out [B, H, D] bf16;
 *   MLA absorbed (parrot/model.py:399-432): q [B, H, L] fp32 (q_f32 = 1),
 *     k_new = the new latent [B, 1, L], v_new = v_cache = NULL (values are
 *     the keys), k_cache = the latent cache [B, 1, max_positions, L],
 *     out [B, H, L] fp32 (out_f32 = 1), scale = head_dim^-0.5.
 * Supported (D, H / KVH): (96, 4), (96, 1), (128, 8), (32, 2), (32, 4).
 * q_row_stride / kv_row_stride: elements between batch rows of q and of
 * k_new / v_new (0 = packed), so q, k and v can be views of one projection.
 * partials: parrot_decode_attention_scratch_bytes() of scratch, zero-filled
 * before its first use (it ends every call zero-filled where that matters: the
 * per-group arrival counters after the partials); calls that share it must be
 * ordered on one stream.  A position outside [0, max_positions) is recorded in
 * status and nothing is written. */
int parrot_decode_attention_bf16(void* out, int out_f32, const void* q, int q_f32,
                                 long long q_row_stride, const void* k_new, const void* v_new,
                                 long long kv_row_stride, void* k_cache, void* v_cache,
                                 const int* pos_dev, int batch, int n_heads, int n_kv_heads,
                                 int max_positions, int head_dim, int window, float scale,
                                 void* partials, size_t partial_bytes, int* status,
                                 void* stream);

/* parrot_decode_attention_bf16 for the local GQA layers with the rotary
 * embedding applied inside (replaces parrot_rope_inplace_at_bf16 on the q and
 * k heads followed by parrot_decode_attention_bf16; model.py:206-216 then
 * :303-328): q is bf16 and read unrotated, the query is rotated as it is
 * loaded and the new key as it is appended, with the same bf16 rounding, so
 * outputs and cache rows are bit-identical to the two calls.  cos_table /
 * sin_table: bf16 [rope_positions, head_dim / 2], rope_positions >=
 * max_positions.  k_new / v_new in memory stay unrotated. */
int parrot_decode_attention_rope_bf16(void* out, int out_f32, const void* q,
                                      long long q_row_stride, const void* k_new,
                                      const void* v_new, long long kv_row_stride, void* k_cache,
                                      void* v_cache, const int* pos_dev, int batch, int n_heads,
                                      int n_kv_heads, int max_positions, int head_dim,
                                      int window, float scale, const void* cos_table,
                                      const void* sin_table, int rope_positions,
                                      void* partials, size_t partial_bytes, int* status,
                                      void* stream);

/* y[t, n] = sum_k x[t, k] w[n, k] for a decode step's projections
 * (model.py:303-328 q/k/v and out, 399-432 the latent down-projection and the
 * absorbed query / output), replacing F.linear there: fp32 accumulation and one
 * rounding of the result to y's type.  rows <= 8, n_out % 16 == 0, k_in % 8
 * == 0 and <= 1024; x [rows, k_in] and w [n_out, k_in] (nn.Linear layout)
 * contiguous and 16-byte aligned, each bf16 or fp32 (the *_f32 flags); y
 * [rows, n_out].  The weights are read before the kernel's grid dependency
 * wait, so they must not be written by the kernel launched just before. */
int parrot_linear_small(void* y, int y_f32, const void* x, int x_f32, const void* w, int w_f32,
                        int rows, int n_out, int k_in, void* stream);

/* Scratch bytes parrot_decode_attention_bf16 needs for these sizes. */
size_t parrot_decode_attention_scratch_bytes(int batch, int n_heads, int max_positions,
                                             int head_dim);

/* ------------------------------------------------------------------------
 * MoE block: router + top-2 + capacity grouping + grouped SwiGLU experts +
 * shared expert + weighted combine (+ residual add).
 * ---------------------------------------------------------------------- */
typedef struct parrot_moe_dims {
  int tokens;      /* T, flattened tokens (0 allowed) */
  int dim;         /* d, % 128 == 0, <= 1024 */
  int n_experts;   /* E, 2..32 */
  int top_k;       /* must be 2 */
  int expert_dim;  /* H, % 64 == 0 */
  int shared_dim;  /* Hs, % 64 == 0 */
  int capacity;    /* slots per expert; 0 selects parrot_moe_capacity();
                      -1 packs all rows per expert, experts in id order (no capacity
                      region: the expert-parallel send layout); -2 slot mode: a
                      region of 2T rows per expert that the router fills itself,
                      see parrot_depthmix_route_bf16 */
} parrot_moe_dims;

/* Expert weights start in torch.nn.Linear [out, in] layout and are packed
 * once into the tiled layout the GEMMs stream: gate_up / shared_gate_up by
 * parrot_pack_gate_up_bf16, down / shared_down by parrot_pack_down_bf16. */
typedef struct parrot_moe_weights {
  const void* router;          /* [E, d], nn.Linear layout */
  const float* router_bias;    /* [E] fp32 logit offset or NULL (harness only) */
  const void* gate_up;         /* E * 2H * d elements, parrot_pack_gate_up_bf16 */
  const void* down;            /* E * d * H elements, parrot_pack_down_bf16 */
  const void* shared_gate_up;  /* 2Hs * d elements, parrot_pack_gate_up_bf16 */
  const void* shared_down;     /* d * Hs elements, parrot_pack_down_bf16 */
} parrot_moe_weights;

typedef struct parrot_moe_outputs {
  void* out;              /* [T, d] bf16, required */
  const void* residual;   /* [T, d] or NULL: out = bf16(residual + moe(x)) */
  float* probs;           /* [T, E] router softmax, or NULL */
  long long* indices;     /* [T, 2] int64 expert ids, or NULL */
  float* weights;         /* [T, 2] renormalised top-2 weights, or NULL */
  int* positions;         /* [2T] grouped row of each assignment, or NULL */
  int* counts;            /* [E] assignments per expert, or NULL */
  float* stats;           /* [E + 1]: utilisation[E], aux loss; or NULL */
} parrot_moe_outputs;

/* Byte offsets of the buffers inside one MoE workspace (for inspection). */
typedef struct parrot_moe_layout {
  size_t indices, weights, positions;
  size_t chunk_hist;      /* [ceil(T/32), E] int32 expert histogram per 32-token chunk */
  size_t tile_hist;       /* [route_blocks, E] int32 per router tile (32 tokens up to
                             T = 4096, else 128) */
  size_t tile_probsum;    /* [route_blocks, E] f32 router probability sums per tile */
  size_t counts, seg_rows, seg_base, stats, status;
  size_t row_dst, row_w;  /* per grouped row: token-major slot, route weight */
  size_t grouped;         /* [E*C + 2T, d] token rows grouped by expert */
  size_t hidden;          /* [E*C + 2T, H] SwiGLU hidden, same row order */
  size_t contrib;         /* [2T, d] bf16(bf16(y) * bf16(w)), slot 2t + (lower expert id first) */
  size_t shared_hidden, shared_y, total;
  int capacity, grouped_rows;
  int route_blocks;       /* router CTAs: ceil(T / 32) up to T = 4096, else ceil(T / 128) */
  int reserved;
} parrot_moe_layout;

/* Default capacity: max(8, ceil8(ceil(2 * 2T / E))), metal_moe.py:388-391. */
int parrot_moe_capacity(int tokens, int n_experts);

/* Fills `layout`; returns PARROT_EINVAL for unsupported dims. */
int parrot_moe_workspace_layout(const parrot_moe_dims* dims, parrot_moe_layout* layout);

/* Zeroes the status word of a fresh workspace (call once after allocating;
 * a zero-filled allocation needs no call).  Enqueued on `stream`. */
int parrot_moe_workspace_init(void* workspace, const parrot_moe_dims* dims, void* stream);

/* Pack gate/up for the fused SwiGLU GEMM.  Logical packed row p of matrix m
 * is gate (p % 16 < 8) or up of feature (p / 128) * 64 + (p % 128) / 16 * 8 +
 * p % 8 (within each 16-row group: 8 gate rows, then the same features' up);
 * rows are stored as 128-row x 64-column tiles, each a contiguous 16 KB block,
 * ordered (m, row tile, column slab).  gate, up: [n_mats, hidden, dim];
 * dst: n_mats * 2 * hidden * dim elements; hidden % 64 == 0, dim % 64 == 0.
 * Replaces the weight packing of metal_moe.py:105-131 (pack_combined_weights). */
int parrot_pack_gate_up_bf16(void* dst, const void* gate, const void* up, int n_mats, int hidden,
                             int dim, void* stream);

/* Elementwise bf16 SiLU exactly as the SwiGLU epilogue of the expert GEMMs
 * evaluates it: y = bf16(x / (1 + expf(-x))) in fp32, the value PyTorch's
 * F.silu gives for a bf16 tensor (parrot/model.py:448 and :460,
 * Expert.forward / SharedExpert.forward).  x, y: n bf16 values.  The epilogue
 * takes a fast path for almost every input and reads a 65,536-entry table for
 * the rest; this entry runs the same code so it can be checked exhaustively. */
int parrot_silu_bf16(const void* x, void* y, int64_t n, void* stream);

/* Pack [n_mats, rows, cols] (down projections, [d, H]) into the same tiled
 * layout: 128 x 64 tiles ordered (m, row tile, column slab).
 * rows % 128 == 0, cols % 64 == 0.  Replaces metal_moe.py:97-99 (torch.stack of
 * the expert down weights). */
int parrot_pack_down_bf16(void* dst, const void* src, int n_mats, int rows, int cols,
                          void* stream);

/* Whole MoE block.  Replaces parrot/model.py:505-569 (MoE.forward: router
 * :521-527, per-expert dispatch loop :545-551, router statistics :554-569)
 * and :571-585 (MoE.inference with addend), plus the Metal route/group/
 * gather path metal_moe.py:58-81, 372-416 (moe_bf16.metal:67-134, 650-777).
 * x: [T, d].  `workspace` holds parrot_moe_workspace_layout(dims).total bytes. */
int parrot_moe_forward_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                            const void* x, const parrot_moe_outputs* outputs, void* workspace,
                            size_t workspace_bytes, void* stream);

/* The MoE block without its final combine: route, grouping and both expert
 * GEMMs, leaving the weighted routed contributions at layout.contrib
 * ([2T, d], token-major, row 2t + j the token's j-th lowest expert id) and the
 * shared expert output at layout.shared_y ([T, d]) in `workspace`;
 * outputs->out is not used (may be NULL).  The caller finishes the block with
 * parrot_depthmix_moe_bf16 — the combine of model.py:546-551 (+ the residual
 * add of :702) folded into the next Block AttnRes depth mix — before the
 * workspace is used again. */
int parrot_moe_forward_deferred_bf16(const parrot_moe_dims* dims,
                                     const parrot_moe_weights* weights, const void* x,
                                     const parrot_moe_outputs* outputs, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* parrot_depthmix_bf16 (with its optional pending residual) whose normalised
 * output is the input of an MoE block, with that block's router folded in:
 * besides the depth mix it computes the router logits, softmax, top-2 and
 * renormalised weights of every output row (model.py:521-527, the router of
 * parrot_moe_forward_bf16) into `workspace` (the block's workspace for
 * `dims`), plus outputs->probs / indices / weights when non-NULL.
 * rows == dims->tokens <= 4096; out_norm_weight required.  The block then
 * runs from its grouping on with parrot_moe_forward_routed_bf16.  One launch
 * instead of a depth mix and a router launch.  The logits' summation order
 * differs from the router kernel's: expert ids follow this call's own
 * probabilities.
 * Slot mode, when dims->capacity == -2 (every expert a region of 2T rows,
 * which it cannot overflow): this call also does the grouping.  Each assignment
 * takes the next slot of its expert from a per-expert counter kept in the
 * workspace's zeroed status region, and its row, position, contribution slot
 * and route weight are written there and then; the group kernel does not
 * run.  Rows of one expert are in no particular order within its region
 * (positions say where each went; the block output does not depend on it).
 * The call must be followed by parrot_moe_forward_routed_bf16 on the same
 * workspace, which reads the counters and leaves them zero.  Counters left
 * set by a routing call whose block never ran are caught: a slot past the
 * expert's region is reported in the status word (PARROT code 2) and nothing
 * is written there; parrot_moe_workspace_init zeroes the counters again. */
int parrot_depthmix_route_bf16(void* out, const void* const* sources, int n_sources,
                               const void* query, const void* key_norm_weight, float key_eps,
                               const void* out_norm_weight, float out_eps, void* mix_out,
                               const void* pending_base, const void* pending_delta,
                               void* pending_out, int rows, int dim,
                               const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                               const parrot_moe_outputs* outputs, void* workspace,
                               size_t workspace_bytes, void* stream);

/* The MoE block after parrot_depthmix_route_bf16 routed its input x:
 * grouping, experts and (deferred == 0) the combine, as
 * parrot_moe_forward_bf16 / (deferred != 0) parrot_moe_forward_deferred_bf16
 * from their grouping on.  outputs->probs / indices / weights must be NULL
 * (the routing call writes them).  In slot mode (above) the grouping was done
 * by the routing call: the GEMMs take the expert counters as their segments,
 * the down projection writes counts, statistics and positions and zeroes the
 * counters.  parrot_moe_forward_bf16 / _deferred_bf16 / _static_bf16 with
 * dims->capacity == -2 run slot mode with their own router kernel (no group
 * kernel; positions in no particular order within an expert). */
int parrot_moe_forward_routed_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                   const void* x, const parrot_moe_outputs* outputs, int deferred,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* Whole MoE block without a caller-provided workspace, for callers that
 * cannot allocate device memory at the point of the call (a runtime that owns
 * all device memory and forbids allocation on its hot path, or code that must
 * not enter an allocator).  Same computation and arguments as
 * parrot_moe_forward_bf16; the workspace is a 4 MiB array compiled into this
 * library, one per device that loads it, kept until the process exits —
 * enough for Parrot XL widths (d 768, 16 experts of 512, shared 256) up to 192
 * tokens.  Dims whose workspace (parrot_moe_workspace_layout) exceeds 4 MiB are
 * rejected with PARROT_EINVAL.  It calls no allocator.  The first call on a
 * device looks up the array's device address (and, like any first MoE call,
 * builds the SiLU table there); make it before any stream capture.  The
 * address is cached with the id of the CUDA context it was found in; a call
 * made in another context (after cudaDeviceReset, or under a caller's own
 * context) looks it up again, so that call is a first call too.  All calls
 * share the one array: calls whose GPU work overlaps (other streams, other
 * threads) race and must be serialised by the caller.
 * No counterpart in the reference. */
int parrot_moe_forward_static_bf16(const parrot_moe_dims* dims,
                                   const parrot_moe_weights* weights, const void* x,
                                   const parrot_moe_outputs* outputs, void* stream);

/* Router + grouping only (metal_moe.py:58-81 metal_route, plus the slot
 * scatter of moe_bf16.metal:678-696).  Leaves its results in the workspace
 * and copies the optional outputs (probs, indices, weights, positions,
 * counts, stats). */
int parrot_moe_route_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                          const void* x, const parrot_moe_outputs* outputs, void* workspace,
                          size_t workspace_bytes, void* stream);

/* The whole MoE block at decode batch sizes (tokens <= 16), in two kernels:
 * every CTA routes all tokens, then computes 32 SwiGLU features of one
 * expert for the tokens routed to it (the shared expert for all); a second
 * kernel takes (token, 16 output columns) and produces the two routed down
 * rows, the shared one and their combine (+ residual) exactly as
 * parrot_moe_forward_bf16 rounds them.  Same arguments as
 * parrot_moe_forward_bf16; outputs->positions / counts / stats must be NULL.
 * Replaces model.py:571-585 (MoE.inference) at decode, and the Metal decode
 * MoE lanes (metal_moe.py:182-221, moe_bf16.metal:898-1024). */
int parrot_moe_decode_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                           const void* x, const parrot_moe_outputs* outputs, void* workspace,
                           size_t workspace_bytes, void* stream);

/* parrot_moe_decode_bf16 after parrot_depthmix_route_bf16 routed its input x
 * (rows == tokens <= 4 with a non-slot dims->capacity): the gate/up kernel
 * reads the routing from the workspace instead of computing it, and the down
 * kernel fetches its expert rows before its dependency wait (the routing was
 * written two launches earlier).  outputs->probs / indices / weights must be
 * NULL (the routing call writes them). */
int parrot_moe_decode_routed_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                  const void* x, const parrot_moe_outputs* outputs,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Expert GEMMs + shared expert + combine on a workspace filled by
 * parrot_moe_route_bf16 for the same x (metal_moe.py:372-416 after routing). */
int parrot_moe_experts_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                            const void* x, const parrot_moe_outputs* outputs, void* workspace,
                            size_t workspace_bytes, void* stream);

/* One grouped-GEMM stage on a workspace filled by parrot_moe_route_bf16
 * (stage 0: gate_up + SwiGLU for routed and shared experts; stage 1: down).
 * Used to time the tensor-core kernel on its own; the result is the same as
 * the corresponding part of parrot_moe_experts_bf16 (cuda_training.py:26-30,
 * the torch._grouped_mm pair it replaces). */
int parrot_moe_gemm_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                         const void* x, void* workspace, size_t workspace_bytes, int stage,
                         void* stream);

/* Number of kernels this library has enqueued since it was loaded
 * (instrumentation; no reference counterpart). */
unsigned long long parrot_b200_launch_count(void);

/* Copies the workspace status word {code, site, info, 0} to host memory
 * (synchronises `stream`).  code 0 = ok. */
int parrot_moe_read_status(const void* workspace, const parrot_moe_dims* dims, int* host_status4,
                           void* stream);

/* ---- expert parallelism ----------------------------------------------------
 * The reference runs every expert on one device; these four calls split the
 * same computation (model.py:521-551) across ep_ranks devices that each own
 * n_experts / ep_ranks experts, round-robin: expert e lives on rank
 * e % ep_ranks as local expert e / ep_ranks.  The exchange between them (an
 * all-to-all of row counts, of token rows, and back of expert outputs) is the
 * caller's, over NCCL; these calls only touch local memory.  The result equals
 * parrot_moe_forward_bf16 on the same tokens bit for bit.
 *
 * Router + grouping for expert parallelism.  dims->capacity must be -1: the
 * workspace's grouped rows [2T, d] then hold every assignment packed by
 * destination rank, then local expert, then ascending token (the reference's
 * torch.where order, model.py:548).  outputs->counts (optional) receives the
 * per-expert row counts; out/residual are unused. */
int parrot_moe_ep_dispatch_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                                const void* x, const parrot_moe_outputs* outputs, int ep_ranks,
                                void* workspace, size_t workspace_bytes, void* stream);

/* The shared expert (model.py:546, `self.shared(flat)`) on this rank's own
 * tokens, into the workspace; only weights->shared_gate_up/shared_down are read. */
int parrot_moe_shared_ffn_bf16(const parrot_moe_dims* dims, const parrot_moe_weights* weights,
                               const void* x, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Grouped SwiGLU experts over received rows (model.py:443-448 per expert):
 * x [rows, dim] is cut into n_segments contiguous segments (device int arrays
 * seg_rows, seg_base: first row; seg_expert: which of the n_mats packed
 * matrices, parrot_pack_gate_up_bf16 / parrot_pack_down_bf16 layout).
 * hidden [rows, expert_dim] is scratch; y [rows, dim] receives the unweighted
 * expert outputs in the order of x.  status: device int[4], or NULL. */
int parrot_moe_expert_ffn_bf16(int rows, int dim, int expert_dim, int n_mats, int n_segments,
                               const int* seg_rows, const int* seg_base, const int* seg_expert,
                               const void* gate_up, const void* down, const void* x,
                               void* hidden, void* y, int* status, void* stream);

/* Combine for expert parallelism (model.py:551): y [2T, d] holds the expert
 * outputs returned in the dispatch's grouped-row order; out = shared output +
 * route-weighted outputs in ascending expert order (+ residual when non-NULL).
 * Reads indices, weights, positions and the shared output from the workspace
 * of parrot_moe_ep_dispatch_bf16 / parrot_moe_shared_ffn_bf16. */
int parrot_moe_ep_combine_bf16(const parrot_moe_dims* dims, const void* y, const void* workspace,
                               size_t workspace_bytes, const void* residual, void* out,
                               void* stream);

/* ---- greedy next token -----------------------------------------------------
 * The tied LM-head projection fused with the argmax over the vocabulary:
 *   out[t] = argmax_v bf16(sum_k hidden[t, k] * weight[v, k])   (int64)
 * fp32 accumulation, each logit rounded to bf16 before the comparison (as
 * F.linear on bf16 tensors), the lowest v among equal values (as
 * torch.argmax); the [rows, vocab] logits are never written.  Replaces
 * parrot/model.py:927-931 (decode_next: F.linear(normalized,
 * embedding.weight).argmax(-1)) and the Metal vocab_argmax_partials_bf16 /
 * vocab_argmax_reduce_bf16 kernels (moe_bf16.metal:1541-1621, bound in
 * metal_moe.py:329-353).  hidden [rows, dim], weight [vocab, dim] bf16;
 * rows <= 8, dim % 8 == 0 and <= 1024.  scratch: 256-byte aligned,
 * parrot_vocab_argmax_scratch_bytes() bytes, zero-filled before its first
 * use (the kernel leaves its counter at zero); calls sharing a scratch must
 * be ordered on one stream. */
size_t parrot_vocab_argmax_scratch_bytes(void);
int parrot_vocab_argmax_bf16(long long* out, const void* hidden, const void* weight, int rows,
                             int dim, int vocab, void* scratch, size_t scratch_bytes,
                             void* stream);

/* Row-wise argmax of bf16 logits [rows, cols] into int64 out[rows], lowest
 * column among equal maxima: the argmax(-1) of decode_next (model.py:927-931)
 * when more than 8 token rows make the projection a GEMM.  cols % 8 == 0. */
int parrot_argmax_rows_bf16(long long* out, const void* logits, int rows, int cols, void* stream);

/* ---- expert-parallel exchange over peer memory ----------------------------
 * The same expert-parallel MoE block (model.py:521-551 split over ranks as
 * above) with the exchange done by these kernels instead of NCCL: every rank
 * owns one EP buffer (parrot_ep_buffer_layout; zero-filled once when
 * allocated) that every other rank maps into its address space with
 * parrot_ipc_export / parrot_ipc_import (CUDA IPC, one node, NVLink /
 * NVSwitch).  One call of the block on a rank, all on one stream:
 *   parrot_moe_ep_dispatch_bf16      router + grouping (capacity -1)
 *   parrot_moe_ep_send_bf16          rows + counts into every rank's buffer
 *   parrot_moe_shared_ffn_bf16       shared expert (overlaps the arrivals)
 *   parrot_moe_ep_receive            wait for every source; segment table
 *   parrot_moe_ep_experts_bf16       local experts on the received rows
 *   parrot_moe_ep_return_bf16        outputs back into every source's buffer
 *   parrot_moe_ep_combine_peer_bf16  wait for every return; combine (+ residual)
 * or, with the copies folded into the kernels that produce the rows:
 *   parrot_moe_ep_dispatch_send_bf16   router + grouping storing each row into
 *                                      its destination's receive region; counts
 *   parrot_moe_shared_ffn_bf16, parrot_moe_ep_receive
 *   parrot_moe_ep_experts_return_bf16  local experts, the down GEMM storing each
 *                                      output into its source's return region
 *   parrot_moe_ep_combine_peer_bf16
 * Both sequences leave the same bytes in every buffer the combine reads and
 * may be mixed from call to call.
 * Nothing is read back to the host and every size is fixed by max_tokens, so
 * the sequence can be captured in a CUDA graph.  Every rank must make the
 * same calls in the same order (a rank with no tokens still calls them).
 * Each flag wait is bounded by wait_ns; a wait that runs out records
 * {1 (timeout), site, rank} in the EP buffer's status word
 * (parrot_ep_read_status), counts the missing rank's rows as zero and
 * returns.  No reference counterpart (the reference has no multi-GPU path). */
#define PARROT_EP_MAX_RANKS 8

typedef struct parrot_ep_dims {
  int ranks;        /* G, 1..8 */
  int rank;         /* this process's rank */
  int max_tokens;   /* most tokens any rank passes to one call: sizes the regions */
  int dim;          /* d, as parrot_moe_dims */
  int n_experts;    /* E */
  int expert_dim;   /* H */
  unsigned long long wait_ns;  /* limit of each flag wait; 0 selects 2 s */
  /* Placement.  slots = 0: round-robin, expert e on rank e % G as local slot
   * e / G (G must divide E).  Otherwise this rank holds `slots` experts
   * (ranks * slots <= 64) and plan[q][j] is the global expert of rank q's
   * slot j whose rows THIS rank sends there, or -1: every expert must appear
   * exactly once in this rank's plan.  An expert that every rank holds may be
   * planned to this rank itself (each source computes its own rows of it). */
  int slots;
  signed char plan[PARROT_EP_MAX_RANKS][32];
} parrot_ep_dims;

/* Byte offsets inside one EP buffer. */
typedef struct parrot_ep_layout {
  /* written by the other ranks */
  size_t flags_in;    /* [8] u32 arrival flag of each source */
  size_t flags_back;  /* [8] u32 return flag of each expert rank */
  size_t meta;        /* [8, 33] int32: each source's counts per local expert, then its row base */
  size_t recv_rows;   /* [G, 2 * max_tokens, d] rows received, one region per source */
  size_t back_rows;   /* [2 * max_tokens, d] expert outputs of this rank's rows, dispatch order */
  /* this rank only */
  size_t epoch, counters, status;
  size_t seg_rows, seg_base, seg_expert;  /* [E] segment table of the received rows */
  size_t back_n, back_base;               /* [8] per source: rows received, their base there */
  size_t hidden;      /* [G * 2 * max_tokens, H] */
  size_t y;           /* [G * 2 * max_tokens, d] expert outputs */
  size_t total;
  int region_rows;    /* 2 * max_tokens */
  int reserved;
} parrot_ep_layout;

/* buffers[r]: rank r's EP buffer as mapped in this process (buffers[rank] is
 * this rank's own); entries >= ranks are ignored. */
typedef struct parrot_ep_peers {
  void* buffers[PARROT_EP_MAX_RANKS];
} parrot_ep_peers;

int parrot_ep_buffer_layout(const parrot_ep_dims* ep, parrot_ep_layout* layout);

/* CUDA IPC of a device allocation: `handle` (64 bytes) names the allocation
 * holding `ptr`, `offset` is ptr's offset in it.  parrot_ipc_import maps the
 * allocation into this process (current device) with peer access enabled and
 * returns the pointer plus the mapping's base, which parrot_ipc_close unmaps.
 * Set-up only (outside the per-call path). */
int parrot_ipc_export(const void* ptr, void* handle, unsigned long long* offset);
int parrot_ipc_import(const void* handle, unsigned long long offset, void** ptr, void** base);
int parrot_ipc_close(void* base);

/* Router + grouping for the peer exchange: parrot_moe_ep_dispatch_bf16 with
 * the rows packed in the order of ep's plan (destination rank major, then
 * the destination's slot order, then ascending token). */
int parrot_moe_ep_dispatch_planned_bf16(const parrot_moe_dims* dims,
                                        const parrot_moe_weights* weights, const void* x,
                                        const parrot_moe_outputs* outputs,
                                        const parrot_ep_dims* ep, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* Stores this rank's dispatched rows (workspace of
 * parrot_moe_ep_dispatch_planned_bf16 with the same ep, dims->tokens <=
 * ep->max_tokens) into each destination's receive region for this source,
 * with the per-slot counts and the rows' base in this rank's dispatch order,
 * then raises this rank's arrival flag there. */
int parrot_moe_ep_send_bf16(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                            const parrot_ep_peers* peers, const void* workspace,
                            size_t workspace_bytes, void* stream);

/* parrot_moe_ep_dispatch_planned_bf16 then parrot_moe_ep_send_bf16 without
 * the copy: the grouping kernel stores every dispatched row straight into
 * its destination's receive region (peer memory, 16-byte stores) and fences
 * them at system scope; the send kernel then writes the counts and row base
 * and raises the arrival flags.  The workspace's grouped rows are not
 * written.  dims as parrot_moe_ep_send_bf16 (capacity -1); with no tokens
 * only the counts and flags are sent. */
int parrot_moe_ep_dispatch_send_bf16(const parrot_moe_dims* dims,
                                     const parrot_moe_weights* weights, const void* x,
                                     const parrot_moe_outputs* outputs, const parrot_ep_dims* ep,
                                     const parrot_ep_peers* peers, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Waits for every source's arrival flag, then writes the segment table of the
 * received rows (one segment per (source, local slot)) into the buffer. */
int parrot_moe_ep_receive(const parrot_ep_dims* ep, void* buffer, void* stream);

/* The local experts (packed gate_up / down of this rank's slots, in slot
 * order, parrot_pack_gate_up_bf16 / parrot_pack_down_bf16 layout) on the
 * received rows, by the segment table; outputs into the buffer's y. */
int parrot_moe_ep_experts_bf16(const parrot_ep_dims* ep, void* buffer, const void* gate_up,
                               const void* down, void* stream);

/* Stores each source's expert outputs back into that source's buffer, in its
 * dispatch order, then raises this rank's return flag there. */
int parrot_moe_ep_return_bf16(const parrot_ep_dims* ep, const parrot_ep_peers* peers,
                              void* stream);

/* parrot_moe_ep_experts_bf16 then parrot_moe_ep_return_bf16 without the
 * copy: the down GEMM's epilogue stores each output row straight into its
 * source's return region (peer memory, 16-byte stores, at the row base the
 * source sent) and fences at system scope; a one-block kernel then raises
 * the return flags.  The buffer's y is not written. */
int parrot_moe_ep_experts_return_bf16(const parrot_ep_dims* ep, const parrot_ep_peers* peers,
                                      const void* gate_up, const void* down, void* stream);

/* Waits for every expert rank's return flag, then parrot_moe_ep_combine_bf16
 * on the returned rows (buffer's back_rows). */
int parrot_moe_ep_combine_peer_bf16(const parrot_moe_dims* dims, const parrot_ep_dims* ep,
                                    const void* buffer, const void* workspace,
                                    size_t workspace_bytes, const void* residual, void* out,
                                    void* stream);

/* Copies the EP buffer's status word {code, site, info, 0} to host memory
 * (synchronises `stream`). */
int parrot_ep_read_status(const parrot_ep_dims* ep, const void* buffer, int* host_status4,
                          void* stream);

/* ---- self-test --------------------------------------------------------------
 * The failure path of the kernels' bounded mbarrier waits, without a fault: a
 * one-warp kernel waits on an mbarrier nobody arrives at through the same wait
 * loop the grouped GEMM and the router use, limited to limit_ns (1 us .. 1 s)
 * instead of their 2 s.  device_out8 (8 int32, 16-byte aligned, device memory)
 * receives the status word the wait writes {1 (timeout), 90 (site), 0 (block),
 * 0}, the wait's result (0: it gave up), the CTA abort flag it set (1) and the
 * microseconds it waited.  No reference counterpart. */
int parrot_selftest_wait_timeout(unsigned long long limit_ns, int* device_out8, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PARROT_B200_H */
