/*
 * hier_b200.h - C ABI of libhier_b200.so, the B200 (sm_100a) implementation of
 * Multics' hierarchical group attention.
 *
 * Every entry point takes plain device pointers, element counts/strides and a
 * CUDA stream (as void*), returns a status code (HIER_OK on success) and
 * never allocates device memory itself: callers pass output buffers and, where
 * a kernel needs scratch space, a workspace whose size is given by the
 * matching *_workspace_size call.  On failure the message of the last error
 * of the calling thread is available from hier_last_error().
 *
 * Reference interfaces (TencentARC/Multics, paths relative to the checkout)
 * that each entry point replaces are cited beside it.
 */
#ifndef HIER_B200_H
#define HIER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python host layer maps them onto the exception types the
 * reference raises: VALUE -> ValueError, NOTIMPL -> NotImplementedError,
 * RUNTIME/CUDA -> RuntimeError, ASSERT -> AssertionError. */
#define HIER_OK 0
#define HIER_EVALUE 1
#define HIER_ENOTIMPL 2
#define HIER_ERUNTIME 3
#define HIER_EASSERT 4
#define HIER_ECUDA 5

/* Last error message / code of the calling thread ("" / HIER_OK if none). */
const char* hier_last_error(void);
int hier_last_error_code(void);
/* ABI version, bumped on any signature change. */
int hier_abi_version(void);

/*
 * Grouping description shared by the mask and metadata builders.  Mirrors the
 * tensors normalised by _prepare_hier_group_tensors /
 * _prepare_hier_membership_tensors (multics/models/hier_masks.py:22-71,
 * 127-193).  All pointers are device pointers; the host layer has already
 * validated shapes and ranges with the reference's messages.
 *   labels      int64 [T,P]   (membership_mode == 0)
 *   membership  uint8 [T,N,P] (membership_mode == 1)
 *   global_only uint8 [T,P]   (membership_mode == 1)
 *   active      uint8 [T,N]   (both modes; labels mode: scatter of labels or
 *                              the caller's active_group)
 */
typedef struct hier_grouping {
  int32_t P, T, L, N, KL, KG;
  int32_t n_block;    /* num_frame_per_block */
  int32_t local_attn; /* local_attn_size, -1 = unlimited */
  int32_t direct;     /* direct_player */
  int32_t no_local;   /* hier_no_local_hub */
  int32_t membership_mode;
  const int64_t* labels;
  const uint8_t* membership;
  const uint8_t* global_only;
  const uint8_t* active;
} hier_grouping;

/* ---------------------------------------------------------------------------
 * Masks
 * ------------------------------------------------------------------------- */

/* Dense bool mask rows [row0, row0+nrows) of the [S,S] hierarchical mask into
 * out (uint8 [nrows, S]).  Replaces build_stage2_hier_self_attn_mask
 * (multics/models/hier_masks.py:364-507) and its membership variant
 * (hier_masks.py:510-641).  Bit-exact. */
int hier_dense_mask(const hier_grouping* g, int64_t row0, int64_t nrows, uint8_t* out,
                    void* stream);

/* Workspace bytes for hier_block_mask_build / hier_block_plan_build. */
int hier_block_workspace_size(const hier_grouping* g, size_t* bytes);

/* 128x128 block classification of the mask padded to S_pad = ceil(S/128)*128,
 * with the same partial / full block lists as the Flex BlockMask built by
 * build_stage2_hier_flex_block_mask (hier_masks.py:722-934, membership
 * variant :937-1149): per query block the number of partial blocks and of
 * full blocks, and the CSR-concatenated ascending block indices (offsets are
 * exclusive scans of the counts).  Outputs (device int32):
 *   kv_num [nb], kv_off [nb+1], kv_idx [nb*nb capacity]
 *   full_num [nb], full_off [nb+1], full_idx [nb*nb capacity]
 * totals (device int32 [2]) receives (#partial, #full). */
int hier_block_mask_build(const hier_grouping* g, void* workspace, int32_t* kv_num,
                          int32_t* kv_off, int32_t* kv_idx, int32_t* full_num,
                          int32_t* full_off, int32_t* full_idx, int32_t* totals,
                          void* stream);

/* Size of the fixed device scratch buffer used by
 * hier_block_mask_build_static (bytes). */
#define HIER_STATIC_SCRATCH_BYTES (4u << 20)

/* Allocation-free variant of hier_block_mask_build.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory on the
 * call path, such as a serving loop whose device memory is entirely
 * pre-reserved by its own allocator, or a foreign-language binding with no
 * device allocator from which to pass a workspace.  Same inputs and outputs
 * as hier_block_mask_build, minus the workspace: the scratch (unit matrix and
 * block classes, align256(U*U) + align256(nb*nb) bytes with U = P*T + T*N + T
 * and nb = ceil(S/128)) lives in a file-scope device array of
 * HIER_STATIC_SCRATCH_BYTES that every GPU loading the library holds until
 * the process exits.  Larger problems are rejected with HIER_EVALUE.  Call it
 * with the stream's device current.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and should come before any
 * stream capture.  Every call uses the same array: calls that overlap on the
 * GPU (different streams, or different host threads on one device) race on
 * it.  The kernels overwrite every scratch byte they read, so stale contents
 * of an earlier call never reach the results.  Never allocates or frees
 * device memory. */
int hier_block_mask_build_static(const hier_grouping* g, int32_t* kv_num, int32_t* kv_off,
                                 int32_t* kv_idx, int32_t* full_num, int32_t* full_off,
                                 int32_t* full_idx, int32_t* totals, void* stream);

/* Attention work plan for the full-sequence hierarchical layout, built from
 * the block classification of hier_block_mask_build (same workspace, after
 * it).  Query blocks are paired: pair p = query blocks 2p and 2p+1 (the two
 * halves the attention kernel computes together).  Writes
 *   q_pairs [np][8]  = (q_start0, q_rows0, q_start1, q_rows1, kv_begin, kv_end,
 *       0, 0), np = ceil(nb/2); a missing second block has q_rows1 = 0;
 *   kv_tiles [<= n_partial + n_full][4] = (k_row0, k_row1, mask0, mask1):
 *       ascending key blocks used by either half; k_row0/k_row1 are the pool
 *       rows of the two 64-key halves of the block (page_table != NULL maps
 *       logical 64-key pages to physical pages: page p holds keys
 *       [64p, 64p+64)); mask_h = -1 full block for half h, -2 block not used
 *       by half h, otherwise an index into row_masks;
 *   row_masks [n_partial][128][4] uint32 = per-row key bitmask of each partial
 *       block, in the order of the Flex partial list (bit c of word c/32 set
 *       <=> key c of the block is visible);
 *   order [np] = pairs sorted by descending number of key tiles;
 *   n_kv_tiles (device int32) = number of kv_tiles entries written.
 * The full-sequence layout is the reference's dense/Flex mask semantics
 * (hier_masks.py:364-1149), so inactive local-hub rows keep their self edge. */
int hier_block_plan_build(const hier_grouping* g, void* workspace, const int32_t* kv_off,
                          const int32_t* kv_idx, const int32_t* full_off,
                          const int32_t* full_idx, const int32_t* page_table,
                          int32_t* q_pairs, int32_t* kv_tiles, uint32_t* row_masks,
                          int32_t* order, int32_t* n_kv_tiles, void* stream);

/* Workspace bytes for hier_dense_block_mask_build / hier_dense_block_plan_build. */
int hier_dense_block_workspace_size(int64_t S, size_t* bytes);

/* The same block classification and lists as hier_block_mask_build, read
 * from a caller's dense mask instead of a grouping: mask is uint8/bool
 * [S, ld] on the device (row stride ld >= S; any non-zero byte allows the
 * pair, as flash_attention's mask.to(bool) does), or NULL for no mask (every
 * pair inside [0,S)^2 allowed).  Replaces the dense-mask and unmasked calls
 * of flash_attention (multics/models/attention.py:39-54, the sdpa path of
 * SelfAttention.forward, attention.py:436-442). */
int hier_dense_block_mask_build(const uint8_t* mask, int64_t S, int64_t ld, void* workspace,
                                int32_t* kv_num, int32_t* kv_off, int32_t* kv_idx,
                                int32_t* full_num, int32_t* full_off, int32_t* full_idx,
                                int32_t* totals, void* stream);

/* Attention work plan (the formats of hier_block_plan_build, no page table)
 * of the classification hier_dense_block_mask_build left in the workspace;
 * row_masks hold the mask's own bits of every partial block. */
int hier_dense_block_plan_build(const uint8_t* mask, int64_t S, int64_t ld, void* workspace,
                                const int32_t* kv_off, const int32_t* kv_idx, int32_t* q_pairs,
                                int32_t* kv_tiles, uint32_t* row_masks, int32_t* order,
                                int32_t* n_kv_tiles, void* stream);

/* Split-KV form of a query-pair plan: pair p becomes out pair p*chunks + c
 * over part c of its key-tile list [b + len*c/chunks, b + len*(c+1)/chunks),
 * with q_pairs[7] = 1 | c << 8 (partial rows in slot c, see
 * hier_partial_out); order [n_pairs*chunks] (or NULL) ranks them by work.
 * The slots are merged by hier_lse_gather_merge.  The input pairs must not
 * be partial already.  No counterpart in the reference (a scheduling
 * device: shorter CTAs for plans with few, long pairs). */
int hier_plan_split_kv(const int32_t* q_pairs, int32_t n_pairs, int32_t chunks,
                       int32_t* out_pairs, int32_t* order, void* stream);

/* Batched attention under one bool mask [Lq, Lk] shared by every batch entry
 * (query row b*Lq + i sees key row b*Lk + j iff mask[i*ld + j] != 0): the
 * reference's flash_attention(q, k, v, num_heads, mask) with a mask that
 * broadcasts over the batch (multics/models/attention.py:39-54), as the DiT
 * block's action branch calls it: the per-frame mouse attention with
 * get_temporal_block_causal_mask (hier_masks.py:1152-1166, blocks.py:441-447,
 * 684-686), the keyboard cross-attention with the repeated frame mask
 * (blocks.py:446-448,693-697) and their cached forms (blocks.py:256-375).
 * hier_shared_mask_plan_size gives the plan's extent: n_pairs query pairs and
 * tiles_per_pair kv_tiles entries reserved per pair; the caller allocates
 * q_pairs [n_pairs][8], kv_tiles [n_pairs * tiles_per_pair][4], tile_masks
 * [n_pairs * tiles_per_pair * 2][128][4] uint32 and order [n_pairs] (or
 * passes NULL for the identity order).  Sequences of at most 64 rows are
 * packed several to a 128-row tile with block-diagonal masks.  With aligned
 * != 0 the plan is instead cut on the 128-row grid of the flat rows: query
 * tiles are rows [128 i, 128 i + 128) of the B*Lq rows and key tiles start at
 * multiples of 128 of the B*Lk rows, per-row masks carrying the batch
 * diagonal; that is the form the backward (hier_bwd_plan_transpose,
 * hier_attn_bwd_dq, hier_attn_bwd_dkv) takes, at the price of partial tiles
 * for short sequences.  The plan runs on hier_attn_fwd (keys and values
 * [B*Lk, H*D]).  Errors: HIER_EVALUE for non-positive sizes, more than
 * 2^24 - 256 key rows, or a NULL mask / ld < Lk. */
int hier_shared_mask_plan_size(int64_t B, int64_t Lq, int64_t Lk, int32_t aligned,
                               int32_t* n_pairs, int32_t* tiles_per_pair);
int hier_shared_mask_plan_build(const uint8_t* mask, int64_t ld, int64_t B, int64_t Lq,
                                int64_t Lk, int32_t aligned, int32_t* q_pairs,
                                int32_t* kv_tiles, uint32_t* tile_masks, int32_t* order,
                                void* stream);

/* ---------------------------------------------------------------------------
 * Fused Q/K prologue
 * ------------------------------------------------------------------------- */

/* q = RoPE(RMSNorm(qx + cam @ wcq^T) * nqw), k likewise, for S tokens of
 * dimension dim = H * D (bf16 in, bf16 out), computed in fp32.  Replaces the
 * post-projection part of SelfAttention._project_self_attn_qkv
 * (multics/models/attention.py:355-365): camera adapter add
 * (_apply_camera_qk, attention.py:307-320, bias-free, cam_dim inputs),
 * RMSNorm over the full dim (attention.py:231-242, eps) and rope_apply
 * (multics/models/rope.py:248-254).  cam may be NULL (no camera tokens).
 * freqs: float32 [freqs_rows, D/2, 2] (cos, sin), shared by all heads; token
 * r uses row r % freqs_rows (freqs_rows = S: one row per token; the frame
 * count: a batch of sequences flattened to rows, as the per-frame action
 * attention's [frames, 1, D/2] table broadcasts over its batch).
 * Row strides are in elements.  out_rows (int32 [S], may be NULL) writes
 * token r's q and k to row out_rows[r] of q_out / k_out; k_out_rows (may be
 * NULL: out_rows) gives k its own rows, e.g. the physical rows of a paged
 * key pool.  dim = H*D a multiple of 128 up to 3072, D dividing 256, cam_dim
 * 12 or 16. */
int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                 int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                 const void* nkw, const float* freqs, int64_t freqs_rows, int64_t S, int32_t H,
                 int32_t D, float eps, void* q_out, void* k_out, int64_t out_stride,
                 const int32_t* out_rows, const int32_t* k_out_rows, void* stream);

/* Backward of hier_prep_qk (training): given the gradients gq, gk of the
 * roped q and k, writes dqx, dkx (bf16, the gradients of the projections
 * qx, kx) and the norm weights' gradients as partial rows dw_part
 * [2][n_warps][dim] fp32 (q then k; the caller sums over n_warps, from
 * hier_prep_qk_bwd_partials).  With y = x + cam @ Wc^T, yh = y * rstd and
 * g_n = the gradient rotated back by the RoPE table:
 *   dx = rstd * (g_n * w - yh * mean(g_n * w * yh)),  dw = sum_rows g_n * yh.
 * The camera adapters' gradient is dx^T @ cam (a GEMM left to the caller);
 * camera tokens get no gradient.  Replaces the autograd of the reference's
 * _project_self_attn_qkv (multics/models/attention.py:355-365) for the part
 * after the projections.  Other arguments as hier_prep_qk (no row maps). */
int hier_prep_qk_bwd_partials(int64_t S, int32_t* n_warps);
int hier_prep_qk_bwd(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                     int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                     const void* nkw, const float* freqs, int64_t freqs_rows, int64_t S,
                     int32_t H, int32_t D, float eps, const void* gq, const void* gk,
                     int64_t g_stride, void* dqx, void* dkx, int64_t dx_stride, float* dw_part,
                     void* stream);

/* ---------------------------------------------------------------------------
 * Attention
 * ------------------------------------------------------------------------- */

/* Block-sparse flash attention forward on sm_100a (tcgen05 MMA with TMEM
 * accumulators, TMA-staged tiles, online softmax), bf16 in/out, D = 128.
 *   q   bf16 [q_rows_total, H*D] (row stride q_stride elements)
 *   k,v bf16 [kv_rows_total, H*D] key/value pool (row stride kv_stride)
 *   out bf16 [q_rows_total, H*D] (row stride out_stride); only rows covered
 *       by q_pairs are written; rows whose key set is empty are written as 0
 *       (the cached backends' contract, hier_segmented_attention.py:104-109).
 *   q_pairs [n_pairs][8], kv_tiles [][4], row_masks, order [n_pairs] (or
 *       NULL) in the format of hier_block_plan_build: each CTA computes the
 *       two 128-row query tiles of a pair for one head, pairs taken in the
 *       order of order[] for every head.
 *   dev_err: device int32, set non-zero if a pipeline wait timed out.
 * Replaces the attention kernels of the reference backends: masked SDPA
 * (attention.py:39-54), FlexAttention (attention.py:322-353), the Triton
 * segmented / tiled128 kernels (kernels/hier_segmented_attention.py:27-114,
 * kernels/hier_tiled_attention.py:52-146), aten FA2 varlen
 * (kernels/hier_packed_attention.py:230-242) and FlashInfer paged prefill
 * (kernels/hier_paged_attention.py:238-266). */
int hier_attn_fwd(const void* q, int64_t q_rows_total, int64_t q_stride, const void* k,
                  const void* v, int64_t kv_rows_total, int64_t kv_stride, void* out,
                  int64_t out_stride, int32_t H, int32_t D, const int32_t* q_pairs,
                  int32_t n_pairs, const int32_t* kv_tiles, const uint32_t* row_masks,
                  const int32_t* order, float softmax_scale, int32_t* dev_err, void* stream);

/* Maximum number of key/value tensors (streams) one attention launch reads. */
#define HIER_MAX_KV_STREAMS 32

/* hier_attn_fwd over keys/values held in several tensors ("streams", e.g. one
 * rolling cache per player, per local-hub group and the global hub), read in
 * place: no pool concatenation (the reference copies every cache into one
 * pool per call, hier_segmented_attention.py:484-495,
 * hier_paged_attention.py:182-191).  Stream s is k[s], v[s]: bf16
 * [stream_rows[s], H*D] with row stride kv_stride[s] elements (device
 * pointers in a host array).  A key-box row of kv_tiles is
 * (s << 24) | row-within-stream.  tile_masks holds mask_rows entries of four
 * uint32 per partial tile: 128 (one key bitmask per query row, the format of
 * hier_block_plan_build) or 1 (one key bitmask shared by every query row, the
 * format of hier_cached_build); a query pair whose q_pairs[6] is 1 uses 128
 * (its mask index then counts 128-entry masks) whatever mask_rows says.
 * lse (float [q_rows_total][H], may be NULL)
 * receives per written row and head log2(sum_j 2^(s_j)) of the scaled scores
 * s_j = q.k_j * softmax_scale * log2(e) (-inf for rows without keys), so that
 * partial results over disjoint key sets merge as
 * O = sum_r 2^(lse_r - M) O_r / sum_r 2^(lse_r - M).  out_rows (int32
 * [q_rows_total], may be NULL) sends query row r's output and lse to row
 * out_rows[r] (a query order other than the output order, e.g. hub rows
 * grouped by group while the output keeps the sequence order).  part (may
 * be NULL): a second query tensor and the destination of partial rows (see
 * hier_partial_out).  Other arguments as hier_attn_fwd. */
/* Rows of a query-pair plan beyond the main query tensor: query rows from
 * q2_row0 on are read from q2 (row r at q2 row r - q2_row0); the outputs of
 * pairs flagged in q_pairs[7] (bit 0) are partial rows, written to o at row
 * r - row0 + (q_pairs[7] >> 8) * slot_rows with their log2-sum-exp in lse
 * ([rows][H]) for a later merge (hier_lse_gather_*): bits 8 and up select a
 * slot, so that pairs over disjoint parts of one key list (split-KV) keep
 * their partial rows apart. */
typedef struct hier_partial_out {
  const void* q2;
  int64_t q2_rows, q2_stride, q2_row0;
  void* o;
  int64_t o_stride;
  float* lse;
  int64_t row0;
  int64_t slot_rows;
} hier_partial_out;

int hier_attn_fwd_streams(const void* q, int64_t q_rows_total, int64_t q_stride,
                          int32_t n_streams, const void* const* k, const void* const* v,
                          const int64_t* stream_rows, const int64_t* kv_stride, void* out,
                          int64_t out_stride, const int32_t* out_rows, int32_t H, int32_t D,
                          const int32_t* q_pairs,
                          int32_t n_pairs, const int32_t* kv_tiles, const uint32_t* tile_masks,
                          int32_t mask_rows, const int32_t* order, float softmax_scale,
                          float* lse, const hier_partial_out* part, int32_t* dev_err,
                          void* stream);

/* ---------------------------------------------------------------------------
 * Attention backward (training)
 * ------------------------------------------------------------------------- */

/* Gradients of hier_attn_fwd / hier_attn_fwd_streams over a 128x128 block
 * plan (hier_block_plan_build without a page table, or
 * hier_dense_block_plan_build), in place of the FlexAttention backward the
 * reference trains with (multics/models/attention.py:322-353, the Flex
 * Jacobian of forward_hier_tiled_ste, attention.py:367-434).  With
 * s = q.k * scale * log2(e), P = 2^(s - lse) (lse from the forward, log2
 * units), dP = dO.v and Delta = rowsum(dO * O):
 *   dQ = scale * (P * (dP - Delta)) K,  dK = scale * (P * (dP - Delta))^T Q,
 *   dV = P^T dO.
 * Tensors are bf16 [rows, H*128] (row strides in elements, multiples of 8,
 * 16-byte aligned bases).  Every dQ, dK and dV row is written once (rows
 * without keys or queries: 0); no atomics. */

/* delta [H][rows_pad] = rowsum(dO * O) per head (fp32) and lse_t [H][rows_pad]
 * = the forward's lse [rows][H] transposed, +inf for rows without keys and
 * for the padding rows (rows_pad: a multiple of 128, >= rows). */
int hier_attn_bwd_prep(const void* o, int64_t o_stride, const void* dout, int64_t do_stride,
                       const float* lse, int64_t rows, int32_t H, int32_t D, float* delta,
                       float* lse_t, int64_t rows_pad, void* stream);

/* Key-major form of a block plan: per key block kb (keys [128 kb, 128 kb +
 * 128)) the query blocks that see it, k_ent [capacity][4] = (q_start,
 * q_rows, mask selector (-1 full, else an index into t_masks), q_start/128)
 * at k_off[kb] .. k_off[kb+1] (ascending q_start), and t_masks
 * [n_masks][128][4] = row_masks transposed (word w bit b of key row j: query
 * row 32w + b).  capacity >= the plan's (entry, half) references (n_partial +
 * n_full of the block classification).  workspace: int32 [2 * n_kb].
 * *status (device) gets bit 0 if the plan is not an aligned single-stream
 * block plan, bit 1 if capacity is too small. */
int hier_bwd_plan_transpose(const int32_t* q_pairs, int32_t n_pairs, const int32_t* kv_tiles,
                            const uint32_t* row_masks, int32_t n_masks, int32_t n_kb,
                            int32_t* workspace, int32_t* k_off, int32_t* k_ent,
                            int32_t capacity, uint32_t* t_masks, int32_t* status,
                            void* stream);

/* dQ over the forward's query-major plan (q_pairs, kv_tiles, row_masks with
 * mask_rows 128 or 1 as in hier_attn_fwd_streams): one CTA per (query tile,
 * head).  dout has the rows of q. */
int hier_attn_bwd_dq(const void* q, int64_t q_rows, int64_t q_stride, const void* k,
                     const void* v, int64_t kv_rows, int64_t kv_stride, const void* dout,
                     int64_t do_stride, const float* lse_t, const float* delta,
                     int64_t rows_pad, int32_t H, int32_t D, const int32_t* q_pairs,
                     int32_t n_pairs, const int32_t* kv_tiles, const uint32_t* row_masks,
                     int32_t mask_rows, float softmax_scale, void* dq, int64_t dq_stride,
                     int32_t* dev_err, void* stream);

/* dK and dV over the key-major plan of hier_bwd_plan_transpose: one CTA per
 * (key block, head); n_kb * 128 >= kv_rows. */
int hier_attn_bwd_dkv(const void* q, int64_t q_rows, int64_t q_stride, const void* k,
                      const void* v, int64_t kv_rows, int64_t kv_stride, const void* dout,
                      int64_t do_stride, const float* lse_t, const float* delta,
                      int64_t rows_pad, int32_t H, int32_t D, const int32_t* k_off,
                      const int32_t* k_ent, const uint32_t* t_masks, int32_t n_kb,
                      float softmax_scale, void* dk, int64_t dk_stride, void* dv,
                      int64_t dv_stride, int32_t* dev_err, void* stream);

/* ---------------------------------------------------------------------------
 * Cached (rolling key/value cache) step
 * ------------------------------------------------------------------------- */

/* One cached step: the query block of n_frames new frames (player rows,
 * then local-hub rows, then global-hub rows, as causal_forward_hier_hub
 * orders them, multics/models/attention.py:456-1005) against the retained
 * frames of every cache.  Mirrors the arguments of _build_metadata
 * (multics/models/kernels/hier_segmented_attention.py:156-395) with the
 * per-token tensors of the cached-backend plugin signature
 * (hier_paged_attention.py:79-106) instead of host tuples.  Device pointers:
 *   agent_frames[p]  int64 [fa*L]   frame id of every cached token of player p
 *   local_frames[g]  int64 [fl*KL]  (no_local: unused, fl = 0, K_L = 0)
 *   local_active[g]  uint8 [fl*KL]  token activity of local-hub caches
 *   global_frames    int64 [fg*KG]
 *   labels           int64 [n_frames, P]   (membership_mode == 0)
 *   q_active         uint8 [n_frames, N]
 *   membership       uint8 [T_mem, N, P]   (membership_mode == 1), indexed by
 *   global_only      uint8 [T_mem, P]       absolute frame id */
typedef struct hier_cached_grouping {
  int32_t P, N, L, KL, KG;
  int32_t n_frames, n_block, local_attn, direct, no_local, membership_mode;
  int32_t fa, fl, fg; /* retained frames per agent / local / global cache */
  int32_t T_mem;
  const int64_t* agent_frames[HIER_MAX_KV_STREAMS];
  const int64_t* local_frames[HIER_MAX_KV_STREAMS];
  const uint8_t* local_active[HIER_MAX_KV_STREAMS];
  const int64_t* global_frames;
  const int64_t* labels;
  const uint8_t* q_active;
  const uint8_t* membership;
  const uint8_t* global_only;
} hier_cached_grouping;

typedef struct hier_cached_sizes_t {
  int32_t n_seg;         /* segments: P*n + N*n (unless no_local) + n */
  int32_t n_prog;        /* block_m programs */
  int32_t n_pairs;       /* attention query pairs */
  int32_t n_streams;     /* key/value streams: P agents, N local (unless no_local), global */
  int32_t n_cand;        /* candidate runs per segment */
  int32_t tile_capacity; /* upper bound of attention key tiles */
  int64_t q_rows;        /* query rows of the step */
  int64_t pool_rows;     /* rows of the reference's concatenated pool */
} hier_cached_sizes_t;

/* Host-only sizes of a cached step (validates the grouping with the
 * reference's messages). */
int hier_cached_sizes(const hier_cached_grouping* g, int32_t block_m, hier_cached_sizes_t* out);

/* Per segment: number of keys (kv_count, as _build_metadata) and of 64-row
 * key boxes of the attention plan.  status (device int32, may be NULL) gets
 * bit 0 set if a membership / global_only frame is out of range. */
int hier_cached_count(const hier_cached_grouping* g, int32_t* kv_count, int32_t* n_boxes,
                      int32_t* status, void* stream);

/* Fill the outputs of a cached step; any group may be NULL to skip it.
 *   prog_qbase/prog_nq/prog_seg [n_prog]: block_m programs (bit-exact);
 *   kv_index [n_seg, kv_width] int32, zero padded (bit-exact for
 *       kv_width = ceil64(max kv_count), as _build_metadata);
 *   q_pairs [n_pairs][8], kv_tiles [tile_capacity][4], tile_masks
 *       [tile_capacity][4] (mask_rows = 1), order [n_pairs]: the attention
 *       plan for hier_attn_fwd_streams; with n_boxes from hier_cached_count
 *       the segments' tiles are packed, with n_boxes NULL each segment gets
 *       tile_capacity / n_seg tiles (no count launch needed).
 * status bit 1 is set if the plan exceeds tile_capacity.  No host sync. */
int hier_cached_build(const hier_cached_grouping* g, int32_t block_m, const int32_t* n_boxes,
                      int32_t* prog_qbase, int32_t* prog_nq, int32_t* prog_seg,
                      int32_t* kv_index, int32_t kv_width, int32_t* q_pairs, int32_t* kv_tiles,
                      uint32_t* tile_masks, int32_t tile_capacity, int32_t* order,
                      int32_t* status, void* stream);

/* Packed hub rows for the attention plan of a cached step.  A local-hub
 * segment has K_L query rows but its members' whole cached history as keys,
 * and a group's segments at the n query frames see almost the same keys; so
 * the plan can pack them: pack g (g < N) = the rows of group g at every
 * query frame (n*K_L rows, frame-major: row f*K_L + s is hub slot s of group
 * g at query frame f), pack N = the global-hub rows (n*K_G, frame-major).  A
 * pack's key list is the union of its frames' candidate runs; its tiles carry
 * 128-row masks (a row sees the keys its own segment attends to).  Packing
 * applies when n*K_L <= 128 and n*K_G <= 128 (n_packs = 0 otherwise, and
 * without local hubs).  The packed rows are a second query block
 * (hier_partial_out.q2, rows from q2_row0 on) written back through out_rows.
 * The per-segment metadata (_build_metadata's contract) is unchanged. */
typedef struct hier_cached_pack_sizes_t {
  int32_t n_packs;       /* N + (K_G > 0), or 0 */
  int32_t q2_rows;       /* packed query rows: n*(N*K_L + K_G) */
  int32_t agent_pairs;   /* the plan's player pairs: q_pairs rows [0, agent_pairs) */
  int32_t tile_capacity; /* upper bound of the packs' key tiles */
} hier_cached_pack_sizes_t;

int hier_cached_pack_sizes(const hier_cached_grouping* g, hier_cached_pack_sizes_t* out);

/* 64-row key boxes of each pack (n_boxes [n_packs]). */
int hier_cached_pack_count(const hier_cached_grouping* g, int32_t* n_boxes, int32_t* status,
                           void* stream);

/* After hier_cached_build (n_boxes from hier_cached_pack_count, or NULL:
 * each pack gets (tile_end - tile_base) / n_packs tiles): the packs' pairs at q_pairs rows [agent_pairs,
 * agent_pairs + n_packs) (replacing the hub segments' pairs, so the plan
 * has agent_pairs + n_packs pairs), their tiles at kv_tiles rows
 * [tile_base, tile_end), their 128-row masks from index mask_base of
 * tile_masks counted in 128-entry units (mask_base * 128 >= the per-tile
 * masks in use), packed row i read as query row q2_row0 + i; order
 * [agent_pairs + n_packs] ranks all pairs.  status bit 1: capacity
 * exceeded. */
int hier_cached_pack_build(const hier_cached_grouping* g, const int32_t* n_boxes,
                           int32_t tile_base, int32_t tile_end, int32_t mask_base,
                           int32_t q2_row0, int32_t* q_pairs, int32_t* kv_tiles,
                           uint32_t* tile_masks, int32_t* order, int32_t* status, void* stream);

/* Workspace bytes for hier_varlen_plan_build. */
int hier_varlen_workspace_size(int32_t n_seg, size_t* bytes);

/* Packed varlen plan of _get_varlen_plan (hier_packed_attention.py:32-102)
 * from one-program-per-segment metadata: over the segments with rows and
 * keys, q_index (int64 [sum q]) = their query rows, k_index (int64 [sum k]) =
 * their kv_index rows, cu_q / cu_k (int32 [active+1]); page_indices (int32
 * [sum k], may be NULL) = k_index as the page table of page size 1
 * (hier_paged_attention.py:232-249); scalars (int64 [5]) = max_q, max_k,
 * min_k_index, max_k_index, number of active segments. */
int hier_varlen_plan_build(const int32_t* prog_qbase, const int32_t* prog_nq,
                           const int32_t* kv_index, int32_t kv_width, const int32_t* kv_count,
                           int32_t n_seg, void* workspace, int64_t* q_index, int64_t* k_index,
                           int32_t* cu_q, int32_t* cu_k, int32_t* page_indices, int64_t* scalars,
                           void* stream);

/* ---------------------------------------------------------------------------
 * Tiled128 block layouts
 * ------------------------------------------------------------------------- */

#define HIER_TILED_FULL 0   /* build_hier_tiled_full_sequence_layouts */
#define HIER_TILED_CACHED 1 /* build_hier_tiled_cached_layout */

/* Inputs of the Tiled128 layout builders
 * (multics/models/kernels/hier_tiled_attention.py:244-429, 474-655).  Device
 * pointers.  Full sequence (mode 0): T frames, labels int64 [T, P], active
 * uint8 [T, N] (labels constant inside each block of n_block frames, checked
 * by the host layer).  Cached (mode 1): n_frames query frames, labels int64
 * [n_frames, P], active = q_active uint8 [n_frames, N], and the per-token
 * cache tensors as in hier_cached_grouping (fa / fl / fg retained frames). */
typedef struct hier_tiled_grouping {
  int32_t mode;
  int32_t P, N, L, KL, KG, n_block, local_attn, direct;
  int32_t T;
  int32_t n_frames, fa, fl, fg;
  const int64_t* labels;
  const uint8_t* active;
  const int64_t* agent_frames[HIER_MAX_KV_STREAMS];
  const int64_t* local_frames[HIER_MAX_KV_STREAMS];
  const uint8_t* local_active[HIER_MAX_KV_STREAMS];
  const int64_t* global_frames;
} hier_tiled_grouping;

typedef struct hier_tiled_sizes_t {
  int32_t n_layouts;     /* T / n_block (full) or 1 (cached) */
  int32_t n_seg;         /* segments per layout */
  int32_t n_prog;        /* BLOCK_M=16 programs per layout */
  int32_t n_pairs;       /* attention query pairs per layout */
  int32_t tile_capacity; /* upper bound of attention key tiles, all layouts */
  int32_t reserved;
  int64_t q_rows;        /* query rows */
} hier_tiled_sizes_t;

int hier_tiled_sizes(const hier_tiled_grouping* g, hier_tiled_sizes_t* out);

/* Per (layout, segment), layout-major: kv_count (kept 128-slot chunks x 128,
 * as the reference), attention key boxes, and slots [2] int64 = (logical =
 * valid slots, dense slots).  status bit 2: a query frame is missing from an
 * agent cache (the reference's KeyError). */
int hier_tiled_count(const hier_tiled_grouping* g, int32_t* kv_count, int32_t* n_boxes,
                     int64_t* slots, int32_t* status, void* stream);

/* Fill the layouts (NULL groups skipped): programs [n_layouts*n_prog];
 * kv_index (int32) / kv_valid (uint8) of layout b at element offset
 * kv_off[b] with row width kv_width[b] (device arrays; bit-exact for
 * kv_width = ceil128(max kv_count of the layout)); and one attention plan
 * over all layouts (q_pairs [n_layouts*n_pairs][8], kv_tiles / tile_masks
 * [tile_capacity][4], order) for hier_attn_fwd_streams with mask_rows = 1 on
 * the full-sequence (or concatenated cached) key/value pool. */
int hier_tiled_build(const hier_tiled_grouping* g, const int32_t* n_boxes, const int64_t* kv_off,
                     const int32_t* kv_width, int32_t* prog_qbase, int32_t* prog_nq,
                     int32_t* prog_seg, int32_t* kv_index, uint8_t* kv_valid, int32_t* q_pairs,
                     int32_t* kv_tiles, uint32_t* tile_masks, int32_t tile_capacity,
                     int32_t* order, int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Player-sharded execution (one rank per GPU)
 * ------------------------------------------------------------------------- */

/* One rank's share of a full-sequence layer (labels mode), or with one
 * shard (every player local with all its strips and hub partials, hub_keys
 * = 1) the whole layer.  The rank holds the rows of n_local players (row
 * slots in local_player order) and computes the given 256-row strips of
 * them, so players can be split between ranks by strips when their count
 * does not divide the ranks.  Its query rows:
 *   [0, own_rows)           its local players' rows (slot, frame, patch);
 *   [own_rows, V)           every hub row, group-major: local hub (g, f, slot)
 *                           at own_rows + (g*T + f)*K_L + slot, then global hub
 *                           (f, slot) at own_rows + T*N*K_L + f*K_G + slot
 *                           (V = own_rows + hub_rows);
 *   [V + o, V + o + hub_partial_rows) per hub-partial player (k-th slot with
 *                           hub_partials set) and frame t the K_L rows of the
 *                           local hub of its group at t, row
 *                           V + o + (k*T + t)*K_L + slot (a second query
 *                           tensor: hier_partial_out.q2 with q2_row0 = V + o;
 *                           o = hub_partial_row0 places the rank's partials in
 *                           a buffer shared by the ranks).
 * Key/value streams for hier_attn_fwd_streams: 0 = its local players' rows, 1 =
 * the hub rows (same order), and for each remote group-mate unit (o, f) (the
 * L rows of player o at frame f) the stream-packed first row
 * remote_key[o*T + f] = (stream << 24) | row (-1 if absent): a buffer of
 * frames fetched before the launch, or the owning rank's buffer mapped from
 * its GPU (read in place over NVLink).
 * Player rows get their full key sets (a group-mate frame held by no local
 * slot comes from remote_key).  A hub row is split into partial rows over
 * disjoint key sets: per member player (third block, on the rank computing
 * that player's hub partials) and over the hub tokens (second block, when
 * hub_keys is set); hub
 * pairs are flagged in q_pairs[7] and written as partial rows
 * (hier_partial_out.row0 = own_rows: hub-key partials at [0, hub_rows),
 * player partials at hub_rows + o onwards), then merged with
 * hier_lse_gather_merge.  Query pairs are two 128-row tiles of 256-row strips of
 * one block; their key tiles cover exactly the key units some row attends
 * to and carry a 128-row mask per half where a half sees part of a tile
 * (q_pairs[6] = 1; launch with mask_rows 128).  An inactive local hub
 * attends to itself only.  The edges are those of the dense mask
 * (multics/models/hier_masks.py:364-507); no reference counterpart exists
 * for the sharding itself: the reference runs every player on one device. */
#define HIER_SHARD_MAX_LOCAL 16

typedef struct hier_shard_desc {
  int32_t P, N, L, KL, KG, T, n_block, local_attn, direct;
  int32_t n_local;          /* players whose rows this rank holds */
  int32_t hub_keys;
  int32_t hub_partial_row0; /* o: first hub-partial row (0 for one shard) */
  const int64_t* labels;      /* [T, P] */
  const uint8_t* active;      /* [T, N] */
  const int32_t* remote_key;  /* [P*T] */
  int32_t local_player[HIER_SHARD_MAX_LOCAL]; /* absolute player of each local row slot */
  int32_t strip_begin[HIER_SHARD_MAX_LOCAL];  /* the 256-row strips [begin, end) of the */
  int32_t strip_end[HIER_SHARD_MAX_LOCAL];    /*   slot's player this rank computes */
  int32_t hub_partials[HIER_SHARD_MAX_LOCAL]; /* 1: this rank computes the player's hub partials */
  /* Paged player rows (key/value stream 0) in pages of 64 rows: logical row
   * r of stream 0 lives at physical row page_table[r / 64] * 64 + r % 64 of
   * the stream's tensors (n_pages >= ceil(own_rows / 64) entries).  NULL: rows
   * in place.  Paging needs a single shard holding every player. */
  const int32_t* page_table;
  int32_t n_pages;
  /* With hub_keys set: the hub-key pairs this rank computes (one group's
   * T*K_L local-hub rows or the T*K_G global-hub rows per 256-row strip, in
   * the order local group 0 .. N-1, then global): [hub_key_first,
   * hub_key_first + hub_key_count), or all of them for hub_key_count = 0.
   * Spread over the ranks, each hub-token partial row is computed on one
   * rank; hier_lse_gather_merge_peers reads it there (local_owner). */
  int32_t hub_key_first;
  int32_t hub_key_count;
} hier_shard_desc;

typedef struct hier_shard_sizes_t {
  int32_t n_pairs;          /* player strips, hub-partial strips, hub-key pairs */
  int32_t n_player_pairs;   /* the player strips, pairs [0, n_player_pairs) */
  int32_t n_counts;         /* int32 entries of the per-pair counts */
  int32_t reserved;
  int64_t own_rows;         /* the rank's player rows */
  int64_t hub_rows;         /* T*(N*K_L + K_G) */
  int64_t hub_partial_rows; /* hub-partial players * T*K_L */
} hier_shard_sizes_t;

int hier_shard_sizes(const hier_shard_desc* g, hier_shard_sizes_t* out);

/* First pass: per pair its key tiles and 128-row masks (counts, int32
 * [n_counts]) and their totals (int32 [2] on the device: key tiles, masks),
 * from which the caller sizes kv_tiles ([tiles][4] int32) and tile_masks
 * ([masks][128][4] uint32).  Status bit 3: a remote unit the plan needs has
 * no slot.  No host sync. */
int hier_shard_count(const hier_shard_desc* g, int32_t* counts, int32_t* totals,
                     int32_t* status, void* stream);

/* Second pass: the plan (q_pairs [n_pairs][8], kv_tiles, tile_masks, order
 * [n_pairs] or NULL: every pair by descending work); status bit 1: tile
 * capacity, bit 4: mask capacity, bit 5: a pair touches more pages of the
 * paged stream than the builder's page list holds.  With a page table the
 * player keys of a pair are covered page by page (every row of a page it
 * touches, masked by the unit-level edges), so each 64-row key box is one
 * physical page, the reference's paged KV layout
 * (kernels/hier_paged_attention.py:209-260) with 64-token pages. */
int hier_shard_build(const hier_shard_desc* g, const int32_t* counts, int32_t* q_pairs,
                     int32_t* kv_tiles, int32_t tile_capacity, uint32_t* tile_masks,
                     int64_t mask_capacity, int32_t* order, int32_t* status, void* stream);

/* Bounds check of an attention work plan (q_pairs [n_pairs][8], kv_tiles
 * [n_tiles][4], order [n_pairs] or NULL) before a launch, for plans that a
 * caller built, stored or received: every pair's key-tile range inside
 * [0, n_tiles), its query rows inside [0, q_rows_total) (count a second query
 * block's rows in) and at most 128 per tile, every selector -1, -2 or a
 * row-mask index below n_masks, every 64-row key box in an existing stream
 * (stream index row >> 24 below n_streams) starting before the stream's end
 * plus 64 rows (row & 0xFFFFFF below stream_rows[stream] + 64: the second
 * box of a block plan's last tile may start past the end; rows past the end
 * read as zero), every order entry below n_pairs.  The check reads a table entry
 * only after checking its index.  status (device int32, cleared first): bit
 * 0 key-tile range, bit 1 query rows, bit 2 selector, bit 3 key rows or
 * stream, bit 4 order.  stream_rows is a host array of n_streams (1..32)
 * entries.  Partial-row destinations are not checked.  No host sync.  This
 * is the metadata-corruption check the reference's plugin performs on the
 * host (kernels/hier_packed_attention.py:224-225), on the device. */
int hier_plan_check(const int32_t* q_pairs, int32_t n_pairs, const int32_t* kv_tiles,
                    int64_t n_tiles, int64_t n_masks, const int32_t* order, int64_t q_rows_total,
                    const int64_t* stream_rows, int32_t n_streams, int32_t* status, void* stream);

/* Merge of partial rows over disjoint key sets.  Target t has the partial
 * rows rows[off[t] .. off[t+1]) of o (bf16 [.., H*D], row stride o_stride)
 * with log2-sum-exp lse ([..][H]); out[out_rows ? out_rows[t] : t] =
 * sum_i 2^(lse_i - M) o_i / sum_i 2^(lse_i - M) (bf16, M the largest lse_i,
 * 0 without keys).  Across ranks the partial rows are all-gathered first, or
 * read in place (hier_lse_gather_merge_peers). */
int hier_lse_gather_merge(const void* o, int64_t o_stride, const float* lse, int32_t H, int32_t D,
                          const int32_t* off, const int32_t* rows, int64_t n_targets, void* out,
                          int64_t out_stride, const int32_t* out_rows, void* stream);

/* hier_lse_gather_merge over partial rows that stay in the memory of the
 * rank that computed them: o_bases / lse_bases are device arrays of n_ranks
 * pointers (this rank's own buffers and the other ranks' buffers mapped into
 * this GPU's address space, e.g. symmetric memory); partial row pr < local_rows
 * is read from rank local_owner[pr] (rank self when local_owner is NULL), a
 * higher row from rank (pr - local_rows) / slot_rows, at the same row of that
 * rank's buffer.  The caller orders the reads after
 * every rank's writes (a collective on the stream after the attention).
 * (Having the attention kernels write each partial row into every rank's
 * buffer instead was measured slower at 8 GPUs: the NVLink stores slow the
 * attention launch more than the merge saves.) */
int hier_lse_gather_merge_peers(const void* const* o_bases, const float* const* lse_bases,
                                int32_t n_ranks, int32_t self, int64_t local_rows,
                                int64_t slot_rows, int64_t o_stride, int32_t H, int32_t D,
                                const int32_t* off, const int32_t* rows, int64_t n_targets,
                                void* out, int64_t out_stride, const int32_t* out_rows,
                                const int32_t* local_owner, void* stream);

/* ---------------------------------------------------------------------------
 * Self-test of the tensor-core operand encodings (no reference counterpart):
 * with A, B bf16 [128,128] row-major,
 *   c_ss = A @ B^T   (both operands K-major in shared memory)
 *   c_mn = A @ B     (B MN-major in shared memory)
 *   c_ts = A @ B     (A read from tensor memory, B MN-major)
 * as fp32 [128,128]. */
int hier_selftest_umma(const void* a, const void* b, float* c_ss, float* c_mn, float* c_ts,
                       int32_t* dev_err, void* stream);

/* Self-test of the bounded pipeline wait (no reference counterpart; the
 * reference has no device-side waits): one thread waits, giving up after
 * limit_cycles SM clock cycles (1 .. 4e9, the kernels' own limit), on a
 * barrier phase that nothing completes.  Afterwards *dev_err holds
 * 1 (wait timed out) | (30 << 8) (wait site) if it was 0, and *dev_cycles the
 * cycles waited (-1 if the wait had not given up).  This is how every kernel
 * of the library reports a stalled pipeline instead of hanging the device. */
int hier_selftest_wait_timeout(int64_t limit_cycles, int32_t* dev_err, int64_t* dev_cycles,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HIER_B200_H */
