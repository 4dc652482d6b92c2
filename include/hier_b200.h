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
 * freqs: float32 [S, D/2, 2] (cos, sin) per token, shared by all heads.
 * Row strides are in elements. */
int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                 int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                 const void* nkw, const float* freqs, int64_t S, int32_t H, int32_t D,
                 float eps, void* q_out, void* k_out, int64_t out_stride, void* stream);

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
 *       two 128-row query tiles of a pair for one head.
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

/* ---------------------------------------------------------------------------
 * Self-test of the tensor-core operand encodings (no reference counterpart):
 * with A, B bf16 [128,128] row-major,
 *   c_ss = A @ B^T   (both operands K-major in shared memory)
 *   c_mn = A @ B     (B MN-major in shared memory)
 *   c_ts = A @ B     (A read from tensor memory, B MN-major)
 * as fp32 [128,128]. */
int hier_selftest_umma(const void* a, const void* b, float* c_ss, float* c_mn, float* c_ts,
                       int32_t* dev_err, void* stream);

/* Self-test of the FMA-pipe exp2 used for part of the softmax exponentials
 * (no reference counterpart): y[i] = 2^x[i] for n fp32 values, 0 for
 * x <= -127. */
int hier_selftest_exp2(const float* x, float* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HIER_B200_H */
