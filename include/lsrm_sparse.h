/*
 * lsrm_sparse.h — C ABI of the B200 (sm_100a) variable-block native sparse
 * attention library (liblsrm_sparse.so).
 *
 * The library replaces the hot path of LSRM's sparse volume decoder
 * (chenxiex/Large-Sparse-Reconstruction-Model): the Triton kernels of
 * sparse/ops/triton_native_sparse_attention_impl_kvcentric.py, the pure-torch
 * scorer sparse/ops/block_score.py, the flash-attn calls of the compressed
 * and window branches, the segment-mean compression and the gated merge of
 * sparse/module/spatial_sparse_attention.py.
 *
 * Conventions (all entry points):
 *   - plain device pointers, sizes and element strides; no framework types;
 *   - `stream` is a cudaStream_t passed as void*; nothing synchronises the
 *     host; work is enqueued on `stream` only;
 *   - return 0 on success or a negative LSRM_ERR_* code; a message for the
 *     last failure of the calling thread is returned by lsrm_last_error();
 *   - device-side problems (bad indices, timeouts) are OR-ed into the int
 *     pointed to by `err_flags` (device memory, may be NULL) as LSRM_ERR_*
 *     bits; callers that want them read the word after the stream completes;
 *   - `workspace` is caller-owned device memory of at least the size reported
 *     by the matching *_workspace_bytes() query; the library never allocates.
 *   - token-major layouts: q/o/dq [total_q, Hq, D], k/v/dk/dv [total_k, Hkv, D]
 *     (head stride D, token stride given), LSE [Hq, total_q] fp32.
 *   - dtype: LSRM_DTYPE_BF16 or LSRM_DTYPE_F16 for q/k/v/o and grads.
 */
#ifndef LSRM_SPARSE_H_
#define LSRM_SPARSE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSRM_ABI_VERSION 2

/* return codes (negative) and device error bits (positive) */
#define LSRM_OK 0
#define LSRM_ERR_INVALID_ARG (-1)
#define LSRM_ERR_UNSUPPORTED (-2)
#define LSRM_ERR_ALIGNMENT (-3)
#define LSRM_ERR_CUDA (-4)
#define LSRM_ERR_WORKSPACE (-5)
/* device error-word bits */
#define LSRM_ERR_TIMEOUT 0x1          /* a bounded wait ran out (kernel tore down) */
#define LSRM_ERR_DUPLICATE_BLOCK 0x2  /* a query listed one block twice */
#define LSRM_ERR_CAPACITY 0x4         /* a work list exceeded its capacity */
#define LSRM_ERR_BAD_INDEX 0x8        /* metadata out of range */

#define LSRM_DTYPE_F16 0
#define LSRM_DTYPE_BF16 1

/* Variable-length metadata shared by the attention entry points (device
 * pointers, int32).  Mirrors the arguments of native_sparse_attend
 * (sparse/ops/triton_native_sparse_attention_impl_kvcentric.py:1382-1393). */
typedef struct lsrm_varlen {
  int32_t num_seqs;                       /* B */
  int32_t total_q;                        /* Nq */
  int32_t total_k;                        /* Nk */
  int32_t num_blocks;                     /* total KV blocks (len(cu_block_include_tokens) - 1) */
  const int32_t* cu_seqlens_q;            /* [B+1] */
  const int32_t* cu_seqlens_k;            /* [B+1] */
  const int32_t* cu_seqblocks;            /* [B+1] block offsets per sequence */
  const int32_t* cu_block_include_tokens; /* [num_blocks+1] global token offsets */
} lsrm_varlen;

/* Attention problem shape and operand layout. */
typedef struct lsrm_attn_shape {
  int32_t num_q_heads;   /* Hq */
  int32_t num_kv_heads;  /* Hkv; Hq % Hkv == 0, G = Hq/Hkv a power of two <= 128 */
  int32_t head_dim;      /* D: 16, 32 or 64 */
  int32_t dtype;         /* LSRM_DTYPE_* */
  int64_t q_token_stride;  /* elements between consecutive tokens of q/o/do/dq */
  int64_t kv_token_stride; /* elements between consecutive tokens of k/v/dk/dv */
  float softmax_scale;     /* <= 0 selects 1/sqrt(D) */
} lsrm_attn_shape;

/* ---------------------------------------------------------------------- */
/* Library information                                                      */
/* ---------------------------------------------------------------------- */
int lsrm_abi_version(void);
const char* lsrm_last_error(void);
/* Returns the number of kernels this library launched since load (all
 * entry points, all threads); used by benchmarks to count launches. */
uint64_t lsrm_launch_count(void);

/* Kernel timing (tracing): while enabled, every entry point records a CUDA
 * event pair on its stream around each kernel it launches.
 * lsrm_profile_enable(1) starts (and clears), lsrm_profile_collect()
 * synchronises on the recorded events and folds them into per-kernel totals
 * (returns the number of distinct kernels, or < 0), lsrm_profile_get() reads
 * one total.  Off by default; no reference counterpart (the reference times
 * with host wall clocks, test_lrm_vol_sparse.py:1374-1401). */
void lsrm_profile_enable(int on);
int lsrm_profile_collect(void);
int lsrm_profile_get(int index, char* name, int name_cap, double* total_ms, uint64_t* launches);

/* ---------------------------------------------------------------------- */
/* Selected-block attention (the reference's NSA op)                        */
/* ---------------------------------------------------------------------- */

/* Workspace needed by lsrm_select_attn_fwd/_bwd for `topk` selections per
 * row.  `selection_rows` is total_q for per-token selection or the number of
 * query blocks when `cu_query_blocks` is used (see below). */
size_t lsrm_select_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t topk,
                                   int32_t num_query_blocks);

/* Forward of sparse/ops/triton_native_sparse_attention.py:17-41 /
 * native_sparse_attn_forward (kvcentric.py:931-1010):
 *   out [Nq,Hq,D], lse_log2 [Hq,Nq] (log2 units, as the reference's Lse).
 * block_topk: [Hkv, rows, topk] int32 sequence-local block ids (-1 = none);
 * rows = Nq (per-token selection, the reference) or the number of query blocks
 * when `cu_query_blocks` (global token offsets of query blocks, [nqb+1]) is
 * non-NULL (one selection per query block, an extension).
 * A query whose list has no valid id gets a NaN row and -inf LSE, as in the
 * reference.  A block id listed twice for one query is rejected
 * (LSRM_ERR_DUPLICATE_BLOCK in err_flags). */
int lsrm_select_attn_fwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* k,
                         const void* v, const int32_t* block_topk, int32_t topk, const int32_t* cu_query_blocks,
                         int32_t num_query_blocks, void* out, float* lse_log2, void* workspace,
                         size_t workspace_bytes, int* err_flags, void* stream);

/* Backward of NSA (kvcentric.py:1018-1263): dq, dk, dv (same dtype as q).
 * `workspace` must be the one the forward used (its selection plan is
 * reused) or freshly sized; `delta` receives rowsum(o*do) [Hq,Nq] fp32.
 * Accumulation order is fixed: dK/dV sum query tiles in ascending order. */
int lsrm_select_attn_bwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* k,
                         const void* v, const void* out, const float* lse_log2, const void* dout,
                         const int32_t* block_topk, int32_t topk, const int32_t* cu_query_blocks,
                         int32_t num_query_blocks, void* dq, void* dk, void* dv, float* delta, void* workspace,
                         size_t workspace_bytes, int* err_flags, void* stream);

/* Scratch size of lsrm_select_attn_fwd_noalloc: 16 MiB of device memory that
 * every GPU loading this library holds until the process exits. */
#define LSRM_NOALLOC_SCRATCH_BYTES (16u << 20)

/* lsrm_select_attn_fwd without allocation or caller workspace.  No
 * counterpart in the reference: it exists for callers that may not allocate
 * device memory (plugin hosts that own every device allocation, latency-bound
 * loops that must not enter the driver allocator).  Same inputs, outputs and
 * results as lsrm_select_attn_fwd; the selection plan lives in a fixed
 * LSRM_NOALLOC_SCRATCH_BYTES device array inside the library.  Problems whose
 * plan exceeds it are rejected with LSRM_ERR_WORKSPACE and a message.  The
 * array's device address differs per CUDA context, so the first call in each
 * context (each device's primary context, or a context the host made current)
 * resolves it (make that first call before any stream capture); all calls in
 * a context share the array, so calls that overlap on the GPU race on it. */
int lsrm_select_attn_fwd_noalloc(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q,
                                 const void* k, const void* v, const int32_t* block_topk, int32_t topk,
                                 const int32_t* cu_query_blocks, int32_t num_query_blocks, void* out,
                                 float* lse_log2, int* err_flags, void* stream);

/* ---------------------------------------------------------------------- */
/* Dense-range branches                                                     */
/* ---------------------------------------------------------------------- */

/* Workspace for the compressed / window / sliding-window entries.  With more
 * than one query head per kv head the dense kernels run over kv heads
 * repeated num_q_heads / num_kv_heads times (one query head each); the
 * workspace then also holds the repeated k / v and their gradients. */
size_t lsrm_dense_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode);

#define LSRM_DENSE_COMPRESSED 0 /* q vs all compressed blocks of its sequence */
#define LSRM_DENSE_INTRA_BLOCK 1 /* full attention inside each block */
#define LSRM_DENSE_SLIDING 2     /* |i-j| <= window/2 inside each sequence */

/* Compressed branch (replaces flash_attn_varlen_func(q, ck, cv,
 * cu_seqlens_q, cu_seqblocks, ..., return_attn_probs=True) at
 * sparse/module/spatial_sparse_attention.py:121-143): k/v are the compressed
 * tokens [num_blocks, Hkv, D]; keys of sequence b are rows
 * [cu_seqblocks[b], cu_seqblocks[b+1]).  lse_ln: natural-log LSE [Hq,Nq].
 * Intra-block window (sparse/ops/block_window_attention.py:14-31): q, k, v
 * are the same token sequence, segments = cu_block_include_tokens.
 * Sliding window (extension): segments = sequences, band |i-j| <= window/2. */
int lsrm_dense_attn_fwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode, int32_t window,
                        const void* q, const void* k, const void* v, void* out, float* lse, void* workspace,
                        size_t workspace_bytes, int* err_flags, void* stream);

/* Backward of the above; `lse` is what the forward returned (natural log for
 * LSRM_DENSE_COMPRESSED, log2 otherwise). */
int lsrm_dense_attn_bwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode, int32_t window,
                        const void* q, const void* k, const void* v, const void* out, const float* lse,
                        const void* dout, void* dq, void* dk, void* dv, float* delta, void* workspace,
                        size_t workspace_bytes, int* err_flags, void* stream);

/* ---------------------------------------------------------------------- */
/* Block scoring + deterministic top-k (sparse/ops/block_score.py:16-98)    */
/* ---------------------------------------------------------------------- */

/* score[h,i,b] = sum_g exp2(dot(q[i,hG+g], ck[b,h]) * float(sm_scale*1.44269504)
 *                          - lse_ln[hG+g,i] * 1.44269504f)
 * evaluated in float32 with a fixed operation order (the dot product
 * accumulates channel 0..D-1 with separately rounded multiply and add; exp2 is
 * a fixed range-reduction + degree-7 Taylor evaluation), so results are
 * reproducible bit for bit.  Top-k keeps the largest scores, ties to the
 * lowest block id, then sorts ids ascending and pads with -1.
 * Per-token: out [Hkv, Nq, topk].  With cu_query_blocks: out [Hkv, nqb,
 * topk], the score of a query block being the float32 sum of its tokens'
 * scores in ascending token order; force_self always selects block j for
 * query block j of a sequence.  `q` may be fp16/bf16 (shape->dtype); ck has
 * the same dtype; lse_ln fp32.  sm_scale <= 0 selects 1/sqrt(D); the scale
 * used is float(sm_scale * 1.44269504) evaluated in double.  Per query block
 * the scores come from tensor cores with certified error bounds and only the
 * blocks the bounds leave undecided are scored exactly (same indices); that
 * path needs `workspace` of lsrm_block_topk_workspace_bytes (the compressed
 * keys' norms and every (query block, kv head)'s score bounds, fp32); the
 * per-token path needs none (0 bytes). */
size_t lsrm_block_topk_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t topk,
                                       int32_t num_query_blocks);
int lsrm_block_topk(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* ck,
                    const float* lse_ln, int32_t topk, const int32_t* cu_query_blocks, int32_t num_query_blocks,
                    int32_t force_self, double sm_scale, int32_t* block_topk, void* workspace,
                    size_t workspace_bytes, int* err_flags, void* stream);

/* ---------------------------------------------------------------------- */
/* Compression (SpatialSparseAttentionIn, spatial_sparse_attention.py:27-67) */
/* ---------------------------------------------------------------------- */

/* out[b, c] = mean_{t in block b} x[t, c]; x [Nk, C] row stride `x_stride`,
 * out [num_blocks, C] contiguous; empty blocks give NaN (segment_reduce). */
int lsrm_block_mean_fwd(int32_t num_blocks, int32_t channels, int32_t dtype, const int32_t* cu_block_include_tokens,
                        const void* x, int64_t x_stride, void* out, void* stream);
/* dx[t, c] = dout[block(t), c] / len(block); dx [Nk, C] contiguous. */
int lsrm_block_mean_bwd(int32_t num_blocks, int32_t channels, int32_t dtype, const int32_t* cu_block_include_tokens,
                        int32_t total_tokens, const void* dout, void* dx, void* stream);

/* Non-affine LayerNorm (fp32 math) of r = x + h, the epilogue of
 * SparseResBlock (sparse/module/residual_block.py:31-34), fused with the
 * block mean: y[t] = LN(x[t]+h[t]) (optional, may be NULL) and
 * out[b] = mean_{t in b} y[t].  mean/rstd [Nk] fp32 are saved for backward. */
int lsrm_resnorm_mean_fwd(int32_t num_blocks, int32_t total_tokens, int32_t channels, int32_t dtype,
                          const int32_t* cu_block_include_tokens, const void* x, const void* h, float eps, void* y,
                          void* out, float* mean, float* rstd, void* stream);
/* Backward: given dout [nb, C] (grad of the block mean) -> dr [Nk, C] (grad
 * of x + h, same for both). */
int lsrm_resnorm_mean_bwd(int32_t num_blocks, int32_t total_tokens, int32_t channels, int32_t dtype,
                          const int32_t* cu_block_include_tokens, const void* x, const void* h, const float* mean,
                          const float* rstd, const void* dout, void* dr, void* stream);

/* ---------------------------------------------------------------------- */
/* Gated merge (SpatialSparseAttentionOut, spatial_sparse_attention.py:226-270) */
/* ---------------------------------------------------------------------- */

/* out[t, c] = sum_i sigmoid(z[t, gate_col(i, c)]) * branch_i[t, c], where z are
 * the gate logits [N, n_branch*G_w] (G_w = C for per-channel gates, Hq for
 * per-head gates whose value is shared by the D channels of a head).
 * branches: array of n_branch device pointers, each [N, C] contiguous. */
int lsrm_gate_merge_fwd(int32_t total_tokens, int32_t channels, int32_t n_branch, int32_t per_head,
                        int32_t head_dim, int32_t dtype, const void* z, const void* const* branches, void* out,
                        void* stream);
/* dz [N, n_branch*G_w] and dbranch_i [N, C]. */
int lsrm_gate_merge_bwd(int32_t total_tokens, int32_t channels, int32_t n_branch, int32_t per_head,
                        int32_t head_dim, int32_t dtype, const void* z, const void* const* branches,
                        const void* dout, void* dz, void* const* dbranches, void* stream);

/* ---------------------------------------------------------------------- */
/* Block metadata of sparse voxel sequences                                 */
/* ---------------------------------------------------------------------- */
/* Sort key of sort_volume_blocks (misc/sparse_utils.py:126-152): coords
 * [n, 4] int32 (batch, z, y, x), 16-byte aligned; keys[i] int64 orders the
 * voxels by batch, block cell (z, y, x) and position inside the cell.  The
 * caller sorts by the key (a library sort) and permutes its tensors. */
int lsrm_volume_sort_keys(int64_t n_tokens, const int32_t* coords, int32_t volume_res, int32_t block_size,
                          int64_t* keys, void* stream);

/* sort_image_blocks (misc/sparse_utils.py:95-124): keys [n] int64 of image
 * tokens coords [n, 4] int32 (batch, view, patch row, patch column) with the
 * reference's offsets (views = the view count it reads as coords[:, 1].max() + 1,
 * patch_res = input_image_res[1] / patch_size); argsort of the keys is the
 * block-major order. */
int lsrm_image_sort_keys(int64_t n_tokens, const int32_t* coords, int32_t views, int32_t patch_res,
                         int32_t block_size, int64_t* keys, void* stream);

/* compute_block_separation (misc/sparse_utils.py:592-641): coords
 * [n, dim+1] int32 (batch, then dim coordinates), grouped by batch; host
 * arrays block_size[dim], resolution[dim] (cells per dimension =
 * resolution / block_size).  Writes cu_seqlens [batch+1], cu_seqblocks
 * [batch+1], cu_block_include_tokens [num_blocks+1] (capacity n+1) and the
 * device scalar num_blocks: per batch element, the token count of every
 * non-empty cell in cell order (first coordinate most significant); cells
 * outside the grid are not counted.  Batch ids out of range set
 * LSRM_ERR_BAD_INDEX in err_flags (required). */
size_t lsrm_block_separation_workspace_bytes(int32_t dim, const int32_t* block_size, const int32_t* resolution,
                                             int32_t batch);
int lsrm_block_separation(int64_t n_tokens, const int32_t* coords, int32_t dim, const int32_t* block_size,
                          const int32_t* resolution, int32_t batch, int32_t* cu_seqlens, int32_t* cu_seqblocks,
                          int32_t* cu_block_include_tokens, int32_t* num_blocks, void* workspace,
                          size_t workspace_bytes, int* err_flags, void* stream);

/* ---------------------------------------------------------------------- */
/* Ulysses sequence <-> head exchange (sequence parallelism over W ranks)   */
/* ---------------------------------------------------------------------- */
/* Replaces the layout side of the reference's sequence-parallel exchange
 * (models_sparse/utils.py:326-474 all-gathers its KV tokens; here queries,
 * keys, values and gate logits are moved once by all_to_all_single).  A
 * rank's head slice holds hp = H/W heads (H >= W) or one head shared by
 * W/H ranks (H < W, grouped-query kv heads).  Both calls need 16-byte
 * aligned buffers and hp*D*2 a multiple of 16 bytes.
 *
 * pack:   src [n, H, D] (token stride given) -> dst [W, n, hp, D] contiguous;
 *         rank p's slice holds heads starting at (p / rep) * hp.
 * unpack: src [W, n, hp, D] -> dst [n, H, D]; the rep replicas of a head
 *         are summed in rank order in fp32 (the backward of pack). */
int lsrm_ulysses_pack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world, int32_t dtype,
                      int64_t src_token_stride, const void* src, void* dst, void* stream);
int lsrm_ulysses_unpack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world, int32_t dtype,
                        const void* src, int64_t dst_token_stride, void* dst, void* stream);

/* Geometric volume-to-volume block selection (build_volume_to_volume_attn
 * with use_3d_aware_attn, misc/sparse_utils.py:1203-1279): coords [n, 4]
 * int32 (batch, z, y, x) in block order, with cu_seqblocks [batch+1] and
 * cu_block_include_tokens from lsrm_block_separation.  Each token's point is
 * 2 * (c / (volume_res - 1) - 0.5) * radius (radius = bbox_radius * 1.05, as
 * the reference; x, y, z from columns 3, 2, 1); block centres are the fp32
 * sequential means of their tokens' points (written to centroids, scratch of
 * 3 * n floats).  block_topk [n, topk] (topk <= 64): per token the topk blocks
 * of its batch element with the smallest squared distance (ties to the lower
 * id), as sorted sequence-local ids, -1 padding.  Batch ids out of range set
 * LSRM_ERR_BAD_INDEX in err_flags (required). */
int lsrm_volume_block_topk(const int32_t* coords, int64_t n_tokens, const int32_t* cu_seqblocks,
                           const int32_t* cu_block_include_tokens, int32_t batch, int32_t volume_res, float radius,
                           int32_t topk, float* centroids, int32_t* block_topk, int* err_flags, void* stream);

/* Image-to-volume block selection (build_image_to_volume_attn with
 * use_3d_aware_attn, misc/sparse_utils.py:901-988): as lsrm_volume_block_topk,
 * but the query points are given (points [n_points, 3] float32, e.g. from
 * lsrm_image_token_points; point_coords [n_points, 4] int32 only for the batch
 * id in column 0) and the block centres come from the voxels volume_coords
 * [n_voxels, 4] in block order (centroids: scratch of 3 * n_voxels floats). */
int lsrm_points_volume_block_topk(const float* points, const int32_t* point_coords, int64_t n_points,
                                  const int32_t* volume_coords, int64_t n_voxels, const int32_t* cu_seqblocks,
                                  const int32_t* cu_block_include_tokens, int32_t batch, int32_t volume_res,
                                  float radius, int32_t topk, float* centroids, int32_t* block_topk, int* err_flags,
                                  void* stream);

/* from_volcoords_to_points (misc/sparse_utils.py:644-650): points [n, 3]
 * float32 = 2 * (c / (volume_res - 1) - 0.5) * radius for (x, y, z) = coords
 * columns (3, 2, 1), radius = bbox_radius * 1.05 as the reference passes. */
int lsrm_voxel_points(const int32_t* coords, int64_t n_tokens, int32_t volume_res, float radius, float* points,
                      void* stream);

/* ---------------------------------------------------------------------- */
/* Image-side 3D-aware attention maps (misc/sparse_utils.py:653-1200)       */
/* ---------------------------------------------------------------------- */
/* from_imcoords_to_points (:653-687): image_coords [n, 4] int32 (batch, view,
 * patch row, patch column); surface_points [B, M, S, S, 3] and surface_masks
 * [B, M, S, S] float32 (S a multiple of patch_res, the patch grid per side).
 * points [n, 3]: the surface point of the token's patch whose mask value is
 * largest (the first in row-major order on ties).  Coordinates out of range
 * set LSRM_ERR_BAD_INDEX in err_flags (required) and give (0, 0, 0). */
int lsrm_image_token_points(const int32_t* image_coords, int64_t n_tokens, const float* surface_points,
                            const float* surface_masks, int32_t batch, int32_t views, int32_t surface_res,
                            int32_t patch_res, float* points, int* err_flags, void* stream);

/* The view-block selection of build_volume_to_image_attn (:991-1200) and
 * build_image_to_image_attn (:690-898) with use_3d_aware_attn, for query
 * points [n, 3] float32 (voxel points or image-token points) whose batch id
 * is column 0 of point_coords [n, 4] int32.
 *   mask_input     view v = b * views + m at mask_input + v * mask_image_stride,
 *                  [image_h, image_w] float32, non-negative; a block of
 *                  (patch_size * block_size)^2 pixels is selected when some
 *                  value is non-zero (blocks numbered row-major per view).
 *   surface_points [B, M, S, S, 3], surface_masks [B, M, S, S] float32; a
 *                  block owns an (S / blocks per side)^2 tile of them; a point
 *                  is valid when its mask > 0.2.
 *   world_to_cam   [B, M, 4, 4] (the inverse of the camera-to-world matrix),
 *   tan_half_fov   [B, M] = tan(fov / 2), both computed by the caller with the
 *                  reference's calls; crop [B, M, 4] = (origin - 1, rows
 *                  start, columns start, crop size - 1), or NULL without crop.
 * Per view with selected blocks, the win (<= 25) blocks nearest to the
 * point's projection in block units; each candidate's value is the smallest
 * distance to its valid points, capped at max_dist when it has an invalid
 * one (max_dist when it has none).  block_topk [n, topk]: the min(C, topk)
 * smallest of the C candidates (views * win <= 512), in candidate order
 * (view, then nearness), as block ids offset by the selected-block count of
 * the earlier views; -1 padding.  Ties go to the lower position.  The
 * workspace size comes from lsrm_view_block_topk_workspace_bytes (0 for
 * unsupported geometry).  Blocks per side must be equal and divide S. */
int64_t lsrm_view_block_topk_workspace_bytes(int32_t batch, int32_t views, int32_t image_h, int32_t image_w,
                                             int32_t surface_res, int32_t patch_size, int32_t block_size, int32_t win,
                                             int64_t n_queries);
int lsrm_view_block_topk(const float* points, const int32_t* point_coords, int64_t n_queries, int32_t batch,
                         int32_t views, const float* mask_input, int64_t mask_image_stride, int32_t image_h,
                         int32_t image_w, const float* surface_points, const float* surface_masks,
                         int32_t surface_res, int32_t patch_size, int32_t block_size, const float* world_to_cam,
                         const float* tan_half_fov, const float* crop, int32_t win, int32_t topk, float max_dist,
                         int32_t* block_topk, void* workspace, int64_t workspace_bytes, int* err_flags, void* stream);

/* ---------------------------------------------------------------------- */
/* Volume output preparation (models_sparse/voldecoder.py:196-268)          */
/* ---------------------------------------------------------------------- */
/* VolTransformer.prepare_volume_output on the device, no host sync.
 * volume: [n_tokens, channels * u^3] elements of elem_bytes (2 or 4), each
 * token's features channel-major (c * u^3 + s); volume_index: [n_tokens, 4]
 * int32 (batch, z, y, x), grouped by ascending batch id in [0, batch_size),
 * coordinates in [0, vol_res), unique per batch element (the reference's
 * assumptions; a batch id without tokens gets an empty range).  Writes
 *   sparse_feat  [n_tokens * u^3, channels]: row i * u^3 + s is token i's
 *                sub-voxel s = (dz * u + dy) * u + dx,
 *   cu_seqlens   [batch_size + 1] and seqlens [batch_size], in sub-voxels,
 *   index_volume [batch_size, R, R, R] int32 (R = vol_res * u): -1, or the
 *                sequence-local row of the sub-voxel at (z*u+dz, y*u+dy, x*u+dx).
 * Out-of-range batch ids or coordinates, or tokens not grouped by batch, set
 * LSRM_ERR_BAD_INDEX in err_flags (required) and are skipped. */
int lsrm_prepare_volume_output(const void* volume, int32_t elem_bytes, const int32_t* volume_index, int64_t n_tokens,
                               int32_t channels, int32_t upsample_scale, int32_t vol_res, int32_t batch_size,
                               void* sparse_feat, int32_t* cu_seqlens, int32_t* seqlens, int32_t* index_volume,
                               int* err_flags, void* stream);

/* Per-head LayerNorm fused with the Ulysses pack (models_sparse/utils.py:
 * 21-23 LayerNorm32, :133-134 non-affine over head_dim, :239-270 q / k /
 * compressed-k normalisation before the sequence-parallel exchange).
 * pack: src [n, H, D] (token stride src_token_stride elements) ->
 *   dst [W, n, H/W, D] (rank-major head slices; W = 1: [n, H, D]), each
 *   (token, head) row normalised in fp32: (x - mean) / sqrt(var + eps),
 *   biased variance, cast back to dtype.  H % W == 0, D in 16..256 (powers
 *   of two), 16-byte aligned rows.
 * bwd: the gradient of pack: src (the same x), grad_packed [W, n, H/W, D] ->
 *   grad_src [n, H, D] contiguous (statistics recomputed from x). */
int lsrm_head_layernorm_pack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world, int32_t dtype,
                             int64_t src_token_stride, float eps, const void* src, void* dst, void* stream);
int lsrm_head_layernorm_pack_bwd(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world, int32_t dtype,
                                 int64_t src_token_stride, float eps, const void* src, const void* grad_packed,
                                 void* grad_src, void* stream);

/* Projection GEMM with the per-head LayerNorm in its epilogue: replaces
 * CrossAttention's q / k / v projections (models_sparse/utils.py:114-127,
 * q_proj_x / k_proj_x / v_proj_x, and the y side) followed by
 * _normalize_qkv's LayerNorm32 of q and k (:239-270).
 * fwd: Y = x W^T (+ bias) for x [M, K] (token stride x_token_stride
 *   elements) and W [N, K] bf16 (the Linears' weights stacked), fp32
 *   accumulation on the tensor cores.  The N columns are the segments in
 *   order; segment s writes its columns of bf16(Y) to `out` and/or the
 *   per-head LayerNorm of bf16(Y) (non-affine over head_dim columns, fp32
 *   statistics, biased variance, eps) to `out_norm`, each [M, cols]
 *   contiguous and 16-byte aligned, and 1/std of each normalised head to
 *   rstd [M, N / head_dim].  K a multiple of 64, head_dim 32 or 64, up to 4
 *   segments.  err_flags required (a bounded wait that ran out sets
 *   LSRM_ERR_TIMEOUT).
 * bwd: grad_pre [M, N] bf16 = the gradient of Y given, per segment, the
 *   gradient of `out` (grad_out) and/or of `out_norm` (grad_norm, with the
 *   forward's out_norm and rstd); any of them may be NULL.  The input and
 *   weight gradients are then grad_pre W and grad_pre^T x. */
typedef struct {
  int32_t cols;     /* GEMM columns of this segment, a multiple of head_dim */
  int32_t reserved;
  void* out;        /* [M, cols] bf16 result, or NULL */
  void* out_norm;   /* [M, cols] bf16 per-head LayerNorm of the result, or NULL */
} lsrm_qkv_segment;

typedef struct {
  int32_t cols;
  int32_t reserved;
  const void* out_norm;   /* the forward's normalised output (needed with grad_norm) */
  const void* grad_out;   /* gradient of the raw output, or NULL */
  const void* grad_norm;  /* gradient of the normalised output, or NULL */
} lsrm_qkv_grad_segment;

int lsrm_qkv_norm_fwd(int64_t M, int32_t K, int32_t N, int32_t head_dim, const void* x, int64_t x_token_stride,
                      const void* w, const void* bias, const lsrm_qkv_segment* segs, int32_t n_segs, float eps,
                      float* rstd, int* err_flags, void* stream);
int lsrm_qkv_norm_bwd(int64_t M, int32_t N, int32_t head_dim, const lsrm_qkv_grad_segment* segs, int32_t n_segs,
                      const float* rstd, void* grad_pre, void* stream);

/* ---------------------------------------------------------------------- */
/* Self-test of the tcgen05 / TMA building blocks (used by the GPU tests)   */
/* ---------------------------------------------------------------------- */
/* a, b, v: [128, D] bf16; p: [128, 128] bf16; c1 = a @ b^T [128,128] fp32,
 * c2 = p @ v [128, D] fp32.  D = 32 or 64. */
int lsrm_umma_selftest(int32_t head_dim, const void* a, const void* b, const void* p, const void* v, float* c1,
                       float* c2, int* err_flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LSRM_SPARSE_H_ */
