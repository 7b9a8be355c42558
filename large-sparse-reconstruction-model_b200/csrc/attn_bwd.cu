// Host entry points of the backward attention paths.
#include <algorithm>

#include "attn_bwd.cuh"
#include "attn_host.h"
#include "host_util.h"

namespace lsrm {

// Sums the split partials of dK/dV in split order (deterministic) and casts.
constexpr int kReduceRows = 16;
template <bool BF16, int D>
__global__ void dkdv_reduce_kernel_d(DkvParams p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  // grid (KV tile, kv head, 2 x row groups of kReduceRows): every thread sums
  // 4 consecutive channels of one row over the splits, in split order
  const int kt_idx = blockIdx.x, h = blockIdx.y, which = blockIdx.z & 1, rg = blockIdx.z >> 1;
  if (kt_idx >= *p.n_kvtiles) return;
  const QTile kt = p.kvtiles[kt_idx];
  T* out = static_cast<T*>(which == 0 ? p.dk : p.dv);
  const size_t split_stride = (size_t)p.hkv * p.kvtiles_ub * 128 * D;
  const float* base = p.partial + ((((size_t)which * p.n_split) * p.hkv + h) * p.kvtiles_ub + kt_idx) * 128 * D;
  const int r_end = min(kt.n_q, (rg + 1) * kReduceRows);
  for (int i = threadIdx.x; i < kReduceRows * D / 4; i += blockDim.x) {
    const int r = rg * kReduceRows + (i * 4) / D, d = (i * 4) % D;
    if (r >= r_end) break;
    const float* src = base + (size_t)r * D + d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < p.n_split; ++sp) {
      const float4 x = *reinterpret_cast<const float4*>(src + sp * split_stride);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    T* o = out + (size_t)(kt.q_start + r) * p.kv_tok_stride + (size_t)h * D + d;
    o[0] = (T)acc.x;
    o[1] = (T)acc.y;
    o[2] = (T)acc.z;
    o[3] = (T)acc.w;
  }
}

// Select mode: dK / dV of every item that was cut into pieces = the sum of
// its pieces' fp32 slots in piece order (deterministic), cast.  grid (split
// item, 2 x row groups of kReduceRows).
template <bool BF16, int D>
__global__ void dkdv_piece_reduce_kernel(DkvParams p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int k = blockIdx.x;
  if (k >= p.sched_ctr[2]) return;
  const int4 si = p.split_items[k];
  const int item = si.x, slot0 = si.y, pieces = si.z;
  if (!dcheck(item >= 0 && item < p.hkv * p.kvtiles_ub && slot0 >= 0 && pieces >= 1 &&
                  slot0 + pieces <= p.piece_slots,
              kDcChunks, p.err))
    return;
  const int h = item / p.kvtiles_ub, kt_idx = item - h * p.kvtiles_ub;
  const QTile kt = p.kvtiles[kt_idx];
  const int which = blockIdx.y & 1, rg = blockIdx.y >> 1;
  T* out = static_cast<T*>(which == 0 ? p.dk : p.dv);
  const int r_end = min(kt.n_q, (rg + 1) * kReduceRows);
  for (int i = threadIdx.x; i < kReduceRows * D / 4; i += blockDim.x) {
    const int r = rg * kReduceRows + (i * 4) / D, d = (i * 4) % D;
    if (r >= r_end) break;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int pc = 0; pc < pieces; ++pc) {
      const float4 x = *reinterpret_cast<const float4*>(p.piece_partial +
                                                        (((size_t)(slot0 + pc) * 2 + which) * 128 + r) * D + d);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    T* o = out + (size_t)(kt.q_start + r) * p.kv_tok_stride + (size_t)h * D + d;
    o[0] = (T)acc.x;
    o[1] = (T)acc.y;
    o[2] = (T)acc.z;
    o[3] = (T)acc.w;
  }
}

// Zeroes rows [*start, total) of dk and dv (tokens outside every KV tile).
__global__ void zero_tail_kernel(uint16_t* dk, uint16_t* dv, const int32_t* start, long long total, long long stride,
                                 int row_elems) {
  const long long s = *start;
  const long long n = (total - s) * (long long)row_elems;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = s + i / row_elems, c = i % row_elems;
    dk[r * stride + c] = 0;
    dv[r * stride + c] = 0;
  }
}

template <int D, bool BF16, int MODE>
static int launch_dq_t(const CUtensorMap& mq, const CUtensorMap& mdo, const KVMaps& kv, const DqParams& p, int grid_x,
                       int hkv, cudaStream_t s) {
  constexpr int STAGES = 6;
  using L = DqSmem<D, STAGES>;
  auto kern = attn_dq_kernel<D, BF16, MODE, STAGES>;
  LSRM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
  ProfScope ps(MODE == kSelect ? "attn_dq_select" : (MODE == kBand ? "attn_dq_sliding" : "attn_dq_range"), s);
  // persistent: one CTA per SM walks the (tile, head) items
  DqParams pp = p;
  pp.hkv = hkv;
  const int grid = (int)std::min<long long>((long long)grid_x * hkv, num_sms());
  kern<<<dim3(grid, 1), kDqThreads, L::ALLOC, s>>>(mq, mdo, kv, pp);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

template <int MODE>
static int launch_dq(int D, bool bf16, const CUtensorMap& mq, const CUtensorMap& mdo, const KVMaps& kv,
                     const DqParams& p, int grid_x, int hkv, cudaStream_t s) {
  if (grid_x <= 0) return LSRM_OK;
  if (D == 64)
    return bf16 ? launch_dq_t<64, true, MODE>(mq, mdo, kv, p, grid_x, hkv, s)
                : launch_dq_t<64, false, MODE>(mq, mdo, kv, p, grid_x, hkv, s);
  if (D == 16)
    return bf16 ? launch_dq_t<16, true, MODE>(mq, mdo, kv, p, grid_x, hkv, s)
                : launch_dq_t<16, false, MODE>(mq, mdo, kv, p, grid_x, hkv, s);
  return bf16 ? launch_dq_t<32, true, MODE>(mq, mdo, kv, p, grid_x, hkv, s)
              : launch_dq_t<32, false, MODE>(mq, mdo, kv, p, grid_x, hkv, s);
}

template <int D, bool BF16, int MODE>
static int launch_dkdv_t(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const CUtensorMap& mdo,
                         const QMaps& qm, const DkvParams& p, int grid_x, int hkv, cudaStream_t s) {
  constexpr int STAGES = 6;
  using L = DkvSmem<D, STAGES>;
  auto kern = attn_dkdv_kernel<D, BF16, MODE, STAGES>;
  LSRM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
  DkvParams pp = p;
  pp.hkv = hkv;
  {
    ProfScope ps(MODE == kSelect ? "attn_dkdv_select" : (MODE == kBand ? "attn_dkdv_sliding" : "attn_dkdv_range"), s);
    // persistent: one CTA per SM walks the work items
    const long long items = p.kv_sched ? (long long)grid_x * hkv + p.piece_slots : (long long)grid_x * hkv * p.n_split;
    const int grid = (int)std::min<long long>(items, num_sms());
    kern<<<dim3(grid, 1), kDkvThreads, L::ALLOC, s>>>(mk, mv, mq, mdo, qm, pp);
    LSRM_LAUNCH_CHECK();
  }
  if (p.kv_sched && p.piece_slots > 0) {
    ProfScope ps("dkdv_piece_reduce", s);
    dkdv_piece_reduce_kernel<BF16, D>
        <<<dim3(std::max(p.piece_slots / 2, 1), 2 * (128 / kReduceRows)), 256, 0, s>>>(pp);
    LSRM_LAUNCH_CHECK();
  }
  if (p.n_split > 1) {
    ProfScope ps("dkdv_split_reduce", s);
    dkdv_reduce_kernel_d<BF16, D><<<dim3(grid_x, hkv, 2 * (128 / kReduceRows)), 256, 0, s>>>(p);
    LSRM_LAUNCH_CHECK();
  }
  return LSRM_OK;
}

template <int MODE>
static int launch_dkdv(int D, bool bf16, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq,
                       const CUtensorMap& mdo, const QMaps& qm, const DkvParams& p, int grid_x, int hkv,
                       cudaStream_t s) {
  if (grid_x <= 0) return LSRM_OK;
  if (D == 64)
    return bf16 ? launch_dkdv_t<64, true, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s)
                : launch_dkdv_t<64, false, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s);
  if (D == 16)
    return bf16 ? launch_dkdv_t<16, true, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s)
                : launch_dkdv_t<16, false, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s);
  return bf16 ? launch_dkdv_t<32, true, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s)
              : launch_dkdv_t<32, false, MODE>(mk, mv, mq, mdo, qm, p, grid_x, hkv, s);
}

static int launch_zero_tail(void* dk, void* dv, const int32_t* start, long long total, long long stride,
                            int row_elems, cudaStream_t s) {
  ProfScope ps("zero_tail", s);
  zero_tail_kernel<<<148, 256, 0, s>>>(static_cast<uint16_t*>(dk), static_cast<uint16_t*>(dv), start, total, stride,
                                       row_elems);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

// Split factor of the dense-branch dK/dV: enough CTAs to fill the GPU when
// few KV tiles exist (the compressed branch), at least 16 chunks per split.
static int dense_split(const lsrm_varlen* m, const lsrm_attn_shape* sh, int mode, int kvtiles_ub) {
  if (mode != LSRM_DENSE_COMPRESSED) return 1;
  const int G = sh->num_q_heads / sh->num_kv_heads;
  const int qpc = kKvQRows / G;
  // compressed keys are few (one per block): split every KV tile's queries
  // so that the grid is ~16 waves of 148 SMs (balanced), partial sums are
  // reduced in a fixed order afterwards
  const long long ctas = (long long)std::max(m->num_blocks / kRows + m->num_seqs, 1) * sh->num_kv_heads;
  int n = (int)std::min<long long>(32, (16 * 148 + ctas - 1) / ctas);
  const long long chunks_per_seq = std::max<long long>(1, (long long)m->total_q / std::max(m->num_seqs, 1) / qpc);
  n = (int)std::max<long long>(1, std::min<long long>(n, chunks_per_seq / 16));
  (void)kvtiles_ub;
  return n;
}

size_t dense_bwd_extra_bytes(const lsrm_varlen* m, const lsrm_attn_shape* sh, int mode) {
  int G = sh->num_q_heads / std::max(sh->num_kv_heads, 1);
  DensePlan p = make_dense_plan(m, G, mode, nullptr);
  const int n = dense_split(m, sh, mode, p.kvtiles_ub);
  if (n <= 1) return 0;
  return 2ull * n * sh->num_kv_heads * (size_t)p.kvtiles_ub * kRows * sh->head_dim * sizeof(float);
}

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_select_attn_bwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q,
                                    const void* k, const void* v, const void* out, const float* lse_log2,
                                    const void* dout, const int32_t* block_topk, int32_t topk,
                                    const int32_t* cu_query_blocks, int32_t num_query_blocks, void* dq, void* dk,
                                    void* dv, float* delta, void* workspace, size_t workspace_bytes, int* err_flags,
                                    void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(G <= 64, "the backward supports up to 64 query heads per kv head (got %d)", G);
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(num_query_blocks == 0 || cu_query_blocks, "num_query_blocks > 0 needs cu_query_blocks");
  const size_t need = lsrm_select_workspace_bytes(meta, shape, topk, num_query_blocks);
  if (workspace_bytes < need || !workspace) {
    set_error("workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int D = shape->head_dim, hkv = shape->num_kv_heads;
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  const int row_elems = hkv * D;
  if (meta->total_q == 0) {
    if (meta->total_k > 0) {
      LSRM_CUDA_TRY(cudaMemsetAsync(dk, 0, (size_t)meta->total_k * shape->kv_token_stride * 2, s));
      LSRM_CUDA_TRY(cudaMemsetAsync(dv, 0, (size_t)meta->total_k * shape->kv_token_stride * 2, s));
    }
    return LSRM_OK;
  }
  SelectPlan plan = make_select_plan(meta, G, hkv, topk, num_query_blocks, workspace);
  int* err = err_flags ? err_flags : reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + plan.bytes);
  const int qpt = kRows / G;
  const bool qblock = num_query_blocks > 0;
  if ((rc = launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, qblock ? kTilesQBlock : kTilesSeq, qpt, meta,
                               cu_query_blocks, qblock ? num_query_blocks : meta->num_seqs, 0, err, s)))
    return rc;
  if ((rc = launch_build_unions(plan, meta, block_topk, topk, qblock ? num_query_blocks : meta->total_q, G, err, s)))
    return rc;
  if ((rc = launch_build_reverse(plan, err, s))) return rc;
  if ((rc = launch_build_tiles(plan.kvtiles, plan.n_kvtiles, plan.kvtiles_ub, kTilesKVBlock, kRows, meta, nullptr,
                               meta->num_blocks, 0, err, s)))
    return rc;
  if ((rc = launch_build_kv_schedule(plan, G, num_sms(), s))) return rc;
  const float scale = softmax_scale_of(shape);
  // dQ (+ delta)
  {
    CUtensorMap mq, mdo;
    KVMaps kv;
    if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt))) return rc;
    if ((rc = make_tmap_3d(&mdo, dout, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt)))
      return rc;
    if ((rc = make_kv_maps(kv.k, kv.v, kNumBoxes, k, v, D, hkv, meta->total_k, shape->kv_token_stride))) return rc;
    DqParams p{};
    p.tiles = plan.tiles;
    p.n_tiles = plan.n_tiles;
    p.union_cnt = plan.union_cnt;
    p.union_ngroups = plan.union_ngroups;
    p.union_blk = plan.union_blk;
    p.union_mask = plan.union_mask;
    p.tiles_ub = plan.tiles_ub;
    p.union_cap = plan.union_cap;
    p.cu_block_include_tokens = meta->cu_block_include_tokens;
    p.num_blocks = meta->num_blocks;
    p.out = out;
    p.dout = dout;
    p.lse = lse_log2;
    p.delta = delta;
    p.dq = dq;
    p.q_tok_stride = shape->q_token_stride;
    p.total_q = meta->total_q;
    p.total_k = meta->total_k;
    p.G = G;
    p.scale_log2 = scale * 1.44269504f;
    p.scale = scale;
    p.err = err;
    if ((rc = launch_dq<kSelect>(D, bf16, mq, mdo, kv, p, plan.tiles_ub, hkv, s))) return rc;
  }
  // dK, dV
  {
    CUtensorMap mk, mv;
    if ((rc = make_tmap_3d(&mk, k, D, hkv, meta->total_k, shape->kv_token_stride, 1, kRows))) return rc;
    if ((rc = make_tmap_3d(&mv, v, D, hkv, meta->total_k, shape->kv_token_stride, 1, kRows))) return rc;
    DkvParams p{};
    p.q = q;
    p.dout = dout;
    p.q_tok_stride = shape->q_token_stride;
    p.kvtiles = plan.kvtiles;
    p.n_kvtiles = plan.n_kvtiles;
    p.kvtiles_ub = plan.kvtiles_ub;
    p.qtiles = plan.tiles;
    p.rev_off = plan.rev_off;
    p.rev_entries = plan.rev_entries;
    p.union_mask = plan.union_mask;
    p.tiles_ub = plan.tiles_ub;
    p.union_cap = plan.union_cap;
    p.num_blocks = meta->num_blocks;
    p.lse = lse_log2;
    p.delta = delta;
    p.dk = dk;
    p.dv = dv;
    p.partial = nullptr;
    p.n_split = 1;
    p.kv_sched = plan.kv_sched;
    p.item_nch = plan.item_nch;
    p.item_rng = plan.item_rng;
    p.item_src = plan.item_src;
    p.piece_partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.bytes + 256);
    p.split_items = plan.split_items;
    p.sched_ctr = plan.sched_ctr;
    p.piece_slots = plan.piece_slots;
    p.kv_tok_stride = shape->kv_token_stride;
    p.total_q = meta->total_q;
    p.total_k = meta->total_k;
    p.G = G;
    p.hkv = hkv;
    p.scale_log2 = scale * 1.44269504f;
    p.scale = scale;
    p.err = err;
    // query rows: TMA boxes of whole query windows (G <= 8), else cp.async gathers
    QMaps qm;
    for (int i = 0; i < 4; ++i) {
      if (G <= 8) {
        if ((rc = make_tmap_3d(&qm.q[i], q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G,
                               (8 / G) << i)))
          return rc;
        if ((rc = make_tmap_3d(&qm.dout[i], dout, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G,
                               (8 / G) << i)))
          return rc;
      } else {
        qm.q[i] = mk;
        qm.dout[i] = mv;
      }
    }
    if ((rc = launch_dkdv<kSelect>(D, bf16, mk, mv, mk, mv, qm, p, plan.kvtiles_ub, hkv, s))) return rc;
  }
  return launch_zero_tail(dk, dv, meta->cu_block_include_tokens + meta->num_blocks, meta->total_k,
                          shape->kv_token_stride, row_elems, s);
}

namespace lsrm {

// dk / dv [n, hkv, D] (row stride `stride`) = sum over the R copies of each
// kv head in src [n, hkv * R, D], in copy order, fp32.
template <typename T>
__global__ void sum_kv_head_copies_kernel(const T* __restrict__ src, T* __restrict__ dst, long long stride,
                                          long long n, int hkv, int R, int D) {
  const long long total = n * hkv * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int h = (int)((i / D) % hkv);
    const long long t = i / ((long long)D * hkv);
    const T* row = src + ((t * hkv + h) * R) * (long long)D + d;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc += (float)row[(long long)r * D];
    dst[t * stride + (long long)h * D + d] = (T)acc;
  }
}

static int sum_kv_head_copies(const void* src, void* dst, long long stride, long long n, int hkv, int R, int D,
                              bool bf16, cudaStream_t s) {
  if (n <= 0) return LSRM_OK;
  const long long total = n * hkv * D;
  const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  ProfScope ps("dense_regroup", s);
  if (bf16)
    sum_kv_head_copies_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(src),
                                                                  static_cast<__nv_bfloat16*>(dst), stride, n, hkv, R,
                                                                  D);
  else
    sum_kv_head_copies_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(src), static_cast<__half*>(dst),
                                                           stride, n, hkv, R, D);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

// The dense backward with at most kDenseMaxG query heads per kv head; the
// workspace holds `need` bytes (dense_ws_direct).
static int dense_bwd_direct(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode, int window,
                            const void* q, const void* k, const void* v, const void* out, const float* lse,
                            const void* dout, void* dq, void* dk, void* dv, float* delta, void* workspace,
                            size_t need, int* err_flags, cudaStream_t s) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(G <= kDenseMaxG, "dense kernels take at most %d query heads per kv head (got %d)", kDenseMaxG, G);
  const int D = shape->head_dim, hkv = shape->num_kv_heads;
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  const long long nk = (mode == LSRM_DENSE_COMPRESSED) ? meta->num_blocks : meta->total_k;
  const int row_elems = hkv * D;
  DensePlan plan = make_dense_plan(meta, G, mode, workspace);
  uint8_t* extra = static_cast<uint8_t*>(workspace) + plan.bytes;
  int* err = err_flags ? err_flags : reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + need - 256);
  if ((rc = dense_fwd_tiles(meta, G, mode, window, plan, err, s))) return rc;
  const int kind = mode == LSRM_DENSE_COMPRESSED ? kTilesCompressed
                   : mode == LSRM_DENSE_INTRA_BLOCK ? kTilesKVBlock
                                                    : kTilesKVSeq;
  const int nseg = mode == LSRM_DENSE_INTRA_BLOCK ? meta->num_blocks : meta->num_seqs;
  if ((rc = launch_build_tiles(plan.kvtiles, plan.n_kvtiles, plan.kvtiles_ub, kind, kRows, meta, nullptr, nseg,
                               mode == LSRM_DENSE_SLIDING ? window : 0, err, s)))
    return rc;
  const float scale = softmax_scale_of(shape);
  const int qpt = kRows / G;
  {
    CUtensorMap mq, mdo;
    KVMaps kv;
    if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt))) return rc;
    if ((rc = make_tmap_3d(&mdo, dout, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt)))
      return rc;
    if ((rc = make_kv_maps(kv.k, kv.v, kNumBoxes, k, v, D, hkv, nk, shape->kv_token_stride))) return rc;
    DqParams p{};
    p.tiles = plan.tiles;
    p.n_tiles = plan.n_tiles;
    p.out = out;
    p.dout = dout;
    p.lse = lse;
    p.delta = delta;
    p.dq = dq;
    p.q_tok_stride = shape->q_token_stride;
    p.total_q = meta->total_q;
    p.total_k = (int)nk;
    p.G = G;
    p.scale_log2 = scale * 1.44269504f;
    p.scale = scale;
    p.half_window = window / 2;
    p.lse_natural = mode == LSRM_DENSE_COMPRESSED;
    p.err = err;
    rc = (mode == LSRM_DENSE_SLIDING) ? launch_dq<kBand>(D, bf16, mq, mdo, kv, p, plan.tiles_ub, hkv, s)
                                      : launch_dq<kRange>(D, bf16, mq, mdo, kv, p, plan.tiles_ub, hkv, s);
    if (rc) return rc;
  }
  {
    CUtensorMap mk, mv, mq, mdo;
    const int qpc = kKvQRows / G;
    if ((rc = make_tmap_3d(&mk, k, D, hkv, nk, shape->kv_token_stride, 1, kRows))) return rc;
    if ((rc = make_tmap_3d(&mv, v, D, hkv, nk, shape->kv_token_stride, 1, kRows))) return rc;
    if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpc))) return rc;
    if ((rc = make_tmap_3d(&mdo, dout, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpc)))
      return rc;
    DkvParams p{};
    p.q = q;
    p.dout = dout;
    p.q_tok_stride = shape->q_token_stride;
    p.kvtiles = plan.kvtiles;
    p.n_kvtiles = plan.n_kvtiles;
    p.kvtiles_ub = plan.kvtiles_ub;
    p.lse = lse;
    p.delta = delta;
    p.dk = dk;
    p.dv = dv;
    p.n_split = dense_split(meta, shape, mode, plan.kvtiles_ub);
    p.partial = p.n_split > 1 ? reinterpret_cast<float*>(extra) : nullptr;
    p.kv_tok_stride = shape->kv_token_stride;
    p.total_q = meta->total_q;
    p.total_k = (int)nk;
    p.G = G;
    p.hkv = hkv;
    p.scale_log2 = scale * 1.44269504f;
    p.scale = scale;
    p.half_window = window / 2;
    p.lse_natural = mode == LSRM_DENSE_COMPRESSED;
    p.err = err;
    QMaps qm;  // unused by the dense branches
    for (int i = 0; i < 4; ++i) {
      qm.q[i] = mq;
      qm.dout[i] = mdo;
    }
    rc = (mode == LSRM_DENSE_SLIDING) ? launch_dkdv<kBand>(D, bf16, mk, mv, mq, mdo, qm, p, plan.kvtiles_ub, hkv, s)
                                      : launch_dkdv<kRange>(D, bf16, mk, mv, mq, mdo, qm, p, plan.kvtiles_ub, hkv, s);
    if (rc) return rc;
  }
  const int32_t* start = mode == LSRM_DENSE_COMPRESSED   ? meta->cu_seqblocks + meta->num_seqs
                         : mode == LSRM_DENSE_INTRA_BLOCK ? meta->cu_block_include_tokens + meta->num_blocks
                                                          : meta->cu_seqlens_k + meta->num_seqs;
  return launch_zero_tail(dk, dv, start, nk, shape->kv_token_stride, row_elems, s);
}

}  // namespace lsrm

extern "C" int lsrm_dense_attn_bwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode,
                                   int32_t window, const void* q, const void* k, const void* v, const void* out,
                                   const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta,
                                   void* workspace, size_t workspace_bytes, int* err_flags, void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(G <= 64, "the backward supports up to 64 query heads per kv head (got %d)", G);
  LSRM_CHECK_ARG(mode >= 0 && mode <= 2, "unknown dense mode %d", mode);
  LSRM_CHECK_ARG(mode == LSRM_DENSE_COMPRESSED || meta->total_q == meta->total_k,
                 "window branches attend inside one token sequence (total_q == total_k)");
  const size_t need = lsrm_dense_workspace_bytes(meta, shape, mode);
  if (workspace_bytes < need || !workspace) {
    set_error("workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long nk = (mode == LSRM_DENSE_COMPRESSED) ? meta->num_blocks : meta->total_k;
  if (meta->total_q == 0) {
    if (nk > 0) {
      LSRM_CUDA_TRY(cudaMemsetAsync(dk, 0, (size_t)nk * shape->kv_token_stride * 2, s));
      LSRM_CUDA_TRY(cudaMemsetAsync(dv, 0, (size_t)nk * shape->kv_token_stride * 2, s));
    }
    return LSRM_OK;
  }
  if (G <= kDenseMaxG)
    return dense_bwd_direct(meta, shape, mode, window, q, k, v, out, lse, dout, dq, dk, dv, delta, workspace, need,
                            err_flags, s);
  // regrouped as in the forward: repeated kv heads in, their gradients summed
  // back per kv head afterwards
  const DenseRegroup r = dense_regroup(meta, shape, mode);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  void* k2 = base + r.inner;
  void* v2 = base + r.inner + r.buf;
  void* dk2 = base + r.inner + 2 * r.buf;
  void* dv2 = base + r.inner + 3 * r.buf;
  const int hkv = shape->num_kv_heads, D = shape->head_dim;
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  if ((rc = repeat_kv_heads(k, shape->kv_token_stride, k2, r.nk, hkv, r.R, D, s))) return rc;
  if ((rc = repeat_kv_heads(v, shape->kv_token_stride, v2, r.nk, hkv, r.R, D, s))) return rc;
  if ((rc = dense_bwd_direct(meta, &r.shape, mode, window, q, k2, v2, out, lse, dout, dq, dk2, dv2, delta, workspace,
                             r.inner, err_flags, s)))
    return rc;
  if ((rc = sum_kv_head_copies(dk2, dk, shape->kv_token_stride, r.nk, hkv, r.R, D, bf16, s))) return rc;
  return sum_kv_head_copies(dv2, dv, shape->kv_token_stride, r.nk, hkv, r.R, D, bf16, s);
}
