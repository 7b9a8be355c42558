// Host entry points of the forward attention paths.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "attn_fwd.cuh"
#include "attn_host.h"
#include "host_util.h"

namespace lsrm {

template <int D, bool BF16, int MODE>
static int launch_fwd_t(const CUtensorMap& mq, const KVMaps& kv, const FwdParams& p, int grid_x, int hkv,
                        cudaStream_t s) {
  constexpr int STAGES = 5;
  using L = FwdSmem<D, STAGES>;
  auto kern = attn_fwd_kernel<D, BF16, MODE, STAGES>;
  LSRM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
  ProfScope ps(MODE == kSelect ? "attn_fwd_select" : (MODE == kBand ? "attn_fwd_sliding" : "attn_fwd_range"), s);
  // persistent: one CTA per SM walks the (tile, head) items
  FwdParams pp = p;
  pp.hkv = hkv;
  const long long items_ub = (long long)grid_x * hkv;
  const int grid = (int)std::min<long long>(items_ub, num_sms());
  kern<<<dim3(grid, 1), kFwdThreads, L::ALLOC, s>>>(mq, kv, pp);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

template <int MODE>
static int launch_fwd(int D, bool bf16, const CUtensorMap& mq, const KVMaps& kv, const FwdParams& p, int grid_x,
                      int hkv, cudaStream_t s) {
  if (grid_x <= 0) return LSRM_OK;
  if (D == 64) {
    return bf16 ? launch_fwd_t<64, true, MODE>(mq, kv, p, grid_x, hkv, s)
                : launch_fwd_t<64, false, MODE>(mq, kv, p, grid_x, hkv, s);
  }
  if (D == 16)
    return bf16 ? launch_fwd_t<16, true, MODE>(mq, kv, p, grid_x, hkv, s)
                : launch_fwd_t<16, false, MODE>(mq, kv, p, grid_x, hkv, s);
  return bf16 ? launch_fwd_t<32, true, MODE>(mq, kv, p, grid_x, hkv, s)
              : launch_fwd_t<32, false, MODE>(mq, kv, p, grid_x, hkv, s);
}

int check_shape(const lsrm_varlen* m, const lsrm_attn_shape* sh, int& G) {
  LSRM_CHECK_ARG(m && sh, "null metadata / shape");
  LSRM_CHECK_ARG(sh->head_dim == 16 || sh->head_dim == 32 || sh->head_dim == 64, "head_dim must be 16, 32 or 64 (got %d)",
                 sh->head_dim);
  LSRM_CHECK_ARG(sh->dtype == LSRM_DTYPE_BF16 || sh->dtype == LSRM_DTYPE_F16, "dtype must be bf16 or fp16");
  LSRM_CHECK_ARG(sh->num_kv_heads > 0 && sh->num_q_heads % sh->num_kv_heads == 0,
                 "num_q_heads (%d) must be a multiple of num_kv_heads (%d)", sh->num_q_heads, sh->num_kv_heads);
  G = sh->num_q_heads / sh->num_kv_heads;
  LSRM_CHECK_ARG(G <= 128 && (G & (G - 1)) == 0, "query heads per kv head (%d) must be a power of two <= 128", G);
  LSRM_CHECK_ARG(m->num_seqs >= 1 && m->total_q >= 0 && m->total_k >= 0 && m->num_blocks >= 0, "bad varlen sizes");
  LSRM_CHECK_ARG(sh->q_token_stride >= (int64_t)sh->num_q_heads * sh->head_dim, "q token stride too small");
  LSRM_CHECK_ARG(sh->kv_token_stride >= (int64_t)sh->num_kv_heads * sh->head_dim, "kv token stride too small");
  return LSRM_OK;
}

float softmax_scale_of(const lsrm_attn_shape* sh) {
  return sh->softmax_scale > 0.f ? sh->softmax_scale : 1.0f / std::sqrt((float)sh->head_dim);
}

}  // namespace lsrm

using namespace lsrm;

extern "C" size_t lsrm_select_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t topk,
                                              int32_t num_query_blocks) {
  int G = 1;
  if (check_shape(meta, shape, G) != LSRM_OK || topk < 1) return 0;
  SelectPlan p = make_select_plan(meta, G, shape->num_kv_heads, topk, num_query_blocks, nullptr);
  return p.bytes + 256 + piece_partial_bytes(p, shape->head_dim);  // + internal error word, dK/dV pieces
}

extern "C" int lsrm_select_attn_fwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q,
                                    const void* k, const void* v, const int32_t* block_topk, int32_t topk,
                                    const int32_t* cu_query_blocks, int32_t num_query_blocks, void* out,
                                    float* lse_log2, void* workspace, size_t workspace_bytes, int* err_flags,
                                    void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(num_query_blocks == 0 || cu_query_blocks, "num_query_blocks > 0 needs cu_query_blocks");
  const size_t need = lsrm_select_workspace_bytes(meta, shape, topk, num_query_blocks);
  if (workspace_bytes < need || !workspace) {
    set_error("workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  if (meta->total_q == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SelectPlan plan = make_select_plan(meta, G, shape->num_kv_heads, topk, num_query_blocks, workspace);
  int* err = err_flags ? err_flags : reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + plan.bytes);
  const int qpt = kRows / G;
  const bool qblock = num_query_blocks > 0;
  if ((rc = launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, qblock ? kTilesQBlock : kTilesSeq, qpt, meta,
                               cu_query_blocks, qblock ? num_query_blocks : meta->num_seqs, 0, err, s)))
    return rc;
  if ((rc = launch_build_unions(plan, meta, block_topk, topk, qblock ? num_query_blocks : meta->total_q, G, err, s)))
    return rc;
  const int D = shape->head_dim;
  CUtensorMap mq;
  KVMaps kv;
  if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt))) return rc;
  if ((rc = make_kv_maps(kv.k, kv.v, kNumBoxes, k, v, D, shape->num_kv_heads, meta->total_k, shape->kv_token_stride)))
    return rc;
  FwdParams p{};
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
  p.lse = lse_log2;
  p.q_tok_stride = shape->q_token_stride;
  p.num_q_heads = shape->num_q_heads;
  p.total_q = meta->total_q;
  p.total_k = meta->total_k;
  p.G = G;
  p.scale_log2 = softmax_scale_of(shape) * 1.44269504f;
  p.half_window = 0;
  p.lse_natural = 0;
  p.err = err;
  return launch_fwd<kSelect>(D, shape->dtype == LSRM_DTYPE_BF16, mq, kv, p, plan.tiles_ub, shape->num_kv_heads, s);
}

namespace lsrm {

// Workspace of the dense kernels run directly (G <= kDenseMaxG).
size_t dense_ws_direct(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode) {
  int G = 1;
  if (check_shape(meta, shape, G) != LSRM_OK) return 0;
  DensePlan p = make_dense_plan(meta, G, mode, nullptr);
  return p.bytes + dense_bwd_extra_bytes(meta, shape, mode) + 256;
}

DenseRegroup dense_regroup(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode) {
  DenseRegroup r{};
  r.shape = *shape;
  const int G = shape->num_q_heads / shape->num_kv_heads;
  r.R = G > kDenseMaxG ? G / kDenseMaxG : 1;
  r.nk = (mode == LSRM_DENSE_COMPRESSED) ? meta->num_blocks : meta->total_k;
  if (r.R > 1) {
    r.shape.num_kv_heads = shape->num_kv_heads * r.R;
    r.shape.kv_token_stride = (int64_t)r.shape.num_kv_heads * shape->head_dim;
  }
  r.inner = align_up(dense_ws_direct(meta, &r.shape, mode), 256);
  r.buf = align_up((size_t)std::max<long long>(r.nk, 1) * r.shape.num_kv_heads * shape->head_dim * 2, 256);
  return r;
}

// k / v [n, hkv, D] (row stride `stride` elements) -> [n, hkv * R, D] with
// head h copied to heads h*R .. h*R+R-1; 16-byte moves.
__global__ void repeat_kv_heads_kernel(const uint4* __restrict__ src, long long stride_v, uint4* __restrict__ dst,
                                       long long n, int hkv, int R, int vpr) {
  const long long total = n * hkv * R * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % vpr);
    const long long hr = i / vpr;
    const int h = (int)((hr / R) % hkv);
    const long long t = hr / ((long long)R * hkv);
    dst[i] = src[t * stride_v + (long long)h * vpr + c];
  }
}

int repeat_kv_heads(const void* src, long long stride, void* dst, long long n, int hkv, int R, int D,
                    cudaStream_t s) {
  if (n <= 0) return LSRM_OK;
  const int vpr = D * 2 / 16;  // 16-byte vectors per head row
  const long long total = n * hkv * R * vpr;
  const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  ProfScope ps("dense_regroup", s);
  repeat_kv_heads_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), stride * 2 / 16,
                                              static_cast<uint4*>(dst), n, hkv, R, vpr);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

int dense_fwd_tiles(const lsrm_varlen* meta, int G, int mode, int window, DensePlan& plan, int* err, cudaStream_t s) {
  const int qpt = kRows / G;
  if (mode == LSRM_DENSE_COMPRESSED)
    return launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, 5 /*seq rows, compressed kv*/, qpt, meta,
                              nullptr, meta->num_seqs, 0, err, s);
  if (mode == LSRM_DENSE_INTRA_BLOCK)
    return launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, kTilesKVBlock, qpt, meta, nullptr,
                              meta->num_blocks, 0, err, s);
  return launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, kTilesSeq, qpt, meta, nullptr, meta->num_seqs,
                            window, err, s);
}

// The dense forward with at most kDenseMaxG query heads per kv head; the
// workspace holds `need` bytes (dense_ws_direct).
static int dense_fwd_direct(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode, int window,
                            const void* q, const void* k, const void* v, void* out, float* lse, void* workspace,
                            size_t need, int* err_flags, cudaStream_t s) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(G <= kDenseMaxG, "dense kernels take at most %d query heads per kv head (got %d)", kDenseMaxG, G);
  DensePlan plan = make_dense_plan(meta, G, mode, workspace);
  int* err = err_flags ? err_flags : reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + need - 256);
  if ((rc = dense_fwd_tiles(meta, G, mode, window, plan, err, s))) return rc;
  const int D = shape->head_dim, qpt = kRows / G;
  const long long nk = (mode == LSRM_DENSE_COMPRESSED) ? meta->num_blocks : meta->total_k;
  CUtensorMap mq;
  KVMaps kv;
  if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt))) return rc;
  if ((rc = make_kv_maps(kv.k, kv.v, kNumBoxes, k, v, D, shape->num_kv_heads, nk, shape->kv_token_stride))) return rc;
  FwdParams p{};
  p.tiles = plan.tiles;
  p.n_tiles = plan.n_tiles;
  p.out = out;
  p.lse = lse;
  p.q_tok_stride = shape->q_token_stride;
  p.num_q_heads = shape->num_q_heads;
  p.total_q = meta->total_q;
  p.total_k = (int)nk;
  p.G = G;
  p.scale_log2 = softmax_scale_of(shape) * 1.44269504f;
  p.half_window = window / 2;
  p.lse_natural = (mode == LSRM_DENSE_COMPRESSED) ? 1 : 0;
  p.err = err;
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  if (mode == LSRM_DENSE_SLIDING)
    return launch_fwd<kBand>(D, bf16, mq, kv, p, plan.tiles_ub, shape->num_kv_heads, s);
  return launch_fwd<kRange>(D, bf16, mq, kv, p, plan.tiles_ub, shape->num_kv_heads, s);
}

}  // namespace lsrm

extern "C" size_t lsrm_dense_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode) {
  int G = 1;
  if (check_shape(meta, shape, G) != LSRM_OK) return 0;
  if (G <= kDenseMaxG) return dense_ws_direct(meta, shape, mode);
  const DenseRegroup r = dense_regroup(meta, shape, mode);
  return r.inner + 4 * r.buf;  // inner workspace, repeated k / v, their gradients
}

extern "C" int lsrm_dense_attn_fwd(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int32_t mode,
                                   int32_t window, const void* q, const void* k, const void* v, void* out, float* lse,
                                   void* workspace, size_t workspace_bytes, int* err_flags, void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(mode >= 0 && mode <= 2, "unknown dense mode %d", mode);
  LSRM_CHECK_ARG(mode != LSRM_DENSE_SLIDING || window >= 0, "window must be >= 0");
  LSRM_CHECK_ARG(mode == LSRM_DENSE_COMPRESSED || meta->total_q == meta->total_k,
                 "window branches attend inside one token sequence (total_q == total_k)");
  const size_t need = lsrm_dense_workspace_bytes(meta, shape, mode);
  if (workspace_bytes < need || !workspace) {
    set_error("workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  if (meta->total_q == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (G <= kDenseMaxG)
    return dense_fwd_direct(meta, shape, mode, window, q, k, v, out, lse, workspace, need, err_flags, s);
  // more query heads per kv head than the dense kernels take: repeat every kv
  // head R times and run with kDenseMaxG (the query heads, the output and the
  // LSE are the same; only the grouping changes)
  const DenseRegroup r = dense_regroup(meta, shape, mode);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  void* k2 = base + r.inner;
  void* v2 = base + r.inner + r.buf;
  const int hkv = shape->num_kv_heads, D = shape->head_dim;
  if ((rc = repeat_kv_heads(k, shape->kv_token_stride, k2, r.nk, hkv, r.R, D, s))) return rc;
  if ((rc = repeat_kv_heads(v, shape->kv_token_stride, v2, r.nk, hkv, r.R, D, s))) return rc;
  return dense_fwd_direct(meta, &r.shape, mode, window, q, k2, v2, out, lse, workspace, r.inner, err_flags, s);
}

// ---------------------------------------------------------------------------
// Selected-block forward without any allocation
//
// For callers that may not allocate device memory themselves: plugin hosts
// that own every device allocation (an inference server's fixed arena, another
// framework's operator interface), and latency-critical loops that must not
// call the driver allocator (cudaMalloc can synchronise the device and stall).
// The plan scratch (query tiles and per-tile block unions) lives in one
// file-scope device array that every GPU loading this library holds until the
// process exits.  Every call shares it and it keeps the previous call's
// contents; calls that overlap on the GPU (different streams, different host
// threads) race on it.
// ---------------------------------------------------------------------------

namespace lsrm {

static __device__ __align__(256) uint8_t g_select_fwd_scratch[LSRM_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array.  A __device__ array has its own address
// in every CUDA context (the runtime's primary context of each device, a
// driver-API context a plugin host made current, a context re-created after
// cudaDeviceReset), so the address is resolved on the first call in each
// context and cached under the context's process-unique id (cuCtxGetId), which
// a destroyed context never passes on to a new one.  Host code cannot use the
// symbol itself: on the host it names a stand-in, not device memory.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

static int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  constexpr int kSlots = 64;
  static unsigned long long ids[kSlots] = {};
  static void* ptrs[kSlots] = {};
  static int next_slot = 0;
  std::lock_guard<std::mutex> g(mu);
  if (!get_current || !get_id) {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) != cudaSuccess ||
        qa != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) != cudaSuccess ||
        qb != cudaDriverEntryPointSuccess) {
      set_error("cuCtxGetCurrent / cuCtxGetId are unavailable from the driver");
      return LSRM_ERR_CUDA;
    }
    get_current = reinterpret_cast<CtxGetCurrentFn>(a);
    get_id = reinterpret_cast<CtxGetIdFn>(b);
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) {
    set_error("cuCtxGetCurrent failed");
    return LSRM_ERR_CUDA;
  }
  void* p = nullptr;
  if (!ctx) {  // no context current yet: the runtime makes its primary context current here
    LSRM_CUDA_TRY(cudaGetSymbolAddress(&p, g_select_fwd_scratch));
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) {
      set_error("no CUDA context is current");
      return LSRM_ERR_CUDA;
    }
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS || id == 0) {
    set_error("cuCtxGetId failed");
    return LSRM_ERR_CUDA;
  }
  for (int i = 0; i < kSlots; ++i) {
    if (ids[i] == id) {
      *out = ptrs[i];
      return LSRM_OK;
    }
  }
  if (!p) LSRM_CUDA_TRY(cudaGetSymbolAddress(&p, g_select_fwd_scratch));
  ids[next_slot] = id;  // oldest entry makes room once every slot is taken
  ptrs[next_slot] = p;
  next_slot = (next_slot + 1) % kSlots;
  *out = p;
  return LSRM_OK;
}

}  // namespace lsrm

extern "C" int lsrm_select_attn_fwd_noalloc(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q,
                                            const void* k, const void* v, const int32_t* block_topk, int32_t topk,
                                            const int32_t* cu_query_blocks, int32_t num_query_blocks, void* out,
                                            float* lse_log2, int* err_flags, void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(num_query_blocks == 0 || cu_query_blocks, "num_query_blocks > 0 needs cu_query_blocks");
  // forward-only carve of the selection plan: tiles, tile count, unions
  SelectPlan plan = make_select_plan(meta, G, shape->num_kv_heads, topk, num_query_blocks, nullptr);
  const size_t hkv = (size_t)shape->num_kv_heads;
  const size_t ent = hkv * plan.tiles_ub * plan.union_cap;
  size_t need = 0;
  auto carve_off = [&](size_t bytes) {
    const size_t off = need;
    need += align_up(bytes, 256);
    return off;
  };
  const size_t o_tiles = carve_off(sizeof(QTile) * plan.tiles_ub);
  const size_t o_ntiles = carve_off(16);
  const size_t o_cnt = carve_off(sizeof(int) * hkv * plan.tiles_ub);
  const size_t o_ngroups = carve_off(sizeof(int) * hkv * plan.tiles_ub);
  const size_t o_blk = carve_off(sizeof(int) * ent);
  const size_t o_mask = carve_off(sizeof(uint4) * ent);
  const size_t o_err = carve_off(sizeof(int));
  if (need > (size_t)LSRM_NOALLOC_SCRATCH_BYTES) {
    set_error("lsrm_select_attn_fwd_noalloc: this problem needs %zu bytes of plan scratch, more than the fixed %zu; "
              "use lsrm_select_attn_fwd with a caller-provided workspace",
              need, (size_t)LSRM_NOALLOC_SCRATCH_BYTES);
    return LSRM_ERR_WORKSPACE;
  }
  if (meta->total_q == 0) return LSRM_OK;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch_ptr(&scratch))) return rc;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  plan.tiles = reinterpret_cast<QTile*>(base + o_tiles);
  plan.n_tiles = reinterpret_cast<int*>(base + o_ntiles);
  plan.union_cnt = reinterpret_cast<int*>(base + o_cnt);
  plan.union_ngroups = reinterpret_cast<int*>(base + o_ngroups);
  plan.union_blk = reinterpret_cast<int*>(base + o_blk);
  plan.union_mask = reinterpret_cast<uint4*>(base + o_mask);
  plan.kvtiles = nullptr;
  plan.n_kvtiles = nullptr;
  plan.rev_off = nullptr;
  plan.rev_cursor = nullptr;
  plan.rev_entries = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = err_flags;
  if (!err) {  // the internal error word must start clear on every call
    err = reinterpret_cast<int*>(base + o_err);
    LSRM_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), s));
  }
  const int qpt = kRows / G;
  const bool qblock = num_query_blocks > 0;
  if ((rc = launch_build_tiles(plan.tiles, plan.n_tiles, plan.tiles_ub, qblock ? kTilesQBlock : kTilesSeq, qpt, meta,
                               cu_query_blocks, qblock ? num_query_blocks : meta->num_seqs, 0, err, s)))
    return rc;
  if ((rc = launch_build_unions(plan, meta, block_topk, topk, qblock ? num_query_blocks : meta->total_q, G, err, s)))
    return rc;
  const int D = shape->head_dim;
  CUtensorMap mq;
  KVMaps kv;
  if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, qpt))) return rc;
  if ((rc = make_kv_maps(kv.k, kv.v, kNumBoxes, k, v, D, shape->num_kv_heads, meta->total_k, shape->kv_token_stride)))
    return rc;
  FwdParams p{};
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
  p.lse = lse_log2;
  p.q_tok_stride = shape->q_token_stride;
  p.num_q_heads = shape->num_q_heads;
  p.total_q = meta->total_q;
  p.total_k = meta->total_k;
  p.G = G;
  p.scale_log2 = softmax_scale_of(shape) * 1.44269504f;
  p.half_window = 0;
  p.lse_natural = 0;
  p.err = err;
  return launch_fwd<kSelect>(D, shape->dtype == LSRM_DTYPE_BF16, mq, kv, p, plan.tiles_ub, shape->num_kv_heads, s);
}
