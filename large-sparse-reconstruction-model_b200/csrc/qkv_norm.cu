// Projection GEMM with the per-head LayerNorm32 in its epilogue (sm_100a).
//
// Y = X W^T (+ b) for X [M, K] and W [N, K] (nn.Linear layout), bf16 in, fp32
// accumulation on the tensor cores.  Persistent CTAs walk 128 x 256 output
// tiles (row tiles outer, so the CTAs working at one time share X rows in
// L2; W is small enough to stay there): warp 0 streams 64-wide K chunks of X
// and W by TMA into a 4-stage ring, warp 1 issues tcgen05.mma (M = 128,
// N = 256, K = 16, both operands K-major from shared memory; at N = 256 the
// products are bound by the tensor pipe rather than by shared-memory operand
// reads) into one of two TMEM accumulators (2 x 256 columns), and warps 2-5
// (one output row per thread) empty a finished accumulator while the next
// tile accumulates in the other.
//
// The N columns are cut into segments (CrossAttention's q, k and v
// projections).  Per segment the epilogue writes the bf16 result, its
// per-head LayerNorm (non-affine over `head_dim` columns; fp32 statistics of
// the bf16-rounded values, i.e. LayerNorm32 applied to the Linear's bf16
// output as models_sparse/utils.py:239-270 does), or both, and records 1/std
// of every normalised head group for the backward.
//
// qkv_norm_bwd_kernel turns the gradients of the outputs into the gradient
// of the pre-norm result Y (the non-affine LayerNorm backward from the
// normalised output and 1/std: dy = rstd * (g - mean(g) - yhat * mean(g *
// yhat)), plus the gradient of the raw output); the weight and input
// gradients are then two plain GEMMs.
#include "common.cuh"
#include "host_util.h"

namespace lsrm {
namespace {

constexpr int kQnBM = 128, kQnBN = 256, kQnBK = 64, kQnStages = 4;
constexpr int kQnThreads = 192;                  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kQnTileA = kQnBM * kQnBK * 2;      // bytes of one 128 x 64 bf16 tile of X
constexpr int kQnTileB = kQnBN * kQnBK * 2;      // bytes of one 256 x 64 bf16 tile of W
constexpr int kQnMaxSeg = 4;
constexpr int kQnTmemCols = 2 * kQnBN;          // two accumulators

struct QnSeg {
  int col0, cols;  // GEMM columns [col0, col0 + cols)
  void* out;       // [M, cols] bf16 result, or null
  void* out_norm;  // [M, cols] bf16 per-head LayerNorm of the result, or null
};

struct QnParams {
  int M, N, K;
  int heads_total;  // N / head_dim: width of the rstd rows
  const __nv_bfloat16* bias;
  QnSeg seg[kQnMaxSeg];
  int n_seg;
  float eps;
  float* rstd;  // [M, heads_total]
  int* err;
};

struct QnSmem {
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = kQnStages * kQnTileA;
  static constexpr int OFF_BAR = OFF_B + kQnStages * kQnTileB;
  // full[S], empty[S], acc_full[2], acc_empty[2], mma_done
  static constexpr int NBAR = 2 * kQnStages + 5;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;  // + alignment of the swizzled tiles
  static_assert(ALLOC <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ int qn_segment(const QnParams& p, int col) {
  int s = 0;
  while (s + 1 < p.n_seg && col >= p.seg[s + 1].col0) ++s;
  return s;
}

template <int D>
__device__ __forceinline__ void store_row_bf16(void* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < D; c += 8) {
    uint4 pk;
    pk.x = pack_bf16(v[c], v[c + 1]);
    pk.y = pack_bf16(v[c + 2], v[c + 3]);
    pk.z = pack_bf16(v[c + 4], v[c + 5]);
    pk.w = pack_bf16(v[c + 6], v[c + 7]);
    d[c / 8] = pk;
  }
}

template <int D>
__device__ __forceinline__ void load_row_bf16(const void* src, float* v) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int c = 0; c < D; c += 8) {
    const uint4 x = s[c / 8];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&x);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[c + j] = __bfloat162float(e[j]);
  }
}

template <int D>
__global__ void __launch_bounds__(kQnThreads, 1)
    qkv_norm_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                         const QnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + QnSmem::OFF_A;
  uint8_t* sB = smem + QnSmem::OFF_B;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + QnSmem::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + kQnStages;
  uint64_t* acc_full = bars + 2 * kQnStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + QnSmem::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + QnSmem::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kQnBM - 1) / kQnBM, n_tiles = (p.N + kQnBN - 1) / kQnBN;
  const int n_items = m_tiles * n_tiles;
  const int kc_n = p.K / kQnBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kQnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      int J = 0, last = -1;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        const int m0 = (i / n_tiles) * kQnBM, n0 = (i % n_tiles) * kQnBN;
        for (int kc = 0; kc < kc_n; ++kc, ++J) {
          const int s = J % kQnStages;
          if (!mbar_wait(&empty[s], ((J / kQnStages) & 1) ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kQnTileA + kQnTileB);
          tma_load_3d(sA + s * kQnTileA, &tm_x, 0, kc, m0, &full[s]);
          tma_load_3d(sB + s * kQnTileB, &tm_w, 0, kc, n0, &full[s]);
          last = J;
        }
      }
      if (!ok)  // teardown after an abort: the copies still in flight land before the CTA exits
        for (int j = max(0, last - kQnStages + 1); j <= last; ++j)
          mbar_wait_drain(&full[j % kQnStages], (j / kQnStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(1u, 0, 0, kQnBM, kQnBN);
      int J = 0, it = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it) {
        const int b = it & 1;
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * kQnBN;
        for (int kc = 0; kc < kc_n; ++kc, ++J) {
          const int s = J % kQnStages;
          if (!mbar_wait(&full[s], (J / kQnStages) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * kQnTileA), b_base = smem_u32(sB + s * kQnTileB);
#pragma unroll
          for (int ks = 0; ks < kQnBK / 16; ++ks)
            umma_f16(acc, make_sdesc(a_base + ks * 32, 16, 8 * 128, kSw128),
                     make_sdesc(b_base + ks * 32, 16, 8 * 128, kSw128), idesc, (kc > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&empty[s]);  // the stage is free once these products have read it
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    // warp w reads TMEM lanes 32*(w%4).. : thread = one output row of the tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float inv_d = 1.0f / D;
    int it = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++it) {
      const int b = it & 1;
      const int m0 = (i / n_tiles) * kQnBM, n0 = (i % n_tiles) * kQnBN;
      if (!warp_wait(&acc_full[b], (it >> 1) & 1, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = m0 + r;
      const bool row_ok = row < p.M;
#pragma unroll 1
      for (int g = 0; g < kQnBN / D; ++g) {
        const int col = n0 + g * D;
        if (col >= p.N) break;  // the same for every lane of the warp
        float v[D];
        tmem_load_cols<D>(tmem + b * kQnBN + g * D + lane_base, v);
        tmem_wait_ld();
        if (row_ok) {
          const QnSeg& sg = p.seg[qn_segment(p, col)];
          const int lc = col - sg.col0;
#pragma unroll
          for (int c = 0; c < D; ++c) {
            float x = v[c];
            if (p.bias) x += __bfloat162float(p.bias[col + c]);
            v[c] = __bfloat162float(__float2bfloat16_rn(x));  // the Linear's bf16 output
          }
          if (sg.out)
            store_row_bf16<D>(static_cast<__nv_bfloat16*>(sg.out) + (size_t)row * sg.cols + lc, v);
          if (sg.out_norm) {
            float mean = 0.f;
#pragma unroll
            for (int c = 0; c < D; ++c) mean += v[c];
            mean *= inv_d;
            float var = 0.f;
#pragma unroll
            for (int c = 0; c < D; ++c) {
              const float t = v[c] - mean;
              var = fmaf(t, t, var);
            }
            const float rs = rsqrtf(var * inv_d + p.eps);
            p.rstd[(size_t)row * p.heads_total + col / D] = rs;
#pragma unroll
            for (int c = 0; c < D; ++c) v[c] = (v[c] - mean) * rs;
            store_row_bf16<D>(static_cast<__nv_bfloat16*>(sg.out_norm) + (size_t)row * sg.cols + lc, v);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kQnTmemCols);
  }
}

struct QnGradSeg {
  int col0, cols;
  const void* out_norm;   // forward's normalised output (or null)
  const void* grad_out;   // gradient of the raw output (or null)
  const void* grad_norm;  // gradient of the normalised output (or null)
};

struct QnBwdParams {
  long long M;
  int N, heads_total;
  QnGradSeg seg[kQnMaxSeg];
  int n_seg;
  const float* rstd;
  void* grad_pre;  // [M, N] bf16
};

// One thread per (row, head group): neighbouring threads take neighbouring
// groups of one row, so every warp reads and writes contiguous rows.
template <int D>
__global__ void qkv_norm_bwd_kernel(const QnBwdParams p) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.M * p.heads_total) return;
  const long long row = idx / p.heads_total;
  const int g = (int)(idx - row * p.heads_total);
  const int col = g * D;
  int s = 0;
  while (s + 1 < p.n_seg && col >= p.seg[s + 1].col0) ++s;
  const QnGradSeg& sg = p.seg[s];
  const size_t off = (size_t)row * sg.cols + (col - sg.col0);
  float dy[D];
#pragma unroll
  for (int c = 0; c < D; ++c) dy[c] = 0.f;
  if (sg.grad_out) load_row_bf16<D>(static_cast<const __nv_bfloat16*>(sg.grad_out) + off, dy);
  if (sg.grad_norm && sg.out_norm) {
    float gv[D], yh[D];
    load_row_bf16<D>(static_cast<const __nv_bfloat16*>(sg.grad_norm) + off, gv);
    load_row_bf16<D>(static_cast<const __nv_bfloat16*>(sg.out_norm) + off, yh);
    float mg = 0.f, mgy = 0.f;
#pragma unroll
    for (int c = 0; c < D; ++c) {
      mg += gv[c];
      mgy = fmaf(gv[c], yh[c], mgy);
    }
    mg *= 1.0f / D;
    mgy *= 1.0f / D;
    const float rs = p.rstd[(size_t)row * p.heads_total + g];
#pragma unroll
    for (int c = 0; c < D; ++c) dy[c] += rs * (gv[c] - mg - yh[c] * mgy);
  }
  store_row_bf16<D>(static_cast<__nv_bfloat16*>(p.grad_pre) + (size_t)row * p.N + col, dy);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace
}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_qkv_norm_fwd(int64_t M, int32_t K, int32_t N, int32_t head_dim, const void* x,
                                 int64_t x_token_stride, const void* w, const void* bias,
                                 const lsrm_qkv_segment* segs, int32_t n_segs, float eps, float* rstd,
                                 int* err_flags, void* stream) {
  LSRM_CHECK_ARG(M >= 0 && M <= INT32_MAX, "rows must be in [0, 2^31) (got %lld)", (long long)M);
  LSRM_CHECK_ARG(K >= kQnBK && K % kQnBK == 0, "K must be a positive multiple of %d (got %d)", kQnBK, K);
  LSRM_CHECK_ARG(head_dim == 32 || head_dim == 64, "head_dim must be 32 or 64 (got %d)", head_dim);
  LSRM_CHECK_ARG(N >= head_dim && N % head_dim == 0, "N must be a positive multiple of head_dim (got %d)", N);
  LSRM_CHECK_ARG(n_segs >= 1 && n_segs <= kQnMaxSeg && segs, "between 1 and %d segments", kQnMaxSeg);
  LSRM_CHECK_ARG(x && w && err_flags, "x, w and err_flags are required");
  LSRM_CHECK_ARG(x_token_stride >= K, "x token stride %lld is below K = %d", (long long)x_token_stride, K);
  QnParams p{};
  p.M = (int)M;
  p.N = N;
  p.K = K;
  p.heads_total = N / head_dim;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.n_seg = n_segs;
  p.eps = eps;
  p.rstd = rstd;
  p.err = err_flags;
  int col = 0;
  for (int s = 0; s < n_segs; ++s) {
    const lsrm_qkv_segment& sg = segs[s];
    LSRM_CHECK_ARG(sg.cols > 0 && sg.cols % head_dim == 0, "segment %d: cols %d is not a positive multiple of %d", s,
                   sg.cols, head_dim);
    LSRM_CHECK_ARG(sg.out || sg.out_norm, "segment %d has no output", s);
    LSRM_CHECK_ARG((!sg.out || aligned16(sg.out)) && (!sg.out_norm || aligned16(sg.out_norm)),
                   "segment %d: outputs must be 16-byte aligned", s);
    LSRM_CHECK_ARG(!sg.out_norm || rstd, "segment %d is normalised: rstd is required", s);
    p.seg[s] = QnSeg{col, sg.cols, sg.out, sg.out_norm};
    col += sg.cols;
  }
  LSRM_CHECK_ARG(col == N, "segments cover %d columns, N is %d", col, N);
  if (M == 0) return LSRM_OK;
  CUtensorMap tm_x, tm_w;
  int rc;
  // K is read in chunks of 64 elements (128 B): {64, K / 64, rows} with 128B swizzle, box of 128 rows
  if ((rc = make_tmap_3d(&tm_x, x, kQnBK, K / kQnBK, M, x_token_stride, 1, kQnBM))) return rc;
  if ((rc = make_tmap_3d(&tm_w, w, kQnBK, K / kQnBK, N, K, 1, kQnBN))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long items = ((M + kQnBM - 1) / kQnBM) * (long long)((N + kQnBN - 1) / kQnBN);
  const int grid = (int)std::min<long long>(items, num_sms());
  ProfScope ps("qkv_norm_gemm", s);
  if (head_dim == 64) {
    LSRM_CUDA_TRY(cudaFuncSetAttribute(qkv_norm_gemm_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       QnSmem::ALLOC));
    qkv_norm_gemm_kernel<64><<<grid, kQnThreads, QnSmem::ALLOC, s>>>(tm_x, tm_w, p);
  } else {
    LSRM_CUDA_TRY(cudaFuncSetAttribute(qkv_norm_gemm_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       QnSmem::ALLOC));
    qkv_norm_gemm_kernel<32><<<grid, kQnThreads, QnSmem::ALLOC, s>>>(tm_x, tm_w, p);
  }
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_qkv_norm_bwd(int64_t M, int32_t N, int32_t head_dim, const lsrm_qkv_grad_segment* segs,
                                 int32_t n_segs, const float* rstd, void* grad_pre, void* stream) {
  LSRM_CHECK_ARG(M >= 0, "rows must be non-negative");
  LSRM_CHECK_ARG(head_dim == 32 || head_dim == 64, "head_dim must be 32 or 64 (got %d)", head_dim);
  LSRM_CHECK_ARG(N >= head_dim && N % head_dim == 0, "N must be a positive multiple of head_dim (got %d)", N);
  LSRM_CHECK_ARG(n_segs >= 1 && n_segs <= kQnMaxSeg && segs, "between 1 and %d segments", kQnMaxSeg);
  LSRM_CHECK_ARG(grad_pre && aligned16(grad_pre), "grad_pre is required and must be 16-byte aligned");
  QnBwdParams p{};
  p.M = M;
  p.N = N;
  p.heads_total = N / head_dim;
  p.n_seg = n_segs;
  p.rstd = rstd;
  p.grad_pre = grad_pre;
  int col = 0;
  for (int s = 0; s < n_segs; ++s) {
    const lsrm_qkv_grad_segment& sg = segs[s];
    LSRM_CHECK_ARG(sg.cols > 0 && sg.cols % head_dim == 0, "segment %d: cols %d is not a positive multiple of %d", s,
                   sg.cols, head_dim);
    LSRM_CHECK_ARG((!sg.out_norm || aligned16(sg.out_norm)) && (!sg.grad_out || aligned16(sg.grad_out)) &&
                       (!sg.grad_norm || aligned16(sg.grad_norm)),
                   "segment %d: tensors must be 16-byte aligned", s);
    LSRM_CHECK_ARG(!sg.grad_norm || (sg.out_norm && rstd), "segment %d: a normalised gradient needs out_norm and rstd",
                   s);
    p.seg[s] = QnGradSeg{col, sg.cols, sg.out_norm, sg.grad_out, sg.grad_norm};
    col += sg.cols;
  }
  LSRM_CHECK_ARG(col == N, "segments cover %d columns, N is %d", col, N);
  if (M == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long n = M * (long long)p.heads_total;
  const int threads = 256;
  const long long blocks = (n + threads - 1) / threads;
  LSRM_CHECK_ARG(blocks <= INT32_MAX, "too many rows");
  ProfScope ps("qkv_norm_bwd", s);
  if (head_dim == 64)
    qkv_norm_bwd_kernel<64><<<(int)blocks, threads, 0, s>>>(p);
  else
    qkv_norm_bwd_kernel<32><<<(int)blocks, threads, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
