// Block scoring + deterministic top-k (the reference's get_block_score,
// sparse/ops/block_score.py:16-98) with a fixed float32 operation order, so
// the selected indices are reproducible bit for bit on any device:
//   dot    = sum_{j=0..D-1} q_j * k_j      (separately rounded mul, add)
//   t      = dot * qk_scale - lse_ln * 1.44269504f
//   score  = sum_{g=0..G-1} exp2_fixed(t_g)
//   agg    = sum over the row's tokens in ascending order (query blocks)
// then the k largest scores (ties to the lowest block id), sorted ascending,
// padded with -1.  exp2_fixed: n = rint(t), f = t - n, degree-7 Taylor
// polynomial of exp(f ln 2) by Horner's rule, times 2^n; t < -125.5 -> 0.
//
// One CTA (256 threads) per (row, kv head); thread b scores blocks b, b+256,
// ..., keeping its block's compressed key in registers while the row's
// queries stream through shared memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>
#include <cstring>

#include "attn_host.h"
#include "host_util.h"
#include "score_exact.cuh"

namespace lsrm {

int launch_qblock_topk_fast(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* ck,
                            const float* lse_ln, int topk, const int32_t* cu_query_blocks, int num_query_blocks,
                            int force_self, double qk_scale, int32_t* out, void* workspace, size_t workspace_bytes,
                            int* err, cudaStream_t s);
size_t fast_scorer_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int num_query_blocks);

struct ScoreParams {
  const void* q;
  const void* ck;
  const float* lse;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_cblocks;  // compressed_cu_seqlens
  const int32_t* cu_qblocks;  // null: one row per token
  int32_t* out;
  long long q_tok_stride;
  long long ck_tok_stride;
  int num_seqs;
  int total_q;
  int G;
  int topk;
  int force_self;
  int tq;  // tokens staged per pass
  float qk_scale;
};

constexpr int kScoreThreads = 256;

template <typename T, int D>
__global__ void __launch_bounds__(kScoreThreads) block_topk_kernel(ScoreParams p) {
  extern __shared__ float sm[];
  const int row = blockIdx.x, h = blockIdx.y;
  const int G = p.G;
  int r0, r1;
  if (p.cu_qblocks) {
    r0 = p.cu_qblocks[row];
    r1 = p.cu_qblocks[row + 1];
  } else {
    r0 = row;
    r1 = row + 1;
  }
  int lo = 0, hi = p.num_seqs + 1;  // sequence of token r0
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (p.cu_seqlens_q[mid] > r0) hi = mid;
    else lo = mid + 1;
  }
  const int seq = max(lo - 1, 0);
  const int blk0 = p.cu_cblocks[seq];
  const int nb = p.cu_cblocks[seq + 1] - blk0;
  const int row_self = p.cu_qblocks ? row - 0 : -1;  // query block index (global)
  float* scores = sm;                        // [nb]
  float* qs = sm + ((nb + 3) & ~3);          // [tq][G][D]
  float* ls = qs + (size_t)p.tq * G * D;     // [tq][G]
  __shared__ float red_s[kScoreThreads / 32];
  __shared__ int red_i[kScoreThreads / 32];
  __shared__ int chosen[64];

  const float l2e = __uint_as_float(0x3FB8AA3Bu);  // 1.44269504f
  for (int b0 = 0; b0 < nb; b0 += kScoreThreads) {
    const int b = b0 + threadIdx.x;
    const bool valid = b < nb;
    float kr[D];
    if (valid) {
      const T* src = static_cast<const T*>(p.ck) + (size_t)(blk0 + b) * p.ck_tok_stride + (size_t)h * D;
#pragma unroll
      for (int j = 0; j < D; ++j) kr[j] = (float)src[j];
    }
    float agg = 0.f;
    for (int t0 = r0; t0 < r1; t0 += p.tq) {
      const int nt = min(p.tq, r1 - t0);
      __syncthreads();
      for (int i = threadIdx.x; i < nt * G * D; i += kScoreThreads) {
        const int t = i / (G * D), rem = i % (G * D), g = rem / D, j = rem % D;
        qs[i] = (float)static_cast<const T*>(p.q)[(size_t)(t0 + t) * p.q_tok_stride + (size_t)(h * G + g) * D + j];
      }
      for (int i = threadIdx.x; i < nt * G; i += kScoreThreads) {
        const int t = i / G, g = i % G;
        ls[i] = __fmul_rn(p.lse[(size_t)(h * G + g) * p.total_q + t0 + t], l2e);
      }
      __syncthreads();
      if (valid) {
        for (int t = 0; t < nt; ++t) {
          float s = 0.f;
          for (int g = 0; g < G; ++g) {
            const float* qv = qs + ((size_t)t * G + g) * D;
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < D; ++j) dot = __fadd_rn(dot, __fmul_rn(qv[j], kr[j]));
            const float tt = __fsub_rn(__fmul_rn(dot, p.qk_scale), ls[t * G + g]);
            s = __fadd_rn(s, exp2_fixed(tt));
          }
          agg = __fadd_rn(agg, s);
        }
        scores[b] = agg;
      }
    }
    if (valid && r1 <= r0) scores[b] = 0.f;
  }
  __syncthreads();

  // selection: forced self block first, then k rounds of arg-max
  const int kk = min(p.topk, nb);
  int n_chosen = 0;
  if (p.force_self && p.cu_qblocks) {
    // query block j of a sequence owns KV block j of that sequence
    int qb_lo = 0, qb_hi = row + 1;  // first query block of the sequence
    while (qb_lo < qb_hi) {
      const int mid = (qb_lo + qb_hi) >> 1;
      if (p.cu_qblocks[mid] >= p.cu_seqlens_q[seq]) qb_hi = mid;
      else qb_lo = mid + 1;
    }
    const int self = row - qb_lo;
    if (self >= 0 && self < nb && kk > 0) {
      if (threadIdx.x == 0) chosen[0] = self;
      if (threadIdx.x == 0) scores[self] = -1.f;
      n_chosen = 1;
    }
    __syncthreads();
  }
  (void)row_self;
  for (; n_chosen < kk; ++n_chosen) {
    float best = -1.f;
    int bid = INT_MAX;
    for (int b = threadIdx.x; b < nb; b += kScoreThreads) {
      const float s = scores[b];
      if (s > best || (s == best && b < bid)) {
        best = s;
        bid = b;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      if (os > best || (os == best && oi < bid)) {
        best = os;
        bid = oi;
      }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
      red_s[w] = best;
      red_i[w] = bid;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bs = red_s[0];
      int bi = red_i[0];
      for (int i = 1; i < kScoreThreads / 32; ++i)
        if (red_s[i] > bs || (red_s[i] == bs && red_i[i] < bi)) {
          bs = red_s[i];
          bi = red_i[i];
        }
      chosen[n_chosen] = bi;
      scores[bi] = -1.f;
    }
    __syncthreads();
  }
  // ascending order (ids are distinct): rank by counting
  int32_t* dst = p.out + ((size_t)h * gridDim.x + row) * p.topk;
  for (int i = threadIdx.x; i < p.topk; i += kScoreThreads) {
    if (i < kk) {
      const int id = chosen[i];
      int rank = 0;
      for (int j = 0; j < kk; ++j) rank += chosen[j] < id;
      dst[rank] = id;
    } else {
      dst[i] = -1;
    }
  }
}

template <typename T, int D>
static int launch_topk_t(const ScoreParams& p, int rows, int hkv, size_t smem, cudaStream_t s) {
  LSRM_CUDA_TRY(
      cudaFuncSetAttribute(block_topk_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ProfScope ps("block_topk", s);
  block_topk_kernel<T, D><<<dim3(rows, hkv), kScoreThreads, smem, s>>>(p);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

}  // namespace lsrm

using namespace lsrm;

extern "C" size_t lsrm_block_topk_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape,
                                                  int32_t topk, int32_t num_query_blocks) {
  int G = 1;
  if (check_shape(meta, shape, G) || topk < 1 || topk > 64) return 0;
  return fast_scorer_workspace_bytes(meta, shape, num_query_blocks);
}

extern "C" int lsrm_block_topk(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* ck,
                               const float* lse_ln, int32_t topk, const int32_t* cu_query_blocks,
                               int32_t num_query_blocks, int32_t force_self, double sm_scale, int32_t* block_topk,
                               void* workspace, size_t workspace_bytes, int* err_flags, void* stream) {
  int G = 1, rc;
  if ((rc = check_shape(meta, shape, G))) return rc;
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(num_query_blocks == 0 || cu_query_blocks, "num_query_blocks > 0 needs cu_query_blocks");
  LSRM_CHECK_ARG(!force_self || cu_query_blocks, "force_self needs query blocks");
  const int D = shape->head_dim;
  LSRM_CHECK_ARG(G * D <= 8192, "query heads per kv head x head_dim (%d) exceeds 8192", G * D);
  const double scale = sm_scale > 0 ? sm_scale : 1.0 / std::sqrt((double)D);
  ScoreParams p{};
  p.q = q;
  p.ck = ck;
  p.lse = lse_ln;
  p.cu_seqlens_q = meta->cu_seqlens_q;
  p.cu_cblocks = meta->cu_seqblocks;
  p.cu_qblocks = num_query_blocks > 0 ? cu_query_blocks : nullptr;
  p.out = block_topk;
  p.q_tok_stride = shape->q_token_stride;
  p.ck_tok_stride = shape->kv_token_stride;
  p.num_seqs = meta->num_seqs;
  p.total_q = meta->total_q;
  p.G = G;
  p.topk = topk;
  p.force_self = force_self;
  p.tq = std::max(1, std::min(64, 4096 / (G * D)));
  p.qk_scale = (float)(scale * 1.44269504);
  const int rows = num_query_blocks > 0 ? num_query_blocks : meta->total_q;
  if (rows == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Per-query-block selection: tensor-core scores with exact refinement
  // (same indices); LSRM_SCORER=exact forces the exact scorer everywhere.
  const char* mode = getenv("LSRM_SCORER");
  if (num_query_blocks > 0 && !(mode && strcmp(mode, "exact") == 0)) {
    int* err = err_flags;
    rc = launch_qblock_topk_fast(meta, shape, q, ck, lse_ln, topk, cu_query_blocks, num_query_blocks, force_self,
                                 scale * 1.44269504, block_topk, workspace, workspace_bytes, err, s);
    if (rc != LSRM_ERR_UNSUPPORTED) return rc;
  }
  const size_t nb_cap = ((size_t)std::max(meta->num_blocks, 1) + 3) & ~size_t(3);
  const size_t smem = (nb_cap + (size_t)p.tq * G * D + (size_t)p.tq * G) * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("block_topk: %d compressed blocks do not fit the on-chip score buffer", meta->num_blocks);
    return LSRM_ERR_UNSUPPORTED;
  }
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  if (D == 64)
    return bf16 ? launch_topk_t<__nv_bfloat16, 64>(p, rows, shape->num_kv_heads, smem, s)
                : launch_topk_t<__half, 64>(p, rows, shape->num_kv_heads, smem, s);
  if (D == 16)
    return bf16 ? launch_topk_t<__nv_bfloat16, 16>(p, rows, shape->num_kv_heads, smem, s)
                : launch_topk_t<__half, 16>(p, rows, shape->num_kv_heads, smem, s);
  return bf16 ? launch_topk_t<__nv_bfloat16, 32>(p, rows, shape->num_kv_heads, smem, s)
              : launch_topk_t<__half, 32>(p, rows, shape->num_kv_heads, smem, s);
}
