// Per-query-block block selection with tensor-core scores and exact
// refinement.  One CTA per (query block, kv head); 320 threads: 8 reduce
// warps, a TMA producer warp, an MMA warp.
//
// 1. Fast scores.  For each chunk of 128 compressed blocks of the sequence,
//    S^T = CK_chunk . Q^T (M = 128 blocks, N <= 128 query rows of the query
//    block per pass, tcgen05, fp32 accumulators in TMEM, double-buffered in
//    256 columns so that two CTAs share an SM and one's selection phase
//    overlaps the other's tensor-core phase).  Reduce warp
//    w owns block row 32*(w%4)+lane and half of the columns; each element
//    adds e = exp2(t), t = s*qk_scale - lse2, to the block's fast score and
//    e*t to a second sum, and keeps the largest t; with the pass's largest
//    |q| and |lse2| these give a rigorous error bound (below).
// 2. Certified selection.  With U = fast + bound and L = fast - bound, let T
//    be the k'-th largest L and T' the (k'+1)-th largest U (k' = k minus the
//    forced own block).  Blocks with U < T are certainly outside the top-k;
//    blocks with L > T' are certainly inside (at most k' blocks have U > T',
//    the block among them, so at most k'-1 others can score above it).  Only
//    the blocks in between (the ambiguous candidates) get their score
//    recomputed with the exact fixed-order arithmetic of score_exact.cuh, and
//    the best of them by (exact score desc, block id asc) fill the remaining
//    places.  T and T' come from exact radix selects.  This is the same set
//    the exact scorer selects, so the indices stay bit-exact.
//
// Error bound per block (generous by construction):
//   |fast dot - exact dot| <= 2^-16 |q| |ck|       (fp32 accumulation of 64
//                                                    exact bf16 products, both
//                                                    sides, 4x margin)
//   |t error| <= qk_scale 2^-16 |q||ck| + 2^-20 (2|t| + 2|lse2| + 1)
//   |e error| <= e (0.7 |t error| + 2^-19)          (ex2 vs exp2_fixed)
//   sum error <= 2 (n + 1) 2^-23 sum e + n 2^-120   (both accumulations; flush)
// and the whole bound is doubled.  The sums over a block's elements use
//   sum e |q|        <= max|q| sum e                (the pass's largest |q|)
//   sum e (2|t| + 2|lse2| + 1) <= 2 (-sum e t + 2 max(t, 0) sum e)
//                                 + (2 max|lse2| + 1) sum e
// (|t| = -t + 2 max(t, 0)), so each element costs one exp2 and three
// accumulations.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>
#include <cmath>

#include "attn_host.h"
#include "common.cuh"
#include "host_util.h"
#include "score_exact.cuh"

namespace lsrm {

constexpr int kSfThreads = 320;
constexpr int kSfReduceThreads = 256;
constexpr int kSfCols = 128;  // query rows per pass: 2 x 128 TMEM columns, so two CTAs share an SM
constexpr int kSfStages = 3;

struct FastScoreParams {
  const void* q;
  const void* ck;
  const float* lse;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_cblocks;
  const int32_t* cu_qblocks;
  int32_t* out;
  long long q_tok_stride;
  long long ck_tok_stride;
  int num_seqs;
  int total_q;
  int G;
  int topk;
  int force_self;
  int nb_cap;      // blocks per sequence the bound slices and shared arrays hold
  int nb_total;    // compressed blocks of all sequences (the norm table's row length)
  int nqb;         // query blocks
  int hkv;         // kv heads
  const float* ckn;  // [Hkv, nb_total] norms of the compressed keys
  float* bounds;     // [Hkv, nqb, 2, nb_cap] lower / upper score bounds
  float qk_scale;
  int* err;
};

template <int D>
struct SfLayout {
  static constexpr int RB = 2 * D;
  static constexpr int QT = kSfCols * RB;
  static constexpr int CKT = 128 * RB;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_CK = QT;
  static constexpr int OFF_COLS = OFF_CK + kSfStages * CKT;  // lse2[128], qn[128], the pass's max |q|, max |lse2|
  static constexpr int OFF_BAR = OFF_COLS + 2 * kSfCols * 4 + 16;
  static constexpr int NBAR = 2 * kSfStages + 2 + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_ARR = OFF_MISC + 64;
  // per-block arrays, one per column half: fast score SF, |q|-weighted sum WS
  // and t-term sum TS [2][nb_cap each]
  static size_t bytes(int nb_cap) { return (size_t)OFF_ARR + 24ull * nb_cap + 1024; }
};

constexpr int kSelThreads = 256;  // 8 warps, one (query block, kv head) item each
constexpr int kSelCandCap = 256;  // ambiguous candidates held per item (more: exact scores of every block)
constexpr int kSelBatch = 8;      // candidates whose exact terms are computed together
constexpr int kSelTerms = 512;    // exact-stage terms held per warp
constexpr int kSelUnroll = 8;     // bound loads per lane in flight in the selects and the candidate sweep

// |ck| of every (compressed block, kv head), fp32 (exact conversion of the
// 16-bit values, fused multiply-add accumulation).
template <typename T, int D>
__global__ void ck_norms_kernel(const T* __restrict__ ck, long long stride, int hkv, int nb, float* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)nb * hkv) return;
  const int b = (int)(i / hkv), h = (int)(i - (long long)b * hkv);
  const uint4* r4 = reinterpret_cast<const uint4*>(ck + (size_t)b * stride + (size_t)h * D);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint4 u = r4[c];
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf((float)e[j], (float)e[j], acc);
  }
  out[(size_t)h * nb + b] = sqrtf(acc);
}

// Row of D 16-bit values -> fp32 (exact conversion), 16-byte loads.
template <typename T, int D>
__device__ __forceinline__ void load_row_f32(const T* __restrict__ row, float* out) {
  const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint4 u = r4[c];
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[c * 8 + i] = (float)e[i];
  }
}

__device__ __forceinline__ void reduce_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kSfReduceThreads) : "memory"); }

// Order-preserving map of a float to uint32, descending: larger floats give
// smaller keys (-inf and +inf included; no NaN reaches it).
__device__ __forceinline__ uint32_t desc_key(float x) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t asc = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ~asc;
}

// The k-th largest of vals[0..n) (1 <= k <= n), exactly, by an MSB-first
// 8-bit radix select.  Block-wide: every thread of the CTA calls it.
__device__ float kth_largest(const float* vals, int n, int k, uint32_t* hist, int* misc) {
  uint32_t prefix = 0u, mask = 0u;
  int kk = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    // warp-aggregated counts: the keys crowd into few bins (similar magnitudes)
    const int lane = threadIdx.x & 31;
    for (int b0 = threadIdx.x - lane; b0 < n; b0 += blockDim.x) {
      const int b = b0 + lane;
      const uint32_t key = b < n ? desc_key(vals[b]) : 0u;
      const bool m = b < n && (key & mask) == prefix;
      const uint32_t bin = m ? ((key >> shift) & 255u) : 256u + lane;
      const uint32_t peers = __match_any_sync(0xffffffffu, bin);
      if (m && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint32_t c[8], tot = 0u;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = hist[lane * 8 + i];
        tot += c[i];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t excl = incl - tot;
      // the lane whose range of 8 bins holds the kk-th key
      if (excl < (uint32_t)kk && (uint32_t)kk <= incl) {
        uint32_t run = excl;
        int d = lane * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (run + c[i] >= (uint32_t)kk) {
            d = lane * 8 + i;
            break;
          }
          run += c[i];
        }
        misc[0] = d;
        misc[1] = kk - (int)run;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)misc[0] << shift;
    mask |= 255u << shift;
    kk = misc[1];
    __syncthreads();
  }
  const uint32_t asc = ~prefix;
  return __uint_as_float((asc & 0x80000000u) ? (asc & 0x7fffffffu) : ~asc);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kSfThreads, 2)
    qblock_scores_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_ck,
                            const FastScoreParams p) {
  using L = SfLayout<D>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int RB = L::RB;
  constexpr uint64_t SWZ = swz_for_row_bytes(RB);
  constexpr uint32_t AB = BF16 ? 1u : 0u;
  const int qb = blockIdx.x, h = blockIdx.y;
  const int G = p.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int r0 = p.cu_qblocks[qb], r1 = p.cu_qblocks[qb + 1];
  int lo = 0, hi = p.num_seqs + 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (p.cu_seqlens_q[mid] > r0) hi = mid;
    else lo = mid + 1;
  }
  const int seq = max(lo - 1, 0);
  const int blk0 = p.cu_cblocks[seq];
  const int nb = p.cu_cblocks[seq + 1] - blk0;
  const int ncols_total = max(r1 - r0, 0) * G;
  const int tpp = kSfCols / G;  // tokens per pass
  const int n_pass = (ncols_total + kSfCols - 1) / kSfCols;
  const int n_ck = (nb + 127) / 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sCK = smem + L::OFF_CK;
  float* col_lse2 = reinterpret_cast<float*>(smem + L::OFF_COLS);
  float* col_qn = col_lse2 + kSfCols;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* ck_full = bars;
  uint64_t* ck_empty = bars + kSfStages;
  uint64_t* q_full = bars + 2 * kSfStages;
  uint64_t* q_free = q_full + 1;
  uint64_t* s_full = q_free + 1;
  uint64_t* s_free = s_full + 2;
  uint64_t* mma_done = s_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  float* SF = reinterpret_cast<float*>(smem + L::OFF_ARR);  // [2][nb_cap]: the two column halves' sums
  float* WS = SF + 2 * p.nb_cap;
  float* TS = WS + 2 * p.nb_cap;

  if (nb > p.nb_cap) {  // the host sizes nb_cap from the total block count
    if (threadIdx.x == 0) atomicOr(p.err, LSRM_ERR_CAPACITY);
    return;
  }
  for (int b = threadIdx.x; b < 2 * p.nb_cap; b += kSfThreads) {
    SF[b] = 0.f;
    WS[b] = 0.f;
    TS[b] = 0.f;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSfStages; ++i) {
      mbar_init(&ck_full[i], 1);
      mbar_init(&ck_empty[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 2 * kSfCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const float sl2 = p.qk_scale;

  if (warp == 8) {
    if (lane == 0) {
      for (int ps = 0; ps < n_pass; ++ps) {
        if (ps > 0 && !mbar_wait(q_free, (ps - 1) & 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(q_full, L::QT);
        tma_load_3d(sQ, &tm_q, 0, h * G, r0 + ps * tpp, q_full);
        bool ok = true;
        for (int c = 0; c < n_ck; ++c) {
          const int j = ps * n_ck + c, s = j % kSfStages;
          if (!mbar_wait(&ck_empty[s], ((j / kSfStages) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&ck_full[s], L::CKT);
          tma_load_3d(sCK + s * L::CKT, &tm_ck, 0, h, blk0 + c * 128, &ck_full[s]);
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    if (lane == 0) {
      bool ok = true;
      for (int ps = 0; ps < n_pass && ok; ++ps) {
        const int ncols = min(kSfCols, ncols_total - ps * kSfCols);
        // whole 32-column slices: every column the reduce warps read is a computed (finite) product
        const uint32_t n_mma = (uint32_t)((ncols + 31) / 32 * 32);
        const uint32_t idesc = make_idesc(AB, 0, 0, 128, n_mma);
        if (!mbar_wait(q_full, ps & 1, abort_flag, p.err)) break;
        tc_fence_after();
        for (int c = 0; c < n_ck; ++c) {
          const int j = ps * n_ck + c, s = j % kSfStages, sb = j & 1;
          if (!mbar_wait(&ck_full[s], (j / kSfStages) & 1, abort_flag, p.err)) { ok = false; break; }
          if (!mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ckb = smem_u32(sCK + s * L::CKT), qb_s = smem_u32(sQ);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_f16(tmem + sb * kSfCols, make_sdesc(ckb + ks * 32, 16, 8 * RB, SWZ),
                     make_sdesc(qb_s + ks * 32, 16, 8 * RB, SWZ), idesc, ks > 0);
          umma_commit(&s_full[sb]);
          umma_commit(&ck_empty[s]);
        }
        umma_commit(q_free);
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ reduce warps ---------------------------
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float l2e = __uint_as_float(0x3FB8AA3Bu);
    bool ok = true;
    float* col_max = col_qn + kSfCols;  // [0] max |q|, [1] max |lse2| of the pass (non-negative: int order)
    for (int ps = 0; ps < n_pass && ok; ++ps) {
      const int ncols = min(kSfCols, ncols_total - ps * kSfCols);
      reduce_bar();
      if (threadIdx.x < 2) col_max[threadIdx.x] = 0.f;
      reduce_bar();
      {
        const int t = threadIdx.x;  // column of this pass
        // padding columns: a huge finite lse2 makes e exactly 0, so e * t is exactly 0 too
        float l2 = 1e30f, qn = 0.f;
        if (t < ncols) {
          const int tok = r0 + ps * tpp + t / G, g = t % G;
          l2 = p.lse[(size_t)(h * G + g) * p.total_q + tok] * l2e;
          float qv[D];
          load_row_f32<T, D>(static_cast<const T*>(p.q) + (size_t)tok * p.q_tok_stride + (size_t)(h * G + g) * D, qv);
#pragma unroll
          for (int j = 0; j < D; ++j) qn = fmaf(qv[j], qv[j], qn);
          qn = sqrtf(qn);
          atomicMax(reinterpret_cast<int*>(&col_max[0]), __float_as_int(qn));
          atomicMax(reinterpret_cast<int*>(&col_max[1]), __float_as_int(fabsf(l2)));
        }
        if (t < kSfCols) {
          col_lse2[t] = l2;
          col_qn[t] = qn;
        }
      }
      reduce_bar();
      const float qmax = col_max[0], l2max = col_max[1];
      for (int c = 0; c < n_ck; ++c) {
        const int j = ps * n_ck + c, sb = j & 1;
        if (!warp_wait(&s_full[sb], (j >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        float acc_e = 0.f, acc_te = 0.f, tmax = -INFINITY;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int col0 = (2 * x + half) * 32;  // halves interleave 32-column slices
          if (col0 < ncols) {
            float sv[32];
            tmem_ld32(tmem + sb * kSfCols + lane_base + col0, sv);
            tmem_wait_ld();
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(&col_lse2[col0 + c4]);
              const float l2v[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float t = fmaf(sv[c4 + i], sl2, -l2v[i]);
                const float e = ex2(t);
                acc_e += e;
                acc_te = fmaf(e, t, acc_te);
                tmax = fmaxf(tmax, t);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        // each half keeps its own sums (no exchange per chunk): the bound of a
        // block is the sum of the halves' bounds
        const int b = c * 128 + row;
        if (b < nb) {
          const size_t hb = (size_t)half * p.nb_cap + b;
          const float tm = fmaxf(tmax, 0.f);
          SF[hb] += acc_e;
          WS[hb] += qmax * acc_e;  // >= sum e |q|
          // >= sum e (2|t| + 2|lse2| + 1)
          TS[hb] += 2.f * (fmaxf(-acc_te, 0.f) + 2.f * tm * acc_e) + (2.f * l2max + 1.f) * acc_e;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kSfCols);
  }
  if (*abort_flag) return;

  // ------------------------- certified bounds ------------------------------
  // lower (L) and upper (U) bound of every block's score, written to this
  // (query block, kv head)'s slice of the bounds workspace; the forced own
  // block gets -inf in both (it is chosen apart from the ranking)
  int self = -1;
  if (p.force_self && min(p.topk, nb) > 0) {
    int qb_lo = 0, qb_hi = qb + 1;
    while (qb_lo < qb_hi) {
      const int mid = (qb_lo + qb_hi) >> 1;
      if (p.cu_qblocks[mid] >= p.cu_seqlens_q[seq]) qb_hi = mid;
      else qb_lo = mid + 1;
    }
    const int sidx = qb - qb_lo;
    if (sidx >= 0 && sidx < nb) self = sidx;
  }
  const float n_f = (float)ncols_total;
  float* Lg = p.bounds + ((size_t)h * p.nqb + qb) * 2 * p.nb_cap;
  float* Ug = Lg + p.nb_cap;
  for (int b = threadIdx.x; b < nb; b += kSfThreads) {
    const float ckn = p.ckn[(size_t)h * p.nb_total + blk0 + b];
    const float sf = SF[b] + SF[p.nb_cap + b];
    const float ws = WS[b] + WS[p.nb_cap + b], ts = TS[b] + TS[p.nb_cap + b];
    const float e = 2.f * (0.7f * (sl2 * 0x1p-16f * ckn * ws + 0x1p-20f * ts) +
                           (0x1p-19f + (n_f + 1.f) * 0x1p-22f) * sf + n_f * 0x1p-120f);
    Lg[b] = (b == self) ? -INFINITY : sf - e;
    Ug[b] = (b == self) ? -INFINITY : sf + e;
  }
}

// Selection of one (query block, kv head) from its certified bounds (see the
// top of this file), one warp per item and eight items per CTA: thresholds by
// warp-level exact radix selects over the bounds (read from L2, no block-wide
// barriers), certainly chosen blocks directly, the ambiguous ones by the exact
// fixed-order score.  Small per-warp shared memory, so many items share an SM
// and hide the latency of the bound and query-row loads.
template <int D>
struct SelWarpMem {
  uint32_t hist[256];               // radix-select histogram
  int cand[kSelCandCap];            // ambiguous candidates
  float cand_exact[kSelCandCap];    // their exact scores
  int chosen[64];
  float terms[kSelTerms];           // exact-stage terms of a candidate batch
  uint16_t ckrow[kSelBatch][D];     // the batch's compressed key rows
  int misc[8];
};

// The k-th largest (1 <= k <= n) of vals[0..n), exactly, by an MSB-first
// 8-bit radix select; warp-wide (no block barriers).
__device__ float warp_kth_largest(const float* __restrict__ vals, int n, int k, uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0u, mask = 0u;
  int kk = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = lane; i < 256; i += 32) hist[i] = 0u;
    __syncwarp();
    for (int b0 = 0; b0 < n; b0 += 32 * kSelUnroll) {
      float v[kSelUnroll];  // the loads of several rounds in flight at once
#pragma unroll
      for (int j = 0; j < kSelUnroll; ++j) {
        const int b = b0 + 32 * j + lane;
        v[j] = b < n ? vals[b] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kSelUnroll; ++j) {
        const int b = b0 + 32 * j + lane;
        const uint32_t key = b < n ? desc_key(v[j]) : 0u;
        const bool m = b < n && (key & mask) == prefix;
        const uint32_t bin = m ? ((key >> shift) & 255u) : 256u + lane;
        const uint32_t peers = __match_any_sync(0xffffffffu, bin);
        if (m && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
      }
    }
    __syncwarp();
    uint32_t c[8], tot = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      c[i] = hist[lane * 8 + i];
      tot += c[i];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - tot;
    int d = -1, rem = 0;
    if (excl < (uint32_t)kk && (uint32_t)kk <= incl) {
      uint32_t run = excl;
      d = lane * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (run + c[i] >= (uint32_t)kk) {
          d = lane * 8 + i;
          break;
        }
        run += c[i];
      }
      rem = kk - (int)run;
    }
    const uint32_t who = __ballot_sync(0xffffffffu, d >= 0);
    const int src = __ffs(who) - 1;
    d = __shfl_sync(0xffffffffu, d, src);
    kk = __shfl_sync(0xffffffffu, rem, src);
    prefix |= (uint32_t)d << shift;
    mask |= 255u << shift;
    __syncwarp();
  }
  const uint32_t asc = ~prefix;
  return __uint_as_float((asc & 0x80000000u) ? (asc & 0x7fffffffu) : ~asc);
}

// Exact fixed-order scores of blocks ids[0..n) of one (query block, kv
// head): sum over the block's tokens in ascending order of (sum over the G
// heads in order of exp2_fixed(dot * qk_scale - lse2)), the dot product over
// channels 0..D-1 with separately rounded multiply and add.  Warp-wide;
// results in out[0..n).
template <int D, typename T>
__device__ void warp_exact_scores(const FastScoreParams& p, SelWarpMem<D>& wm, const int* ids, int n, int blk0,
                                  int h, int r0, int ncols_total, float* out) {
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const float l2e = __uint_as_float(0x3FB8AA3Bu);
  const int bat = max(1, min(kSelBatch, kSelTerms / G));  // nbat * G <= kSelTerms (G <= 128)
  for (int c0 = 0; c0 < n; c0 += bat) {
    const int nbat = min(bat, n - c0);
    __syncwarp();
    for (int idx = lane; idx < nbat * (D / 8); idx += 32) {
      const int ci = idx / (D / 8), v = idx % (D / 8);
      reinterpret_cast<uint4*>(wm.ckrow[ci])[v] = reinterpret_cast<const uint4*>(
          static_cast<const T*>(p.ck) + (size_t)(blk0 + ids[c0 + ci]) * p.ck_tok_stride + (size_t)h * D)[v];
    }
    float run = 0.f;  // lane ci < nbat: candidate c0 + ci's ordered sum
    // token-aligned column chunks whose terms fit the scratch
    const int cchunk = max(G, kSelTerms / nbat / G * G);
    for (int cc0 = 0; cc0 < ncols_total; cc0 += cchunk) {
      const int nc = min(cchunk, ncols_total - cc0);
      __syncwarp();
      // lane = column: its query row is read once and serves every candidate
      // of the batch (each dot still accumulates channels 0..D-1 in order)
      for (int cl = lane; cl < nc; cl += 32) {
        const int col = cc0 + cl;
        const int tok = r0 + col / G, g = col % G;
        const uint4* qr = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (size_t)tok * p.q_tok_stride +
                                                         (size_t)(h * G + g) * D);
        float dot[kSelBatch];
#pragma unroll
        for (int ci = 0; ci < kSelBatch; ++ci) dot[ci] = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < D / 8; ++c8) {
          const uint4 qu = qr[c8];
          const T* qe = reinterpret_cast<const T*>(&qu);
#pragma unroll
          for (int ci = 0; ci < kSelBatch; ++ci) {
            if (ci < nbat) {
              const uint4 ku = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(wm.ckrow[ci]) + c8 * 8);
              const T* ke = reinterpret_cast<const T*>(&ku);
#pragma unroll
              for (int i = 0; i < 8; ++i) dot[ci] = __fadd_rn(dot[ci], __fmul_rn((float)qe[i], (float)ke[i]));
            }
          }
        }
        const float lse2 = __fmul_rn(p.lse[(size_t)(h * G + g) * p.total_q + tok], l2e);
#pragma unroll
        for (int ci = 0; ci < kSelBatch; ++ci)
          if (ci < nbat) wm.terms[ci * nc + cl] = exp2_fixed(__fsub_rn(__fmul_rn(dot[ci], p.qk_scale), lse2));
      }
      __syncwarp();
      if (lane < nbat) {
        const float* e = wm.terms + (size_t)lane * nc;
        if (G == 1) {
          for (int t = 0; t < nc; ++t) run = __fadd_rn(run, __fadd_rn(0.f, e[t]));
        } else {
          for (int t = 0; t < nc / G; ++t) {
            float st = 0.f;
            for (int g = 0; g < G; ++g) st = __fadd_rn(st, e[t * G + g]);
            run = __fadd_rn(run, st);
          }
        }
      }
    }
    if (lane < nbat) out[c0 + lane] = run;
  }
  __syncwarp();
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kSelThreads, 4) qblock_select_kernel(const FastScoreParams p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  SelWarpMem<D>& wm = reinterpret_cast<SelWarpMem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127))[warp];
  const int item = blockIdx.x * (kSelThreads / 32) + warp;  // h * nqb + qb
  if (item >= p.nqb * p.hkv) return;
  const int h = item / p.nqb, qb = item - h * p.nqb;
  const int G = p.G;
  const int r0 = p.cu_qblocks[qb], r1 = p.cu_qblocks[qb + 1];
  int lo = 0, hi = p.num_seqs + 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (p.cu_seqlens_q[mid] > r0) hi = mid;
    else lo = mid + 1;
  }
  const int seq = max(lo - 1, 0);
  const int blk0 = p.cu_cblocks[seq];
  const int nb = p.cu_cblocks[seq + 1] - blk0;
  const int ncols_total = max(r1 - r0, 0) * G;
  int32_t* dst = p.out + ((size_t)h * p.nqb + qb) * p.topk;
  if (nb > p.nb_cap) {
    if (lane == 0) atomicOr(p.err, LSRM_ERR_CAPACITY);
    for (int i = lane; i < p.topk; i += 32) dst[i] = -1;
    return;
  }
  float* Lg = p.bounds + ((size_t)h * p.nqb + qb) * 2 * p.nb_cap;  // the fallback overwrites it with exact scores
  const float* Ug = Lg + p.nb_cap;
  const int kk = min(p.topk, nb);
  int self = -1;
  if (p.force_self && kk > 0) {
    int qb_lo = 0, qb_hi = qb + 1;
    while (qb_lo < qb_hi) {
      const int mid = (qb_lo + qb_hi) >> 1;
      if (p.cu_qblocks[mid] >= p.cu_seqlens_q[seq]) qb_hi = mid;
      else qb_lo = mid + 1;
    }
    const int sidx = qb - qb_lo;
    if (sidx >= 0 && sidx < nb) self = sidx;
  }
  const int kp = kk - (self >= 0 ? 1 : 0);
  float thr = -INFINITY, thr_hi = -INFINITY;
  if (kp > 0) thr = warp_kth_largest(Lg, nb, kp, wm.hist);
  if (kp > 0 && kp < nb) thr_hi = warp_kth_largest(Ug, nb, kp + 1, wm.hist);
  // candidates whose upper bound reaches thr: certainly chosen ones straight
  // to `chosen`, the ambiguous rest to `cand` (warp-aggregated appends)
  int n_ch = 0, n_cand = 0;
  bool overflow = false;
  if (self >= 0 && lane == 0) wm.chosen[0] = self;
  n_ch = self >= 0 ? 1 : 0;
  if (kp > 0) {
    for (int b0 = 0; b0 < nb; b0 += 32 * kSelUnroll) {
      float uv[kSelUnroll], lv[kSelUnroll];
#pragma unroll
      for (int j = 0; j < kSelUnroll; ++j) {
        const int b = b0 + 32 * j + lane;
        uv[j] = b < nb ? Ug[b] : -INFINITY;
        lv[j] = b < nb ? Lg[b] : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < kSelUnroll; ++j) {
      const int b = b0 + 32 * j + lane;
      bool sure = false, amb = false;
      if (b < nb && b != self) {
        if (uv[j] >= thr) {
          if (lv[j] > thr_hi) sure = true;
          else amb = true;
        }
      }
      const uint32_t ms = __ballot_sync(0xffffffffu, sure), ma = __ballot_sync(0xffffffffu, amb);
      const uint32_t below = (1u << lane) - 1u;
      if (sure) {
        const int slot = n_ch + __popc(ms & below);
        if (slot < 64) wm.chosen[slot] = b;
      }
      if (amb) {
        const int slot = n_cand + __popc(ma & below);
        if (slot < kSelCandCap) wm.cand[slot] = b;
      }
      n_ch += __popc(ms);
      n_cand += __popc(ma);
      }
    }
    overflow = n_cand > kSelCandCap;
  }
  __syncwarp();
  const int slots = kp - (n_ch - (self >= 0 ? 1 : 0));
  if (overflow) {
    // more ambiguous blocks than the list holds: exact scores of every block
    // (in place of the lower bounds), then the kp best by (exact desc, id asc)
    n_ch = self >= 0 ? 1 : 0;
    for (int b0 = 0; b0 < nb; b0 += kSelCandCap) {
      const int m = min(kSelCandCap, nb - b0);
      for (int i = lane; i < m; i += 32) wm.cand[i] = b0 + i;
      __syncwarp();
      warp_exact_scores<D, T>(p, wm, wm.cand, m, blk0, h, r0, ncols_total, Lg + b0);
    }
    __syncwarp();
    if (self >= 0 && lane == 0) Lg[self] = -INFINITY;
    __syncwarp();
    for (int r = 0; r < kp; ++r) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int b = lane; b < nb; b += 32) {
        const float v = Lg[b];
        if (v > bv || (v == bv && b < bi)) {
          bv = v;
          bi = b;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi == INT_MAX || bv == -INFINITY) break;
      if (lane == 0) {
        wm.chosen[n_ch] = bi;
        Lg[bi] = -INFINITY;
      }
      ++n_ch;
      __syncwarp();
    }
  } else if (slots > 0 && n_cand > 0) {
    if (n_cand <= slots) {
      for (int i = lane; i < n_cand; i += 32)
        if (n_ch + i < 64) wm.chosen[n_ch + i] = wm.cand[i];
      n_ch += n_cand;
    } else {
      warp_exact_scores<D, T>(p, wm, wm.cand, n_cand, blk0, h, r0, ncols_total, wm.cand_exact);
      // a candidate is chosen when fewer than `slots` of them beat it
      int taken = 0;
      for (int i0 = 0; i0 < n_cand; i0 += 32) {
        const int i = i0 + lane;
        bool take = false;
        if (i < n_cand) {
          const float v = wm.cand_exact[i];
          const int id = wm.cand[i];
          int beat = 0;
          for (int j = 0; j < n_cand; ++j) {
            const float w = wm.cand_exact[j];
            beat += (w > v) || (w == v && wm.cand[j] < id);
          }
          take = beat < slots;
        }
        const uint32_t mt = __ballot_sync(0xffffffffu, take);
        if (take) {
          const int slot = n_ch + taken + __popc(mt & ((1u << lane) - 1u));
          if (slot < 64) wm.chosen[slot] = wm.cand[i];
        }
        taken += __popc(mt);
      }
      n_ch += taken;
    }
  }
  __syncwarp();
  if (n_ch > kk) {  // only reachable with non-finite scores
    if (lane == 0) atomicOr(p.err, LSRM_ERR_CAPACITY);
    n_ch = kk;
  }
  for (int i = lane; i < p.topk; i += 32) {
    if (i < n_ch) {
      const int id = wm.chosen[i];
      int rank = 0;
      for (int j = 0; j < n_ch; ++j) rank += wm.chosen[j] < id;
      if (rank < p.topk) dst[rank] = id;
    } else {
      dst[i] = -1;
    }
  }
}

template <int D, bool BF16>
static int launch_fast_t(const CUtensorMap& mq, const CUtensorMap& mck, const FastScoreParams& p, int hkv,
                         size_t smem_scores, size_t smem_select, long long ck_stride, cudaStream_t s) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  {
    ProfScope ps("block_topk_norms", s);
    const long long n = (long long)p.nb_total * hkv;
    ck_norms_kernel<T, D><<<(int)((n + 255) / 256), 256, 0, s>>>(static_cast<const T*>(p.ck), ck_stride, hkv,
                                                                 p.nb_total, const_cast<float*>(p.ckn));
    LSRM_LAUNCH_CHECK();
  }
  LSRM_CUDA_TRY(cudaFuncSetAttribute(qblock_scores_kernel<D, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_scores));
  {
    ProfScope ps("block_topk_fast", s);
    qblock_scores_kernel<D, BF16><<<dim3(p.nqb, hkv), kSfThreads, smem_scores, s>>>(mq, mck, p);
    LSRM_LAUNCH_CHECK();
  }
  if (smem_select > 48 * 1024)
    LSRM_CUDA_TRY(cudaFuncSetAttribute(qblock_select_kernel<D, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_select));
  {
    ProfScope ps("block_topk_select", s);
    const long long items = (long long)p.nqb * hkv, per = kSelThreads / 32;
    qblock_select_kernel<D, BF16><<<(int)((items + per - 1) / per), kSelThreads, smem_select, s>>>(p);
    LSRM_LAUNCH_CHECK();
  }
  return LSRM_OK;
}

// Shared-memory sizes of the fast path's two kernels, 0 when it does not fit
// (the exact scorer then serves the call).
static void fast_smem(int D, int G, int nb_cap, size_t* scores, size_t* select) {
  *scores = D == 64 ? SfLayout<64>::bytes(nb_cap) : D == 32 ? SfLayout<32>::bytes(nb_cap) : SfLayout<16>::bytes(nb_cap);
  constexpr int W = kSelThreads / 32;
  *select = 128 + W * (D == 64 ? sizeof(SelWarpMem<64>) : D == 32 ? sizeof(SelWarpMem<32>) : sizeof(SelWarpMem<16>));
  if (G > kSfCols || *scores > 220 * 1024 || *select > 220 * 1024) *scores = *select = 0;
}

// Workspace of the fast path: the key norms and the per-(query block, kv
// head) score bounds; 0 when the fast path does not serve the problem.
size_t fast_scorer_workspace_bytes(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int num_query_blocks) {
  if (num_query_blocks <= 0 || !meta || !shape || shape->num_kv_heads <= 0) return 0;
  const int G = shape->num_q_heads / shape->num_kv_heads;
  const int nb_cap = std::max(meta->num_blocks, 1);
  size_t a, b;
  fast_smem(shape->head_dim, G, nb_cap, &a, &b);
  if (!a) return 0;
  const size_t hkv = (size_t)shape->num_kv_heads;
  return align_up(4 * hkv * nb_cap, 256) + align_up(8 * hkv * (size_t)num_query_blocks * nb_cap, 256);
}

// Returns LSRM_ERR_UNSUPPORTED (without launching) when the problem does not
// fit the fast path; the caller then uses the exact scorer.
int launch_qblock_topk_fast(const lsrm_varlen* meta, const lsrm_attn_shape* shape, const void* q, const void* ck,
                            const float* lse_ln, int topk, const int32_t* cu_query_blocks, int num_query_blocks,
                            int force_self, double qk_scale, int32_t* out, void* workspace, size_t workspace_bytes,
                            int* err, cudaStream_t s) {
  const int D = shape->head_dim;
  const int G = shape->num_q_heads / shape->num_kv_heads;
  const int nb_cap = std::max(meta->num_blocks, 1);
  size_t smem_scores, smem_select;
  fast_smem(D, G, nb_cap, &smem_scores, &smem_select);
  if (!smem_scores) return LSRM_ERR_UNSUPPORTED;
  const size_t need = fast_scorer_workspace_bytes(meta, shape, num_query_blocks);
  if (!workspace || workspace_bytes < need) {
    set_error("block_topk: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  // 256 TMEM columns per scores CTA: two CTAs may share an SM (their 512 columns fit)
  CUtensorMap mq, mck;
  int rc;
  if ((rc = make_tmap_3d(&mq, q, D, shape->num_q_heads, meta->total_q, shape->q_token_stride, G, kSfCols / G)))
    return rc;
  if ((rc = make_tmap_3d(&mck, ck, D, shape->num_kv_heads, meta->num_blocks, shape->kv_token_stride, 1, 128))) return rc;
  const size_t hkv = (size_t)shape->num_kv_heads;
  FastScoreParams p{};
  p.q = q;
  p.ck = ck;
  p.lse = lse_ln;
  p.cu_seqlens_q = meta->cu_seqlens_q;
  p.cu_cblocks = meta->cu_seqblocks;
  p.cu_qblocks = cu_query_blocks;
  p.out = out;
  p.q_tok_stride = shape->q_token_stride;
  p.ck_tok_stride = shape->kv_token_stride;
  p.num_seqs = meta->num_seqs;
  p.total_q = meta->total_q;
  p.G = G;
  p.topk = topk;
  p.force_self = force_self;
  p.nb_cap = nb_cap;
  p.nb_total = meta->num_blocks;
  p.nqb = num_query_blocks;
  p.hkv = (int)hkv;
  p.ckn = static_cast<const float*>(workspace);
  p.bounds = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align_up(4 * hkv * nb_cap, 256));
  p.qk_scale = (float)qk_scale;
  p.err = err;
  const bool bf16 = shape->dtype == LSRM_DTYPE_BF16;
  const long long cks = shape->kv_token_stride;
  if (D == 64)
    return bf16 ? launch_fast_t<64, true>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s)
                : launch_fast_t<64, false>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s);
  if (D == 32)
    return bf16 ? launch_fast_t<32, true>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s)
                : launch_fast_t<32, false>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s);
  return bf16 ? launch_fast_t<16, true>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s)
              : launch_fast_t<16, false>(mq, mck, p, (int)hkv, smem_scores, smem_select, cks, s);
}

}  // namespace lsrm
