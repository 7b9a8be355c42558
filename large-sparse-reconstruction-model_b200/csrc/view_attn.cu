// Image-side block selection of the reference's 3D-aware attention maps
// (misc/sparse_utils.py:653-1200, with use_3d_aware_attn):
//
//   lsrm_image_token_points   from_imcoords_to_points (:653-687): per image
//                             token the surface point of its patch with the
//                             largest mask value (first in row-major order).
//   lsrm_view_block_topk      the block selection of build_volume_to_image_attn
//                             (:991-1200) and build_image_to_image_attn
//                             (:690-898) for query points (voxels or image
//                             tokens): per view, the ``win`` selected blocks
//                             nearest to the point's projection; per such
//                             candidate the smallest masked 3D distance to the
//                             block's surface points (compute_block_topk_dist_
//                             chunked, :16-56); over all views the ``topk``
//                             smallest, listed in candidate order.
//
// The reference gathers [chunk, win, points, 3] tensors per view; here one
// warp owns 32 consecutive queries (neighbours in the sorted token order, so
// their windows overlap) and walks the union of their windows once per view:
// each block's valid surface points (packed once per launch) are streamed as
// warp-wide broadcast loads and every lane folds them into its own minimum.
// Arithmetic follows the reference's fp32 operations in order, without
// contraction: the projection is torch's CPU matmul (a fused multiply-add
// chain over k = 0..3), distances are (dx^2 + dy^2) + dz^2, the candidate
// value is sqrt (correctly rounded) of the smallest valid distance, capped at
// max_dist when the block has an invalid point.  Ties go to the lower
// position (the reference leaves them to torch.topk).
#include <algorithm>
#include <cstdint>

#include "host_util.h"

namespace lsrm {

namespace {

constexpr int kMaxCand = 512;  // views * window per query
constexpr int kMaxWin = 25;

struct ViewGeom {
  int B, M, H, W, S;
  int bp;   // block size in pixels (patch_size * block_size)
  int bw;   // blocks per row (== per column)
  int nbi;  // blocks per image
  int ib;   // surface points per block side
  int P;    // surface points per block
  int T;    // tile side (surface points): ceil(ib / 4), so at most 4 x 4 tiles per block
  int nt;   // tiles per block side
  int NT;   // tiles per block (<= kMaxTiles)
  int TC;   // points per tile, rounded up to a multiple of 4
  int R;    // floats per packed block record
  int win, Cmax;
};

// A packed block record (floats): per tile its valid-point count (as int) and
// bounding box (lo xyz, hi xyz), then the points as x[NT * TC], y[...], z[...],
// tile t's valid points at [t * TC, t * TC + count), +inf up to the next
// multiple of 4.
constexpr int kMaxTiles = 16;
constexpr int kHdr = kMaxTiles * 7;  // counts, then boxes

int va_grid(long long work, int threads) {
  return (int)std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, 1ll << 30));
}

__global__ void image_token_points_kernel(const int4* __restrict__ coords, long long n, const float* __restrict__ sp,
                                          const float* __restrict__ sm, int B, int M, int S, int pr,
                                          float* __restrict__ out, int* err) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int4 c = coords[t];  // (batch, image, patch row, patch column)
  if (c.x < 0 || c.x >= B || c.y < 0 || c.y >= M || c.z < 0 || c.z >= pr || c.w < 0 || c.w >= pr) {
    atomicOr(err, LSRM_ERR_BAD_INDEX);
    out[3 * t] = out[3 * t + 1] = out[3 * t + 2] = 0.f;
    return;
  }
  const int ps = S / pr;
  const long long img = (long long)c.x * M + c.y;
  const float* mk = sm + img * S * S;
  int by = c.z * ps, bx = c.w * ps;
  float best = mk[(long long)by * S + bx];
  int bi = 0;
  for (int j = 1; j < ps * ps; ++j) {  // first maximum in row-major order
    const float v = mk[(long long)(by + j / ps) * S + bx + j % ps];
    if (v > best) {
      best = v;
      bi = j;
    }
  }
  const float* p = sp + ((img * S + by + bi / ps) * S + bx + bi % ps) * 3;
  out[3 * t] = p[0];
  out[3 * t + 1] = p[1];
  out[3 * t + 2] = p[2];
}

// One CTA per (image, block): whether the block's pixel mask has a non-zero
// value, and its valid surface points (mask > 0.2) packed tile by tile with
// each tile's bounding box (the order inside a tile is free: only the minimum
// distance is used; the +inf pads are never a minimum).
__global__ void view_block_prep_kernel(const float* __restrict__ mask, long long img_stride,
                                       const float* __restrict__ sp, const float* __restrict__ sm, ViewGeom g,
                                       int* __restrict__ cnt, int* __restrict__ selflag, float* __restrict__ packed) {
  const int blk = blockIdx.x, bm = blockIdx.y;
  const int by = blk / g.bw, bx = blk % g.bw;
  const float* mi = mask + (long long)bm * img_stride;
  int any = 0;
  for (int i = threadIdx.x; i < g.bp * g.bp && !any; i += blockDim.x) {
    const int y = i / g.bp, x = i % g.bp;
    any = mi[(long long)(by * g.bp + y) * g.W + bx * g.bp + x] != 0.f;
  }
  any = __syncthreads_or(any);
  __shared__ int tcount[kMaxTiles];
  if (threadIdx.x < kMaxTiles) tcount[threadIdx.x] = 0;
  __syncthreads();
  const long long gb = (long long)bm * g.nbi + blk;
  float* rec = packed + gb * g.R;
  float* X = rec + kHdr;
  const int span = g.NT * g.TC;
  for (int i = threadIdx.x; i < g.P; i += blockDim.x) {
    const int iy = i / g.ib, ix = i % g.ib;
    const long long pix = ((long long)bm * g.S + by * g.ib + iy) * g.S + bx * g.ib + ix;
    if (sm[pix] > 0.2f) {
      const int t = (iy / g.T) * g.nt + ix / g.T;
      const int slot = t * g.TC + atomicAdd(&tcount[t], 1);
      X[slot] = sp[3 * pix];
      X[span + slot] = sp[3 * pix + 1];
      X[2 * span + slot] = sp[3 * pix + 2];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int t = warp; t < kMaxTiles; t += nwarps) {  // per tile: pads and bounding box
    const int c = t < g.NT ? tcount[t] : 0;
    float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int i = lane; i < c; i += 32) {
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const float v = X[a * span + t * g.TC + i];
        lo[a] = fminf(lo[a], v);
        hi[a] = fmaxf(hi[a], v);
      }
    }
#pragma unroll
    for (int a = 0; a < 3; ++a) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
        hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
      }
    }
    if (t < g.NT && lane < 3 && c + lane < ((c + 3) & ~3)) {
#pragma unroll
      for (int a = 0; a < 3; ++a) X[a * span + t * g.TC + c + lane] = INFINITY;
    }
    if (lane == 0) {
      reinterpret_cast<int*>(rec)[t] = c;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        rec[kMaxTiles + 6 * t + a] = lo[a];
        rec[kMaxTiles + 6 * t + 3 + a] = hi[a];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0;
    for (int t = 0; t < g.NT; ++t) c += tcount[t];
    cnt[gb] = c;
    selflag[gb] = any;
  }
}

// Packed fp32 pairs (sm_100): two independent IEEE round-to-nearest
// operations per instruction, bit-identical to the scalar ones.
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_splat(float v) {
  const unsigned long long u = __float_as_uint(v);
  return u | (u << 32);
}
__device__ __forceinline__ float f2_min(unsigned long long v, float m) {
  return fminf(fminf(m, __uint_as_float((unsigned)v)), __uint_as_float((unsigned)(v >> 32)));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// One warp per batch element: the selected blocks of each view in row-major
// order, and per view (selected count, block offset, candidate offset,
// window size).
__global__ void view_image_list_kernel(const int* __restrict__ selflag, ViewGeom g, int* __restrict__ sel_list,
                                       int4* __restrict__ img_info, int* __restrict__ cand_total) {
  const int b = blockIdx.x, lane = threadIdx.x;
  int blk_off = 0, cand_off = 0;
  for (int m = 0; m < g.M; ++m) {
    const long long bm = (long long)b * g.M + m;
    int nsel = 0;
    for (int base = 0; base < g.nbi; base += 32) {
      const int j = base + lane;
      const bool f = j < g.nbi && selflag[bm * g.nbi + j];
      const unsigned bal = __ballot_sync(0xffffffffu, f);
      if (f) sel_list[bm * g.nbi + nsel + __popc(bal & ((1u << lane) - 1))] = j;
      nsel += __popc(bal);
    }
    const int wm = min(g.win, nsel);
    if (lane == 0) img_info[bm] = make_int4(nsel, blk_off, cand_off, wm);
    blk_off += nsel;
    cand_off += wm;
  }
  if (lane == 0) cand_total[b] = cand_off;
}

// Lane = query, CTA = 128 consecutive queries.  Per view (and per batch
// element present in the CTA, normally one): every lane projects its point and
// keeps the WM nearest selected blocks; the CTA marks the union of its
// windows in a shared bitmap, then streams the union's blocks through two
// shared-memory buffers (cp.async, the next block loading while the current
// one is evaluated).  A warp evaluates a staged block only when one of its
// lanes has it in its window; every lane of such a warp folds the block's
// points into its own minimum with packed fp32 pairs, 4 points per step.
constexpr int kCandThreads = 128;

// Copies block blk's packed record into stage buffer buf.
__device__ __forceinline__ void stage_points(int blk, int buf, long long gbase, int R,
                                             const float* __restrict__ packed, float* stage, int tid) {
  const float* src = packed + (gbase + blk) * R;
  float* dst = stage + buf * R;
  for (int i = tid; i < (R >> 2); i += kCandThreads) cp_async16(dst + 4 * i, src + 4 * i);
}

// Folds tile t of a staged record into the lane's minimum (4 points per step).
__device__ __forceinline__ float tile_min(const float* rec, int t, int TC, int span, unsigned long long P2x,
                                          unsigned long long P2y, unsigned long long P2z, float mn) {
  const int c4 = (reinterpret_cast<const int*>(rec)[t] + 3) >> 2;
  const float* base = rec + kHdr + t * TC;
  const ulonglong2* X = reinterpret_cast<const ulonglong2*>(base);
  const ulonglong2* Y = reinterpret_cast<const ulonglong2*>(base + span);
  const ulonglong2* Z = reinterpret_cast<const ulonglong2*>(base + 2 * span);
  float mn1 = INFINITY;
#pragma unroll 2
  for (int i = 0; i < c4; ++i) {
    const ulonglong2 x = X[i], y = Y[i], z = Z[i];
    {
      const unsigned long long dx = f2_sub(P2x, x.x), dy = f2_sub(P2y, y.x), dz = f2_sub(P2z, z.x);
      mn = f2_min(f2_add(f2_add(f2_mul(dx, dx), f2_mul(dy, dy)), f2_mul(dz, dz)), mn);
    }
    {
      const unsigned long long dx = f2_sub(P2x, x.y), dy = f2_sub(P2y, y.y), dz = f2_sub(P2z, z.y);
      mn1 = f2_min(f2_add(f2_add(f2_mul(dx, dx), f2_mul(dy, dy)), f2_mul(dz, dz)), mn1);
    }
  }
  return fminf(mn, mn1);
}

template <int WM>
__global__ void __launch_bounds__(kCandThreads, (WM <= 9 ? 8 : 6)) view_candidates_kernel(
    const float* __restrict__ pts, const int32_t* __restrict__ qc, long long n, ViewGeom g,
    const float* __restrict__ w2c, const float* __restrict__ tan_half, const float* __restrict__ crop,
    float max_dist, const int* __restrict__ sel_list, const int4* __restrict__ img_info,
    const int* __restrict__ cnt, const float* __restrict__ packed, float* __restrict__ cand_val,
    int* __restrict__ cand_id, int* err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int nwords = (g.nbi + 31) >> 5;
  float* stage = reinterpret_cast<float*>(smem_raw);                  // [2][R]
  unsigned* bitmap = reinterpret_cast<unsigned*>(stage + 2 * g.R);    // [nwords]
  int* ulist = reinterpret_cast<int*>(bitmap + nwords);               // [nbi]
  __shared__ int s_ucount, s_blo, s_bhi;

  const int tid = threadIdx.x, lane = tid & 31;
  const long long q = (long long)blockIdx.x * kCandThreads + tid;
  const bool in_range = q < n;
  int b = in_range ? qc[4 * q] : 0;
  const bool live = in_range && b >= 0 && b < g.B;
  if (in_range && !live) atomicOr(err, LSRM_ERR_BAD_INDEX);
  if (tid == 0) {
    s_blo = INT32_MAX;
    s_bhi = -1;
  }
  for (int w = tid; w < nwords; w += kCandThreads) bitmap[w] = 0u;
  __syncthreads();
  if (live) {
    atomicMin(&s_blo, b);
    atomicMax(&s_bhi, b);
  }
  float px = 0.f, py = 0.f, pz = 0.f;
  if (live) {
    px = pts[3 * q];
    py = pts[3 * q + 1];
    pz = pts[3 * q + 2];
  }
  const unsigned long long P2x = f2_splat(px), P2y = f2_splat(py), P2z = f2_splat(pz);
  __syncthreads();
  const int blo = s_blo, bhi = s_bhi;  // no live query: blo > bhi, nothing to do

  for (int m = 0; m < g.M; ++m) {
    for (int bb = blo; bb <= bhi; ++bb) {
      const bool mine_b = live && b == bb;
      const int bm = bb * g.M + m;
      const int4 info = img_info[bm];  // (selected, block offset, candidate offset, window)
      const int wm = mine_b ? info.w : 0;
      float bd[WM];
      int bj[WM], key[WM];
      float val[WM];
#pragma unroll
      for (int i = 0; i < WM; ++i) {
        bd[i] = INFINITY;
        bj[i] = INT32_MAX;
        key[i] = -1;
        val[i] = 0.f;
      }
      const int* sl = sel_list + (long long)bm * g.nbi;
      if (wm > 0) {
        const float* W = w2c + (long long)bm * 16;
        float pc[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {  // [p, 1] @ world_to_cam^T, k = 0..3 as one fused chain
          float t = __fmul_rn(px, W[4 * r]);
          t = __fmaf_rn(py, W[4 * r + 1], t);
          t = __fmaf_rn(pz, W[4 * r + 2], t);
          pc[r] = __fadd_rn(t, W[4 * r + 3]);
        }
        const float den = fmaxf(-pc[2], 1e-6f);
        const float th = tan_half[bm];
        float u = __fmul_rn(0.5f, __fadd_rn(__fdiv_rn(__fdiv_rn(pc[0], den), th), 1.f));
        float v = __fmul_rn(0.5f, __fadd_rn(__fdiv_rn(__fdiv_rn(-pc[1], den), th), 1.f));
        const float s1 = (float)(g.S - 1);
        if (crop) {
          const float* c = crop + (long long)bm * 4;  // (origin - 1, rows start, columns start, crop - 1)
          u = __fmul_rn(__fdiv_rn(__fsub_rn(__fmul_rn(u, c[0]), c[2]), c[3]), s1);
          v = __fmul_rn(__fdiv_rn(__fsub_rn(__fmul_rn(v, c[0]), c[1]), c[3]), s1);
        } else {
          u = __fmul_rn(u, s1);
          v = __fmul_rn(v, s1);
        }
        const float fib = (float)g.ib;
        const float bxq = __fdiv_rn(u, fib), byq = __fdiv_rn(v, fib);
        float worst = INFINITY;
        int filled = 0;
        for (int j = 0; j < info.x; ++j) {
          const int blk = sl[j];
          const float dx = __fsub_rn(bxq, (float)(blk % g.bw) + 0.5f);
          const float dy = __fsub_rn(byq, (float)(blk / g.bw) + 0.5f);
          float d = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
          if (d != d) d = INFINITY;  // non-finite input: rank last, keep the slots filled
          // positions arrive in increasing order: an equal distance never displaces an earlier one
          if (filled < wm || d < worst) {
            float cd = d;
            int cj = j;
#pragma unroll
            for (int i = 0; i < WM; ++i) {  // insertion into the sorted slots [0, wm); empty slots hold (inf, INT_MAX)
              if (i < wm && (cd < bd[i] || (cd == bd[i] && cj < bj[i]))) {
                const float td = bd[i];
                const int tj = bj[i];
                bd[i] = cd;
                bj[i] = cj;
                cd = td;
                cj = tj;
              }
            }
            filled = min(filled + 1, wm);
#pragma unroll
            for (int i = 0; i < WM; ++i)
              if (i == wm - 1) worst = bd[i];
          }
        }
#pragma unroll
        for (int i = 0; i < WM; ++i) {
          if (i < wm) {
            key[i] = sl[bj[i]];
            atomicOr(&bitmap[key[i] >> 5], 1u << (key[i] & 31));
          }
        }
      }
      __syncthreads();
      if (tid < 32) {  // the union in ascending block order; the bitmap is cleared for the next round
        int base = 0;
        for (int w0 = 0; w0 < nwords; w0 += 32) {
          const int w = w0 + lane;
          const unsigned bits = w < nwords ? bitmap[w] : 0u;
          if (w < nwords) bitmap[w] = 0u;
          const int c = __popc(bits);
          int incl = c;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
          }
          int pos = base + incl - c;
          for (unsigned x = bits; x; x &= x - 1) ulist[pos++] = (w << 5) + __ffs(x) - 1;
          base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) s_ucount = base;
      }
      __syncthreads();
      const int ucount = s_ucount;
      const long long gbase = (long long)bm * g.nbi;
      if (ucount > 0) stage_points(ulist[0], 0, gbase, g.R, packed, stage, tid);
      cp_async_commit();
      for (int u = 0; u < ucount; ++u) {
        if (u + 1 < ucount) stage_points(ulist[u + 1], (u + 1) & 1, gbase, g.R, packed, stage, tid);
        cp_async_commit();
        cp_async_wait1();
        __syncthreads();
        const int blk = ulist[u];
        bool want = false;
#pragma unroll
        for (int i = 0; i < WM; ++i) want |= key[i] == blk;
        if (__any_sync(0xffffffffu, want)) {
          const int c = cnt[gbase + blk];
          const float* rec = stage + (u & 1) * g.R;
          const int span = g.NT * g.TC;
          // per tile a lower bound of every point's d^2: the box gap per axis, squared and summed in the
          // same order (each rounded step is monotone, so no point of the tile can come out below it)
          float lb[kMaxTiles];
          int first = 0;
          float best = INFINITY;
#pragma unroll
          for (int t = 0; t < kMaxTiles; ++t) {
            lb[t] = INFINITY;
            if (t < g.NT) {
              const float* bx = rec + kMaxTiles + 6 * t;
              const float gx = fmaxf(fmaxf(__fsub_rn(bx[0], px), __fsub_rn(px, bx[3])), 0.f);
              const float gy = fmaxf(fmaxf(__fsub_rn(bx[1], py), __fsub_rn(py, bx[4])), 0.f);
              const float gz = fmaxf(fmaxf(__fsub_rn(bx[2], pz), __fsub_rn(pz, bx[5])), 0.f);
              lb[t] = __fadd_rn(__fadd_rn(__fmul_rn(gx, gx), __fmul_rn(gy, gy)), __fmul_rn(gz, gz));
              if (lb[t] < best) {
                best = lb[t];
                first = t;
              }
            }
          }
          // the tiles some lane bounds lowest first, then the others unless no lane can improve
          const unsigned firsts = __reduce_or_sync(0xffffffffu, best < INFINITY ? 1u << first : 0u);
          float mn = INFINITY;
          for (unsigned f = firsts; f; f &= f - 1)
            mn = tile_min(rec, __ffs(f) - 1, g.TC, span, P2x, P2y, P2z, mn);
#pragma unroll
          for (int t = 0; t < kMaxTiles; ++t) {
            if (t < g.NT && !((firsts >> t) & 1u) && __any_sync(0xffffffffu, lb[t] < mn))
              mn = tile_min(rec, t, g.TC, span, P2x, P2y, P2z, mn);
          }
          float dist = __fsqrt_rn(mn);
          if (c < g.P) dist = fminf(dist, max_dist);
#pragma unroll
          for (int i = 0; i < WM; ++i)
            if (key[i] == blk) val[i] = dist;
        }
        __syncthreads();  // the buffer is refilled two blocks later
      }
      if (wm > 0) {
        const long long base = q * g.Cmax + info.z;
#pragma unroll
        for (int i = 0; i < WM; ++i) {
          if (i < wm) {
            cand_val[base + i] = val[i];
            cand_id[base + i] = bj[i] + info.y;
          }
        }
      }
    }
  }
}

// Warp = query: keep the K = min(C, topk) candidates smallest by (value,
// position), in position order, pad with -1.  Values are non-negative
// floats (distances or +inf), whose bit patterns order like the values: the
// K-th smallest pattern is found bit by bit from the top (31 rounds of a
// warp-wide count), then the candidates below it and, in position order, as
// many equal to it as are missing are kept.
template <int R>
__global__ void __launch_bounds__(256) view_final_kernel(const int32_t* __restrict__ qc, long long n, int B,
                                                         const int* __restrict__ cand_total, int Cmax, int topk,
                                                         const float* __restrict__ cand_val,
                                                         const int* __restrict__ cand_id, int32_t* __restrict__ out) {
  const long long q = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (q >= n) return;  // warp-uniform
  const int b = qc[4 * q];
  const int C = (b >= 0 && b < B) ? cand_total[b] : 0;
  const int K = min(C, topk);
  unsigned key[R];
  int id[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int pos = r * 32 + lane;
    key[r] = pos < C ? __float_as_uint(cand_val[q * Cmax + pos]) : 0xffffffffu;  // padding sorts last
    id[r] = pos < C ? cand_id[q * Cmax + pos] : -1;
  }
  unsigned T = 0;  // the largest pattern with fewer than K keys below it = the K-th smallest key
  if (K > 0) {
    for (int bit = 30; bit >= 0; --bit) {  // bit 31 (sign) is clear in every key
      const unsigned cand = T | (1u << bit);
      int below = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) below += __popc(__ballot_sync(0xffffffffu, key[r] < cand));
      if (below < K) T = cand;
    }
  }
  int below = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) below += __popc(__ballot_sync(0xffffffffu, key[r] < T));
  const int need = K - below;  // keys equal to T to keep, the first ones by position
  const unsigned lt_mask = (1u << lane) - 1;
  int base = 0, eq_seen = 0;
  int32_t* o = out + q * topk;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const bool valid = r * 32 + lane < C;
    const bool eq = valid && key[r] == T;
    const unsigned be = __ballot_sync(0xffffffffu, eq);
    const bool sel = K > 0 && valid && (key[r] < T || (eq && eq_seen + __popc(be & lt_mask) < need));
    eq_seen += __popc(be);
    const unsigned bal = __ballot_sync(0xffffffffu, sel);
    if (sel) o[base + __popc(bal & lt_mask)] = id[r];
    base += __popc(bal);
  }
  for (int s = K + lane; s < topk; s += 32) o[s] = -1;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct ViewWs {
  int *cnt, *selflag, *sel_list, *cand_total;
  int4* img_info;
  float* packed;
  float* cand_val;
  int* cand_id;
  size_t bytes;
};

ViewWs view_ws_layout(const ViewGeom& g, long long n, char* base) {
  ViewWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  const size_t nb = (size_t)g.B * g.M * g.nbi;
  w.cnt = (int*)take(nb * 4);
  w.selflag = (int*)take(nb * 4);
  w.sel_list = (int*)take(nb * 4);
  w.img_info = (int4*)take((size_t)g.B * g.M * 16);
  w.cand_total = (int*)take((size_t)g.B * 4);
  w.packed = (float*)take(nb * g.R * 4);
  w.cand_val = (float*)take((size_t)n * g.Cmax * 4);
  w.cand_id = (int*)take((size_t)n * g.Cmax * 4);
  w.bytes = off;
  return w;
}

size_t cand_smem_bytes(const ViewGeom& g) {
  return (size_t)2 * g.R * 4 + (size_t)((g.nbi + 31) / 32) * 4 + (size_t)g.nbi * 4;
}

int view_geom(int32_t batch, int32_t views, int32_t H, int32_t W, int32_t S, int32_t patch, int32_t block, int32_t win,
              ViewGeom* g) {
  LSRM_CHECK_ARG(batch >= 1 && views >= 1 && H >= 1 && W >= 1 && S >= 1 && patch >= 1 && block >= 1, "bad sizes");
  const int bp = patch * block;
  LSRM_CHECK_ARG(H % bp == 0 && W % bp == 0, "image size (%d x %d) must be a multiple of patch*block (%d)", H, W,
                 bp);
  const int bh = H / bp, bw = W / bp;
  LSRM_CHECK_ARG(bh == bw && S % bh == 0,
                 "blocks per side must agree (%d x %d) and divide the surface resolution (%d)", bh, bw, S);
  LSRM_CHECK_ARG(win >= 1 && win <= kMaxWin, "window must be in [1, %d] (got %d)", kMaxWin, win);
  LSRM_CHECK_ARG((long long)views * win <= kMaxCand, "views * window must be <= %d (got %d)", kMaxCand, views * win);
  g->B = batch;
  g->M = views;
  g->H = H;
  g->W = W;
  g->S = S;
  g->bp = bp;
  g->bw = bw;
  g->nbi = bh * bw;
  g->ib = S / bh;
  g->P = g->ib * g->ib;
  g->T = (g->ib + 3) / 4;
  g->nt = (g->ib + g->T - 1) / g->T;
  g->NT = g->nt * g->nt;
  g->TC = (g->T * g->T + 3) & ~3;
  g->R = (kHdr + 3 * g->NT * g->TC + 3) & ~3;
  LSRM_CHECK_ARG(cand_smem_bytes(*g) <= 200 * 1024, "surface points per block (%d) exceed the shared-memory stage",
                 g->P);
  g->win = win;
  g->Cmax = views * win;
  return LSRM_OK;
}

template <int WM>
int launch_candidates(const float* pts, const int32_t* qc, long long n, const ViewGeom& g, const float* w2c,
                      const float* th, const float* crop, float max_dist, const ViewWs& w, int* err, cudaStream_t s) {
  const size_t smem = cand_smem_bytes(g);
  if (smem > 48 * 1024)
    LSRM_CUDA_TRY(cudaFuncSetAttribute(view_candidates_kernel<WM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  view_candidates_kernel<WM><<<va_grid(n, kCandThreads), kCandThreads, smem, s>>>(
      pts, qc, n, g, w2c, th, crop, max_dist, w.sel_list, w.img_info, w.cnt, w.packed, w.cand_val, w.cand_id, err);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

template <int R>
int launch_final(const int32_t* qc, long long n, const ViewGeom& g, int topk, const ViewWs& w, int32_t* out,
                 cudaStream_t s) {
  view_final_kernel<R><<<va_grid(n * 32, 256), 256, 0, s>>>(qc, n, g.B, w.cand_total, g.Cmax, topk, w.cand_val,
                                                             w.cand_id, out);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

}  // namespace

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_image_token_points(const int32_t* image_coords, int64_t n_tokens, const float* surface_points,
                                       const float* surface_masks, int32_t batch, int32_t views, int32_t surface_res,
                                       int32_t patch_res, float* points, int* err_flags, void* stream) {
  LSRM_CHECK_ARG(n_tokens >= 0 && batch >= 1 && views >= 1 && patch_res >= 1 && surface_res >= patch_res,
                 "bad sizes");
  LSRM_CHECK_ARG(surface_res % patch_res == 0, "surface resolution (%d) must be a multiple of the patch grid (%d)",
                 surface_res, patch_res);
  LSRM_CHECK_ARG(((uintptr_t)image_coords & 15) == 0, "image coords must be 16-byte aligned ([n, 4] int32)");
  LSRM_CHECK_ARG(err_flags != nullptr, "err_flags is required");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  image_token_points_kernel<<<va_grid(n_tokens, 256), 256, 0, s>>>(
      reinterpret_cast<const int4*>(image_coords), n_tokens, surface_points, surface_masks, batch, views, surface_res,
      patch_res, points, err_flags);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int64_t lsrm_view_block_topk_workspace_bytes(int32_t batch, int32_t views, int32_t image_h,
                                                        int32_t image_w, int32_t surface_res, int32_t patch_size,
                                                        int32_t block_size, int32_t win, int64_t n_queries) {
  ViewGeom g;
  if (view_geom(batch, views, image_h, image_w, surface_res, patch_size, block_size, win, &g) != LSRM_OK) return 0;
  return (int64_t)view_ws_layout(g, n_queries, nullptr).bytes;
}

extern "C" int lsrm_view_block_topk(const float* points, const int32_t* point_coords, int64_t n_queries,
                                    int32_t batch, int32_t views, const float* mask_input,
                                    int64_t mask_image_stride, int32_t image_h, int32_t image_w,
                                    const float* surface_points, const float* surface_masks, int32_t surface_res,
                                    int32_t patch_size, int32_t block_size, const float* world_to_cam,
                                    const float* tan_half_fov, const float* crop, int32_t win, int32_t topk,
                                    float max_dist, int32_t* block_topk, void* workspace, int64_t workspace_bytes,
                                    int* err_flags, void* stream) {
  ViewGeom g;
  int rc = view_geom(batch, views, image_h, image_w, surface_res, patch_size, block_size, win, &g);
  if (rc) return rc;
  LSRM_CHECK_ARG(n_queries >= 0 && n_queries < (1ll << 31), "bad query count");
  LSRM_CHECK_ARG(topk >= 1, "topk must be >= 1");
  LSRM_CHECK_ARG(mask_image_stride >= (int64_t)image_h * image_w, "mask image stride must be >= H*W");
  LSRM_CHECK_ARG(((uintptr_t)point_coords & 15) == 0, "point coords must be 16-byte aligned ([n, 4] int32)");
  LSRM_CHECK_ARG(err_flags != nullptr, "err_flags is required");
  const ViewWs need = view_ws_layout(g, n_queries, nullptr);
  if (workspace_bytes < (int64_t)need.bytes || (need.bytes && workspace == nullptr)) {
    set_error("workspace of %lld bytes is smaller than the %zu needed", (long long)workspace_bytes, need.bytes);
    return LSRM_ERR_WORKSPACE;
  }
  if (n_queries == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("view_block_topk", s);
  const ViewWs w = view_ws_layout(g, n_queries, static_cast<char*>(workspace));
  view_block_prep_kernel<<<dim3(g.nbi, g.B * g.M), 256, 0, s>>>(mask_input, mask_image_stride, surface_points,
                                                                 surface_masks, g, w.cnt, w.selflag, w.packed);
  LSRM_LAUNCH_CHECK();
  view_image_list_kernel<<<g.B, 32, 0, s>>>(w.selflag, g, w.sel_list, w.img_info, w.cand_total);
  LSRM_LAUNCH_CHECK();
  if (win <= 4)
    rc = launch_candidates<4>(points, point_coords, n_queries, g, world_to_cam, tan_half_fov, crop, max_dist, w,
                              err_flags, s);
  else if (win <= 9)
    rc = launch_candidates<9>(points, point_coords, n_queries, g, world_to_cam, tan_half_fov, crop, max_dist, w,
                              err_flags, s);
  else if (win <= 16)
    rc = launch_candidates<16>(points, point_coords, n_queries, g, world_to_cam, tan_half_fov, crop, max_dist, w,
                               err_flags, s);
  else
    rc = launch_candidates<25>(points, point_coords, n_queries, g, world_to_cam, tan_half_fov, crop, max_dist, w,
                               err_flags, s);
  if (rc) return rc;
  const int rows = (g.Cmax + 31) / 32;
  if (rows <= 1) return launch_final<1>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 2) return launch_final<2>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 3) return launch_final<3>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 4) return launch_final<4>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 5) return launch_final<5>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 6) return launch_final<6>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 8) return launch_final<8>(point_coords, n_queries, g, topk, w, block_topk, s);
  if (rows <= 12) return launch_final<12>(point_coords, n_queries, g, topk, w, block_topk, s);
  return launch_final<16>(point_coords, n_queries, g, topk, w, block_topk, s);
}
