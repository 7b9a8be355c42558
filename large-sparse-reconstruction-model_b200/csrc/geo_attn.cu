// Geometric volume-to-volume block selection (build_volume_to_volume_attn
// with use_3d_aware_attn, misc/sparse_utils.py:1203-1279): every voxel token
// selects the topk blocks of its batch element whose centroid is nearest to
// the token's point, as sorted sequence-local block ids (-1 padding when the
// element has fewer blocks).
//
// The reference materialises an [n, blocks] distance matrix per batch element
// and runs torch.topk on it; here one thread per token streams the block
// centroids of its element (L1-resident, the same for every thread of a CTA)
// and keeps the k best in registers.  Arithmetic follows the reference's
// fp32 operations in order, with no fused multiply-add:
//   point  (x, y, z) = 2 * (c / (res - 1) - 0.5) * r   (from_volcoords_to_points, :644-650)
//   centre = sequential fp32 sum of its tokens' points / count (torch.segment_reduce mean)
//   d^2    = ((dx*dx + dy*dy) + dz*dz)
// and ranks by d^2 (ties to the lower block id): the reference ranks
// sqrt(d^2), which is monotone, so the selected sets agree except where
// rounding inside sqrt makes distinct d^2 equal (a tie the reference breaks
// arbitrarily).
#include <algorithm>
#include <cstdint>

#include "host_util.h"

namespace lsrm {

namespace {

int geo_grid(long long work, int threads) {
  return (int)std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, 1ll << 30));
}

__device__ __forceinline__ float3 voxel_point(const int4 c, float den, float r) {
  // 2 * (c / (res - 1) - 0.5) * r, evaluated left to right in fp32 (IEEE division)
  auto f = [&](int v) { return __fmul_rn(__fmul_rn(2.f, __fsub_rn(__fdiv_rn((float)v, den), 0.5f)), r); };
  return make_float3(f(c.w), f(c.z), f(c.y));  // (x, y, z) from (batch, z, y, x)
}

// Block centroids, one warp per block: the lanes load and convert 32
// tokens at a time, lane 0 adds them in token order (the sequential fp32 sum
// of the reference's segment_reduce) from the lanes' registers.
__global__ void geo_centroid_kernel(const int32_t* __restrict__ coords, const int32_t* __restrict__ cu_sb, int batch,
                                    const int32_t* __restrict__ cu_blk, float den, float r, long long cap,
                                    float* __restrict__ cent) {
  const long long j = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= cap || j >= cu_sb[batch]) return;  // warp-uniform
  const int t0 = cu_blk[j], t1 = cu_blk[j + 1];
  float sx = 0.f, sy = 0.f, sz = 0.f;
  for (int b = t0; b < t1; b += 32) {
    float3 p = make_float3(0.f, 0.f, 0.f);
    if (b + lane < t1) p = voxel_point(reinterpret_cast<const int4*>(coords)[b + lane], den, r);
    const int m = min(32, t1 - b);
    for (int i = 0; i < m; ++i) {
      const float px = __shfl_sync(0xffffffffu, p.x, i), py = __shfl_sync(0xffffffffu, p.y, i),
                  pz = __shfl_sync(0xffffffffu, p.z, i);
      sx = __fadd_rn(sx, px);
      sy = __fadd_rn(sy, py);
      sz = __fadd_rn(sz, pz);
    }
  }
  if (lane == 0) {
    const float n = (float)(t1 - t0);
    cent[3 * j] = __fdiv_rn(sx, n);
    cent[3 * j + 1] = __fdiv_rn(sy, n);
    cent[3 * j + 2] = __fdiv_rn(sz, n);
  }
}

// Per token: the k nearest blocks of its element (k <= K), sorted by id.
// The token's point is its voxel's (coords [n, 4]) or, with ``qpts``, given
// ([n, 3] floats; coords column 0 still names the batch element).
template <int K>
__global__ void geo_topk_kernel(const int32_t* __restrict__ coords, const float* __restrict__ qpts, long long n,
                                const int32_t* __restrict__ cu_sb, int batch, const float* __restrict__ cent,
                                float den, float r, int k, int32_t* __restrict__ out, int* err) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int4 c = reinterpret_cast<const int4*>(coords)[t];
  int32_t* o = out + t * k;
  if (c.x < 0 || c.x >= batch) {
    atomicOr(err, LSRM_ERR_BAD_INDEX);
    for (int i = 0; i < k; ++i) o[i] = -1;
    return;
  }
  const float3 p = qpts ? make_float3(qpts[3 * t], qpts[3 * t + 1], qpts[3 * t + 2]) : voxel_point(c, den, r);
  const int b0 = cu_sb[c.x], nb = cu_sb[c.x + 1] - b0;
  float bd[K];
  int bi[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    bd[i] = INFINITY;
    bi[i] = INT32_MAX;
  }
  float worst = INFINITY;  // the k-th best distance so far (slot k-1)
  int filled = 0;
  constexpr int U = 4;  // candidates whose loads and distances are computed ahead of the insertion checks
  for (int j0 = 0; j0 < nb; j0 += U) {
    float d2u[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = min(j0 + u, nb - 1);
      const float* q = cent + 3 * (size_t)(b0 + j);
      const float dx = __fsub_rn(p.x, __ldg(q)), dy = __fsub_rn(p.y, __ldg(q + 1)), dz = __fsub_rn(p.z, __ldg(q + 2));
      d2u[u] = __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
    const int j = j0 + u;
    const float d2 = d2u[u];
    // ids arrive in increasing order: an equal distance never displaces an earlier id
    if (j < nb && (filled < k || d2 < worst)) {
      float cd = d2;
      int ci = j;
#pragma unroll
      for (int i = 0; i < K; ++i) {  // insertion into the sorted slots [0, k)
        if (i < k && (cd < bd[i] || (cd == bd[i] && ci < bi[i]))) {
          const float td = bd[i];
          const int ti = bi[i];
          bd[i] = cd;
          bi[i] = ci;
          cd = td;
          ci = ti;
        }
      }
      filled = min(filled + 1, k);
#pragma unroll
      for (int i = 0; i < K; ++i)
        if (i == k - 1) worst = bd[i];
    }
    }
  }
  // the selected ids in ascending order (the reference sorts topk's indices)
#pragma unroll
  for (int i = 1; i < K; ++i) {
#pragma unroll
    for (int m = i; m > 0; --m) {
      if (m < k && bi[m] < bi[m - 1]) {
        const int ti = bi[m];
        bi[m] = bi[m - 1];
        bi[m - 1] = ti;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < K; ++i)
    if (i < k) o[i] = (i < nb) ? bi[i] : -1;
}

template <int K>
int launch_geo_topk(const int32_t* coords, const float* qpts, long long n, const int32_t* cu_sb, int batch,
                    const float* cent, float den, float r, int k, int32_t* out, int* err, cudaStream_t s) {
  geo_topk_kernel<K><<<geo_grid(n, 128), 128, 0, s>>>(coords, qpts, n, cu_sb, batch, cent, den, r, k, out, err);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

int dispatch_geo_topk(const int32_t* coords, const float* qpts, long long n, const int32_t* cu_sb, int batch,
                      const float* cent, float den, float r, int k, int32_t* out, int* err, cudaStream_t s) {
  if (k <= 8) return launch_geo_topk<8>(coords, qpts, n, cu_sb, batch, cent, den, r, k, out, err, s);
  if (k <= 16) return launch_geo_topk<16>(coords, qpts, n, cu_sb, batch, cent, den, r, k, out, err, s);
  if (k <= 32) return launch_geo_topk<32>(coords, qpts, n, cu_sb, batch, cent, den, r, k, out, err, s);
  return launch_geo_topk<64>(coords, qpts, n, cu_sb, batch, cent, den, r, k, out, err, s);
}

__global__ void voxel_points_kernel(const int32_t* __restrict__ coords, long long n, float den, float r,
                                    float* __restrict__ pts) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const float3 p = voxel_point(reinterpret_cast<const int4*>(coords)[t], den, r);
  pts[3 * t] = p.x;
  pts[3 * t + 1] = p.y;
  pts[3 * t + 2] = p.z;
}

}  // namespace

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_volume_block_topk(const int32_t* coords, int64_t n_tokens, const int32_t* cu_seqblocks,
                                      const int32_t* cu_block_include_tokens, int32_t batch, int32_t volume_res,
                                      float radius, int32_t topk, float* centroids, int32_t* block_topk,
                                      int* err_flags, void* stream) {
  LSRM_CHECK_ARG(n_tokens >= 0 && n_tokens < (1ll << 31) && batch >= 1 && volume_res >= 2, "bad sizes");
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(((uintptr_t)coords & 15) == 0, "coords must be 16-byte aligned ([n, 4] int32)");
  LSRM_CHECK_ARG(err_flags != nullptr, "err_flags is required");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("volume_block_topk", s);
  const float den = (float)(volume_res - 1);
  geo_centroid_kernel<<<geo_grid(n_tokens * 32, 256), 256, 0, s>>>(coords, cu_seqblocks, batch,
                                                                   cu_block_include_tokens, den, radius, n_tokens,
                                                                   centroids);
  LSRM_LAUNCH_CHECK();
  return dispatch_geo_topk(coords, nullptr, n_tokens, cu_seqblocks, batch, centroids, den, radius, topk, block_topk,
                           err_flags, s);
}

extern "C" int lsrm_points_volume_block_topk(const float* points, const int32_t* point_coords, int64_t n_points,
                                             const int32_t* volume_coords, int64_t n_voxels,
                                             const int32_t* cu_seqblocks, const int32_t* cu_block_include_tokens,
                                             int32_t batch, int32_t volume_res, float radius, int32_t topk,
                                             float* centroids, int32_t* block_topk, int* err_flags, void* stream) {
  LSRM_CHECK_ARG(n_points >= 0 && n_points < (1ll << 31) && n_voxels >= 0 && n_voxels < (1ll << 31) && batch >= 1 &&
                     volume_res >= 2,
                 "bad sizes");
  LSRM_CHECK_ARG(topk >= 1 && topk <= 64, "topk must be in [1, 64] (got %d)", topk);
  LSRM_CHECK_ARG(((uintptr_t)point_coords & 15) == 0 && ((uintptr_t)volume_coords & 15) == 0,
                 "coords must be 16-byte aligned ([n, 4] int32)");
  LSRM_CHECK_ARG(err_flags != nullptr && points != nullptr, "points and err_flags are required");
  if (n_points == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("points_volume_block_topk", s);
  const float den = (float)(volume_res - 1);
  if (n_voxels > 0) {
    geo_centroid_kernel<<<geo_grid(n_voxels * 32, 256), 256, 0, s>>>(volume_coords, cu_seqblocks, batch,
                                                                     cu_block_include_tokens, den, radius, n_voxels,
                                                                     centroids);
    LSRM_LAUNCH_CHECK();
  }
  return dispatch_geo_topk(point_coords, points, n_points, cu_seqblocks, batch, centroids, den, radius, topk,
                           block_topk, err_flags, s);
}

extern "C" int lsrm_voxel_points(const int32_t* coords, int64_t n_tokens, int32_t volume_res, float radius,
                                 float* points, void* stream) {
  LSRM_CHECK_ARG(n_tokens >= 0 && volume_res >= 2, "bad sizes");
  LSRM_CHECK_ARG(((uintptr_t)coords & 15) == 0, "coords must be 16-byte aligned ([n, 4] int32)");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  voxel_points_kernel<<<geo_grid(n_tokens, 256), 256, 0, s>>>(coords, n_tokens, (float)(volume_res - 1), radius,
                                                              points);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
