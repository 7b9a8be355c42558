// Output formatting of the upsampled volume decoder (the step after the
// sparse transformer): VolTransformer.prepare_volume_output,
// models_sparse/voldecoder.py:196-268, on the device and without host syncs.
//
// Token i carries C * S features (S = u^3 sub-voxels, channel-major:
// element c * S + s).  The step writes
//   sparse_feat  [N * S, C]      row i * S + s = token i's sub-voxel s,
//   cu_seqlens   [B + 1]         batch boundaries counted in sub-voxels,
//   seqlens      [B],
//   index_volume [B, Ru, Ru, Ru] -1, or the sequence-local row of the
//                                sub-voxel at (z*u+dz, y*u+dy, x*u+dx),
// with s = (dz * u + dy) * u + dx (the reference's meshgrid "ij" order).
//
// All of it is HBM-bound byte movement: the feature transpose reads and
// writes N*C*S elements once (a warp stages one token's C x S block in shared
// memory, padded against bank conflicts, and writes it back S x C, both
// sides coalesced); the index volume is a memset to -1 and one 4-byte
// scatter per sub-voxel.
#include <algorithm>
#include <cstdint>

#include "host_util.h"

namespace lsrm {

namespace {

constexpr int kTrWarps = 8;  // warps per CTA of the transpose, one token at a time each

int vo_grid(long long work, int threads) {
  return (int)std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, 1ll << 30));
}

// out[i][s][c] = in[i][c][s] for every token i (E: 2- or 4-byte elements).
template <typename E>
__global__ void __launch_bounds__(kTrWarps * 32) volume_transpose_kernel(const E* __restrict__ in, E* __restrict__ out,
                                                                        long long n_tok, int C, int S) {
  extern __shared__ uint32_t tr_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = C * S, stride = S + 1;  // staging row of a channel: S elements + 1 pad
  E* wb = reinterpret_cast<E*>(tr_smem) + (size_t)warp * C * stride;
  for (long long i = (long long)blockIdx.x * kTrWarps + warp; i < n_tok; i += (long long)gridDim.x * kTrWarps) {
    const E* src = in + i * per;
    E* dst = out + i * per;
    for (int k = lane; k < per; k += 32) {
      const int c = k / S, s = k - c * S;
      wb[c * stride + s] = src[k];
    }
    __syncwarp();
    for (int k = lane; k < per; k += 32) {
      const int s = k / C, c = k - s * C;
      dst[k] = wb[c * stride + s];
    }
    __syncwarp();
  }
}

// The same transpose for power-of-two C and S (the common C = 32, u = 2 or 4):
// 16-byte loads and stores, shift / mask indexing, kTpw tokens per warp
// iteration so that each lane keeps several loads in flight.  Requires
// C * S * sizeof(E) % 16 == 0, C % (16 / sizeof(E)) == 0 and 16-byte
// aligned rows.
constexpr int kTpw = 4;
template <typename E>
__global__ void __launch_bounds__(kTrWarps * 32) volume_transpose_vec_kernel(const uint4* __restrict__ in,
                                                                            uint4* __restrict__ out, long long n_tok,
                                                                            int lgC, int lgS) {
  extern __shared__ uint32_t tr_smem[];
  constexpr int V = 16 / (int)sizeof(E);  // elements per 16-byte chunk
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = 1 << lgC, S = 1 << lgS, stride = S + 1;
  const int chunks = (C << lgS) / V;  // per token
  E* wb = reinterpret_cast<E*>(tr_smem) + (size_t)warp * kTpw * C * stride;
  for (long long i0 = ((long long)blockIdx.x * kTrWarps + warp) * kTpw; i0 < n_tok;
       i0 += (long long)gridDim.x * kTrWarps * kTpw) {
    const int nt = n_tok - i0 < kTpw ? (int)(n_tok - i0) : kTpw;
    for (int q = lane; q < nt * chunks; q += 32) {
      const int t = q / chunks, r = q - t * chunks;
      const uint4 x = in[(i0 + t) * chunks + r];
      const E* e = reinterpret_cast<const E*>(&x);
      E* tb = wb + t * C * stride;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int k = r * V + j;
        tb[(k >> lgS) * stride + (k & (S - 1))] = e[j];
      }
    }
    __syncwarp();
    for (int q = lane; q < nt * chunks; q += 32) {
      const int t = q / chunks, r = q - t * chunks;
      const int k0 = r * V, sv = k0 >> lgC, c0 = k0 & (C - 1);
      const E* tb = wb + t * C * stride;
      uint4 x;
      E* e = reinterpret_cast<E*>(&x);
#pragma unroll
      for (int j = 0; j < V; ++j) e[j] = tb[(c0 + j) * stride + sv];
      out[(i0 + t) * chunks + r] = x;
    }
    __syncwarp();
  }
}

// cu[b] = first sub-voxel row of batch element b.  Tokens are grouped by
// batch id in ascending order; a batch id without tokens gets an empty range.
__global__ void volume_cu_kernel(const int32_t* __restrict__ vidx, long long n_tok, int B, int S, int32_t* cu,
                                 int* err) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i > n_tok) return;
  const int prev = i == 0 ? -1 : vidx[(i - 1) * 4];
  const int cur = i == n_tok ? B : vidx[i * 4];
  if (i < n_tok && (cur < 0 || cur >= B)) {
    atomicOr(err, LSRM_ERR_BAD_INDEX);
    return;
  }
  if (cur < prev) {  // not grouped by ascending batch id
    atomicOr(err, LSRM_ERR_BAD_INDEX);
    return;
  }
  for (int b = prev + 1; b <= cur; ++b) cu[b] = (int32_t)(i * S);
}

// index_volume[b, z, y, x] = row of the sub-voxel inside its sequence; the
// first B threads also write seqlens (cu is complete when this kernel runs).
__global__ void volume_scatter_kernel(const int32_t* __restrict__ vidx, long long n_sub, int u, int S, int B,
                                      int Ru, const int32_t* __restrict__ cu, int32_t* __restrict__ index_volume,
                                      int32_t* __restrict__ seqlens, int* err) {
  const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (j < B) seqlens[j] = cu[j + 1] - cu[j];
  if (j >= n_sub) return;
  const long long i = j / S;
  const int s = (int)(j - i * S);
  const int4 t = reinterpret_cast<const int4*>(vidx)[i];  // batch, z, y, x
  const int dz = s / (u * u), dy = (s / u) % u, dx = s % u;
  const int z = t.y * u + dz, y = t.z * u + dy, x = t.w * u + dx;
  if (t.x < 0 || t.x >= B || z < 0 || z >= Ru || y < 0 || y >= Ru || x < 0 || x >= Ru) {
    atomicOr(err, LSRM_ERR_BAD_INDEX);
    return;
  }
  index_volume[((long long)(t.x * (long long)Ru + z) * Ru + y) * Ru + x] = (int32_t)(j - cu[t.x]);
}

}  // namespace

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_prepare_volume_output(const void* volume, int32_t elem_bytes, const int32_t* volume_index,
                                          int64_t n_tokens, int32_t channels, int32_t upsample_scale,
                                          int32_t vol_res, int32_t batch_size, void* sparse_feat,
                                          int32_t* cu_seqlens, int32_t* seqlens, int32_t* index_volume,
                                          int* err_flags, void* stream) {
  LSRM_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "elem_bytes must be 2 or 4 (got %d)", elem_bytes);
  LSRM_CHECK_ARG(n_tokens >= 0 && channels > 0 && upsample_scale > 0 && vol_res > 0 && batch_size > 0,
                 "bad sizes");
  const long long S = (long long)upsample_scale * upsample_scale * upsample_scale;
  const long long Ru = (long long)vol_res * upsample_scale;
  LSRM_CHECK_ARG(n_tokens * S < (1ll << 31), "more than 2^31 sub-voxels");
  LSRM_CHECK_ARG(Ru < (1 << 20) && Ru * Ru * Ru * batch_size < (1ll << 40), "index volume too large");
  const size_t stage = (size_t)kTrWarps * channels * (S + 1) * elem_bytes;
  LSRM_CHECK_ARG(stage <= 200 * 1024, "channels x upsample_scale^3 too large for the staged transpose");
  LSRM_CHECK_ARG(((uintptr_t)volume_index & 15) == 0, "volume_index must be 16-byte aligned ([n, 4] int32)");
  LSRM_CHECK_ARG(err_flags != nullptr, "err_flags is required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("volume_output", s);
  const size_t vol_bytes = (size_t)batch_size * Ru * Ru * Ru * sizeof(int32_t);
  LSRM_CUDA_TRY(cudaMemsetAsync(index_volume, 0xff, vol_bytes, s));  // -1 everywhere
  volume_cu_kernel<<<vo_grid(n_tokens + 1, 256), 256, 0, s>>>(volume_index, n_tokens, batch_size, (int)S, cu_seqlens,
                                                              err_flags);
  LSRM_LAUNCH_CHECK();
  if (n_tokens == 0) {  // no sub-voxel: only the (empty) lengths
    volume_scatter_kernel<<<vo_grid(batch_size, 256), 256, 0, s>>>(volume_index, 0, upsample_scale, (int)S,
                                                                   batch_size, (int)Ru, cu_seqlens, index_volume,
                                                                   seqlens, err_flags);
    LSRM_LAUNCH_CHECK();
    return LSRM_OK;
  }
  const auto pow2 = [](long long x) { return x > 0 && (x & (x - 1)) == 0; };
  const int V = 16 / elem_bytes;
  if (pow2(channels) && pow2(S) && channels % V == 0 && ((uintptr_t)volume & 15) == 0 &&
      ((uintptr_t)sparse_feat & 15) == 0) {
    const int lgC = __builtin_ctz((unsigned)channels), lgS = __builtin_ctzll((unsigned long long)S);
    const size_t vstage = (size_t)kTrWarps * kTpw * channels * (S + 1) * elem_bytes;
    const int grid_v =
        (int)std::min<long long>((n_tokens + kTrWarps * kTpw - 1) / (kTrWarps * kTpw), (long long)num_sms() * 8);
    if (vstage <= 200 * 1024) {
      if (elem_bytes == 2) {
        if (vstage > 48 * 1024)
          LSRM_CUDA_TRY(cudaFuncSetAttribute(volume_transpose_vec_kernel<uint16_t>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vstage));
        volume_transpose_vec_kernel<uint16_t><<<grid_v, kTrWarps * 32, vstage, s>>>(
            static_cast<const uint4*>(volume), static_cast<uint4*>(sparse_feat), n_tokens, lgC, lgS);
      } else {
        if (vstage > 48 * 1024)
          LSRM_CUDA_TRY(cudaFuncSetAttribute(volume_transpose_vec_kernel<uint32_t>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vstage));
        volume_transpose_vec_kernel<uint32_t><<<grid_v, kTrWarps * 32, vstage, s>>>(
            static_cast<const uint4*>(volume), static_cast<uint4*>(sparse_feat), n_tokens, lgC, lgS);
      }
      LSRM_LAUNCH_CHECK();
      volume_scatter_kernel<<<vo_grid(std::max<long long>(n_tokens * S, batch_size), 256), 256, 0, s>>>(
          volume_index, n_tokens * S, upsample_scale, (int)S, batch_size, (int)Ru, cu_seqlens, index_volume, seqlens,
          err_flags);
      LSRM_LAUNCH_CHECK();
      return LSRM_OK;
    }
  }
  const int grid_tr = (int)std::min<long long>((n_tokens + kTrWarps - 1) / kTrWarps, (long long)num_sms() * 8);
  if (elem_bytes == 2) {
    if (stage > 48 * 1024)
      LSRM_CUDA_TRY(cudaFuncSetAttribute(volume_transpose_kernel<uint16_t>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stage));
    volume_transpose_kernel<uint16_t><<<grid_tr, kTrWarps * 32, stage, s>>>(
        static_cast<const uint16_t*>(volume), static_cast<uint16_t*>(sparse_feat), n_tokens, channels, (int)S);
  } else {
    if (stage > 48 * 1024)
      LSRM_CUDA_TRY(cudaFuncSetAttribute(volume_transpose_kernel<uint32_t>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stage));
    volume_transpose_kernel<uint32_t><<<grid_tr, kTrWarps * 32, stage, s>>>(
        static_cast<const uint32_t*>(volume), static_cast<uint32_t*>(sparse_feat), n_tokens, channels, (int)S);
  }
  LSRM_LAUNCH_CHECK();
  volume_scatter_kernel<<<vo_grid(std::max<long long>(n_tokens * S, batch_size), 256), 256, 0, s>>>(
      volume_index, n_tokens * S, upsample_scale, (int)S, batch_size, (int)Ru, cu_seqlens, index_volume, seqlens,
      err_flags);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
