// Per-head LayerNorm fused with the Ulysses head-slice pack.
//
// The reference's CrossAttention normalises q, k and the compressed keys per
// head with a non-affine LayerNorm evaluated in fp32 (LayerNorm32 over
// head_dim, eps 1e-5, models_sparse/utils.py:21-23, 133-134, 239-270), then
// moves them to other ranks; here one pass reads x [n, H, D] and writes the
// normalised rows straight into the rank-major layout [W, n, H/W, D] that the
// all-to-all sends (W = 1: the plain per-head LayerNorm, same layout as x).
// The backward reads x again (mean and 1/std are recomputed, nothing is
// saved) and the packed gradient, and writes dx [n, H, D]:
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)).
// A group of D/8 lanes owns one (token, head) row (16-byte accesses); rows
// are independent, so this is one HBM-bound pass each way.
#include <algorithm>
#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_util.h"

namespace lsrm {

namespace {

int hn_grid(long long work, int threads) {
  return (int)std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, (long long)num_sms() * 16));
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = (float)e[i];
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = (T)f[i];
  return u;
}

// sum over the GL lanes of a row group (GL a power of two <= 32)
template <int GL>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = GL / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int D>
__global__ void head_ln_pack_kernel(const uint4* __restrict__ src, long long src_stride_vec, uint4* __restrict__ dst,
                                    long long n, int H, int hp, float eps) {
  constexpr int GL = D / 8, RPW = 32 / GL;  // lanes per row (8 elements each), rows per warp step
  const long long rows = n * H;
  const int lane = threadIdx.x & 31, l = lane % GL;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long warps = (long long)gridDim.x * blockDim.x >> 5;
  // warp-uniform trip count: the group shuffles below need the whole warp
  for (long long base = warp * RPW; base < rows; base += warps * RPW) {
    const long long row = base + lane / GL;
    const bool live = row < rows;
    const long long t = live ? row / H : 0;
    const int h = live ? (int)(row - t * H) : 0;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) unpack8<T>(src[t * src_stride_vec + (long long)h * GL + l], v);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
    const float mean = group_sum<GL>(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] -= mean;
      q = fmaf(v[i], v[i], q);
    }
    const float rstd = 1.f / sqrtf(group_sum<GL>(q) / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= rstd;
    if (live) {
      const int r = h / hp, hh = h - r * hp;
      dst[((r * n + t) * hp + hh) * GL + l] = pack8<T>(v);
    }
  }
}

template <typename T, int D>
__global__ void head_ln_pack_bwd_kernel(const uint4* __restrict__ src, long long src_stride_vec,
                                        const uint4* __restrict__ gpk, uint4* __restrict__ dx, long long n, int H,
                                        int hp, float eps) {
  constexpr int GL = D / 8, RPW = 32 / GL;
  const long long rows = n * H;
  const int lane = threadIdx.x & 31, l = lane % GL;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long warps = (long long)gridDim.x * blockDim.x >> 5;
  for (long long base = warp * RPW; base < rows; base += warps * RPW) {
    const long long row = base + lane / GL;
    const bool live = row < rows;
    const long long t = live ? row / H : 0;
    const int h = live ? (int)(row - t * H) : 0;
    const int r = h / hp, hh = h - r * hp;
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
      unpack8<T>(src[t * src_stride_vec + (long long)h * GL + l], x);
      unpack8<T>(gpk[((r * n + t) * hp + hh) * GL + l], g);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += x[i];
    const float mean = group_sum<GL>(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] -= mean;
      q = fmaf(x[i], x[i], q);
    }
    const float rstd = 1.f / sqrtf(group_sum<GL>(q) / (float)D + eps);
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] *= rstd;  // xhat
      sg += g[i];
      sgx = fmaf(g[i], x[i], sgx);
    }
    const float mg = group_sum<GL>(sg) / (float)D, mgx = group_sum<GL>(sgx) / (float)D;
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = rstd * (g[i] - mg - x[i] * mgx);
    if (live) dx[(t * H + h) * GL + l] = pack8<T>(g);
  }
}

template <typename T>
int launch_ln(bool bwd, int D, const void* src, long long stride_vec, const void* gpk, void* dst, long long n, int H,
              int hp, float eps, cudaStream_t s) {
  const long long threads = n * H * (D / 8);  // one lane per 16 bytes of a row
  const int grid = hn_grid(threads, 256);
#define LN_CASE(DD)                                                                                             \
  if (D == DD) {                                                                                                \
    if (bwd)                                                                                                    \
      head_ln_pack_bwd_kernel<T, DD><<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), stride_vec,           \
                                                          static_cast<const uint4*>(gpk), static_cast<uint4*>(dst), \
                                                          n, H, hp, eps);                                       \
    else                                                                                                        \
      head_ln_pack_kernel<T, DD><<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), stride_vec,               \
                                                      static_cast<uint4*>(dst), n, H, hp, eps);                 \
    LSRM_LAUNCH_CHECK();                                                                                        \
    return LSRM_OK;                                                                                             \
  }
  LN_CASE(16) LN_CASE(32) LN_CASE(64) LN_CASE(128) LN_CASE(256)
#undef LN_CASE
  return LSRM_ERR_UNSUPPORTED;
}

int check_ln_args(int32_t n, int32_t H, int32_t D, int32_t W, int32_t dtype, int64_t stride, const void* src) {
  LSRM_CHECK_ARG(n >= 0 && H >= 1 && W >= 1, "bad sizes");
  LSRM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128 || D == 256, "head_dim must be 16..256, a power of two");
  LSRM_CHECK_ARG(H % W == 0, "num_heads (%d) must be a multiple of world (%d)", H, W);
  LSRM_CHECK_ARG(dtype == LSRM_DTYPE_BF16 || dtype == LSRM_DTYPE_F16, "dtype must be bf16 or fp16");
  LSRM_CHECK_ARG(stride >= (int64_t)H * D && stride % 8 == 0, "src token stride must be >= H*D and a multiple of 8");
  LSRM_CHECK_ARG(((uintptr_t)src & 15) == 0, "src must be 16-byte aligned");
  return LSRM_OK;
}

}  // namespace

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_head_layernorm_pack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world,
                                        int32_t dtype, int64_t src_token_stride, float eps, const void* src, void* dst,
                                        void* stream) {
  int rc = check_ln_args(n_tokens, num_heads, head_dim, world, dtype, src_token_stride, src);
  if (rc) return rc;
  LSRM_CHECK_ARG(((uintptr_t)dst & 15) == 0, "dst must be 16-byte aligned");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("head_layernorm_pack", s);
  const int hp = num_heads / world;
  return dtype == LSRM_DTYPE_BF16
             ? launch_ln<__nv_bfloat16>(false, head_dim, src, src_token_stride / 8, nullptr, dst, n_tokens,
                                        num_heads, hp, eps, s)
             : launch_ln<__half>(false, head_dim, src, src_token_stride / 8, nullptr, dst, n_tokens, num_heads, hp, eps,
                                 s);
}

extern "C" int lsrm_head_layernorm_pack_bwd(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world,
                                            int32_t dtype, int64_t src_token_stride, float eps, const void* src,
                                            const void* grad_packed, void* grad_src, void* stream) {
  int rc = check_ln_args(n_tokens, num_heads, head_dim, world, dtype, src_token_stride, src);
  if (rc) return rc;
  LSRM_CHECK_ARG(((uintptr_t)grad_packed & 15) == 0 && ((uintptr_t)grad_src & 15) == 0,
                 "gradients must be 16-byte aligned");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("head_layernorm_pack_bwd", s);
  const int hp = num_heads / world;
  return dtype == LSRM_DTYPE_BF16
             ? launch_ln<__nv_bfloat16>(true, head_dim, src, src_token_stride / 8, grad_packed, grad_src, n_tokens,
                                        num_heads, hp, eps, s)
             : launch_ln<__half>(true, head_dim, src, src_token_stride / 8, grad_packed, grad_src, n_tokens, num_heads,
                                 hp, eps, s);
}
