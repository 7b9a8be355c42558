// HBM-bound kernels of the sparse-attention module: block-mean compression,
// the residual + LayerNorm + block-mean epilogue of SparseResBlock, and the
// sigmoid-gated merge of the attention branches.  16-byte vector accesses,
// fp32 math, one pass over the data.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_util.h"

namespace lsrm {

template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ void to_float(float* f) const {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (float)e[i];
  }
  __device__ __forceinline__ void from_float(const float* f) {
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = (T)f[i];
  }
};

// ----------------------------- block mean ----------------------------------
// grid: blocks; 256 threads = kMeanCg channel groups of 8 x (256 / kMeanCg)
// token slices (cg = tid % cgp, slice = tid / cgp, cgp a power of two >= the
// channel groups, at most 256).  Slice s sums tokens t0 + s, t0 + s + slices,
// ...; slice 0 then adds the slices' sums in slice order.
constexpr int kMeanThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kMeanThreads)
    block_mean_fwd_kernel(const int32_t* __restrict__ cu, const T* __restrict__ x, long long x_stride,
                          T* __restrict__ out, int C, int nb, int cgp) {
  __shared__ float part[kMeanThreads * 8];
  const int b = blockIdx.x;
  if (b >= nb) return;
  const int t0 = cu[b], t1 = cu[b + 1];
  const float inv = t1 > t0 ? 1.f / (float)(t1 - t0) : __int_as_float(0x7fc00000);
  const int cg = threadIdx.x % cgp, sl = threadIdx.x / cgp, slices = kMeanThreads / cgp;
  for (int cb = 0; cb < C; cb += cgp * 8) {
    const int c = cb + cg * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (c < C) {
      int t = t0 + sl;
      for (; t + 3 * slices < t1; t += 4 * slices) {
        Vec8<T> v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[u].raw = *reinterpret_cast<const uint4*>(x + (size_t)(t + u * slices) * x_stride + c);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[8];
          v[u].to_float(f);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += f[i];
        }
      }
      for (; t < t1; t += slices) {
        Vec8<T> v;
        v.raw = *reinterpret_cast<const uint4*>(x + (size_t)t * x_stride + c);
        float f[8];
        v.to_float(f);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += f[i];
      }
    }
    if (slices > 1) {
      __syncthreads();  // the previous channel round's partial sums are consumed
#pragma unroll
      for (int i = 0; i < 8; ++i) part[threadIdx.x * 8 + i] = acc[i];
      __syncthreads();
      if (sl == 0) {
        for (int s2 = 1; s2 < slices; ++s2)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += part[(s2 * cgp + cg) * 8 + i];
      }
    }
    if (sl == 0 && c < C) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= inv;
      Vec8<T> o;
      o.from_float(acc);
      *reinterpret_cast<uint4*>(out + (size_t)b * C + c) = o.raw;
    }
  }
}

template <typename T>
__global__ void block_mean_bwd_kernel(const int32_t* __restrict__ cu, const T* __restrict__ dout, T* __restrict__ dx,
                                      int C, int nb) {
  const int b = blockIdx.x;
  if (b >= nb) return;
  const int t0 = cu[b], t1 = cu[b + 1];
  if (t1 <= t0) return;
  const float inv = 1.f / (float)(t1 - t0);
  for (int c = threadIdx.x * 8; c < C; c += blockDim.x * 8) {
    Vec8<T> g;
    g.raw = *reinterpret_cast<const uint4*>(dout + (size_t)b * C + c);
    float f[8];
    g.to_float(f);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] *= inv;
    Vec8<T> o;
    o.from_float(f);
    for (int t = t0; t < t1; ++t) *reinterpret_cast<uint4*>(dx + (size_t)t * C + c) = o.raw;
  }
}

// --------------------- residual + LayerNorm + block mean --------------------
// One CTA per block; per token, the CTA reduces mean / variance over C.
constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// Each thread owns 8 channels (C <= 8 * kNormThreads = 2048).
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    resnorm_mean_fwd_kernel(const int32_t* __restrict__ cu, const T* __restrict__ x, const T* __restrict__ h, int C,
                            float eps, T* __restrict__ y, T* __restrict__ out, float* __restrict__ mean_out,
                            float* __restrict__ rstd_out, int nb) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  if (b >= nb) return;
  const int t0 = cu[b], t1 = cu[b + 1];
  const int c = threadIdx.x * 8;
  const bool active = c < C;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int t = t0; t < t1; ++t) {
    float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) {
      Vec8<T> a, bb;
      a.raw = *reinterpret_cast<const uint4*>(x + (size_t)t * C + c);
      bb.raw = *reinterpret_cast<const uint4*>(h + (size_t)t * C + c);
      float fa[8], fb[8];
      a.to_float(fa);
      bb.to_float(fb);
      // the reference adds in the input dtype, then LayerNorm32 upcasts
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = (float)(T)(fa[i] + fb[i]);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += r[i];
    const float mu = block_sum(s, red) / (float)C;
    float v = 0.f;
    if (active) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v += (r[i] - mu) * (r[i] - mu);
    }
    const float var = block_sum(v, red) / (float)C;
    const float rs = rsqrtf(var + eps);
    if (threadIdx.x == 0) {
      mean_out[t] = mu;
      rstd_out[t] = rs;
    }
    if (active) {
      float yn[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) yn[i] = (r[i] - mu) * rs;
      Vec8<T> o;
      o.from_float(yn);
      if (y) *reinterpret_cast<uint4*>(y + (size_t)t * C + c) = o.raw;
      // block mean of the LayerNorm output as the reference sees it (input dtype)
      float yr[8];
      o.to_float(yr);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += yr[i];
    }
  }
  if (active) {
    const float inv = t1 > t0 ? 1.f / (float)(t1 - t0) : __int_as_float(0x7fc00000);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
    Vec8<T> o;
    o.from_float(acc);
    *reinterpret_cast<uint4*>(out + (size_t)b * C + c) = o.raw;
  }
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    resnorm_mean_bwd_kernel(const int32_t* __restrict__ cu, const T* __restrict__ x, const T* __restrict__ h, int C,
                            const float* __restrict__ mean, const float* __restrict__ rstd, const T* __restrict__ dout,
                            T* __restrict__ dr, int nb) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  if (b >= nb) return;
  const int t0 = cu[b], t1 = cu[b + 1];
  if (t1 <= t0) return;
  const int c = threadIdx.x * 8;
  const bool active = c < C;
  float dy[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (active) {
    Vec8<T> g;
    g.raw = *reinterpret_cast<const uint4*>(dout + (size_t)b * C + c);
    g.to_float(dy);
    const float inv = 1.f / (float)(t1 - t0);
#pragma unroll
    for (int i = 0; i < 8; ++i) dy[i] *= inv;
  }
  for (int t = t0; t < t1; ++t) {
    const float mu = mean[t], rs = rstd[t];
    float yh[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) {
      Vec8<T> a, bb;
      a.raw = *reinterpret_cast<const uint4*>(x + (size_t)t * C + c);
      bb.raw = *reinterpret_cast<const uint4*>(h + (size_t)t * C + c);
      float fa[8], fb[8];
      a.to_float(fa);
      bb.to_float(fb);
#pragma unroll
      for (int i = 0; i < 8; ++i) yh[i] = ((float)(T)(fa[i] + fb[i]) - mu) * rs;
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s1 += dy[i];
      s2 += dy[i] * yh[i];
    }
    const float m1 = block_sum(s1, red) / (float)C;
    const float m2 = block_sum(s2, red) / (float)C;
    if (active) {
      float g[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] = rs * (dy[i] - m1 - yh[i] * m2);
      Vec8<T> o;
      o.from_float(g);
      *reinterpret_cast<uint4*>(dr + (size_t)t * C + c) = o.raw;
    }
  }
}

// ------------------------------ gated merge ---------------------------------
constexpr int kMaxBranch = 3;

struct GateArgs {
  const void* br[kMaxBranch];
  void* dbr[kMaxBranch];
};

__device__ __forceinline__ float sigmoidf_(float z) { return 1.f / (1.f + __expf(-z)); }

// Thread = 8 consecutive channels of one token.
template <typename T, bool PER_HEAD>
__global__ void gate_merge_fwd_kernel(long long n, int C, int nbr, int H, int D, const T* __restrict__ z, GateArgs a,
                                      T* __restrict__ out) {
  const int vecs = C / 8;
  const int zw = PER_HEAD ? nbr * H : nbr * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * vecs;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / vecs;
    const int c = (int)(i % vecs) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int b = 0; b < nbr; ++b) {
      Vec8<T> v;
      v.raw = *reinterpret_cast<const uint4*>(static_cast<const T*>(a.br[b]) + t * C + c);
      float f[8];
      v.to_float(f);
      if (PER_HEAD) {
        const float g = sigmoidf_((float)z[t * zw + b * H + c / D]);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += g * f[e];
      } else {
        Vec8<T> zz;
        zz.raw = *reinterpret_cast<const uint4*>(z + t * zw + b * C + c);
        float fz[8];
        zz.to_float(fz);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += sigmoidf_(fz[e]) * f[e];
      }
    }
    Vec8<T> o;
    o.from_float(acc);
    *reinterpret_cast<uint4*>(out + t * C + c) = o.raw;
  }
}

template <typename T, bool PER_HEAD>
__global__ void gate_merge_bwd_kernel(long long n, int C, int nbr, int H, int D, const T* __restrict__ z, GateArgs a,
                                      const T* __restrict__ dout, T* __restrict__ dz) {
  const int vecs = C / 8;
  const int zw = PER_HEAD ? nbr * H : nbr * C;
  const int lanes_per_head = D / 8;  // consecutive lanes share a head (D/8 <= 32)
  for (long long base = blockIdx.x * (long long)blockDim.x; base < n * vecs; base += (long long)gridDim.x * blockDim.x) {
    const long long i = base + threadIdx.x;
    const bool live = i < n * vecs;
    const long long t = live ? i / vecs : 0;
    const int c = live ? (int)(i % vecs) * 8 : 0;
    float go[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
      Vec8<T> g;
      g.raw = *reinterpret_cast<const uint4*>(dout + t * C + c);
      g.to_float(go);
    }
    for (int b = 0; b < nbr; ++b) {
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (live) {
        Vec8<T> v;
        v.raw = *reinterpret_cast<const uint4*>(static_cast<const T*>(a.br[b]) + t * C + c);
        v.to_float(f);
      }
      if (PER_HEAD) {
        const float g = live ? sigmoidf_((float)z[t * zw + b * H + c / D]) : 0.f;
        float part = 0.f;
        float db[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          db[e] = g * go[e];
          part += go[e] * f[e];
        }
        // reduce over the lanes of one head (aligned groups of D/8 lanes)
        for (int o = 1; o < lanes_per_head; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (live) {
          Vec8<T> o;
          o.from_float(db);
          *reinterpret_cast<uint4*>(static_cast<T*>(a.dbr[b]) + t * C + c) = o.raw;
          if ((c % D) == 0) dz[t * zw + b * H + c / D] = (T)(part * g * (1.f - g));
        }
      } else if (live) {
        Vec8<T> zz;
        zz.raw = *reinterpret_cast<const uint4*>(z + t * zw + b * C + c);
        float fz[8], db[8], dzz[8];
        zz.to_float(fz);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float g = sigmoidf_(fz[e]);
          db[e] = g * go[e];
          dzz[e] = go[e] * f[e] * g * (1.f - g);
        }
        Vec8<T> o1, o2;
        o1.from_float(db);
        o2.from_float(dzz);
        *reinterpret_cast<uint4*>(static_cast<T*>(a.dbr[b]) + t * C + c) = o1.raw;
        *reinterpret_cast<uint4*>(dz + t * zw + b * C + c) = o2.raw;
      }
    }
  }
}

static int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  return (int)std::min<long long>(std::max<long long>(g, 1), 148LL * 16);
}

}  // namespace lsrm

using namespace lsrm;

#define DISPATCH_T(dtype, ...)                     \
  do {                                             \
    if ((dtype) == LSRM_DTYPE_BF16) {              \
      using T = __nv_bfloat16;                     \
      __VA_ARGS__;                                 \
    } else {                                       \
      using T = __half;                            \
      __VA_ARGS__;                                 \
    }                                              \
  } while (0)

extern "C" int lsrm_block_mean_fwd(int32_t num_blocks, int32_t channels, int32_t dtype,
                                   const int32_t* cu_block_include_tokens, const void* x, int64_t x_stride, void* out,
                                   void* stream) {
  LSRM_CHECK_ARG(channels > 0 && channels % 8 == 0, "channels must be a positive multiple of 8");
  LSRM_CHECK_ARG(x_stride % 8 == 0, "x row stride must be a multiple of 8 elements");
  if (num_blocks <= 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int cgp = 1;  // channel groups of 8, rounded up to a power of two, at most the block's threads
  while (cgp < channels / 8 && cgp < kMeanThreads) cgp *= 2;
  ProfScope ps("block_mean_fwd", s);
  DISPATCH_T(dtype, (block_mean_fwd_kernel<T><<<num_blocks, kMeanThreads, 0, s>>>(
                        cu_block_include_tokens, static_cast<const T*>(x), x_stride, static_cast<T*>(out), channels,
                        num_blocks, cgp)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_block_mean_bwd(int32_t num_blocks, int32_t channels, int32_t dtype,
                                   const int32_t* cu_block_include_tokens, int32_t total_tokens, const void* dout,
                                   void* dx, void* stream) {
  LSRM_CHECK_ARG(channels > 0 && channels % 8 == 0, "channels must be a positive multiple of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (total_tokens > 0) LSRM_CUDA_TRY(cudaMemsetAsync(dx, 0, (size_t)total_tokens * channels * 2, s));
  if (num_blocks <= 0) return LSRM_OK;
  const int threads = std::min(256, std::max(32, (channels / 8 + 31) / 32 * 32));
  ProfScope ps("block_mean_bwd", s);
  DISPATCH_T(dtype, (block_mean_bwd_kernel<T><<<num_blocks, threads, 0, s>>>(
                        cu_block_include_tokens, static_cast<const T*>(dout), static_cast<T*>(dx), channels,
                        num_blocks)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_resnorm_mean_fwd(int32_t num_blocks, int32_t total_tokens, int32_t channels, int32_t dtype,
                                     const int32_t* cu_block_include_tokens, const void* x, const void* h, float eps,
                                     void* y, void* out, float* mean, float* rstd, void* stream) {
  LSRM_CHECK_ARG(channels > 0 && channels % 8 == 0 && channels <= 8 * kNormThreads,
                 "channels must be a multiple of 8 and <= %d", 8 * kNormThreads);
  (void)total_tokens;
  if (num_blocks <= 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = std::max(32, (channels / 8 + 31) / 32 * 32);
  ProfScope ps("resnorm_mean_fwd", s);
  DISPATCH_T(dtype, (resnorm_mean_fwd_kernel<T><<<num_blocks, threads, 0, s>>>(
                        cu_block_include_tokens, static_cast<const T*>(x), static_cast<const T*>(h), channels, eps,
                        static_cast<T*>(y), static_cast<T*>(out), mean, rstd, num_blocks)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_resnorm_mean_bwd(int32_t num_blocks, int32_t total_tokens, int32_t channels, int32_t dtype,
                                     const int32_t* cu_block_include_tokens, const void* x, const void* h,
                                     const float* mean, const float* rstd, const void* dout, void* dr, void* stream) {
  LSRM_CHECK_ARG(channels > 0 && channels % 8 == 0 && channels <= 8 * kNormThreads,
                 "channels must be a multiple of 8 and <= %d", 8 * kNormThreads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (total_tokens > 0) LSRM_CUDA_TRY(cudaMemsetAsync(dr, 0, (size_t)total_tokens * channels * 2, s));
  if (num_blocks <= 0) return LSRM_OK;
  const int threads = std::max(32, (channels / 8 + 31) / 32 * 32);
  ProfScope ps("resnorm_mean_bwd", s);
  DISPATCH_T(dtype, (resnorm_mean_bwd_kernel<T><<<num_blocks, threads, 0, s>>>(
                        cu_block_include_tokens, static_cast<const T*>(x), static_cast<const T*>(h), channels, mean,
                        rstd, static_cast<const T*>(dout), static_cast<T*>(dr), num_blocks)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_gate_merge_fwd(int32_t total_tokens, int32_t channels, int32_t n_branch, int32_t per_head,
                                   int32_t head_dim, int32_t dtype, const void* z, const void* const* branches,
                                   void* out, void* stream) {
  LSRM_CHECK_ARG(n_branch >= 1 && n_branch <= kMaxBranch, "n_branch must be 1..%d", kMaxBranch);
  LSRM_CHECK_ARG(channels % 8 == 0, "channels must be a multiple of 8");
  LSRM_CHECK_ARG(!per_head || (head_dim % 8 == 0 && channels % head_dim == 0), "bad head_dim for per-head gates");
  if (total_tokens <= 0) return LSRM_OK;
  GateArgs a{};
  for (int i = 0; i < n_branch; ++i) a.br[i] = branches[i];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long work = (long long)total_tokens * (channels / 8);
  const int H = per_head ? channels / head_dim : 0;
  ProfScope ps("gate_merge_fwd", s);
  DISPATCH_T(dtype, if (per_head) gate_merge_fwd_kernel<T, true><<<grid_for(work, 256), 256, 0, s>>>(
                        total_tokens, channels, n_branch, H, head_dim, static_cast<const T*>(z), a,
                        static_cast<T*>(out));
             else gate_merge_fwd_kernel<T, false><<<grid_for(work, 256), 256, 0, s>>>(
                 total_tokens, channels, n_branch, H, head_dim, static_cast<const T*>(z), a, static_cast<T*>(out)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_gate_merge_bwd(int32_t total_tokens, int32_t channels, int32_t n_branch, int32_t per_head,
                                   int32_t head_dim, int32_t dtype, const void* z, const void* const* branches,
                                   const void* dout, void* dz, void* const* dbranches, void* stream) {
  LSRM_CHECK_ARG(n_branch >= 1 && n_branch <= kMaxBranch, "n_branch must be 1..%d", kMaxBranch);
  LSRM_CHECK_ARG(channels % 8 == 0, "channels must be a multiple of 8");
  LSRM_CHECK_ARG(!per_head || (head_dim % 8 == 0 && channels % head_dim == 0 && head_dim / 8 <= 32 &&
                               ((head_dim / 8) & (head_dim / 8 - 1)) == 0),
                 "bad head_dim for per-head gates");
  if (total_tokens <= 0) return LSRM_OK;
  GateArgs a{};
  for (int i = 0; i < n_branch; ++i) {
    a.br[i] = branches[i];
    a.dbr[i] = dbranches[i];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long work = (long long)total_tokens * (channels / 8);
  const int H = per_head ? channels / head_dim : 0;
  ProfScope ps("gate_merge_bwd", s);
  DISPATCH_T(dtype, if (per_head) gate_merge_bwd_kernel<T, true><<<grid_for(work, 256), 256, 0, s>>>(
                        total_tokens, channels, n_branch, H, head_dim, static_cast<const T*>(z), a,
                        static_cast<const T*>(dout), static_cast<T*>(dz));
             else gate_merge_bwd_kernel<T, false><<<grid_for(work, 256), 256, 0, s>>>(
                 total_tokens, channels, n_branch, H, head_dim, static_cast<const T*>(z), a,
                 static_cast<const T*>(dout), static_cast<T*>(dz)));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
