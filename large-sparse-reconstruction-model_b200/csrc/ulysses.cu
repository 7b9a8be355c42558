// Ulysses sequence <-> head exchange layouts.
//
// A rank holding n tokens of the sequence and all H heads sends, to each of
// the W ranks of the group, the head slice that rank computes.  pack writes
// those slices contiguously, rank-major, so that one all_to_all_single moves
// them; after the exchange the received buffer is already token-major
// ([sum of the ranks' tokens, heads per rank, D], because every rank's tokens
// are one contiguous, Morton-ordered run of whole blocks).  unpack is the
// inverse for the return trip (and the backward of pack): it also sums the
// copies of a head that was replicated to several ranks (grouped-query heads
// when H < W), in rank order, in fp32, so the result is deterministic.
//
// Both are HBM-bound copies: 16-byte vectors, one read and one write of every
// byte (unpack with replication reads each replica once).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "host_util.h"

namespace lsrm {

namespace {

struct Layout {
  long long n;        // tokens on this side
  int chunk_vec;      // 16-byte vectors in one (token, rank) slice: hp * D * elem / 16
  int world;          // ranks
  int rep;            // ranks sharing one head slice (1 unless H < world)
  long long tok_vec;  // 16-byte vectors between consecutive tokens of the token-major side
};

// dst[p][t][:] = src[t][(p / rep) * chunk : ...]
__global__ void ulysses_pack_kernel(Layout L, const uint4* __restrict__ src, uint4* __restrict__ dst) {
  const long long per_rank = L.n * L.chunk_vec;
  const long long total = per_rank * L.world;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(i / per_rank);
    const long long r = i - (long long)p * per_rank;
    const long long t = r / L.chunk_vec;
    const int c = (int)(r - t * L.chunk_vec);
    dst[i] = src[t * L.tok_vec + (long long)(p / L.rep) * L.chunk_vec + c];
  }
}

// dst[t][g * chunk : ...] = sum_{j < rep} src[g * rep + j][t][:]   (rep == 1: a copy)
template <typename T>
__global__ void ulysses_unpack_kernel(Layout L, const uint4* __restrict__ src, uint4* __restrict__ dst) {
  const int groups = L.world / L.rep;
  const long long per_tok = (long long)groups * L.chunk_vec;
  const long long total = L.n * per_tok;
  const long long per_rank = L.n * L.chunk_vec;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / per_tok;
    const int r = (int)(i - t * per_tok);
    const int g = r / L.chunk_vec;
    const int c = r - g * L.chunk_vec;
    const long long s0 = (long long)(g * L.rep) * per_rank + t * L.chunk_vec + c;
    uint4 out;
    if (L.rep == 1) {
      out = src[s0];
    } else {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int j = 0; j < L.rep; ++j) {
        const uint4 v = src[s0 + (long long)j * per_rank];
        const T* x = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += (float)x[e];
      }
      T* o = reinterpret_cast<T*>(&out);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (T)acc[e];
    }
    dst[t * L.tok_vec + r] = out;
  }
}

int make_layout(Layout& L, long long n, int heads, int head_dim, int world, int dtype, long long token_stride) {
  LSRM_CHECK_ARG(n >= 0 && heads >= 1 && world >= 1, "bad sizes");
  LSRM_CHECK_ARG(dtype == LSRM_DTYPE_BF16 || dtype == LSRM_DTYPE_F16, "dtype must be bf16 or fp16");
  LSRM_CHECK_ARG(heads % world == 0 || world % heads == 0,
                 "heads (%d) and world size (%d) must divide one another", heads, world);
  const int hp = heads >= world ? heads / world : 1;
  LSRM_CHECK_ARG((hp * head_dim * 2) % 16 == 0, "a rank's head slice must be a multiple of 16 bytes");
  LSRM_CHECK_ARG(token_stride >= (long long)heads * head_dim && (token_stride * 2) % 16 == 0,
                 "token stride must cover the heads and be a multiple of 16 bytes");
  L.n = n;
  L.chunk_vec = hp * head_dim * 2 / 16;
  L.world = world;
  L.rep = heads >= world ? 1 : world / heads;
  L.tok_vec = token_stride * 2 / 16;
  return LSRM_OK;
}

int grid_of(long long work) {
  const long long g = (work + 255) / 256;
  return (int)std::min<long long>(std::max<long long>(g, 1), 148LL * 8);
}

}  // namespace
}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_ulysses_pack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world, int32_t dtype,
                                 int64_t src_token_stride, const void* src, void* dst, void* stream) {
  Layout L{};
  int rc;
  if ((rc = make_layout(L, n_tokens, num_heads, head_dim, world, dtype, src_token_stride))) return rc;
  LSRM_CHECK_ARG(((uintptr_t)src | (uintptr_t)dst) % 16 == 0, "src/dst must be 16-byte aligned");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("ulysses_pack", s);
  ulysses_pack_kernel<<<grid_of(L.n * L.chunk_vec * world), 256, 0, s>>>(L, static_cast<const uint4*>(src),
                                                                          static_cast<uint4*>(dst));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_ulysses_unpack(int32_t n_tokens, int32_t num_heads, int32_t head_dim, int32_t world,
                                   int32_t dtype, const void* src, int64_t dst_token_stride, void* dst,
                                   void* stream) {
  Layout L{};
  int rc;
  if ((rc = make_layout(L, n_tokens, num_heads, head_dim, world, dtype, dst_token_stride))) return rc;
  LSRM_CHECK_ARG(((uintptr_t)src | (uintptr_t)dst) % 16 == 0, "src/dst must be 16-byte aligned");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long work = L.n * (world / L.rep) * L.chunk_vec;
  ProfScope ps("ulysses_unpack", s);
  if (dtype == LSRM_DTYPE_BF16)
    ulysses_unpack_kernel<__nv_bfloat16><<<grid_of(work), 256, 0, s>>>(L, static_cast<const uint4*>(src),
                                                                       static_cast<uint4*>(dst));
  else
    ulysses_unpack_kernel<__half><<<grid_of(work), 256, 0, s>>>(L, static_cast<const uint4*>(src),
                                                                static_cast<uint4*>(dst));
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
