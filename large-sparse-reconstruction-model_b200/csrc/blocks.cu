// Block metadata of a sparse voxel (or image-patch) sequence, on the device.
//
// sort keys: the order in which voxels are laid out so that every block is a
//   contiguous run of tokens (batch, block cell, position inside the cell).
// block separation: per batch element, the token count of every non-empty
//   block cell in cell order -> cu_seqlens, cu_seqblocks,
//   cu_block_include_tokens.  Counting is order independent (a histogram),
//   as in the reference; coordinates whose cell lies outside the grid are not
//   counted.
//
// Both are integer, HBM-bound passes: one read of the coordinates, atomic
// histogram updates in L2, and scans over the (batch x cells) histogram.
#include <algorithm>

#include "host_util.h"

namespace lsrm {

namespace {

constexpr int kScanThreads = 1024;
constexpr int kScanPerThread = 4;
constexpr int kScanTile = kScanThreads * kScanPerThread;  // histogram bins per CTA

struct SepParams {
  const int32_t* coords;  // [n, dim + 1]: batch, then dim coordinates
  long long n;
  int dim;
  int batch;
  int block_size[3];
  long long mult[3];      // flattening multipliers of the cell coordinates
  long long cells;        // cells per batch element
  int32_t* hist;          // [batch * cells] token counts
  int32_t* seq_count;     // [batch] tokens per batch element
  int* err;
};

__global__ void volume_keys_kernel(const int32_t* __restrict__ coords, long long n, int res, int bs,
                                   int64_t* __restrict__ keys) {
  const long long r3 = (long long)res * res * res, r2b = (long long)res * res * bs, rb2 = (long long)res * bs * bs;
  const long long b3 = (long long)bs * bs * bs, b2 = (long long)bs * bs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int4 c = reinterpret_cast<const int4*>(coords)[i];
    keys[i] = r3 * c.x + r2b * (c.y / bs) + rb2 * (c.z / bs) + b3 * (c.w / bs) + b2 * (c.y % bs) +
              (long long)bs * (c.z % bs) + (c.w % bs);
  }
}

// sort_image_blocks (misc/sparse_utils.py:95-124): image tokens (batch, view,
// patch row, patch column) by batch, view, block row, block column, then row
// and column inside the block, with the reference's offsets.
__global__ void image_keys_kernel(const int32_t* __restrict__ coords, long long n, int views, int pr, int bs,
                                  int64_t* __restrict__ keys) {
  const long long o1 = (long long)views * pr * pr, o2 = (long long)pr * pr, o3 = (long long)pr * bs,
                  o4 = (long long)bs * bs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int4 c = reinterpret_cast<const int4*>(coords)[i];
    keys[i] = o1 * c.x + o2 * c.y + o3 * (c.z / bs) + o4 * (c.w / bs) + (long long)bs * (c.z % bs) + (c.w % bs);
  }
}

__global__ void block_hist_kernel(SepParams p) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n; i += (long long)gridDim.x * blockDim.x) {
    const int32_t* c = p.coords + i * (p.dim + 1);
    const int b = c[0];
    if (b < 0 || b >= p.batch) {
      atomicOr(p.err, LSRM_ERR_BAD_INDEX);
      continue;
    }
    atomicAdd(&p.seq_count[b], 1);
    // flattened cell id with floor division; like a histogram over
    // [0, cells), ids outside that range are not counted
    long long cell = 0;
    for (int d = 0; d < p.dim; ++d) {
      const int v = c[1 + d], bs = p.block_size[d];
      const int q = v >= 0 ? v / bs : -((-v + bs - 1) / bs);
      cell += p.mult[d] * q;
    }
    if (cell >= 0 && cell < p.cells) atomicAdd(&p.hist[(long long)b * p.cells + cell], 1);
  }
}

// Per CTA tile of bins: number of non-empty bins and tokens.
__global__ void __launch_bounds__(kScanThreads) hist_tile_sums_kernel(const int32_t* __restrict__ hist, long long bins,
                                                                      int2* __restrict__ tile_sums) {
  __shared__ int2 red[kScanThreads / 32];
  const long long base = (long long)blockIdx.x * kScanTile + threadIdx.x * kScanPerThread;
  int nz = 0, tok = 0;
#pragma unroll
  for (int k = 0; k < kScanPerThread; ++k) {
    const long long i = base + k;
    const int v = i < bins ? hist[i] : 0;
    nz += v > 0;
    tok += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nz += __shfl_xor_sync(0xffffffffu, nz, o);
    tok += __shfl_xor_sync(0xffffffffu, tok, o);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_int2(nz, tok);
  __syncthreads();
  if (threadIdx.x < 32) {
    int2 v = threadIdx.x < kScanThreads / 32 ? red[threadIdx.x] : make_int2(0, 0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = v;
  }
}

// Exclusive scan of the tile sums (one CTA) and of the per-batch token
// counts -> cu_seqlens.
__global__ void __launch_bounds__(kScanThreads) tile_scan_kernel(int2* tile_sums, int n_tiles, const int32_t* seq_count,
                                                                 int batch, int32_t* cu_seqlens) {
  __shared__ int2 carry_s;
  if (threadIdx.x == 0) carry_s = make_int2(0, 0);
  __syncthreads();
  for (int b0 = 0; b0 < n_tiles; b0 += kScanThreads) {
    const int i = b0 + threadIdx.x;
    int2 v = i < n_tiles ? tile_sums[i] : make_int2(0, 0);
    int2 incl = v;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl.x, o), y = __shfl_up_sync(0xffffffffu, incl.y, o);
      if (lane >= o) {
        incl.x += x;
        incl.y += y;
      }
    }
    __shared__ int2 wsum[kScanThreads / 32];
    if (lane == 31) wsum[w] = incl;
    __syncthreads();
    if (w == 0) {
      int2 s = wsum[lane];
      int2 si = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, si.x, o), y = __shfl_up_sync(0xffffffffu, si.y, o);
        if (lane >= o) {
          si.x += x;
          si.y += y;
        }
      }
      wsum[lane] = make_int2(si.x - s.x, si.y - s.y);  // exclusive warp offsets
    }
    __syncthreads();
    const int2 c = carry_s;
    if (i < n_tiles) tile_sums[i] = make_int2(c.x + wsum[w].x + incl.x - v.x, c.y + wsum[w].y + incl.y - v.y);
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) carry_s = make_int2(c.x + wsum[w].x + incl.x, c.y + wsum[w].y + incl.y);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < batch; ++b) {
      cu_seqlens[b] = acc;
      acc += seq_count[b];
    }
    cu_seqlens[batch] = acc;
  }
}

// Writes the offsets of every non-empty bin, cu_seqblocks and the totals.
__global__ void __launch_bounds__(kScanThreads) hist_emit_kernel(const int32_t* __restrict__ hist, long long bins,
                                                                 long long cells, int batch,
                                                                 const int2* __restrict__ tile_off, int n_tiles,
                                                                 int32_t* __restrict__ cu_blk,
                                                                 int32_t* __restrict__ cu_seqblocks,
                                                                 int32_t* __restrict__ num_blocks) {
  __shared__ int2 wsum[kScanThreads / 32];
  const long long base = (long long)blockIdx.x * kScanTile + threadIdx.x * kScanPerThread;
  int v[kScanPerThread];
  int nz = 0, tok = 0;
#pragma unroll
  for (int k = 0; k < kScanPerThread; ++k) {
    const long long i = base + k;
    v[k] = i < bins ? hist[i] : 0;
    nz += v[k] > 0;
    tok += v[k];
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int nzi = nz, toki = tok;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, nzi, o), y = __shfl_up_sync(0xffffffffu, toki, o);
    if (lane >= o) {
      nzi += x;
      toki += y;
    }
  }
  if (lane == 31) wsum[w] = make_int2(nzi, toki);
  __syncthreads();
  if (w == 0) {
    const int2 s = wsum[lane];
    int2 si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, si.x, o), y = __shfl_up_sync(0xffffffffu, si.y, o);
      if (lane >= o) {
        si.x += x;
        si.y += y;
      }
    }
    wsum[lane] = make_int2(si.x - s.x, si.y - s.y);
  }
  __syncthreads();
  int rank = tile_off[blockIdx.x].x + wsum[w].x + nzi - nz;   // non-empty bins before this thread's first
  int tokp = tile_off[blockIdx.x].y + wsum[w].y + toki - tok;  // tokens before it
#pragma unroll
  for (int k = 0; k < kScanPerThread; ++k) {
    const long long i = base + k;
    if (i >= bins) break;
    if (i % cells == 0) cu_seqblocks[i / cells] = rank;
    if (v[k] > 0) {
      cu_blk[rank] = tokp;
      ++rank;
      tokp += v[k];
    }
  }
  if (blockIdx.x == n_tiles - 1 && threadIdx.x == kScanThreads - 1) {
    const int2 last = tile_off[n_tiles - 1];
    // totals: this tile's exclusive offset plus its own sums (the last thread's inclusive values)
    const int total_nz = last.x + wsum[w].x + nzi, total_tok = last.y + wsum[w].y + toki;
    cu_blk[total_nz] = total_tok;
    cu_seqblocks[batch] = total_nz;
    *num_blocks = total_nz;
  }
}

int grid_of(long long work, int threads) {
  return (int)std::min<long long>(std::max<long long>((work + threads - 1) / threads, 1), 148LL * 8);
}

}  // namespace

size_t separation_workspace(int dim, const int* block_size, const int* resolution, int batch, long long* cells_out) {
  long long cells = 1;
  for (int d = 0; d < dim; ++d) cells *= resolution[d] / std::max(block_size[d], 1);
  if (cells_out) *cells_out = cells;
  const long long bins = cells * batch;
  const long long tiles = (bins + kScanTile - 1) / kScanTile;
  return (size_t)bins * 4 + (size_t)batch * 4 + (size_t)tiles * 8 + 256;
}

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_volume_sort_keys(int64_t n_tokens, const int32_t* coords, int32_t volume_res, int32_t block_size,
                                     int64_t* keys, void* stream) {
  LSRM_CHECK_ARG(n_tokens >= 0 && volume_res > 0 && block_size > 0, "bad sizes");
  LSRM_CHECK_ARG(volume_res % block_size == 0, "volume_res must be a multiple of block_size");
  LSRM_CHECK_ARG(((uintptr_t)coords & 15) == 0, "coords must be 16-byte aligned ([n, 4] int32)");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps("volume_keys", s);
  volume_keys_kernel<<<grid_of(n_tokens, 256), 256, 0, s>>>(coords, n_tokens, volume_res, block_size, keys);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" int lsrm_image_sort_keys(int64_t n_tokens, const int32_t* coords, int32_t views, int32_t patch_res,
                                    int32_t block_size, int64_t* keys, void* stream) {
  LSRM_CHECK_ARG(n_tokens >= 0 && views > 0 && patch_res > 0 && block_size > 0, "bad sizes");
  LSRM_CHECK_ARG(((uintptr_t)coords & 15) == 0, "coords must be 16-byte aligned ([n, 4] int32)");
  if (n_tokens == 0) return LSRM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  image_keys_kernel<<<grid_of(n_tokens, 256), 256, 0, s>>>(coords, n_tokens, views, patch_res, block_size, keys);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

extern "C" size_t lsrm_block_separation_workspace_bytes(int32_t dim, const int32_t* block_size,
                                                        const int32_t* resolution, int32_t batch) {
  if (dim < 1 || dim > 3 || batch < 1 || !block_size || !resolution) return 0;
  return separation_workspace(dim, block_size, resolution, batch, nullptr);
}

extern "C" int lsrm_block_separation(int64_t n_tokens, const int32_t* coords, int32_t dim, const int32_t* block_size,
                                     const int32_t* resolution, int32_t batch, int32_t* cu_seqlens,
                                     int32_t* cu_seqblocks, int32_t* cu_block_include_tokens, int32_t* num_blocks,
                                     void* workspace, size_t workspace_bytes, int* err_flags, void* stream) {
  LSRM_CHECK_ARG(dim >= 1 && dim <= 3, "dim must be 1, 2 or 3 (got %d)", dim);
  LSRM_CHECK_ARG(batch >= 1 && n_tokens >= 0 && n_tokens < (1ll << 31), "bad sizes");
  LSRM_CHECK_ARG(block_size && resolution, "null block_size / resolution");
  for (int d = 0; d < dim; ++d)
    LSRM_CHECK_ARG(block_size[d] > 0 && resolution[d] >= block_size[d],
                   "block_size must be positive and resolution at least one block (dim %d)", d);
  long long cells = 0;
  const size_t need = separation_workspace(dim, block_size, resolution, batch, &cells);
  if (!workspace || workspace_bytes < need) {
    set_error("workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    return LSRM_ERR_WORKSPACE;
  }
  const long long bins = cells * batch;
  LSRM_CHECK_ARG(bins < (1ll << 31), "too many block cells");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SepParams p{};
  p.coords = coords;
  p.n = n_tokens;
  p.dim = dim;
  p.batch = batch;
  p.cells = cells;
  long long m = 1;
  for (int d = dim - 1; d >= 0; --d) {  // first coordinate most significant
    p.block_size[d] = block_size[d];
    p.mult[d] = m;
    m *= resolution[d] / block_size[d];
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.hist = reinterpret_cast<int32_t*>(ws);
  p.seq_count = reinterpret_cast<int32_t*>(ws + (size_t)bins * 4);
  const int n_tiles = (int)((bins + kScanTile - 1) / kScanTile);
  int2* tile = reinterpret_cast<int2*>(ws + (((size_t)bins * 4 + (size_t)batch * 4 + 7) / 8) * 8);
  int* err = err_flags;
  if (!err) {
    set_error("err_flags is required (metadata is validated on the device)");
    return LSRM_ERR_INVALID_ARG;
  }
  p.err = err;
  ProfScope ps("block_separation", s);
  LSRM_CUDA_TRY(cudaMemsetAsync(ws, 0, (size_t)bins * 4 + (size_t)batch * 4, s));
  if (n_tokens > 0) {
    block_hist_kernel<<<grid_of(n_tokens, 256), 256, 0, s>>>(p);
    LSRM_LAUNCH_CHECK();
  }
  hist_tile_sums_kernel<<<n_tiles, kScanThreads, 0, s>>>(p.hist, bins, tile);
  LSRM_LAUNCH_CHECK();
  tile_scan_kernel<<<1, kScanThreads, 0, s>>>(tile, n_tiles, p.seq_count, batch, cu_seqlens);
  LSRM_LAUNCH_CHECK();
  hist_emit_kernel<<<n_tiles, kScanThreads, 0, s>>>(p.hist, bins, cells, batch, tile, n_tiles, cu_block_include_tokens,
                                                    cu_seqblocks, num_blocks);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
