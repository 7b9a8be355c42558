// Plan-building kernels: tile lists, per-tile selection unions, reverse map.
// All integer work; deterministic outputs (the reverse map is sorted).
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"
#include "plan.cuh"

namespace lsrm {

// ---------------------------------------------------------------------------
// Block-wide exclusive scan (blockDim.x a multiple of 32, <= 1024).
// ---------------------------------------------------------------------------
__device__ int block_exclusive_scan(int v, int* total, int* scratch /* >= 33 ints */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? scratch[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) scratch[lane] = w;  // inclusive warp totals
    if (lane == nw - 1) scratch[32] = w;
  }
  __syncthreads();
  const int base = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[32];
  const int res = base + x - v;
  __syncthreads();
  return res;
}

__device__ __forceinline__ int upper_bound_i32(const int32_t* a, int n, int x) {
  // first index i in [0, n) with a[i] > x
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] > x) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// Segment i -> [row_lo, row_hi) (the tile rows), [oth_lo, oth_hi) (the range
// the tile iterates over), sequence index, selection row.
__device__ void segment_info(int kind, int i, const lsrm_varlen& m, const int32_t* cu_seg, int window, int& row_lo,
                             int& row_hi, int& oth_lo, int& oth_hi, int& seq, int& sel_row) {
  sel_row = -1;
  switch (kind) {
    case kTilesSeq:
      row_lo = m.cu_seqlens_q[i];
      row_hi = m.cu_seqlens_q[i + 1];
      oth_lo = m.cu_seqlens_k[i];
      oth_hi = m.cu_seqlens_k[i + 1];
      seq = i;
      break;
    case kTilesQBlock:
      row_lo = cu_seg[i];
      row_hi = cu_seg[i + 1];
      seq = upper_bound_i32(m.cu_seqlens_q, m.num_seqs + 1, row_lo) - 1;
      oth_lo = m.cu_seqlens_k[seq];
      oth_hi = m.cu_seqlens_k[seq + 1];
      sel_row = i;
      break;
    case kTilesKVBlock:
      row_lo = m.cu_block_include_tokens[i];
      row_hi = m.cu_block_include_tokens[i + 1];
      oth_lo = row_lo;
      oth_hi = row_hi;
      seq = upper_bound_i32(m.cu_seqblocks, m.num_seqs + 1, i) - 1;
      break;
    case kTilesCompressed:  // rows = compressed keys of sequence i, other = its queries
      row_lo = m.cu_seqblocks[i];
      row_hi = m.cu_seqblocks[i + 1];
      oth_lo = m.cu_seqlens_q[i];
      oth_hi = m.cu_seqlens_q[i + 1];
      seq = i;
      break;
    default:  // kTilesKVSeq: rows = keys of sequence i, other = its queries
      row_lo = m.cu_seqlens_k[i];
      row_hi = m.cu_seqlens_k[i + 1];
      oth_lo = m.cu_seqlens_q[i];
      oth_hi = m.cu_seqlens_q[i + 1];
      seq = i;
      break;
  }
  (void)window;
}

// Forward tiles of the compressed branch: rows = queries of sequence i,
// other = compressed keys of sequence i.  Encoded as kind 5 internally.
constexpr int kTilesSeqCompressedKV = 5;

__global__ void build_tiles_kernel(QTile* tiles, int* n_tiles, int tiles_ub, int kind, int rows_per_tile,
                                   lsrm_varlen m, const int32_t* cu_seg, int n_seg, int window, int* err) {
  __shared__ int scratch[40];
  __shared__ int s_off[1024], s_cnt[1024];  // the chunk's segments: first tile (chunk-relative), tile count
  int base = 0;
  const int half = window / 2;
  const int k = (kind == kTilesSeqCompressedKV) ? kTilesSeq : kind;
  auto seg = [&](int i, int& row_lo, int& row_hi, int& oth_lo, int& oth_hi, int& sq, int& sel_row) {
    segment_info(k, i, m, cu_seg, window, row_lo, row_hi, oth_lo, oth_hi, sq, sel_row);
    if (kind == kTilesSeqCompressedKV) {
      oth_lo = m.cu_seqblocks[i];
      oth_hi = m.cu_seqblocks[i + 1];
    }
  };
  for (int c0 = 0; c0 < n_seg; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    int cnt = 0;
    if (i < n_seg) {
      int row_lo, row_hi, oth_lo, oth_hi, sq, sel_row;
      seg(i, row_lo, row_hi, oth_lo, oth_hi, sq, sel_row);
      if (row_hi > row_lo) cnt = (row_hi - row_lo + rows_per_tile - 1) / rows_per_tile;
    }
    int total;
    const int off = block_exclusive_scan(cnt, &total, scratch);
    s_off[threadIdx.x] = off;
    s_cnt[threadIdx.x] = cnt;
    __syncthreads();
    // the chunk's tiles, one thread each: segment by binary search of the offsets
    const int nseg_chunk = min((int)blockDim.x, n_seg - c0);
    for (int t_all = threadIdx.x; t_all < total; t_all += blockDim.x) {
      // the last segment whose first tile is <= t_all; an empty segment shares
      // its offset with the next one, so the last such segment holds t_all
      int lo = 0, hi = nseg_chunk - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= t_all) lo = mid;
        else hi = mid - 1;
      }
      const int idx = base + t_all;
      if (idx >= tiles_ub) {
        atomicOr(err, LSRM_ERR_CAPACITY);
        continue;
      }
      const int si = c0 + lo, t = t_all - s_off[lo];
      int row_lo, row_hi, oth_lo, oth_hi, sq, sel_row;
      seg(si, row_lo, row_hi, oth_lo, oth_hi, sq, sel_row);
      QTile q;
      q.q_start = row_lo + t * rows_per_tile;
      q.n_q = min(rows_per_tile, row_hi - q.q_start);
      q.kv_lo = oth_lo;
      q.kv_hi = oth_hi;
      if (window > 0) {
        // band |i - j| <= window/2 (query and key token indices of one sequence)
        q.kv_lo = max(oth_lo, q.q_start - half);
        q.kv_hi = min(oth_hi, q.q_start + q.n_q + half);
      }
      q.seq = sq;
      q.sel_row = sel_row;
      q.seg = si;
      q.pad = 0;
      tiles[idx] = q;
    }
    base += total;
    __syncthreads();  // s_off / s_cnt are rewritten by the next chunk
  }
  if (threadIdx.x == 0) *n_tiles = min(base, tiles_ub);
}

// ---------------------------------------------------------------------------
// Unions of selected blocks per (tile, kv head)
// ---------------------------------------------------------------------------
constexpr int kUnionThreads = 256;
constexpr int kMaxUnionEntries = 8192;

__global__ void __launch_bounds__(kUnionThreads)
    build_unions_kernel(SelectPlan p, lsrm_varlen m, const int32_t* __restrict__ block_topk, int topk, int sel_rows,
                        int G, int* err) {
  extern __shared__ int sm[];
  const int t = blockIdx.x, h = blockIdx.y;
  if (t >= *p.n_tiles) return;
  const QTile tile = p.tiles[t];
  const int blk0 = m.cu_seqblocks[tile.seq];
  const int nb_seq = m.cu_seqblocks[tile.seq + 1] - blk0;
  const bool per_block = tile.sel_row >= 0;
  const int E = per_block ? topk : tile.n_q * topk;
  int P = 1;
  while (P < E) P <<= 1;
  int* keys = sm;                  // [P]
  int* ids = sm + P;               // [P] unique ids
  uint32_t* masks = reinterpret_cast<uint32_t*>(sm + 2 * P);  // [cap][4]
  __shared__ int scratch[40];
  __shared__ int s_count, s_dup;
  const int32_t* sel = block_topk + (size_t)h * sel_rows * topk;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    int v = INT32_MAX;
    if (i < E) {
      const int row = per_block ? tile.sel_row : tile.q_start + i / topk;
      if (dcheck(row >= 0 && row < sel_rows, kDcSelRow, err)) {
        const int id = sel[(size_t)row * topk + (i % topk)];
        if (id >= 0 && id < nb_seq) v = id;
      }
    }
    keys[i] = v;
  }
  if (threadIdx.x == 0) s_dup = 0;
  __syncthreads();
  // bitonic sort, ascending
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const int a = keys[i], b = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // unique: each thread owns a contiguous run of the sorted keys
  const int per = (P + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(P, i0 + per);
  int cnt = 0;
  for (int i = i0; i < i1; ++i) {
    const int v = keys[i];
    if (v == INT32_MAX) continue;
    if (i == 0 || keys[i - 1] != v) ++cnt;
    else if (per_block) s_dup = 1;  // one selection row listing a block twice
  }
  int total;
  int pos = block_exclusive_scan(cnt, &total, scratch);
  for (int i = i0; i < i1; ++i) {
    const int v = keys[i];
    if (v == INT32_MAX) continue;
    if (i == 0 || keys[i - 1] != v) ids[pos++] = v;
  }
  if (threadIdx.x == 0) s_count = total;
  __syncthreads();
  const int U = s_count;
  if (U > p.union_cap) {
    if (threadIdx.x == 0) atomicOr(err, LSRM_ERR_CAPACITY);
    return;
  }
  for (int i = threadIdx.x; i < U * 4; i += blockDim.x) masks[i] = 0u;
  __syncthreads();
  if (per_block) {
    for (int u = threadIdx.x; u < U; u += blockDim.x)
      for (int w = 0; w < 4; ++w) {
        const int lo = w * 32;
        uint32_t bits = 0;
        if (tile.n_q > lo) bits = (tile.n_q - lo >= 32) ? 0xffffffffu : ((1u << (tile.n_q - lo)) - 1u);
        masks[u * 4 + w] = bits;
      }
  } else {
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
      const int r = i / topk;
      if (!dcheck(tile.q_start + r < sel_rows, kDcSelRow, err)) continue;
      const int id = sel[(size_t)(tile.q_start + r) * topk + (i % topk)];
      if (id < 0 || id >= nb_seq) continue;
      int lo = 0, hi = U;  // lower bound of id in ids[0..U)
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (ids[mid] < id) lo = mid + 1;
        else hi = mid;
      }
      const uint32_t bit = 1u << (r & 31);
      const uint32_t old = atomicOr(&masks[lo * 4 + (r >> 5)], bit);
      if (old & bit) s_dup = 1;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && s_dup) atomicOr(err, LSRM_ERR_DUPLICATE_BLOCK);
  // write the union, count 8-row groups for the chunk count
  const size_t base = ((size_t)h * p.tiles_ub + t) * p.union_cap;
  int groups = 0;
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int gb = blk0 + ids[u];
    p.union_blk[base + u] = gb;
    p.union_mask[base + u] = make_uint4(masks[u * 4], masks[u * 4 + 1], masks[u * 4 + 2], masks[u * 4 + 3]);
    const int t0 = max(m.cu_block_include_tokens[gb], tile.kv_lo);
    const int t1 = min(m.cu_block_include_tokens[gb + 1], tile.kv_hi);
    if (t1 > t0) groups += (t1 - t0 + kGroupRows - 1) / kGroupRows;
  }
  int gtotal;
  block_exclusive_scan(groups, &gtotal, scratch);
  if (threadIdx.x == 0) {
    p.union_cnt[(size_t)h * p.tiles_ub + t] = U;
    p.union_ngroups[(size_t)h * p.tiles_ub + t] = gtotal;
  }
}

// ---------------------------------------------------------------------------
// Reverse map: (kv head, block) -> ascending list of (tile, union entry)
// ---------------------------------------------------------------------------
__global__ void rev_count_kernel(SelectPlan p) {
  const int t = blockIdx.x, h = blockIdx.y;
  if (t >= *p.n_tiles) return;
  const size_t base = ((size_t)h * p.tiles_ub + t) * p.union_cap;
  const int U = p.union_cnt[(size_t)h * p.tiles_ub + t];
  for (int u = threadIdx.x; u < U; u += blockDim.x)
    atomicAdd(&p.rev_off[(size_t)h * (p.num_blocks + 1) + p.union_blk[base + u] + 1], 1);
}

__global__ void rev_scan_kernel(SelectPlan p) {
  __shared__ int scratch[40];
  const int h = blockIdx.x;
  int* off = p.rev_off + (size_t)h * (p.num_blocks + 1);
  int* cur = p.rev_cursor + (size_t)h * p.num_blocks;
  int run = 0;
  for (int c0 = 0; c0 < p.num_blocks; c0 += blockDim.x) {
    const int b = c0 + threadIdx.x;
    const int v = b < p.num_blocks ? off[b + 1] : 0;
    int total;
    const int ex = run + block_exclusive_scan(v, &total, scratch);
    if (b < p.num_blocks) {
      off[b + 1] = ex + v;
      cur[b] = ex;
    }
    run += total;
  }
  if (threadIdx.x == 0) off[0] = 0;
}

__global__ void rev_fill_kernel(SelectPlan p, int* err) {
  const int t = blockIdx.x, h = blockIdx.y;
  if (t >= *p.n_tiles) return;
  const size_t base = ((size_t)h * p.tiles_ub + t) * p.union_cap;
  const int U = p.union_cnt[(size_t)h * p.tiles_ub + t];
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int b = p.union_blk[base + u];
    const int pos = atomicAdd(&p.rev_cursor[(size_t)h * p.num_blocks + b], 1);
    if (dcheck(pos >= 0 && (long long)pos < (long long)p.tiles_ub * p.union_cap, kDcRevFill, err))
      p.rev_entries[(size_t)h * p.tiles_ub * p.union_cap + pos] = make_int2(t, u);
  }
}

// Per-block sort of the reverse lists (bitonic, in shared memory).  Keys are
// (tile, union slot); a block appears at most once per tile, so a list holds
// at most one entry per query tile.  When tile and slot fit in 19 + 13 bits
// the key is 32-bit and a list may hold kRevSortMax32 entries, otherwise 64-bit
// and kRevSortMax64; a longer list is left unsorted and flagged
// (LSRM_ERR_CAPACITY).  Two launches: lists of up to kRevSortSmall entries in
// small CTAs (many per SM), then the longer ones with the full capacity.
constexpr int kRevSortMax32 = 32768;  // 128 KB of keys
constexpr int kRevSortMax64 = 16384;  // 128 KB of keys
constexpr int kRevSortSmall = 2048;
constexpr int kRevSlotBits = 13;

template <typename K, bool SMALL>
__global__ void __launch_bounds__(256) rev_sort_kernel(SelectPlan p, int* err) {
  extern __shared__ __align__(16) unsigned char rs_smem[];
  K* keys = reinterpret_cast<K*>(rs_smem);
  constexpr bool k32 = sizeof(K) == 4;
  constexpr int cap = SMALL ? kRevSortSmall : k32 ? kRevSortMax32 : kRevSortMax64;
  const int b = blockIdx.x, h = blockIdx.y;
  const int* off = p.rev_off + (size_t)h * (p.num_blocks + 1);
  const int s = off[b], e = off[b + 1], n = e - s;
  if (n <= 1 || (SMALL ? n > kRevSortSmall : n <= kRevSortSmall)) return;  // the other launch's list
  if (n > cap) {
    if (threadIdx.x == 0) atomicOr(err, LSRM_ERR_CAPACITY);
    return;
  }
  int2* ent = p.rev_entries + (size_t)h * p.tiles_ub * p.union_cap + s;
  int P = 1;
  while (P < n) P <<= 1;
  const K kmax = ~K(0);
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    K k = kmax;
    if (i < n) {
      const int2 x = ent[i];
      k = k32 ? (K)(((uint32_t)x.x << kRevSlotBits) | (uint32_t)x.y)
              : (K)(((unsigned long long)(uint32_t)x.x << 32) | (uint32_t)x.y);
    }
    keys[i] = k;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const K a = keys[i], c = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > c) == up) {
            keys[i] = c;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const K k = keys[i];
    ent[i] = k32 ? make_int2((int)(k >> kRevSlotBits), (int)(k & ((1u << kRevSlotBits) - 1u)))
                 : make_int2((int)((unsigned long long)k >> 32), (int)((unsigned long long)k & 0xffffffffull));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static size_t carve(uint8_t*& cur, size_t bytes) {
  size_t a = align_up(bytes, 256);
  cur += a;
  return a;
}

SelectPlan make_select_plan(const lsrm_varlen* m, int G, int hkv, int topk, int num_qblocks, void* ws) {
  SelectPlan p{};
  const int qpt = kRows / G;
  const long long nq = m->total_q, nk = m->total_k;
  const bool qblock = num_qblocks > 0;
  p.tiles_ub = (int)(ceil_div<long long>(nq, qpt) + m->num_seqs + (qblock ? num_qblocks : 0) + 1);
  p.union_cap = (int)std::min<long long>(qblock ? topk : (long long)qpt * topk, std::max(m->num_blocks, 1));
  p.kvtiles_ub = (int)(ceil_div<long long>(nk, kRows) + m->num_blocks + 1);
  p.hkv = hkv;
  p.num_blocks = m->num_blocks;
  uint8_t* base = static_cast<uint8_t*>(ws);
  uint8_t* cur = base;
  auto take = [&](size_t bytes) {
    uint8_t* r = cur;
    carve(cur, bytes);
    return r;
  };
  const size_t ent = (size_t)hkv * p.tiles_ub * p.union_cap;
  p.tiles = reinterpret_cast<QTile*>(take(sizeof(QTile) * p.tiles_ub));
  p.n_tiles = reinterpret_cast<int*>(take(16));
  p.union_cnt = reinterpret_cast<int*>(take(sizeof(int) * hkv * p.tiles_ub));
  p.union_ngroups = reinterpret_cast<int*>(take(sizeof(int) * hkv * p.tiles_ub));
  p.union_blk = reinterpret_cast<int*>(take(sizeof(int) * ent));
  p.union_mask = reinterpret_cast<uint4*>(take(sizeof(uint4) * ent));
  p.kvtiles = reinterpret_cast<QTile*>(take(sizeof(QTile) * p.kvtiles_ub));
  p.n_kvtiles = reinterpret_cast<int*>(take(16));
  p.rev_off = reinterpret_cast<int*>(take(sizeof(int) * hkv * ((size_t)m->num_blocks + 1)));
  p.rev_cursor = reinterpret_cast<int*>(take(sizeof(int) * hkv * (size_t)std::max(m->num_blocks, 1)));
  p.rev_entries = reinterpret_cast<int2*>(take(sizeof(int2) * ent));
  const size_t items = (size_t)hkv * p.kvtiles_ub;
  p.piece_slots = (int)std::min<size_t>(kMaxPieceSlots, items);
  const size_t entries = items + p.piece_slots;
  p.kv_sched = reinterpret_cast<int*>(take(sizeof(int) * entries));
  p.sched_key = reinterpret_cast<int*>(take(sizeof(int) * entries));
  p.item_nch = reinterpret_cast<int*>(take(sizeof(int) * entries));
  p.item_rng = reinterpret_cast<int2*>(take(sizeof(int2) * entries));
  p.item_src = reinterpret_cast<int*>(take(sizeof(int) * p.piece_slots));
  p.item_slot = reinterpret_cast<int*>(take(sizeof(int) * items));
  p.sched_bins = reinterpret_cast<int*>(take(sizeof(int) * 2 * kSchedBins));
  p.sched_ctr = reinterpret_cast<int*>(take(sizeof(int) * 4));
  p.split_items = reinterpret_cast<int4*>(take(sizeof(int4) * p.piece_slots));
  p.bytes = (size_t)(cur - base);
  return p;
}

DensePlan make_dense_plan(const lsrm_varlen* m, int G, int mode, void* ws) {
  DensePlan p{};
  const int qpt = kRows / G;
  const long long nq = m->total_q, nk = m->total_k;
  long long nseg_q = (mode == LSRM_DENSE_INTRA_BLOCK) ? m->num_blocks : m->num_seqs;
  p.tiles_ub = (int)(ceil_div<long long>(nq, qpt) + nseg_q + 1);
  long long nrows_k = (mode == LSRM_DENSE_COMPRESSED) ? m->num_blocks : nk;
  long long nseg_k = (mode == LSRM_DENSE_INTRA_BLOCK) ? m->num_blocks : m->num_seqs;
  p.kvtiles_ub = (int)(ceil_div<long long>(nrows_k, kRows) + nseg_k + 1);
  uint8_t* base = static_cast<uint8_t*>(ws);
  uint8_t* cur = base;
  auto take = [&](size_t bytes) {
    uint8_t* r = cur;
    carve(cur, bytes);
    return r;
  };
  p.tiles = reinterpret_cast<QTile*>(take(sizeof(QTile) * p.tiles_ub));
  p.n_tiles = reinterpret_cast<int*>(take(16));
  p.kvtiles = reinterpret_cast<QTile*>(take(sizeof(QTile) * p.kvtiles_ub));
  p.n_kvtiles = reinterpret_cast<int*>(take(16));
  p.bytes = (size_t)(cur - base);
  return p;
}

int launch_build_tiles(QTile* tiles, int* n_tiles, int tiles_ub, int kind, int rows_per_tile, const lsrm_varlen* m,
                       const int32_t* cu_segments, int n_segments, int window, int* err, cudaStream_t s) {
  ProfScope ps("plan_tiles", s);
  build_tiles_kernel<<<1, 1024, 0, s>>>(tiles, n_tiles, tiles_ub, kind, rows_per_tile, *m, cu_segments, n_segments,
                                        window, err);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

int launch_build_unions(const SelectPlan& p, const lsrm_varlen* m, const int32_t* block_topk, int topk, int sel_rows,
                        int G, int* err, cudaStream_t s) {
  const int qpt = kRows / G;
  const int E = (sel_rows == m->total_q) ? qpt * topk : topk;
  int P = 1;
  while (P < std::max(E, 1)) P <<= 1;
  if (P > kMaxUnionEntries) {
    set_error("queries per tile (%d) x topk (%d) exceeds %d", qpt, topk, kMaxUnionEntries);
    return LSRM_ERR_UNSUPPORTED;
  }
  const size_t smem = sizeof(int) * 2 * P + sizeof(uint32_t) * 4 * (size_t)p.union_cap;
  if (smem > 200 * 1024) {
    set_error("union builder needs %zu bytes of shared memory", smem);
    return LSRM_ERR_UNSUPPORTED;
  }
  LSRM_CUDA_TRY(cudaFuncSetAttribute(build_unions_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(p.tiles_ub, p.hkv);
  ProfScope ps("plan_unions", s);
  build_unions_kernel<<<grid, kUnionThreads, smem, s>>>(p, *m, block_topk, topk, sel_rows, G, err);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

// dK/dV schedule.  Every (kv head, KV tile) item gets its number of 64-query
// chunks (the queries that selected the tile's block); an item much longer
// than the average load of one CTA is cut into pieces (runs of its reverse
// list, each accumulated into its own fp32 slot and summed afterwards in
// piece order), and the work entries are listed heaviest bucket first, so the
// longest CTAs start early instead of trailing the launch.  Order inside a
// bucket is arbitrary; it does not change any result.
// The chunk count follows the dK/dV kernel's rule: a run of the block's
// reverse list is read in segments of kRevCacheCap entries from its first
// entry (one shared-memory cache fill each); within a segment, G <= 8 runs in
// 8-row query groups (chunks of 8 groups), G > 8 in chunks of 64/G gathered
// queries.  One warp per item: the lanes stride over each segment's entries.
__device__ __forceinline__ int run_chunks(const SelectPlan& p, int h, int e0, int e1, int G) {
  const int qpc = 64 / G, W = G <= 8 ? 8 / G : 1;
  const int lane = threadIdx.x & 31;
  const int2* ent = p.rev_entries + (size_t)h * p.tiles_ub * p.union_cap;
  const bool grouped = G <= 8;
  int chunks = 0;
  for (int s0 = e0; s0 < e1; s0 += kRevCacheCap) {
    const int s1 = min(e1, s0 + kRevCacheCap);
    int nq = 0, ng = 0;
    for (int e = s0 + lane; e < s1; e += 32) {
      const int2 x = ent[e];
      const uint4 m = p.union_mask[((size_t)h * p.tiles_ub + x.x) * p.union_cap + x.y];
      nq += __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w);
      if (grouped) ng += window_count(m, W);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nq += __shfl_xor_sync(0xffffffffu, nq, o);
      ng += __shfl_xor_sync(0xffffffffu, ng, o);
    }
    chunks += grouped ? (ng + 7) / 8 : (nq + qpc - 1) / qpc;
  }
  return chunks;
}

__device__ __forceinline__ int sched_bin(int chunks) { return kSchedBins - 1 - min(chunks, kSchedBins - 1); }

// Pass 1: chunks of every item (whole list), their total; the piece entries
// start empty.
__global__ void sched_count_kernel(SelectPlan p, int G) {
  const int items = p.hkv * p.kvtiles_ub;
  const int n_kv = *p.n_kvtiles;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < p.piece_slots; j += gridDim.x * blockDim.x) {
    p.item_nch[items + j] = 0;
    p.item_rng[items + j] = make_int2(-1, 0);
    p.sched_key[items + j] = kSchedBins - 1;
    p.item_src[j] = 0;
  }
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < items; i += warps) {
    const int h = i / p.kvtiles_ub, kt = i - h * p.kvtiles_ub;
    int chunks = 0, e0 = 0, e1 = 0;
    if (kt < n_kv) {
      const int blk = p.kvtiles[kt].seg;
      const int* off = p.rev_off + (size_t)h * (p.num_blocks + 1);
      e0 = off[blk];
      e1 = off[blk + 1];
      chunks = run_chunks(p, h, e0, e1, G);
    }
    if (lane == 0) {
      p.item_nch[i] = chunks;
      p.item_rng[i] = make_int2(0, e1 - e0);
      if (chunks) atomicAdd(&p.sched_ctr[0], chunks);
    }
  }
}

// Pieces of one item: an item of more than half the average load of a CTA
// (total / 2 ctas chunks, at least 2 * kMinPieceChunks) is cut into up to
// kMaxPieces runs of equal entry counts, each about that long — the CTAs walk
// the heaviest-first list in a fixed snake order, so no single entry may hold
// much more than half a CTA's share.  1: the item stays whole.
__device__ __forceinline__ int item_pieces(int nch, int n_ent, bool valid, int target, int* per) {
  *per = n_ent;
  if (!valid || nch <= target || nch < 2 * kMinPieceChunks) return 1;
  const int want = min(min(kMaxPieces, (nch + target - 1) / target), min(n_ent, nch / kMinPieceChunks));
  if (want <= 1) return 1;
  *per = (n_ent + want - 1) / want;
  return (n_ent + *per - 1) / *per;
}

__device__ __forceinline__ int piece_target(const SelectPlan& p, int ctas) {
  return max((p.sched_ctr[0] + 2 * ctas - 1) / (2 * ctas), kMinPieceChunks);
}

// Pass 2 (one block): piece slots in item order — an exclusive scan of the
// pieces of every item to be cut; an item whose pieces would pass the last
// slot stays whole.  The choice depends on the item order alone, so the
// schedule (and every sum) is the same from run to run.
constexpr int kSlotThreads = 1024;
__global__ void __launch_bounds__(kSlotThreads) sched_slots_kernel(SelectPlan p, int ctas) {
  __shared__ int wsum[32];
  const int items = p.hkv * p.kvtiles_ub;
  const int n_kv = *p.n_kvtiles;
  const int target = piece_target(p, ctas);
  const int per_t = (items + kSlotThreads - 1) / kSlotThreads;
  const int i0 = threadIdx.x * per_t, i1 = min(items, i0 + per_t);
  auto pieces_of = [&](int i) {
    const int kt = i % p.kvtiles_ub;
    int per;
    const int pc = item_pieces(p.item_nch[i], p.item_rng[i].y, kt < n_kv, target, &per);
    return pc > 1 ? pc : 0;
  };
  int own = 0;
  for (int i = i0; i < i1; ++i) own += pieces_of(i);
  // block exclusive scan of `own`
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int x = wsum[lane];
    int xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += y;
    }
    wsum[lane] = xi - x;
  }
  __syncthreads();
  int pre = wsum[w] + incl - own;
  for (int i = i0; i < i1; ++i) {
    const int pc = pieces_of(i);
    p.item_slot[i] = pc > 0 && pre + pc <= p.piece_slots ? pre : -1;
    pre += pc;
  }
}

// Pass 3: the pieces of every item given slots (their runs, chunk counts and
// buckets); every item gets its bucket.
__global__ void sched_split_kernel(SelectPlan p, int G, int ctas) {
  const int items = p.hkv * p.kvtiles_ub;
  const int n_kv = *p.n_kvtiles;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int target = piece_target(p, ctas);
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < items; i += warps) {
    const int h = i / p.kvtiles_ub, kt = i - h * p.kvtiles_ub;
    const int nch = p.item_nch[i];
    const int n_ent = p.item_rng[i].y;
    const int slot0 = p.item_slot[i];
    if (slot0 < 0) {
      if (lane == 0) p.sched_key[i] = kt < n_kv ? sched_bin(nch) : kSchedBins - 1;
      continue;
    }
    int per;
    const int pieces = item_pieces(nch, n_ent, kt < n_kv, target, &per);
    const int e0 = p.rev_off[(size_t)h * (p.num_blocks + 1) + p.kvtiles[kt].seg];
    for (int k = 0; k < pieces; ++k) {
      const int lo = k * per, cnt = min(per, n_ent - lo);
      const int c = run_chunks(p, h, e0 + lo, e0 + lo + cnt, G);
      if (lane == 0) {
        const int j = items + slot0 + k;
        p.item_nch[j] = c;
        p.item_rng[j] = make_int2(lo, cnt);
        p.item_src[slot0 + k] = i;
        p.sched_key[j] = sched_bin(c);
      }
    }
    if (lane == 0) {
      p.item_rng[i] = make_int2(-1, 0);
      p.sched_key[i] = kSchedBins - 1;
      p.split_items[atomicAdd(&p.sched_ctr[2], 1)] = make_int4(i, slot0, pieces, 0);
    }
  }
}

__global__ void sched_bins_kernel(SelectPlan p) {
  const int entries = p.hkv * p.kvtiles_ub + p.piece_slots;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < entries; j += gridDim.x * blockDim.x)
    atomicAdd(&p.sched_bins[p.sched_key[j]], 1);
}

__global__ void sched_scan_kernel(SelectPlan p) {
  // one warp per 32 bins, serial over warps (1024 bins)
  __shared__ int wsum[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int v = p.sched_bins[threadIdx.x];
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int x = wsum[lane];
    int xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += y;
    }
    wsum[lane] = xi - x;
  }
  __syncthreads();
  p.sched_bins[kSchedBins + threadIdx.x] = wsum[w] + incl - v;
}

__global__ void sched_scatter_kernel(SelectPlan p) {
  const int entries = p.hkv * p.kvtiles_ub + p.piece_slots;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < entries; i += gridDim.x * blockDim.x) {
    const int pos = atomicAdd(&p.sched_bins[kSchedBins + p.sched_key[i]], 1);
    p.kv_sched[pos] = i;
  }
}

int launch_build_kv_schedule(const SelectPlan& p, int G, int ctas, cudaStream_t s) {
  ProfScope ps("plan_schedule", s);
  LSRM_CUDA_TRY(cudaMemsetAsync(p.sched_bins, 0, sizeof(int) * kSchedBins, s));
  LSRM_CUDA_TRY(cudaMemsetAsync(p.sched_ctr, 0, sizeof(int) * 4, s));
  const int items = p.hkv * p.kvtiles_ub;
  const int entries = items + p.piece_slots;
  const int grid = std::min((entries + 255) / 256, 148 * 8);
  const int warp_grid = std::min((items + 7) / 8, 148 * 16);  // 8 items (warps) per block
  sched_count_kernel<<<warp_grid, 256, 0, s>>>(p, G);
  LSRM_LAUNCH_CHECK();
  sched_slots_kernel<<<1, kSlotThreads, 0, s>>>(p, std::max(ctas, 1));
  LSRM_LAUNCH_CHECK();
  sched_split_kernel<<<warp_grid, 256, 0, s>>>(p, G, std::max(ctas, 1));
  LSRM_LAUNCH_CHECK();
  sched_bins_kernel<<<grid, 256, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  sched_scan_kernel<<<1, kSchedBins, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  sched_scatter_kernel<<<grid, 256, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

int launch_build_reverse(const SelectPlan& p, int* err, cudaStream_t s) {
  ProfScope ps("plan_reverse", s);
  LSRM_CUDA_TRY(cudaMemsetAsync(p.rev_off, 0, sizeof(int) * p.hkv * ((size_t)p.num_blocks + 1), s));
  dim3 grid(p.tiles_ub, p.hkv);
  rev_count_kernel<<<grid, 128, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  rev_scan_kernel<<<p.hkv, 1024, 0, s>>>(p);
  LSRM_LAUNCH_CHECK();
  rev_fill_kernel<<<grid, 128, 0, s>>>(p, err);
  LSRM_LAUNCH_CHECK();
  const dim3 grid_sort(std::max(p.num_blocks, 1), p.hkv);
  // 32-bit keys when tile < 2^19 - 1 and slot < 2^13 (no key equals the padding key ~0)
  if (p.tiles_ub < (1 << (32 - kRevSlotBits)) && p.union_cap <= (1 << kRevSlotBits)) {
    rev_sort_kernel<uint32_t, true><<<grid_sort, 256, kRevSortSmall * (int)sizeof(uint32_t), s>>>(p, err);
    LSRM_LAUNCH_CHECK();
    const int smem = kRevSortMax32 * (int)sizeof(uint32_t);
    LSRM_CUDA_TRY(
        cudaFuncSetAttribute(rev_sort_kernel<uint32_t, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    rev_sort_kernel<uint32_t, false><<<grid_sort, 256, smem, s>>>(p, err);
  } else {
    rev_sort_kernel<unsigned long long, true>
        <<<grid_sort, 256, kRevSortSmall * (int)sizeof(unsigned long long), s>>>(p, err);
    LSRM_LAUNCH_CHECK();
    const int smem = kRevSortMax64 * (int)sizeof(unsigned long long);
    LSRM_CUDA_TRY(cudaFuncSetAttribute(rev_sort_kernel<unsigned long long, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    rev_sort_kernel<unsigned long long, false><<<grid_sort, 256, smem, s>>>(p, err);
  }
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}

}  // namespace lsrm
