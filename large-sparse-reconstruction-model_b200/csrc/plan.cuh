// Work decomposition shared by the attention kernels.
//
// A query tile is up to 128 MMA rows: QPT = 128 / G queries x G query heads
// of one KV head.  Query tiles never straddle a sequence (and, when query
// blocks are given, never straddle a query block).  For selected-block
// attention each (tile, kv head) carries the ascending union of the blocks its
// queries selected and, per union entry, the bitmask of tile queries that
// selected it; the KV side of the kernels walks that union in 8-token groups.
// The backward's reverse map lists, per (kv head, block), the (tile, entry)
// pairs in ascending tile order, so dK/dV accumulate in a fixed order.
#pragma once

#include <cstdint>
#include <cuda.h>

#include "lsrm_sparse.h"

namespace lsrm {

struct QTile {
  int q_start;  // first query (global token index)
  int n_q;      // queries in the tile
  int kv_lo;    // KV token range the tile may read (sequence or block range)
  int kv_hi;
  int seq;      // sequence index
  int sel_row;  // selection row for per-query-block selection, else -1
  int seg;      // segment index the tile came from (block / query block / sequence)
  int pad;
};

// Tile-list builder modes.
enum TileKind : int {
  kTilesSeq = 0,        // segments = sequences of the query side
  kTilesQBlock = 1,     // segments = query blocks (selection per query block)
  kTilesKVBlock = 2,    // segments = KV blocks (intra-block window; dK/dV tiles)
  kTilesCompressed = 3, // segments = compressed-key ranges of sequences (dK/dV)
  kTilesKVSeq = 4,      // segments = KV sequences (sliding-window dK/dV)
};

constexpr int kRows = 128;     // MMA M (rows of a query or KV tile)
constexpr int kKVChunk = 128;  // keys per KV chunk (MMA N of S = Q K^T)
constexpr int kGroupRows = 8;  // rows per TMA gather group in select mode
constexpr int kGroupsPerChunk = kKVChunk / kGroupRows;

// TMA maps over K and V with box heights 8, 16, 32, 64, 128 rows; used to
// load runs of consecutive 8-token groups with as few copies as possible.
constexpr int kNumBoxes = 5;
struct KVMaps {
  CUtensorMap k[kNumBoxes];
  CUtensorMap v[kNumBoxes];
};

// Workspace layout for selected-block attention.
struct SelectPlan {
  int tiles_ub;      // capacity of the tile list
  int union_cap;     // union entries per (tile, head)
  int kvtiles_ub;    // capacity of the KV tile list
  int hkv;
  int num_blocks;
  int piece_slots;   // dK/dV work entries for the pieces of long items
  // device pointers into the workspace
  QTile* tiles;
  int* n_tiles;            // [1]
  int* union_cnt;          // [hkv][tiles_ub]
  int* union_ngroups;       // [hkv][tiles_ub] 8-token groups of the union
  int* union_blk;          // [hkv][tiles_ub][cap] global block ids
  uint4* union_mask;       // [hkv][tiles_ub][cap] query bits within the tile
  QTile* kvtiles;          // dK/dV tiles (one block's keys, <= 128)
  int* n_kvtiles;          // [1]
  int* rev_off;            // [hkv][num_blocks+1]
  int* rev_cursor;         // [hkv][num_blocks]
  int2* rev_entries;       // [hkv][tiles_ub*cap] (tile, union entry index)
  // dK/dV work entries: e < hkv*kvtiles_ub is the item (kv head, KV tile)
  // e = h*kvtiles_ub + tile over the block's whole reverse list; e =
  // hkv*kvtiles_ub + slot is a piece of a long item (a run of its list,
  // accumulated into its own fp32 slot and summed afterwards)
  int* kv_sched;           // [entries] work entries, heaviest first
  int* item_nch;           // [entries] query chunks of each entry
  int2* item_rng;          // [entries] {first entry, entries} of the block's list; x < 0: split into pieces
  int* item_src;           // [piece_slots] the item each piece belongs to
  int* item_slot;          // [hkv*kvtiles_ub] first piece slot of an item that is cut, else -1
  int* sched_key;          // [entries] bucket of each entry
  int* sched_bins;         // [2*kSchedBins] bucket counts, then cursors
  int* sched_ctr;          // [4] chunks of all items, 0, split items, 0
  int4* split_items;       // [piece_slots] {item, first slot, pieces, 0} of every split item
  size_t bytes;
};

constexpr int kMaxPieceSlots = 256;  // pieces of long dK/dV items per launch
constexpr int kMaxPieces = 8;        // pieces of one item
constexpr int kMinPieceChunks = 8;   // no piece shorter than this many chunks

constexpr int kSchedBins = 1024;  // dK/dV schedule buckets (query chunks, capped)

// dK/dV reverse-map cache capacity (entries of one block kept in shared memory)
constexpr int kRevCacheCap = 1024;

// Query groups (G <= 8): a tile's 128 MMA rows are 16 windows of 8 rows,
// window w = queries [w*W, w*W + W) of the tile, W = 8/G.  A group is one
// non-empty window of one reverse-map entry; its bits say which of its W
// queries selected the block.
__device__ __forceinline__ uint32_t window_bits(const uint4& m, int w, int W) {
  const int o = w * W;
  const uint32_t word = (o >> 5) == 0 ? m.x : (o >> 5) == 1 ? m.y : (o >> 5) == 2 ? m.z : m.w;
  return (word >> (o & 31)) & ((1u << W) - 1u);
}

// Number of non-empty windows (W in {1, 2, 4, 8}) of a 128-bit mask.
__device__ __forceinline__ int window_count(const uint4& m, int W) {
  auto f = [&](uint32_t x) {
    if (W >= 2) x |= x >> 1;
    if (W >= 4) x |= x >> 2;
    if (W >= 8) x |= x >> 4;
    const uint32_t keep = W == 1 ? 0xffffffffu : W == 2 ? 0x55555555u : W == 4 ? 0x11111111u : 0x01010101u;
    return __popc(x & keep);
  };
  return f(m.x) + f(m.y) + f(m.z) + f(m.w);
}

__device__ __forceinline__ uint32_t window_mask(const uint4& m, int W) {
  uint32_t wm = 0u;
#pragma unroll
  for (int w = 0; w < 16; ++w) wm |= (window_bits(m, w, W) != 0u ? 1u : 0u) << w;
  return wm;
}

struct DensePlan {
  int tiles_ub;
  int kvtiles_ub;
  QTile* tiles;
  int* n_tiles;
  QTile* kvtiles;
  int* n_kvtiles;
  size_t bytes;
};

// fp32 dK and dV of every piece slot: [piece_slots][2][kRows][D].
inline size_t piece_partial_bytes(const SelectPlan& p, int D) {
  return (size_t)p.piece_slots * 2 * kRows * D * sizeof(float);
}

// Host helpers (plan.cu).
SelectPlan make_select_plan(const lsrm_varlen* m, int G, int hkv, int topk, int num_qblocks, void* ws);
DensePlan make_dense_plan(const lsrm_varlen* m, int G, int mode, void* ws);

// Enqueue the plan-building kernels.  Return 0 or an LSRM error code.
int launch_build_tiles(QTile* tiles, int* n_tiles, int tiles_ub, int kind, int rows_per_tile, const lsrm_varlen* m,
                       const int32_t* cu_segments, int n_segments, int window, int* err, cudaStream_t s);
int launch_build_unions(const SelectPlan& p, const lsrm_varlen* m, const int32_t* block_topk, int topk,
                        int sel_rows, int G, int* err, cudaStream_t s);
int launch_build_reverse(const SelectPlan& p, int* err, cudaStream_t s);
int launch_build_kv_schedule(const SelectPlan& p, int G, int ctas, cudaStream_t s);

}  // namespace lsrm
