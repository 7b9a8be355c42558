// Forward attention kernel for sm_100a: one CTA per (query tile, kv head).
//
// Roles (352 threads):
//   warps 0-7  softmax: warps w and w+4 own MMA rows 32*(w%4).. (row r =
//              query r/G, head r%G) and split each 128-key chunk into two
//              64-key halves; they read S = Q K^T from TMEM, apply the row's
//              key mask, exchange the partial row max through shared memory
//              (online softmax in log2 units), write their half of P
//              (bf16/fp16) to TMEM, and each folds half of O's columns of
//              P V from TMEM into fp32 registers.
//   warp 8     producer: TMA loads of the Q tile and of K/V chunks (128 keys)
//              into a STAGES-deep ring.
//   warp 9     MMA issuer (lane 0): S_j = Q K_j^T (M=128, N=128).
//   warp 10    MMA issuer (lane 0): O_j = P_j V_j (M=128, N=D), P read from
//              TMEM.  S, P and PV are double-buffered in TMEM.
//
// KV chunk sources:
//   kSelect : the union of the blocks selected by the tile's queries, walked
//             in 8-token groups (one TMA box per group); a per-group query
//             bitmask tells each row which groups it may attend.
//   kRange  : a contiguous key range (compressed keys of the sequence, or the
//             tokens of one block), 128-key TMA boxes.
//   kBand   : a contiguous range with the band |i - j| <= half.
#pragma once

#include "common.cuh"
#include "plan.cuh"

namespace lsrm {

enum AttnMode : int { kSelect = 0, kRange = 1, kBand = 2 };

struct FwdParams {
  const QTile* tiles;
  const int* n_tiles;
  // select mode
  const int* union_cnt;
  const int* union_ngroups;
  const int* union_blk;
  const uint4* union_mask;
  int tiles_ub;
  int union_cap;
  const int32_t* cu_block_include_tokens;
  int num_blocks;
  // outputs
  void* out;
  float* lse;
  long long q_tok_stride;
  int num_q_heads;
  int total_q;
  int total_k;
  int G;
  float scale_log2;
  int half_window;
  int lse_natural;  // write ln-based LSE (compressed branch) instead of log2
  int hkv;          // kv heads (work items are tile x head)
  int* err;
};

struct ChunkMeta {
  uint32_t colmask[4];     // select: columns holding a key of the chunk
  uint32_t qmask[16][4];   // select: per group, the tile queries that may attend it
  int row0[16];            // select: first key token of each group (-1 = unused)
  int kv_start;            // range modes: first key token of the chunk
  int n_valid;             // range modes: keys in the chunk
  int pad[2];
};

template <int D, int STAGES>
struct FwdSmem {
  static constexpr int RB = 2 * D;
  static constexpr int TILE = 128 * RB;
  static constexpr int OFF_Q = 0;                 // two Q tiles (persistent CTAs prefetch the next)
  static constexpr int OFF_K = OFF_Q + 2 * TILE;
  static constexpr int OFF_V = OFF_K + STAGES * TILE;
  static constexpr int OFF_XCH = OFF_V + STAGES * TILE;  // row max / sum exchange [item parity][max|sum][half][128]
  static constexpr int OFF_META = OFF_XCH + 2 * 4 * 128 * 4;
  static constexpr int OFF_BAR = OFF_META + STAGES * (int)sizeof(ChunkMeta);
  // barriers: kv_full[S], kv_empty[S], q_full[2], q_empty[2], s_full[2], s_free[2],
  // p_full[2], p_free[2], pv_full[2], pv_free[2], mma_done, pv_mma_done, pair[4]
  static constexpr int NBAR = 2 * STAGES + 4 + 12 + 2 + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_UC = (OFF_MISC + 16 + 15) / 16 * 16;  // select mode: the tile's union
  static constexpr int BYTES = OFF_UC + (int)sizeof(UnionCache);
  static constexpr int ALLOC = (BYTES + 1024 > kOneCtaPerSmSmem) ? BYTES + 1024 : kOneCtaPerSmSmem;
  static_assert(OFF_UC % 16 == 0, "union cache must be 16-byte aligned");
  static_assert(ALLOC <= 227 * 1024, "shared memory budget");
};

constexpr int kFwdThreads = 352;


template <int D, bool BF16, int MODE, int STAGES>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ KVMaps kv,
                    const FwdParams prm) {
  using L = FwdSmem<D, STAGES>;
  constexpr int RB = L::RB;
  constexpr uint64_t SWZ = swz_for_row_bytes(RB);
  constexpr uint32_t AB = BF16 ? 1u : 0u;

  // Persistent CTAs: work item i = (tile i / Hkv, kv head i % Hkv) for
  // i = blockIdx.x, blockIdx.x + gridDim.x, ...  Every role walks the same
  // items; chunk counters J run on across items, so the ring barriers'
  // phases continue, and the producer fetches the next item's Q tile and
  // KV chunks while the softmax warps finish the current one.
  const int hkv_n = gridDim.y;  // 1: heads are folded into the item index
  (void)hkv_n;
  const int n_items = (*prm.n_tiles) * prm.hkv;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  ChunkMeta* meta = reinterpret_cast<ChunkMeta*>(smem + L::OFF_META);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + STAGES;
  uint64_t* q_full = bars + 2 * STAGES;
  uint64_t* q_empty = q_full + 2;
  uint64_t* s_full = q_empty + 2;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* p_free = p_full + 2;
  uint64_t* pv_full = p_free + 2;
  uint64_t* pv_free = pv_full + 2;
  uint64_t* mma_done = pv_free + 2;
  uint64_t* pv_mma_done = mma_done + 1;
  uint64_t* pair_mb = pv_mma_done + 1;  // [4]: the two softmax warps of a row quarter met at the item's end
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = prm.G;

  // per-item decode: tile, head, KV chunks (select: union size and base)
  struct Item {
    QTile tile;
    int tile_idx, h, n_chunks, U;
    size_t ubase;
  };
  auto item_of = [&](int i) {
    Item it;
    it.tile_idx = i / prm.hkv;
    it.h = i - it.tile_idx * prm.hkv;
    it.tile = prm.tiles[it.tile_idx];
    it.U = 0;
    it.ubase = 0;
    if constexpr (MODE == kSelect) {
      const size_t th = (size_t)it.h * prm.tiles_ub + it.tile_idx;
      it.ubase = th * prm.union_cap;
      it.U = prm.union_cnt[th];
      it.n_chunks = (prm.union_ngroups[th] + kGroupsPerChunk - 1) / kGroupsPerChunk;
      if (!dcheck((unsigned)it.U <= (unsigned)prm.union_cap, kDcUnion, prm.err)) it.U = it.n_chunks = 0;
    } else {
      it.n_chunks = it.tile.kv_hi > it.tile.kv_lo ? (it.tile.kv_hi - it.tile.kv_lo + kKVChunk - 1) / kKVChunk : 0;
    }
    if (!dcheck(it.tile.q_start >= 0 && it.tile.n_q >= 0 && it.tile.q_start + it.tile.n_q <= prm.total_q &&
                    it.n_chunks >= 0,
                kDcQTile, prm.err))
      it.tile.n_q = it.n_chunks = 0;
    return it;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_free[i], 1);
      mbar_init(&pv_full[i], i == 0 ? 8 : 1);  // pv_full[0]: o_free (the softmax warps read O)
      mbar_init(&pv_free[i], 8);
    }
    mbar_init(mma_done, 1);
    mbar_init(pv_mma_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_mb[i], 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S0 [0,128), S1 [128,256), O0 [256,256+D) and O1 [256+D, 256+2D)
  // (the output accumulated over keys 0-63 and 64-127 of every chunk, each
  // half on its own running row max), P0 [384,448), P1 [448,512) (16-bit
  // pairs: the A operand of P V)
  const uint32_t tm_s0 = tmem, tm_o0 = tmem + 256, tm_p0 = tmem + 384;
  uint64_t* o_free = &pv_full[0];  // the softmax warps have read O of the item

  if (warp == 8) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) tma_prefetch_desc(&tm_q);
    if (lane < kNumBoxes) {
      tma_prefetch_desc(&kv.k[lane]);
      tma_prefetch_desc(&kv.v[lane]);
    }
    UnionCache& uc = *reinterpret_cast<UnionCache*>(smem + L::OFF_UC);
    int J = 0, issued = 0, it_n = 0, q_loads = 0;  // chunks issued (all items), items started, Q tiles issued
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
      const Item w = item_of(i);
      const QTile& tile = w.tile;
      const int h = w.h, qb = it_n & 1;
      if (!warp_wait(&q_empty[qb], ((it_n >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[qb], L::TILE);
        tma_load_3d(sQ + qb * L::TILE, &tm_q, 0, h * G, tile.q_start, &q_full[qb]);
      }
      q_loads = it_n + 1;
      bool cached = false;
      if constexpr (MODE == kSelect)
        cached = union_cache_fill(uc, w.U, prm.union_blk, prm.union_mask, w.ubase, prm.cu_block_include_tokens,
                                  tile.kv_lo, tile.kv_hi, prm.num_blocks, prm.err);
      if (cached) {
        // the whole warp lays out each chunk (one lane per group) and issues its boxes
        int ucur = 0;
        for (int j = 0; j < w.n_chunks; ++j, ++J) {
          const int s = J % STAGES;
          if (!warp_wait(&kv_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          ChunkMeta& mt = meta[s];
          const int r = union_cache_chunk<kGroupsPerChunk>(uc, j, mt.row0, mt.qmask, mt.colmask, ucur);
          __syncwarp();
          if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], 2 * L::TILE);
          __syncwarp();
          issue_group_runs<kGroupsPerChunk, RB>(r, sK + s * L::TILE, sV + s * L::TILE, kv.k, kv.v, h, prm.total_k,
                                                &kv_full[s]);
          issued = J + 1;
        }
      } else {
        if (lane == 0) {
          int u = -1, tcur = 0, tend = 0;  // select-mode walk state (unions too large for the cache)
          for (int j = 0; j < w.n_chunks; ++j, ++J) {
            const int s = J % STAGES;
            if (!mbar_wait(&kv_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
            ChunkMeta& mt = meta[s];
            uint8_t* dK = sK + s * L::TILE;
            uint8_t* dV = sV + s * L::TILE;
            if constexpr (MODE == kSelect) {
              uint32_t cm[4] = {0u, 0u, 0u, 0u};
              for (int g = 0; g < kGroupsPerChunk; ++g) {
                while (tcur >= tend && u + 1 < w.U) {
                  ++u;
                  const int gb = prm.union_blk[w.ubase + u];
                  if (!dcheck((unsigned)gb < (unsigned)prm.num_blocks, kDcUnion, prm.err)) continue;
                  tcur = max(prm.cu_block_include_tokens[gb], tile.kv_lo);
                  tend = min(prm.cu_block_include_tokens[gb + 1], tile.kv_hi);
                }
                if (tcur < tend) {
                  const int cnt = min(kGroupRows, tend - tcur);
                  mt.row0[g] = tcur;
                  const uint4 qm = prm.union_mask[w.ubase + u];
                  mt.qmask[g][0] = qm.x;
                  mt.qmask[g][1] = qm.y;
                  mt.qmask[g][2] = qm.z;
                  mt.qmask[g][3] = qm.w;
                  cm[g >> 2] |= ((1u << cnt) - 1u) << ((g & 3) * 8);
                  tcur += cnt;
                } else {
                  mt.row0[g] = -1;
                  mt.qmask[g][0] = mt.qmask[g][1] = mt.qmask[g][2] = mt.qmask[g][3] = 0u;
                }
              }
              for (int x = 0; x < 4; ++x) mt.colmask[x] = cm[x];
              mbar_arrive_expect_tx(&kv_full[s], 2 * L::TILE);
              // unused groups read past the end of the tensor: zero fill
              load_group_runs<kGroupsPerChunk, RB>(mt.row0, dK, dV, kv.k, kv.v, h, prm.total_k, &kv_full[s]);
            } else {
              const int k0 = tile.kv_lo + j * kKVChunk;
              mt.kv_start = k0;
              mt.n_valid = min(kKVChunk, tile.kv_hi - k0);
              mbar_arrive_expect_tx(&kv_full[s], 2 * L::TILE);
              tma_load_3d(dK, &kv.k[kNumBoxes - 1], 0, h, k0, &kv_full[s]);
              tma_load_3d(dV, &kv.v[kNumBoxes - 1], 0, h, k0, &kv_full[s]);
            }
            issued = J + 1;
          }
        }
        // lane 0 advanced J and may have hit an abort: share both
        J = __shfl_sync(0xffffffffu, J, 0);
        issued = __shfl_sync(0xffffffffu, issued, 0);
        ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      }
    }
    // Teardown after an abort: let issued copies land before the CTA exits.
    if (lane == 0 && *abort_flag) {
      for (int k = max(0, q_loads - 2); k < q_loads; ++k) mbar_wait_drain(&q_full[k & 1], (k >> 1) & 1);
      for (int j = max(0, issued - STAGES); j < issued; ++j) mbar_wait_drain(&kv_full[j % STAGES], (j / STAGES) & 1);
    }
    __syncwarp();
  } else if (warp == 9) {
    // --------------------------- MMA issuer: S = Q K^T ----------------------
    // Two threads issue the tensor-core work (one spends ~90 cycles per
    // tcgen05.mma in short bursts): this one S, warp 10 the P V products.
    if (lane == 0) {
      const uint32_t idesc_qk = make_idesc(AB, 0, 0, 128, 128);
      bool ok = true;
      int J = 0, it_n = 0;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
        const int n_chunks = item_of(i).n_chunks, qb = it_n & 1;
        if (!mbar_wait(&q_full[qb], (it_n >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
        const uint32_t q_base = smem_u32(sQ + qb * L::TILE);
        for (int j = 0; j < n_chunks; ++j, ++J) {
          const int s = J % STAGES, sb = J & 1;
          if (!mbar_wait(&kv_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
          if (!mbar_wait(&s_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * L::TILE);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint64_t da = make_sdesc(q_base + ks * 32, 16, 8 * RB, SWZ);
            const uint64_t db = make_sdesc(k_base + ks * 32, 16, 8 * RB, SWZ);
            umma_f16(tm_s0 + sb * 128, da, db, idesc_qk, ks > 0);
          }
          umma_commit(&s_full[sb]);
        }
        if (!ok) break;
        umma_commit(&q_empty[qb]);  // the item's Q tile is free once its S products are done
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
    __syncwarp();
  } else if (warp == 10) {
    // --------------------------- MMA issuer: O += P_j V_j ------------------
    // Two accumulations per chunk, O0 += P[:, 0:64] V[0:64] and
    // O1 += P[:, 64:128] V[64:128] (the two softmax warps of a row quarter
    // scale their halves independently).  S_j is complete once P_j is written
    // (the softmax warps read it first), so this thread's commit alone
    // releases the chunk's K / V stage; its commit on p_free also tells the
    // softmax warps that O holds chunk j.
    if (lane == 0) {
      const uint32_t idesc_pv = make_idesc(AB, 0, 1, 128, D);
      bool ok = true;
      int J = 0, it_n = 0;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
        const int n_chunks = item_of(i).n_chunks;
        // the previous item's O must have been read out before chunk 0 overwrites it
        if (!mbar_wait(o_free, (it_n & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
        for (int j = 0; j < n_chunks; ++j, ++J) {
          const int pb = J & 1, s = J % STAGES;
          if (!mbar_wait(&p_full[pb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t v_base = smem_u32(sV + s * L::TILE);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t db = make_sdesc(v_base + (hh * 4 + ks) * 16 * RB, L::TILE, 8 * RB, SWZ);
              umma_f16_ts(tm_o0 + hh * D, tm_p0 + pb * 64 + hh * 32 + ks * 8, db, idesc_pv,
                          (j > 0 || ks > 0) ? 1u : 0u);
            }
          umma_commit(&p_free[pb]);
          umma_commit(&kv_empty[s]);
        }
      }
      umma_commit(pv_mma_done);
      mbar_wait_drain(pv_mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax -------------------------------
    // Warps w and w+4 share the rows of TMEM lane quarter w & 3 and take key
    // columns 0-63 and 64-127 of every chunk.  Each keeps its own running row
    // max m and sum l over its columns and its own output half O_h in TMEM,
    // so the pair never synchronises inside an item.  The max is lazy: P =
    // exp2(s - m) may reach 2^8 before O_h and l are rescaled to a new max
    // (fp32 accumulators, bf16 P keeps its relative precision), which skips
    // nearly every rescale after the first chunks.  At the end of an item the
    // pair combines (m, l) once and each warp writes half of the output
    // columns from both O halves.
    constexpr int DH = D / 2;         // output columns written by each warp of a pair
    constexpr float kLazy = 8.f;      // log2 headroom before a rescale
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // MMA row
    const int qloc = r / G;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tm_oh = tm_o0 + half * D;  // this warp's output half
    const float sl2 = prm.scale_log2;
    float* xch = reinterpret_cast<float*>(smem + L::OFF_XCH);  // [max|sum][half][128]
    bool ok = true;

    int J = 0, it_n = 0;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++it_n) {
    const Item w = item_of(it);
    const QTile& tile = w.tile;
    const int n_chunks = w.n_chunks;
    const int hq = w.h * G + (r % G);
    const int qi = tile.q_start + qloc;
    const bool row_valid = qloc < tile.n_q;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n_chunks; ++j, ++J) {
      const int s = J % STAGES, sb = J & 1;
      if (!warp_wait(&s_full[sb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
      if (!warp_wait(&kv_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      // key-validity mask of this row for the warp's 64 columns (2 words)
      uint32_t vm[2];
      const ChunkMeta& mt = meta[s];
      if constexpr (MODE == kSelect) {
        const int wq = qloc >> 5, b = qloc & 31;
#pragma unroll
        for (int xx = 0; xx < 2; ++xx) {
          const int x = 2 * half + xx;
          uint32_t e = 0u;
#pragma unroll
          for (int y = 0; y < 4; ++y)
            if ((mt.qmask[x * 4 + y][wq] >> b) & 1u) e |= 0xffu << (y * 8);
          vm[xx] = e & mt.colmask[x];
        }
      } else {
        int lo = 0, hi = mt.n_valid;  // valid columns [lo, hi)
        if constexpr (MODE == kBand) {
          lo = max(lo, qi - prm.half_window - mt.kv_start);
          hi = min(hi, qi + prm.half_window + 1 - mt.kv_start);
        }
#pragma unroll
        for (int xx = 0; xx < 2; ++xx) {
          const int x = 2 * half + xx;
          const int a = max(lo - 32 * x, 0), bnd = min(hi - 32 * x, 32);
          uint32_t e = 0u;
          if (bnd > a) e = ((bnd - a) == 32 ? 0xffffffffu : ((1u << (bnd - a)) - 1u)) << a;
          vm[xx] = e;
        }
      }
      const uint32_t tm_s = tm_s0 + sb * 128 + lane_base + half * 64;
      float sv[2][32];
      tmem_ld32(tm_s, sv[0]);
      tmem_ld32(tm_s + 32, sv[1]);
      tmem_wait_ld();
      // S of this chunk is in registers: the TMEM buffer can be refilled
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      // every row of the warp attends all 64 columns (rows past the tile do
      // not matter): no per-element masking
      const bool full = __all_sync(0xffffffffu, !row_valid || (vm[0] & vm[1]) == 0xffffffffu);
      float mx = -INFINITY;
      if (full) {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int xx = 0; xx < 2; ++xx)
#pragma unroll
          for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[xx][c]);
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      } else {
#pragma unroll
        for (int xx = 0; xx < 2; ++xx)
#pragma unroll
          for (int c = 0; c < 32; ++c) mx = fmaxf(mx, ((vm[xx] >> c) & 1u) ? sv[xx][c] : -INFINITY);
      }
      const float cand = mx * sl2;
      if (j == 0) {
        m = cand;  // O_h is overwritten by this chunk's product, l starts at 0
      } else {
        const bool need = cand > m + kLazy;
        if (__any_sync(0xffffffffu, need)) {
          // rescale this warp's rows of O_h to the new max: the previous
          // chunk's product into O_h must have landed first
          const int pj = J - 1;
          if (!warp_wait(&p_free[pj & 1], (pj >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const float m_new = need ? cand : m;
          // unchanged rows keep their scale (also m == m_new == -inf: no key
          // yet); m == -inf with a finite m_new scales zeros by 0
          const float alpha = (m_new == m) ? 1.f : ex2(m - m_new);
          l *= alpha;
          m = m_new;
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 16) {
            float ov[16];
            tmem_load_cols<16>(tm_oh + c0 + lane_base, ov);
            tmem_wait_ld();
            uint32_t ou[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) ou[c] = __float_as_uint(ov[c] * alpha);
            tmem_st16(tm_oh + c0 + lane_base, ou);
          }
          tmem_wait_st();
        }
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      // probabilities -> P: this warp's 64 keys as 16-bit pairs into TMEM
      // columns [half*32, half*32+32) of the P buffer (operand A of P V)
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[2][16];
#pragma unroll
      for (int xx = 0; xx < 2; ++xx) {
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float e = ex2(fmaf(sv[xx][c], sl2, -m_use));
            sv[xx][c] = e;
            rs4[c & 3] += e;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float e = ex2(fmaf(sv[xx][c], sl2, -m_use));  // unconditional: no branch per element
            const float pv = ((vm[xx] >> c) & 1u) ? e : 0.f;
            sv[xx][c] = pv;
            rs4[c & 3] += pv;
          }
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[xx][c] = pack2<BF16>(sv[xx][2 * c], sv[xx][2 * c + 1]);
      }
      if (!warp_wait(&p_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      tmem_st16(tm_p0 + sb * 64 + half * 32 + lane_base, pk[0]);
      tmem_st16(tm_p0 + sb * 64 + half * 32 + 16 + lane_base, pk[1]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
    }
    // epilogue: wait for the item's last product, combine the pair's (m, l)
    // once, and write this warp's output columns from both O halves
    if (ok && n_chunks > 0) {
      const int pj = J - 1;
      ok = warp_wait(&p_free[pj & 1], (pj >> 1) & 1, abort_flag, prm.err);
    }
    if (ok) {
      // the pair meets on an mbarrier (a bounded wait, so a partner that
      // aborted cannot hold this warp); slots alternate by item, and a warp
      // cannot reach item n+2 before its partner has read item n's values
      float* xb = xch + (it_n & 1) * 512;
      xb[half * 128 + r] = m;
      xb[256 + half * 128 + r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&pair_mb[quarter]);
      ok = warp_wait(&pair_mb[quarter], it_n & 1, abort_flag, prm.err);
    }
    if (ok) {
      const float* xb = xch + (it_n & 1) * 512;
      const float m0 = xb[r], m1 = xb[128 + r];
      const float l0 = xb[256 + r], l1 = xb[256 + 128 + r];
      const float mm = fmaxf(m0, m1);
      const float c0 = (m0 == -INFINITY) ? 0.f : ex2(m0 - mm);
      const float c1 = (m1 == -INFINITY) ? 0.f : ex2(m1 - mm);
      const float lt = l0 * c0 + l1 * c1;  // same order in both warps
      float o[DH];
      if (n_chunks > 0) {
        float o1[DH];
        tc_fence_after();
        tmem_load_cols<DH>(tm_o0 + half * DH + lane_base, o);
        tmem_load_cols<DH>(tm_o0 + D + half * DH + lane_base, o1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < DH; ++c) o[c] = o[c] * c0 + o1[c] * c1;
      } else {
#pragma unroll
        for (int c = 0; c < DH; ++c) o[c] = 0.f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);  // O of this item is read
      if (row_valid) {
        const float inv = (lt > 0.f) ? 1.f / lt : __int_as_float(0x7fc00000);
        uint8_t* orow =
            static_cast<uint8_t*>(prm.out) + ((size_t)qi * prm.q_tok_stride + (size_t)hq * D + half * DH) * 2;
        if (dcheck(qi < prm.total_q && hq < prm.num_q_heads, kDcOutRow, prm.err)) {
#pragma unroll
          for (int c = 0; c < DH; c += 8) {
            uint4 pk;
            pk.x = pack2<BF16>(o[c] * inv, o[c + 1] * inv);
            pk.y = pack2<BF16>(o[c + 2] * inv, o[c + 3] * inv);
            pk.z = pack2<BF16>(o[c + 4] * inv, o[c + 5] * inv);
            pk.w = pack2<BF16>(o[c + 6] * inv, o[c + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 2) = pk;
          }
          if (half == 0) {
            float lse = (lt > 0.f) ? mm + __log2f(lt) : -INFINITY;
            if (prm.lse_natural) lse *= 0.69314718055994531f;
            prm.lse[(size_t)hq * prm.total_q + qi] = lse;
          }
        }
      }
    }
    }  // items
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace lsrm
