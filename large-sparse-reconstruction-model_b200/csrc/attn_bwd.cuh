// Backward attention kernels for sm_100a.
//
// attn_dq_kernel — one CTA per (query tile, kv head), 64-key chunks:
//   S_j = Q K_j^T, dP_j = dO V_j^T (TMEM, double-buffered); the 4 compute
//   warps form dS = P (dP - delta) * scale with P = exp2(S*scale*log2e - lse)
//   and the row's key mask, write dS to shared memory; dQ += dS K_j
//   accumulates in TMEM and is written once.  Row r also computes
//   delta = rowsum(O * dO) in its prologue and stores it for dK/dV.
//
// attn_dkdv_kernel — one CTA per (KV tile of <= 128 keys, kv head[, split]):
//   the queries attending the tile are gathered 64 MMA rows at a time (for
//   selected-block attention: the tiles listed by the sorted reverse map and
//   their query bitmasks; for dense branches: a contiguous query range);
//   S^T = K Q_c^T, dP^T = V dO_c^T; the compute warps (row = key) form P^T and
//   dS^T; dV += P^T dO_c and dK += dS^T Q_c accumulate in TMEM.  Single writer
//   per KV tile, query chunks in ascending order: deterministic.
#pragma once

#include <climits>

#include "attn_fwd.cuh"
#include "common.cuh"
#include "plan.cuh"

namespace lsrm {

constexpr int kDqChunk = 64;     // keys per dQ chunk
constexpr int kDqGroups = kDqChunk / kGroupRows;
constexpr int kKvQRows = 64;     // query rows per dK/dV chunk

struct DqParams {
  const QTile* tiles;
  const int* n_tiles;
  const int* union_cnt;
  const int* union_ngroups;
  const int* union_blk;
  const uint4* union_mask;
  int tiles_ub;
  int union_cap;
  const int32_t* cu_block_include_tokens;
  int num_blocks;
  const void* out;
  const void* dout;
  const float* lse;
  float* delta;
  void* dq;
  long long q_tok_stride;
  int total_q;
  int total_k;
  int G;
  float scale_log2;
  float scale;
  int half_window;
  int lse_natural;
  int hkv;  // kv heads (work items are tile x head)
  int* err;
};

struct DqMeta {
  uint32_t colmask[2];
  uint32_t qmask[kDqGroups][4];
  int row0[kDqGroups];
  int kv_start;
  int n_valid;
};

template <int D, int STAGES>
struct DqSmem {
  static constexpr int RB = 2 * D;
  static constexpr int QTILE = 128 * RB;
  static constexpr int KTILE = kDqChunk * RB;
  static constexpr int OFF_Q = 0;            // two Q tiles and two dO tiles (the next item's prefetch)
  static constexpr int OFF_DO = 2 * QTILE;
  static constexpr int OFF_K = 4 * QTILE;
  static constexpr int OFF_V = OFF_K + STAGES * KTILE;
  static constexpr int OFF_META = OFF_V + STAGES * KTILE;  // dS lives in TMEM
  static constexpr int OFF_BAR = OFF_META + STAGES * (int)sizeof(DqMeta);
  // kv_full[S], kv_empty[S], qdo_full[2], qdo_empty[2], sd_full[2], sd_free[2],
  // ds_full[2], ds_free[2], dq_done, dq_free, mma_done, dq_mma_done, uc_empty, uc_full
  static constexpr int NBAR = 2 * STAGES + 4 + 8 + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_UC = (OFF_MISC + 16 + 15) / 16 * 16;  // select mode: the tile's union
  static constexpr int BYTES = OFF_UC + (int)sizeof(UnionCache);
  static constexpr int ALLOC = (BYTES + 1024 > kOneCtaPerSmSmem) ? BYTES + 1024 : kOneCtaPerSmSmem;
  static_assert(ALLOC <= 227 * 1024, "shared memory budget");
};

// Fills the groups of one select-mode chunk by walking the union.
template <int NG>
__device__ __forceinline__ void walk_union_groups(int& u, int& tcur, int& tend, int U, const int* union_blk,
                                                  const uint4* union_mask, size_t ubase, const int32_t* cu_blk,
                                                  int kv_lo, int kv_hi, int* row0, uint32_t (*qmask)[4],
                                                  uint32_t* colmask, int num_blocks, int* err) {
  uint32_t cm[NG / 4];
#pragma unroll
  for (int w = 0; w < NG / 4; ++w) cm[w] = 0u;
  for (int g = 0; g < NG; ++g) {
    while (tcur >= tend && u + 1 < U) {
      ++u;
      const int gb = union_blk[ubase + u];
      if (!dcheck((unsigned)gb < (unsigned)num_blocks, kDcUnion, err)) continue;  // tcur == tend: next entry
      tcur = max(cu_blk[gb], kv_lo);
      tend = min(cu_blk[gb + 1], kv_hi);
    }
    if (tcur < tend) {
      const int cnt = min(kGroupRows, tend - tcur);
      row0[g] = tcur;
      const uint4 qm = union_mask[ubase + u];
      qmask[g][0] = qm.x;
      qmask[g][1] = qm.y;
      qmask[g][2] = qm.z;
      qmask[g][3] = qm.w;
      cm[g >> 2] |= ((1u << cnt) - 1u) << ((g & 3) * 8);
      tcur += cnt;
    } else {
      row0[g] = -1;
      qmask[g][0] = qmask[g][1] = qmask[g][2] = qmask[g][3] = 0u;
    }
  }
#pragma unroll
  for (int w = 0; w < NG / 4; ++w) colmask[w] = cm[w];
}

// Threads of the dQ kernel: 8 compute warps (two per TMEM lane quarter,
// splitting the 64 key columns of a chunk), two producer warps (8 and 11,
// alternate chunks) and two MMA-issuing warps (9: S / dP, 10: dQ).
constexpr int kDqThreads = 384;

template <int D, bool BF16, int MODE, int STAGES>
__global__ void __launch_bounds__(kDqThreads, 1)
    attn_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                   const __grid_constant__ KVMaps kv, const DqParams prm) {
  using L = DqSmem<D, STAGES>;
  constexpr int RB = L::RB;
  constexpr uint64_t SWZ = swz_for_row_bytes(RB);
  constexpr uint32_t AB = BF16 ? 1u : 0u;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;

  // Persistent CTAs over (tile, kv head) items; see attn_fwd_kernel.
  const int n_items = (*prm.n_tiles) * prm.hkv;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  DqMeta* meta = reinterpret_cast<DqMeta*>(smem + L::OFF_META);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + STAGES;
  uint64_t* qdo_full = bars + 2 * STAGES;
  uint64_t* qdo_empty = qdo_full + 2;
  uint64_t* sd_full = qdo_empty + 2;
  uint64_t* sd_free = sd_full + 2;
  uint64_t* ds_full = sd_free + 2;
  uint64_t* ds_free = ds_full + 2;
  uint64_t* dq_done = ds_free + 2;
  uint64_t* dq_free = dq_done + 1;
  uint64_t* mma_done = dq_free + 1;
  uint64_t* dq_mma_done = mma_done + 1;
  uint64_t* uc_empty = dq_mma_done + 1;  // both producer warps are done with the union cache (count 2)
  uint64_t* uc_full = uc_empty + 1;      // warp 8 has filled it for the next item (count 1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = prm.G;

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
      it.n_chunks = (prm.union_ngroups[th] + kDqGroups - 1) / kDqGroups;
      if (!dcheck((unsigned)it.U <= (unsigned)prm.union_cap, kDcUnion, prm.err)) it.U = it.n_chunks = 0;
    } else {
      it.n_chunks = it.tile.kv_hi > it.tile.kv_lo ? (it.tile.kv_hi - it.tile.kv_lo + kDqChunk - 1) / kDqChunk : 0;
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
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&sd_full[i], 1);
      mbar_init(&sd_free[i], 8);
      mbar_init(&ds_full[i], 8);
      mbar_init(&ds_free[i], 1);
    }
    mbar_init(dq_done, 1);
    mbar_init(dq_free, 8);
    mbar_init(mma_done, 1);
    mbar_init(dq_mma_done, 1);
    mbar_init(uc_empty, 2);
    mbar_init(uc_full, 1);
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
  // TMEM: S0 [0,64) S1 [64,128) dP0 [128,192) dP1 [192,256) dQ [256, 256+D)
  // dS 0/1 [384,416) [416,448): 16-bit pairs, the A operand of the dQ product
  const uint32_t tm_s0 = tmem, tm_dp0 = tmem + 128, tm_dq = tmem + 256, tm_ds = tmem + 384;

  if (warp == 8 || warp == 11) {
    // ------------------------------ producers -----------------------------
    // Warp 8 loads each item's Q / dO tiles and fills the union cache (the
    // two warps hand it over through uc_empty / uc_full); the warps then lay
    // out and load alternate chunks.  Dense modes: alternate chunks, one box
    // per operand.  A select-mode union too large for the cache is walked by
    // lane 0 of warp 8 alone.
    const int pw = warp == 8 ? 0 : 1;
    if (pw == 0) {
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_do);
      }
      if (lane < kNumBoxes) {
        tma_prefetch_desc(&kv.k[lane]);
        tma_prefetch_desc(&kv.v[lane]);
      }
    }
    UnionCache& uc = *reinterpret_cast<UnionCache*>(smem + L::OFF_UC);
    int Jbase = 0, it_n = 0, q_loads = 0, cache_uses = 0;
    int hist[STAGES];  // this warp's last STAGES issued chunks (teardown drain), newest first
#pragma unroll
    for (int k = 0; k < STAGES; ++k) hist[k] = -1;
    auto note_issued = [&](int J) {
#pragma unroll
      for (int k = STAGES - 1; k > 0; --k) hist[k] = hist[k - 1];
      hist[0] = J;
    };
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
      const Item w = item_of(i);
      const QTile& tile = w.tile;
      const int h = w.h, qb = it_n & 1;
      if (pw == 0) {
        if (!warp_wait(&qdo_empty[qb], ((it_n >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&qdo_full[qb], 2 * L::QTILE);
          tma_load_3d(sQ + qb * L::QTILE, &tm_q, 0, h * G, tile.q_start, &qdo_full[qb]);
          tma_load_3d(sDO + qb * L::QTILE, &tm_do, 0, h * G, tile.q_start, &qdo_full[qb]);
        }
        q_loads = it_n + 1;
      }
      const bool cached = MODE == kSelect && w.U <= kUnionCacheCap;
      if (cached) {
        const uint32_t par = cache_uses & 1;
        ++cache_uses;
        if (lane == 0) mbar_arrive(uc_empty);
        if (pw == 0) {
          if (!warp_wait(uc_empty, par, abort_flag, prm.err)) { ok = false; break; }
          union_cache_fill(uc, w.U, prm.union_blk, prm.union_mask, w.ubase, prm.cu_block_include_tokens, tile.kv_lo,
                           tile.kv_hi, prm.num_blocks, prm.err);
          __syncwarp();
          if (lane == 0) mbar_arrive(uc_full);
        } else {
          if (!warp_wait(uc_full, par, abort_flag, prm.err)) { ok = false; break; }
        }
        int ucur = 0;
        for (int j = pw; j < w.n_chunks; j += 2) {
          const int J = Jbase + j, s = J % STAGES;
          if (!warp_wait(&kv_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          DqMeta& mt = meta[s];
          const int r = union_cache_chunk<kDqGroups>(uc, j, mt.row0, mt.qmask, mt.colmask, ucur);
          __syncwarp();
          if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], 2 * L::KTILE);
          __syncwarp();
          issue_group_runs<kDqGroups, RB>(r, sK + s * L::KTILE, sV + s * L::KTILE, kv.k, kv.v, h, prm.total_k,
                                          &kv_full[s]);
          note_issued(J);
        }
      } else if (MODE != kSelect) {
        for (int j = pw; j < w.n_chunks; j += 2) {
          const int J = Jbase + j, s = J % STAGES;
          if (!warp_wait(&kv_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          if (lane == 0) {
            DqMeta& mt = meta[s];
            const int k0 = tile.kv_lo + j * kDqChunk;
            mt.kv_start = k0;
            mt.n_valid = min(kDqChunk, tile.kv_hi - k0);
            mbar_arrive_expect_tx(&kv_full[s], 2 * L::KTILE);
            tma_load_3d(sK + s * L::KTILE, &kv.k[3], 0, h, k0, &kv_full[s]);  // 64-row box
            tma_load_3d(sV + s * L::KTILE, &kv.v[3], 0, h, k0, &kv_full[s]);
          }
          note_issued(J);
        }
      } else if (pw == 0) {
        if (lane == 0) {
          int u = -1, tcur = 0, tend = 0;
          for (int j = 0; j < w.n_chunks; ++j) {
            const int J = Jbase + j, s = J % STAGES;
            if (!mbar_wait(&kv_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
            DqMeta& mt = meta[s];
            walk_union_groups<kDqGroups>(u, tcur, tend, w.U, prm.union_blk, prm.union_mask, w.ubase,
                                         prm.cu_block_include_tokens, tile.kv_lo, tile.kv_hi, mt.row0, mt.qmask,
                                         mt.colmask, prm.num_blocks, prm.err);
            mbar_arrive_expect_tx(&kv_full[s], 2 * L::KTILE);
            load_group_runs<kDqGroups, RB>(mt.row0, sK + s * L::KTILE, sV + s * L::KTILE, kv.k, kv.v, h, prm.total_k,
                                           &kv_full[s]);
            note_issued(J);
          }
        }
        ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
#pragma unroll
        for (int k = 0; k < STAGES; ++k) hist[k] = __shfl_sync(0xffffffffu, hist[k], 0);
      }
      Jbase += w.n_chunks;
    }
    // Teardown after an abort: let this warp's issued copies land before the CTA exits.
    if (lane == 0 && *abort_flag) {
      if (pw == 0)
        for (int k = max(0, q_loads - 2); k < q_loads; ++k) mbar_wait_drain(&qdo_full[k & 1], (k >> 1) & 1);
#pragma unroll
      for (int k = 0; k < STAGES; ++k)
        if (hist[k] >= 0) mbar_wait_drain(&kv_full[hist[k] % STAGES], (hist[k] / STAGES) & 1);
    }
    __syncwarp();
  } else if (warp == 9) {
    // --------------------------- MMA issuer: S, dP --------------------------
    // One thread issues S = Q K^T and dP = dO V^T of every chunk, warp 10 the
    // dQ accumulation (one issuing thread spends ~90 cycles per tcgen05.mma
    // in short bursts; two keep the tensor pipe busy).
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc(AB, 0, 0, 128, kDqChunk);
      bool ok = true;
      int J = 0, it_n = 0;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
        const int n_chunks = item_of(i).n_chunks, qb = it_n & 1;
        if (!mbar_wait(&qdo_full[qb], (it_n >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
        const uint32_t q_base = smem_u32(sQ + qb * L::QTILE), do_base = smem_u32(sDO + qb * L::QTILE);
        for (int j = 0; j < n_chunks; ++j, ++J) {
          const int s = J % STAGES, sb = J & 1;
          if (!mbar_wait(&kv_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
          if (!mbar_wait(&sd_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * L::KTILE), v_base = smem_u32(sV + s * L::KTILE);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            umma_f16(tm_s0 + sb * kDqChunk, make_sdesc(q_base + ks * 32, 16, 8 * RB, SWZ),
                     make_sdesc(k_base + ks * 32, 16, 8 * RB, SWZ), idesc_s, ks > 0);
          }
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            umma_f16(tm_dp0 + sb * kDqChunk, make_sdesc(do_base + ks * 32, 16, 8 * RB, SWZ),
                     make_sdesc(v_base + ks * 32, 16, 8 * RB, SWZ), idesc_s, ks > 0);
          }
          umma_commit(&sd_full[sb]);
        }
        if (!ok) break;
        umma_commit(&qdo_empty[qb]);  // Q / dO tiles free once the item's S and dP products are done
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------- MMA issuer: dQ += dS K -----------------------
    // The chunk's S / dP products are complete once its dS is written (the
    // compute warps read them first), so this thread's commit alone releases
    // the chunk's K / V stage.
    if (lane == 0) {
      const uint32_t idesc_dq = make_idesc(AB, 0, 1, 128, D);
      bool ok = true;
      int J = 0, it_n = 0;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it_n) {
        const int n_chunks = item_of(i).n_chunks;
        // the previous item's dQ accumulator must have been read out first
        if (!mbar_wait(dq_free, (it_n & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
        for (int j = 0; j < n_chunks; ++j, ++J) {
          const int pb = J & 1, s = J % STAGES;
          if (!mbar_wait(&ds_full[pb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * L::KTILE);
#pragma unroll
          for (int ks = 0; ks < kDqChunk / 16; ++ks) {
            const uint64_t db = make_sdesc(k_base + ks * 16 * RB, L::KTILE, 8 * RB, SWZ);
            umma_f16_ts(tm_dq, tm_ds + pb * 32 + ks * 8, db, idesc_dq, (j > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&ds_free[pb]);
          umma_commit(&kv_empty[s]);
        }
        if (!ok) break;
        umma_commit(dq_done);  // one completion per item
      }
      umma_commit(dq_mma_done);
      mbar_wait_drain(dq_mma_done, 0);
    }
    __syncwarp();
  } else {
    // warp w: rows 32*(w%4).., key columns 32*(w/4).. of each chunk
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int qloc = r / G;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = prm.scale_log2, scale = prm.scale;
    bool ok = true;
    int J = 0, it_n = 0;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++it_n) {
    const Item w = item_of(it);
    const QTile& tile = w.tile;
    const int n_chunks = w.n_chunks;
    const int hq = w.h * G + (r % G);
    const int qi = tile.q_start + qloc;
    const bool row_valid = qloc < tile.n_q;
    float lse2 = 0.f, delta = 0.f;
    if (row_valid) {
      lse2 = prm.lse[(size_t)hq * prm.total_q + qi];
      if (prm.lse_natural) lse2 *= 1.4426950408889634f;
      const size_t off = ((size_t)qi * prm.q_tok_stride + (size_t)hq * D);
      const uint4* orow = reinterpret_cast<const uint4*>(static_cast<const T*>(prm.out) + off);
      const uint4* grow = reinterpret_cast<const uint4*>(static_cast<const T*>(prm.dout) + off);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 a = orow[c], b = grow[c];
        const T* ae = reinterpret_cast<const T*>(&a);
        const T* be = reinterpret_cast<const T*>(&b);
#pragma unroll
        for (int e = 0; e < 8; ++e) delta = fmaf((float)ae[e], (float)be[e], delta);
      }
      if (half == 0) prm.delta[(size_t)hq * prm.total_q + qi] = delta;
    }
    for (int j = 0; j < n_chunks; ++j, ++J) {
      const int s = J % STAGES, sb = J & 1;
      if (!warp_wait(&sd_full[sb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
      if (!warp_wait(&kv_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      const DqMeta& mt = meta[s];
      uint32_t vm;  // valid columns of this warp's 32-column slice
      if constexpr (MODE == kSelect) {
        const int wq = qloc >> 5, b = qloc & 31;
        uint32_t e = 0u;
#pragma unroll
        for (int y = 0; y < 4; ++y)
          if ((mt.qmask[half * 4 + y][wq] >> b) & 1u) e |= 0xffu << (y * 8);
        vm = e & mt.colmask[half];
      } else {
        int lo = 0, hi = mt.n_valid;
        if constexpr (MODE == kBand) {
          lo = max(lo, qi - prm.half_window - mt.kv_start);
          hi = min(hi, qi + prm.half_window + 1 - mt.kv_start);
        }
        const int a = max(lo - 32 * half, 0), bnd = min(hi - 32 * half, 32);
        vm = 0u;
        if (bnd > a) vm = ((bnd - a) == 32 ? 0xffffffffu : ((1u << (bnd - a)) - 1u)) << a;
      }
      float sv[32], dp[32];
      tmem_ld32(tm_s0 + sb * kDqChunk + lane_base + half * 32, sv);
      tmem_ld32(tm_dp0 + sb * kDqChunk + lane_base + half * 32, dp);
      tmem_wait_ld();
      // S / dP of this chunk are in registers: release the TMEM buffers early
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sd_free[sb]);
      if (__all_sync(0xffffffffu, !row_valid || vm == 0xffffffffu)) {  // no masking needed
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p = ex2(fmaf(sv[c], sl2, -lse2));
          sv[c] = p * (dp[c] - delta) * scale;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const bool valid = (vm >> c) & 1u;
          const float p = ex2(fmaf(sv[c], sl2, -lse2));
          sv[c] = valid ? p * (dp[c] - delta) * scale : 0.f;
        }
      }
      // row r's 32 key columns of dS, 16-bit pairs, into this warp's TMEM
      // lanes (the dQ MMA reads them as operand A)
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) pk[c] = pack2<BF16>(sv[2 * c], sv[2 * c + 1]);
      if (!warp_wait(&ds_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      tmem_st16(tm_ds + sb * 32 + half * 16 + lane_base, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[sb]);
    }
    if (!ok) break;
    // warps of half 0 write dQ (every lane takes part in the warp-collective
    // TMEM load, only valid rows store); then all eight warps release the
    // accumulator for the next item
    if (!warp_wait(dq_done, it_n & 1, abort_flag, prm.err)) { ok = false; break; }
    if (half == 0) {
      tc_fence_after();
      uint8_t* drow = static_cast<uint8_t*>(prm.dq) + ((size_t)qi * prm.q_tok_stride + (size_t)hq * D) * 2;
      float v[D];
      if (n_chunks > 0) {
        tmem_load_cols<D>(tm_dq + lane_base, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int c = 0; c < D; ++c) v[c] = 0.f;
      }
      if (row_valid) {
#pragma unroll
        for (int c = 0; c < D; c += 8) {
          uint4 pk;
          pk.x = pack2<BF16>(v[c], v[c + 1]);
          pk.y = pack2<BF16>(v[c + 2], v[c + 3]);
          pk.z = pack2<BF16>(v[c + 4], v[c + 5]);
          pk.w = pack2<BF16>(v[c + 6], v[c + 7]);
          *reinterpret_cast<uint4*>(drow + c * 2) = pk;
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(dq_free);
    }  // items
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dK / dV
// ---------------------------------------------------------------------------

struct DkvParams {
  const QTile* kvtiles;
  const int* n_kvtiles;
  int kvtiles_ub;
  // select mode: reverse map
  const QTile* qtiles;
  const int* rev_off;
  const int2* rev_entries;
  const uint4* union_mask;
  int tiles_ub;
  int union_cap;
  int num_blocks;
  // query-side operands, gathered row by row with cp.async
  const void* q;
  const void* dout;
  long long q_tok_stride;
  // per-row statistics [Hq, Nq]
  const float* lse;
  const float* delta;
  void* dk;
  void* dv;
  float* partial;  // [split][hkv][kvtiles_ub][128][D] x 2 when n_split > 1
  int n_split;
  const int* kv_sched;  // select mode: work entries, heaviest first (items, then pieces of long items)
  const int* item_nch;  // select mode: query chunks of each work entry
  const int2* item_rng; // select mode: {first entry, entries} of the block's list; x < 0: item split
  const int* item_src;  // select mode: the item of each piece
  float* piece_partial; // select mode: [piece_slots][2][128][D] fp32 dK / dV of each piece
  const int4* split_items;  // select mode: {item, first slot, pieces, 0}
  const int* sched_ctr;     // select mode: [2] = number of split items
  int piece_slots;
  long long kv_tok_stride;
  int total_q;
  int total_k;
  int G;
  int hkv;
  float scale_log2;
  float scale;
  int half_window;
  int lse_natural;
  int* err;
};

struct KvMeta {
  float lse2[kKvQRows];
  float delta[kKvQRows];
  int qidx[kKvQRows];   // query token of each row (-1: padding)
  int qlist[kKvQRows];  // query tokens of the chunk (G rows each)
  int n_rows;
  int pad[3];
};

// The reverse map of one KV block in shared memory: the (query tile, union
// slot) entries that selected it, as the tile's first query token, the
// 128-bit mask of its queries and the exclusive prefix of the masks' bit
// counts, so the queries of any chunk are found without a sequential walk
// (capacity kRevCacheCap entries).

struct RevCache {
  int tq0[kRevCacheCap];
  int prefix[kRevCacheCap];  // queries before the entry
  int gstart[kRevCacheCap];  // query groups before the entry (G <= 8)
  int wmask[kRevCacheCap];   // the entry's non-empty query windows (16 bits)
  uint4 mask[kRevCacheCap];
  int n;       // entries of the segment held
  int total;   // queries
  int groups;  // query groups (G <= 8): 8 rows = 8/G queries of one window
  int pad;
};


// Position of the n-th (0-based) set bit of `word` (n < popc(word)).
__device__ __forceinline__ int nth_set_bit(uint32_t word, int n) {
  int pos = 0;
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const uint32_t low = word & ((1u << width) - 1u);
    const int c = __popc(low);
    if (n >= c) {
      n -= c;
      word >>= width;
      pos += width;
    } else {
      word = low;
    }
  }
  return pos;
}

template <int D, int STAGES>
struct DkvSmem {
  static constexpr int RB = 2 * D;
  static constexpr int KTILE = 128 * RB;
  static constexpr int QTILE = kKvQRows * RB;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = KTILE;
  static constexpr int OFF_Q = 2 * KTILE;
  static constexpr int OFF_DO = OFF_Q + STAGES * QTILE;
  static constexpr int OFF_META = OFF_DO + STAGES * QTILE;  // P^T / dS^T live in TMEM
  static constexpr int OFF_BAR = OFF_META + STAGES * (int)sizeof(KvMeta);
  // kv_full, kv_empty, q_full[S], q_empty[S], st_full[2], st_free[2], pds_full[2], pds_free[2],
  // acc_done, acc_free, mma_done, rc_empty, rc_full, acc_mma_done
  static constexpr int NBAR = 2 + 2 * STAGES + 8 + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_RC = (OFF_MISC + 32 + 15) / 16 * 16;  // select mode: the block's reverse map
  static constexpr int BYTES = OFF_RC + (int)sizeof(RevCache);
  static constexpr int ALLOC = (BYTES + 1024 > kOneCtaPerSmSmem) ? BYTES + 1024 : kOneCtaPerSmSmem;
  static_assert(ALLOC <= 227 * 1024, "shared memory budget");
};


// Threads of the dK/dV kernel: 8 compute warps (two per TMEM lane quarter,
// splitting the 64 query columns of a chunk), two producer warps and two
// MMA-issuing warps.
constexpr int kDkvThreads = 384;
constexpr int kDkvProducerWarp = 8;
constexpr int kDkvMmaWarp = 9;
constexpr int kDkvProducer2Warp = 10;  // select mode: gathers every other chunk
constexpr int kDkvAccWarp = 11;        // issues the dV / dK accumulation MMAs

// Warp-wide fill of the reverse cache with entries [e0, e0 + n) of kv head
// `h`'s reverse map (one segment of a block's list, n <= kRevCacheCap).
__device__ __forceinline__ void rev_cache_fill(RevCache& rc, const DkvParams& prm, int h, int e0, int n) {
  const int lane = threadIdx.x & 31;
  n = max(0, min(n, kRevCacheCap));
  const int2* ent = prm.rev_entries + (size_t)h * prm.tiles_ub * prm.union_cap;
  int carry = 0, gcarry = 0;
  for (int b0 = 0; b0 < n; b0 += 32) {
    const int i = b0 + lane;
    int cnt = 0, gcnt = 0;
    if (i < n) {
      const int2 x = ent[e0 + i];
      const bool good = dcheck((unsigned)x.x < (unsigned)prm.tiles_ub && (unsigned)x.y < (unsigned)prm.union_cap,
                               kDcRevEntry, prm.err);
      const uint4 m = good ? prm.union_mask[((size_t)h * prm.tiles_ub + x.x) * prm.union_cap + x.y]
                           : make_uint4(0u, 0u, 0u, 0u);
      rc.tq0[i] = good ? prm.qtiles[x.x].q_start : 0;
      rc.mask[i] = m;
      cnt = __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w);
      if (prm.G <= 8) {
        const uint32_t wm = window_mask(m, 8 / prm.G);
        rc.wmask[i] = (int)wm;
        gcnt = __popc(wm);
      }
    }
    int incl = cnt, gincl = gcnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o), gy = __shfl_up_sync(0xffffffffu, gincl, o);
      if (lane >= o) {
        incl += y;
        gincl += gy;
      }
    }
    if (i < n) {
      rc.prefix[i] = carry + incl - cnt;
      rc.gstart[i] = gcarry + gincl - gcnt;
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
    gcarry += __shfl_sync(0xffffffffu, gincl, 31);
  }
  if (lane == 0) {
    rc.n = n;
    rc.total = carry;
    rc.groups = gcarry;
  }
  __syncwarp();
}

// Queries c*qpc .. c*qpc+qpc-1 of the cached list into qlist (-1 past the
// end); returns how many are real.  Warp-wide.  cursor[k] (per lane, start
// at 0) keeps the entry of the lane's k-th slot between calls with
// increasing c: it only moves forward, so a short scan replaces a search.
__device__ __forceinline__ int rev_cache_chunk(const RevCache& rc, int c, int qpc, int* qlist, int* cursor) {
  const int lane = threadIdx.x & 31;
  const int base = c * qpc;
  const int n = max(0, min(qpc, rc.total - base));
#pragma unroll
  for (int k = 0; k < kKvQRows / 32; ++k) {
    const int i = lane + 32 * k;
    if (i >= qpc) break;
    int q = -1;
    if (i < n) {
      const int t = base + i;
      int lo = cursor[k];  // last entry with prefix <= t (entries with no query never are)
      while (lo + 1 < rc.n && rc.prefix[lo + 1] <= t) ++lo;
      cursor[k] = lo;
      int rank = t - rc.prefix[lo];
      const uint4 m = rc.mask[lo];
      int w = 0;
      uint32_t word = m.x;
      int cw = __popc(m.x);
      if (rank >= cw) {
        rank -= cw;
        w = 1;
        word = m.y;
        cw = __popc(m.y);
        if (rank >= cw) {
          rank -= cw;
          w = 2;
          word = m.z;
          cw = __popc(m.z);
          if (rank >= cw) {
            rank -= cw;
            w = 3;
            word = m.w;
          }
        }
      }
      q = rc.tq0[lo] + 32 * w + nth_set_bit(word, rank);
    }
    qlist[i] = q;
  }
  return n;
}

// Query-window boxes of the select-mode producer: box heights 8 << i rows
// ((8/G) << i tokens of G heads), i = 0..3.
struct QMaps {
  CUtensorMap q[4];
  CUtensorMap dout[4];
};

template <int D, bool BF16, int MODE, int STAGES>
__global__ void __launch_bounds__(kDkvThreads, 1)
    attn_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ QMaps qm, const DkvParams prm) {
  using L = DkvSmem<D, STAGES>;
  constexpr int RB = L::RB;
  constexpr uint64_t SWZ = swz_for_row_bytes(RB);
  constexpr uint32_t AB = BF16 ? 1u : 0u;

  // Persistent CTAs walk the work items: select mode the heaviest-first
  // schedule (kv head, KV tile); dense modes (kv head, KV tile, query
  // split).  Every role decodes the same items in the same order; per-chunk
  // ring phases run on across items and the K/V tile, the reverse-map cache
  // and the dK/dV accumulators are handed from item to item by barriers, so
  // the next item's loads overlap the current item's tail.
  const int G = prm.G;
  const int qpc = kKvQRows / G;  // queries per chunk (gather path)
  const int n_items = prm.kv_sched ? prm.hkv * prm.kvtiles_ub + prm.piece_slots
                                   : prm.hkv * prm.kvtiles_ub * prm.n_split;
  const int n_kv = *prm.n_kvtiles;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  KvMeta* meta = reinterpret_cast<KvMeta*>(smem + L::OFF_META);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* q_full = bars + 2;
  uint64_t* q_empty = q_full + STAGES;
  uint64_t* st_full = q_empty + STAGES;
  uint64_t* st_free = st_full + 2;
  uint64_t* pds_full = st_free + 2;
  uint64_t* pds_free = pds_full + 2;
  uint64_t* acc_done = pds_free + 2;
  uint64_t* acc_free = acc_done + 1;
  uint64_t* mma_done = acc_free + 1;
  uint64_t* rc_empty = mma_done + 1;  // both producer warps are done with the cache (count 2)
  uint64_t* rc_full = rc_empty + 1;   // warp 8 has filled it for the next item (count 1)
  uint64_t* acc_mma_done = rc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  struct KvItem {
    QTile kt;
    int kt_idx, h, split, n_chunks, q_lo, q_hi;
    int slot, e_lo, e_cnt;  // select mode: piece slot (-1: the whole item) and its run of the list
    bool skip;
  };
  auto item_of = [&](int i) {
    KvItem it;
    it.split = 0;
    it.slot = -1;
    it.e_lo = it.e_cnt = 0;
    int sched_e = 0;
    if (prm.kv_sched) {
      const int n_whole = prm.hkv * prm.kvtiles_ub;
      sched_e = prm.kv_sched[i];
      int src = sched_e;
      if (!dcheck((unsigned)sched_e < (unsigned)(n_whole + prm.piece_slots), kDcKvTile, prm.err)) {
        it.skip = true;
        return it;
      }
      if (sched_e >= n_whole) {
        it.slot = sched_e - n_whole;
        src = prm.item_src[it.slot];
      }
      const int2 rg = prm.item_rng[sched_e];
      if (rg.x < 0 || !dcheck((unsigned)src < (unsigned)n_whole, kDcKvTile, prm.err)) {  // split, or unused
        it.skip = true;
        return it;
      }
      it.e_lo = rg.x;
      it.e_cnt = rg.y;
      it.h = src / prm.kvtiles_ub;
      it.kt_idx = src - it.h * prm.kvtiles_ub;
    } else {
      const int per_h = prm.kvtiles_ub * prm.n_split;
      it.h = i / per_h;
      const int rem = i - it.h * per_h;
      it.kt_idx = rem / prm.n_split;
      it.split = rem - it.kt_idx * prm.n_split;
    }
    it.skip = it.kt_idx >= n_kv;
    it.n_chunks = 0;
    it.q_lo = it.q_hi = 0;
    if (it.skip) return it;
    it.kt = prm.kvtiles[it.kt_idx];  // rows = keys [q_start, q_start + n_q)
    it.q_lo = it.kt.kv_lo;
    it.q_hi = it.kt.kv_hi;
    if (!dcheck(it.kt.q_start >= 0 && it.kt.n_q >= 0 && it.kt.n_q <= 128 && it.kt.q_start + it.kt.n_q <= prm.total_k &&
                    (MODE != kSelect || (unsigned)it.kt.seg < (unsigned)prm.num_blocks),
                kDcKvTile, prm.err)) {
      it.skip = true;
      return it;
    }
    if constexpr (MODE == kSelect) {
      it.n_chunks = prm.item_nch[sched_e];
      if (!dcheck(it.n_chunks >= 0, kDcChunks, prm.err)) it.n_chunks = 0;
    } else {
      const int nq = max(it.q_hi - it.q_lo, 0);
      const int per = ((nq + prm.n_split - 1) / prm.n_split + qpc - 1) / qpc * qpc;
      it.q_lo = min(it.kt.kv_lo + it.split * per, it.kt.kv_hi);
      it.q_hi = min(it.q_lo + per, it.kt.kv_hi);
      it.n_chunks = (max(it.q_hi - it.q_lo, 0) + qpc - 1) / qpc;
    }
    return it;
  };

  // round k of the walk: items in snake order (k odd: reversed), so a CTA
  // that drew a heavy item of the heaviest-first list draws a light one next
  // (select mode; the dense modes' items are uniform and walk in order)
  auto item_at = [&](int k) {
    const bool rev = prm.kv_sched && (k & 1);
    return k * (int)gridDim.x + (rev ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
  };

  RevCache& rc = *reinterpret_cast<RevCache*>(smem + L::OFF_RC);
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st_full[i], 1);
      mbar_init(&st_free[i], 8);
      mbar_init(&pds_full[i], 8);
      mbar_init(&pds_free[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(acc_free, 8);
    mbar_init(mma_done, 1);
    mbar_init(rc_empty, 2);
    mbar_init(rc_full, 1);
    mbar_init(acc_mma_done, 1);
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
  const int lg_g = __ffs(G) - 1;  // G is a power of two
  // TMEM: St0 [0,64) St1 [64,128) dPt0 [128,192) dPt1 [192,256) dK [256,256+D) dV [256+D, 256+2D)
  // P^T 0/1 [384,416) [416,448), dS^T 0/1 [448,480) [480,512): 16-bit pairs, the A operand of dV / dK
  const uint32_t tm_st0 = tmem, tm_dpt0 = tmem + 128, tm_dk = tmem + 256, tm_dv = tmem + 256 + D;
  const uint32_t tm_pt = tmem + 384, tm_dst = tmem + 448;

  if (warp == kDkvProducerWarp || warp == kDkvProducer2Warp) {
    // ------------------------------ producers -----------------------------
    // Per item: warp 8 loads the K/V tile once the previous item's S^T /
    // dP^T products are done and, in select mode, fills the reverse-map cache
    // with each segment of the block's list in turn (both producer warps meet
    // at barriers before and after every fill, the cache being shared).
    // Query rows: select mode with G <= 8 in 8-row windows by TMA (grouped),
    // G > 8 gathered with 16-byte cp.async from the cache; dense modes one
    // TMA box per operand.  The two warps take alternate chunks and publish a
    // chunk as soon as its copies have landed.
    const int pw = warp == kDkvProducerWarp ? 0 : 1;
    if (MODE == kSelect && lane < 4) {
      tma_prefetch_desc(&qm.q[lane]);
      tma_prefetch_desc(&qm.dout[lane]);
    }
    constexpr int CPR = RB / 16;  // 16-byte chunks per row
    const uint8_t* qbase = static_cast<const uint8_t*>(prm.q);
    const uint8_t* dobase = static_cast<const uint8_t*>(prm.dout);
    const int W = G <= 8 ? 8 / G : 1;  // queries per 8-row window
    int Jbase = 0, it_n = 0, kv_loads = 0, cache_uses = 0;
    int last_issued_J = -1;             // this warp's last issued chunk (global index), for teardown
    bool ok = true;
    for (int rnd = 0, i = item_at(0); i < n_items && ok; i = item_at(++rnd)) {
      const KvItem w = item_of(i);
      if (w.skip) continue;
      const int h = w.h;
      const QTile& kt = w.kt;
      const int n_chunks = w.n_chunks;
      // Select mode: the block's reverse list streams through the shared-memory
      // cache in segments of at most kRevCacheCap entries.  Per segment both
      // warps release the cache, warp 8 refills it, and the segment's chunks
      // are produced (the warps alternate); the last segment pads up to the
      // item's scheduled chunk count.  Dense modes: one segment, no cache.
      int e_first = 0, e_count = 0;
      if constexpr (MODE == kSelect) {
        const int* off = prm.rev_off + (size_t)h * (prm.num_blocks + 1);
        e_first = off[kt.seg];
        e_count = off[kt.seg + 1] - e_first;
        if (w.slot >= 0) {  // a piece: its run of the list
          if (!dcheck(w.e_lo >= 0 && w.e_cnt >= 0 && w.e_lo + w.e_cnt <= e_count, kDcRevRange, prm.err))
            e_count = 0;
          else {
            e_first += w.e_lo;
            e_count = w.e_cnt;
          }
        }
        if (!dcheck(e_first >= 0 && e_count >= 0 &&
                        (long long)e_first + e_count <= (long long)prm.tiles_ub * prm.union_cap,
                    kDcRevRange, prm.err))
          e_first = e_count = 0;
      }
      const int n_seg = MODE == kSelect ? (e_count + kRevCacheCap - 1) / kRevCacheCap : 1;
      const bool have_rc = MODE == kSelect && n_seg > 0;
      const bool grouped = MODE == kSelect && G <= 8;
      auto publish = [&](int ci) {  // ci: chunk index within the item
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[(Jbase + ci) % STAGES]);
      };
      int cbase = 0;  // the current segment's first chunk within the item
      for (int sg = 0; sg < (n_seg > 0 ? n_seg : 1) && ok; ++sg) {
        if (have_rc) {
          const uint32_t par = cache_uses & 1;
          ++cache_uses;
          if (lane == 0) mbar_arrive(rc_empty);
          if (pw == 0) {
            if (!warp_wait(rc_empty, par, abort_flag, prm.err)) { ok = false; break; }
            rev_cache_fill(rc, prm, h, e_first + sg * kRevCacheCap, min(kRevCacheCap, e_count - sg * kRevCacheCap));
            __syncwarp();
            if (lane == 0) mbar_arrive(rc_full);
          } else {
            if (!warp_wait(rc_full, par, abort_flag, prm.err)) { ok = false; break; }
          }
        }
        if (sg == 0 && pw == 0) {
          if (!warp_wait(kv_empty, (it_n & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(kv_full, 2 * L::KTILE);
            tma_load_3d(sK, &tm_k, 0, h, kt.q_start, kv_full);
            tma_load_3d(sV, &tm_v, 0, h, kt.q_start, kv_full);
          }
          kv_loads = it_n + 1;
        }
        const int rc_n = have_rc ? rc.n : 0, rc_groups = have_rc ? rc.groups : 0;
        const int own = !have_rc ? 0 : grouped ? (rc_groups + 7) / 8 : (rc.total + qpc - 1) / qpc;
        int nch = max(n_chunks - cbase, 0);  // the last segment pads up to the scheduled count
        if (sg + 1 < n_seg) nch = min(own, nch);
        else if (own > nch && lane == 0 && pw == 0) atomicOr(prm.err, LSRM_ERR_CAPACITY);  // plan disagrees
        int issued = 0, published = 0;  // in this warp's own chunk sequence of this segment
        int rcur[kKvQRows / 32] = {};   // reverse-cache cursors of this lane
        // grouped path: this lane's current cache entry (index, first group,
        // next entry's first group, windows, first query, query mask)
        int e_lo = -1, e_gs = 0, e_gnext = 0, e_tq0 = 0;
        uint32_t e_wm = 0u;
        uint4 e_mask = make_uint4(0u, 0u, 0u, 0u);
        for (int cl = pw; cl < nch; cl += 2) {
          const int ci = cbase + cl;  // chunk within the item
          const int J = Jbase + ci;
          const int s = J % STAGES;
          if (!warp_wait(&q_empty[s], ((J / STAGES) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          last_issued_J = J;
          KvMeta& mt = meta[s];
          if (grouped) {
            // 8 groups of 8 rows: lane g < 8 finds its group's window; each
            // group lands by TMA at an 8-row boundary (boxes of whole windows,
            // merged when adjacent); rows whose query did not select the block
            // get lse = +inf, so their P and dS are exactly zero
            int tok = -1;
            uint32_t bits = 0u;
            if (lane < 8) {
              const int gg = 8 * cl + lane;
              if (gg < rc_groups) {
                // the lane's entry only moves forward: step over gstart alone,
                // then fetch the entry's fields once (shared-memory loads are
                // slow while the tensor pipe streams its operands)
                bool moved = false;
                while (e_gnext <= gg) {
                  ++e_lo;
                  e_gs = e_gnext;
                  e_gnext = e_lo + 1 < rc_n ? rc.gstart[e_lo + 1] : INT_MAX;
                  moved = true;
                }
                if (moved) {
                  e_wm = (uint32_t)rc.wmask[e_lo];
                  e_tq0 = rc.tq0[e_lo];
                  e_mask = rc.mask[e_lo];
                }
                const int wdx = nth_set_bit(e_wm, gg - e_gs);
                tok = e_tq0 + wdx * W;
                bits = window_bits(e_mask, wdx, W);
              }
            }
#pragma unroll
            for (int k = 0; k < kKvQRows / 32; ++k) {
              const int row = lane + 32 * k, grp = row >> 3, rr = row & 7;
              const int t = __shfl_sync(0xffffffffu, tok, grp);
              const uint32_t bb = __shfl_sync(0xffffffffu, bits, grp);
              const int qq = rr >> lg_g, g = rr & (G - 1);
              const bool valid = t >= 0 && ((bb >> qq) & 1u) && dcheck(t + qq < prm.total_q, kDcQRow, prm.err);
              mt.qidx[row] = valid ? t + qq : -1;
              if (valid) {
                const size_t si = (size_t)(h * G + g) * prm.total_q + (t + qq);
                cp_async_4(smem_u32(&mt.lse2[row]), prm.lse + si);
                cp_async_4(smem_u32(&mt.delta[row]), prm.delta + si);
              } else {
                mt.lse2[row] = INFINITY;
                mt.delta[row] = 0.f;
              }
            }
            if (lane == 0) {
              mt.n_rows = kKvQRows;
              mbar_expect_tx(&q_full[s], 2 * L::QTILE);
            }
            __syncwarp();
            issue_group_runs<8, RB>(tok, sQ + s * L::QTILE, sDO + s * L::QTILE, qm.q, qm.dout, h * G, prm.total_q,
                                    &q_full[s], W);
          } else {
            int n = 0;
            if constexpr (MODE == kSelect) {
              if (have_rc) {
                n = rev_cache_chunk(rc, cl, qpc, mt.qlist, rcur);
              } else {  // an empty list: padding chunks only
                for (int i2 = lane; i2 < qpc; i2 += 32) mt.qlist[i2] = -1;
              }
            } else {
              const int q0 = w.q_lo + ci * qpc;
              n = max(0, min(qpc, w.q_hi - q0));
              for (int i2 = lane; i2 < qpc; i2 += 32) mt.qlist[i2] = i2 < n ? q0 + i2 : -1;
            }
            if (lane == 0) mt.n_rows = n * G;
            __syncwarp();
            for (int row = lane; row < kKvQRows; row += 32) {
              int q = mt.qlist[row >> lg_g];
              const int g = row & (G - 1);
              if (q >= 0 && !dcheck(q < prm.total_q, kDcQRow, prm.err)) q = -1;
              mt.qidx[row] = q;
              if (q >= 0) {
                const size_t si = (size_t)(h * G + g) * prm.total_q + q;
                cp_async_4(smem_u32(&mt.lse2[row]), prm.lse + si);
                cp_async_4(smem_u32(&mt.delta[row]), prm.delta + si);
              } else {
                mt.lse2[row] = 0.f;
                mt.delta[row] = 0.f;
              }
            }
            __syncwarp();
            const uint32_t dq_s = smem_u32(sQ + s * L::QTILE), ddo_s = smem_u32(sDO + s * L::QTILE);
            if constexpr (MODE != kSelect) {
              // contiguous queries: one TMA box per operand; rows past the range are
              // other tokens' data (finite, masked) or zero fill past the tensor
              if (lane == 0) {
                const int q0 = w.q_lo + ci * qpc;
                mbar_expect_tx(&q_full[s], 2 * L::QTILE);
                tma_load_3d(sQ + s * L::QTILE, &tm_q, 0, h * G, q0, &q_full[s]);
                tma_load_3d(sDO + s * L::QTILE, &tm_do, 0, h * G, q0, &q_full[s]);
              }
            } else {
              // lane: 16-byte column j of rows r0, r0 + 32/CPR, ...; the head and
              // column offsets are folded into the lane's base pointers
              const int j = lane % CPR, r0 = lane / CPR;
              const uint8_t* qb = qbase + ((size_t)h * G * D) * 2 + (size_t)j * 16;
              const uint8_t* db = dobase + ((size_t)h * G * D) * 2 + (size_t)j * 16;
              const size_t tok_bytes = (size_t)prm.q_tok_stride * 2;
#pragma unroll
              for (int row = r0; row < kKvQRows; row += 32 / CPR) {
                const int q = mt.qidx[row];
                const uint32_t o = swz_offset<RB>(row, j);
                if (q >= 0) {
                  const size_t off2 = (size_t)q * tok_bytes + (size_t)(row & (G - 1)) * (D * 2);
                  cp_async_16(dq_s + o, qb + off2);
                  cp_async_16(ddo_s + o, db + off2);
                } else {  // padding rows: zeros, so P^T dO and dS^T Q add nothing
                  st_shared_v4(dq_s + o, 0u, 0u, 0u, 0u);
                  st_shared_v4(ddo_s + o, 0u, 0u, 0u, 0u);
                }
              }
            }
          }
          cp_async_commit();
          ++issued;
          cp_async_wait<0>();
          publish(cbase + pw + 2 * published);
          ++published;
        }
        cp_async_wait<0>();
        for (; published < issued; ++published) publish(cbase + pw + 2 * published);
        cbase += nch;
      }
      Jbase += n_chunks;
      ++it_n;
    }
    if (lane == 0 && *abort_flag) {
      if (pw == 0 && kv_loads > 0) mbar_wait_drain(kv_full, (kv_loads - 1) & 1);
      if (last_issued_J >= 0) mbar_wait_drain(&q_full[last_issued_J % STAGES], (last_issued_J / STAGES) & 1);
    }
    __syncwarp();
  } else if (warp == kDkvMmaWarp) {
    // --------------------------- MMA issuer: S^T, dP^T ----------------------
    // Two threads issue the tensor-core work: this one S^T = K Q^T and
    // dP^T = V dO^T of every chunk, warp 11 the dV / dK accumulation.  One
    // issuing thread spends ~90 cycles per tcgen05.mma in bursts of 8; two
    // keep the pipe near its operand-read rate (~56 cycles per 128x64x16).
    if (lane == 0) {
      const uint32_t idesc_st = make_idesc(AB, 0, 0, 128, kKvQRows);
      bool ok = true;
      int Jbase = 0, it_n = 0;
      for (int rnd = 0, i = item_at(0); i < n_items && ok; i = item_at(++rnd)) {
        const KvItem w = item_of(i);
        if (w.skip) continue;
        const int n_chunks = w.n_chunks;
        if (!mbar_wait(kv_full, it_n & 1, abort_flag, prm.err)) { ok = false; break; }
        for (int c = 0; c < n_chunks; ++c) {
          const int J = Jbase + c;
          const int s = J % STAGES, sb = J & 1;
          if (!mbar_wait(&q_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
          if (!mbar_wait(&st_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t kb = smem_u32(sK), vb = smem_u32(sV);
          const uint32_t qb = smem_u32(sQ + s * L::QTILE), dob = smem_u32(sDO + s * L::QTILE);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_f16(tm_st0 + sb * kKvQRows, make_sdesc(kb + ks * 32, 16, 8 * RB, SWZ),
                     make_sdesc(qb + ks * 32, 16, 8 * RB, SWZ), idesc_st, ks > 0);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_f16(tm_dpt0 + sb * kKvQRows, make_sdesc(vb + ks * 32, 16, 8 * RB, SWZ),
                     make_sdesc(dob + ks * 32, 16, 8 * RB, SWZ), idesc_st, ks > 0);
          umma_commit(&st_full[sb]);
        }
        if (!ok) break;
        umma_commit(kv_empty);  // K / V are free once the item's S^T and dP^T products are done
        Jbase += n_chunks;
        ++it_n;
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
    __syncwarp();
  } else if (warp == kDkvAccWarp) {
    // ------------------------ MMA issuer: dV, dK ----------------------------
    // dV += P^T dO, dK += dS^T Q of each chunk once the compute warps have
    // written P^T / dS^T.  The chunk's S^T / dP^T products are complete by
    // then (the compute warps read them first), so this thread's commit
    // alone releases the chunk's Q / dO stage.
    if (lane == 0) {
      const uint32_t idesc_acc = make_idesc(AB, 0, 1, 128, D);
      bool ok = true;
      int Jbase = 0, it_n = 0;
      for (int rnd = 0, i = item_at(0); i < n_items && ok; i = item_at(++rnd)) {
        const KvItem w = item_of(i);
        if (w.skip) continue;
        const int n_chunks = w.n_chunks;
        // the previous item's accumulators must have been read out first
        if (!mbar_wait(acc_free, (it_n & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
        for (int c = 0; c < n_chunks; ++c) {
          const int J = Jbase + c;
          const int pb = J & 1, s = J % STAGES;
          const uint32_t accum0 = c > 0 ? 1u : 0u;
          if (!mbar_wait(&pds_full[pb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qb = smem_u32(sQ + s * L::QTILE), dob = smem_u32(sDO + s * L::QTILE);
#pragma unroll
          for (int ks = 0; ks < kKvQRows / 16; ++ks)
            umma_f16_ts(tm_dv, tm_pt + pb * 32 + ks * 8, make_sdesc(dob + ks * 16 * RB, L::QTILE, 8 * RB, SWZ),
                        idesc_acc, ks > 0 ? 1u : accum0);
#pragma unroll
          for (int ks = 0; ks < kKvQRows / 16; ++ks)
            umma_f16_ts(tm_dk, tm_dst + pb * 32 + ks * 8, make_sdesc(qb + ks * 16 * RB, L::QTILE, 8 * RB, SWZ),
                        idesc_acc, ks > 0 ? 1u : accum0);
          umma_commit(&pds_free[pb]);
          umma_commit(&q_empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_done);  // one completion per item
        Jbase += n_chunks;
        ++it_n;
      }
      umma_commit(acc_mma_done);
      mbar_wait_drain(acc_mma_done, 0);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------ P^T / dS^T -----------------------------
    // warp w: key rows 32*(w%4).., query columns 32*(w/4).. of each chunk
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // key row
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = prm.scale_log2, scale = prm.scale;
    const float lse_mul = prm.lse_natural ? 1.4426950408889634f : 1.f;
    bool ok = true;
    int Jbase = 0, it_n = 0;
    for (int rnd = 0, it = item_at(0); it < n_items && ok; it = item_at(++rnd)) {
    const KvItem w = item_of(it);
    if (w.skip) continue;
    const QTile& kt = w.kt;
    const int n_chunks = w.n_chunks, h = w.h, split = w.split, kt_idx = w.kt_idx;
    const bool row_valid = r < kt.n_q;
    const int kidx = kt.q_start + r;
    for (int c = 0; c < n_chunks; ++c) {
      const int J = Jbase + c;
      const int s = J % STAGES, sb = J & 1;
      if (!warp_wait(&st_full[sb], (J >> 1) & 1, abort_flag, prm.err)) { ok = false; break; }
      if (!warp_wait(&q_full[s], (J / STAGES) & 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      const KvMeta& mt = meta[s];
      const int n_rows = mt.n_rows;
      float st[32], dpt[32];
      tmem_ld32(tm_st0 + sb * kKvQRows + lane_base + half * 32, st);
      tmem_ld32(tm_dpt0 + sb * kKvQRows + lane_base + half * 32, dpt);
      tmem_wait_ld();
      // S^T / dP^T of this chunk are in registers: release the TMEM buffer early
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st_free[sb]);
      float lse_c[32], dl_c[32];
#pragma unroll
      for (int v4 = 0; v4 < 8; ++v4) {  // per-column statistics, 16-byte broadcast loads
        const float4 a = *reinterpret_cast<const float4*>(&mt.lse2[half * 32 + v4 * 4]);
        const float4 b = *reinterpret_cast<const float4*>(&mt.delta[half * 32 + v4 * 4]);
        lse_c[v4 * 4 + 0] = a.x * lse_mul;
        lse_c[v4 * 4 + 1] = a.y * lse_mul;
        lse_c[v4 * 4 + 2] = a.z * lse_mul;
        lse_c[v4 * 4 + 3] = a.w * lse_mul;
        dl_c[v4 * 4 + 0] = b.x;
        dl_c[v4 * 4 + 1] = b.y;
        dl_c[v4 * 4 + 2] = b.z;
        dl_c[v4 * 4 + 3] = b.w;
      }
      // Select mode needs no mask: padding columns hold zero Q / dO rows with
      // zero LSE and delta, so P^T dO and dS^T Q get nothing from them, and
      // key rows past the tile are never stored.  Range mode: full chunks
      // need none either.
      if (MODE == kSelect || (MODE == kRange && n_rows >= half * 32 + 32)) {
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const float p = ex2(fmaf(st[cc], sl2, -lse_c[cc]));
          st[cc] = p;
          dpt[cc] = p * (dpt[cc] - dl_c[cc]) * scale;
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const int col = half * 32 + cc;
          bool valid = row_valid && col < n_rows;
          if constexpr (MODE == kBand) valid = valid && abs(mt.qidx[col] - kidx) <= prm.half_window;
          // unconditional ex2, then select: a conditional asm call becomes a branch per element
          const float e = ex2(fmaf(st[cc], sl2, -lse_c[cc]));
          const float p = valid ? e : 0.f;
          st[cc] = p;
          dpt[cc] = valid ? p * (dpt[cc] - dl_c[cc]) * scale : 0.f;
        }
      }
      // key row r's 32 query columns of P^T and dS^T, 16-bit pairs, into
      // this warp's TMEM lanes (the dV / dK MMAs read them as operand A)
      uint32_t pk[16], dk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        pk[j] = pack2<BF16>(st[2 * j], st[2 * j + 1]);
        dk[j] = pack2<BF16>(dpt[2 * j], dpt[2 * j + 1]);
      }
      if (!warp_wait(&pds_free[sb], ((J >> 1) & 1) ^ 1, abort_flag, prm.err)) { ok = false; break; }
      tc_fence_after();
      tmem_st16(tm_pt + sb * 32 + half * 16 + lane_base, pk);
      tmem_st16(tm_dst + sb * 32 + half * 16 + lane_base, dk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pds_full[sb]);
    }
    if (!ok) break;
    // epilogue: warps of half 0 write dK, of half 1 write dV (key row r);
    // then all eight warps hand the accumulators to the next item
    if (!warp_wait(acc_done, it_n & 1, abort_flag, prm.err)) { ok = false; break; }
    {
      tc_fence_after();
      const int which = half;
      const uint32_t tm_acc = which == 0 ? tm_dk : tm_dv;
      float v[D];
      if (n_chunks > 0) {
        tmem_load_cols<D>(tm_acc + lane_base, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int cc = 0; cc < D; ++cc) v[cc] = 0.f;
      }
      if (row_valid && dcheck(kidx < prm.total_k, kDcKvOut, prm.err)) {
        if (MODE == kSelect && w.slot >= 0) {  // a piece: fp32 into its slot, summed after the launch
          float* dst_p = prm.piece_partial + (((size_t)w.slot * 2 + which) * 128 + r) * D;
#pragma unroll
          for (int cc = 0; cc < D; cc += 4)
            *reinterpret_cast<float4*>(dst_p + cc) = make_float4(v[cc], v[cc + 1], v[cc + 2], v[cc + 3]);
        } else if (prm.n_split > 1) {
          float* dst_p = prm.partial +
                         ((((size_t)which * prm.n_split + split) * prm.hkv + h) * prm.kvtiles_ub + kt_idx) * 128 * D +
                         (size_t)r * D;
#pragma unroll
          for (int cc = 0; cc < D; cc += 4)
            *reinterpret_cast<float4*>(dst_p + cc) = make_float4(v[cc], v[cc + 1], v[cc + 2], v[cc + 3]);
        } else {
          uint8_t* drow = static_cast<uint8_t*>(which == 0 ? prm.dk : prm.dv) +
                          ((size_t)kidx * prm.kv_tok_stride + (size_t)h * D) * 2;
#pragma unroll
          for (int cc = 0; cc < D; cc += 8) {
            uint4 pk;
            pk.x = pack2<BF16>(v[cc], v[cc + 1]);
            pk.y = pack2<BF16>(v[cc + 2], v[cc + 3]);
            pk.z = pack2<BF16>(v[cc + 4], v[cc + 5]);
            pk.w = pack2<BF16>(v[cc + 6], v[cc + 7]);
            *reinterpret_cast<uint4*>(drow + cc * 2) = pk;
          }
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(acc_free);
    Jbase += n_chunks;
    ++it_n;
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
