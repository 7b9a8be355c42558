// Device primitives for the sm_100a kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (UMMA + TMEM) wrappers and shared-memory matrix
// descriptors.  Everything here is inline PTX written for this library.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "lsrm_sparse.h"

namespace lsrm {

// ---------------------------------------------------------------------------
// Error word shared by the kernels of one call (device memory, host reads it
// back only when asked).  Bits are the LSRM_ERR_* codes of lsrm_sparse.h.
// ---------------------------------------------------------------------------

// Every spin-wait gives up after this many nanoseconds (globaltimer), sets the
// error word and makes the CTA tear down cleanly.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Device-side index checks, compiled in with -DLSRM_DEVICE_CHECKS (build.py
// --device-checks): a data-dependent index is tested before use; a failed
// test sets LSRM_ERR_BAD_INDEX plus the site's bit (1 << (8 + site)) in the
// error word and the access is skipped.  Release builds compile every check
// to `true`.
enum DcheckSite : int {
  kDcUnion = 0,     // union size above its capacity, or a union block id out of range
  kDcQTile = 1,     // a query tile outside the query tensor
  kDcKvRow = 2,     // a key group row outside the key tensor
  kDcOutRow = 3,    // an output / dQ row outside the query tensor
  kDcRevRange = 4,  // a reverse-list range outside the entry array
  kDcRevEntry = 5,  // a reverse entry (tile, union slot) out of range
  kDcQRow = 6,      // a dK/dV query row outside the query tensor
  kDcKvOut = 7,     // a dK/dV key row outside the key tensor
  kDcSelRow = 8,    // a selection row out of range (union builder)
  kDcRevFill = 9,   // a reverse-map fill position out of range
  kDcKvTile = 10,   // a dK/dV tile whose block or rows are out of range
  kDcChunks = 11,   // a work item's chunk count out of range
};

#ifdef LSRM_DEVICE_CHECKS
__device__ __forceinline__ bool dcheck(bool ok, int site, int* err) {
  if (!ok && err) atomicOr(err, LSRM_ERR_BAD_INDEX | (1 << (8 + site)));
  return ok;
}
#else
__device__ __forceinline__ bool dcheck(bool, int, int*) { return true; }
#endif

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ----------------------------- mbarrier ------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Adds transaction bytes to the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false when
// the CTA-wide abort flag is raised or the time limit passes (which raises the
// flag and records LSRM_ERR_TIMEOUT in the error word).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  uint32_t spins = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((++spins & 63u) == 0) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, LSRM_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Teardown wait (ignores the abort flag): lets copies or MMAs already in
// flight finish before the CTA exits; gives up after 200 ms.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_test(bar, parity)) {
    if (globaltimer() - t0 > 200000000ull) return false;
  }
  return true;
}

// Warp-uniform wait: every lane polls, the warp proceeds only if all lanes
// saw the phase complete (so warp-collective instructions that follow never
// run with lanes diverged on an abort path).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err));
}

// ------------------------------- TMA ----------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled load (no multicast) into this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------ tcgen05 -------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/fp16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B with A (M = 128 rows x K = 16, K-major) read from TMEM: row m
// in lane m, the 16-bit elements k = 2j, 2j+1 packed in column a_tmem + j
// (low half first); B from shared memory as in umma_f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread i of the warp gets lane (base+i),
// columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}

// This warp's 32 lanes x 16 consecutive 32-bit TMEM columns from v[0..16)
// (thread i writes lane base+i); complete with tmem_wait_st().
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------- UMMA descriptors ------------------------------------

// Swizzle codes of the sm_100 shared-memory matrix descriptor (bits 61-63).
enum : uint64_t { kSwNone = 0, kSw128 = 2, kSw64 = 4, kSw32 = 6 };

// Shared-memory matrix descriptor: start address, leading/stride byte
// offsets (16-byte units), descriptor version 1 (bit 46), swizzle mode.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint64_t swz) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= swz << 61;
  return d;
}

// Instruction descriptor for kind::f16: fp32 accumulate, A/B element type
// (0 = fp16, 1 = bf16), A/B major (0 = K-major, 1 = MN-major), M, N.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_type, uint32_t a_mn_major, uint32_t b_mn_major,
                                                  uint32_t M, uint32_t N) {
  return (1u << 4) | (ab_type << 7) | (ab_type << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Dynamic shared memory requested by every kernel that allocates all 512
// TMEM columns: more than half of an SM's 228 KB, so one CTA per SM.
constexpr int kOneCtaPerSmSmem = 116 * 1024;

// Swizzle mode matching a row of RB bytes (TMA box inner extent).
__host__ __device__ constexpr uint64_t swz_for_row_bytes(int RB) {
  return RB == 128 ? kSw128 : (RB == 64 ? kSw64 : kSw32);
}

// Loads N (8, 16 or a multiple of 32) consecutive fp32 TMEM columns of this
// warp's 32 lanes into v[0..N).
template <int N>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float* v) {
  if constexpr (N == 8) {
    tmem_ld8(taddr, v);
  } else if constexpr (N == 16) {
    tmem_ld16(taddr, v);
  } else {
#pragma unroll
    for (int c = 0; c < N; c += 32) tmem_ld32(taddr + c, v + c);
  }
}

// Byte offset of the 16-byte chunk `chunk` of row `row` inside a tile whose
// rows are `row_bytes` (= swizzle span: 128, 64 or 32) long, in the TMA /
// UMMA swizzled layout (XOR of the 16-byte chunk index with the row index
// inside the 8-row atom).
template <int ROW_BYTES>
__device__ __forceinline__ uint32_t swz_offset(int row, int chunk) {
  constexpr int kChunks = ROW_BYTES / 16;  // 8, 4 or 2
  if constexpr (kChunks == 8) {
    return row * ROW_BYTES + ((chunk ^ (row & 7)) << 4);
  } else if constexpr (kChunks == 4) {
    return row * ROW_BYTES + ((chunk ^ ((row >> 1) & 3)) << 4);
  } else {
    return row * ROW_BYTES + ((chunk ^ ((row >> 2) & 1)) << 4);
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) return pack_bf16(a, b);
  else return pack_f16(a, b);
}

__device__ __forceinline__ void st_shared_v4(uint32_t saddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Ampere-style asynchronous copies (global -> shared, through L2).
__device__ __forceinline__ void cp_async_16(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace lsrm

namespace lsrm {

// Loads the groups of a select-mode chunk: row0[g] is the first key token of
// 8-row group g (-1: unused, zero filled).  Runs of groups that are
// contiguous in memory are split into power-of-two boxes (8..128 rows) of the
// maps in `maps_k`/`maps_v` (box heights 8 << i).  Destinations stay aligned
// to 8 rows (the swizzle atom).
template <int NG, int RB>
__device__ __forceinline__ void load_group_runs(const int* row0, uint8_t* dK, uint8_t* dV, const CUtensorMap* maps_k,
                                                const CUtensorMap* maps_v, int h, int oob_row, uint64_t* bar) {
  int g = 0;
  while (g < NG) {
    const int r = row0[g];
    int n = 1;
    if (r >= 0) {
      while (g + n < NG && row0[g + n] == r + 8 * n) ++n;
    } else {
      while (g + n < NG && row0[g + n] < 0) ++n;
    }
    int done = 0;
    while (done < n) {
      const int rem = n - done;
      const int mi = 31 - __clz(rem);  // largest power of two <= rem
      const int piece = 1 << mi;
      const int row = r >= 0 ? r + 8 * done : oob_row;
      tma_load_3d(dK + (g + done) * 8 * RB, &maps_k[mi], 0, h, row, bar);
      tma_load_3d(dV + (g + done) * 8 * RB, &maps_v[mi], 0, h, row, bar);
      done += piece;
    }
    g += n;
  }
}

}  // namespace lsrm

namespace lsrm {

// ---------------------------------------------------------------------------
// Union cache: a tile's selected blocks in shared memory, so a producer warp
// can lay out the 8-token groups of any KV chunk with one lane per group.
// ---------------------------------------------------------------------------
constexpr int kUnionCacheCap = 512;

struct UnionCache {
  int t0[kUnionCacheCap];     // first token (clipped to the tile's KV range)
  int t1[kUnionCacheCap];     // end token
  int gstart[kUnionCacheCap]; // first group index (exclusive prefix of group counts)
  uint4 mask[kUnionCacheCap]; // queries of the tile that selected the block
  int n;                      // entries cached (== U when the union fits)
  int groups;                 // total groups
};

// Warp-wide fill (all 32 lanes).  Returns false when the union does not fit.
__device__ __forceinline__ bool union_cache_fill(UnionCache& uc, int U, const int* union_blk, const uint4* union_mask,
                                                 size_t ubase, const int32_t* cu_blk, int kv_lo, int kv_hi,
                                                 int num_blocks, int* err) {
  const int lane = threadIdx.x & 31;
  if (U > kUnionCacheCap) return false;
  int carry = 0;
  for (int b0 = 0; b0 < U; b0 += 32) {
    const int e = b0 + lane;
    int t0 = 0, t1 = 0, g = 0;
    uint4 m = make_uint4(0u, 0u, 0u, 0u);
    if (e < U && dcheck((unsigned)union_blk[ubase + e] < (unsigned)num_blocks, kDcUnion, err)) {
      const int gb = union_blk[ubase + e];
      t0 = max(cu_blk[gb], kv_lo);
      t1 = min(cu_blk[gb + 1], kv_hi);
      if (t1 < t0) t1 = t0;
      g = (t1 - t0 + 7) >> 3;
      m = union_mask[ubase + e];
    }
    int incl = g;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (e < U) {
      uc.t0[e] = t0;
      uc.t1[e] = t1;
      uc.gstart[e] = carry + incl - g;
      uc.mask[e] = m;
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    uc.n = U;
    uc.groups = carry;
  }
  __syncwarp();
  return true;
}

// Lays out groups [NG*j, NG*j+NG) of the union into row0 / qmask / colmask
// (one lane per group, lanes >= NG idle).  Warp-wide.  Returns the lane's
// group's first token (-1: no group).
//
// `cursor` (per lane, start at 0) remembers the lane's entry between calls
// with increasing j: the lane's group only moves forward, so the entry is
// found by a short forward scan instead of a search.
template <int NG>
__device__ __forceinline__ int union_cache_chunk(const UnionCache& uc, int j, int* row0, uint32_t (*qmask)[4],
                                                 uint32_t* colmask, int& cursor) {
  const int lane = threadIdx.x & 31;
  uint32_t bits = 0u;
  int r = -1;
  if (lane < NG) {
    const int g = NG * j + lane;
    if (g < uc.groups) {
      int lo = cursor;  // last entry with gstart <= g (empty entries never are)
      while (lo + 1 < uc.n && uc.gstart[lo + 1] <= g) ++lo;
      cursor = lo;
      r = uc.t0[lo] + 8 * (g - uc.gstart[lo]);
      const int cnt = min(8, uc.t1[lo] - r);
      const uint4 m = uc.mask[lo];
      qmask[lane][0] = m.x;
      qmask[lane][1] = m.y;
      qmask[lane][2] = m.z;
      qmask[lane][3] = m.w;
      bits = ((1u << cnt) - 1u) << ((lane & 3) * 8);
    } else {
      qmask[lane][0] = qmask[lane][1] = qmask[lane][2] = qmask[lane][3] = 0u;
    }
    row0[lane] = r;
  }
  // colmask word w collects the bytes of groups 4w..4w+3
  bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
  if (lane < NG && (lane & 3) == 0) colmask[lane >> 2] = bits;
  return r;
}

// Issues the TMA loads of one chunk's groups, lanes in parallel.  Runs of
// groups contiguous in memory (or runs of unused groups, read past the end of
// the tensor: zero fill) are split greedily into power-of-two boxes
// (8 << i rows, maps[i]); the box's first group's lane g issues its first
// operand and lane g + NG its second in the same instruction (a TMA issue
// holds the issuing warp ~150-300 cycles; lanes that issue together share
// it).  `r` is lane g's group's first token (-1 unused); consecutive groups
// of a run are `step` tokens apart (a group is 8 rows: 8 tokens of one head,
// or 8/G tokens of G heads).  Warp-wide; the caller has armed `bar` with the
// chunk's bytes.
template <int NG, int RB>
__device__ __forceinline__ void issue_group_runs(int r, uint8_t* dK, uint8_t* dV, const CUtensorMap* maps_k,
                                                 const CUtensorMap* maps_v, int h, int oob_row, uint64_t* bar,
                                                 int step = 8) {
  static_assert(2 * NG <= 32, "two lanes per group");
  const int lane = threadIdx.x & 31;
  const int prev = __shfl_up_sync(0xffffffffu, r, 1);
  const bool cont = lane > 0 && lane < NG && ((r >= 0 && prev == r - step) || (r < 0 && prev < 0));
  const uint32_t starts = __ballot_sync(0xffffffffu, lane < NG && !cont) | (1u << NG);
  int go = 0, hb = 0;
  if (lane < NG) {
    const int s0 = 31 - __clz(starts & ((2u << lane) - 1u));        // this run's first group
    const int s1 = __ffs(starts & ~((2u << lane) - 1u)) - 1;         // next run's first group
    const int n = s1 - s0, d = lane - s0;
    hb = 31 - __clz(n - d);                                          // largest box that fits
    go = d == ((n >> (hb + 1)) << (hb + 1));
  }
  const int g = lane < NG ? lane : lane - NG;
  go = __shfl_sync(0xffffffffu, go, g);
  hb = __shfl_sync(0xffffffffu, hb, g);
  const int rg = __shfl_sync(0xffffffffu, r, g);
  if (lane < 2 * NG && go) {
    const bool second = lane >= NG;
    tma_load_3d((second ? dV : dK) + g * 8 * RB, second ? &maps_v[hb] : &maps_k[hb], 0, h, rg >= 0 ? rg : oob_row,
                bar);
  }
}

}  // namespace lsrm
