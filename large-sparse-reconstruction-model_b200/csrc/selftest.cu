// Self-test of the UMMA building blocks with exactly the operand forms the
// attention kernels use:
//   c1 = a @ b^T   (A, B K-major, TMA-loaded, swizzled rows of 2*D bytes)
//   c2 = p @ v     (A = P written by threads in the K-major 128B-swizzled
//                   layout, B = V MN-major, TMA-loaded)
// One CTA, 6 warps: warps 0-3 write P and read TMEM, warp 4 issues TMA + MMA.
#include "common.cuh"
#include "host_util.h"

namespace lsrm {

template <int D>
__global__ void __launch_bounds__(192, 1)
    umma_selftest_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_v, const __nv_bfloat16* __restrict__ p,
                         float* __restrict__ c1, float* __restrict__ c2, int* err) {
  constexpr int RB = 2 * D;         // bytes per row of a / b / v tiles
  constexpr int TILE = 128 * RB;    // bytes per 128-row tile
  constexpr uint64_t SWZ = swz_for_row_bytes(RB);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = sa + TILE;
  uint8_t* sv = sb + TILE;
  uint8_t* sp = sv + TILE;  // 2 regions of 128 rows x 128 B
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * 128 * 128);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 128) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // P into shared memory, K-major, 128B swizzle, keys 0-63 in region 0.
  if (threadIdx.x < 128) {
    const int r = threadIdx.x;
    for (int c = 0; c < 16; ++c) {
      const uint4 val = *reinterpret_cast<const uint4*>(p + r * 128 + c * 8);
      const int region = c / 8, ch = c % 8;
      const uint32_t addr = smem_u32(sp + region * 128 * 128) + swz_offset<128>(r, ch);
      st_shared_v4(addr, val.x, val.y, val.z, val.w);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bars[0], 3 * TILE);
      tma_load_3d(sa, &map_a, 0, 0, 0, &bars[0]);
      tma_load_3d(sb, &map_b, 0, 0, 0, &bars[0]);
      tma_load_3d(sv, &map_v, 0, 0, 0, &bars[0]);
      if (mbar_wait(&bars[0], 0, abort_flag, err)) {
        tc_fence_after();
        const uint32_t id1 = make_idesc(1, 0, 0, 128, 128);
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t da = make_sdesc(smem_u32(sa) + ks * 32, 16, 8 * RB, SWZ);
          const uint64_t db = make_sdesc(smem_u32(sb) + ks * 32, 16, 8 * RB, SWZ);
          umma_f16(tmem, da, db, id1, ks > 0);
        }
        const uint32_t id2 = make_idesc(1, 0, 1, 128, D);
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t da = make_sdesc(smem_u32(sp) + (ks / 4) * 128 * 128 + (ks % 4) * 32, 16, 1024, kSw128);
          const uint64_t db = make_sdesc(smem_u32(sv) + ks * 16 * RB, TILE, 8 * RB, SWZ);
          umma_f16(tmem + 128, da, db, id2, ks > 0);
        }
        umma_commit(&bars[1]);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    if (mbar_wait(&bars[1], 0, abort_flag, err)) {
      tc_fence_after();
      const int row = warp * 32 + lane;
      const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
      float v[32];
      for (int c = 0; c < 128; c += 32) {
        tmem_ld32(tmem + lane_base + c, v);
        tmem_wait_ld();
        for (int j = 0; j < 32; ++j) c1[row * 128 + c + j] = v[j];
      }
      float w[D];
      tmem_load_cols<D>(tmem + lane_base + 128, w);
      tmem_wait_ld();
      for (int j = 0; j < D; ++j) c2[row * D + j] = w[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace lsrm

using namespace lsrm;

extern "C" int lsrm_umma_selftest(int32_t head_dim, const void* a, const void* b, const void* p, const void* v,
                                  float* c1, float* c2, int* err_flags, void* stream) {
  LSRM_CHECK_ARG(head_dim == 16 || head_dim == 32 || head_dim == 64, "head_dim must be 16, 32 or 64, got %d", head_dim);
  CUtensorMap ma, mb, mv;
  int rc;
  if ((rc = make_tmap_3d(&ma, a, head_dim, 1, 128, head_dim, 1, 128))) return rc;
  if ((rc = make_tmap_3d(&mb, b, head_dim, 1, 128, head_dim, 1, 128))) return rc;
  if ((rc = make_tmap_3d(&mv, v, head_dim, 1, 128, head_dim, 1, 128))) return rc;
  const size_t smem = 1024 + 3 * 128 * head_dim * 2 + 2 * 128 * 128 + 64;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64) {
    LSRM_CUDA_TRY(cudaFuncSetAttribute(umma_selftest_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    umma_selftest_kernel<64><<<1, 192, smem, s>>>(ma, mb, mv, static_cast<const __nv_bfloat16*>(p), c1, c2,
                                                  err_flags);
  } else if (head_dim == 16) {
    LSRM_CUDA_TRY(cudaFuncSetAttribute(umma_selftest_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    umma_selftest_kernel<16><<<1, 192, smem, s>>>(ma, mb, mv, static_cast<const __nv_bfloat16*>(p), c1, c2,
                                                  err_flags);
  } else {
    LSRM_CUDA_TRY(cudaFuncSetAttribute(umma_selftest_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    umma_selftest_kernel<32><<<1, 192, smem, s>>>(ma, mb, mv, static_cast<const __nv_bfloat16*>(p), c1, c2,
                                                  err_flags);
  }
  LSRM_LAUNCH_CHECK();
  return LSRM_OK;
}
