#include "host_util.h"

#include <cstdarg>
#include <mutex>

namespace lsrm {

static thread_local std::string t_last_error;
std::atomic<uint64_t> g_launch_count{0};

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_3d(CUtensorMap* map, const void* base, int D, int n_head, long long n_tok, long long tok_stride,
                 int box_h, int box_n) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return LSRM_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("tensor base address %p is not 16-byte aligned", base);
    return LSRM_ERR_ALIGNMENT;
  }
  if ((tok_stride * 2) % 16 != 0) {
    set_error("token stride %lld elements is not a multiple of 16 bytes", tok_stride);
    return LSRM_ERR_ALIGNMENT;
  }
  if (n_tok < 1) n_tok = 1;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)n_head, (cuuint64_t)n_tok};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)tok_stride * 2};
  cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)box_h, (cuuint32_t)box_n};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMapSwizzle swz = (D * 2 == 128) ? CU_TENSOR_MAP_SWIZZLE_128B
                           : (D * 2 == 64) ? CU_TENSOR_MAP_SWIZZLE_64B
                                           : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): D=%d heads=%d tokens=%lld stride=%lld box=(%d,%d,%d)", (int)r, D,
              n_head, n_tok, tok_stride, D, box_h, box_n);
    return LSRM_ERR_CUDA;
  }
  return LSRM_OK;
}

}  // namespace lsrm

extern "C" {

int lsrm_abi_version(void) { return LSRM_ABI_VERSION; }

const char* lsrm_last_error(void) { return lsrm::t_last_error.c_str(); }

uint64_t lsrm_launch_count(void) { return lsrm::g_launch_count.load(); }

}  // extern "C"
