#include "host_util.h"

#include <cstdarg>
#include <mutex>
#include <string>
#include <vector>

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

int make_kv_maps(CUtensorMap* maps_k, CUtensorMap* maps_v, int n, const void* k, const void* v, int D, int n_head,
                 long long n_tok, long long tok_stride) {
  for (int i = 0; i < n; ++i) {
    int rc;
    if ((rc = make_tmap_3d(&maps_k[i], k, D, n_head, n_tok, tok_stride, 1, 8 << i))) return rc;
    if ((rc = make_tmap_3d(&maps_v[i], v, D, n_head, n_tok, tok_stride, 1, 8 << i))) return rc;
  }
  return LSRM_OK;
}

int num_sms() {
  static int cache[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// ------------------------------ profiler ----------------------------------
struct ProfRecord {
  std::string name;
  cudaEvent_t start, stop;
};
static std::mutex g_prof_mu;
static std::vector<ProfRecord> g_prof_records;
static std::atomic<int> g_prof_on{0};
struct ProfTotal {
  std::string name;
  double ms;
  uint64_t launches;
};
static std::vector<ProfTotal> g_prof_totals;

ProfScope::ProfScope(const char* name, cudaStream_t s) : stream_(s) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  ProfRecord r;
  r.name = name;
  if (cudaEventCreate(&r.start) != cudaSuccess) return;
  if (cudaEventCreate(&r.stop) != cudaSuccess) {
    cudaEventDestroy(r.start);
    return;
  }
  cudaEventRecord(r.start, s);
  std::lock_guard<std::mutex> g(g_prof_mu);
  slot_ = (int)g_prof_records.size();
  g_prof_records.push_back(r);
}

ProfScope::~ProfScope() {
  if (slot_ < 0) return;
  cudaEvent_t stop;
  {
    std::lock_guard<std::mutex> g(g_prof_mu);
    stop = g_prof_records[slot_].stop;
  }
  cudaEventRecord(stop, stream_);
}

}  // namespace lsrm

extern "C" {

void lsrm_profile_enable(int on) {
  std::lock_guard<std::mutex> g(lsrm::g_prof_mu);
  for (auto& r : lsrm::g_prof_records) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  lsrm::g_prof_records.clear();
  lsrm::g_prof_totals.clear();
  lsrm::g_prof_on.store(on ? 1 : 0);
}

int lsrm_profile_collect(void) {
  std::lock_guard<std::mutex> g(lsrm::g_prof_mu);
  for (auto& r : lsrm::g_prof_records) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess || cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) {
      lsrm::set_error("profile: event query failed");
      return -1;
    }
    bool found = false;
    for (auto& t : lsrm::g_prof_totals)
      if (t.name == r.name) {
        t.ms += ms;
        t.launches += 1;
        found = true;
        break;
      }
    if (!found) lsrm::g_prof_totals.push_back({r.name, (double)ms, 1});
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  lsrm::g_prof_records.clear();
  return (int)lsrm::g_prof_totals.size();
}

int lsrm_profile_get(int index, char* name, int name_cap, double* total_ms, uint64_t* launches) {
  std::lock_guard<std::mutex> g(lsrm::g_prof_mu);
  if (index < 0 || index >= (int)lsrm::g_prof_totals.size()) return LSRM_ERR_INVALID_ARG;
  const auto& t = lsrm::g_prof_totals[index];
  if (name && name_cap > 0) snprintf(name, name_cap, "%s", t.name.c_str());
  if (total_ms) *total_ms = t.ms;
  if (launches) *launches = t.launches;
  return LSRM_OK;
}


int lsrm_abi_version(void) { return LSRM_ABI_VERSION; }

const char* lsrm_last_error(void) { return lsrm::t_last_error.c_str(); }

uint64_t lsrm_launch_count(void) { return lsrm::g_launch_count.load(); }

}  // extern "C"
