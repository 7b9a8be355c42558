// Host-side helpers shared by the entry points: thread-local error text,
// launch counter, TMA tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>

#include "lsrm_sparse.h"

namespace lsrm {

void set_error(const char* fmt, ...);

// Streaming multiprocessors of the current device (cached per device).
int num_sms();
extern std::atomic<uint64_t> g_launch_count;

inline void count_launch(uint64_t n = 1) { g_launch_count.fetch_add(n, std::memory_order_relaxed); }

#define LSRM_CHECK_ARG(cond, ...)            \
  do {                                       \
    if (!(cond)) {                           \
      ::lsrm::set_error(__VA_ARGS__);        \
      return LSRM_ERR_INVALID_ARG;           \
    }                                        \
  } while (0)

#define LSRM_CUDA_TRY(expr)                                                            \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess) {                                                           \
      ::lsrm::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                        __LINE__);                                                     \
      return LSRM_ERR_CUDA;                                                            \
    }                                                                                  \
  } while (0)

// Checks for a launch error right after a <<<>>> launch.
#define LSRM_LAUNCH_CHECK()                                                            \
  do {                                                                                 \
    ::lsrm::count_launch();                                                            \
    cudaError_t _e = cudaGetLastError();                                               \
    if (_e != cudaSuccess) {                                                           \
      ::lsrm::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e), __FILE__, \
                        __LINE__);                                                     \
      return LSRM_ERR_CUDA;                                                            \
    }                                                                                  \
  } while (0)

// Kernel timing: while profiling is enabled (lsrm_profile_enable), a
// ProfScope records a CUDA event pair on the launching stream around the
// launches made in its lifetime, keyed by name.
class ProfScope {
 public:
  ProfScope(const char* name, cudaStream_t s);
  ~ProfScope();

 private:
  int slot_ = -1;
  cudaStream_t stream_;
};

// Encodes a 3-D tiled tensor map over a [n_tok, n_head, D] 16-bit tensor:
// dims {D, n_head, n_tok}, strides in elements (head stride D, token stride
// `tok_stride`), box {D, box_h, box_n}, swizzle matched to the row size
// (D*2 = 128 B -> 128B swizzle, 64 B -> 64B swizzle).  Out-of-range rows
// read as zero.
int make_tmap_3d(CUtensorMap* map, const void* base, int D, int n_head, long long n_tok, long long tok_stride,
                 int box_h, int box_n);

// Fills maps_k/maps_v (box heights 8 << i rows, i < n) over k and v.
int make_kv_maps(CUtensorMap* maps_k, CUtensorMap* maps_v, int n, const void* k, const void* v, int D, int n_head,
                 long long n_tok, long long tok_stride);

template <typename T>
inline T ceil_div(T a, T b) {
  return (a + b - 1) / b;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace lsrm
