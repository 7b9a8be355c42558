// Host-side declarations shared by the attention entry points.
#pragma once

#include <cuda_runtime.h>

#include "lsrm_sparse.h"
#include "plan.cuh"

namespace lsrm {

// Validates metadata / shape; sets G = Hq / Hkv.
int check_shape(const lsrm_varlen* m, const lsrm_attn_shape* sh, int& G);
float softmax_scale_of(const lsrm_attn_shape* sh);
// Extra workspace of the dense-branch backward (split-KV partial sums).
size_t dense_bwd_extra_bytes(const lsrm_varlen* m, const lsrm_attn_shape* sh, int mode);
int dense_fwd_tiles(const lsrm_varlen* meta, int G, int mode, int window, DensePlan& plan, int* err, cudaStream_t s);

// The dense kernels run with kDenseMaxG query heads per kv head at most.
// Larger groups run over kv heads repeated R = G / kDenseMaxG times (the
// query heads, outputs and LSE are unchanged; the dK / dV of the copies are
// summed back per kv head).  The dense dK/dV kernel ended in a device fault
// in the 24-layer decoder at 131k voxels with 8 query heads per kv head, and
// again with 4 (the 8-head groups regrouped), while every run with one query
// head per kv head, the same decoder included, is clean; the cause is not
// found, so the dense kernels only run with one.
constexpr int kDenseMaxG = 1;
struct DenseRegroup {
  lsrm_attn_shape shape;  // kv heads x R, dense kv rows
  int R;                  // copies of each kv head
  long long nk;           // kv rows (tokens, or compressed blocks)
  size_t inner;           // workspace of the direct kernels for `shape` (256-aligned)
  size_t buf;             // bytes of one repeated k / v / dk / dv buffer (256-aligned)
};
size_t dense_ws_direct(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode);
DenseRegroup dense_regroup(const lsrm_varlen* meta, const lsrm_attn_shape* shape, int mode);
int repeat_kv_heads(const void* src, long long stride, void* dst, long long n, int hkv, int R, int D,
                    cudaStream_t s);

}  // namespace lsrm
