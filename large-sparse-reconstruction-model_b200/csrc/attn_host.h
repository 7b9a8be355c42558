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

}  // namespace lsrm
