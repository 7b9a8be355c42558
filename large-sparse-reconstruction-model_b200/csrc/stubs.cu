// Entry points not yet implemented: they fail loudly.
#include "attn_host.h"
#include "host_util.h"


#define LSRM_STUB(name) \
  ::lsrm::set_error(#name " is not implemented in this build"); \
  return LSRM_ERR_UNSUPPORTED;

extern "C" {
int lsrm_block_topk(const lsrm_varlen*, const lsrm_attn_shape*, const void*, const void*, const float*, int32_t,
                    const int32_t*, int32_t, int32_t, float, int32_t*, int*, void*) { LSRM_STUB(lsrm_block_topk) }
int lsrm_block_mean_fwd(int32_t, int32_t, int32_t, const int32_t*, const void*, int64_t, void*, void*) {
  LSRM_STUB(lsrm_block_mean_fwd) }
int lsrm_block_mean_bwd(int32_t, int32_t, int32_t, const int32_t*, int32_t, const void*, void*, void*) {
  LSRM_STUB(lsrm_block_mean_bwd) }
int lsrm_resnorm_mean_fwd(int32_t, int32_t, int32_t, int32_t, const int32_t*, const void*, const void*, float, void*,
                          void*, float*, float*, void*) { LSRM_STUB(lsrm_resnorm_mean_fwd) }
int lsrm_resnorm_mean_bwd(int32_t, int32_t, int32_t, int32_t, const int32_t*, const void*, const void*, const float*,
                          const float*, const void*, void*, void*) { LSRM_STUB(lsrm_resnorm_mean_bwd) }
int lsrm_gate_merge_fwd(int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, const void*, const void* const*, void*,
                        void*) { LSRM_STUB(lsrm_gate_merge_fwd) }
int lsrm_gate_merge_bwd(int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, const void*, const void* const*,
                        const void*, void*, void* const*, void*) { LSRM_STUB(lsrm_gate_merge_bwd) }
}
