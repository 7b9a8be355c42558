// Fixed-order float32 scoring arithmetic shared by the exact and the fast
// block scorers (and restated by the CPU oracle):
//   dot    = sum_{j=0..D-1} q_j * k_j      (separately rounded mul, add)
//   t      = dot * qk_scale - lse_ln * 1.44269504f
//   score  = sum_{g=0..G-1} exp2_fixed(t_g)
//   agg    = sum over a query block's tokens in ascending order
// exp2_fixed: n = rint(t), f = t - n, degree-7 Taylor polynomial of
// exp(f ln 2) by Horner's rule, times 2^n; t < -125.5 -> 0.
#pragma once

namespace lsrm {

__device__ __forceinline__ float exp2_fixed(float t) {
  const float n = rintf(t);
  if (n < -125.f) return 0.f;
  if (n > 127.f) return INFINITY;
  const float f = __fsub_rn(t, n);
  float r = __uint_as_float(0x377FE5FEu);
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x39218489u));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3AAEC3FFu));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3C1D955Bu));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3D635847u));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3E75FDF0u));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3F317218u));
  r = __fadd_rn(__fmul_rn(r, f), __uint_as_float(0x3F800000u));
  const float sc = __int_as_float(((int)n + 127) << 23);
  return __fmul_rn(r, sc);
}

template <typename T, int D>
__device__ __forceinline__ float exact_dot(const T* __restrict__ a, const T* __restrict__ b) {
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < D; ++j) dot = __fadd_rn(dot, __fmul_rn((float)a[j], (float)b[j]));
  return dot;
}

}  // namespace lsrm
