// SwiGLU arithmetic shared by the standalone kernel and the gate/up GEMM
// epilogue, so both produce the same bits from the same 16-bit g and u.
#pragma once

#include <cuda_runtime.h>

namespace lsek {

// silu(g) * u in fp32 with the optional clamp of ref_swiglu
// (tests/test_reference.py:110-125): g = min(g, L), u = clamp(u, -L, L).
// silu(g) = g / (1 + e^-g).
//
// The quotient uses the fast approximate division: an IEEE-rounded division
// costs enough instructions per element that the standalone kernel becomes
// issue-bound below the HBM stream rate (5.2 vs 6.2 TB/s at 65536 x 2048 on
// a B200).  Both __expf and __fdividef are within a few fp32 ulps of their
// exact results for the g that matter, which leaves the 16-bit result within
// one 16-bit ulp of silu(g) * u.  For g < -87 (1 + e^-g > 2^126) the quotient
// is 0 where the exact value is below 2^-120.
__device__ __forceinline__ float swiglu_f32(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  const float s = __fdividef(g, __fadd_rn(1.0f, __expf(-g)));
  return __fmul_rn(s, u);
}

}  // namespace lsek
