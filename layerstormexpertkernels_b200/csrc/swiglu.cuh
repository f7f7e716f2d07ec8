// SwiGLU arithmetic shared by the standalone kernel and the gate/up GEMM
// epilogue, so both produce the same bits from the same 16-bit g and u.
#pragma once

#include <cuda_runtime.h>

namespace lsek {

// silu(g) * u in fp32 with the optional clamp of ref_swiglu
// (tests/test_reference.py:110-125): g = min(g, L), u = clamp(u, -L, L).
// silu(g) = g / (1 + e^-g).
__device__ __forceinline__ float swiglu_f32(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, __expf(-g)));
  return __fmul_rn(s, u);
}

}  // namespace lsek
