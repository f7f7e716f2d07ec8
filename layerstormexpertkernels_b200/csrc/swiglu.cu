// Fused SwiGLU: out[n, j] = silu(g) * u, g = in[n, j], u = in[n, d + j].
// Grid-stride over 8-element vectors of the output; each step reads 16 bytes
// of gate and 16 bytes of up and writes 16 bytes, so the kernel is a pure
// HBM stream (6 bytes per output element).  Replaces fused_swiglu_bf16
// (smxx/activation/fused_swiglu.cu:32-89), which runs one block per row.
#include "common.cuh"
#include "swiglu.cuh"

namespace lsek {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(T* __restrict__ out,
                                                         const T* __restrict__ in, int64_t N,
                                                         int d, float limit) {
  const int vpr = d / 8;
  const int64_t total = N * vpr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / vpr;
    const int v = static_cast<int>(i - n * vpr);
    const T* g = in + n * 2 * d + static_cast<int64_t>(v) * 8;
    const uint4 graw = ldg_nc_v4(g);
    const uint4 uraw = ldg_nc_v4(g + d);
    const T* ge = reinterpret_cast<const T*>(&graw);
    const T* ue = reinterpret_cast<const T*>(&uraw);
    uint4 oraw;
    T* oe = reinterpret_cast<T*>(&oraw);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      oe[j] = Elem<T>::from_f(swiglu_f32(Elem<T>::to_f(ge[j]), Elem<T>::to_f(ue[j]), limit));
    *reinterpret_cast<uint4*>(out + n * d + static_cast<int64_t>(v) * 8) = oraw;
  }
}

template <typename T>
__global__ void swiglu_scalar_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t N,
                                     int d, float limit) {
  const int64_t total = N * d;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / d;
    const int j = static_cast<int>(i - n * d);
    const float g = Elem<T>::to_f(in[n * 2 * d + j]);
    const float u = Elem<T>::to_f(in[n * 2 * d + d + j]);
    out[i] = Elem<T>::from_f(swiglu_f32(g, u, limit));
  }
}

template <typename T>
lsek_status launch_swiglu_t(void* out, const void* in, int64_t N, int d, float limit,
                            cudaStream_t st) {
  const bool vec_ok = d % 8 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int threads = 256;
  const int64_t items = vec_ok ? N * (d / 8) : N * d;
  int64_t grid = ceil_div(items, threads);
  const int64_t cap = 32ll * num_sms();
  if (grid > cap) grid = cap;
  if (vec_ok)
    swiglu_vec_kernel<T><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<T*>(out), static_cast<const T*>(in), N, d, limit);
  else
    swiglu_scalar_kernel<T><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<T*>(out), static_cast<const T*>(in), N, d, limit);
  return check_launch("fused_swiglu");
}

}  // namespace
}  // namespace lsek

extern "C" lsek_status lsek_fused_swiglu(void* output, const void* input, int32_t num_tokens,
                                         int32_t d, float swiglu_limit, int32_t dtype,
                                         void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(num_tokens >= 0 && d >= 0, "fused_swiglu: sizes must be >= 0");
  LSEK_REQUIRE(swiglu_limit >= 0.0f, "fused_swiglu: swiglu_limit must be >= 0 (0 = no clamp)");
  LSEK_REQUIRE(dtype == LSEK_BF16 || dtype == LSEK_FP16, "fused_swiglu: dtype must be bf16 or fp16");
  if (num_tokens == 0 || d == 0) return LSEK_OK;
  LSEK_REQUIRE(output && input, "fused_swiglu: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == LSEK_BF16
             ? launch_swiglu_t<__nv_bfloat16>(output, input, num_tokens, d, swiglu_limit, st)
             : launch_swiglu_t<__half>(output, input, num_tokens, d, swiglu_limit, st);
}
