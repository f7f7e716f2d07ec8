// Shared helpers for the sm_100a kernels of liblsek: status plumbing, dtype
// conversions, and the bounded waits every spin in this library goes through.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "lsek.h"

namespace lsek {

// ---- host-side status plumbing ---------------------------------------------

// Records `msg` as the calling thread's last error and returns `st`.
lsek_status fail(lsek_status st, const char* fmt, ...);
// Returns LSEK_OK, or LSEK_ERR_CUDA with the launch error recorded.
lsek_status check_launch(const char* what);

#define LSEK_REQUIRE(cond, ...)                                  \
  do {                                                           \
    if (!(cond)) return ::lsek::fail(LSEK_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define LSEK_CUDA_TRY(expr)                                                 \
  do {                                                                      \
    cudaError_t e_ = (expr);                                                \
    if (e_ != cudaSuccess)                                                  \
      return ::lsek::fail(LSEK_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

int num_sms();  // SM count of the current device (cached per device)

// One-time setup (e.g. raising a kernel's shared-memory limit) that must be
// repeated for every device the library is used on.
struct PerDeviceOnce {
  std::atomic<uint64_t> done{0};
};
template <class F>
cudaError_t once_per_device(PerDeviceOnce& once, F&& f) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (once.done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = f();
  if (e == cudaSuccess) once.done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// ---- device-side error word --------------------------------------------------

// Codes a kernel records when its bounded wait expires; read back (and
// cleared) by lsek_device_error.  Each translation unit with waiting kernels
// keeps its own word (grouped_gemm.cu, ep.cu); lsek_device_error reads both.
enum DeviceError : int32_t {
  kDevErrNone = 0,
  kDevErrGemmProducerWait = 1,
  kDevErrGemmMmaWait = 2,
  kDevErrGemmEpilogueWait = 3,
  kDevErrEpDispatchWait = 4,   // a peer's dispatch rows did not arrive in time
  kDevErrEpCombineWait = 5,    // a peer's combine slots did not arrive in time
};

// Nanoseconds since an arbitrary epoch (globaltimer); used to bound waits.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound on any single wait inside a kernel of this library.  Real waits
// last microseconds; 2 s means a peer of the wait is gone.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ---- element types ------------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// Eight 16-bit elements in one 16-byte vector.
template <typename T>
struct alignas(16) Vec8 {
  T v[8];
};

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__host__ __device__ constexpr inline int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

}  // namespace lsek
