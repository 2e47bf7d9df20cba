// Shared helpers for the B200 drafter-step library: error reporting, dtype
// traits, launch accounting and small device utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/pe_b200.h"

namespace pe {

// ---------------------------------------------------------------- errors ----
void set_error(const char* fmt, ...);
int64_t& launch_counter();

#define PE_CHECK_ARG(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::pe::set_error(__VA_ARGS__);        \
      return PE_ERR_ARG;                   \
    }                                      \
  } while (0)

#define PE_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess) {                                                           \
      ::pe::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                      __LINE__);                                                       \
      return PE_ERR_CUDA;                                                              \
    }                                                                                  \
  } while (0)

// after a <<<>>> launch: record it and surface launch-configuration errors
#define PE_LAUNCHED()                                                                 \
  do {                                                                                \
    ++::pe::launch_counter();                                                         \
    cudaError_t _e = cudaPeekAtLastError();                                           \
    if (_e != cudaSuccess) {                                                          \
      ::pe::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e),     \
                      __FILE__, __LINE__);                                            \
      (void)cudaGetLastError();                                                       \
      return PE_ERR_CUDA;                                                             \
    }                                                                                 \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// --------------------------------------------------------------- dtypes -----
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
// round-trip through the storage type (identity for fp32)
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_f(from_f<T>(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// number of SMs of the current device (cached per device)
int sm_count();

// Library-owned non-blocking stream of the current device (slot 0..3), created on
// first use; kernels independent of the caller's stream run there and are joined
// back with events, so callers still see one ordered stream.
cudaStream_t side_stream(int slot);
// Timing-disabled event i (0..31) of the current device, reused across calls.
cudaEvent_t pool_event(int i);

// dispatch a lambda templated on the storage type
#define PE_DISPATCH(dtype, T, ...)                                   \
  [&]() -> int {                                                    \
    if ((dtype) == PE_F32) {                                        \
      using T = float;                                              \
      return __VA_ARGS__();                                         \
    } else if ((dtype) == PE_BF16) {                                \
      using T = __nv_bfloat16;                                      \
      return __VA_ARGS__();                                         \
    }                                                               \
    ::pe::set_error("unsupported dtype code %d", (int)(dtype));     \
    return PE_ERR_ARG;                                              \
  }()

}  // namespace pe
