// Shared helpers for the fkb200 kernels: status plumbing, element-type traits,
// 16-byte vector loads/stores with cache hints, warp reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/fkb200.h"

namespace fk {

// ---------------------------------------------------------------- status -------------
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int launch_status(const char* what);  // FK_OK or FK_ERR_LAUNCH after a launch
int num_sms();                         // SM count of the current device (cached per device)

#define FK_CHECK_ARG(cond, ...)                                   \
  do {                                                            \
    if (!(cond)) return ::fk::fail(FK_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool valid_dtype(int d) { return d == FK_F32 || d == FK_F16 || d == FK_BF16; }
inline int dtype_size(int d) { return d == FK_F32 ? 4 : 2; }

// ---------------------------------------------------------------- element traits -----
template <typename T> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// A 16-byte packet of T elements.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 u;
    T e[N];
  };
};

// Streaming (evict-first) 16-byte global load / store.
template <typename T>
__device__ __forceinline__ Vec16<T> ld_stream(const T* p) {
  Vec16<T> v;
  v.u = __ldcs(reinterpret_cast<const uint4*>(p));
  return v;
}
template <typename T>
__device__ __forceinline__ Vec16<T> ld_keep(const T* p) {
  Vec16<T> v;
  v.u = __ldg(reinterpret_cast<const uint4*>(p));
  return v;
}
template <typename T>
__device__ __forceinline__ void st_stream(T* p, const Vec16<T>& v) {
  __stcs(reinterpret_cast<uint4*>(p), v.u);
}
template <typename T>
__device__ __forceinline__ void st_plain(T* p, const Vec16<T>& v) {
  *reinterpret_cast<uint4*>(p) = v.u;
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

// Sigmoid for the elementwise kernels.  16-bit element types use the fast exponential
// and reciprocal (their outputs round to 8/11 mantissa bits); fp32 uses expf and IEEE
// division.
template <typename T>
__device__ __forceinline__ float sigmoidf_t(float x) {
  return __fdividef(1.0f, 1.0f + __expf(-x));
}
template <>
__device__ __forceinline__ float sigmoidf_t<float>(float x) {
  return 1.0f / (1.0f + expf(-x));
}

}  // namespace fk

// Dispatch helper: runs BODY with `scalar_t` bound to the element type of `dtype`.
#define FK_DISPATCH_DTYPE(dtype, ...)                       \
  switch (dtype) {                                          \
    case FK_F32: { using scalar_t = float; __VA_ARGS__; break; }          \
    case FK_F16: { using scalar_t = __half; __VA_ARGS__; break; }         \
    case FK_BF16: { using scalar_t = __nv_bfloat16; __VA_ARGS__; break; } \
    default: return ::fk::fail(FK_ERR_INVALID_ARG, "bad dtype code %d", (int)(dtype)); \
  }
