// Shared helpers for the Motif B200 kernels: dtype conversion, vector loads,
// warp/block reductions, error reporting for the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "motif_b200.h"

namespace motif {

// ---- error reporting (host) ----------------------------------------------
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- dtype traits ------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round a float through the storage dtype and back (models a materialised
// intermediate tensor of that dtype).
template <typename T>
__device__ __forceinline__ float round_through(float v) { return to_f<T>(from_f<T>(v)); }

// ---- vector loads of N consecutive elements into floats ----------------------
// The pointer must be aligned to N*sizeof(T) bytes (callers guarantee it).
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[N]) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES == 16) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else if constexpr (BYTES == 8) {
    uint2 r = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else if constexpr (BYTES == 4) {
    uint32_t r = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else if constexpr (BYTES == 32) {
    uint4 r0 = reinterpret_cast<const uint4*>(p)[0];
    uint4 r1 = reinterpret_cast<const uint4*>(p)[1];
    const T* e0 = reinterpret_cast<const T*>(&r0);
    const T* e1 = reinterpret_cast<const T*>(&r1);
#pragma unroll
    for (int i = 0; i < N / 2; ++i) out[i] = to_f<T>(e0[i]);
#pragma unroll
    for (int i = 0; i < N / 2; ++i) out[N / 2 + i] = to_f<T>(e1[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T* p, const float (&in)[N]) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES == 16) {
    uint4 r;
    T* e = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint4*>(p) = r;
  } else if constexpr (BYTES == 8) {
    uint2 r;
    T* e = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint2*>(p) = r;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f<T>(in[i]);
  }
}

// Programmatic dependent launch: let the next kernel in the stream (if it was
// launched with programmatic stream serialization) start its independent
// prologue — the quantized GEMV streams its weights — while this one runs. The
// dependent still waits for this grid's completion before reading its outputs.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n"); }

// ---- reductions ----------------------------------------------------------------
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

// Sum of NV values across the whole block; every thread gets the totals.
// `scratch` must hold 32*NV floats. Block size must be a multiple of 32.
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
  __syncthreads();  // scratch may be reused by the caller between calls
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) scratch[i * 32 + warp] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float t = (lane < nwarps) ? scratch[i * 32 + lane] : 0.0f;
    v[i] = warp_sum(t);
  }
}

}  // namespace motif

// Dispatch a body over the three activation dtypes.
#define MOTIF_DISPATCH_FLOAT(dtype, T, ...)                                  \
  switch (dtype) {                                                           \
    case MOTIF_F16: {                                                        \
      using T = __half;                                                      \
      __VA_ARGS__;                                                           \
    } break;                                                                 \
    case MOTIF_BF16: {                                                       \
      using T = __nv_bfloat16;                                               \
      __VA_ARGS__;                                                           \
    } break;                                                                 \
    case MOTIF_F32: {                                                        \
      using T = float;                                                       \
      __VA_ARGS__;                                                           \
    } break;                                                                 \
    default:                                                                 \
      return ::motif::fail(MOTIF_ERR_DTYPE, "unsupported dtype code %d", (int)(dtype)); \
  }

#define MOTIF_REQUIRE(cond, code, ...)                 \
  do {                                                 \
    if (!(cond)) return ::motif::fail(code, __VA_ARGS__); \
  } while (0)
