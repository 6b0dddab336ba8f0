// Shared helpers for the MantisNet sm_100a kernels: status handling, the
// device error word, and vectorised row loads/stores.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mantis_b200.h"

namespace mb {

// ---------------------------------------------------------------- status --
int fail(int status, const char* fmt, ...);
int launch_status(const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#define MB_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) return ::mb::fail(MB_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

// Device error word: first nonzero code wins; kernels skip the bad access.
enum DeviceError : uint32_t {
  ERR_NONE = 0,
  ERR_INDEX = 1,       // an index array held a value out of range
  ERR_UNSORTED = 2,    // keys that must be sorted were not
  ERR_RUN_BOUND = 3,   // a CSR run was malformed
};
// Defined here: the library is one translation unit (mantis_b200.cu).
__device__ uint32_t g_device_error = 0;
__device__ __forceinline__ void report(uint32_t code) { atomicCAS(&g_device_error, 0u, code); }

// --------------------------------------------------------------- dtypes --
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Load VEC consecutive elements (VEC * sizeof(T) bytes, naturally aligned).
template <int VEC>
__device__ __forceinline__ void load_vec(const float* __restrict__ p, float* out) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 4; ++i) {
      float4 f = __ldg(reinterpret_cast<const float4*>(p) + i);
      out[4 * i] = f.x; out[4 * i + 1] = f.y; out[4 * i + 2] = f.z; out[4 * i + 3] = f.w;
    }
  } else if constexpr (VEC == 2) {
    float2 f = __ldg(reinterpret_cast<const float2*>(p));
    out[0] = f.x; out[1] = f.y;
  } else {
    out[0] = __ldg(p);
  }
}

template <int VEC>
__device__ __forceinline__ void load_vec(const __nv_bfloat16* __restrict__ p, float* out) {
  if constexpr (VEC % 8 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 8; ++i) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + i);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        out[8 * i + 2 * j] = f.x; out[8 * i + 2 * j + 1] = f.y;
      }
    }
  } else if constexpr (VEC == 4) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  } else if constexpr (VEC == 2) {
    unsigned int u = __ldg(reinterpret_cast<const unsigned int*>(p));
    float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
    out[0] = a.x; out[1] = a.y;
  } else {
    out[0] = __bfloat162float(p[0]);
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(float* p, const float* v) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    p[0] = v[0];
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(__nv_bfloat16* p, const float* v) {
  if constexpr (VEC % 8 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 8; ++i) {
      uint4 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
      reinterpret_cast<uint4*>(p)[i] = u;
    }
  } else if constexpr (VEC == 4) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(v[0], v[1]);
    h[1] = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = u;
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  } else {
    p[0] = __float2bfloat16_rn(v[0]);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
// Sum over aligned groups of `group` lanes (power of two <= 32).
__device__ __forceinline__ float group_sum(float x, int group) {
  for (int o = group >> 1; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

inline bool aligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }
inline int dtype_size(int dt) { return dt == MB_BF16 ? 2 : 4; }
inline bool valid_dtype(int dt) { return dt == MB_F32 || dt == MB_BF16; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Per-lane vector width VEC in {8,4,2,1} such that width % (32 * VEC) == 0
// (0 when width is not a multiple of 32). Attention kernels need this exact
// tiling; row kernels use row_vec, which falls back to a guarded VEC = 1.
inline int pick_vec(int64_t width) {
  if (width % 256 == 0) return 8;
  if (width % 128 == 0) return 4;
  if (width % 64 == 0) return 2;
  if (width % 32 == 0) return 1;
  return 0;
}
inline int row_vec(int64_t width) { return width <= 0 ? 0 : (pick_vec(width) ? pick_vec(width) : 1); }

}  // namespace mb

// Dispatch helpers: expand a body over runtime dtype / VEC choices.
#define MB_DISPATCH_T(dt, T, ...)                 \
  [&] {                                           \
    if ((dt) == MB_BF16) {                        \
      using T = __nv_bfloat16;                    \
      return __VA_ARGS__();                       \
    } else {                                      \
      using T = float;                            \
      return __VA_ARGS__();                       \
    }                                             \
  }()

#define MB_DISPATCH_CH(ch, C, ...)                          \
  [&] {                                                     \
    switch (ch) {                                           \
      case 1: { constexpr int C = 1; return __VA_ARGS__(); } \
      case 2: { constexpr int C = 2; return __VA_ARGS__(); } \
      default: { constexpr int C = 4; return __VA_ARGS__(); } \
    }                                                       \
  }()

#define MB_DISPATCH_VEC(vec, V, ...)                        \
  [&] {                                                     \
    switch (vec) {                                          \
      case 8: { constexpr int V = 8; return __VA_ARGS__(); } \
      case 4: { constexpr int V = 4; return __VA_ARGS__(); } \
      case 2: { constexpr int V = 2; return __VA_ARGS__(); } \
      default: { constexpr int V = 1; return __VA_ARGS__(); } \
    }                                                       \
  }()
