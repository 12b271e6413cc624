// Shared helpers for the kvcompress_b200 CUDA kernels (sm_100a).
//
// Element types: the compressed cell x is (m, T, d) row-major in one of
// f32 / f16 / bf16.  Kernels read it through Elt<T>, do arithmetic in fp32,
// and round back to T exactly where the reference rounds (torch's bf16/fp16
// ops widen to fp32, compute, round to nearest even).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <cstring>
#include <string>

#include "kvc_b200.h"

namespace kvc {

// ---------------------------------------------------------------------------
// error state (thread-local, read by kvc_last_error)
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elt;

template <> struct Elt<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float round(float v) { return v; }
  static __device__ __forceinline__ float from(float v) { return v; }
  static __device__ __forceinline__ float to_f32(float v) { return v; }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
};

__device__ __forceinline__ float round_dt(float v, int dt) {
  if (dt == KVC_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == KVC_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float load_dt(const void* base, int64_t i, int dt) {
  if (dt == KVC_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  if (dt == KVC_F16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}

__device__ __forceinline__ void store_dt(void* base, int64_t i, float v, int dt) {
  if (dt == KVC_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else if (dt == KVC_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// Order-preserving map float -> int32 (for atomicMin / atomicMax on floats).
__device__ __forceinline__ int32_t ordered_bits(float f) {
  int32_t b = __float_as_int(f);
  return b ^ ((b >> 31) & 0x7FFFFFFF);
}
__host__ __device__ __forceinline__ float from_ordered_bits(int32_t b) {
#ifdef __CUDA_ARCH__
  return __int_as_float(b ^ ((b >> 31) & 0x7FFFFFFF));
#else
  int32_t u = b ^ ((b >> 31) & 0x7FFFFFFF);
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// Per-cell device pointers, passed to kernels by value.
struct CellPtrs {
  const void* p[KVC_MAX_CELLS];
};
struct CellPtrsMut {
  void* p[KVC_MAX_CELLS];
};

inline size_t dtype_size(int dt) { return dt == KVC_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == KVC_F32 || dt == KVC_F16 || dt == KVC_BF16; }

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms();

}  // namespace kvc

#define KVC_DISPATCH_DTYPE(dt, T, ...)                   \
  do {                                                   \
    if ((dt) == KVC_F32) {                               \
      using T = float;                                   \
      __VA_ARGS__;                                       \
    } else if ((dt) == KVC_F16) {                        \
      using T = __half;                                  \
      __VA_ARGS__;                                       \
    } else {                                             \
      using T = __nv_bfloat16;                           \
      __VA_ARGS__;                                       \
    }                                                    \
  } while (0)
