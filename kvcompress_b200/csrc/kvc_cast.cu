// Elementwise dtype casts for the identity / fp8 baselines
// (kvcompress/compressor/identity.py:68-117 with dispatch.py:106-125).
//
// float8_e4m3fn follows torch's Tensor.to semantics: round to nearest even
// on the 3-bit mantissa, subnormals with step 2^-9, and no saturation --
// values whose rounding leaves the finite range (|x| > 464) and inf/NaN
// become NaN (0x7F / 0xFF).  The conversion is written out on the float32
// bit pattern from the format definition (1 sign, 4 exponent with bias 7,
// 3 mantissa bits; S.1111.111 is NaN, there is no infinity).
#include <algorithm>

#include "kvc_common.cuh"

namespace kvc {
namespace {

__device__ __forceinline__ uint8_t f32_to_e4m3fn(float f) {
  uint32_t u = __float_as_uint(f);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  u &= 0x7FFFFFFFu;
  if (u >= 0x7F800000u) return sign | 0x7F;           // inf / NaN
  if (u >= 0x43F00000u) return sign | 0x7F;           // >= 480: past the finite range
  if (u < 0x3C800000u) {                              // below 2^-6: subnormal grid
    const float q = rintf(__uint_as_float(u) * 512.0f);  // multiples of 2^-9, exact scaling
    return sign | (uint8_t)q;                         // q == 8 encodes 2^-6 (exp 1, mant 0)
  }
  // normal: rebias exponent (127 -> 7) and round the mantissa to 3 bits
  const uint32_t odd = (u >> 20) & 1u;
  u += ((uint32_t)(7 - 127) << 23) + 0x7FFFFu + odd;
  return sign | (uint8_t)(u >> 20);
}

__device__ __forceinline__ float e4m3fn_to_f32(uint8_t b) {
  const uint32_t sign = (uint32_t)(b & 0x80) << 24;
  const uint32_t e = (b >> 3) & 0xF, m = b & 0x7;
  if (e == 0xF && m == 0x7) return __uint_as_float(sign | 0x7FC00000u);
  float v;
  if (e == 0) v = (float)m * 0.001953125f;  // m * 2^-9
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return __uint_as_float(__float_as_uint(v) | sign);
}

__device__ __forceinline__ float load_any(const void* p, int64_t i, int dt) {
  if (dt == KVC_FP8E4M3) return e4m3fn_to_f32(static_cast<const uint8_t*>(p)[i]);
  return load_dt(p, i, dt);
}

__device__ __forceinline__ void store_any(void* p, int64_t i, float v, int dt) {
  if (dt == KVC_FP8E4M3) static_cast<uint8_t*>(p)[i] = f32_to_e4m3fn(v);
  else store_dt(p, i, v, dt);
}

__global__ void cast_kernel(int64_t n, const void* __restrict__ in, int in_dt, void* __restrict__ out,
                            int out_dt) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_any(out, i, load_any(in, i, in_dt), out_dt);
}

bool cast_dtype_ok(int dt) { return dtype_ok(dt) || dt == KVC_FP8E4M3; }

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" int kvc_cast(int64_t n, const void* in, int in_dtype, void* out, int out_dtype,
                        void* stream) {
  if (n < 0) return fail(KVC_ERR_SHAPE, "kvc_cast: negative size");
  if (!cast_dtype_ok(in_dtype) || !cast_dtype_ok(out_dtype)) return fail(KVC_ERR_DTYPE, "kvc_cast: bad dtype");
  if (n == 0) return KVC_OK;
  if (!in || !out) return fail(KVC_ERR_ARG, "kvc_cast: NULL pointer");
  const int blocks = (int)std::min<int64_t>(ceil_div(n, 256), 16LL * num_sms());
  cast_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(n, in, in_dtype, out, out_dtype);
  return check_launch("cast_kernel");
}
