// Quantiser arithmetic shared by the SIMT and tensor-core kernels
// (IntQuantizer, kvcompress/compressor/quantization.py:300-452).
#pragma once

#include "kvc_common.cuh"

namespace kvc {

__device__ __forceinline__ void qrange(int bits, int symmetric, int& qmin, int& qmax) {
  if (symmetric) {
    qmin = -(1 << (bits - 1));
    qmax = (1 << (bits - 1)) - 1;
  } else {
    qmin = 0;
    qmax = (1 << bits) - 1;
  }
}

// scale / zero point from min/max, in the arithmetic of `dt`
// (IntQuantizer.compute_params, quantization.py:437-452).
__device__ __forceinline__ void params_from_minmax(float mn, float mx, int bits, int symmetric, int dt, float& scale,
                                   int32_t& zp) {
  int qmin, qmax;
  qrange(bits, symmetric, qmin, qmax);
  const float eps = round_dt(1e-12f, dt);
  if (symmetric) {
    float am = fmaxf(fabsf(mn), fabsf(mx));
    am = fmaxf(am, eps);
    scale = round_dt(__fdiv_rn(am, (float)qmax), dt);
    zp = 0;
  } else {
    float rng = fmaxf(round_dt(mx - mn, dt), eps);
    scale = round_dt(__fdiv_rn(rng, (float)(qmax - qmin)), dt);
    const float ratio = round_dt(__fdiv_rn(mn, scale), dt);
    const float z = round_dt((float)qmin - ratio, dt);
    zp = (int32_t)rintf(z);
  }
}

__device__ __forceinline__ int quantize_one(float v, float s, int32_t zp, int qmin, int qmax,
                                            int dt_arith) {
  float sc;
  if (dt_arith != KVC_F32) {
    sc = round_dt(__fdiv_rn(v, s), dt_arith);
    sc = round_dt(sc + (float)zp, dt_arith);
  } else {
    sc = __fadd_rn(__fdiv_rn(v, s), (float)zp);
  }
  float r = rintf(sc);
  r = fminf(fmaxf(r, (float)qmin), (float)qmax);
  return (int)r;
}

}  // namespace kvc
