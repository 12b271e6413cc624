// Decode plan of the tensor-core decompress: the part of a decode that does
// not depend on the token range (codes tensor maps, factor pointers, and the
// per-cell B images in the caller's workspace), so that a stream of
// token-range decodes launches only the Tucker-term and decode kernels.
#pragma once

#include "kvc_common.cuh"
#include "kvc_tma.cuh"

namespace kvc {

struct TcDecodePlan {
  TmaMaps cmaps;          // codes of every cell: (m, T, d * bits / 8) uint8
  CellPtrs core, ut, ud;  // Tucker factors (rt > 0)
  uint8_t* bimg;          // workspace: B images, [cell][two or three terms (+ Tucker block)]
  float* tmp;             // workspace: Tucker row terms of the current range
  int64_t m, t;
  int n_cells, d, bits, rt, rd, factor_dtype, out_dtype;
};

int tc_decode_plan_init(TcDecodePlan* p, int n_cells, const uint8_t* const* codes, const float* const* scale,
                        int bits, const void* const* core, const void* const* u_token,
                        const void* const* u_feature, int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd,
                        const float* proj, int out_dtype, void* workspace, size_t ws_bytes, cudaStream_t st);
int tc_decode_plan_run(const TcDecodePlan* p, int64_t t0, int64_t t1, void* const* out, cudaStream_t st);

}  // namespace kvc
