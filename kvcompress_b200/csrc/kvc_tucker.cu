// Row-times-small-matrix products of the partial Tucker decomposition
// (SIMT tiled GEMM, fp32 accumulation, one rounding to the cell dtype):
//
//  * kvc_project_feature: x_proj = x  x_3 U_d  (tucker.py:251), stored in the
//    token-unfolding layout (T, m*rd) that mode_n_unfold(x_proj, 1) reads
//    (tucker.py:254), so the token Gram and the core read it contiguously.
//  * kvc_apply_basis: U_T = A_t M (the lift q @ u_b of svd.py:285 expressed
//    on the token unfolding A_t), rounded like svd.py:507-510.
#include <algorithm>

#include "kvc_common.cuh"

namespace kvc {
namespace {

constexpr int TM = 64, TN = 64, TK = 32, NT = 256;

template <typename TB>
struct BLoad;
template <>
struct BLoad<double> {
  static __device__ __forceinline__ float get(const void* b, int64_t i) {
    return (float)static_cast<const double*>(b)[i];
  }
};
template <>
struct BLoad<float> {
  static __device__ __forceinline__ float get(const void* b, int64_t i) {
    return static_cast<const float*>(b)[i];
  }
};
template <>
struct BLoad<__half> {
  static __device__ __forceinline__ float get(const void* b, int64_t i) {
    return __half2float(static_cast<const __half*>(b)[i]);
  }
};
template <>
struct BLoad<__nv_bfloat16> {
  static __device__ __forceinline__ float get(const void* b, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(b)[i]);
  }
};

// out = round_T(A (rows x K) * B (K x N)); PROJECT scatters row i = h*T + t
// to out[t][h*N + j], otherwise out[i][j].
template <typename TA, typename TB, bool PROJECT>
__global__ void __launch_bounds__(NT)
rowmat_kernel(CellPtrs A, CellPtrs B, int64_t rows, int K, int N, int64_t T, int m,
              CellPtrsMut out) {
  const int cell = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.x * TM;
  const int j0 = blockIdx.y * TN;
  const TA* __restrict__ a = static_cast<const TA*>(A.p[cell]);
  const void* b = B.p[cell];
  __shared__ float sA[TK][TM + 4];
  __shared__ __align__(16) float sB[TK][TN];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[u][v] = 0.f;
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int e = threadIdx.x; e < TM * TK; e += NT) {
      const int rr = e / TK, kk = e % TK;
      const int64_t r = r0 + rr;
      const int k = k0 + kk;
      sA[kk][rr] = (r < rows && k < K) ? Elt<TA>::to_f32(a[r * K + k]) : 0.f;
    }
    for (int e = threadIdx.x; e < TK * TN; e += NT) {
      const int kk = e / TN, jj = e % TN;
      const int k = k0 + kk, j = j0 + jj;
      sB[kk][jj] = (k < K && j < N) ? BLoad<TB>::get(b, (int64_t)k * N + j) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float av[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) av[u] = sA[kk][ty * 4 + u];
      const float4 bv = *reinterpret_cast<const float4*>(&sB[kk][tx * 4]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc[u][0] = fmaf(av[u], bv.x, acc[u][0]);
        acc[u][1] = fmaf(av[u], bv.y, acc[u][1]);
        acc[u][2] = fmaf(av[u], bv.z, acc[u][2]);
        acc[u][3] = fmaf(av[u], bv.w, acc[u][3]);
      }
    }
    __syncthreads();
  }
  TA* o = static_cast<TA*>(out.p[cell]);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t r = r0 + ty * 4 + u;
    if (r >= rows) continue;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int j = j0 + tx * 4 + v;
      if (j >= N) continue;
      int64_t idx;
      if (PROJECT) {
        const int64_t h = r / T, t = r % T;
        idx = t * ((int64_t)m * N) + h * N + j;
      } else {
        idx = r * N + j;
      }
      o[idx] = Elt<TA>::from(acc[u][v]);
    }
  }
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" int kvc_project_feature(int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                                   int dtype, const void* const* u_feature, int rd,
                                   void* const* x_proj_t, void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_project_feature: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || rd <= 0 || rd > d) return fail(KVC_ERR_SHAPE, "kvc_project_feature: bad shape");
  if (!dtype_ok(dtype)) return fail(KVC_ERR_DTYPE, "kvc_project_feature: bad dtype");
  CellPtrs xa, ub;
  CellPtrsMut o;
  for (int c = 0; c < n_cells; ++c) {
    if (!x[c] || !u_feature[c] || !x_proj_t[c]) return fail(KVC_ERR_ARG, "kvc_project_feature: NULL pointer");
    xa.p[c] = x[c];
    ub.p[c] = u_feature[c];
    o.p[c] = x_proj_t[c];
  }
  const int64_t rows = m * t;
  dim3 grid((unsigned)ceil_div(rows, TM), (unsigned)ceil_div(rd, TN), n_cells);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KVC_DISPATCH_DTYPE(dtype, T,
                     rowmat_kernel<T, T, true><<<grid, NT, 0, st>>>(xa, ub, rows, d, rd, t, (int)m, o));
  return check_launch("rowmat_kernel(project)");
}

extern "C" int kvc_apply_basis(int n_cells, const void* const* a, int64_t rows, int p, int dtype,
                               const double* mat, int r, void* const* out, void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_apply_basis: bad n_cells");
  if (rows <= 0 || p <= 0 || r <= 0) return fail(KVC_ERR_SHAPE, "kvc_apply_basis: bad shape");
  if (!dtype_ok(dtype)) return fail(KVC_ERR_DTYPE, "kvc_apply_basis: bad dtype");
  if (!mat) return fail(KVC_ERR_ARG, "kvc_apply_basis: NULL basis");
  CellPtrs aa, mm;
  CellPtrsMut o;
  for (int c = 0; c < n_cells; ++c) {
    if (!a[c] || !out[c]) return fail(KVC_ERR_ARG, "kvc_apply_basis: NULL pointer");
    aa.p[c] = a[c];
    mm.p[c] = mat + (int64_t)c * p * r;
    o.p[c] = out[c];
  }
  dim3 grid((unsigned)ceil_div(rows, TM), (unsigned)ceil_div(r, TN), n_cells);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KVC_DISPATCH_DTYPE(dtype, T,
                     rowmat_kernel<T, double, false><<<grid, NT, 0, st>>>(aa, mm, rows, p, r, 1, 1, o));
  return check_launch("rowmat_kernel(apply)");
}
