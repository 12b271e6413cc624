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
#include "kvc_sched.cuh"
#include "kvc_tc.cuh"
#include "kvc_tma.cuh"

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

// x_proj for small feature ranks (rd <= RDM): LPR lanes share a row, each
// loads 16 bytes with one vector load, multiplies by its slice of U_d held in
// registers, and the partial sums meet with a butterfly of shuffles.  Each
// thread keeps UNROLL rows in flight.  Bandwidth-bound.
template <typename T, int RDM, int LPR>
__global__ void __launch_bounds__(256) project_small_kernel(CellPtrs X, CellPtrs U, int64_t rows, int d, int rd,
                                                           int64_t T_, int m, CellPtrsMut out) {
  constexpr int EPL = 16 / sizeof(T);  // elements per lane
  constexpr int UNROLL = 4;
  const int cell = blockIdx.y;
  const T* x = static_cast<const T*>(X.p[cell]);
  const T* u = static_cast<const T*>(U.p[cell]);
  T* o = static_cast<T*>(out.p[cell]);
  const int lane = threadIdx.x & 31;
  const int pos = lane % LPR;
  float uv[EPL][RDM];
#pragma unroll
  for (int e = 0; e < EPL; ++e)
#pragma unroll
    for (int r = 0; r < RDM; ++r) uv[e][r] = r < rd ? Elt<T>::to_f32(u[(int64_t)(pos * EPL + e) * rd + r]) : 0.f;
  const int64_t groups = (int64_t)gridDim.x * (blockDim.x / LPR);
  // the loop bound is warp-uniform (every lane reaches the shuffles)
  const int64_t warp_gid = (int64_t)blockIdx.x * (blockDim.x / LPR) + (threadIdx.x & ~31) / LPR;
  for (int64_t wbase = warp_gid; wbase < rows; wbase += groups * UNROLL) {
    const int64_t base = wbase + lane / LPR;
    uint4 raw[UNROLL];
#pragma unroll
    for (int q = 0; q < UNROLL; ++q) {
      const int64_t row = base + q * groups;
      raw[q] = row < rows ? *reinterpret_cast<const uint4*>(x + row * d + pos * EPL) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < UNROLL; ++q) {
      const int64_t row = base + q * groups;
      const T* e = reinterpret_cast<const T*>(&raw[q]);
      float acc[RDM];
#pragma unroll
      for (int r = 0; r < RDM; ++r) {
        acc[r] = 0.f;
#pragma unroll
        for (int k = 0; k < EPL; ++k) acc[r] = fmaf(Elt<T>::to_f32(e[k]), uv[k][r], acc[r]);
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
      }
      if (pos < rd && row < rows) {
        const int64_t h = row / T_, t = row % T_;
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < RDM; ++r)
          if (r == pos) v = acc[r];
        o[t * ((int64_t)m * rd) + h * rd + pos] = Elt<T>::from(v);
      }
    }
  }
}

// x_proj for bf16 cells with rd == 1 and d = 8 * LPR: LPR lanes per row,
// each holding 8 values as 4 packed pairs; fp32 accumulation in packed
// pairs (even / odd elements), then a butterfly over the row's lanes.
// Four rows per thread in flight.
template <int LPR>
__global__ void __launch_bounds__(256) project_rd1_bf16_kernel(CellPtrs X, CellPtrs U, int64_t rows, int d,
                                                              int64_t T_, int m, CellPtrsMut out) {
  constexpr int UNROLL = 4;
  const int cell = blockIdx.y;
  const uint4* x = static_cast<const uint4*>(X.p[cell]);
  const uint16_t* u = static_cast<const uint16_t*>(U.p[cell]);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out.p[cell]);
  const int lane = threadIdx.x & 31;
  const int pos = lane % LPR;
  // this lane's 8 entries of u_feature (a column of d), as packed fp32 pairs
  uint64_t u2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float lo = __uint_as_float((uint32_t)u[pos * 8 + 2 * q] << 16);
    const float hi = __uint_as_float((uint32_t)u[pos * 8 + 2 * q + 1] << 16);
    u2[q] = tc::f2_pack(lo, hi);
  }
  const int64_t groups = (int64_t)gridDim.x * (blockDim.x / LPR);
  const int64_t warp_gid = (int64_t)blockIdx.x * (blockDim.x / LPR) + (threadIdx.x & ~31) / LPR;
  const int rows_per_chunk = d / 8;  // uint4 per row
  for (int64_t wbase = warp_gid; wbase < rows; wbase += groups * UNROLL) {  // warp-uniform bound
    const int64_t base = wbase + lane / LPR;
    uint4 raw[UNROLL];
#pragma unroll
    for (int q = 0; q < UNROLL; ++q) {
      const int64_t row = base + q * groups;
      raw[q] = row < rows ? __ldg(x + row * rows_per_chunk + pos) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < UNROLL; ++q) {
      const uint32_t w[4] = {raw[q].x, raw[q].y, raw[q].z, raw[q].w};
      uint64_t acc = tc::f2_pack(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        acc = tc::f2_fma(tc::f2_pack(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u)), u2[i], acc);
      float a0, a1;
      tc::f2_unpack(acc, a0, a1);
      float sum = a0 + a1;
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const int64_t row = base + q * groups;
      if (pos == 0 && row < rows) {
        const int64_t h = row / T_, t = row % T_;
        o[t * m + h] = __float2bfloat16_rn(sum);
      }
    }
  }
}

// x_proj for bf16 cells with rd == 1 and d = 64 or 128, streamed by TMA:
// tiles of 128 rows (one head, 128 tokens) in (cell, token block, head)
// order, heads fastest, so the scattered 2-byte outputs of one token block
// meet in L2 before they are written back.  Each CTA owns a contiguous run
// of tiles; one producer thread keeps NS tiles in flight (SWIZZLE_128B boxes
// of 64 columns), and two consumer threads share a row: thread (r, half)
// sums the 64 (or 32) products of its half in packed fp32 pairs, and the
// halves meet by a shuffle.  A quarter-warp holds 8 rows of one half, so
// the swizzle puts its 16-byte reads in 8 different bank groups.
constexpr int PJ_ROWS = 128, PJ_THREADS = 288;  // 8 consumer warps + 1 producer warp

template <int D, int NS>
struct PjLayout {
  static constexpr uint32_t STAGE = PJ_ROWS * D * 2;
  static constexpr uint32_t OFF_RING = NS * STAGE;
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t BYTES = OFF_BAR + 2 * NS * 8 + 1024;
};

struct PjArgs {
  CellPtrs u;
  CellPtrsMut out;
  int64_t t, tb, units, per_cta;  // tokens, token blocks per head, tiles, tiles per CTA
  int m;
};

template <int D, int NS>
__global__ void __launch_bounds__(PJ_THREADS, 1)
    project_rd1_tma_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ PjArgs A) {
  using L = PjLayout<D, NS>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  constexpr int HALF = D / 2;     // elements per thread
  constexpr int NCH = HALF / 8;   // 16-byte chunks per thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = tc::smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + NS;
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 8);  // one arrive per consumer warp
    }
    tc::mbar_fence_init();
  }
  __syncthreads();
  if (warp == 8) {
    if (lane == 0) {
      sched::Cursor cur(A.per_cta, A.units);
      for (int it = 0;; ++it) {
        const int64_t u = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)u);
        const int st = it % NS;
        if (!tc::mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x501)) break;
        if (u < 0) {
          tc::mbar_arrive(&full[st]);
          break;
        }
        const int cell = (int)(u / (A.tb * A.m));
        const int64_t r = u % (A.tb * A.m);
        const int y = (int)((r % A.m) * A.t + (r / A.m) * PJ_ROWS);  // row of the cell's (m * T) x D view
        tc::mbar_expect_tx(&full[st], L::STAGE);
#pragma unroll
        for (int hcol = 0; hcol < D / 64; ++hcol)
          tc::tma_load_2d(sbase + st * L::STAGE + hcol * PJ_ROWS * 128, &xmaps.m[cell], hcol * 64, y, &full[st]);
      }
    }
    __syncwarp();
  } else {
    // thread -> (row, half): lanes 0-7 and 16-23 hold half 0, 8-15 and 24-31 half 1
    const int half = (threadIdx.x >> 3) & 1;
    const int row = (threadIdx.x & 7) | ((threadIdx.x >> 4) << 3);
    uint64_t u2[HALF / 2];  // this half of u_feature as packed fp32 pairs
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int st = it % NS;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x502))) break;
      const int32_t u = sched::ring_get(ring, it);
      if (u < 0) break;
      const int cell = (int)(u / (A.tb * A.m));
      if (cell != cur_cell) {
        const uint16_t* uf = static_cast<const uint16_t*>(A.u.p[cell]) + half * HALF;
#pragma unroll
        for (int q = 0; q < HALF / 2; ++q)
          u2[q] = tc::f2_pack(__uint_as_float((uint32_t)uf[2 * q] << 16), __uint_as_float((uint32_t)uf[2 * q + 1] << 16));
        cur_cell = cell;
      }
      // half 0 = columns 0-63 (first box), half 1 = 64-127 (D = 128); for
      // D = 64 both halves share the one box, 32 columns each
      const uint8_t* rs = smem + st * L::STAGE + (D == 128 ? half * PJ_ROWS * 128 : 0) + row * 128;
      uint64_t acc = tc::f2_pack(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int chunk = (D == 128 ? c : half * NCH + c) ^ (row & 7);  // SWIZZLE_128B
        const uint4 raw = *reinterpret_cast<const uint4*>(rs + chunk * 16);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc = tc::f2_fma(tc::f2_pack(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u)),
                           u2[c * 4 + i], acc);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[st]);  // the stage has been read
      float a0, a1;
      tc::f2_unpack(acc, a0, a1);
      float sum = a0 + a1;
      sum += __shfl_xor_sync(0xffffffffu, sum, 8);
      const int64_t r = u % (A.tb * A.m);
      const int64_t h = r % A.m, tok = (r / A.m) * PJ_ROWS + row;
      if (half == 0 && tok < A.t)
        static_cast<__nv_bfloat16*>(A.out.p[cell])[tok * A.m + h] = __float2bfloat16_rn(sum);
    }
  }
}

// out (rows x N) = round_T(A (rows x K) * M (K x N)) for K <= 64, N <= 16:
// one thread per row, M in shared memory as float, fp32 accumulation in k
// order (the same arithmetic as rowmat_kernel).  SKN: the column count
// rounded up to 1, 2, 4, 8 or 16, so a rank-1 basis costs one FMA and one
// shared-memory read per element, not sixteen predicated ones.
constexpr int SKK = 64, SKN_MAX = 16;
template <typename T, int SKN>
__global__ void __launch_bounds__(256) rowmat_skinny_kernel(CellPtrs A, const double* __restrict__ mat, int64_t rows,
                                                            int K, int N, CellPtrsMut out) {
  __shared__ float sM[SKK * SKN_MAX];
  const int cell = blockIdx.y;
  const double* m = mat + (int64_t)cell * K * N;
  for (int i = threadIdx.x; i < K * N; i += blockDim.x) sM[i] = (float)m[i];
  __syncthreads();
  const T* a = static_cast<const T*>(A.p[cell]);
  T* o = static_cast<T*>(out.p[cell]);
  // 16-bit rows of a multiple of 8 elements on 16-byte boundaries: the whole
  // row in flight at once (up to eight 16-byte loads per thread)
  const bool vec = sizeof(T) == 2 && K % 8 == 0 && (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    float acc[SKN];
#pragma unroll
    for (int j = 0; j < SKN; ++j) acc[j] = 0.f;
    bool done = false;
    if constexpr (sizeof(T) == 2) {
      if (vec) {
        done = true;
        uint4 raw[SKK / 8];
        const uint4* src = reinterpret_cast<const uint4*>(a + r * K);
#pragma unroll
        for (int c = 0; c < SKK / 8; ++c)
          if (c < K / 8) raw[c] = __ldg(src + c);
#pragma unroll
        for (int c = 0; c < SKK / 8; ++c) {
          if (c >= K / 8) break;
          const T* e = reinterpret_cast<const T*>(&raw[c]);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float av = Elt<T>::to_f32(e[q]);
            const int k = c * 8 + q;
#pragma unroll
            for (int j = 0; j < SKN; ++j)
              if (j < N) acc[j] = fmaf(av, sM[k * N + j], acc[j]);
          }
        }
      }
    }
    if (!done) {
      for (int k = 0; k < K; ++k) {
        const float av = Elt<T>::to_f32(a[r * K + k]);
#pragma unroll
        for (int j = 0; j < SKN; ++j)
          if (j < N) acc[j] = fmaf(av, sM[k * N + j], acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < SKN; ++j)
      if (j < N) o[r * N + j] = Elt<T>::from(acc[j]);
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int lpr = (int)(d * dtype_size(dtype) / 16);
  bool aligned = (d * dtype_size(dtype)) % 16 == 0;
  for (int c = 0; c < n_cells; ++c) aligned = aligned && (reinterpret_cast<uintptr_t>(x[c]) & 15u) == 0;
  if (rd == 1 && dtype == KVC_BF16 && aligned && (d == 64 || d == 128) && rows < (1LL << 31)) {
    TmaMaps xm;
    int rc;
    for (int c = 0; c < n_cells; ++c) {
      const uint64_t dims[2] = {(uint64_t)d, (uint64_t)rows};
      const uint64_t strides[1] = {(uint64_t)d * 2};
      const uint32_t box[2] = {64u, (uint32_t)PJ_ROWS};
      if ((rc = encode_tma(&xm.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x[c], dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    }
    PjArgs a;
    a.u = ub;
    a.out = o;
    a.t = t;
    a.m = (int)m;
    a.tb = ceil_div(t, PJ_ROWS);
    a.units = (int64_t)n_cells * m * a.tb;
    const int64_t ctas = std::min<int64_t>(a.units, num_sms());
    a.per_cta = ceil_div(a.units, ctas);
    const dim3 grid((unsigned)ceil_div(a.units, a.per_cta));
    if (d == 128) {
      auto kern = project_rd1_tma_kernel<128, 6>;
      constexpr size_t sm = PjLayout<128, 6>::BYTES;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return fail(KVC_ERR_LAUNCH, "kvc_project_feature: cudaFuncSetAttribute");
      kern<<<grid, PJ_THREADS, sm, st>>>(xm, a);
    } else {
      auto kern = project_rd1_tma_kernel<64, 8>;
      constexpr size_t sm = PjLayout<64, 8>::BYTES;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return fail(KVC_ERR_LAUNCH, "kvc_project_feature: cudaFuncSetAttribute");
      kern<<<grid, PJ_THREADS, sm, st>>>(xm, a);
    }
    return check_launch("project_rd1_tma_kernel");
  }
  if (rd == 1 && dtype == KVC_BF16 && aligned && (lpr == 8 || lpr == 16)) {
    const int64_t per_block = 256 / lpr * 4;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, per_block),
                                                                    ceil_div(8LL * num_sms(), n_cells)));
    dim3 grid(blocks, n_cells);
    if (lpr == 8) project_rd1_bf16_kernel<8><<<grid, 256, 0, st>>>(xa, ub, rows, d, t, (int)m, o);
    else project_rd1_bf16_kernel<16><<<grid, 256, 0, st>>>(xa, ub, rows, d, t, (int)m, o);
    return check_launch("project_rd1_bf16_kernel");
  }
  if (rd <= 4 && aligned && (lpr == 8 || lpr == 16 || lpr == 32)) {
    const int64_t per_block = 256 / lpr * 4;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, per_block),
                                                                    ceil_div(8LL * num_sms(), n_cells)));
    dim3 grid(blocks, n_cells);
#define KVC_PROJ(R, L)                                                                                \
  KVC_DISPATCH_DTYPE(dtype, T, project_small_kernel<T, R, L><<<grid, 256, 0, st>>>(xa, ub, rows, d, rd, t, \
                                                                                   (int)m, o))
    if (rd == 1) {
      if (lpr == 8) KVC_PROJ(1, 8);
      else if (lpr == 16) KVC_PROJ(1, 16);
      else KVC_PROJ(1, 32);
    } else {
      if (lpr == 8) KVC_PROJ(4, 8);
      else if (lpr == 16) KVC_PROJ(4, 16);
      else KVC_PROJ(4, 32);
    }
#undef KVC_PROJ
    return check_launch("project_small_kernel");
  }
  dim3 grid((unsigned)ceil_div(rows, TM), (unsigned)ceil_div(rd, TN), n_cells);
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p <= SKK && r <= SKN_MAX) {
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 256), ceil_div(16LL * num_sms(), n_cells)));
    const dim3 grid(blocks, n_cells);
#define KVC_ROWMAT_SKINNY(NN) \
  KVC_DISPATCH_DTYPE(dtype, T, rowmat_skinny_kernel<T, NN><<<grid, 256, 0, st>>>(aa, mat, rows, p, r, o))
    if (r <= 1) KVC_ROWMAT_SKINNY(1);
    else if (r <= 2) KVC_ROWMAT_SKINNY(2);
    else if (r <= 4) KVC_ROWMAT_SKINNY(4);
    else if (r <= 8) KVC_ROWMAT_SKINNY(8);
    else KVC_ROWMAT_SKINNY(16);
#undef KVC_ROWMAT_SKINNY
    return check_launch("rowmat_skinny_kernel");
  }
  dim3 grid((unsigned)ceil_div(rows, TM), (unsigned)ceil_div(r, TN), n_cells);
  KVC_DISPATCH_DTYPE(dtype, T,
                     rowmat_kernel<T, double, false><<<grid, NT, 0, st>>>(aa, mm, rows, p, r, 1, 1, o));
  return check_launch("rowmat_kernel(apply)");
}
