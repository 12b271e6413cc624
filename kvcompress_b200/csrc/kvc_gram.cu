// Column Gram / cross products A^T B over a long row axis (SIMT, fp32 FMA).
//
// Used for
//  * the feature-mode Gram + sketch  [x^T x | x^T Omega]  (kvc_gram),
//  * the token-mode Gram  x_proj_t^T x_proj_t             (kvc_gram, k = 0),
//  * the Tucker core       u_token^T x_proj_t              (kvc_core).
// The row axis is split into chunks; each block accumulates one 64x64
// output tile of one chunk in fp32 and writes it to the workspace; a second
// kernel sums the chunks in a fixed order in fp64, so results are
// bit-reproducible run to run.
#include <algorithm>

#include "kvc_common.cuh"

namespace kvc {

bool tc_gram_eligible(int dtype, int p, int k);
size_t tc_gram_workspace(int n_cells, int64_t rows);
int tc_gram_launch(int n_cells, const void* const* a, int64_t rows, const float* omega, int k, double* out,
                   void* workspace, size_t ws_bytes, cudaStream_t st);
int kernel_policy();

namespace {

constexpr int TB = 64;   // output tile edge
constexpr int RB = 32;   // rows staged per iteration
constexpr int NT = 256;  // threads per block (16 x 16, 4x4 outputs each)

// One operand's RB x W stage (rows r0.., columns c0.. of a row-major matrix
// with ld columns, the columns past ncols zero) held in registers until it
// is stored to shared memory, so the next stage's loads are in flight while
// the current one is multiplied.  16-bit operands whose row length is a
// multiple of 8 on 16-byte boundaries take one 16-byte load per thread
// (W = 64 only).
template <typename T, int W = TB>
struct StageRegs {
  uint4 v;
  float s[RB * W / NT];

  __device__ __forceinline__ void load(const T* __restrict__ base, int64_t r0, int64_t r_end, int c0, int ncols,
                                       int ld, bool vec, const float* __restrict__ extra, int q1) {
    if constexpr (sizeof(T) == 2 && W == TB) {
      if (vec) {
        const int rr = threadIdx.x >> 3, col = c0 + ((threadIdx.x & 7) << 3);
        const int64_t r = r0 + rr;
        v = (r < r_end && col < ncols) ? __ldg(reinterpret_cast<const uint4*>(base + r * ld + col))
                                       : make_uint4(0u, 0u, 0u, 0u);
        return;
      }
    }
#pragma unroll
    for (int u = 0; u < RB * W / NT; ++u) {
      const int e = threadIdx.x + u * NT;
      const int rr = e / W, cc = e % W;
      const int64_t r = r0 + rr;
      const int c = c0 + cc;
      float val = 0.f;
      if (r < r_end) {
        if (c < q1) val = Elt<T>::to_f32(base[r * ld + c]);
        else if (c < ncols) val = extra[r * (ncols - q1) + (c - q1)];
      }
      s[u] = val;
    }
  }

  __device__ __forceinline__ void store(float (*sm)[W], bool vec) {
    if constexpr (sizeof(T) == 2 && W == TB) {
      if (vec) {
        const int rr = threadIdx.x >> 3, cb = (threadIdx.x & 7) << 3;
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q) sm[rr][cb + q] = Elt<T>::to_f32(e[q]);
        return;
      }
    }
#pragma unroll
    for (int u = 0; u < RB * W / NT; ++u) {
      const int e = threadIdx.x + u * NT;
      sm[e / W][e % W] = s[u];
    }
  }
};

// CW output columns a thread (tiles of 64 x 16 CW): 4, or 5 for outputs
// of 65 to 80 columns (a d = 64 Gram with its sketch in one tile).
template <typename TA, typename TB1, int CW>
__global__ void __launch_bounds__(NT)
atb_partial_kernel(CellPtrs A, CellPtrs B1, const float* __restrict__ B2, int64_t rows, int p,
                   int q1, int q2, int chunks, int64_t chunk_rows, float* __restrict__ partial, int vec_a,
                   int vec_b) {
  constexpr int TJ = 16 * CW;
  const int cell = blockIdx.z;
  const int chunk = blockIdx.x;
  const int q = q1 + q2;
  const int tiles_j = (q + TJ - 1) / TJ;
  const int ti = blockIdx.y / tiles_j, tj = blockIdx.y % tiles_j;
  const int i0 = ti * TB, j0 = tj * TJ;
  const TA* __restrict__ a = static_cast<const TA*>(A.p[cell]);
  const TB1* __restrict__ b1 = static_cast<const TB1*>(B1.p[cell]);
  __shared__ __align__(16) float sA[RB][TB];
  __shared__ __align__(16) float sB[RB][TJ];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][CW];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < CW; ++v) acc[u][v] = 0.f;

  const int64_t r_begin = (int64_t)chunk * chunk_rows;
  const int64_t r_end = r_begin + chunk_rows < rows ? r_begin + chunk_rows : rows;
  StageRegs<TA> ra;
  StageRegs<TB1, TJ> rb;
  ra.load(a, r_begin, r_end, i0, p, p, vec_a, nullptr, p);
  rb.load(b1, r_begin, r_end, j0, q, q1, vec_b, B2, q1);
  for (int64_t r0 = r_begin; r0 < r_end; r0 += RB) {
    ra.store(sA, vec_a);
    rb.store(sB, vec_b);
    __syncthreads();
    if (r0 + RB < r_end) {
      ra.load(a, r0 + RB, r_end, i0, p, p, vec_a, nullptr, p);
      rb.load(b1, r0 + RB, r_end, j0, q, q1, vec_b, B2, q1);
    }
#pragma unroll 4
    for (int rr = 0; rr < RB; ++rr) {
      const float4 a4 = *reinterpret_cast<const float4*>(&sA[rr][ty * 4]);
      const float av[4] = {a4.x, a4.y, a4.z, a4.w};
      float bv[CW];
      if constexpr (CW == 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(&sB[rr][tx * 4]);
        bv[0] = b4.x;
        bv[1] = b4.y;
        bv[2] = b4.z;
        bv[3] = b4.w;
      } else {
        // column stride 5: the 16 columns groups of a half warp hit distinct banks
#pragma unroll
        for (int v = 0; v < CW; ++v) bv[v] = sB[rr][tx * CW + v];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < CW; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
  float* out = partial + ((int64_t)cell * chunks + chunk) * (int64_t)p * q;
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < CW; ++v) {
      const int i = i0 + ty * 4 + u, j = j0 + tx * CW + v;
      if (i < p && j < q) out[(int64_t)i * q + j] = acc[u][v];
    }
}

// Skinny variant (p + q <= SK_MAXPQ, or p <= SK_MAXP_WIDE with p + q <=
// SK_MAXPQ_WIDE): one block loads a chunk of SK_ROWS rows of A and [B1 | B2]
// into shared memory with independent loads, then each thread sums one or
// more outputs over the chunk.  Used for the token Gram (p = m * rd) and the
// Tucker core (p = rt), whose operands are a few columns wide: the tiled
// kernel above would serialise its loads there, or (one row of A) compute a
// 64 x 64 tile for one row of outputs.
constexpr int SK_ROWS = 256;
constexpr int SK_MAXPQ = 48;
// a few rows of A (the Tucker core's u_token^T, rt <= 8) against up to 120
// columns: the tiled kernel would compute a 64 x 64 tile for each of them
constexpr int SK_MAXP_WIDE = 8, SK_MAXPQ_WIDE = 128;

template <typename TA, typename TB1>
__global__ void __launch_bounds__(NT)
atb_skinny_kernel(CellPtrs A, CellPtrs B1, const float* __restrict__ B2, int64_t rows, int p, int q1, int q2,
                  int chunks, float* __restrict__ partial) {
  extern __shared__ float sk[];
  const int cell = blockIdx.y;
  const int chunk = blockIdx.x;
  const int q = q1 + q2;
  float* sA = sk;                  // [SK_ROWS][p]
  float* sB = sk + SK_ROWS * p;    // [SK_ROWS][q]
  const int64_t r0 = (int64_t)chunk * SK_ROWS;
  const int nr = (int)(rows - r0 < SK_ROWS ? rows - r0 : SK_ROWS);
  const TA* __restrict__ a = static_cast<const TA*>(A.p[cell]) + r0 * p;
  const TB1* __restrict__ b1 = static_cast<const TB1*>(B1.p[cell]) + r0 * q1;
  const float* __restrict__ b2 = B2 ? B2 + r0 * q2 : nullptr;
  const int na = nr * p;
#pragma unroll 4
  for (int e = threadIdx.x; e < SK_ROWS * p; e += NT) sA[e] = e < na ? Elt<TA>::to_f32(a[e]) : 0.f;
  const int nb1 = nr * q1;
#pragma unroll 4
  for (int e = threadIdx.x; e < SK_ROWS * q1; e += NT) {
    const int r = e / q1, j = e % q1;
    sB[r * q + j] = e < nb1 ? Elt<TB1>::to_f32(b1[e]) : 0.f;
  }
  if (q2 > 0) {
    const int nb2 = nr * q2;
#pragma unroll 4
    for (int e = threadIdx.x; e < SK_ROWS * q2; e += NT) {
      const int r = e / q2, j = e % q2;
      sB[r * q + q1 + j] = e < nb2 ? b2[e] : 0.f;
    }
  }
  __syncthreads();
  float* out = partial + ((int64_t)cell * chunks + chunk) * (int64_t)p * q;
  for (int o = threadIdx.x; o < p * q; o += NT) {
    const int i = o / q, j = o % q;
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
    for (int r = 0; r < SK_ROWS; r += 2) {
      acc0 = fmaf(sA[r * p + i], sB[r * q + j], acc0);
      acc1 = fmaf(sA[(r + 1) * p + i], sB[(r + 1) * q + j], acc1);
    }
    out[o] = acc0 + acc1;
  }
}

// Sum partials over chunks (fixed order, fp64) into the Gram layout
// [A^T B1 (p x q1) | A^T B2 (p x q2) | trace] at `stride` doubles per cell.
__global__ void gram_reduce_kernel(const float* __restrict__ partial, int n_cells, int chunks, int p,
                                   int q1, int q2, double* __restrict__ out, int64_t stride) {
  const int q = q1 + q2;
  const int64_t total = (int64_t)n_cells * p * q;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int cell = (int)(idx / ((int64_t)p * q));
    const int64_t e = idx % ((int64_t)p * q);
    const int i = (int)(e / q), j = (int)(e % q);
    const float* src = partial + (int64_t)cell * chunks * p * q + e;
    double s = 0.0;
    for (int c = 0; c < chunks; ++c) s += (double)src[(int64_t)c * p * q];
    double* o = out + cell * stride;
    if (j < q1) o[(int64_t)i * q1 + j] = s;
    else o[(int64_t)p * q1 + (int64_t)i * q2 + (j - q1)] = s;
  }
}

// trace of each cell's Gram, one warp per cell (fixed order: lane partial
// sums over i = lane + 32 j, then a butterfly)
__global__ void gram_trace_kernel(double* out, int n_cells, int p, int q2, int64_t stride) {
  const int cell = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (cell >= n_cells) return;
  double* o = out + cell * stride;
  double s = 0.0;
  for (int i = lane; i < p; i += 32) s += o[(int64_t)i * p + i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) o[(int64_t)p * p + (int64_t)p * q2] = s;
}

// core[h, a, r] = C[a, h*rd + r] with C = u_token^T x_proj_t (rt x m*rd).
template <typename T>
__global__ void core_reduce_kernel(const float* __restrict__ partial, int n_cells, int chunks,
                                   int rt, int m, int rd, CellPtrsMut core) {
  const int q = m * rd;
  const int64_t total = (int64_t)n_cells * rt * q;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int cell = (int)(idx / ((int64_t)rt * q));
    const int64_t e = idx % ((int64_t)rt * q);
    const int a = (int)(e / q), c = (int)(e % q);
    const int h = c / rd, r = c % rd;
    const float* src = partial + (int64_t)cell * chunks * rt * q + e;
    double s = 0.0;
    for (int ch = 0; ch < chunks; ++ch) s += (double)src[(int64_t)ch * rt * q];
    T* dst = static_cast<T*>(core.p[cell]);
    dst[((int64_t)h * rt + a) * rd + r] = Elt<T>::from((float)s);
  }
}

// Output columns a thread of atb_partial_kernel takes: 5 when the columns
// fit one 80-wide tile but not a 64-wide one.
int cols_per_thread(int q) { return q > TB && q <= 80 ? 5 : 4; }

struct ChunkPlan {
  int chunks;
  int64_t chunk_rows;
  int tiles;
  bool skinny;
};

// The chunking depends on the row count only (never on the batch size or
// the GPU), so a cell gets bit-identical sums whether it is compressed alone
// or batched with other layers.
ChunkPlan plan_chunks(int n_cells, int64_t rows, int p, int q) {
  (void)n_cells;
  ChunkPlan pl;
  pl.skinny = p + q <= SK_MAXPQ || (p <= SK_MAXP_WIDE && p + q <= SK_MAXPQ_WIDE);
  if (pl.skinny) {
    pl.tiles = 1;
    pl.chunk_rows = SK_ROWS;
    pl.chunks = (int)std::max<int64_t>(1, ceil_div(rows, SK_ROWS));
    return pl;
  }
  pl.tiles = (int)(ceil_div(p, TB) * ceil_div(q, 16 * cols_per_thread(q)));
  // narrow outputs (a feature Gram of d = 64 and its sketch: two tiles) get
  // shorter chunks, so a few cells still fill the GPU with blocks
  int64_t cr = std::max<int64_t>(pl.tiles <= 4 ? 512 : 2048, ceil_div(rows, 128));
  cr = ceil_div(cr, RB) * RB;
  pl.chunk_rows = cr;
  pl.chunks = (int)std::max<int64_t>(1, ceil_div(rows, cr));
  return pl;
}

// 16-bit rows of a multiple of 8 elements, every cell's base on a 16-byte boundary
template <typename T>
bool rows_vectorizable(const CellPtrs& x, int n_cells, int width) {
  if constexpr (sizeof(T) != 2) {
    return false;
  } else {
    if (width % 8 != 0) return false;
    for (int c = 0; c < n_cells; ++c)
      if (reinterpret_cast<uintptr_t>(x.p[c]) & 15u) return false;
    return true;
  }
}

template <typename TA, typename TB1>
int launch_partial(int n_cells, const CellPtrs& a, const CellPtrs& b1, const float* b2, int64_t rows,
                   int p, int q1, int q2, const ChunkPlan& pl, float* partial, cudaStream_t st) {
  if (pl.skinny) {
    const size_t smem = (size_t)SK_ROWS * (p + q1 + q2) * sizeof(float);  // at most 128 KB
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(atb_skinny_kernel<TA, TB1>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("atb_skinny_kernel: ") + cudaGetErrorString(e));
    }
    atb_skinny_kernel<TA, TB1><<<dim3(pl.chunks, n_cells), NT, smem, st>>>(a, b1, b2, rows, p, q1, q2, pl.chunks,
                                                                           partial);
    return check_launch("atb_skinny_kernel");
  }
  dim3 grid(pl.chunks, pl.tiles, n_cells);
  const int vec_a = rows_vectorizable<TA>(a, n_cells, p);
  const int vec_b = q2 == 0 && rows_vectorizable<TB1>(b1, n_cells, q1);
  if (cols_per_thread(q1 + q2) == 5)
    atb_partial_kernel<TA, TB1, 5><<<grid, NT, 0, st>>>(a, b1, b2, rows, p, q1, q2, pl.chunks, pl.chunk_rows, partial,
                                                        vec_a, 0);
  else
    atb_partial_kernel<TA, TB1, 4><<<grid, NT, 0, st>>>(a, b1, b2, rows, p, q1, q2, pl.chunks, pl.chunk_rows, partial,
                                                        vec_a, vec_b);
  return check_launch("atb_partial_kernel");
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" size_t kvc_gram_workspace_bytes(int n_cells, int64_t rows, int p, int k) {
  if (n_cells <= 0 || rows <= 0 || p <= 0 || k < 0) return 0;
  ChunkPlan pl = plan_chunks(n_cells, rows, p, p + k);
  size_t simt = (size_t)n_cells * pl.chunks * (size_t)p * (p + k) * sizeof(float);
  return std::max(simt, tc_gram_eligible(KVC_BF16, p, k) ? tc_gram_workspace(n_cells, rows) : (size_t)0);
}

extern "C" int kvc_gram(int n_cells, const void* const* a, int64_t rows, int p, int dtype,
                        const float* omega, int k, double* out, void* workspace, size_t ws_bytes,
                        void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_gram: bad n_cells");
  if (rows <= 0 || p <= 0 || k < 0) return fail(KVC_ERR_SHAPE, "kvc_gram: bad shape");
  if (!dtype_ok(dtype)) return fail(KVC_ERR_DTYPE, "kvc_gram: bad dtype");
  if (k > 0 && omega == nullptr) return fail(KVC_ERR_ARG, "kvc_gram: omega is NULL");
  if (!out) return fail(KVC_ERR_ARG, "kvc_gram: out is NULL");
  ChunkPlan pl = plan_chunks(n_cells, rows, p, p + k);
  const size_t need = (size_t)n_cells * pl.chunks * (size_t)p * (p + k) * sizeof(float);
  if (!workspace || ws_bytes < need) return fail(KVC_ERR_WORKSPACE, "kvc_gram: workspace too small");
  CellPtrs ap;
  bool aligned = true;
  for (int c = 0; c < n_cells; ++c) {
    if (!a[c]) return fail(KVC_ERR_ARG, "kvc_gram: NULL cell pointer");
    ap.p[c] = a[c];
    aligned = aligned && (reinterpret_cast<uintptr_t>(a[c]) & 15u) == 0;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t stride = (int64_t)p * p + (int64_t)p * k + 1;
  int rc;
  if (kernel_policy() != 1 && k > 0 && aligned && tc_gram_eligible(dtype, p, k) &&
      ws_bytes >= tc_gram_workspace(n_cells, rows)) {
    if ((rc = tc_gram_launch(n_cells, a, rows, omega, k, out, workspace, ws_bytes, st))) return rc;
    gram_trace_kernel<<<(n_cells + 3) / 4, 128, 0, st>>>(out, n_cells, p, k, stride);
    return check_launch("gram_trace_kernel");
  }
  float* partial = static_cast<float*>(workspace);
  KVC_DISPATCH_DTYPE(dtype, T, rc = launch_partial<T, T>(n_cells, ap, ap, omega, rows, p, p, k, pl,
                                                         partial, st));
  if (rc) return rc;
  const int64_t total = (int64_t)n_cells * p * (p + k);
  const int blocks = (int)std::min<int64_t>(ceil_div(total, 256), 8 * num_sms());
  gram_reduce_kernel<<<blocks, 256, 0, st>>>(partial, n_cells, pl.chunks, p, p, k, out, stride);
  if ((rc = check_launch("gram_reduce_kernel"))) return rc;
  gram_trace_kernel<<<(n_cells + 3) / 4, 128, 0, st>>>(out, n_cells, p, k, stride);
  return check_launch("gram_trace_kernel");
}

extern "C" size_t kvc_core_workspace_bytes(int n_cells, int64_t t, int m, int rd, int rt) {
  if (n_cells <= 0 || t <= 0 || m <= 0 || rd <= 0 || rt <= 0) return 0;
  ChunkPlan pl = plan_chunks(n_cells, t, rt, m * rd);
  return (size_t)n_cells * pl.chunks * (size_t)rt * m * rd * sizeof(float);
}

extern "C" int kvc_core(int n_cells, const void* const* x_proj_t, const void* const* u_token,
                        int64_t t, int m, int rd, int rt, int dtype, void* const* core,
                        void* workspace, size_t ws_bytes, void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_core: bad n_cells");
  if (t <= 0 || m <= 0 || rd <= 0 || rt <= 0) return fail(KVC_ERR_SHAPE, "kvc_core: bad shape");
  if (!dtype_ok(dtype)) return fail(KVC_ERR_DTYPE, "kvc_core: bad dtype");
  const int q = m * rd;
  ChunkPlan pl = plan_chunks(n_cells, t, rt, q);
  const size_t need = (size_t)n_cells * pl.chunks * (size_t)rt * q * sizeof(float);
  if (!workspace || ws_bytes < need) return fail(KVC_ERR_WORKSPACE, "kvc_core: workspace too small");
  CellPtrs ut, xp;
  CellPtrsMut cp;
  for (int c = 0; c < n_cells; ++c) {
    if (!x_proj_t[c] || !u_token[c] || !core[c]) return fail(KVC_ERR_ARG, "kvc_core: NULL pointer");
    ut.p[c] = u_token[c];
    xp.p[c] = x_proj_t[c];
    cp.p[c] = core[c];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(workspace);
  int rc;
  KVC_DISPATCH_DTYPE(dtype, T, rc = launch_partial<T, T>(n_cells, ut, xp, nullptr, t, rt, q, 0, pl,
                                                         partial, st));
  if (rc) return rc;
  const int64_t total = (int64_t)n_cells * rt * q;
  const int blocks = (int)std::min<int64_t>(ceil_div(total, 256), 8 * num_sms());
  KVC_DISPATCH_DTYPE(dtype, T,
                     core_reduce_kernel<T><<<blocks, 256, 0, st>>>(partial, n_cells, pl.chunks, rt,
                                                                   m, rd, cp));
  return check_launch("core_reduce_kernel");
}
