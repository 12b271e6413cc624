// Small dense solvers for the Tucker bases, one thread block per cell, fp64.
//
// The reference's SVD.randomise (kvcompress/compressor/svd.py:221-316) makes
// five passes over the unfolding A (sketch, two power iterations, Q^T A, the
// Frobenius norm) and then small QR / SVD calls.  Here A is only seen through
// its Gram (kvc_gram), so every remaining step is a small dense problem:
//
//   LEFT  (feature mode, Gram G = A A^T, p = d):
//     Q = orth(Y0), Q = orth(G Q) twice      == orth(G^2 A Omega)
//     C = Q^T G Q = B B^T (B = Q^T A)         -> Ritz pairs (lambda, V)
//     U = Q V[:, :rank]                      (== q @ u_b, svd.py:285)
//   RIGHT (token mode, Gram H = A^T A, p = m * rd):
//     every column of the sketch is A w; orth() runs in the H inner product
//     (<A w, A v> = w^T H v): W = orth_H(Omega), W = orth_H(H W) twice,
//     C = (H W)^T (H W) = B B^T, U = A (W V[:, :rank]) -> basis M = W V.
//   EXACT: eigenpairs of G (LEFT) or H (RIGHT, U = A V Lambda^{-1/2}).
//
// orth() is CholeskyQR2 with rank dropping (a column whose Cholesky pivot
// falls below 1e-10 of its norm is set to zero).  Only the `rank` leading
// eigenpairs are computed, by the selected-eigenpair method of LAPACK's
// dsyevx (Householder tridiagonalisation, bisection on Sturm counts,
// inverse iteration, back-transformation; kvc_eig.cuh).  Every loop has a
// fixed trip count bound.
#include <algorithm>
#include <cmath>

#include "kvc_common.cuh"
#include "kvc_eig.cuh"

namespace kvc {
namespace {

constexpr int SNT = 512;
constexpr int MAX_DIM = 2046;  // largest p and k of the general solver

// C (M x N) = op(A) * B.  A is M x K row-major, or K x M when transA.
__device__ void blk_gemm(double* __restrict__ C, const double* __restrict__ A, bool transA,
                         const double* __restrict__ B, int M, int N, int K) {
  for (int idx = threadIdx.x; idx < M * N; idx += blockDim.x) {
    const int i = idx / N, j = idx % N;
    double s = 0.0;
    if (!transA)
      for (int k = 0; k < K; ++k) s = fma(A[(int64_t)i * K + k], B[(int64_t)k * N + j], s);
    else
      for (int k = 0; k < K; ++k) s = fma(A[(int64_t)k * M + i], B[(int64_t)k * N + j], s);
    C[idx] = s;
  }
  __syncthreads();
}

// One CholeskyQR pass: Y (p x k) <- Y R^{-1} with R^T R = Y^T Mtx Y
// (Mtx = identity when NULL).  Z: p x k scratch, S: k x k scratch.
__device__ void blk_cholqr(double* Y, int p, int k, const double* Mtx, double* Z, double* S) {
  const double* MY = Y;
  if (Mtx) {
    blk_gemm(Z, Mtx, false, Y, p, k, p);
    MY = Z;
  }
  blk_gemm(S, Y, true, MY, k, k, p);
  __shared__ double rjj_s;
  for (int j = 0; j < k; ++j) {
    if (threadIdx.x == 0) {
      const double orig = S[(int64_t)j * k + j];
      double d = orig;
      for (int i = 0; i < j; ++i) d -= S[(int64_t)i * k + j] * S[(int64_t)i * k + j];
      const double r = (orig > 0.0 && d > 1e-10 * orig) ? sqrt(d) : 0.0;
      S[(int64_t)j * k + j] = r;
      rjj_s = r;
    }
    __syncthreads();
    const double rjj = rjj_s;
    for (int l = j + 1 + threadIdx.x; l < k; l += blockDim.x) {
      double v = S[(int64_t)j * k + l];
      for (int i = 0; i < j; ++i) v -= S[(int64_t)i * k + j] * S[(int64_t)i * k + l];
      S[(int64_t)j * k + l] = rjj > 0.0 ? v / rjj : 0.0;
    }
    __syncthreads();
  }
  for (int r = threadIdx.x; r < p; r += blockDim.x) {
    double* y = Y + (int64_t)r * k;
    for (int j = 0; j < k; ++j) {
      double v = y[j];
      for (int i = 0; i < j; ++i) v -= y[i] * S[(int64_t)i * k + j];
      const double rjj = S[(int64_t)j * k + j];
      y[j] = rjj > 0.0 ? v / rjj : 0.0;
    }
  }
  __syncthreads();
}

__device__ void blk_orth2(double* Y, int p, int k, const double* Mtx, double* Z, double* S) {
  blk_cholqr(Y, p, k, Mtx, Z, S);
  blk_cholqr(Y, p, k, Mtx, Z, S);
}

struct SolveArgs {
  int mode, side, p, k, rank, n_power, basis_dtype;
  int64_t n_other;
  const double* gram;
  int64_t gram_stride;
  const float* omega;
  void* basis;
  double* sv2;
  double* tail;
  double* ws;
  int64_t ws_cell;
};

// Workspace layout of the general solver per cell (doubles):
//   exact:      A (p x p) | Zt (rank x p) | vec (8 p) | lam (p) | eig scratch
//   randomised: Q (p x k) | Z (p x k) | S (k x k) | C (k x k) | Zt (k x k) |
//               vec (8 k) | lam (k) | eig scratch
// where the eigensolver's scratch is 3 n doubles for each of min(n, SNT)
// threads (n = p exact, k randomised).
__host__ __device__ inline int64_t eig_scratch_doubles(int n) { return 3LL * n * (n < SNT ? n : SNT); }

__global__ void __launch_bounds__(SNT) sketch_solve_kernel(SolveArgs a) {
  __shared__ double red[64];
  __shared__ int cnt[SNT];
  const int cell = blockIdx.x;
  const int p = a.p, k = a.k, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* ws = a.ws + cell * a.ws_cell;
  __shared__ double nrm_s;

  if (a.mode == KVC_SVD_EXACT) {
    double* A = ws;                               // p x p
    double* Zt = A + (int64_t)p * p;              // rank x p
    double* vec = Zt + (int64_t)rank * p;         // 8 p
    double* lam = vec + eig::vec_doubles(p);      // p
    double* scr = lam + p;
    double part = 0.0;
    for (int64_t i = threadIdx.x; i < (int64_t)p * p; i += blockDim.x) {
      const double g = gram[i];
      A[i] = g;
      if (i / p == i % p) part += g;
    }
    const double total = eig::block_sum(part, red);  // trace = |A|_F^2 (its barriers order the copy)
    eig::eig_top(A, p, p, rank, lam, Zt, p, vec, cnt, red, scr);
    const int64_t max_rank = a.n_other < p ? a.n_other : p;
    if (threadIdx.x == 0) {
      double kept = 0.0;
      for (int i = 0; i < rank; ++i) kept += fmax(lam[i], 0.0);
      const double t = total > 0.0 ? (total - kept) / total : 0.0;
      a.tail[cell] = (rank >= max_rank || !(total > 0.0)) ? 0.0 : fmax(t, 0.0);
      if (a.sv2)
        for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = fmax(lam[i], 0.0);
    }
    if (a.side == KVC_SIDE_LEFT) {
      for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
        const int i = (int)(idx / rank), r = (int)(idx % rank);
        store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)Zt[(int64_t)r * p + i], a.basis_dtype);
      }
    } else {
      const double lmax = fmax(lam[0], 0.0);
      double* M = static_cast<double*>(a.basis) + (int64_t)cell * p * rank;
      for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
        const int i = (int)(idx / rank), r = (int)(idx % rank);
        const double l = lam[r];
        M[idx] = (l > 1e-14 * lmax && l > 0.0) ? Zt[(int64_t)r * p + i] / sqrt(l) : 0.0;
      }
    }
    return;
  }

  // randomised
  double* Q = ws;                                 // p x k
  double* Z = Q + (int64_t)p * k;                 // p x k
  double* S = Z + (int64_t)p * k;                 // k x k
  double* C = S + (int64_t)k * k;                 // k x k
  double* Zt = C + (int64_t)k * k;                // k x k (rank rows used)
  double* vec = Zt + (int64_t)k * k;              // 8 k
  double* lam = vec + eig::vec_doubles(k);        // k
  double* scr = lam + k;
  const double* Mtx = nullptr;
  const double* G = gram;
  if (a.side == KVC_SIDE_LEFT) {
    const double* y0 = gram + (int64_t)p * p;
    for (int64_t i = threadIdx.x; i < (int64_t)p * k; i += blockDim.x) Q[i] = y0[i];
    if (threadIdx.x == 0) nrm_s = gram[(int64_t)p * p + (int64_t)p * k];
  } else {
    Mtx = gram;
    for (int64_t i = threadIdx.x; i < (int64_t)p * k; i += blockDim.x) Q[i] = (double)a.omega[i];
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int i = 0; i < p; ++i) t += gram[(int64_t)i * p + i];
      nrm_s = t;
    }
  }
  __syncthreads();
  blk_orth2(Q, p, k, Mtx, Z, S);
  for (int it = 0; it < a.n_power; ++it) {
    blk_gemm(Z, G, false, Q, p, k, p);
    for (int64_t i = threadIdx.x; i < (int64_t)p * k; i += blockDim.x) Q[i] = Z[i];
    __syncthreads();
    blk_orth2(Q, p, k, Mtx, Z, S);
  }
  blk_gemm(Z, G, false, Q, p, k, p);              // Z = G Q (or H W)
  if (a.side == KVC_SIDE_LEFT) blk_gemm(C, Q, true, Z, k, k, p);   // Q^T G Q
  else blk_gemm(C, Z, true, Z, k, k, p);                           // (H W)^T (H W)
  eig::eig_top(C, k, k, rank, lam, Zt, k, vec, cnt, red, scr);
  if (threadIdx.x == 0) {
    double retained = 0.0;
    for (int i = 0; i < rank; ++i) retained += fmax(lam[i], 0.0);
    const double nrm = nrm_s;
    double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[cell] = t > 0.0 ? t : 0.0;
    if (a.sv2)
      for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = fmax(lam[i], 0.0);
  }
  // basis = Q V[:, :rank] (V's columns are Zt's rows)
  for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
    const int i = (int)(idx / rank), r = (int)(idx % rank);
    double s = 0.0;
    for (int j = 0; j < k; ++j) s = fma(Q[(int64_t)i * k + j], Zt[(int64_t)r * k + j], s);
    if (a.side == KVC_SIDE_LEFT) store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)s, a.basis_dtype);
    else static_cast<double*>(a.basis)[(int64_t)cell * p * rank + idx] = s;
  }
}

// ---------------------------------------------------------------------------
// Shared-memory solver for the common randomised case (p <= 128, k <= 32).
// Same algorithm and outputs as sketch_solve_kernel above, laid out for
// latency: every operand lives in shared memory and every step is a short
// block-wide phase (the Cholesky's trailing updates, the inverse of R by
// parallel back-substitution, Q = Y R^{-1} as a product, one phase of 2 x 2
// block updates per Jacobi round), so no single warp runs a long chain of
// dependent fp64 operations.  Square roots and reciprocals take an fp32
// hardware estimate refined by two Newton-Raphson steps in fp64.
// ---------------------------------------------------------------------------
constexpr int SM_P = 128;
constexpr int SM_K = 32;
constexpr int SM_QS = SM_K + 2;  // row stride (doubles) of Q and Z: even, so rows start on 16 bytes
constexpr int SM_NT = 256;

// G | Q | Z | S | C | Zt | vec (8 SM_K) | lam | diag0 (2 SM_K) | red (64) | cnt
size_t small_smem_bytes(int p) {
  return sizeof(double) * (((size_t)p * p + 1) / 2 * 2 + 2 * (size_t)p * SM_QS + 3 * SM_K * SM_K +
                           eig::vec_doubles(SM_K) + 3 * SM_K + 64) +
         sizeof(int) * SM_NT;
}

// 1/sqrt(x) and 1/x for normal positive / nonzero x: fp32 estimate, then two
// Newton-Raphson steps y <- y (3 - x y^2) / 2 and y <- y (2 - x y) (each step
// doubles the correct bits: ~22 -> 44 -> 88).
__device__ __forceinline__ double rsqrt_nr(double x) {
  double y = (double)rsqrtf((float)x);
  y = y * fma(-0.5 * x, y * y, 1.5);
  y = y * fma(-0.5 * x, y * y, 1.5);
  return y;
}
// the fp32 estimate needs x inside the fp32 normal range
__device__ __forceinline__ bool f32_range(double x) { return fabs(x) > 1e-36 && fabs(x) < 1e36; }
__device__ __forceinline__ double rsqrt_any(double x) { return f32_range(x) ? rsqrt_nr(x) : 1.0 / sqrt(x); }

// Z (p x k) = G Q, G symmetric p x p.  Thread: one row, 8 columns.  The
// eight Q values of a step are read as four 16-byte pairs when Q is 16-byte
// aligned (the shared-memory wavefronts of these broadcast reads are what
// bound the product); the FMAs run in the same order either way.
__device__ void sm_gemm(double* Z, const double* G, const double* Q, int p, int k) {
  const int groups = (k + 7) / 8;
  const bool paired = (reinterpret_cast<uintptr_t>(Q) & 15) == 0;
  for (int task = threadIdx.x; task < p * groups; task += blockDim.x) {
    const int i = task % p, jg = task / p;
    double acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0;
    if (paired) {
      for (int kk = 0; kk < p; ++kk) {
        const double g = G[kk * p + i];
        const double2* q = reinterpret_cast<const double2*>(Q + kk * SM_QS + jg * 8);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const double2 v = q[c];
          acc[2 * c] = fma(g, v.x, acc[2 * c]);
          acc[2 * c + 1] = fma(g, v.y, acc[2 * c + 1]);
        }
      }
    } else {
      for (int kk = 0; kk < p; ++kk) {
        const double g = G[kk * p + i];
        const double* q = Q + kk * SM_QS + jg * 8;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = fma(g, q[c], acc[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (jg * 8 + c < k) Z[i * SM_QS + jg * 8 + c] = acc[c];
  }
  __syncthreads();
}

// S (k x k, stride SM_K) = A^T B over p rows; one output per thread, rows in
// a fixed order (two partial sums).
__device__ void sm_colgram(double* S, const double* A, const double* B, int p, int k) {
  for (int o = threadIdx.x; o < k * k; o += blockDim.x) {
    const int i = o / k, j = o % k;
    double s0 = 0.0, s1 = 0.0;
    int r = 0;
    for (; r + 1 < p; r += 2) {
      s0 = fma(A[r * SM_QS + i], B[r * SM_QS + j], s0);
      s1 = fma(A[(r + 1) * SM_QS + i], B[(r + 1) * SM_QS + j], s1);
    }
    if (r < p) s0 = fma(A[r * SM_QS + i], B[r * SM_QS + j], s0);
    S[i * SM_K + j] = s0 + s1;
  }
  __syncthreads();
}

// Cholesky with rank dropping of S (k x k, upper triangle -> R): a column
// whose pivot falls below 1e-10 of its original diagonal is zero.  Then
// X = R^{-1} (upper triangular, zero rows and columns where R was dropped).
// diag0 points to 2 SM_K doubles of scratch.
//
// One barrier per elimination step: step j updates the trailing rows with
// the unscaled row j (S[i][l] -= S[j][i] S[j][l] / d) and scales row j - 1,
// which nobody reads in that phase; 1 / R[j][j] is kept for the
// back-substitution.
__device__ void sm_chol_inv(double* S, double* X, double* diag0, int k) {
  double* rinv = diag0 + SM_K;  // 1 / R[j][j], 0 where the column was dropped
  for (int i = threadIdx.x; i < k; i += blockDim.x) diag0[i] = S[i * SM_K + i];
  __syncthreads();
  for (int j = 0; j < k; ++j) {
    const double d = S[j * SM_K + j], oj = diag0[j];
    const bool keep = oj > 0.0 && d > 1e-10 * oj;
    const double rs = keep ? rsqrt_any(d) : 0.0;
    const double inv_d = rs * rs;
    if (threadIdx.x == 0) rinv[j] = rs;
    // scaling of row j - 1 (R[j-1][l] = S[j-1][l] / R[j-1][j-1], the diagonal
    // included), then the trailing update of rows j + 1 .. k - 1
    const int ns = j > 0 ? k - j + 1 : 0, m = k - 1 - j;
    for (int t = threadIdx.x; t < ns + m * m; t += blockDim.x) {
      if (t < ns) {
        const int l = j - 1 + t;
        S[(j - 1) * SM_K + l] *= rinv[j - 1];
      } else {
        const int u = t - ns, i = j + 1 + u / m, l = j + 1 + u % m;
        if (l >= i) S[i * SM_K + l] = fma(-S[j * SM_K + i] * inv_d, S[j * SM_K + l], S[i * SM_K + l]);
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) S[(k - 1) * SM_K + k - 1] *= rinv[k - 1];
  __syncthreads();
  // X = R^{-1}: column c by back-substitution (columns in parallel)
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    for (int i = k - 1; i >= 0; --i) {
      double v = 0.0;
      if (i <= c) {
        v = i == c ? 1.0 : 0.0;
        for (int jj = i + 1; jj <= c; ++jj) v = fma(-S[i * SM_K + jj], X[jj * SM_K + c], v);
        v *= rinv[i];
      }
      X[i * SM_K + c] = v;
    }
  }
  __syncthreads();
}

// Q (p x k) = Y X, X upper triangular; Y is left untouched
__device__ void sm_apply_rinv(double* Q, const double* Y, const double* X, int p, int k) {
  for (int o = threadIdx.x; o < p * k; o += blockDim.x) {
    const int r = o / k, c = o % k;
    double v = 0.0;
    for (int j = 0; j <= c; ++j) v = fma(Y[r * SM_QS + j], X[j * SM_K + c], v);
    Q[r * SM_QS + c] = v;
  }
  __syncthreads();
}

// One CholeskyQR pass in the inner product of Mtx (identity when NULL):
// Q <- orth(Y); Y's storage becomes scratch.  Returns the new Q.
__device__ double* sm_cholqr(double* Y, double* Z, double* S, double* X, double* diag0, const double* Mtx, int p,
                             int k) {
  if (Mtx) {
    sm_gemm(Z, Mtx, Y, p, k);
    sm_colgram(S, Y, Z, p, k);
  } else {
    sm_colgram(S, Y, Y, p, k);
  }
  sm_chol_inv(S, X, diag0, k);
  sm_apply_rinv(Z, Y, X, p, k);
  return Z;
}

__global__ void __launch_bounds__(SM_NT) sketch_solve_small_kernel(SolveArgs a) {
  extern __shared__ __align__(16) double sm[];
  const int cell = blockIdx.x;
  const int p = a.p, k = a.k, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* G = sm;                       // p x p
  double* Q = G + (p * p + 1) / 2 * 2;  // p x SM_QS, 16-byte aligned
  double* Z = Q + p * SM_QS;            // p x SM_QS
  double* S = Z + p * SM_QS;            // SM_K x SM_K
  double* C = S + SM_K * SM_K;
  double* Zt = C + SM_K * SM_K;         // Ritz vectors as rows (rank x SM_K)
  double* X = C;                        // R^{-1} of the CholeskyQR passes (C is set after them)
  double* vec = Zt + SM_K * SM_K;       // eigensolver vectors
  double* lam = vec + eig::vec_doubles(SM_K);  // SM_K
  double* diag0 = lam + SM_K;           // 2 SM_K
  double* red = diag0 + 2 * SM_K;       // 64 (reduction scratch)
  int* cnt = reinterpret_cast<int*>(red + 64);  // SM_NT
  __shared__ double nrm_s;
  {
    // sixteen loads in flight per thread before their stores (the Gram is
    // 128 KB at p = 128, one L2 round trip per batch)
    constexpr int U = 16;
    const int nt = blockDim.x, pp = p * p;
    int i = threadIdx.x;
    for (; i + (U - 1) * nt < pp; i += U * nt) {
      double v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = __ldcg(gram + i + u * nt);
#pragma unroll
      for (int u = 0; u < U; ++u) G[i + u * nt] = v[u];
    }
    for (; i < pp; i += nt) G[i] = __ldcg(gram + i);
  }
  if (a.side == KVC_SIDE_LEFT) {
    const double* y0 = gram + (int64_t)p * p;
    for (int i = threadIdx.x; i < p * k; i += blockDim.x) Q[(i / k) * SM_QS + i % k] = y0[i];
    if (threadIdx.x == 0) nrm_s = gram[(int64_t)p * p + (int64_t)p * k];
  } else {
    for (int i = threadIdx.x; i < p * k; i += blockDim.x) Q[(i / k) * SM_QS + i % k] = (double)a.omega[i];
  }
  __syncthreads();
  if (a.side == KVC_SIDE_RIGHT && threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < p; ++i) t += G[i * p + i];
    nrm_s = t;
  }
  const double* Mtx = a.side == KVC_SIDE_RIGHT ? G : nullptr;
  // one CholeskyQR pass keeps each power step well conditioned; the final
  // basis gets a second pass for orthogonality to working precision
  double* W = sm_cholqr(Q, Z, S, X, diag0, Mtx, p, k);  // result in Z
  Z = Q;
  Q = W;
  if (a.n_power == 0) {
    W = sm_cholqr(Q, Z, S, X, diag0, Mtx, p, k);
    Z = Q;
    Q = W;
  }
  for (int it = 0; it < a.n_power; ++it) {
    sm_gemm(Z, G, Q, p, k);  // Z = G Q becomes the sketch
    W = Q;
    Q = Z;
    Z = W;
    W = sm_cholqr(Q, Z, S, X, diag0, Mtx, p, k);
    Z = Q;
    Q = W;
    if (it + 1 == a.n_power) {
      W = sm_cholqr(Q, Z, S, X, diag0, Mtx, p, k);
      Z = Q;
      Q = W;
    }
  }
  sm_gemm(Z, G, Q, p, k);  // Z = G Q (or H W)
  if (a.side == KVC_SIDE_LEFT) sm_colgram(C, Q, Z, p, k);  // Q^T G Q
  else sm_colgram(C, Z, Z, p, k);                         // (H W)^T (H W)
  // the rank leading Ritz pairs (eigenpairs of C); the eigensolver's
  // per-thread scratch is in the workspace
  eig::eig_top(C, SM_K, k, rank, lam, Zt, SM_K, vec, cnt, red, a.ws + cell * a.ws_cell);
  if (threadIdx.x == 0) {
    double retained = 0.0;
    for (int i = 0; i < rank; ++i) retained += fmax(lam[i], 0.0);
    const double nrm = nrm_s;
    const double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[cell] = t > 0.0 ? t : 0.0;
    if (a.sv2)
      for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = fmax(lam[i], 0.0);
  }
  // basis = Q V[:, :rank] (V's columns are Zt's rows)
  for (int idx = threadIdx.x; idx < p * rank; idx += blockDim.x) {
    const int i = idx / rank, r = idx % rank;
    double s = 0.0;
    for (int j = 0; j < k; ++j) s = fma(Q[i * SM_QS + j], Zt[r * SM_K + j], s);
    if (a.side == KVC_SIDE_LEFT) store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)s, a.basis_dtype);
    else static_cast<double*>(a.basis)[(int64_t)cell * p * rank + idx] = s;
  }
}

// ---------------------------------------------------------------------------
// Exact mode for p <= 128 (SVD.exact through the Gram, svd.py:181-219): the
// Gram in shared memory, its rank leading eigenpairs by eig::eig_top; the
// eigenvectors and the eigensolver's per-thread scratch in the workspace.
// ---------------------------------------------------------------------------
constexpr int EX_P = 128;

size_t exact_small_smem_bytes(int p) {
  return sizeof(double) * ((size_t)p * p + eig::vec_doubles(p) + p + 64) + sizeof(int) * SM_NT;
}

__global__ void __launch_bounds__(SM_NT) exact_solve_small_kernel(SolveArgs a) {
  extern __shared__ __align__(16) double sm[];
  const int cell = blockIdx.x;
  const int p = a.p, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* G = sm;                              // p x p
  double* vec = G + p * p;                     // eigensolver vectors
  double* lam = vec + eig::vec_doubles(p);     // p
  double* red = lam + p;                       // 64
  int* cnt = reinterpret_cast<int*>(red + 64); // SM_NT
  double* Zt = a.ws + cell * a.ws_cell;        // rank x p
  double* scr = Zt + (int64_t)rank * p;
  {
    constexpr int U = 16;  // loads in flight per thread before their stores
    const int nt = blockDim.x, pp = p * p;
    int i = threadIdx.x;
    for (; i + (U - 1) * nt < pp; i += U * nt) {
      double v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = __ldcg(gram + i + u * nt);
#pragma unroll
      for (int u = 0; u < U; ++u) G[i + u * nt] = v[u];
    }
    for (; i < pp; i += nt) G[i] = __ldcg(gram + i);
  }
  __syncthreads();
  double part = 0.0;
  for (int i = threadIdx.x; i < p; i += blockDim.x) part += G[i * (p + 1)];
  const double total = eig::block_sum(part, red);  // trace = |A|_F^2
  eig::eig_top(G, p, p, rank, lam, Zt, p, vec, cnt, red, scr);
  const int64_t max_rank = a.n_other < p ? a.n_other : p;
  if (threadIdx.x == 0) {
    double kept = 0.0;
    for (int i = 0; i < rank; ++i) kept += fmax(lam[i], 0.0);
    const double t = total > 0.0 ? (total - kept) / total : 0.0;
    a.tail[cell] = (rank >= max_rank || !(total > 0.0)) ? 0.0 : fmax(t, 0.0);
    if (a.sv2)
      for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = fmax(lam[i], 0.0);
  }
  if (a.side == KVC_SIDE_LEFT) {
    for (int idx = threadIdx.x; idx < p * rank; idx += blockDim.x) {
      const int i = idx / rank, r = idx % rank;
      store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)Zt[(int64_t)r * p + i], a.basis_dtype);
    }
  } else {
    const double lmax = fmax(lam[0], 0.0);
    double* M = static_cast<double*>(a.basis) + (int64_t)cell * p * rank;
    for (int idx = threadIdx.x; idx < p * rank; idx += blockDim.x) {
      const int i = idx / rank, r = idx % rank;
      const double l = lam[r];
      M[idx] = (l > 1e-14 * lmax && l > 0.0) ? Zt[(int64_t)r * p + i] / sqrt(l) : 0.0;
    }
  }
}

// Workspace doubles per cell: the general solver's layout (above), which
// also covers the shared-memory kernels' eigenvectors and scratch.
int64_t ws_per_cell(int mode, int p, int k) {
  if (mode == KVC_SVD_EXACT) return 2LL * p * p + eig::vec_doubles(p) + p + eig_scratch_doubles(p);
  return 2LL * p * k + 3LL * k * k + eig::vec_doubles(k) + k + eig_scratch_doubles(k);
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" size_t kvc_sketch_solve_workspace_bytes(int n_cells, int mode, int p, int k) {
  if (n_cells <= 0 || p <= 0) return 0;
  return (size_t)n_cells * ws_per_cell(mode, p, k) * sizeof(double);
}

extern "C" int kvc_sketch_solve(int n_cells, int mode, int side, int p, int64_t n_other, int k,
                                int rank, int n_power, const double* gram, int64_t gram_stride,
                                const float* omega, void* basis_out, int basis_dtype,
                                double* sv2_out, double* tail_out, void* workspace,
                                size_t ws_bytes, void* stream) {
  if (n_cells <= 0) return fail(KVC_ERR_ARG, "kvc_sketch_solve: bad n_cells");
  if (mode != KVC_SVD_EXACT && mode != KVC_SVD_RANDOMISED)
    return fail(KVC_ERR_ARG, "kvc_sketch_solve: bad mode");
  if (side != KVC_SIDE_LEFT && side != KVC_SIDE_RIGHT)
    return fail(KVC_ERR_ARG, "kvc_sketch_solve: bad side");
  if (p <= 0 || p > MAX_DIM || rank <= 0 || rank > p || n_other <= 0)
    return fail(KVC_ERR_SHAPE, "kvc_sketch_solve: bad p/rank");
  if (mode == KVC_SVD_RANDOMISED && (k < rank || k > p || k > MAX_DIM))
    return fail(KVC_ERR_SHAPE, "kvc_sketch_solve: sketch width must satisfy rank <= k <= p");
  if (mode == KVC_SVD_RANDOMISED && (n_power < 0 || n_power > 16))
    return fail(KVC_ERR_ARG, "kvc_sketch_solve: n_power out of range");
  if (side == KVC_SIDE_RIGHT && mode == KVC_SVD_RANDOMISED && !omega)
    return fail(KVC_ERR_ARG, "kvc_sketch_solve: omega is NULL");
  if (side == KVC_SIDE_LEFT && !dtype_ok(basis_dtype))
    return fail(KVC_ERR_DTYPE, "kvc_sketch_solve: bad basis dtype");
  if (side == KVC_SIDE_RIGHT && basis_dtype != KVC_F64)
    return fail(KVC_ERR_DTYPE, "kvc_sketch_solve: right-side basis is float64");
  if (!gram || !basis_out || !tail_out) return fail(KVC_ERR_ARG, "kvc_sketch_solve: NULL pointer");
  const int kk = mode == KVC_SVD_EXACT ? 0 : k;
  const int64_t per = ws_per_cell(mode, p, kk);
  if (!workspace || ws_bytes < (size_t)n_cells * per * sizeof(double))
    return fail(KVC_ERR_WORKSPACE, "kvc_sketch_solve: workspace too small");
  SolveArgs a;
  a.mode = mode;
  a.side = side;
  a.p = p;
  a.k = kk;
  a.rank = rank;
  a.n_power = n_power;
  a.basis_dtype = basis_dtype;
  a.n_other = n_other;
  a.gram = gram;
  a.gram_stride = gram_stride;
  a.omega = omega;
  a.basis = basis_out;
  a.sv2 = sv2_out;
  a.tail = tail_out;
  a.ws = static_cast<double*>(workspace);
  a.ws_cell = per;
  if (mode == KVC_SVD_RANDOMISED && p <= SM_P && kk <= SM_K) {
    const size_t smem = small_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(sketch_solve_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    sketch_solve_small_kernel<<<n_cells, SM_NT, smem, static_cast<cudaStream_t>(stream)>>>(a);
    return check_launch("sketch_solve_small_kernel");
  }
  if (mode == KVC_SVD_EXACT && p <= EX_P) {
    const size_t smem = exact_small_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(exact_solve_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    exact_solve_small_kernel<<<n_cells, SM_NT, smem, static_cast<cudaStream_t>(stream)>>>(a);
    return check_launch("exact_solve_small_kernel");
  }
  sketch_solve_kernel<<<n_cells, SNT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("sketch_solve_kernel");
}
