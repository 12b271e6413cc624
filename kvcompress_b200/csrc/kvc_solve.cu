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
constexpr int MAX_DIM = 2046;     // largest p of the solver
constexpr int MAX_SKETCH = 1024;  // largest sketch width k (the row blocks of W R^{-1} live in shared memory)

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

// Workspace layout per cell (doubles):
//   exact (exact_solve_kernel, p > 128):
//               A (p x p) | Zt (rank x p) | vec (8 p) | lam (p) | eig scratch
//   randomised (the multi-launch path below, p > 128 or k > 32):
//               W (p x k) | Z (p x k) | S (k x k) | C (k x k) | Zt (k x k) |
//               vec (8 k) | lam (k) | rinv (k) | misc (4) | eig scratch
// where the eigensolver's scratch is 3 n doubles for each of min(n, SNT)
// threads (n = p exact, k randomised).
__host__ __device__ inline int64_t eig_scratch_doubles(int n) { return 3LL * n * (n < SNT ? n : SNT); }

// Exact mode for p > 128: the Gram copied to the workspace and its rank
// leading eigenpairs found there (served from L2).
__global__ void __launch_bounds__(SNT) exact_solve_kernel(SolveArgs a) {
  __shared__ double red[64];
  __shared__ int cnt[SNT];
  const int cell = blockIdx.x;
  const int p = a.p, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* ws = a.ws + cell * a.ws_cell;
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
  eig::eig_top(A, p, p, rank, lam, Zt, p, vec, cnt, red, scr, SNT);
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
}

// ---------------------------------------------------------------------------
// Shared-memory solver for the common randomised case (p <= 128, k <= 32).
// Same algorithm and outputs as the multi-launch path for larger problems,
// laid out for latency: every operand lives in shared memory and every step
// is a short block-wide phase (the Cholesky's trailing updates, the inverse of
// R by parallel back-substitution, Q = Y R^{-1} as a product), so no single
// warp runs a long chain of dependent fp64 operations.  Square roots take an
// fp32 hardware estimate refined by two Newton-Raphson steps in fp64.
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
  // per-thread scratch is the Z buffer, free once C is formed
  const int workers = std::max(1, std::min(rank, (p * SM_QS) / (3 * k)));
  eig::eig_top(C, SM_K, k, rank, lam, Zt, SM_K, vec, cnt, red, Z, workers);
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
constexpr size_t SMEM_LIMIT = 227 * 1024;  // dynamic shared memory of one CTA (opt-in maximum)

constexpr int EX_WORKERS = 8;  // threads computing eigenvectors when they fit in shared memory

size_t exact_small_smem_bytes(int p) {
  return sizeof(double) * ((size_t)p * p + eig::vec_doubles(p) + p + 64) + sizeof(int) * SM_NT;
}
// the eigenvectors (rank x p) and EX_WORKERS solve scratches in shared memory too
size_t exact_small_smem_bytes_vectors(int p, int rank) {
  return exact_small_smem_bytes(p) + sizeof(double) * ((size_t)rank * p + 3 * (size_t)p * EX_WORKERS);
}

__global__ void __launch_bounds__(SM_NT) exact_solve_small_kernel(SolveArgs a, int vectors_in_smem) {
  extern __shared__ __align__(16) double sm[];
  const int cell = blockIdx.x;
  const int p = a.p, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* G = sm;                              // p x p
  double* vec = G + p * p;                     // eigensolver vectors
  double* lam = vec + eig::vec_doubles(p);     // p
  double* red = lam + p;                       // 64
  int* cnt = reinterpret_cast<int*>(red + 64); // SM_NT
  double* Zt = vectors_in_smem ? reinterpret_cast<double*>(cnt + SM_NT) : a.ws + cell * a.ws_cell;  // rank x p
  double* scr = Zt + (int64_t)rank * p;
  const int workers = vectors_in_smem ? EX_WORKERS : SM_NT;
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
  eig::eig_top(G, p, p, rank, lam, Zt, p, vec, cnt, red, scr, workers);
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

// ---------------------------------------------------------------------------
// Randomised problems beyond the shared-memory solver (p > 128 or k > 32; the
// q-capped token sketch of FlashJoLT is 513 wide over p = m * rd up to 1024).
// The algorithm of sketch_solve_small_kernel as a sequence of batched
// launches: the products (G W, W^T Z, ...) are fp64 GEMMs over many CTAs; the
// Cholesky of each CholeskyQR pass is one CTA per cell (blocked, the panel
// rows in shared memory); W R^{-1} is a triangular solve over blocks of rows;
// the Ritz pairs come from eig::eig_top on the k x k Ritz matrix.
// ---------------------------------------------------------------------------
struct Gemm {
  const double* A;
  const double* B;
  double* C;
  int M, N, K, lda, ldb, ldc, tA, tB;
  int64_t sA, sB, sC;  // per-cell strides (doubles)
};

constexpr int GT = 64;    // output tile GT x GT
constexpr int GKD = 32;   // depth per stage
constexpr int GNT = 256;  // 16 x 16 threads, 4 x 4 outputs each (strided by 16: conflict-free reads)
constexpr int GPT = GT * GKD / GNT;  // elements of each operand a thread stages per stage

// C = op(A) op(B) per cell (row-major; op = transpose when tA / tB).  The
// next stage's operand elements are loaded into registers while the current
// stage is multiplied, so the loads' latency overlaps the arithmetic.
__global__ void __launch_bounds__(GNT) f64_gemm_kernel(Gemm g) {
  __shared__ double As[GKD][GT + 1];
  __shared__ double Bs[GKD][GT + 1];
  const int cell = blockIdx.z;
  const double* A = g.A + cell * g.sA;
  const double* B = g.B + cell * g.sB;
  double* C = g.C + cell * g.sC;
  const int i0 = blockIdx.y * GT, j0 = blockIdx.x * GT;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  double acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0;
  double pa[GPT], pb[GPT];
  // consecutive threads read consecutive addresses
  auto fetch = [&](int l0) {
#pragma unroll
    for (int q = 0; q < GPT; ++q) {
      const int e = threadIdx.x + q * GNT;
      const int ii = g.tA ? e % GT : e / GKD, la = g.tA ? e / GT : e % GKD;
      const int i = i0 + ii, l = l0 + la;
      pa[q] = (i < g.M && l < g.K) ? (g.tA ? A[(int64_t)l * g.lda + i] : A[(int64_t)i * g.lda + l]) : 0.0;
      const int jj = g.tB ? e / GKD : e % GT, lb = g.tB ? e % GKD : e / GT;
      const int j = j0 + jj, m = l0 + lb;
      pb[q] = (j < g.N && m < g.K) ? (g.tB ? B[(int64_t)j * g.ldb + m] : B[(int64_t)m * g.ldb + j]) : 0.0;
    }
  };
  fetch(0);
  for (int l0 = 0; l0 < g.K; l0 += GKD) {
#pragma unroll
    for (int q = 0; q < GPT; ++q) {
      const int e = threadIdx.x + q * GNT;
      As[g.tA ? e / GT : e % GKD][g.tA ? e % GT : e / GKD] = pa[q];
      Bs[g.tB ? e % GKD : e / GT][g.tB ? e / GKD : e % GT] = pb[q];
    }
    __syncthreads();
    if (l0 + GKD < g.K) fetch(l0 + GKD);
#pragma unroll
    for (int ll = 0; ll < GKD; ++ll) {
      double a[4], b[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r] = As[ll][ty + 16 * r];
#pragma unroll
      for (int c = 0; c < 4; ++c) b[c] = Bs[ll][tx + 16 * c];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fma(a[r], b[c], acc[r][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = i0 + ty + 16 * r, j = j0 + tx + 16 * c;
      if (i < g.M && j < g.N) C[(int64_t)i * g.ldc + j] = acc[r][c];
    }
}

int launch_gemm(const Gemm& g, int n_cells, cudaStream_t st) {
  const dim3 grid((g.N + GT - 1) / GT, (g.M + GT - 1) / GT, n_cells);
  f64_gemm_kernel<<<grid, GNT, 0, st>>>(g);
  return check_launch("f64_gemm_kernel");
}

constexpr int CH_NT = 256;
constexpr int CH_ROWS = 32;  // panel rows (fewer when k is large: the panel lives in shared memory)

int chol_panel_rows(int k) { return std::max(1, std::min(CH_ROWS, (int)(28000 / std::max(k, 1)))); }

// In place per cell: S (k x k, row-major) -> R in its upper triangle with
// S = R^T R (CholeskyQR's Gram), rinv[j] = 1 / R[j][j].  Rank dropping as in
// sm_chol_inv: a pivot at or below 1e-10 of the column's original diagonal
// makes the row of R zero and rinv[j] = 0.  Right-looking, nb panel rows at
// a time: the panel is factored in shared memory (one barrier per column,
// the row scaled one step late), then the trailing upper triangle takes the
// rank-nb update in 4 x 4 register tiles.
__global__ void __launch_bounds__(CH_NT) chol_kernel(double* Sb, int k, int nbmax, int64_t sS, double* rinvb,
                                                     int64_t sR) {
  extern __shared__ double P[];  // nbmax x k
  __shared__ double dg[CH_ROWS], ri[CH_ROWS];
  double* S = Sb + blockIdx.x * sS;
  double* rinv = rinvb + blockIdx.x * sR;
  for (int i = threadIdx.x; i < k; i += blockDim.x) rinv[i] = S[(int64_t)i * k + i];  // original diagonal
  __syncthreads();
  for (int j0 = 0; j0 < k; j0 += nbmax) {
    const int nb = min(nbmax, k - j0), w = k - j0;
    for (int e = threadIdx.x; e < nb * w; e += blockDim.x) {
      const int r = e / w, c = e % w;
      P[r * w + c] = S[(int64_t)(j0 + r) * k + j0 + c];
    }
    for (int r = threadIdx.x; r < nb; r += blockDim.x) dg[r] = rinv[j0 + r];
    __syncthreads();
    for (int j = 0; j < nb; ++j) {
      const double d = P[j * w + j], o = dg[j];
      const bool keep = o > 0.0 && d > 1e-10 * o;
      const double rs = keep ? 1.0 / sqrt(d) : 0.0;
      const double inv_d = rs * rs;
      // row j - 1 takes its scaling one step late; rows i > j the rank-1
      // update by row j (columns c >= i)
      if (j > 0)
        for (int c = j - 1 + threadIdx.x; c < w; c += blockDim.x) P[(j - 1) * w + c] *= ri[j - 1];
      for (int i = j + 1; i < nb; ++i) {
        const double f = P[j * w + i] * inv_d;
        for (int c = i + threadIdx.x; c < w; c += blockDim.x) P[i * w + c] = fma(-f, P[j * w + c], P[i * w + c]);
      }
      if (threadIdx.x == 0) ri[j] = rs;
      __syncthreads();
    }
    for (int c = nb - 1 + threadIdx.x; c < w; c += blockDim.x) P[(nb - 1) * w + c] *= ri[nb - 1];
    __syncthreads();
    // the panel rows of R (upper part) and their inverse pivots
    for (int e = threadIdx.x; e < nb * w; e += blockDim.x) {
      const int r = e / w, c = e % w;
      S[(int64_t)(j0 + r) * k + j0 + c] = c >= r ? P[r * w + c] : 0.0;
    }
    for (int r = threadIdx.x; r < nb; r += blockDim.x) rinv[j0 + r] = ri[r];
    // trailing update of the upper triangle: S[i][c] -= sum_r R[r][i] R[r][c]
    const int m = w - nb, T = (m + 3) / 4;
    for (int t = threadIdx.x; t < T * T; t += blockDim.x) {
      const int ta = t / T, tb = t % T;
      if (tb < ta) continue;
      double acc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0;
      const int ib = nb + 4 * ta, cb = nb + 4 * tb;
      for (int r = 0; r < nb; ++r) {
        double x[4], y[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) x[a] = ib + a < w ? P[r * w + ib + a] : 0.0;
#pragma unroll
        for (int b = 0; b < 4; ++b) y[b] = cb + b < w ? P[r * w + cb + b] : 0.0;
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[a][b] = fma(x[a], y[b], acc[a][b]);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int i = ib + a, c = cb + b;
          if (i < w && c < w && c >= i) S[(int64_t)(j0 + i) * k + j0 + c] -= acc[a][b];
        }
    }
    __syncthreads();
  }
}

// Multi-CTA Cholesky for the wider sketches, left-looking by panels of CHP
// rows, one launch per panel: CTA b of a panel takes the panel rows' columns
// [j0 + 32 b, j0 + 32 b + 32).  It subtracts the earlier panels' rows of R
// (staged 32 x 32 blocks, the next one loaded into registers while the
// current one is used), eliminates the panel's diagonal block (every CTA,
// redundantly: the pivots and multipliers of its columns) with the rank
// dropping of chol_kernel, and writes its columns of the panel rows of R
// into the upper triangle.  The original values come from the lower
// triangle of S (the Gram is a full symmetric product and the upper
// triangle only is overwritten) and from dg0, the original diagonal, so no
// CTA reads what another CTA of the same launch writes.
constexpr int CHP = 32;
constexpr int CHP_MIN_K = 64;  // narrower sketches keep the single-CTA chol_kernel

__global__ void chol_diag_copy_kernel(const double* Sb, int k, int64_t sS, double* dg0b, int64_t sD) {
  const double* S = Sb + blockIdx.y * sS;
  double* dg0 = dg0b + blockIdx.y * sD;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < k; i += gridDim.x * blockDim.x)
    dg0[i] = S[(int64_t)i * k + i];
}

__global__ void __launch_bounds__(256, 1) chol_panel_kernel(double* Sb, int k, int64_t sS, double* rinvb, int64_t sR,
                                                         const double* dg0b, int64_t sD, int j0) {
  __shared__ double D[CHP][CHP + 1];   // the panel's diagonal block: D[r][q], q >= r
  __shared__ double Sl[CHP][CHP + 1];  // the panel rows of this CTA's columns
  __shared__ double A[CHP][CHP + 1];   // R[i0 + i][j0 + r] of the current chunk
  __shared__ double B[CHP][CHP + 1];   // R[i0 + i][c0 + c] of the current chunk
  __shared__ double rsv[CHP];
  __shared__ double dgs[CHP];  // the panel's original diagonal (read once, not per pivot)
  const int cell = blockIdx.y, blk = blockIdx.x;
  double* S = Sb + cell * sS;
  double* rinv = rinvb + cell * sR;
  const double* dg0 = dg0b + cell * sD;
  const int nb = min(CHP, k - j0);
  const int c0 = j0 + blk * CHP, ncol = min(CHP, k - c0);
  const bool diag = blk == 0;
  const int tr = threadIdx.x >> 3, tq = (threadIdx.x & 7) * 4;  // 4 outputs a thread: row tr, columns tq..tq+3
  if ((int)threadIdx.x < nb) dgs[threadIdx.x] = dg0[j0 + threadIdx.x];
  double pd[4], ps[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int qq = tq + q;
    pd[q] = 0.0;
    ps[q] = 0.0;
    if (tr < nb && qq < nb && qq >= tr) pd[q] = qq == tr ? dg0[j0 + tr] : S[(int64_t)(j0 + qq) * k + j0 + tr];
    if (!diag && tr < nb && qq < ncol) ps[q] = S[(int64_t)(c0 + qq) * k + j0 + tr];
  }
  // the earlier panels: P -= sum_{i < j0} R[i][j0 + r] R[i][column]
  double na[4], nbv[4];
  auto fetch = [&](int i0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = threadIdx.x + 256 * j, i = e >> 5, c = e & 31;
      na[j] = c < nb ? S[(int64_t)(i0 + i) * k + j0 + c] : 0.0;
      nbv[j] = (!diag && c < ncol) ? S[(int64_t)(i0 + i) * k + c0 + c] : 0.0;
    }
  };
  if (j0 > 0) fetch(0);
  for (int i0 = 0; i0 < j0; i0 += CHP) {  // j0 is a multiple of CHP: whole chunks of finished rows
    __syncthreads();  // the previous chunk is consumed
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = threadIdx.x + 256 * j, i = e >> 5, c = e & 31;
      A[i][c] = na[j];
      B[i][c] = nbv[j];
    }
    __syncthreads();
    if (i0 + CHP < j0) fetch(i0 + CHP);
#pragma unroll 4
    for (int i = 0; i < CHP; ++i) {
      const double a = A[i][tr];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pd[q] = fma(-a, A[i][tq + q], pd[q]);
        ps[q] = fma(-a, B[i][tq + q], ps[q]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    D[tr][tq + q] = pd[q];
    Sl[tr][tq + q] = ps[q];
  }
  __syncthreads();
  // the panel: pivot r, row r - 1 scaled one step late, rows q > r updated
  // with the unscaled row r times 1 / d
  for (int r = 0; r < nb; ++r) {
    if (threadIdx.x == 0) {
      const double d = D[r][r], o = dgs[r];
      rsv[r] = (o > 0.0 && d > 1e-10 * o) ? 1.0 / sqrt(d) : 0.0;
    }
    __syncthreads();
    const double inv_d = rsv[r] * rsv[r];
    if (r > 0) {
      const double rs = rsv[r - 1];
      for (int x = r - 1 + threadIdx.x; x < nb; x += blockDim.x) D[r - 1][x] *= rs;
      if (!diag && (int)threadIdx.x < ncol) Sl[r - 1][threadIdx.x] *= rs;
    }
    for (int e = threadIdx.x; e < (nb - 1 - r) * CHP; e += blockDim.x) {
      const int q = r + 1 + (e >> 5), x = e & 31;
      const double f = D[r][q] * inv_d;
      if (x >= q && x < nb) D[q][x] = fma(-f, D[r][x], D[q][x]);
      if (!diag && x < ncol) Sl[q][x] = fma(-f, Sl[r][x], Sl[q][x]);
    }
    __syncthreads();
  }
  {
    const double rs = rsv[nb - 1];
    for (int x = nb - 1 + threadIdx.x; x < nb; x += blockDim.x) D[nb - 1][x] *= rs;
    if (!diag && (int)threadIdx.x < ncol) Sl[nb - 1][threadIdx.x] *= rs;
  }
  __syncthreads();
  // the panel rows of R: the diagonal CTA writes the block's upper triangle
  // and the inverse pivots, the others their columns
  for (int e = threadIdx.x; e < nb * CHP; e += blockDim.x) {
    const int r = e >> 5, x = e & 31;
    if (diag) {
      if (x >= r && x < nb) S[(int64_t)(j0 + r) * k + j0 + x] = D[r][x];
    } else if (x < ncol) {
      S[(int64_t)(j0 + r) * k + c0 + x] = Sl[r][x];
    }
  }
  if (diag && (int)threadIdx.x < nb) rinv[j0 + threadIdx.x] = rsv[threadIdx.x];
}

constexpr int TS_ROWS = 16;  // rows of W per CTA: 16 lanes of a warp per row
constexpr int TS_NT = 256;

// Staged blocks of R for the row solves: 32 x 32 doubles at row stride RS_LD
// (padded: every read pattern below is conflict-free), a ring of NBUF of
// them filled by 8-byte cp.async copies (zero outside the k x k matrix)
// NBUF - 1 blocks ahead of their use, so the L2 latency of R overlaps the
// arithmetic instead of sitting in every dependent step.
constexpr int RS_LD = 33;
constexpr int RS_BLOCK = 32 * RS_LD;  // doubles per staged block

__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(valid ? 8 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit8() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait8() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Block s of a row solve's sequence over the nbk x nbk blocks of R:
// forward (w R^{-1}): column blocks jb = 0, 1, ..; in each, the update blocks
// ib < jb then the diagonal; transposed (w R^{-T}): jb = nbk - 1 down to 0;
// in each, the update blocks ib = nbk - 1 .. jb + 1 then the diagonal.
// (rb, cb): the block's row and column block of R.
struct SolveSeq {
  int jb, ib;
};
template <bool TRANS>
__device__ __forceinline__ void seq_first(SolveSeq& q, int nbk) {
  if (TRANS) {
    q.jb = nbk - 1;
    q.ib = nbk - 1;
  } else {
    q.jb = 0;
    q.ib = 0;
  }
}
template <bool TRANS>
__device__ __forceinline__ void seq_next(SolveSeq& q, int nbk) {
  if (TRANS) {
    if (q.ib > q.jb) --q.ib;
    else {
      --q.jb;
      q.ib = nbk - 1;
    }
  } else {
    if (q.ib < q.jb) ++q.ib;
    else {
      ++q.jb;
      q.ib = 0;
    }
  }
}

template <bool TRANS>
__device__ __forceinline__ void stage_block(double* buf, const double* __restrict__ R, int k, const SolveSeq& q) {
  const int rb = TRANS ? q.jb : q.ib, cbk = TRANS ? q.ib : q.jb;
  for (int e = threadIdx.x; e < 1024; e += blockDim.x) {
    const int i = e >> 5, c = e & 31, r = rb * 32 + i, col = cbk * 32 + c;
    const bool ok = r < k && col < k;
    cp_async8(buf + i * RS_LD + c, ok ? R + (int64_t)r * k + col : R, ok);
  }
}

// w <- w R^{-1} (TRANS: w <- w R^{-T}) for the blockDim / 16 rows w of Wl
// (row stride ldw; row threadIdx / 16, lane threadIdx % 16; every thread of
// the block calls it): R upper triangular (k x k, row stride k), rinv its
// inverse pivots, Rs NBUF staged blocks.  Column blocks of 32: the rank
// update by the finished columns (lane l owns columns l and l + 16 of the
// block), then the block's substitution column by column, the 16 lanes of a
// row splitting each dot product.
//   forward:    y_c = (w_c - sum_{i < c} y_i R[i][c]) / R[c][c]
//   transposed: y_j = (w_j - sum_{i > j} y_i R[j][i]) / R[j][j]
template <bool TRANS, int NBUF>
__device__ void rows_solve(double* Wl, int ldw, int k, const double* __restrict__ R,
                           const double* __restrict__ rinv, double* Rs) {
  const int r = threadIdx.x >> 4, lane = threadIdx.x & 15;
  double* wr = Wl + r * ldw;
  const int nbk = (k + 31) / 32;
  const int total = nbk * (nbk + 1) / 2;
  SolveSeq pre, cur;
  seq_first<TRANS>(pre, nbk);
  seq_first<TRANS>(cur, nbk);
  __syncthreads();  // Rs is free (an earlier solve has consumed it)
#pragma unroll 1
  for (int n = 0; n < NBUF - 1; ++n) {
    if (n < total) {
      stage_block<TRANS>(Rs + n * RS_BLOCK, R, k, pre);
      seq_next<TRANS>(pre, nbk);
    }
    cp_async_commit8();
  }
  double a0 = 0.0, a1 = 0.0;
#pragma unroll 1
  for (int n = 0; n < total; ++n) {
    cp_async_wait8<NBUF - 2>();
    __syncthreads();  // block n is in; every thread is done with block n - 1
    if (n + NBUF - 1 < total) {
      stage_block<TRANS>(Rs + ((n + NBUF - 1) % NBUF) * RS_BLOCK, R, k, pre);
      seq_next<TRANS>(pre, nbk);
    }
    cp_async_commit8();
    const double* B = Rs + (n % NBUF) * RS_BLOCK;
    const int J0 = cur.jb * 32, cb = min(32, k - J0);
    if (cur.ib != cur.jb) {
      const int I0 = cur.ib * 32, ni = min(32, k - I0);
      if (!TRANS) {
        // forward update: rows I0 + i of R (all < k: ib < jb), columns J0 + lane (+16)
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
          const double wi = wr[I0 + i];
          a0 = fma(wi, B[i * RS_LD + lane], a0);
          a1 = fma(wi, B[i * RS_LD + lane + 16], a1);
        }
      } else {
        // transposed update: rows J0 + lane (+16) of R, columns I0 + i < k
        for (int i = 0; i < ni; ++i) {
          const double yi = wr[I0 + i];
          a0 = fma(yi, B[lane * RS_LD + i], a0);
          a1 = fma(yi, B[(lane + 16) * RS_LD + i], a1);
        }
      }
    } else {
      // the diagonal block: apply the update, then substitute column by column
      // (the block's inverse pivots in registers, lane l holding columns l
      // and l + 16: one load instead of one dependent load a column)
      const double ri0 = lane < cb ? rinv[J0 + lane] : 0.0, ri1 = lane + 16 < cb ? rinv[J0 + lane + 16] : 0.0;
      if (lane < cb) wr[J0 + lane] -= a0;
      if (lane + 16 < cb) wr[J0 + lane + 16] -= a1;
      a0 = a1 = 0.0;
      __syncwarp();
      if (!TRANS) {
        for (int c = 0; c < cb; ++c) {
          double part = 0.0;
          if (lane < c) part = wr[J0 + lane] * B[lane * RS_LD + c];
          if (lane + 16 < c) part = fma(wr[J0 + lane + 16], B[(lane + 16) * RS_LD + c], part);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o, 16);
          const double ric = __shfl_sync(0xffffffffu, c < 16 ? ri0 : ri1, c & 15, 16);
          if (lane == 0) wr[J0 + c] = (wr[J0 + c] - part) * ric;
          __syncwarp();
        }
      } else {
        for (int c = cb - 1; c >= 0; --c) {
          double part = 0.0;
          if (lane > c && lane < cb) part = wr[J0 + lane] * B[c * RS_LD + lane];
          if (lane + 16 > c && lane + 16 < cb) part = fma(wr[J0 + lane + 16], B[c * RS_LD + lane + 16], part);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o, 16);
          const double ric = __shfl_sync(0xffffffffu, c < 16 ? ri0 : ri1, c & 15, 16);
          if (lane == 0) wr[J0 + c] = (wr[J0 + c] - part) * ric;
          __syncwarp();
        }
      }
    }
    seq_next<TRANS>(cur, nbk);
  }
  cp_async_wait8<0>();
  __syncthreads();
}

__global__ void identity_kernel(double* Ab, int k, int64_t sA) {
  double* A = Ab + blockIdx.y * sA;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < (int64_t)k * k; e += (int64_t)gridDim.x * blockDim.x)
    A[e] = (e / k == e % k) ? 1.0 : 0.0;
}

// W <- W R^{-1} per cell (R upper triangular from chol_kernel, rinv its
// inverse pivots; a dropped column of R gives a zero column of W).  Each CTA
// holds TS_ROWS rows of W in shared memory and sweeps the columns in blocks
// of 32: first the rank update by the finished columns (R read through L1,
// shared by every row), then the block's own forward substitution, column by
// column, with the 16 lanes of a row splitting each dot product.
// X[r][c] (nb rows of stride ldx; zero past k and in rows r >= nr) <-
// src[r][c] (rows of length k, written by an earlier launch): eight loads in
// flight a thread before their stores.
__device__ inline void load_rows(double* X, int ldx, const double* __restrict__ src, int nb, int nr, int k) {
  const int n = nb * ldx;
  for (int e0 = threadIdx.x; e0 < n; e0 += 8 * blockDim.x) {
    double v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * (int)blockDim.x, r = e / ldx, c = e - r * ldx;
      v[q] = (e < n && c < k && r < nr) ? __ldg(src + (int64_t)r * k + c) : 0.0;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * (int)blockDim.x;
      if (e < n) X[e] = v[q];
    }
  }
}

constexpr int TS_NBUF = 8;  // staged blocks of R in flight per CTA

__global__ void __launch_bounds__(TS_NT) trsm_kernel(double* Wb, int p, int k, int64_t sW, const double* Rb,
                                                     int64_t sR, const double* rinvb, int64_t sri) {
  extern __shared__ double Wl[];  // TS_ROWS x k, then TS_NBUF staged blocks of R
  const int cell = blockIdx.y;
  double* W = Wb + cell * sW;
  const double* R = Rb + cell * sR;
  const double* rinv = rinvb + cell * sri;
  const int row0 = blockIdx.x * TS_ROWS;
  const int nr = min(TS_ROWS, p - row0);
  load_rows(Wl, k, W + (int64_t)row0 * k, TS_ROWS, nr, k);
  __syncthreads();
  rows_solve<false, TS_NBUF>(Wl, k, k, R, rinv, Wl + (size_t)TS_ROWS * k);
  for (int e = threadIdx.x; e < nr * k; e += blockDim.x) {
    const int rr = e / k, c = e % k;
    W[(int64_t)(row0 + rr) * k + c] = Wl[e];
  }
}

// Offsets (doubles) of the randomised multi-launch path's per-cell workspace.
struct LrLayout {
  int64_t W, Z, S, C, Zt, vec, lam, rinv, misc, scr, total;
};

LrLayout lr_layout(int p, int k) {
  LrLayout L;
  L.W = 0;
  L.Z = L.W + (int64_t)p * k;
  L.S = L.Z + (int64_t)p * k;
  L.C = L.S + (int64_t)k * k;
  L.Zt = L.C + (int64_t)k * k;
  L.vec = L.Zt + (int64_t)k * k;
  L.lam = L.vec + eig::vec_doubles(k);
  L.rinv = L.lam + k;
  L.misc = L.rinv + k;
  L.scr = L.misc + 4;
  L.total = L.scr + eig_scratch_doubles(k);
  return L;
}

// W = the starting sketch (LEFT: Y0 = A Omega from the Gram buffer; RIGHT:
// Omega), misc[0] = |A|_F^2.
// (grid: blocks x cells; block 0 of a cell also writes misc[0])
__global__ void lr_init_kernel(SolveArgs a, LrLayout L) {
  const int cell = blockIdx.y, p = a.p, k = a.k;
  const double* gram = a.gram + cell * a.gram_stride;
  double* ws = a.ws + cell * a.ws_cell;
  const int64_t n = (int64_t)p * k, step = (int64_t)gridDim.x * blockDim.x;
  if (a.side == KVC_SIDE_LEFT) {
    const double* y0 = gram + (int64_t)p * p;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += step) ws[L.W + i] = y0[i];
    if (blockIdx.x == 0 && threadIdx.x == 0) ws[L.misc] = gram[(int64_t)p * p + (int64_t)p * k];
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += step)
      ws[L.W + i] = (double)a.omega[i];
    if (blockIdx.x == 0) {
      __shared__ double red[64];
      double part = 0.0;
      for (int i = threadIdx.x; i < p; i += blockDim.x) part += gram[(int64_t)i * p + i];
      const double t = eig::block_sum(part, red);
      if (threadIdx.x == 0) ws[L.misc] = t;
    }
  }
}

// The Ritz pairs: the rank leading eigenpairs of C; tail and sv2.
__global__ void __launch_bounds__(SNT) lr_eig_kernel(SolveArgs a, LrLayout L) {
  __shared__ double red[64];
  __shared__ int cnt[SNT];
  const int cell = blockIdx.x, k = a.k, rank = a.rank;
  double* ws = a.ws + cell * a.ws_cell;
  double* lam = ws + L.lam;
  eig::eig_top(ws + L.C, k, k, rank, lam, ws + L.Zt, k, ws + L.vec, cnt, red, ws + L.scr, SNT);
  if (threadIdx.x == 0) {
    double retained = 0.0;
    for (int i = 0; i < rank; ++i) retained += fmax(lam[i], 0.0);
    const double nrm = ws[L.misc];
    const double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[cell] = t > 0.0 ? t : 0.0;
    if (a.sv2)
      for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = fmax(lam[i], 0.0);
  }
}

// LEFT basis: the product in the Z slot rounded to the basis dtype.
__global__ void lr_store_kernel(SolveArgs a, LrLayout L) {
  const int cell = blockIdx.y;
  const double* z = a.ws + cell * a.ws_cell + L.Z;
  const int64_t n = (int64_t)a.p * a.rank;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_dt(a.basis, (int64_t)cell * n + i, (float)z[i], a.basis_dtype);
}

// ---------------------------------------------------------------------------
// The Ritz step of wide sketches when no singular values are asked for (every
// compress call): the span of the `rank` leading Ritz vectors is the
// complement, inside the sketch space, of the s = k - rank trailing ones, and
// s is at most the oversampling.  So only the trailing ones are found: block
// inverse iteration on C + delta I (nb = 16 vectors for s <= 4, else 32;
// (C + delta I)^-1 = R^-1 R^-T formed once from its Cholesky factor, each
// step W <- W (C + delta I)^-1 and CholeskyQR2 of the rows), a
// Rayleigh-Ritz on the nb x nb projection, then
// Householder reflectors H_0 .. H_{s-1} of the s trailing vectors; the basis
// is (W H_0 ... H_{s-1})[:, s:].  Its columns are an orthonormal basis of
// the same Ritz subspace (not ordered by singular value); the tail mass is
// exact: |A|^2 - trace(C) + the s trailing Ritz values.
// ---------------------------------------------------------------------------
constexpr int CP_MIN_K = 129;  // sketches at least this wide take the complement path
constexpr int CP_MAX_S = 16;   // largest k - rank it handles
constexpr int IV_GROUP = 16;   // vectors when 32 do not fit in shared memory
constexpr int IV_MAX = 32;     // vectors of the block inverse iteration (16 threads each)
constexpr int IV_ITERS = 20;   // steps: trailing Ritz values of flat spectra to ~1e-9 of |A|^2
constexpr int CP_NBUF = 4;     // staged blocks of R in flight in the row solves

// C += delta I (delta = 1e-13 of its largest diagonal entry, so the
// Cholesky succeeds on a semi-definite C); misc[1] = trace(C), misc[2] = delta.
__global__ void cp_shift_kernel(double* wsb, int64_t cs, LrLayout L, int k) {
  __shared__ double red[64];
  __shared__ double mm[2];
  double* ws = wsb + blockIdx.x * cs;
  double* C = ws + L.C;
  double tr = 0.0, mx = 0.0;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const double v = C[(int64_t)i * k + i];
    tr += v;
    mx = fmax(mx, v);
  }
  tr = eig::block_sum(tr, red);
  eig::block_minmax(mx, mx, red, mm);
  const double delta = 1e-13 * mm[1] + 1e-300;
  for (int i = threadIdx.x; i < k; i += blockDim.x) C[(int64_t)i * k + i] += delta;
  if (threadIdx.x == 0) {
    ws[L.misc + 1] = tr;
    ws[L.misc + 2] = delta;
  }
}

// CholeskyQR of the nb (<= IV_MAX) rows of X (row stride ldx, length k):
// G = X X^T, its Cholesky L (rank dropping as chol_kernel), X <- L^{-1} X
// column by column.
__device__ inline void cp_orth_rows(double* X, int ldx, int k, int nb, double* G) {
  for (int e = threadIdx.x; e < nb * nb; e += blockDim.x) {
    const int a = e / nb, b = e % nb;
    if (b > a) continue;
    const double* xa = X + a * ldx;
    const double* xb = X + b * ldx;
    double s0 = 0.0, s1 = 0.0;
    int i = 0;
    for (; i + 1 < k; i += 2) {
      s0 = fma(xa[i], xb[i], s0);
      s1 = fma(xa[i + 1], xb[i + 1], s1);
    }
    if (i < k) s0 = fma(xa[i], xb[i], s0);
    G[a * IV_MAX + b] = s0 + s1;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // G = L L^T in place (lower), rank dropping; L[j][j] stored inverted.
    // Left-looking by columns; lane i > j forms L[i][j] (the sums in the
    // order of the scalar recurrence)
    const int lane = threadIdx.x;
    for (int j = 0; j < nb; ++j) {
      const double o = G[j * IV_MAX + j];
      double d = o;
      for (int q = 0; q < j; ++q) d -= G[j * IV_MAX + q] * G[j * IV_MAX + q];
      const double ri = (o > 0.0 && d > 1e-10 * o) ? 1.0 / sqrt(d) : 0.0;
      if (lane > j && lane < nb) {
        double v = G[lane * IV_MAX + j];
        for (int q = 0; q < j; ++q) v -= G[lane * IV_MAX + q] * G[j * IV_MAX + q];
        G[lane * IV_MAX + j] = v * ri;
      }
      __syncwarp();
      if (lane == 0) G[j * IV_MAX + j] = ri;
      __syncwarp();
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    double x[IV_MAX];
#pragma unroll
    for (int q = 0; q < IV_MAX; ++q) x[q] = q < nb ? X[q * ldx + c] : 0.0;
#pragma unroll
    for (int q = 0; q < IV_MAX; ++q) {
      if (q >= nb) break;
      double v = x[q];
      for (int j = 0; j < q; ++j) v -= G[q * IV_MAX + j] * x[j];
      x[q] = v * G[q * IV_MAX + q];
      X[q * ldx + c] = x[q];
    }
  }
  __syncthreads();
}

// The block inverse iteration on nb vectors, in launches: cp_start_kernel
// (the start block, orthonormalised), then per step iv_mult_kernel (X C^-1
// over a grid of one CTA per 32 columns) and iv_orth_kernel (CholeskyQR2 of
// the block), then cp_bottom_kernel.  The block lives in the workspace at
// xoff (nb rows of length k), the product at xnoff.
__global__ void __launch_bounds__(16 * IV_MAX) cp_start_kernel(SolveArgs a, int nb, int ldx, int64_t xoff) {
  extern __shared__ double X[];  // nb rows of stride ldx
  __shared__ double G[IV_MAX * IV_MAX];
  const int k = a.k;
  double* out = a.ws + blockIdx.x * a.ws_cell + xoff;
  for (int e = threadIdx.x; e < nb * ldx; e += blockDim.x) {
    const int r = e / ldx, c = e % ldx;
    X[e] = c < k ? eig::start_entry(r, c) : 0.0;
  }
  __syncthreads();
  cp_orth_rows(X, ldx, k, nb, G);
  cp_orth_rows(X, ldx, k, nb, G);
  for (int e = threadIdx.x; e < nb * k; e += blockDim.x) {
    const int r = e / k, c = e - r * k;
    out[e] = X[r * ldx + c];
  }
}

// Columns [32 jb, 32 jb + 32) of X (C + delta I)^-1 (the inverse in the S
// slot), jb = blockIdx.x: the block's rows in shared memory, the inverse's
// column block streamed through the ring of staged blocks; thread (row
// threadIdx / 16, lane) owns columns lane and lane + 16.
__global__ void __launch_bounds__(16 * IV_MAX) iv_mult_kernel(SolveArgs a, LrLayout L, int nb, int ldx, int64_t xoff,
                                                              int64_t xnoff) {
  extern __shared__ double X[];  // nb rows of stride ldx, then CP_NBUF staged blocks
  const int cell = blockIdx.y, jb = blockIdx.x, k = a.k;
  double* ws = a.ws + cell * a.ws_cell;
  const double* Cinv = ws + L.S;
  const double* xin = ws + xoff;
  double* out = ws + xnoff;
  double* Rs = X + (size_t)nb * ldx;
  load_rows(X, ldx, xin, nb, nb, k);
  const int r = threadIdx.x >> 4, lane = threadIdx.x & 15;
  const double* xr = X + r * ldx;
  const int nbk = (k + 31) / 32;
  auto stage = [&](int ib, double* buf) {
    for (int e = threadIdx.x; e < 1024; e += blockDim.x) {
      const int i = e >> 5, c = e & 31, row = ib * 32 + i, col = jb * 32 + c;
      const bool ok = row < k && col < k;
      cp_async8(buf + i * RS_LD + c, ok ? Cinv + (int64_t)row * k + col : Cinv, ok);
    }
  };
#pragma unroll 1
  for (int n = 0; n < CP_NBUF - 1; ++n) {
    if (n < nbk) stage(n, Rs + n * RS_BLOCK);
    cp_async_commit8();
  }
  double a0 = 0.0, a1 = 0.0;
#pragma unroll 1
  for (int ib = 0; ib < nbk; ++ib) {
    cp_async_wait8<CP_NBUF - 2>();
    __syncthreads();  // block ib is in (and, the first time, the rows of X)
    if (ib + CP_NBUF - 1 < nbk) stage(ib + CP_NBUF - 1, Rs + ((ib + CP_NBUF - 1) % CP_NBUF) * RS_BLOCK);
    cp_async_commit8();
    const double* B = Rs + (ib % CP_NBUF) * RS_BLOCK;
    const int I0 = ib * 32;
    if (k - I0 >= 32) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const double xi = xr[I0 + i];
        a0 = fma(xi, B[i * RS_LD + lane], a0);
        a1 = fma(xi, B[i * RS_LD + lane + 16], a1);
      }
    } else {
      for (int i = 0; i < k - I0; ++i) {
        const double xi = xr[I0 + i];
        a0 = fma(xi, B[i * RS_LD + lane], a0);
        a1 = fma(xi, B[i * RS_LD + lane + 16], a1);
      }
    }
  }
  cp_async_wait8<0>();
  const int c = jb * 32 + lane;
  if (c < k) out[(int64_t)r * k + c] = a0;
  if (c + 16 < k) out[(int64_t)r * k + c + 16] = a1;
}

// CholeskyQR2 of the product block (xnoff) back into the block (xoff).
__global__ void __launch_bounds__(16 * IV_MAX) iv_orth_kernel(SolveArgs a, int nb, int ldx, int64_t xnoff,
                                                              int64_t xoff) {
  extern __shared__ double X[];  // nb rows of stride ldx
  __shared__ double G[IV_MAX * IV_MAX];
  const int k = a.k;
  double* ws = a.ws + blockIdx.x * a.ws_cell;
  const double* xin = ws + xnoff;
  double* out = ws + xoff;
  load_rows(X, ldx, xin, nb, nb, k);
  __syncthreads();
  cp_orth_rows(X, ldx, k, nb, G);
  cp_orth_rows(X, ldx, k, nb, G);
  for (int e = threadIdx.x; e < nb * k; e += blockDim.x) {
    const int r = e / k, c = e - r * k;
    out[e] = X[r * ldx + c];
  }
}

// One CTA of 16 nb threads per cell, after the inverse iteration: the
// Rayleigh-Ritz on the converged block (xoff), the s trailing Ritz vectors,
// their Householder reflectors (v_q in the S slot, rows of length k; tau_q in
// the lam slot) and the tail mass.
__global__ void __launch_bounds__(16 * IV_MAX, 1) cp_bottom_kernel(SolveArgs a, LrLayout L, int s, int nb, int ldx,
                                                                 int64_t xoff) {
  extern __shared__ double X[];  // nb rows of stride ldx
  __shared__ double G[IV_MAX * IV_MAX], T[IV_MAX * IV_MAX], Mb[IV_MAX * 32];
  __shared__ double Zs[CP_MAX_S * IV_MAX], vec[8 * IV_MAX], lam[IV_MAX], red[64];
  __shared__ double scr[3 * IV_MAX * CP_MAX_S];
  __shared__ int cnt[16 * IV_MAX];
  const int cell = blockIdx.x, k = a.k;
  double* ws = a.ws + cell * a.ws_cell;
  const double* R = ws + L.C;
  const double* xin = ws + xoff;
  load_rows(X, ldx, xin, nb, nb, k);
  __syncthreads();
  // T = (X R^T)(X R^T)^T - delta I = X C X^T, 32 columns of M = X R^T at a time
  for (int e = threadIdx.x; e < IV_MAX * IV_MAX; e += blockDim.x) T[e] = 0.0;
  __syncthreads();
  for (int J0 = 0; J0 < k; J0 += 32) {
    for (int e = threadIdx.x; e < nb * 32; e += blockDim.x) {
      const int r = e >> 5, jj = e & 31, j = J0 + jj;
      double m = 0.0;
      if (j < k) {
        const double* xr = X + r * ldx;
        for (int i = j; i < k; ++i) m = fma(xr[i], __ldg(R + (int64_t)j * k + i), m);
      }
      Mb[e] = m;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb * nb; e += blockDim.x) {
      const int r = e / nb, q = e % nb;
      double t = 0.0;
#pragma unroll 8
      for (int jj = 0; jj < 32; ++jj) t = fma(Mb[r * 32 + jj], Mb[q * 32 + jj], t);
      T[r * IV_MAX + q] += t;
    }
    __syncthreads();
  }
  // the s trailing eigenpairs of T = the s leading ones of -T
  const double delta = ws[L.misc + 2];
  for (int e = threadIdx.x; e < IV_MAX * IV_MAX; e += blockDim.x) {
    const int r = e / IV_MAX, q = e % IV_MAX;
    G[e] = (r < nb && q < nb) ? -(T[e] - (r == q ? delta : 0.0)) : 0.0;
  }
  __syncthreads();
  eig::eig_top(G, IV_MAX, nb, s, lam, Zs, IV_MAX, vec, cnt, red, scr, s);
  // tail = 1 - (trace C - sum of the trailing Ritz values) / |A|^2
  if (threadIdx.x == 0) {
    double trailing = 0.0;
    for (int q = 0; q < s; ++q) trailing += fmax(-lam[q], 0.0);
    const double retained = ws[L.misc + 1] - (double)k * delta - trailing;
    const double nrm = ws[L.misc];
    const double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[cell] = t > 0.0 ? t : 0.0;
  }
  // the trailing Ritz vectors X_s = Zs X (s rows), column by column in place
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    double x[IV_MAX];
#pragma unroll
    for (int q = 0; q < IV_MAX; ++q) x[q] = q < nb ? X[q * ldx + c] : 0.0;
    for (int q = 0; q < s; ++q) {
      double v = 0.0;
#pragma unroll
      for (int j = 0; j < IV_MAX; ++j) v = fma(Zs[q * IV_MAX + j], x[j], v);
      X[q * ldx + c] = v;
    }
  }
  __syncthreads();
  // Householder QR of X_s^T (k x s): reflector q on entries q .. k-1
  double* V = ws + L.S;     // v_q as rows of length k
  double* tau = ws + L.lam;
  for (int q = 0; q < s; ++q) {
    double* xq = X + q * ldx;
    double part = 0.0;
    for (int i = q + 1 + threadIdx.x; i < k; i += blockDim.x) part = fma(xq[i], xq[i], part);
    const double sig = eig::block_sum(part, red);
    const double x0 = xq[q];
    double tq = 0.0, v0 = x0;
    if (sig > 0.0 || x0 < 0.0) {
      const double nx = sqrt(fma(x0, x0, sig));
      const double alpha = x0 >= 0.0 ? -nx : nx;
      v0 = x0 - alpha;
      tq = 2.0 / fma(v0, v0, sig);
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x) V[(int64_t)q * k + i] = i < q ? 0.0 : (i == q ? v0 : xq[i]);
    if (threadIdx.x == 0) tau[q] = tq;
    __syncthreads();
    const double* vq = V + (int64_t)q * k;
    for (int q2 = q + 1; q2 < s; ++q2) {
      double* y = X + q2 * ldx;
      double pd = 0.0;
      for (int i = q + threadIdx.x; i < k; i += blockDim.x) pd = fma(vq[i], y[i], pd);
      const double dot = eig::block_sum(pd, red) * tq;
      for (int i = q + threadIdx.x; i < k; i += blockDim.x) y[i] = fma(-dot, vq[i], y[i]);
      __syncthreads();
    }
  }
}

// s = 0: the basis is the sketch space, the tail 1 - trace(C) / |A|^2.
__global__ void cp_tail_kernel(SolveArgs a, LrLayout L, int n_cells) {
  for (int c = threadIdx.x; c < n_cells; c += blockDim.x) {
    const double* ws = a.ws + c * a.ws_cell;
    const double nrm = ws[L.misc];
    const double retained = ws[L.misc + 1];
    const double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[c] = t > 0.0 ? t : 0.0;
  }
}

// basis rows = (w H_0 ... H_{s-1})[s:] for every row w of W (16 rows per
// CTA, 16 lanes per row); the reflectors from cp_bottom_kernel.
__global__ void __launch_bounds__(TS_NT) cp_complement_kernel(SolveArgs a, LrLayout L, int64_t w_off, int s) {
  extern __shared__ double Wl[];  // TS_ROWS x k
  const int cell = blockIdx.y, p = a.p, k = a.k, rank = a.rank;
  const double* ws = a.ws + cell * a.ws_cell;
  const double* W = ws + w_off;
  const double* V = ws + L.S;
  const double* tau = ws + L.lam;
  const int row0 = blockIdx.x * TS_ROWS;
  const int nr = min(TS_ROWS, p - row0);
  for (int e = threadIdx.x; e < TS_ROWS * k; e += blockDim.x) {
    const int r = e / k, c = e % k;
    Wl[e] = r < nr ? W[(int64_t)(row0 + r) * k + c] : 0.0;
  }
  __syncthreads();
  const int r = threadIdx.x >> 4, lane = threadIdx.x & 15;
  double* wr = Wl + r * k;
  for (int q = 0; q < s; ++q) {
    const double* vq = V + (int64_t)q * k;
    double part = 0.0;
    for (int i = q + lane; i < k; i += 16) part = fma(wr[i], __ldg(vq + i), part);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o, 16);
    const double dot = part * tau[q];
    for (int i = q + lane; i < k; i += 16) wr[i] = fma(-dot, __ldg(vq + i), wr[i]);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < nr * rank; e += blockDim.x) {
    const int rr = e / rank, c = e % rank;
    const double v = Wl[rr * k + s + c];
    const int64_t o = ((int64_t)cell * p + row0 + rr) * rank + c;
    if (a.side == KVC_SIDE_RIGHT) static_cast<double*>(a.basis)[o] = v;
    else store_dt(a.basis, o, (float)v, a.basis_dtype);
  }
}

// S -> R (upper triangle, S = R^T R) and rinv for every cell: the panel
// launches for k >= CHP_MIN_K (dg0: k doubles of scratch per cell), else
// chol_kernel.
int chol_launch(double* S, int k, int nbmax, size_t chol_smem, int64_t cs, double* rinv, double* dg0, int n_cells,
                cudaStream_t st) {
  if (k < CHP_MIN_K) {
    chol_kernel<<<n_cells, CH_NT, chol_smem, st>>>(S, k, nbmax, cs, rinv, cs);
    return check_launch("chol_kernel");
  }
  int rc;
  chol_diag_copy_kernel<<<dim3(1, n_cells), 256, 0, st>>>(S, k, cs, dg0, cs);
  if ((rc = check_launch("chol_diag_copy_kernel"))) return rc;
  for (int j0 = 0; j0 < k; j0 += CHP) {
    const dim3 grid((k - j0 + CHP - 1) / CHP, n_cells);
    chol_panel_kernel<<<grid, 256, 0, st>>>(S, k, cs, rinv, cs, dg0, cs, j0);
    if ((rc = check_launch("chol_panel_kernel"))) return rc;
  }
  return KVC_OK;
}

int lr_solve(const SolveArgs& a, int n_cells, cudaStream_t st) {
  const int p = a.p, k = a.k;
  const LrLayout L = lr_layout(p, k);
  const int64_t cs = a.ws_cell;
  double* ws = a.ws;
  const int nbmax = chol_panel_rows(k);
  const size_t chol_smem = sizeof(double) * (size_t)nbmax * k;
  const size_t trsm_smem = sizeof(double) * ((size_t)TS_ROWS * k + (size_t)TS_NBUF * RS_BLOCK);
  cudaError_t e = cudaFuncSetAttribute(chol_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chol_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(trsm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)trsm_smem);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  int rc;
  lr_init_kernel<<<dim3((unsigned)std::min<int64_t>(ceil_div((int64_t)p * k, 256 * 4), 128), n_cells), 256, 0, st>>>(a, L);
  if ((rc = check_launch("lr_init_kernel"))) return rc;
  int64_t cur = L.W, oth = L.Z;  // the current basis and the other p x k slot
  auto gemm = [&](const double* A, int64_t sA, int lda, int tA, const double* B, int64_t sB, int ldb, int tB,
                  double* C, int64_t sC, int ldc, int M, int N, int K) {
    Gemm g{A, B, C, M, N, K, lda, ldb, ldc, tA, tB, sA, sB, sC};
    return launch_gemm(g, n_cells, st);
  };
  // one CholeskyQR pass on the current basis, in the inner product of H (RIGHT) or I (LEFT)
  auto orth = [&]() -> int {
    int r2;
    const double* rhs = ws + cur;
    if (a.side == KVC_SIDE_RIGHT) {
      if ((r2 = gemm(a.gram, a.gram_stride, p, 0, ws + cur, cs, k, 0, ws + oth, cs, k, p, k, p))) return r2;
      rhs = ws + oth;
    }
    if ((r2 = gemm(ws + cur, cs, k, 1, rhs, cs, k, 0, ws + L.S, cs, k, k, k, p))) return r2;
    if ((r2 = chol_launch(ws + L.S, k, nbmax, chol_smem, cs, ws + L.rinv, ws + L.lam, n_cells, st))) return r2;
    const dim3 grid((p + TS_ROWS - 1) / TS_ROWS, n_cells);
    trsm_kernel<<<grid, TS_NT, trsm_smem, st>>>(ws + cur, p, k, cs, ws + L.S, cs, ws + L.rinv, cs);
    return check_launch("trsm_kernel");
  };
  if ((rc = orth())) return rc;
  if (a.n_power == 0 && (rc = orth())) return rc;
  for (int it = 0; it < a.n_power; ++it) {
    // the other slot = G W becomes the sketch
    if ((rc = gemm(a.gram, a.gram_stride, p, 0, ws + cur, cs, k, 0, ws + oth, cs, k, p, k, p))) return rc;
    std::swap(cur, oth);
    if ((rc = orth())) return rc;
    if (it + 1 == a.n_power && (rc = orth())) return rc;
  }
  // Ritz matrix: C = W^T G W (LEFT) or (H W)^T (H W) (RIGHT)
  if ((rc = gemm(a.gram, a.gram_stride, p, 0, ws + cur, cs, k, 0, ws + oth, cs, k, p, k, p))) return rc;
  if (a.side == KVC_SIDE_LEFT) rc = gemm(ws + cur, cs, k, 1, ws + oth, cs, k, 0, ws + L.C, cs, k, k, k, p);
  else rc = gemm(ws + oth, cs, k, 1, ws + oth, cs, k, 0, ws + L.C, cs, k, k, k, p);
  if (rc) return rc;
  const int s = k - a.rank;
  const int ldx = k | 1;  // odd row stride: the rows' Gram reads are conflict-free
  // IV_ITERS steps on 16 vectors for s <= 4 trailing ones, on 32 for
  // s <= 16 where their rows fit in shared memory next to the static arrays
  // and the staged blocks of R (k <= 554); other sketches take the full
  // eigensolver
  const size_t rs_bytes = sizeof(double) * (size_t)CP_NBUF * RS_BLOCK;
  const bool wide_fits = sizeof(double) * (size_t)IV_MAX * ldx + rs_bytes <= 176 * 1024;
  const int nb = s <= 4 ? IV_GROUP : IV_MAX;
  const int iters = IV_ITERS;
  if (k >= CP_MIN_K && s <= CP_MAX_S && (s <= 4 || wide_fits) && !a.sv2) {
    // the complement of the s trailing Ritz vectors
    const int cp_smem = (int)(sizeof(double) * (size_t)TS_ROWS * k);
    const int iv_smem = (int)(sizeof(double) * (size_t)nb * ldx + rs_bytes);
    if ((e = cudaFuncSetAttribute(cp_complement_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cp_smem)) ==
        cudaSuccess)
      e = cudaFuncSetAttribute(cp_bottom_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, iv_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(cp_start_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, iv_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(iv_mult_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, iv_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(iv_orth_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, iv_smem);
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    if (s > 0) {
      cp_shift_kernel<<<n_cells, 256, 0, st>>>(ws, cs, L, k);
      if ((rc = check_launch("cp_shift_kernel"))) return rc;
      if ((rc = chol_launch(ws + L.C, k, nbmax, chol_smem, cs, ws + L.rinv, ws + L.lam, n_cells, st))) return rc;
      // (C + delta I)^-1 = R^-1 R^-T: R^-1 as the rows of I R^-1 (one
      // row-parallel triangular solve), then one product
      identity_kernel<<<dim3(64, n_cells), 256, 0, st>>>(ws + L.Zt, k, cs);
      if ((rc = check_launch("identity_kernel"))) return rc;
      const dim3 tgrid((k + TS_ROWS - 1) / TS_ROWS, n_cells);
      trsm_kernel<<<tgrid, TS_NT, trsm_smem, st>>>(ws + L.Zt, k, k, cs, ws + L.C, cs, ws + L.rinv, cs);
      if ((rc = check_launch("trsm_kernel"))) return rc;
      if ((rc = gemm(ws + L.Zt, cs, k, 0, ws + L.Zt, cs, k, 1, ws + L.S, cs, k, k, k, k))) return rc;
      const int64_t xoff = oth, xnoff = oth + (int64_t)nb * k;  // the free p x k slot (p >= k > 2 nb)
      const int xs_smem = (int)(sizeof(double) * (size_t)nb * ldx);
      cp_start_kernel<<<n_cells, 16 * nb, xs_smem, st>>>(a, nb, ldx, xoff);
      if ((rc = check_launch("cp_start_kernel"))) return rc;
      const dim3 mgrid((k + 31) / 32, n_cells);
      for (int it = 0; it < iters; ++it) {
        iv_mult_kernel<<<mgrid, 16 * nb, iv_smem, st>>>(a, L, nb, ldx, xoff, xnoff);
        if ((rc = check_launch("iv_mult_kernel"))) return rc;
        iv_orth_kernel<<<n_cells, 16 * nb, xs_smem, st>>>(a, nb, ldx, xnoff, xoff);
        if ((rc = check_launch("iv_orth_kernel"))) return rc;
      }
      cp_bottom_kernel<<<n_cells, 16 * nb, xs_smem, st>>>(a, L, s, nb, ldx, xoff);
      if ((rc = check_launch("cp_bottom_kernel"))) return rc;
    } else {
      // the sketch space itself: tail = 1 - trace(C) / |A|^2
      cp_shift_kernel<<<n_cells, 256, 0, st>>>(ws, cs, L, k);
      if ((rc = check_launch("cp_shift_kernel"))) return rc;
      cp_tail_kernel<<<1, 64, 0, st>>>(a, L, n_cells);
      if ((rc = check_launch("cp_tail_kernel"))) return rc;
    }
    const dim3 grid((p + TS_ROWS - 1) / TS_ROWS, n_cells);
    cp_complement_kernel<<<grid, TS_NT, cp_smem, st>>>(a, L, cur, s);
    return check_launch("cp_complement_kernel");
  }
  lr_eig_kernel<<<n_cells, SNT, 0, st>>>(a, L);
  if ((rc = check_launch("lr_eig_kernel"))) return rc;
  // basis = W Zt^T (p x rank)
  if (a.side == KVC_SIDE_RIGHT) {
    return gemm(ws + cur, cs, k, 0, ws + L.Zt, cs, k, 1, static_cast<double*>(a.basis), (int64_t)p * a.rank, a.rank,
                p, a.rank, k);
  }
  if ((rc = gemm(ws + cur, cs, k, 0, ws + L.Zt, cs, k, 1, ws + oth, cs, a.rank, p, a.rank, k))) return rc;
  SolveArgs b = a;
  b.ws = ws;
  // the product sits in the slot `oth`; point the store kernel's Z slot at it
  LrLayout L2 = L;
  L2.Z = oth;
  const dim3 grid(std::max(1, std::min(64, (int)(((int64_t)p * a.rank + 255) / 256))), n_cells);
  lr_store_kernel<<<grid, 256, 0, st>>>(b, L2);
  return check_launch("lr_store_kernel");
}

// Workspace doubles per cell: the general solver's layout (above), which
// also covers the shared-memory kernels' eigenvectors and scratch.
int64_t ws_per_cell(int mode, int p, int k) {
  if (mode == KVC_SVD_EXACT) return 2LL * p * p + eig::vec_doubles(p) + p + eig_scratch_doubles(p);
  return lr_layout(p, k).total;
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
  if (mode == KVC_SVD_RANDOMISED && (k < rank || k > p || k > MAX_SKETCH))
    return fail(KVC_ERR_SHAPE, "kvc_sketch_solve: sketch width must satisfy rank <= k <= min(p, 1024)");
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
    const int in_smem = exact_small_smem_bytes_vectors(p, rank) <= SMEM_LIMIT;
    const size_t smem = in_smem ? exact_small_smem_bytes_vectors(p, rank) : exact_small_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(exact_solve_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    exact_solve_small_kernel<<<n_cells, SM_NT, smem, static_cast<cudaStream_t>(stream)>>>(a, in_smem);
    return check_launch("exact_solve_small_kernel");
  }
  if (mode == KVC_SVD_RANDOMISED) return lr_solve(a, n_cells, static_cast<cudaStream_t>(stream));
  exact_solve_kernel<<<n_cells, SNT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("exact_solve_kernel");
}
