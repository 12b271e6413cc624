// Leading eigenpairs of a small dense symmetric matrix, one thread block per
// matrix, fp64 -- the eigensolve inside the SVD solvers (the SVD of
// B = Q^T A in SVD.randomise, kvcompress/compressor/svd.py:267-285, and the
// full SVD of SVD.exact, svd.py:181-219, both seen through a Gram matrix).
//
// The method is the one of LAPACK's dsyevx (selected eigenpairs):
//   1. Householder reduction to tridiagonal form T = H^T A H
//      (H = H_0 ... H_{n-3}, H_j = I - tau_j v_j v_j^T; dsytrd),
//   2. the wanted eigenvalues of T by bisection on Sturm counts (dstebz),
//      run as multisection: each wanted eigenvalue's interval is split at
//      several points per round, one point per thread,
//   3. their eigenvectors by inverse iteration on T with a tridiagonal LU
//      with partial pivoting, re-orthogonalised against the earlier vectors
//      of a cluster of close eigenvalues (dstein),
//   4. back-transformation by the reflectors (dormtr).
// Sturm counts use the division-free three-term recurrence of the leading
// principal minors det(T_i - x I) with exact power-of-two rescaling, whose
// sign changes count the eigenvalues below x (Sylvester's law of inertia).
//
// Matrices are passed as generic pointers with a row stride, so the same
// routines run on a matrix in shared memory (n up to a few hundred doubles of
// rows) or in global memory (larger n, served from L2).  Every loop has a
// fixed trip-count bound.
#pragma once

#include <cstdint>

namespace kvc {
namespace eig {

constexpr int MAX_ROUNDS = 160;  // multisection rounds (each shrinks an interval >= 2x)
constexpr int INV_ITERS = 3;     // inverse-iteration solves per eigenvector

// Block-wide sum; every thread gets the result.  red: >= 33 doubles of shared
// memory, not used by the caller between the call's barriers.
__device__ inline double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = threadIdx.x < nw ? red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Block-wide min and max of (lo, hi); results in out[0], out[1] (shared).
__device__ inline void block_minmax(double lo, double hi, double* red, double* out) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fmin(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmax(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) {
    red[w] = lo;
    red[16 + w] = hi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    double a = threadIdx.x < nw ? red[threadIdx.x] : lo;
    double b = threadIdx.x < nw ? red[16 + threadIdx.x] : hi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a = fmin(a, __shfl_xor_sync(0xffffffffu, a, o));
      b = fmax(b, __shfl_xor_sync(0xffffffffu, b, o));
    }
    if (threadIdx.x == 0) {
      out[0] = a;
      out[1] = b;
    }
  }
  __syncthreads();
}

// 1. Householder tridiagonalisation of the symmetric n x n matrix A (both
// triangles stored, row stride lda).  On exit d (n) and e (n - 1) hold T's
// diagonal and off-diagonal, tau (n) the reflector scales (tau[j] = 0: no
// reflector at step j), and column j of A below the diagonal holds v_j.
// vs, ps: n doubles of shared scratch each; red: 33 doubles.
__device__ inline void tridiagonalize(double* A, int lda, int n, double* d, double* e, double* tau, double* vs,
                                      double* ps, double* red) {
  for (int j = 0; j + 2 < n; ++j) {
    const int m = n - j - 1;  // trailing size
    double* col = A + (int64_t)(j + 1) * lda + j;  // x_i = col[i * lda]
    double part = 0.0;
    for (int i = 1 + threadIdx.x; i < m; i += blockDim.x) {
      const double x = col[(int64_t)i * lda];
      part = fma(x, x, part);
    }
    const double sig = block_sum(part, red);
    const double x0 = col[0];
    if (threadIdx.x == 0) {
      d[j] = A[(int64_t)j * lda + j];
    }
    if (!(sig > 0.0)) {
      // nothing to annihilate below the sub-diagonal
      if (threadIdx.x == 0) {
        e[j] = x0;
        tau[j] = 0.0;
      }
      __syncthreads();
      continue;
    }
    const double nx = sqrt(fma(x0, x0, sig));
    const double alpha = x0 >= 0.0 ? -nx : nx;
    const double v0 = x0 - alpha;
    const double t = 2.0 / fma(v0, v0, sig);
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const double v = i == 0 ? v0 : col[(int64_t)i * lda];
      vs[i] = v;
    }
    if (threadIdx.x == 0) {
      e[j] = alpha;
      tau[j] = t;
      col[0] = v0;  // v_j kept in column j (the rest of x is already v)
    }
    __syncthreads();
    // p = t S v, S = A[j+1:, j+1:] (columns read: consecutive rows of a
    // group, consecutive addresses); tpr threads split each row's sum when
    // the trailing matrix is small, which shortens the dependent chain
    const double* S = A + (int64_t)(j + 1) * lda + (j + 1);
    int tpr = 1;
    while (tpr < 32 && tpr * 2 * m <= (int)blockDim.x) tpr *= 2;
    const int sub = threadIdx.x & (tpr - 1), rpp = blockDim.x / tpr;
    double kp = 0.0;
    for (int i0 = 0; i0 < m; i0 += rpp) {  // the same trip count for every thread (the shuffles)
      const int i = i0 + (int)threadIdx.x / tpr;
      double acc = 0.0;
      if (i < m)
        for (int k = sub; k < m; k += tpr) acc = fma(S[(int64_t)k * lda + i], vs[k], acc);
      for (int o = tpr >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (i < m && sub == 0) {
        const double p = t * acc;
        ps[i] = p;
        kp = fma(vs[i], p, kp);
      }
    }
    const double K = 0.5 * t * block_sum(kp, red);
    // w = p - K v (in ps)
    for (int i = threadIdx.x; i < m; i += blockDim.x) ps[i] = fma(-K, vs[i], ps[i]);
    __syncthreads();
    // S -= v w^T + w v^T
    double* Sw = A + (int64_t)(j + 1) * lda + (j + 1);
    for (int64_t idx = threadIdx.x; idx < (int64_t)m * m; idx += blockDim.x) {
      const int r = (int)(idx / m), c = (int)(idx % m);
      double* a = Sw + (int64_t)r * lda + c;
      *a = fma(-vs[r], ps[c], fma(-ps[r], vs[c], *a));
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (n >= 2) {
      d[n - 2] = A[(int64_t)(n - 2) * lda + (n - 2)];
      e[n - 2] = A[(int64_t)(n - 1) * lda + (n - 2)];
      tau[n - 2] = 0.0;
    }
    d[n - 1] = A[(int64_t)(n - 1) * lda + (n - 1)];
    tau[n - 1] = 0.0;
  }
  __syncthreads();
}

// Number of eigenvalues of T below x: sign changes of the leading principal
// minors p_i = (d_i - x) p_{i-1} - e_{i-1}^2 p_{i-2}, p_0 = 1, rescaled by
// exact powers of two to stay in range; a zero minor counts as having the
// sign opposite to its predecessor.
__device__ inline int sturm_count(const double* d, const double* e2, int n, double x) {
  double pm = 1.0, p = d[0] - x;
  int c = 0;
  bool prev_neg = false;  // sign of p_0 = 1
  for (int i = 0;; ) {
    bool neg = p < 0.0 || (p == 0.0 && !prev_neg);
    c += (neg != prev_neg);
    prev_neg = neg;
    if (++i >= n) break;
    double pn = fma(d[i] - x, p, -e2[i - 1] * pm);
    pm = p;
    p = pn;
    // rescale the pair by the larger magnitude (the ratio of consecutive
    // minors is a pivot and may be far from one)
    const double a = fmax(fabs(p), fabs(pm));
    if (a > 0x1p+600) {
      p *= 0x1p-600;
      pm *= 0x1p-600;
    } else if (a < 0x1p-600 && a != 0.0) {
      p *= 0x1p+600;
      pm *= 0x1p+600;
    }
  }
  return c;
}

// 2. The r largest eigenvalues of T (d, e; n), descending, into lam[0..r).
// e2 (n - 1), lo / hi (r each), cnt (blockDim.x ints): shared scratch.
// Returns the Gershgorin bound max|lambda| (the scale for tolerances).
__device__ inline double top_eigenvalues(const double* d, const double* e, int n, int r, double* lam, double* e2,
                                         double* lo, double* hi, int* cnt, double* red) {
  __shared__ double s_bounds[2];
  __shared__ int s_any;
  double glo = 1e300, ghi = -1e300;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double el = i > 0 ? fabs(e[i - 1]) : 0.0, er = i + 1 < n ? fabs(e[i]) : 0.0;
    glo = fmin(glo, d[i] - el - er);
    ghi = fmax(ghi, d[i] + el + er);
    if (i + 1 < n) e2[i] = e[i] * e[i];
  }
  block_minmax(glo, ghi, red, s_bounds);
  const double nrm = fmax(fabs(s_bounds[0]), fabs(s_bounds[1]));
  const double pad = 1e-14 * nrm + 1e-280;
  for (int a = threadIdx.x; a < r; a += blockDim.x) {
    lo[a] = s_bounds[0] - pad;
    hi[a] = s_bounds[1] + pad;
  }
  __syncthreads();
  const int nt = blockDim.x;
  const int G = r >= nt ? 1 : nt / r;  // points per interval per round
  for (int round = 0; round < MAX_ROUNDS; ++round) {
    if (threadIdx.x == 0) s_any = 0;
    __syncthreads();
    // every (interval, point) pair; a thread may take several
    for (int base = 0; base < r * G; base += nt) {
      const int task = base + threadIdx.x;
      int c = -1;
      if (task < r * G) {
        const int a = task / G, g = task % G;
        const double l = lo[a], h = hi[a];
        if (h - l > 4e-16 * fmax(fabs(l), fabs(h)) + 1e-300 + 1e-17 * nrm) {
          const double x = l + (h - l) * (double)(g + 1) / (double)(G + 1);
          c = sturm_count(d, e2, n, x);
          s_any = 1;
        }
      }
      cnt[threadIdx.x] = c;
      __syncthreads();
      // the first thread of each interval narrows it: the counts grow with x,
      // so the points with count <= want come first (binary search)
      if (task < r * G && task % G == 0 && cnt[threadIdx.x] >= 0) {
        const int a = task / G;
        const int want = n - 1 - a;  // ascending index of the a-th largest
        const double l = lo[a], h = hi[a];
        int nb = 0, top = G;  // points [0, nb) have count <= want, [top, G) above
        while (nb < top) {
          const int mid = (nb + top) >> 1;
          if (cnt[threadIdx.x + mid] <= want) nb = mid + 1;
          else top = mid;
        }
        if (nb > 0) lo[a] = l + (h - l) * (double)nb / (double)(G + 1);
        if (nb < G) hi[a] = l + (h - l) * (double)(nb + 1) / (double)(G + 1);
      }
      __syncthreads();
    }
    if (!s_any) break;
  }
  for (int a = threadIdx.x; a < r; a += blockDim.x) lam[a] = 0.5 * (lo[a] + hi[a]);
  __syncthreads();
  return nrm;
}

// Deterministic start vector entry in [-1, 1) for eigenvector a, row i.
__device__ inline double start_entry(int a, int i) {
  uint32_t h = (uint32_t)a * 0x9E3779B1u ^ ((uint32_t)i + 0x7F4A7C15u) * 0x85EBCA77u;
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  h *= 0x297A2D39u;
  h ^= h >> 15;
  return (double)(h >> 8) * (1.0 / 8388608.0) - 1.0;
}

// Solve ((T - lam I) / scale) y = y in place by LU with partial pivoting
// (dgtsv's elimination); u1, u2, dd: n doubles of per-thread scratch.  Zero
// pivots are replaced by tiny.  inv_scale = 1 / scale keeps the entries of
// order one whatever the matrix's magnitude.
__device__ inline void tri_solve(const double* d, const double* e, int n, double lam, double inv_scale, double* y,
                                 double* dd, double* u1, double* u2, double tiny) {
  for (int i = 0; i < n; ++i) {
    dd[i] = (d[i] - lam) * inv_scale;
    u1[i] = i + 1 < n ? e[i] * inv_scale : 0.0;
    u2[i] = 0.0;
  }
  for (int i = 0; i + 1 < n; ++i) {
    const double sub = e[i] * inv_scale;  // row i + 1's entry in column i
    if (fabs(dd[i]) >= fabs(sub)) {
      double piv = dd[i];
      if (piv == 0.0) piv = dd[i] = tiny;
      const double f = sub / piv;
      dd[i + 1] = fma(-f, u1[i], dd[i + 1]);
      y[i + 1] = fma(-f, y[i], y[i + 1]);
    } else {
      // swap rows i and i + 1
      const double f = dd[i] / sub;
      dd[i] = sub;
      const double t1 = dd[i + 1];
      dd[i + 1] = fma(-f, t1, u1[i]);
      u1[i] = t1;
      if (i + 2 < n) {
        u2[i] = u1[i + 1];
        u1[i + 1] = -f * u2[i];
      }
      const double yi = y[i];
      y[i] = y[i + 1];
      y[i + 1] = fma(-f, y[i + 1], yi);
    }
  }
  if (dd[n - 1] == 0.0) dd[n - 1] = tiny;
  y[n - 1] /= dd[n - 1];
  if (n >= 2) y[n - 2] = (y[n - 2] - u1[n - 2] * y[n - 1]) / dd[n - 2];
  for (int i = n - 3; i >= 0; --i) y[i] = (y[i] - u1[i] * y[i + 1] - u2[i] * y[i + 2]) / dd[i];
}

// 3. Eigenvectors of T for lam[0..r) (descending) into rows of Zt (r x n,
// row stride ldz): parallel over clusters of eigenvalues closer than
// 1e-7 * nrm (threads 0 .. workers - 1; a cluster's vectors in order, each
// re-orthogonalised against the cluster's earlier ones).  scratch: 3 n
// doubles per worker at scratch + threadIdx.x * sstride; shared memory keeps
// the solves' read-after-write chains short.
__device__ inline void tri_eigenvectors(const double* d, const double* e, int n, const double* lam, int r, double nrm,
                                        double* Zt, int ldz, double* scratch, int64_t sstride, int workers) {
  const double ctol = 1e-7 * nrm;
  const double inv_scale = nrm > 0.0 ? 1.0 / nrm : 1.0;
  const double tiny = 1e-15;
  double* dd = scratch + threadIdx.x * sstride;
  double* u1 = dd + n;
  double* u2 = u1 + n;
  const int nw = workers < (int)blockDim.x ? workers : (int)blockDim.x;
  for (int a0 = threadIdx.x; a0 < r && (int)threadIdx.x < nw; a0 += nw) {
    if (a0 > 0 && lam[a0 - 1] - lam[a0] <= ctol) continue;  // not a cluster start
    int a1 = a0 + 1;
    while (a1 < r && lam[a1 - 1] - lam[a1] <= ctol) ++a1;
    for (int a = a0; a < a1; ++a) {
      double* y = Zt + (int64_t)a * ldz;
      for (int i = 0; i < n; ++i) y[i] = start_entry(a, i);
      for (int it = 0; it < INV_ITERS; ++it) {
        tri_solve(d, e, n, lam[a], inv_scale, y, dd, u1, u2, tiny);
        for (int b = a0; b < a; ++b) {
          const double* z = Zt + (int64_t)b * ldz;
          double s = 0.0;
          for (int i = 0; i < n; ++i) s = fma(z[i], y[i], s);
          for (int i = 0; i < n; ++i) y[i] = fma(-s, z[i], y[i]);
        }
        double s = 0.0;
        for (int i = 0; i < n; ++i) s = fma(y[i], y[i], s);
        const double inv = s > 0.0 ? 1.0 / sqrt(s) : 0.0;
        if (inv == 0.0) {
          for (int i = 0; i < n; ++i) y[i] = start_entry(a + 7919 * (it + 1), i);
          continue;
        }
        for (int i = 0; i < n; ++i) y[i] *= inv;
      }
    }
  }
  __syncthreads();
}

// 4. Z_a <- H_0 ... H_{n-3} Z_a for every row a of Zt (thread-parallel over
// rows): the eigenvectors of A from those of T.  A holds v_j in column j.
__device__ inline void back_transform(const double* A, int lda, const double* tau, int n, double* Zt, int ldz,
                                      int r) {
  for (int a = threadIdx.x; a < r; a += blockDim.x) {
    double* z = Zt + (int64_t)a * ldz;
    for (int j = n - 3; j >= 0; --j) {
      const double t = tau[j];
      if (t == 0.0) continue;
      const double* v = A + (int64_t)(j + 1) * lda + j;
      const int m = n - j - 1;
      double s = 0.0;
      for (int i = 0; i < m; ++i) s = fma(v[(int64_t)i * lda], z[j + 1 + i], s);
      s *= t;
      for (int i = 0; i < m; ++i) z[j + 1 + i] = fma(-s, v[(int64_t)i * lda], z[j + 1 + i]);
    }
  }
  __syncthreads();
}

}  // namespace eig
}  // namespace kvc

namespace kvc {
namespace eig {

// Doubles of shared (or global) vector scratch eig_top needs for size n.
__host__ __device__ constexpr int64_t vec_doubles(int n) { return 8LL * n; }

// The r leading eigenpairs of the symmetric n x n matrix A (destroyed): lam
// (r, descending) and the eigenvectors as rows of Zt (r x n, row stride ldz).
// vec: vec_doubles(n) doubles; cnt: blockDim.x ints; red: 64 doubles (all
// shared); scratch: 3 n doubles for each of the first `workers` threads
// (thread t at scratch + t * 3 n), which compute the eigenvectors.  Returns
// the spectral scale used for the tolerances (a bound on max |lambda|).
__device__ inline double eig_top(double* A, int lda, int n, int r, double* lam, double* Zt, int ldz, double* vec,
                                 int* cnt, double* red, double* scratch, int workers) {
  double* d = vec;
  double* e = d + n;
  double* tau = e + n;
  double* vs = tau + n;
  double* ps = vs + n;
  double* e2 = ps + n;
  double* lo = e2 + n;
  double* hi = lo + n;
  tridiagonalize(A, lda, n, d, e, tau, vs, ps, red);
  const double nrm = top_eigenvalues(d, e, n, r, lam, e2, lo, hi, cnt, red);
  tri_eigenvectors(d, e, n, lam, r, nrm, Zt, ldz, scratch, 3LL * n, workers);
  back_transform(A, lda, tau, n, Zt, ldz, r);
  return nrm;
}

}  // namespace eig
}  // namespace kvc
