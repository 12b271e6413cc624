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
// falls below 1e-10 of its norm is set to zero); the eigensolver is cyclic
// two-sided Jacobi with round-robin parallel ordering.  Every loop has a
// fixed trip count bound (at most 60 sweeps).
#include <algorithm>
#include <cmath>

#include "kvc_common.cuh"

namespace kvc {
namespace {

constexpr int SNT = 512;
constexpr int MAX_SWEEPS = 60;
constexpr int MAX_PAIRS = 1024;

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

__device__ double blk_sum(double v) {
  __shared__ double red[SNT / 32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (int)(blockDim.x / 32) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  __shared__ double res;
  if (threadIdx.x == 0) res = t;
  __syncthreads();
  return res;
}

// Symmetric eigensolver: A (n x n) is destroyed, V receives eigenvectors in
// columns, evals[i] = A[i][i] after convergence (unsorted).
__device__ void blk_jacobi(double* A, double* V, int n, double* evals) {
  __shared__ int pos[2 * MAX_PAIRS];
  __shared__ double cs[MAX_PAIRS], sn[MAX_PAIRS];
  __shared__ int pp[MAX_PAIRS], qq[MAX_PAIRS];
  const int N = n + (n & 1);
  const int H = N / 2;
  for (int64_t idx = threadIdx.x; idx < (int64_t)n * n; idx += blockDim.x)
    V[idx] = (idx / n == idx % n) ? 1.0 : 0.0;
  for (int i = threadIdx.x; i < N; i += blockDim.x) pos[i] = i;
  __syncthreads();
  for (int sweep = 0; sweep < MAX_SWEEPS && n > 1; ++sweep) {
    double off = 0.0, tot = 0.0;
    for (int64_t idx = threadIdx.x; idx < (int64_t)n * n; idx += blockDim.x) {
      const double a = A[idx];
      tot += a * a;
      if (idx / n != idx % n) off += a * a;
    }
    off = blk_sum(off);
    tot = blk_sum(tot);
    if (!(off > 1e-30 * tot)) break;
    for (int round = 0; round < N - 1; ++round) {
      for (int pr = threadIdx.x; pr < H; pr += blockDim.x) {
        int p = pos[pr], q = pos[N - 1 - pr];
        if (p > q) {
          const int t = p;
          p = q;
          q = t;
        }
        double c = 1.0, s = 0.0;
        if (q < n) {
          const double apq = A[(int64_t)p * n + q];
          if (apq != 0.0) {
            const double app = A[(int64_t)p * n + p], aqq = A[(int64_t)q * n + q];
            const double tau = (aqq - app) / (2.0 * apq);
            const double t = (tau >= 0.0 ? 1.0 : -1.0) / (fabs(tau) + sqrt(1.0 + tau * tau));
            c = 1.0 / sqrt(1.0 + t * t);
            s = t * c;
          }
        }
        cs[pr] = c;
        sn[pr] = s;
        pp[pr] = p;
        qq[pr] = q < n ? q : -1;
      }
      __syncthreads();
      // rows: A <- J^T A
      for (int64_t task = threadIdx.x; task < (int64_t)H * n; task += blockDim.x) {
        const int pr = (int)(task / n), j = (int)(task % n);
        const int q = qq[pr];
        if (q < 0 || sn[pr] == 0.0) continue;
        const int p = pp[pr];
        const double c = cs[pr], s = sn[pr];
        const double a = A[(int64_t)p * n + j], b = A[(int64_t)q * n + j];
        A[(int64_t)p * n + j] = c * a - s * b;
        A[(int64_t)q * n + j] = s * a + c * b;
      }
      __syncthreads();
      // columns: A <- A J, V <- V J
      for (int64_t task = threadIdx.x; task < (int64_t)H * n; task += blockDim.x) {
        const int pr = (int)(task / n), i = (int)(task % n);
        const int q = qq[pr];
        if (q < 0 || sn[pr] == 0.0) continue;
        const int p = pp[pr];
        const double c = cs[pr], s = sn[pr];
        double a = A[(int64_t)i * n + p], b = A[(int64_t)i * n + q];
        A[(int64_t)i * n + p] = c * a - s * b;
        A[(int64_t)i * n + q] = s * a + c * b;
        a = V[(int64_t)i * n + p];
        b = V[(int64_t)i * n + q];
        V[(int64_t)i * n + p] = c * a - s * b;
        V[(int64_t)i * n + q] = s * a + c * b;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        const int last = pos[N - 1];
        for (int i = N - 1; i >= 2; --i) pos[i] = pos[i - 1];
        pos[1] = last;
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) evals[i] = A[(int64_t)i * n + i];
  __syncthreads();
}

// order[r] = index of the r-th largest eigenvalue (ties by index).
__device__ void blk_order_desc(const double* ev, int n, int* order) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int r = 0;
    const double v = ev[i];
    for (int j = 0; j < n; ++j) r += (ev[j] > v) || (ev[j] == v && j < i);
    order[r] = i;
  }
  __syncthreads();
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

__global__ void __launch_bounds__(SNT) sketch_solve_kernel(SolveArgs a) {
  const int cell = blockIdx.x;
  const int p = a.p, k = a.k, rank = a.rank;
  const double* gram = a.gram + cell * a.gram_stride;
  double* ws = a.ws + cell * a.ws_cell;
  const int nmax = p > k ? p : k;
  double* ev = ws;                      // nmax
  int* order = reinterpret_cast<int*>(ws + nmax);  // nmax ints (<= nmax doubles)
  double* base = ws + 2 * (int64_t)nmax;
  __shared__ double nrm_s;

  if (a.mode == KVC_SVD_EXACT) {
    double* A = base;                          // p x p
    double* V = base + (int64_t)p * p;         // p x p
    for (int64_t i = threadIdx.x; i < (int64_t)p * p; i += blockDim.x) A[i] = gram[i];
    __syncthreads();
    blk_jacobi(A, V, p, ev);
    for (int i = threadIdx.x; i < p; i += blockDim.x) ev[i] = ev[i] > 0.0 ? ev[i] : 0.0;
    __syncthreads();
    blk_order_desc(ev, p, order);
    const int64_t max_rank = a.n_other < p ? a.n_other : p;
    if (threadIdx.x == 0) {
      double total = 0.0, tail = 0.0;
      for (int i = 0; i < p; ++i) total += ev[order[i]];
      for (int i = rank; i < p; ++i) tail += ev[order[i]];
      a.tail[cell] = (rank >= max_rank || !(total > 0.0)) ? 0.0 : tail / total;
      if (a.sv2)
        for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = ev[order[i]];
    }
    __syncthreads();
    if (a.side == KVC_SIDE_LEFT) {
      for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
        const int i = (int)(idx / rank), r = (int)(idx % rank);
        store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)V[(int64_t)i * p + order[r]],
                 a.basis_dtype);
      }
    } else {
      const double lmax = ev[order[0]];
      double* M = static_cast<double*>(a.basis) + (int64_t)cell * p * rank;
      for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
        const int i = (int)(idx / rank), r = (int)(idx % rank);
        const double lam = ev[order[r]];
        M[idx] = (lam > 1e-14 * lmax && lam > 0.0) ? V[(int64_t)i * p + order[r]] / sqrt(lam) : 0.0;
      }
    }
    return;
  }

  // randomised
  double* Q = base;                               // p x k
  double* Z = Q + (int64_t)p * k;                 // p x k
  double* S = Z + (int64_t)p * k;                 // k x k
  double* C = S + (int64_t)k * k;                 // k x k
  double* V = C + (int64_t)k * k;                 // k x k
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
  blk_jacobi(C, V, k, ev);
  for (int i = threadIdx.x; i < k; i += blockDim.x) ev[i] = ev[i] > 0.0 ? ev[i] : 0.0;
  __syncthreads();
  blk_order_desc(ev, k, order);
  if (threadIdx.x == 0) {
    double retained = 0.0;
    for (int i = 0; i < rank; ++i) retained += ev[order[i]];
    const double nrm = nrm_s;
    double t = nrm > 0.0 ? 1.0 - retained / nrm : 0.0;
    a.tail[cell] = t > 0.0 ? t : 0.0;
    if (a.sv2)
      for (int i = 0; i < rank; ++i) a.sv2[(int64_t)cell * rank + i] = ev[order[i]];
  }
  __syncthreads();
  // basis = Q V[:, order[:rank]]
  for (int64_t idx = threadIdx.x; idx < (int64_t)p * rank; idx += blockDim.x) {
    const int i = (int)(idx / rank), r = (int)(idx % rank);
    const int col = order[r];
    double s = 0.0;
    for (int j = 0; j < k; ++j) s = fma(Q[(int64_t)i * k + j], V[(int64_t)j * k + col], s);
    if (a.side == KVC_SIDE_LEFT) store_dt(a.basis, (int64_t)cell * p * rank + idx, (float)s, a.basis_dtype);
    else static_cast<double*>(a.basis)[(int64_t)cell * p * rank + idx] = s;
  }
}

int64_t ws_per_cell(int mode, int p, int k) {
  const int64_t nmax = std::max(p, k);
  if (mode == KVC_SVD_EXACT) return 2 * nmax + 2LL * p * p;
  return 2 * nmax + 2LL * p * k + 3LL * k * k;
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
  if (p <= 0 || p > 2 * MAX_PAIRS - 2 || rank <= 0 || rank > p || n_other <= 0)
    return fail(KVC_ERR_SHAPE, "kvc_sketch_solve: bad p/rank");
  if (mode == KVC_SVD_RANDOMISED && (k < rank || k > p || k > 2 * MAX_PAIRS - 2))
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
  sketch_solve_kernel<<<n_cells, SNT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("sketch_solve_kernel");
}
