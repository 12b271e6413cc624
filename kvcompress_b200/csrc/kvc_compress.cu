// kvc_compress: the whole JoLT / FlashJoLT compress of a batch of same-shape
// cells in one call (kvcompress/compressor/jolt.py:273-329 with
// partial_tucker_st_hosvd, tucker.py:192-279, and encode_residual,
// residual.py:155-239), issuing the stage entry points of this library in
// order on one stream:
//
//   kvc_gram (feature)  -> kvc_sketch_solve (U_d)  -> kvc_project_feature
//   kvc_gram (token)    -> kvc_sketch_solve (M)    -> kvc_apply_basis (U_T)
//   kvc_core            -> kvc_residual_stats      -> kvc_residual_quant
//   kvc_cast of the factors to the payload's factor dtype
//
// Intermediates (Grams, x_proj, the token-side basis) live in the caller's
// workspace; the factors, tails, scales and codes go to caller-owned batch
// tensors.  The point is the host: one C call of a few tens of microseconds
// replaces a dozen Python-level launches whose host time exceeded the
// kernels' device time on a 64-cell batch.
#include <cstring>

#include "kvc_b200.h"
#include "kvc_common.cuh"

namespace kvc {

// lets the next tensor-core quantise launch on this thread reuse the Tucker
// row terms the stats launch before it left in the shared scratch
void tc_reuse_tucker_rows(bool allow);
void tc_stats_gram_bound(const double* gram, int64_t stride);

namespace {

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Sizes {
  size_t gram_f, gram_t, xproj, mat, sv2, scratch, total;
};

int dsize(int dtype) { return dtype_size(dtype); }

Sizes sizes(int n, int64_t m, int64_t t, int d, int dtype, int rt, int rd, int mode_f, int k_f, int mode_t, int k_t,
            int bits, int scale_mode) {
  Sizes s;
  const int64_t c = m * rd;
  const int kf = mode_f == KVC_SVD_RANDOMISED ? k_f : 0;
  const int kt = mode_t == KVC_SVD_RANDOMISED ? k_t : 0;
  s.gram_f = a256((size_t)n * ((size_t)d * d + (size_t)d * kf + 1) * 8);
  s.gram_t = a256((size_t)n * ((size_t)c * c + 1) * 8);
  s.xproj = a256((size_t)n * t * c * dsize(dtype));
  s.mat = a256((size_t)n * c * rt * 8);
  s.sv2 = a256((size_t)n * (size_t)std::max(rt, rd) * 8);
  size_t scr = kvc_gram_workspace_bytes(n, m * t, d, kf);
  scr = std::max(scr, kvc_sketch_solve_workspace_bytes(n, mode_f, d, kf));
  scr = std::max(scr, kvc_gram_workspace_bytes(n, t, (int)c, 0));
  scr = std::max(scr, kvc_sketch_solve_workspace_bytes(n, mode_t, (int)c, kt));
  scr = std::max(scr, kvc_core_workspace_bytes(n, t, (int)m, rd, rt));
  if (bits > 0) {
    if (scale_mode != KVC_SCALE_GROUP) scr = std::max(scr, kvc_residual_stats_workspace_bytes(n, m * t, d, rd));
    scr = std::max(scr, kvc_residual_quant_workspace_bytes(n, m * t, d, rd));
  }
  s.scratch = a256(scr);
  s.total = s.gram_f + s.gram_t + s.xproj + s.mat + s.sv2 + s.scratch;
  return s;
}

// Optional stage timing: CUDA events recorded around each stage on the
// call's stream (two per stage, in stage order), per calling thread.
thread_local void* const* tl_events = nullptr;
thread_local int tl_n_events = 0;

enum Stage { ST_GRAM_F, ST_SOLVE_F, ST_PROJECT, ST_GRAM_T, ST_SOLVE_T, ST_APPLY, ST_CORE, ST_STATS, ST_QUANT,
             ST_CAST, ST_COUNT };

int mark(int stage, int end, void* stream) {
  const int i = 2 * stage + end;
  if (tl_events && i < tl_n_events && tl_events[i]) {
    const cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(tl_events[i]), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("kvc_compress stage event: ") + cudaGetErrorString(e));
  }
  return KVC_OK;
}

// per-cell pointers of a contiguous (n, ...) batch
template <typename T>
void cell_ptrs(T** out, void* base, int n, size_t stride_bytes) {
  for (int c = 0; c < n; ++c) out[c] = reinterpret_cast<T*>(static_cast<uint8_t*>(base) + c * stride_bytes);
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" size_t kvc_compress_workspace_bytes(int n_cells, int64_t m, int64_t t, int d, int dtype, int rt, int rd,
                                               int mode_f, int k_f, int mode_t, int k_t, int bits, int scale_mode) {
  if (n_cells <= 0 || m <= 0 || t <= 0 || d <= 0 || rt <= 0 || rd <= 0 || !dtype_ok(dtype)) return 0;
  return sizes(n_cells, m, t, d, dtype, rt, rd, mode_f, k_f, mode_t, k_t, bits, scale_mode).total;
}

extern "C" int kvc_trace_stages(void* const* events, int n_events) {
  tl_events = n_events > 0 ? events : nullptr;
  tl_n_events = n_events > 0 ? n_events : 0;
  return KVC_OK;
}

extern "C" int kvc_compress(int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype, int rt, int rd,
                            int mode_f, int k_f, const float* omega_f, int mode_t, int k_t, const float* omega_t,
                            int n_power, const float* proj, int bits, int symmetric, int scale_mode, int group_size,
                            int stat_dtype, int arith_dtype, int factor_dtype, void* core_out, void* u_token_out,
                            void* u_feature_out, void* core_f, void* u_token_f, void* u_feature_f,
                            double* tail_token, double* tail_feature, double* tails_host, void* tails_ready,
                            float* scale_out, int32_t* zp_out, uint8_t* codes_out, void* workspace,
                            size_t ws_bytes, void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_compress: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || rt <= 0 || rd <= 0 || rd > d || rt > t)
    return fail(KVC_ERR_SHAPE, "kvc_compress: bad shape or ranks");
  if (!dtype_ok(dtype) || !dtype_ok(factor_dtype)) return fail(KVC_ERR_DTYPE, "kvc_compress: bad dtype");
  if (bits != 0 && bits != 2 && bits != 4 && bits != 8) return fail(KVC_ERR_ARG, "kvc_compress: bad bits");
  if (!core_out || !u_token_out || !u_feature_out || !tail_token || !tail_feature)
    return fail(KVC_ERR_ARG, "kvc_compress: NULL output");
  if (bits > 0 && (!scale_out || !zp_out || !codes_out || !proj))
    return fail(KVC_ERR_ARG, "kvc_compress: NULL residual output or projection");
  if (mode_f == KVC_SVD_RANDOMISED && !omega_f) return fail(KVC_ERR_ARG, "kvc_compress: NULL feature sketch");
  if (mode_t == KVC_SVD_RANDOMISED && !omega_t) return fail(KVC_ERR_ARG, "kvc_compress: NULL token sketch");
  const Sizes s = sizes(n_cells, m, t, d, dtype, rt, rd, mode_f, k_f, mode_t, k_t, bits, scale_mode);
  if (!workspace || ws_bytes < s.total) return fail(KVC_ERR_WORKSPACE, "kvc_compress: workspace too small");
  const int n = n_cells;
  const int64_t c = m * rd;
  const int kf = mode_f == KVC_SVD_RANDOMISED ? k_f : 0;
  const int kt = mode_t == KVC_SVD_RANDOMISED ? k_t : 0;
  const int es = dtype_size(dtype);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  double* gram_f = reinterpret_cast<double*>(w);
  double* gram_t = reinterpret_cast<double*>(w + s.gram_f);
  uint8_t* xproj = w + s.gram_f + s.gram_t;
  double* mat = reinterpret_cast<double*>(xproj + s.xproj);
  double* sv2 = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(mat) + s.mat);
  void* scratch = reinterpret_cast<uint8_t*>(sv2) + s.sv2;
  const size_t scr = s.scratch;

  const void* xf[KVC_MAX_CELLS];  // each cell as (m*T, d) rows: the same pointers
  void* xp[KVC_MAX_CELLS];
  void* ud[KVC_MAX_CELLS];
  void* ut[KVC_MAX_CELLS];
  void* co[KVC_MAX_CELLS];
  for (int i = 0; i < n; ++i) {
    if (!x[i]) return fail(KVC_ERR_ARG, "kvc_compress: NULL cell");
    xf[i] = x[i];
  }
  cell_ptrs(xp, xproj, n, (size_t)t * c * es);
  cell_ptrs(ud, u_feature_out, n, (size_t)d * rd * es);
  cell_ptrs(ut, u_token_out, n, (size_t)t * rt * es);
  cell_ptrs(co, core_out, n, (size_t)m * rt * rd * es);
  int rc;
  // --- feature mode: A_f = (m*T, d) rows ---
  if ((rc = mark(ST_GRAM_F, 0, stream))) return rc;
  if ((rc = kvc_gram(n, xf, m * t, d, dtype, omega_f, kf, gram_f, scratch, scr, stream))) return rc;
  if ((rc = mark(ST_GRAM_F, 1, stream))) return rc;
  if ((rc = mark(ST_SOLVE_F, 0, stream))) return rc;
  if ((rc = kvc_sketch_solve(n, mode_f, KVC_SIDE_LEFT, d, m * t, kf, rd, n_power, gram_f,
                             (int64_t)d * d + (int64_t)d * kf + 1, nullptr, u_feature_out, dtype, nullptr, tail_feature,
                             scratch, scr, stream)))
    return rc;
  if ((rc = mark(ST_SOLVE_F, 1, stream))) return rc;
  if ((rc = mark(ST_PROJECT, 0, stream))) return rc;
  if ((rc = kvc_project_feature(n, xf, m, t, d, dtype, ud, rd, xp, stream))) return rc;
  if ((rc = mark(ST_PROJECT, 1, stream))) return rc;
  // --- token mode: A_t = (T, m*rd) ---
  if ((rc = mark(ST_GRAM_T, 0, stream))) return rc;
  if ((rc = kvc_gram(n, xp, t, (int)c, dtype, nullptr, 0, gram_t, scratch, scr, stream))) return rc;
  if ((rc = mark(ST_GRAM_T, 1, stream))) return rc;
  if ((rc = mark(ST_SOLVE_T, 0, stream))) return rc;
  if ((rc = kvc_sketch_solve(n, mode_t, KVC_SIDE_RIGHT, (int)c, t, kt, rt, n_power, gram_t, c * c + 1, omega_t,
                             mat, KVC_F64, nullptr, tail_token, scratch, scr, stream)))
    return rc;
  if ((rc = mark(ST_SOLVE_T, 1, stream))) return rc;
  if (tails_host) {
    // the tail masses are final here: copy them out and signal, so the
    // caller can read them while the remaining stages run
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(tails_host, tail_token, (size_t)n * 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(tails_host + n, tail_feature, (size_t)n * 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && tails_ready) e = cudaEventRecord(static_cast<cudaEvent_t>(tails_ready), st);
    if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("kvc_compress tails copy: ") + cudaGetErrorString(e));
  }
  if ((rc = mark(ST_APPLY, 0, stream))) return rc;
  if ((rc = kvc_apply_basis(n, xp, t, (int)c, dtype, mat, rt, ut, stream))) return rc;
  if ((rc = mark(ST_APPLY, 1, stream))) return rc;
  if ((rc = mark(ST_CORE, 0, stream))) return rc;
  if ((rc = kvc_core(n, xp, ut, t, (int)m, rd, rt, dtype, co, scratch, scr, stream))) return rc;
  if ((rc = mark(ST_CORE, 1, stream))) return rc;
  // --- residual ---
  if (bits > 0) {
    const int ns = scale_mode == KVC_SCALE_CHANNEL ? d
                   : scale_mode == KVC_SCALE_GROUP ? (int)(m * t * (d / std::max(group_size, 1)))
                                                   : 1;
    float* sc[KVC_MAX_CELLS];
    int32_t* zz[KVC_MAX_CELLS];
    uint8_t* cd[KVC_MAX_CELLS];
    cell_ptrs(sc, scale_out, n, (size_t)ns * 4);
    cell_ptrs(zz, zp_out, n, (size_t)ns * 4);
    cell_ptrs(cd, codes_out, n, (size_t)m * t * ((d * bits + 7) / 8));
    if ((rc = mark(ST_STATS, 0, stream))) return rc;
    // the feature Gram (still intact) bounds |R| of each cell for the stats pass
    tc_stats_gram_bound(gram_f, (int64_t)d * d + (int64_t)d * kf + 1);
    if (scale_mode != KVC_SCALE_GROUP)
      rc = kvc_residual_stats(n, xf, m, t, d, dtype, co, ut, ud, rt, rd, proj, bits, symmetric, scale_mode,
                              stat_dtype, sc, zz, scratch, scr, stream);
    tc_stats_gram_bound(nullptr, 0);
    if (rc) return rc;
    if ((rc = mark(ST_STATS, 1, stream))) return rc;
    if ((rc = mark(ST_QUANT, 0, stream))) return rc;
    // the stats call just above left the Tucker row terms in the same scratch
    tc_reuse_tucker_rows(true);
    rc = kvc_residual_quant(n, xf, m, t, d, dtype, co, ut, ud, rt, rd, proj, bits, symmetric, scale_mode,
                            group_size, stat_dtype, arith_dtype, sc, zz, cd, scratch, scr, stream);
    tc_reuse_tucker_rows(false);
    if (rc) return rc;
    if ((rc = mark(ST_QUANT, 1, stream))) return rc;
  }
  if ((rc = mark(ST_CAST, 0, stream))) return rc;
  // --- factors in the payload dtype ---
  if (core_f && (rc = kvc_cast((int64_t)n * m * rt * rd, core_out, dtype, core_f, factor_dtype, stream))) return rc;
  if (u_token_f && (rc = kvc_cast((int64_t)n * t * rt, u_token_out, dtype, u_token_f, factor_dtype, stream)))
    return rc;
  if (u_feature_f && (rc = kvc_cast((int64_t)n * d * rd, u_feature_out, dtype, u_feature_f, factor_dtype, stream)))
    return rc;
  if ((rc = mark(ST_CAST, 1, stream))) return rc;
  return KVC_OK;
}
