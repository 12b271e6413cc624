/*
 * kvc_b200.h -- C ABI of the B200-native (sm_100a) kvcompress hot path.
 *
 * The reference (sachncs/kvcompress) is a Python package; its hot path is
 * JoLTCompressor.compress / decompress (kvcompress/compressor/jolt.py:147-253)
 * and FlashJoLTCompressor.compress_cell (kvcompress/compressor/flashjolt.py:
 * 102-169).  This library replaces the torch ops those methods issue; the
 * Python package kvcompress_b200 binds it with ctypes and keeps the
 * reference's Python API on top.  Each entry point names the reference code
 * it replaces.
 *
 * Conventions
 *  - Plain device pointers and sizes; no allocation, no host synchronisation.
 *    `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *  - "cells": one cell is one layer's K or V, shape (m, T, d) row-major with
 *    m = batch * n_kv_heads (kvcompress/cache/compress.py:308-333).  Batched
 *    entry points take a host array of `n_cells` device pointers, all cells
 *    of one call sharing shape, dtype and allocation.
 *  - Element types: KVC_F32 / KVC_F16 / KVC_BF16 for tensors of the cache's
 *    dtype; KVC_F64 for solver buffers.
 *  - Return 0 on success, a negative KVC_ERR_* on failure; the message is in
 *    kvc_last_error() (thread-local).
 *  - Scratch memory: callers pass `workspace` / `ws_bytes`; the matching
 *    *_workspace_bytes() function gives the size needed.  Calls on different
 *    streams with distinct workspaces are independent.
 */
#ifndef KVC_B200_H
#define KVC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  KVC_OK = 0,
  KVC_ERR_ARG = -1,
  KVC_ERR_SHAPE = -2,
  KVC_ERR_DTYPE = -3,
  KVC_ERR_ALIGN = -4,
  KVC_ERR_WORKSPACE = -5,
  KVC_ERR_LAUNCH = -6,
  KVC_ERR_TIMEOUT = -7,
  KVC_ERR_UNSUPPORTED = -8
};

enum { KVC_F32 = 0, KVC_F16 = 1, KVC_BF16 = 2, KVC_F64 = 3, KVC_FP8E4M3 = 4 };

/* Sketch-solver modes. */
enum { KVC_SVD_EXACT = 0, KVC_SVD_RANDOMISED = 1 };
/* Which side of A the Gram lives on (see kvc_sketch_solve). */
enum { KVC_SIDE_LEFT = 0, KVC_SIDE_RIGHT = 1 };
/* Quantiser scale layouts (kvcompress/compressor/quantization.py:410-452). */
enum { KVC_SCALE_CHANNEL = 0, KVC_SCALE_GROUP = 1, KVC_SCALE_TENSOR = 2 };

#define KVC_MAX_CELLS 64

const char* kvc_last_error(void);
int kvc_abi_version(void);
/* Kernels the calling host thread has launched through the library so far
 * (successful launches; a running count, no counterpart in the reference). */
unsigned long long kvc_launch_count(void);

/*
 * Column Gram and sketch of a row-major (rows x p) matrix A per cell:
 *   out = [ A^T A  (p x p) | A^T Omega (p x k) | sum(A*A) ]      (float64)
 * laid out per cell at stride p*p + p*k + 1.
 *
 * Feature mode: A = x viewed as (m*T, d), so A^T A = A_f A_f^T with
 * A_f = mode_n_unfold(x, 2), and A^T Omega = A_f Omega: the sketch product
 * and the two power iterations of SVD.randomise (kvcompress/compressor/
 * svd.py:259-265) and the Frobenius norm (svd.py:289) reduce to this one
 * pass over x.  Token mode: A = x_proj in (T, m*rd) layout, k = 0.
 * `omega` is one (rows x k) float32 matrix shared by every cell (NULL iff
 * k == 0).  Summation order is fixed: results are bit-reproducible.
 */
size_t kvc_gram_workspace_bytes(int n_cells, int64_t rows, int p, int k);
int kvc_gram(int n_cells, const void* const* a, int64_t rows, int p, int dtype,
             const float* omega, int k, double* out, void* workspace, size_t ws_bytes,
             void* stream);

/*
 * Randomised or exact truncated SVD of an A that is only seen through its
 * Gram (replaces SVD.randomise, svd.py:221-316, and SVD.exact, svd.py:181-219).
 *
 * KVC_SIDE_LEFT (feature mode, A is p x n with n large):
 *   gram per cell = kvc_gram output [G = A A^T | Y0 = A Omega | |A|^2].
 *   Randomised: Q = orth(G^2 Y0) by subspace iteration, Ritz pairs of
 *   Q^T G Q; exact: eigenpairs of G.  basis_out = U (p x rank) rounded to
 *   `basis_dtype` (the input dtype, svd.py:507-510).
 * KVC_SIDE_RIGHT (token mode, A is n x p with n = T large):
 *   gram per cell = H = A^T A (p x p, kvc_gram output with k = 0).
 *   `omega` (p x k, float32, shared).  basis_out = M (p x rank, float64)
 *   with U = A M; apply it with kvc_apply_basis.
 * sv2_out: the leading `rank` squared singular values per cell (may be
 * NULL); tail_out: the discarded Frobenius mass per cell, as the reference
 * reports it (svd.py:98-110 exact, svd.py:289-294 randomised).
 * n_other: the long dimension of A (n), so that min(p, n_other) is the
 * SVD's max_rank; n_power: power iterations (SVD.n_power, svd.py:131-142).
 * Supports p <= 2046 and sketch widths k <= 1024 (q <= 512 gives k <= 513).
 * Only the `rank` leading eigenpairs are computed (Householder
 * tridiagonalisation, bisection, inverse iteration: the dsyevx method).
 */
size_t kvc_sketch_solve_workspace_bytes(int n_cells, int mode, int p, int k);
int kvc_sketch_solve(int n_cells, int mode, int side, int p, int64_t n_other, int k, int rank,
                     int n_power, const double* gram, int64_t gram_stride, const float* omega,
                     void* basis_out, int basis_dtype, double* sv2_out, double* tail_out,
                     void* workspace, size_t ws_bytes, void* stream);

/*
 * x_proj = x  x_3 U_d rounded to the cell dtype (tucker.py:251), written in
 * token-unfolding layout (T, m*rd): x_proj_t[t, h*rd + r]
 * (mode_n_unfold(x_proj, 1), tucker.py:254).
 */
int kvc_project_feature(int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                        int dtype, const void* const* u_feature, int rd, void* const* x_proj_t,
                        void* stream);

/* U = A M rounded to dtype: A (rows x p, dtype), M (p x r, float64 per cell
 * at stride p*r), U (rows x r, dtype).  The lift u = q @ u_b of svd.py:285
 * with the rounding of svd.py:507-510. */
int kvc_apply_basis(int n_cells, const void* const* a, int64_t rows, int p, int dtype,
                    const double* mat, int r, void* const* out, void* stream);

/* core[h, a, r] = sum_t x_proj[h, t, r] * u_token[t, a], rounded to dtype
 * (tucker.py:261).  x_proj_t in (T, m*rd) layout, u_token (T, rt). */
size_t kvc_core_workspace_bytes(int n_cells, int64_t t, int m, int rd, int rt);
int kvc_core(int n_cells, const void* const* x_proj_t, const void* const* u_token, int64_t t,
             int m, int rd, int rt, int dtype, void* const* core, void* workspace,
             size_t ws_bytes, void* stream);

/*
 * JL-rotated residual statistics (pass 1 of encode_residual,
 * residual.py:201-216 + IntQuantizer.compute_params, quantization.py:410-452):
 *   R   = x - reconstruct_partial_tucker(core, u_token, u_feature) in the cell
 *         dtype (einsum order of tucker.py:184-189, jolt.py:311)
 *   Rt  = float32(R) @ proj^T                       (residual.py:204-216)
 * and from the per-column (or whole-tensor) min/max of Rt the quantiser's
 * scale (float32) and zero point (int32).  rt = rd = 0 means "no Tucker
 * term" and proj = NULL means "no rotation": then Rt = x, which is the
 * quantize-only baseline (quantization_only.py:125-175) -- its statistics run
 * in the cell dtype (`stat_dtype`), as the reference's do.
 * scale_mode KVC_SCALE_CHANNEL (d values) or KVC_SCALE_TENSOR (1 value).
 * Min and max are exact and order independent, so the tensor-core path
 * reduces them with integer atomics on order-preserving bit patterns and the
 * result is still bit-reproducible.
 */
size_t kvc_residual_stats_workspace_bytes(int n_cells, int64_t rows, int d, int rd);
int kvc_residual_stats(int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype,
                       const void* const* core, const void* const* u_token,
                       const void* const* u_feature, int rt, int rd, const float* proj,
                       int bits, int symmetric, int scale_mode, int stat_dtype,
                       float* const* scale_out, int32_t* const* zp_out, void* workspace,
                       size_t ws_bytes, void* stream);

/*
 * Pass 2 of encode_residual: recompute Rt, quantise
 * q = clamp(rint(Rt / scale + zp)) (quantization.py:311-363) and bit-pack
 * (bit_packing_signed, quantization.py:181-238) into codes
 * (rows x ceil(d*bits/8)) uint8.  With scale_mode KVC_SCALE_GROUP the
 * per-row group scales (rows x d/group) are computed here and written to
 * scale/zp.  arith_dtype: dtype of the divide/add in the per-tensor branch
 * (0-dim promotion, quantization.py:335-336); KVC_F32 elsewhere.
 */
size_t kvc_residual_quant_workspace_bytes(int n_cells, int64_t rows, int d, int rd);
int kvc_residual_quant(int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype,
                       const void* const* core, const void* const* u_token,
                       const void* const* u_feature, int rt, int rd, const float* proj,
                       int bits, int symmetric, int scale_mode, int group_size, int stat_dtype,
                       int arith_dtype, float* const* scale, int32_t* const* zp,
                       uint8_t* const* codes, void* workspace, size_t ws_bytes, void* stream);

/*
 * Fused decompress of JoLT payloads (reconstruct_payload, jolt.py:401-463 with
 * decode_residual, residual.py:242-288):
 *   out = cast( Tucker(core, u_token, u_feature) in float32
 *              + dequant(codes) @ proj , out_dtype )
 * for the token range [t0, t1) of every cell (t0 = 0, t1 = T: the whole
 * cell).  out is (m, t1 - t0, d).  Factors are float16 (factor_dtype).
 * bits == 0: no residual term.  rt = rd = 0 / proj = NULL: the
 * quantize-only decoder (quantization_only.py:177-198).
 */
size_t kvc_decompress_workspace_bytes(int n_cells, int64_t rows, int d, int rd);
int kvc_decompress(int n_cells, const uint8_t* const* codes, const float* const* scale,
                   const int32_t* const* zp, int bits, int symmetric, int scale_mode,
                   int group_size, const void* const* core, const void* const* u_token,
                   const void* const* u_feature, int factor_dtype, int64_t m, int64_t t, int d,
                   int rt, int rd, const float* proj, int64_t t0, int64_t t1, int out_dtype,
                   void* const* out, void* workspace, size_t ws_bytes, void* stream);

/*
 * kvc_decompress without a workspace argument: no counterpart in the
 * reference.  It is for callers that cannot provide device scratch: a host
 * runtime binding this ABI directly with no device allocator of its own, or
 * an engine that forbids device allocation on its decode path.  It runs the
 * same kernels as kvc_decompress, with scratch in a fixed array of
 * KVC_NOALLOC_SCRATCH_BYTES per device inside this library, and allocates
 * nothing.
 *  - Limit: decodes that take the tensor-core decoder (bf16 output at d of
 *    64 or 128, or fp32 output at d = 64; a JL rotation, symmetric
 *    per-channel scales) and whose
 *    kvc_decompress_workspace_bytes(n_cells, m*t, d, rd) exceeds
 *    KVC_NOALLOC_SCRATCH_BYTES fail with KVC_ERR_WORKSPACE (K and V of one
 *    Llama-3-8B layer at 8k tokens need about 0.7 MB).  Other layouts are
 *    decoded by the SIMT kernel, which uses no scratch, at any size.
 *  - The first call on each device (and again after that device's context
 *    was destroyed and re-created) looks up the array's address
 *    (cudaGetSymbolAddress, which may load the module): make it before any
 *    stream capture.
 *  - Nothing in the array has to start at zero; each call writes every byte
 *    it reads.
 *  - One array per device: calls that overlap on the device (different
 *    streams or host threads) race on it.  Calls on one stream are safe.
 */
#define KVC_NOALLOC_SCRATCH_BYTES (8u << 20)
int kvc_decompress_noalloc(int n_cells, const uint8_t* const* codes, const float* const* scale,
                           const int32_t* const* zp, int bits, int symmetric, int scale_mode,
                           int group_size, const void* const* core, const void* const* u_token,
                           const void* const* u_feature, int factor_dtype, int64_t m, int64_t t,
                           int d, int rt, int rd, const float* proj, int64_t t0, int64_t t1,
                           int out_dtype, void* const* out, void* stream);

/*
 * The whole compress of a batch of same-shape cells in one call:
 * partial_tucker_st_hosvd + encode_residual (tucker.py:192-279,
 * residual.py:155-239, as orchestrated by jolt.py:273-329).  Runs kvc_gram,
 * kvc_sketch_solve, kvc_project_feature, kvc_gram, kvc_sketch_solve,
 * kvc_apply_basis, kvc_core, kvc_residual_stats (not for group scales),
 * kvc_residual_quant and the factor casts on one stream.  rt / rd are the
 * clipped ranks, mode_* / k_* the SVD mode and sketch width of each side
 * (omega_f: (m*T, k_f) and omega_t: (m*rd, k_t) float32, NULL for exact).
 * Outputs are contiguous batches, cell-major: core (n, m, rt, rd),
 * u_token (n, T, rt), u_feature (n, d, rd) in the cell dtype; core_f /
 * u_token_f / u_feature_f in factor_dtype (NULL: no cast); tails (n,) fp64,
 * also copied to tails_host (2n doubles, token then feature; host memory,
 * pinned for an asynchronous copy; NULL: no copy) as soon as the solves are
 * done, after which tails_ready (a cudaEvent_t, optional) is recorded;
 * with bits > 0 scales / zero points ((n, d), (n, m*T, d/g) or (n,)) and
 * codes (n, m*T, ceil(d*bits/8)).  Intermediates live in the workspace.
 */
size_t kvc_compress_workspace_bytes(int n_cells, int64_t m, int64_t t, int d, int dtype, int rt, int rd,
                                    int mode_f, int k_f, int mode_t, int k_t, int bits, int scale_mode);
int kvc_compress(int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype, int rt, int rd,
                 int mode_f, int k_f, const float* omega_f, int mode_t, int k_t, const float* omega_t,
                 int n_power, const float* proj, int bits, int symmetric, int scale_mode, int group_size,
                 int stat_dtype, int arith_dtype, int factor_dtype, void* core_out, void* u_token_out,
                 void* u_feature_out, void* core_f, void* u_token_f, void* u_feature_f,
                 double* tail_token, double* tail_feature, double* tails_host, void* tails_ready,
                 float* scale_out, int32_t* zp_out, uint8_t* codes_out, void* workspace, size_t ws_bytes,
                 void* stream);

/* Stage timing of kvc_compress on the calling thread: events[2 i] and
 * events[2 i + 1] (cudaEvent_t) are recorded on the call's stream around
 * stage i = feature Gram, feature solve, projection, token Gram, token
 * solve, U_T, core, residual stats, quantise, casts.  n_events = 0 stops. */
int kvc_trace_stages(void* const* events, int n_events);

/*
 * Token-range decode streams (a consumer that reads the cache in blocks of
 * tokens, e.g. 256-token blocks per layer).  The reference decodes a whole
 * payload per call (reconstruct_payload, jolt.py:401-463); these split that
 * decode into a plan made once per set of payloads and runs over [t0, t1).
 *  - kvc_decode_plan_bytes: size of the caller-owned host buffer of a plan.
 *  - kvc_decode_plan_init: same arguments as kvc_decompress without the
 *    range and outputs.  Builds the codes tensor maps into the plan and each
 *    cell's B image into the workspace (kvc_decompress_workspace_bytes of
 *    the full payloads); the workspace and the payload tensors must stay
 *    alive and unchanged while the plan is used.  Only layouts that take the
 *    tensor-core decode have plans; others return KVC_ERR_UNSUPPORTED
 *    (decode them with kvc_decompress).
 *  - kvc_decode_plan_run: decodes tokens [t0, t1) of every cell into out[c]
 *    ((m, t1 - t0, d) of the plan's out_dtype, 16-byte aligned): for bf16
 *    output one kernel launch for rank-1 factors in fp16 / bf16 over whole
 *    128-token blocks starting at a multiple of 8 (the row terms are formed
 *    inside the decode), two otherwise; bit for bit the same rows as kvc_decompress over that range.  Runs of one plan
 *    share its workspace: issue them on one stream.  While the stream is
 *    being captured into a CUDA graph, a one-kernel run (head_dim 128) is
 *    launched as a programmatic dependent of the previous launch, so
 *    consecutive runs may overlap: give each captured run its own outputs.
 */
size_t kvc_decode_plan_bytes(void);
int kvc_decode_plan_init(void* plan, size_t plan_bytes, int n_cells, const uint8_t* const* codes,
                         const float* const* scale, const int32_t* const* zp, int bits, int symmetric,
                         int scale_mode, int group_size, const void* const* core,
                         const void* const* u_token, const void* const* u_feature, int factor_dtype,
                         int64_t m, int64_t t, int d, int rt, int rd, const float* proj, int out_dtype,
                         void* workspace, size_t ws_bytes, void* stream);
int kvc_decode_plan_run(const void* plan, size_t plan_bytes, int64_t t0, int64_t t1, void* const* out,
                        void* stream);

/*
 * Kernel selection.  Policy 0 (default): the residual encode of bf16 cells
 * with a JL rotation and channel / tensor scales runs on the tcgen05
 * tensor-core kernels for d = 64 with rd <= 4 and d = 128 with rd <= 16
 * (rd > 4: the quantise pass needs 8- or 4-bit codes), that of fp32 cells
 * for d = 64 with rd <= 4 (the residual and Pi each in three bf16 terms,
 * the six products of order up to two: fp32 accuracy), and symmetric
 * per-channel 8/4/2-bit decodes with rd <= 16 run on the tcgen05 decoder
 * for bf16 output at d = 64 / 128 and fp32 output at d = 64 (diag(scale) Pi
 * in three bf16 terms); everything else on the SIMT kernels.  Policy 1: SIMT kernels
 * only (used to cross-check the two).
 * Under policy 0 the quantise pass runs feature-major for d = 128 with 8-
 * or 4-bit codes (Pi / s in TMEM, the rows in shared memory), and inside a
 * compress call (after the stats pass, rank-1 row terms, per-channel
 * scales) in its fp16 two-term mode: Pi / s in two fp16 terms and R scaled
 * by a power of two per cell.  Policy 2: the stats pass in fp16 too (R
 * scaled by a power of two per cell from a bound on |R| inside a compress
 * call, per 128-row tile otherwise).  Policy 3: bf16 operands with
 * the row-major quantise pass; policy 4: bf16 operands with the
 * feature-major one (both for comparison).
 * Process-wide; set it while no call is in flight.
 */
int kvc_set_kernel_policy(int policy);

/* Reads and clears the device-side error word (an mbarrier wait in a
 * tensor-core kernel that gave up records a nonzero code).  Synchronises
 * the device: a diagnostic, not for the hot path. */
int kvc_device_error(int* code);

/* Elementwise cast between KVC_F32/F16/BF16/FP8E4M3 (torch .to semantics:
 * round to nearest even; float8_e4m3fn does not saturate -- magnitudes that
 * round above 448 become NaN).  Used by the fp8/fp16/bf16 identity
 * compressors (identity.py:68-117, dispatch.py:106-125). */
int kvc_cast(int64_t n, const void* in, int in_dtype, void* out, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVC_B200_H */
