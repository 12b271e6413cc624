// JL-rotated residual encode (stats + quantise/pack) and the fused decode,
// general SIMT kernels: every dtype, head_dim <= 256, every Tucker rank and
// every quantiser layout of the reference (symmetric / asymmetric,
// per-channel / per-group / per-tensor, 2/4/8 bits).
//
// Reference semantics followed here (paths relative to the reference root):
//  * residual in the cell dtype: x - einsum("mar,ta,dr->mtd") with the
//    einsum contracted left to right, each product rounded to the dtype
//    (tucker.py:184-189, jolt.py:310-311 / flashjolt.py:148-150);
//  * rotation Rt = float32(R) @ Pi^T (residual.py:204-216);
//  * scale / zero point from column (or tensor) min/max
//    (quantization.py:410-452), quantise with an IEEE divide, round half to
//    even, clamp (quantization.py:340-357), pack (quantization.py:181-238);
//  * decode: unpack, (q - zp) * scale in fp32, @ Pi (residual.py:287), add
//    the fp32 Tucker term, cast (jolt.py:424-463).
#include <algorithm>

#include "kvc_common.cuh"
#include "kvc_plan.cuh"
#include "kvc_quant.cuh"

namespace kvc {

bool tc_residual_eligible(int dtype, int d, int rd, const float* proj, int scale_mode);
bool tc_quant_fm_eligible(int d, int bits, int scale_mode, int arith_dtype);
size_t tc_residual_workspace(int n_cells, int64_t rows, int d, int rd);
int simt_row_terms(const void* const* core, const void* const* ut, int n_cells, int dtype, int64_t m, int64_t t,
                   int rt, int rd, int stride, float* tmp, cudaStream_t st);
static size_t align256_(size_t x) { return (x + 255) & ~(size_t)255; }
int tc_residual_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype,
                       const void* const* core, const void* const* u_token, const void* const* u_feature,
                       int rt, int rd, const float* proj, int bits, int symmetric, int scale_mode,
                       int stat_dtype, int arith_dtype, float* const* scale, int32_t* const* zp,
                       uint8_t* const* codes, void* workspace, size_t ws_bytes, cudaStream_t st);
bool tc_decompress_eligible(int out_dtype, int d, int rd, int bits, int symmetric, int scale_mode,
                            const float* proj);
size_t tc_decompress_workspace(int n_cells, int64_t rows, int d, int rd);
int tc_decompress_launch(int n_cells, const uint8_t* const* codes, const float* const* scale, int bits,
                         const void* const* core, const void* const* u_token, const void* const* u_feature,
                         int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd, const float* proj,
                         int64_t t0, int64_t t1, int out_dtype, void* const* out, void* workspace,
                         size_t ws_bytes, cudaStream_t st);
void tc_reuse_tucker_rows(bool allow);
int tc_read_device_error(int* out);
int tc_gram_read_device_error(int* out);

// 0: tensor cores when eligible (the quantise pass in its fp16 two-term
// mode where it applies), 1: SIMT kernels only, 2: as 0 with the stats pass
// in fp16 too, 3: bf16 operands with the row-major quantise pass, 4: bf16
// operands with the feature-major quantise pass
static int g_policy = 0;
int kernel_policy() { return g_policy; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename P>
static bool all_aligned(int n, P const* ptrs) {
  for (int c = 0; c < n; ++c)
    if (ptrs[c] && !aligned16(ptrs[c])) return false;
  return true;
}

namespace {

constexpr int ROWS = 32;
constexpr int NT = 256;
constexpr int MAXD = 256;

struct ResArgs {
  CellPtrs x, core, ut, ud;
  int64_t m, t, rows;
  int d, rt, rd, dtype;
  const float* proj;  // Pi, row-major d x d (NULL: no rotation)
  int bits, symmetric, scale_mode, group_size, stat_dtype, arith_dtype;
  // stats
  float* partial;  // [cell][block][2][d]
  int blocks_per_cell;
  // quant
  CellPtrsMut scale, zp, codes;
  int code_bytes;
  int pi_in_smem;
  // the Tucker row terms of every row, precomputed ([cell][row][rt_stride],
  // rounded to the cell dtype), or NULL: each tile forms its own
  const float* rowterm;
  int rt_stride;
};

// Load a tile of rows into xs (fp32), subtract the Tucker reconstruction in
// the cell dtype, rotate into rot.  Returns the number of valid rows.
template <typename T>
__device__ int residual_tile(const ResArgs& A, int cell, int64_t r0, float* xs, float* rot,
                             float* tmp, const float* pi_s) {
  const int d = A.d;
  const int nrow = (int)((A.rows - r0) < ROWS ? (A.rows - r0) : ROWS);
  const T* x = static_cast<const T*>(A.x.p[cell]);
  for (int e = threadIdx.x; e < ROWS * d; e += NT) {
    const int rr = e / d, j = e % d;
    xs[e] = rr < nrow ? Elt<T>::to_f32(x[(r0 + rr) * d + j]) : 0.f;
  }
  __syncthreads();
  if (A.rt > 0) {
    const T* core = static_cast<const T*>(A.core.p[cell]);
    const T* ut = static_cast<const T*>(A.ut.p[cell]);
    const T* ud = static_cast<const T*>(A.ud.p[cell]);
    const int rt = A.rt, rd = A.rd;
    for (int e = threadIdx.x; e < ROWS * rd; e += NT) {
      const int rr = e / rd, r = e % rd;
      float s = 0.f;
      if (A.rowterm) {
        if (rr < nrow) s = A.rowterm[((int64_t)cell * A.rows + r0 + rr) * A.rt_stride + r];
      } else {
        if (rr < nrow) {
          const int64_t row = r0 + rr;
          const int64_t h = row / A.t, t = row % A.t;
          const T* cr = core + h * rt * rd + r;
          const T* ur = ut + t * rt;
          for (int a = 0; a < rt; ++a)
            s = fmaf(Elt<T>::to_f32(cr[(int64_t)a * rd]), Elt<T>::to_f32(ur[a]), s);
        }
        s = Elt<T>::round(s);
      }
      tmp[e] = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < ROWS * d; e += NT) {
      const int rr = e / d, j = e % d;
      float s = 0.f;
      for (int r = 0; r < rd; ++r) s = fmaf(tmp[rr * rd + r], Elt<T>::to_f32(ud[(int64_t)j * rd + r]), s);
      xs[e] = Elt<T>::round(xs[e] - Elt<T>::round(s));
    }
    __syncthreads();
  }
  if (A.proj) {
    for (int e = threadIdx.x; e < ROWS * d; e += NT) {
      const int rr = e / d, j = e % d;
      const float* xr = xs + rr * d;
      float s = 0.f;
      if (pi_s) {
        for (int k = 0; k < d; ++k) s = fmaf(xr[k], pi_s[k * d + j], s);
      } else {
        const float* pj = A.proj + (int64_t)j * d;
        for (int k = 0; k < d; ++k) s = fmaf(xr[k], __ldg(pj + k), s);
      }
      rot[e] = s;
    }
  } else {
    for (int e = threadIdx.x; e < ROWS * d; e += NT) rot[e] = xs[e];
  }
  __syncthreads();
  return nrow;
}

// Pi^T into shared memory: pi_s[k * d + j] = Pi[j][k].
__device__ void load_pi_t(const float* proj, int d, float* pi_s) {
  for (int e = threadIdx.x; e < d * d; e += NT) {
    const int j = e / d, k = e % d;
    pi_s[k * d + j] = proj[e];
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(NT) residual_stats_kernel(ResArgs A) {
  extern __shared__ float smem[];
  const int d = A.d;
  float* pi_s = A.pi_in_smem ? smem : nullptr;
  float* xs = smem + (A.pi_in_smem ? d * d : 0);
  float* rot = xs + ROWS * d;
  float* tmp = rot + ROWS * d;
  __shared__ float red_min[NT], red_max[NT];
  const int cell = blockIdx.y;
  if (pi_s) load_pi_t(A.proj, d, pi_s);
  // each thread owns column j = tid % d over rows (tid / d) + k * (NT / d);
  // d <= MAXD == NT, so one pass covers every column.
  const int lanes = NT / d;
  float vmin = __int_as_float(0x7f800000), vmax = -__int_as_float(0x7f800000);
  const int64_t tiles = ceil_div(A.rows, ROWS);
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int nrow = residual_tile<T>(A, cell, tile * ROWS, xs, rot, tmp, pi_s);
    if ((int)threadIdx.x < lanes * d) {
      const int j = threadIdx.x % d, l = threadIdx.x / d;
      for (int rr = l; rr < nrow; rr += lanes) {
        const float v = rot[rr * d + j];
        vmin = fminf(vmin, v);
        vmax = fmaxf(vmax, v);
      }
    }
    __syncthreads();
  }
  // combine the lanes of each column
  float* out = A.partial + ((int64_t)cell * A.blocks_per_cell + blockIdx.x) * 2 * d;
  red_min[threadIdx.x] = vmin;
  red_max[threadIdx.x] = vmax;
  __syncthreads();
  if ((int)threadIdx.x < d) {
    float a = red_min[threadIdx.x], b = red_max[threadIdx.x];
    for (int l = 1; l < lanes; ++l) {
      a = fminf(a, red_min[threadIdx.x + l * d]);
      b = fmaxf(b, red_max[threadIdx.x + l * d]);
    }
    out[threadIdx.x] = a;
    out[d + threadIdx.x] = b;
  }
}

__global__ void stats_finalize_kernel(const float* __restrict__ partial, int n_cells, int blocks,
                                      int d, int bits, int symmetric, int scale_mode, int stat_dt,
                                      CellPtrsMut scale, CellPtrsMut zp) {
  const int cell = blockIdx.x;
  __shared__ float smin[NT], smax[NT];
  const float* base = partial + (int64_t)cell * blocks * 2 * d;
  float tmin = __int_as_float(0x7f800000), tmax = -__int_as_float(0x7f800000);
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float a = __int_as_float(0x7f800000), b = -__int_as_float(0x7f800000);
    for (int bl = 0; bl < blocks; ++bl) {
      a = fminf(a, base[(int64_t)bl * 2 * d + j]);
      b = fmaxf(b, base[(int64_t)bl * 2 * d + d + j]);
    }
    if (scale_mode == KVC_SCALE_CHANNEL) {
      float s;
      int32_t z;
      params_from_minmax(a, b, bits, symmetric, stat_dt, s, z);
      static_cast<float*>(scale.p[cell])[j] = s;
      static_cast<int32_t*>(zp.p[cell])[j] = z;
    }
    tmin = fminf(tmin, a);
    tmax = fmaxf(tmax, b);
  }
  if (scale_mode != KVC_SCALE_TENSOR) return;
  smin[threadIdx.x] = tmin;
  smax[threadIdx.x] = tmax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = smin[0], b = smax[0];
    for (int i = 1; i < (int)blockDim.x; ++i) {
      a = fminf(a, smin[i]);
      b = fmaxf(b, smax[i]);
    }
    float s;
    int32_t z;
    params_from_minmax(a, b, bits, symmetric, stat_dt, s, z);
    static_cast<float*>(scale.p[cell])[0] = s;
    static_cast<int32_t*>(zp.p[cell])[0] = z;
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) residual_quant_kernel(ResArgs A) {
  extern __shared__ float smem[];
  const int d = A.d;
  float* pi_s = A.pi_in_smem ? smem : nullptr;
  float* xs = smem + (A.pi_in_smem ? d * d : 0);
  float* rot = xs + ROWS * d;
  float* tmp = rot + ROWS * d;
  float* gsc = tmp + ROWS * (A.rd > 0 ? A.rd : 1);  // ROWS * (d / group) scales
  int32_t* gzp = reinterpret_cast<int32_t*>(gsc + ROWS * MAXD);
  const int cell = blockIdx.y;
  if (pi_s) load_pi_t(A.proj, d, pi_s);
  int qmin, qmax;
  qrange(A.bits, A.symmetric, qmin, qmax);
  const int offset = A.symmetric ? (1 << (A.bits - 1)) : 0;
  const int per = 8 / A.bits;
  const int mask = (1 << A.bits) - 1;
  const float* scale = static_cast<const float*>(A.scale.p[cell]);
  const int32_t* zp = static_cast<const int32_t*>(A.zp.p[cell]);
  uint8_t* codes = static_cast<uint8_t*>(A.codes.p[cell]);
  const int64_t tiles = ceil_div(A.rows, ROWS);
  const int ng = A.scale_mode == KVC_SCALE_GROUP ? d / A.group_size : 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t r0 = tile * ROWS;
    const int nrow = residual_tile<T>(A, cell, r0, xs, rot, tmp, pi_s);
    if (A.scale_mode == KVC_SCALE_GROUP) {
      for (int e = threadIdx.x; e < nrow * ng; e += NT) {
        const int rr = e / ng, g = e % ng;
        float a = __int_as_float(0x7f800000), b = -__int_as_float(0x7f800000);
        for (int i = 0; i < A.group_size; ++i) {
          const float v = rot[rr * d + g * A.group_size + i];
          a = fminf(a, v);
          b = fmaxf(b, v);
        }
        float s;
        int32_t z;
        params_from_minmax(a, b, A.bits, A.symmetric, A.stat_dtype, s, z);
        gsc[rr * ng + g] = s;
        gzp[rr * ng + g] = z;
        float* so = static_cast<float*>(A.scale.p[cell]);
        int32_t* zo = static_cast<int32_t*>(A.zp.p[cell]);
        so[(r0 + rr) * ng + g] = s;
        zo[(r0 + rr) * ng + g] = z;
      }
      __syncthreads();
    }
    const int cb = A.code_bytes;
    for (int e = threadIdx.x; e < nrow * cb; e += NT) {
      const int rr = e / cb, byte = e % cb;
      unsigned v = 0;
      for (int u = 0; u < per; ++u) {
        const int j = byte * per + u;
        unsigned code = 0;
        if (j < d) {
          float s;
          int32_t z;
          int ad = KVC_F32;
          if (A.scale_mode == KVC_SCALE_CHANNEL) {
            s = scale[j];
            z = zp[j];
          } else if (A.scale_mode == KVC_SCALE_GROUP) {
            s = gsc[rr * ng + j / A.group_size];
            z = gzp[rr * ng + j / A.group_size];
          } else {
            s = scale[0];
            z = zp[0];
            ad = A.arith_dtype;
          }
          const int q = quantize_one(rot[rr * d + j], s, z, qmin, qmax, ad);
          code = (unsigned)((q + offset) & 0xFF) & (unsigned)mask;
        }
        v |= code << (A.bits * (per - 1 - u));
      }
      codes[(r0 + rr) * cb + byte] = (uint8_t)v;
    }
    __syncthreads();
  }
}

// ------------------------------- decode ------------------------------------

struct DecArgs {
  CellPtrs codes, scale, zp, core, ut, ud;
  CellPtrsMut out;
  int bits, symmetric, scale_mode, group_size, factor_dtype, out_dtype;
  int64_t m, t, t0, t1;
  int d, rt, rd, code_bytes;
  const float* proj;  // Pi row-major (flat = deq @ Pi)
  int pi_in_smem;
};

template <typename TOut>
__global__ void __launch_bounds__(NT) decompress_kernel(DecArgs A) {
  extern __shared__ float smem[];
  const int d = A.d;
  float* pi_s = A.pi_in_smem ? smem : nullptr;
  float* deq = smem + (A.pi_in_smem ? d * d : 0);
  float* tmp = deq + ROWS * d;
  const int cell = blockIdx.y;
  if (pi_s) {
    for (int e = threadIdx.x; e < d * d; e += NT) pi_s[e] = A.proj[e];
    __syncthreads();
  }
  const int64_t tl = A.t1 - A.t0;
  const int64_t rows = A.m * tl;
  const int64_t tiles = ceil_div(rows, ROWS);
  const uint8_t* codes = static_cast<const uint8_t*>(A.codes.p[cell]);
  const float* scale = static_cast<const float*>(A.scale.p[cell]);
  const int32_t* zp = static_cast<const int32_t*>(A.zp.p[cell]);
  TOut* out = static_cast<TOut*>(A.out.p[cell]);
  const int offset = A.symmetric ? (1 << (A.bits - 1)) : 0;
  const int per = A.bits > 0 ? 8 / A.bits : 1;
  const int mask = A.bits > 0 ? (1 << A.bits) - 1 : 0;
  const int ng = A.scale_mode == KVC_SCALE_GROUP ? d / A.group_size : 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t o0 = tile * ROWS;
    const int nrow = (int)((rows - o0) < ROWS ? (rows - o0) : ROWS);
    // residual term
    if (A.bits > 0) {
      for (int e = threadIdx.x; e < ROWS * d; e += NT) {
        const int rr = e / d, k = e % d;
        float v = 0.f;
        if (rr < nrow) {
          const int64_t orow = o0 + rr;
          const int64_t h = orow / tl, t = A.t0 + orow % tl;
          const int64_t row = h * A.t + t;
          const uint8_t byte = codes[row * A.code_bytes + k / per];
          const int q = (int)((byte >> (A.bits * (per - 1 - k % per))) & mask) - offset;
          float s;
          int32_t z;
          if (A.scale_mode == KVC_SCALE_CHANNEL) {
            s = scale[k];
            z = zp[k];
          } else if (A.scale_mode == KVC_SCALE_GROUP) {
            s = scale[row * ng + k / A.group_size];
            z = zp[row * ng + k / A.group_size];
          } else {
            s = scale[0];
            z = zp[0];
          }
          v = __fmul_rn((float)(q - z), s);
        }
        deq[e] = v;
      }
      __syncthreads();
    }
    if (A.rt > 0) {
      const int rt = A.rt, rd = A.rd;
      for (int e = threadIdx.x; e < ROWS * rd; e += NT) {
        const int rr = e / rd, r = e % rd;
        float s = 0.f;
        if (rr < nrow) {
          const int64_t orow = o0 + rr;
          const int64_t h = orow / tl, t = A.t0 + orow % tl;
          for (int a = 0; a < rt; ++a)
            s = fmaf(load_dt(A.core.p[cell], (h * rt + a) * rd + r, A.factor_dtype),
                     load_dt(A.ut.p[cell], t * rt + a, A.factor_dtype), s);
        }
        tmp[e] = s;
      }
      __syncthreads();
    }
    for (int e = threadIdx.x; e < nrow * d; e += NT) {
      const int rr = e / d, j = e % d;
      float val = 0.f;
      if (A.rt > 0) {
        for (int r = 0; r < A.rd; ++r)
          val = fmaf(tmp[rr * A.rd + r], load_dt(A.ud.p[cell], (int64_t)j * A.rd + r, A.factor_dtype), val);
      }
      if (A.bits > 0) {
        float f;
        if (A.proj) {
          f = 0.f;
          const float* dr = deq + rr * d;
          if (pi_s) {
            for (int k = 0; k < d; ++k) f = fmaf(dr[k], pi_s[k * d + j], f);
          } else {
            for (int k = 0; k < d; ++k) f = fmaf(dr[k], __ldg(A.proj + (int64_t)k * d + j), f);
          }
        } else {
          f = deq[rr * d + j];
        }
        val = A.rt > 0 ? __fadd_rn(val, f) : f;
      }
      out[(o0 + rr) * d + j] = Elt<TOut>::from(val);
    }
    __syncthreads();
  }
}

int fill_res_args(ResArgs& a, int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                  int dtype, const void* const* core, const void* const* u_token,
                  const void* const* u_feature, int rt, int rd, const float* proj, int bits,
                  int symmetric, int scale_mode, int stat_dtype) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "residual: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || d > MAXD) return fail(KVC_ERR_SHAPE, "residual: bad shape (d <= 256)");
  if (!dtype_ok(dtype) || !dtype_ok(stat_dtype)) return fail(KVC_ERR_DTYPE, "residual: bad dtype");
  if (bits != 2 && bits != 4 && bits != 8) return fail(KVC_ERR_ARG, "residual: bits must be 2, 4 or 8");
  if (rt < 0 || rd < 0 || (rt == 0) != (rd == 0) || rd > d) return fail(KVC_ERR_SHAPE, "residual: bad ranks");
  if (scale_mode < KVC_SCALE_CHANNEL || scale_mode > KVC_SCALE_TENSOR)
    return fail(KVC_ERR_ARG, "residual: bad scale_mode");
  memset(&a, 0, sizeof(a));
  for (int c = 0; c < n_cells; ++c) {
    if (!x[c]) return fail(KVC_ERR_ARG, "residual: NULL x");
    a.x.p[c] = x[c];
    if (rt > 0) {
      if (!core[c] || !u_token[c] || !u_feature[c]) return fail(KVC_ERR_ARG, "residual: NULL factor");
      a.core.p[c] = core[c];
      a.ut.p[c] = u_token[c];
      a.ud.p[c] = u_feature[c];
    }
  }
  a.m = m;
  a.t = t;
  a.rows = m * t;
  a.d = d;
  a.rt = rt;
  a.rd = rd;
  a.dtype = dtype;
  a.proj = proj;
  a.bits = bits;
  a.symmetric = symmetric ? 1 : 0;
  a.scale_mode = scale_mode;
  a.stat_dtype = stat_dtype;
  a.arith_dtype = KVC_F32;
  a.pi_in_smem = (proj && d <= 128) ? 1 : 0;
  return KVC_OK;
}

size_t res_smem(const ResArgs& a, bool quant) {
  size_t f = (a.pi_in_smem ? (size_t)a.d * a.d : 0) + 2 * (size_t)ROWS * a.d +
             (size_t)ROWS * (a.rd > 0 ? a.rd : 1);
  if (quant) f += 2 * (size_t)ROWS * MAXD;
  return f * sizeof(float);
}

// Row terms precomputed once per call (simt_row_terms) from this rt on.
constexpr int ROWTERM_RT = 8;
int rowterm_stride(int rd) { return rd <= 1 ? 1 : (rd <= 4 ? 4 : (rd <= 16 ? 16 : rd)); }
size_t rowterm_bytes(int n_cells, int64_t rows, int rd) {
  return rd > 0 ? align256_(sizeof(float) * (size_t)n_cells * rows * rowterm_stride(rd)) : 0;
}

int blocks_per_cell(int64_t rows, int n_cells) {
  const int64_t tiles = ceil_div(rows, ROWS);
  const int64_t want = ceil_div(4LL * num_sms(), n_cells);
  return (int)std::max<int64_t>(1, std::min<int64_t>(tiles, want));
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" size_t kvc_residual_stats_workspace_bytes(int n_cells, int64_t rows, int d, int rd) {
  if (n_cells <= 0 || rows <= 0 || d <= 0 || rd < 0) return 0;
  return std::max(align256_((size_t)n_cells * blocks_per_cell(rows, n_cells) * 2 * d * sizeof(float)) +
                      rowterm_bytes(n_cells, rows, rd),
                  tc_residual_workspace(n_cells, rows, d, rd));
}

extern "C" size_t kvc_residual_quant_workspace_bytes(int n_cells, int64_t rows, int d, int rd) {
  if (n_cells <= 0 || rows <= 0 || d <= 0 || rd < 0) return 0;
  return std::max(tc_residual_workspace(n_cells, rows, d, rd), rowterm_bytes(n_cells, rows, rd));
}

extern "C" size_t kvc_decompress_workspace_bytes(int n_cells, int64_t rows, int d, int rd) {
  if (n_cells <= 0 || rows <= 0 || d <= 0 || rd < 0) return 0;
  return tc_decompress_workspace(n_cells, rows, d, rd);
}

extern "C" int kvc_set_kernel_policy(int policy) {
  if (policy < 0 || policy > 4)
    return fail(KVC_ERR_ARG,
                "kvc_set_kernel_policy: 0 (auto), 1 (SIMT), 2 (fp16 stats and quantise), 3 (bf16, row-major "
                "quantise) or 4 (bf16, feature-major quantise)");
  g_policy = policy;
  return KVC_OK;
}

extern "C" int kvc_device_error(int* code) {
  if (!code) return fail(KVC_ERR_ARG, "kvc_device_error: NULL");
  int a = 0, b = 0;
  int rc = tc_read_device_error(&a);
  if (rc) return rc;
  if ((rc = tc_gram_read_device_error(&b))) return rc;
  *code = a ? a : b;
  return KVC_OK;
}

extern "C" int kvc_residual_stats(int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                                  int dtype, const void* const* core, const void* const* u_token,
                                  const void* const* u_feature, int rt, int rd, const float* proj,
                                  int bits, int symmetric, int scale_mode, int stat_dtype,
                                  float* const* scale_out, int32_t* const* zp_out, void* workspace,
                                  size_t ws_bytes, void* stream) {
  ResArgs a;
  int rc = fill_res_args(a, n_cells, x, m, t, d, dtype, core, u_token, u_feature, rt, rd, proj, bits,
                         symmetric, scale_mode, stat_dtype);
  if (rc) return rc;
  if (scale_mode == KVC_SCALE_GROUP) return fail(KVC_ERR_ARG, "kvc_residual_stats: group scales need no stats pass");
  cudaStream_t st0 = static_cast<cudaStream_t>(stream);
  if (g_policy != 1 && tc_residual_eligible(dtype, d, rd, proj, scale_mode) && all_aligned(n_cells, x) &&
      workspace && ws_bytes >= tc_residual_workspace(n_cells, m * t, d, rd)) {
    return tc_residual_launch(0, n_cells, x, m, t, d, dtype, core, u_token, u_feature, rt, rd, proj, bits, symmetric,
                              scale_mode, stat_dtype, KVC_F32, scale_out, zp_out, nullptr, workspace, ws_bytes,
                              st0);
  }
  const int bpc = blocks_per_cell(a.rows, n_cells);
  const size_t need = (size_t)n_cells * bpc * 2 * d * sizeof(float);
  if (!workspace || ws_bytes < need) return fail(KVC_ERR_WORKSPACE, "kvc_residual_stats: workspace too small");
  a.partial = static_cast<float*>(workspace);
  a.blocks_per_cell = bpc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rt >= ROWTERM_RT && ws_bytes >= align256_(need) + rowterm_bytes(n_cells, a.rows, rd)) {
    float* rows_tmp = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256_(need));
    if ((rc = simt_row_terms(core, u_token, n_cells, dtype, m, t, rt, rd, rowterm_stride(rd), rows_tmp, st)))
      return rc;
    a.rowterm = rows_tmp;
    a.rt_stride = rowterm_stride(rd);
  }
  CellPtrsMut sc, zz;
  for (int c = 0; c < n_cells; ++c) {
    if (!scale_out[c] || !zp_out[c]) return fail(KVC_ERR_ARG, "kvc_residual_stats: NULL output");
    sc.p[c] = scale_out[c];
    zz.p[c] = zp_out[c];
  }
  const size_t smem = res_smem(a, false);
  dim3 grid(bpc, n_cells);
  KVC_DISPATCH_DTYPE(dtype, T, {
    cudaFuncSetAttribute(residual_stats_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    residual_stats_kernel<T><<<grid, NT, smem, st>>>(a);
  });
  if ((rc = check_launch("residual_stats_kernel"))) return rc;
  stats_finalize_kernel<<<n_cells, NT, 0, st>>>(a.partial, n_cells, bpc, d, bits, a.symmetric,
                                                scale_mode, stat_dtype, sc, zz);
  return check_launch("stats_finalize_kernel");
}

extern "C" int kvc_residual_quant(int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                                  int dtype, const void* const* core, const void* const* u_token,
                                  const void* const* u_feature, int rt, int rd, const float* proj,
                                  int bits, int symmetric, int scale_mode, int group_size,
                                  int stat_dtype, int arith_dtype, float* const* scale,
                                  int32_t* const* zp, uint8_t* const* codes, void* workspace,
                                  size_t ws_bytes, void* stream) {
  ResArgs a;
  int rc = fill_res_args(a, n_cells, x, m, t, d, dtype, core, u_token, u_feature, rt, rd, proj, bits,
                         symmetric, scale_mode, stat_dtype);
  if (rc) return rc;
  if (scale_mode == KVC_SCALE_GROUP && (group_size <= 0 || d % group_size != 0))
    return fail(KVC_ERR_SHAPE, "kvc_residual_quant: d must be divisible by group_size");
  if (!dtype_ok(arith_dtype)) return fail(KVC_ERR_DTYPE, "kvc_residual_quant: bad arith dtype");
  if (g_policy != 1 && scale_mode != KVC_SCALE_GROUP && (bits == 2 || bits == 4 || bits == 8) &&
      tc_residual_eligible(dtype, d, rd, proj, scale_mode) &&
      (rd <= 4 || tc_quant_fm_eligible(d, bits, scale_mode, arith_dtype)) &&
      all_aligned(n_cells, x) && all_aligned(n_cells, codes) && workspace &&
      ws_bytes >= tc_residual_workspace(n_cells, m * t, d, rd)) {
    return tc_residual_launch(1, n_cells, x, m, t, d, dtype, core, u_token, u_feature, rt, rd, proj, bits, symmetric,
                              scale_mode, stat_dtype, arith_dtype, scale, zp, codes, workspace, ws_bytes,
                              static_cast<cudaStream_t>(stream));
  }
  a.group_size = group_size;
  a.arith_dtype = arith_dtype;
  a.code_bytes = (d * bits + 7) / 8;
  for (int c = 0; c < n_cells; ++c) {
    if (!scale[c] || !zp[c] || !codes[c]) return fail(KVC_ERR_ARG, "kvc_residual_quant: NULL output");
    a.scale.p[c] = scale[c];
    a.zp.p[c] = zp[c];
    a.codes.p[c] = codes[c];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rt >= ROWTERM_RT && workspace && ws_bytes >= rowterm_bytes(n_cells, a.rows, rd)) {
    float* rows_tmp = static_cast<float*>(workspace);
    if ((rc = simt_row_terms(core, u_token, n_cells, dtype, m, t, rt, rd, rowterm_stride(rd), rows_tmp, st)))
      return rc;
    a.rowterm = rows_tmp;
    a.rt_stride = rowterm_stride(rd);
  }
  const size_t smem = res_smem(a, true);
  dim3 grid(blocks_per_cell(a.rows, n_cells), n_cells);
  KVC_DISPATCH_DTYPE(dtype, T, {
    cudaFuncSetAttribute(residual_quant_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    residual_quant_kernel<T><<<grid, NT, smem, st>>>(a);
  });
  return check_launch("residual_quant_kernel");
}

extern "C" int kvc_decompress(int n_cells, const uint8_t* const* codes, const float* const* scale,
                              const int32_t* const* zp, int bits, int symmetric, int scale_mode,
                              int group_size, const void* const* core, const void* const* u_token,
                              const void* const* u_feature, int factor_dtype, int64_t m, int64_t t,
                              int d, int rt, int rd, const float* proj, int64_t t0, int64_t t1,
                              int out_dtype, void* const* out, void* workspace, size_t ws_bytes,
                              void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_decompress: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || d > MAXD) return fail(KVC_ERR_SHAPE, "kvc_decompress: bad shape");
  if (t0 < 0 || t1 > t || t0 >= t1) return fail(KVC_ERR_SHAPE, "kvc_decompress: bad token range");
  if (bits != 0 && bits != 2 && bits != 4 && bits != 8) return fail(KVC_ERR_ARG, "kvc_decompress: bad bits");
  if (rt < 0 || rd < 0 || (rt == 0) != (rd == 0) || rd > d) return fail(KVC_ERR_SHAPE, "kvc_decompress: bad ranks");
  if (!dtype_ok(out_dtype) || (rt > 0 && !dtype_ok(factor_dtype)))
    return fail(KVC_ERR_DTYPE, "kvc_decompress: bad dtype");
  if (bits > 0 && scale_mode == KVC_SCALE_GROUP && (group_size <= 0 || d % group_size != 0))
    return fail(KVC_ERR_SHAPE, "kvc_decompress: d must be divisible by group_size");
  for (int c = 0; c < n_cells; ++c) {
    if (!out[c]) return fail(KVC_ERR_ARG, "kvc_decompress: NULL out");
    if (bits > 0 && (!codes[c] || !scale[c] || !zp[c])) return fail(KVC_ERR_ARG, "kvc_decompress: NULL codes");
    if (rt > 0 && (!core[c] || !u_token[c] || !u_feature[c]))
      return fail(KVC_ERR_ARG, "kvc_decompress: NULL factor");
  }
  if (g_policy != 1 && tc_decompress_eligible(out_dtype, d, rd, bits, symmetric, scale_mode, proj) &&
      all_aligned(n_cells, codes) && all_aligned(n_cells, out) && workspace &&
      ws_bytes >= tc_decompress_workspace(n_cells, m * t, d, rd)) {
    return tc_decompress_launch(n_cells, codes, scale, bits, core, u_token, u_feature, factor_dtype, m, t, d, rt,
                                rd, proj, t0, t1, out_dtype, out, workspace, ws_bytes,
                                static_cast<cudaStream_t>(stream));
  }
  DecArgs a;
  memset(&a, 0, sizeof(a));
  for (int c = 0; c < n_cells; ++c) {
    if (!out[c]) return fail(KVC_ERR_ARG, "kvc_decompress: NULL out");
    a.out.p[c] = out[c];
    if (bits > 0) {
      if (!codes[c] || !scale[c] || !zp[c]) return fail(KVC_ERR_ARG, "kvc_decompress: NULL codes");
      a.codes.p[c] = codes[c];
      a.scale.p[c] = scale[c];
      a.zp.p[c] = zp[c];
    }
    if (rt > 0) {
      if (!core[c] || !u_token[c] || !u_feature[c]) return fail(KVC_ERR_ARG, "kvc_decompress: NULL factor");
      a.core.p[c] = core[c];
      a.ut.p[c] = u_token[c];
      a.ud.p[c] = u_feature[c];
    }
  }
  a.bits = bits;
  a.symmetric = symmetric ? 1 : 0;
  a.scale_mode = scale_mode;
  a.group_size = group_size;
  a.factor_dtype = factor_dtype;
  a.out_dtype = out_dtype;
  a.m = m;
  a.t = t;
  a.t0 = t0;
  a.t1 = t1;
  a.d = d;
  a.rt = rt;
  a.rd = rd;
  a.code_bytes = bits > 0 ? (d * bits + 7) / 8 : 0;
  a.proj = bits > 0 ? proj : nullptr;
  a.pi_in_smem = (a.proj && d <= 128) ? 1 : 0;
  const size_t smem = ((a.pi_in_smem ? (size_t)d * d : 0) + (size_t)ROWS * d +
                       (size_t)ROWS * (rd > 0 ? rd : 1)) * sizeof(float);
  const int64_t rows = m * (t1 - t0);
  dim3 grid(blocks_per_cell(rows, n_cells), n_cells);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KVC_DISPATCH_DTYPE(out_dtype, T, {
    cudaFuncSetAttribute(decompress_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    decompress_kernel<T><<<grid, NT, smem, st>>>(a);
  });
  return check_launch("decompress_kernel");
}

// ---------------------------------------------------------------------------
// Decode plans (token-range streams).  A plan is host bytes owned by the
// caller: a magic word, then the TcDecodePlan (copied through an aligned
// local, since the caller's buffer need not be 64-byte aligned).

namespace {
constexpr uint64_t kPlanMagic = 0x6b76635f706c616eull;  // "kvc_plan"
constexpr size_t kPlanHeader = 64;                      // keeps the plan body 64-byte aligned in place
}  // namespace

extern "C" size_t kvc_decode_plan_bytes(void) { return kPlanHeader + sizeof(TcDecodePlan); }

extern "C" int kvc_decode_plan_init(void* plan, size_t plan_bytes, int n_cells, const uint8_t* const* codes,
                                    const float* const* scale, const int32_t* const* zp, int bits, int symmetric,
                                    int scale_mode, int group_size, const void* const* core,
                                    const void* const* u_token, const void* const* u_feature, int factor_dtype,
                                    int64_t m, int64_t t, int d, int rt, int rd, const float* proj, int out_dtype,
                                    void* workspace, size_t ws_bytes, void* stream) {
  if (!plan || plan_bytes < kvc_decode_plan_bytes()) return fail(KVC_ERR_ARG, "kvc_decode_plan_init: plan buffer too small");
  memset(plan, 0, kvc_decode_plan_bytes());
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_decode_plan_init: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || d > MAXD) return fail(KVC_ERR_SHAPE, "kvc_decode_plan_init: bad shape");
  if (bits != 0 && bits != 2 && bits != 4 && bits != 8) return fail(KVC_ERR_ARG, "kvc_decode_plan_init: bad bits");
  if (rt < 0 || rd < 0 || (rt == 0) != (rd == 0) || rd > d)
    return fail(KVC_ERR_SHAPE, "kvc_decode_plan_init: bad ranks");
  if (!dtype_ok(out_dtype) || (rt > 0 && !dtype_ok(factor_dtype)))
    return fail(KVC_ERR_DTYPE, "kvc_decode_plan_init: bad dtype");
  for (int c = 0; c < n_cells; ++c) {
    if (bits > 0 && (!codes[c] || !scale[c] || !zp[c])) return fail(KVC_ERR_ARG, "kvc_decode_plan_init: NULL codes");
    if (rt > 0 && (!core[c] || !u_token[c] || !u_feature[c]))
      return fail(KVC_ERR_ARG, "kvc_decode_plan_init: NULL factor");
  }
  (void)group_size;
  if (!(g_policy != 1 && tc_decompress_eligible(out_dtype, d, rd, bits, symmetric, scale_mode, proj) &&
        all_aligned(n_cells, codes)))
    return fail(KVC_ERR_UNSUPPORTED,
                "kvc_decode_plan_init: no tensor-core plan for this layout (decode with kvc_decompress)");
  TcDecodePlan local;
  const int rc = tc_decode_plan_init(&local, n_cells, codes, scale, bits, core, u_token, u_feature, factor_dtype, m,
                                     t, d, rt, rd, proj, out_dtype, workspace, ws_bytes,
                                     static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  memcpy(static_cast<uint8_t*>(plan) + kPlanHeader, &local, sizeof(local));
  memcpy(plan, &kPlanMagic, sizeof(kPlanMagic));
  return KVC_OK;
}

extern "C" int kvc_decode_plan_run(const void* plan, size_t plan_bytes, int64_t t0, int64_t t1, void* const* out,
                                   void* stream) {
  uint64_t magic = 0;
  if (!plan || plan_bytes < kvc_decode_plan_bytes()) return fail(KVC_ERR_ARG, "kvc_decode_plan_run: plan buffer too small");
  memcpy(&magic, plan, sizeof(magic));
  if (magic != kPlanMagic) return fail(KVC_ERR_ARG, "kvc_decode_plan_run: not an initialised plan");
  TcDecodePlan local;
  memcpy(&local, static_cast<const uint8_t*>(plan) + kPlanHeader, sizeof(local));
  return tc_decode_plan_run(&local, t0, t1, out, static_cast<cudaStream_t>(stream));
}
