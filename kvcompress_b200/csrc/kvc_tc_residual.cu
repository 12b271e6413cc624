// Tensor-core (tcgen05 / TMEM) kernels for the residual encode and the
// fused decode, bf16 caches with head_dim 64 or 128.
//
// Both are persistent, warp-specialised kernels (288 threads, one CTA per
// SM) over 128-row tiles:
//   warps 0-3  producers: build the bf16 A operand of a tile in shared memory
//              (K-major SWIZZLE_128B, two stages)
//   warp 4     one thread issues tcgen05.mma into one of two TMEM
//              accumulators (128 lanes x d fp32 columns each)
//   warps 5-8  epilogue: tcgen05.ld of the accumulator rows, then the
//              per-tile output
//
// Residual encode (kvcompress/compressor/residual.py:201-239):
//   A = R = x - Tucker(x) rounded to bf16 (exact operand), B = the JL matrix
//   Pi split into three bf16 terms (hi + mid + lo = Pi to fp32 precision),
//   so D = R Pi^T to fp32 accuracy.  Mode STATS reduces per-column min / max
//   (butterfly transpose-reduce, order-independent atomics on ordered ints);
//   mode QUANT divides by the scale, rounds half to even, clamps and packs.
// Decode (kvcompress/compressor/jolt.py:424-463, residual.py:242-288):
//   A = the integer codes (exact in bf16), B = diag(scale) Pi split in two
//   bf16 terms; the epilogue adds the fp32 Tucker term and writes the tile.
//
// Tiles are spread over CTAs by a static contiguous partition of the global
// (cell, tile) list (encode) or per cell (decode: B depends on the cell's
// scales).  Every mbarrier wait is bounded (kvc_tc.cuh).
#include <algorithm>
#include <type_traits>

#include "kvc_common.cuh"
#include "kvc_quant.cuh"
#include "kvc_tc.cuh"

namespace kvc {
namespace {

using namespace tc;

constexpr int TILE_M = 128;
constexpr int NTHREADS = 416;  // 4 producer warps, 1 MMA warp, 8 epilogue warps
constexpr int MMA_WARP = 4;
constexpr int NEPI = 256;      // epilogue threads: 2 warps per TMEM lane group
constexpr int RD_MAX = 16;
constexpr int NSTAGE = 3;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// STAGE_EXTRA: per-stage staging bytes beside the A tile (decode: the codes).
template <int D, int NTERM, int STAGE_EXTRA = 0>
struct Layout {
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_BYTES = NTERM * B_TERM;
  static constexpr uint32_t A_BYTES = TILE_M * D * 2;
  static constexpr uint32_t OFF_B = 0;
  static constexpr uint32_t OFF_A = B_BYTES;
  static constexpr uint32_t OFF_X = OFF_A + NSTAGE * A_BYTES;          // staging
  static constexpr uint32_t OFF_UD = OFF_X + NSTAGE * STAGE_EXTRA;
  static constexpr uint32_t OFF_SC = OFF_UD + D * RD_MAX * 4;          // 8 epilogue warps x (scales, zps)
  static constexpr uint32_t OFF_BAR = OFF_SC + 8 * D * 8;
  static constexpr uint32_t NBAR = 2 * NSTAGE + 4;                     // full, empty, acc full, acc empty
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;                // + alignment slack
};

enum { MODE_STATS = 0, MODE_QUANT = 1 };

struct TcResArgs {
  CellPtrs x, core, ut, ud, scale, zp;
  CellPtrsMut codes;
  int n_cells;
  int64_t m, t, rows, tiles_per_cell, tiles_per_cta, total_tiles;
  int rt, rd;
  const void* bops;    // NTERM swizzled B tiles (global)
  int32_t* minmax;     // STATS: [cell][2][d] ordered ints (min, max)
  const float* tmp;    // [cell][row][rd]: sum_a core[h][a][r] u_token[t][a], rounded to the cell dtype
  const float* ud32;   // [cell][d][rd]: u_feature as float
  int bits, symmetric, scale_mode, arith_dtype, code_bytes;
};

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 out;
  uint32_t* w = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    T lo = Elt<T>::from(v[2 * i]), hi = Elt<T>::from(v[2 * i + 1]);
    w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
  }
  return out;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&v)[8]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = Elt<T>::to_f32(e[i]);
}

// ------------------------------------------------------------------------
// residual encode: STATS / QUANT
// ------------------------------------------------------------------------
template <typename T, int D, int NTERM, int MODE, int RDM>
__global__ void __launch_bounds__(NTHREADS, 1) tc_residual_kernel(TcResArgs A) {
  using L = Layout<D, NTERM, TILE_M * RDM * 4>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t tile_begin = (int64_t)blockIdx.x * A.tiles_per_cta;
  const int64_t tile_end = tile_begin + A.tiles_per_cta < A.total_tiles ? tile_begin + A.tiles_per_cta
                                                                       : A.total_tiles;
  const int n_my = (int)(tile_end > tile_begin ? tile_end - tile_begin : 0);

  // ---- set-up: B operand, barriers, TMEM ----
  {
    const uint4* src = static_cast<const uint4*>(A.bops);
    uint4* dst = reinterpret_cast<uint4*>(smem + L::OFF_B);
    for (int i = threadIdx.x; i < (int)(L::B_BYTES / 16); i += NTHREADS) dst[i] = src[i];
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 128);  // producer threads
      mbar_init(&empty[i], 1);   // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);     // tcgen05.commit
      mbar_init(&acce[i], NEPI);  // epilogue threads
    }
    mbar_fence_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tm_holder, 2 * D);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tm_holder;

  if (warp < 4) {
    // ---------------- producers: one row per thread ----------------
    // cp.async the row of x into the swizzled A stage (and its Tucker row
    // term into a private slot), then R = x - Tucker in place.
    constexpr int CH = D / 8;
    const int ptid = threadIdx.x;  // row within the tile
    float* tslot = reinterpret_cast<float*>(smem + L::OFF_X);  // [stage][128][RDM]
    bool ok = true;
    auto issue = [&](int j) {
      const int64_t g = tile_begin + j;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      const int st = j % NSTAGE;
      if (!mbar_wait(&empty[st], (uint32_t)((j / NSTAGE) & 1) ^ 1u, 0x101)) return false;
      if (row < A.rows) {
        const T* x = static_cast<const T*>(A.x.p[cell]) + row * D;
        const uint32_t a_s = sbase + L::OFF_A + st * L::A_BYTES;
#pragma unroll
        for (int c = 0; c < CH; ++c) cp_async16(a_s + sw128_off(ptid, c * 8, TILE_M), x + c * 8);
        if (A.rt > 0) {
          const float* tp = A.tmp + ((int64_t)cell * A.rows + row) * A.rd;
          const uint32_t ts = smem_u32(tslot + (st * TILE_M + ptid) * RDM);
          for (int r = 0; r < A.rd; ++r)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ts + r * 4), "l"(tp + r) : "memory");
        }
      }
      return true;
    };
    for (int j = 0; j < NSTAGE - 1; ++j) {
      if (ok && j < n_my) ok = issue(j);
      cp_async_commit();
    }
    for (int it = 0; it < n_my; ++it) {
      const int jn = it + NSTAGE - 1;
      if (ok && jn < n_my) ok = issue(jn);
      cp_async_commit();
      cp_async_wait<NSTAGE - 1>();
      if (!ok) continue;  // keep the loop shape; the MMA side times out too
      const int st = it % NSTAGE;
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      uint8_t* As = smem + L::OFF_A + st * L::A_BYTES;
      if (row >= A.rows) {
#pragma unroll
        for (int c = 0; c < CH; ++c)
          *reinterpret_cast<uint4*>(As + sw128_off(ptid, c * 8, TILE_M)) = make_uint4(0, 0, 0, 0);
      } else if (A.rt > 0) {
        float tv[RDM];
#pragma unroll
        for (int r = 0; r < RDM; ++r) tv[r] = r < A.rd ? tslot[(st * TILE_M + ptid) * RDM + r] : 0.f;
        const float4* ud = reinterpret_cast<const float4*>(A.ud32 + (int64_t)cell * D * RDM);
#pragma unroll 4
        for (int c = 0; c < CH; ++c) {
          uint4* slot = reinterpret_cast<uint4*>(As + sw128_off(ptid, c * 8, TILE_M));
          float xv[8];
          unpack8<T>(*slot, xv);
          float u[8 * RDM];
#pragma unroll
          for (int q = 0; q < 2 * RDM; ++q) {
            const float4 f = __ldg(ud + c * 2 * RDM + q);
            u[4 * q] = f.x;
            u[4 * q + 1] = f.y;
            u[4 * q + 2] = f.z;
            u[4 * q + 3] = f.w;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float rec = 0.f;
#pragma unroll
            for (int r = 0; r < RDM; ++r) rec = fmaf(tv[r], u[e * RDM + r], rec);
            xv[e] = Elt<T>::round(xv[e] - Elt<T>::round(rec));
          }
          *slot = pack8<T>(xv);
        }
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
    cp_async_wait<0>();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(TILE_M, D, std::is_same<T, __nv_bfloat16>::value);
      int it = 0;
      for (; it < n_my; ++it) {
        const int st = it % NSTAGE, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NSTAGE) & 1), 0x201)) break;
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x202)) break;
        tc_fence_after();
        const uint32_t a_base = sbase + L::OFF_A + st * L::A_BYTES;
        const uint32_t d_tmem = tmem + (uint32_t)(ac * D);
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t ka = (uint32_t)((ks >> 2) * (TILE_M * 128) + (ks & 3) * 32);
            const uint32_t kb = (uint32_t)((ks >> 2) * (D * 128) + (ks & 3) * 32);
            umma_f16(d_tmem, desc_sw128(a_base + ka), desc_sw128(sbase + L::OFF_B + term * L::B_TERM + kb),
                     idesc, (term | ks) ? 1u : 0u);
          }
        }
        umma_commit(&empty[st]);
        umma_commit(&accf[ac]);
      }
      // do not leave while MMAs that write TMEM are still in flight
      if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x203);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: 2 warps per lane group, one column half each ----------------
    const int e = warp - 5;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;  // 32-column chunks per warp
    float* sc_s = reinterpret_cast<float*>(smem + L::OFF_SC) + e * 2 * D;
    int32_t* zp_s = reinterpret_cast<int32_t*>(sc_s + D);
    float rmax[NCH], rmin[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      rmax[c] = -__int_as_float(0x7f800000);
      rmin[c] = __int_as_float(0x7f800000);
    }
    int qmin, qmax;
    qrange(A.bits > 0 ? A.bits : 8, A.symmetric, qmin, qmax);
    const int offset = A.symmetric ? (1 << (A.bits - 1)) : 0;
    int cur_cell = -1;
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      if (cell != cur_cell) {
        if (MODE == MODE_STATS && cur_cell >= 0) {
          int32_t* mm = A.minmax + (int64_t)cur_cell * 2 * D;
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            const int col = (half * NCH + c) * 32 + lane;
            atomicMin(&mm[col], ordered_bits(rmin[c]));
            atomicMax(&mm[D + col], ordered_bits(rmax[c]));
            rmax[c] = -__int_as_float(0x7f800000);
            rmin[c] = __int_as_float(0x7f800000);
          }
        }
        if (MODE == MODE_QUANT) {
          __syncwarp();
          const float* sc = static_cast<const float*>(A.scale.p[cell]);
          const int32_t* zz = static_cast<const int32_t*>(A.zp.p[cell]);
          for (int j = lane; j < D; j += 32) {
            const int jj = A.scale_mode == KVC_SCALE_CHANNEL ? j : 0;
            sc_s[j] = sc[jj];
            zp_s[j] = zz[jj];
          }
          __syncwarp();
        }
        cur_cell = cell;
      }
      const int ac = it & 1;
      if (!mbar_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x301)) break;
      tc_fence_after();
      const int64_t row = tile * TILE_M + rloc;
      const bool valid = row < A.rows;
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        if (MODE == MODE_STATS) {
          float w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            w[j] = valid ? v[j] : __int_as_float(0x7f800000);
            v[j] = valid ? v[j] : -__int_as_float(0x7f800000);
          }
          rmax[cc] = fmaxf(rmax[cc], transpose_reduce32<true>(v));
          rmin[cc] = fminf(rmin[cc], transpose_reduce32<false>(w));
        } else if (valid) {
          const int ad = A.scale_mode == KVC_SCALE_TENSOR ? A.arith_dtype : KVC_F32;
          uint32_t u[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int q = quantize_one(v[j], sc_s[c * 32 + j], zp_s[c * 32 + j], qmin, qmax, ad);
            u[j] = (uint32_t)((q + offset) & 0xFF);
          }
          uint8_t* dst = static_cast<uint8_t*>(A.codes.p[cell]) + row * A.code_bytes;
          if (A.bits == 8) {
            uint4 o0, o1;
            o0.x = u[0] | u[1] << 8 | u[2] << 16 | u[3] << 24;
            o0.y = u[4] | u[5] << 8 | u[6] << 16 | u[7] << 24;
            o0.z = u[8] | u[9] << 8 | u[10] << 16 | u[11] << 24;
            o0.w = u[12] | u[13] << 8 | u[14] << 16 | u[15] << 24;
            o1.x = u[16] | u[17] << 8 | u[18] << 16 | u[19] << 24;
            o1.y = u[20] | u[21] << 8 | u[22] << 16 | u[23] << 24;
            o1.z = u[24] | u[25] << 8 | u[26] << 16 | u[27] << 24;
            o1.w = u[28] | u[29] << 8 | u[30] << 16 | u[31] << 24;
            reinterpret_cast<uint4*>(dst + c * 32)[0] = o0;
            reinterpret_cast<uint4*>(dst + c * 32)[1] = o1;
          } else if (A.bits == 4) {
            uint32_t w4[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              uint32_t acc = 0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t byte = ((u[8 * b + 2 * i] & 0xF) << 4) | (u[8 * b + 2 * i + 1] & 0xF);
                acc |= byte << (8 * i);
              }
              w4[b] = acc;
            }
            *reinterpret_cast<uint4*>(dst + c * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          } else {
            uint32_t w2[2];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              uint32_t acc = 0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int k = 16 * b + 4 * i;
                const uint32_t byte = ((u[k] & 3) << 6) | ((u[k + 1] & 3) << 4) | ((u[k + 2] & 3) << 2) |
                                      (u[k + 3] & 3);
                acc |= byte << (8 * i);
              }
              w2[b] = acc;
            }
            *reinterpret_cast<uint2*>(dst + c * 8) = make_uint2(w2[0], w2[1]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (MODE == MODE_STATS && cur_cell >= 0) {
      int32_t* mm = A.minmax + (int64_t)cur_cell * 2 * D;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int col = (half * NCH + c) * 32 + lane;
        atomicMin(&mm[col], ordered_bits(rmin[c]));
        atomicMax(&mm[D + col], ordered_bits(rmax[c]));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * D);
  }
}

// Per-row Tucker term for the tensor-core kernels:
//   tmp[cell][row][r] = sum_a core[h][a][r] * u_token[t][a]   (rows of [t0, t1))
// rounded to `round_dt` (the compress side rounds it to the cell dtype like
// the reference's einsum intermediate; the decode side keeps fp32), and
// u_feature as float padded to rdm columns.
__global__ void tucker_rows_kernel(CellPtrs core, CellPtrs ut, CellPtrs ud, int fdt, int round_dt_, int64_t m,
                                   int64_t t0, int64_t tl, int rt, int rd, int d, int rdm, float* tmp,
                                   float* ud32) {
  const int cell = blockIdx.y;
  const int64_t rows = m * tl;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows * rd;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / rd;
    const int r = (int)(idx % rd);
    const int64_t h = row / tl, t = t0 + row % tl;
    float acc = 0.f;
    for (int a = 0; a < rt; ++a)
      acc = fmaf(load_dt(core.p[cell], (h * rt + a) * rd + r, fdt), load_dt(ut.p[cell], t * rt + a, fdt), acc);
    tmp[(int64_t)cell * rows * rd + idx] = round_dt(acc, round_dt_);
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < d * rdm; i += blockDim.x) {
      const int j = i / rdm, r = i % rdm;
      ud32[(int64_t)cell * d * rdm + i] = r < rd ? load_dt(ud.p[cell], (int64_t)j * rd + r, fdt) : 0.f;
    }
}

static int rdm_of(int rd) { return rd <= 1 ? 1 : (rd <= 4 ? 4 : 16); }

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// min / max arrays to their identities (ordered ints of +inf / -inf).
__global__ void minmax_init_kernel(int32_t* mm, int n_cells, int d) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_cells * 2 * d) return;
  const bool is_max = (i / d) & 1;
  mm[i] = is_max ? (int32_t)0x807FFFFF : (int32_t)0x7F800000;
}

__global__ void minmax_finalize_kernel(const int32_t* __restrict__ mm, int n_cells, int d, int bits,
                                       int symmetric, int scale_mode, int stat_dt, CellPtrsMut scale,
                                       CellPtrsMut zp) {
  const int cell = blockIdx.x;
  const int32_t* base = mm + (int64_t)cell * 2 * d;
  if (scale_mode == KVC_SCALE_CHANNEL) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float s;
      int32_t z;
      params_from_minmax(from_ordered_bits(base[j]), from_ordered_bits(base[d + j]), bits, symmetric, stat_dt, s, z);
      static_cast<float*>(scale.p[cell])[j] = s;
      static_cast<int32_t*>(zp.p[cell])[j] = z;
    }
  } else if (threadIdx.x == 0) {
    float a = __int_as_float(0x7f800000), b = -__int_as_float(0x7f800000);
    for (int j = 0; j < d; ++j) {
      a = fminf(a, from_ordered_bits(base[j]));
      b = fmaxf(b, from_ordered_bits(base[d + j]));
    }
    float s;
    int32_t z;
    params_from_minmax(a, b, bits, symmetric, stat_dt, s, z);
    static_cast<float*>(scale.p[cell])[0] = s;
    static_cast<int32_t*>(zp.p[cell])[0] = z;
  }
}

// Pi split into NTERM terms of T, laid out as swizzled K-major B tiles:
// B[n][k] = Pi[n][k] (D = R Pi^T).
template <typename T>
__global__ void prep_rotation_kernel(const float* __restrict__ proj, int d, int nterm, uint8_t* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= d * d) return;
  const int n = e / d, k = e % d;
  float rest = proj[e];
  for (int term = 0; term < nterm; ++term) {
    const T v = Elt<T>::from(rest);
    rest -= Elt<T>::to_f32(v);
    *reinterpret_cast<T*>(out + (size_t)term * d * d * 2 + sw128_off(n, k, d)) = v;
  }
}

// ------------------------------------------------------------------------
// decode
// ------------------------------------------------------------------------
struct TcDecArgs {
  CellPtrs codes, core, ut, ud;
  CellPtrsMut out;
  int64_t m, t, t0, t1, rows, tiles_per_cell;
  int tiles_per_cta;
  int rt, rd, bits, code_bytes, factor_dtype;
  const uint8_t* bops;  // per cell: 2 swizzled B tiles of diag(scale) Pi
  const float* tmp;     // [cell][out row][rd] fp32 Tucker row term
  const float* ud32;    // [cell][d][rdm]
};

template <typename TOut, int D, int RDM, int BITS>
__global__ void __launch_bounds__(NTHREADS, 1) tc_decompress_kernel(TcDecArgs A) {
  constexpr int CB = D * BITS / 8;  // code bytes per row
  using L = Layout<D, 2, TILE_M * CB>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  float* ud_s = reinterpret_cast<float*>(smem + L::OFF_UD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cell = blockIdx.y;
  const int64_t tl = A.t1 - A.t0;
  const int64_t tile_begin = (int64_t)blockIdx.x * A.tiles_per_cta;
  const int64_t tile_end = tile_begin + A.tiles_per_cta < A.tiles_per_cell ? tile_begin + A.tiles_per_cta
                                                                         : A.tiles_per_cell;
  const int n_my = (int)(tile_end > tile_begin ? tile_end - tile_begin : 0);
  {
    const uint4* src = reinterpret_cast<const uint4*>(A.bops + (size_t)cell * L::B_BYTES);
    uint4* dst = reinterpret_cast<uint4*>(smem + L::OFF_B);
    for (int i = threadIdx.x; i < (int)(L::B_BYTES / 16); i += NTHREADS) dst[i] = src[i];
  }
  if (A.rt > 0)
    for (int i = threadIdx.x; i < D * RDM; i += NTHREADS) ud_s[i] = A.ud32[(int64_t)cell * D * RDM + i];
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], NEPI);
    }
    mbar_fence_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tm_holder, 2 * D);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tm_holder;

  if (warp < 4) {
    // codes -> (cp.async) staging -> exact integers in bf16 -> swizzled A tile
    const uint8_t* codes = static_cast<const uint8_t*>(A.codes.p[cell]);
    constexpr int LPR = CB / 16;      // lanes per row, 16 code bytes each
    constexpr int RPI = 32 / LPR;
    constexpr int NIT = 32 / RPI;
    constexpr int PER = 8 / BITS;
    constexpr int VALS = 16 * PER;    // values per lane
    constexpr int OFFSET = 1 << (BITS - 1);
    constexpr int MASK = (1 << BITS) - 1;
    const int pos = lane % LPR, sub = lane / LPR;
    bool ok = true;
    auto issue = [&](int j) {
      const int64_t tile = tile_begin + j;
      const int st = j % NSTAGE;
      if (!mbar_wait(&empty[st], (uint32_t)((j / NSTAGE) & 1) ^ 1u, 0x111)) return false;
      const uint32_t c_s = sbase + L::OFF_X + st * (TILE_M * CB);
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int rloc = warp * 32 + i * RPI + sub;
        const int64_t orow = tile * TILE_M + rloc;
        if (orow < A.rows) {
          const int64_t h = orow / tl, t = A.t0 + orow % tl;
          cp_async16(c_s + rloc * CB + pos * 16, codes + (h * A.t + t) * CB + pos * 16);
        }
      }
      return true;
    };
    for (int j = 0; j < NSTAGE - 1; ++j) {
      if (ok && j < n_my) ok = issue(j);
      cp_async_commit();
    }
    for (int it = 0; it < n_my && ok; ++it) {
      const int jn = it + NSTAGE - 1;
      if (jn < n_my) ok = issue(jn);
      cp_async_commit();
      if (!ok) break;
      cp_async_wait<NSTAGE - 1>();
      const int st = it % NSTAGE;
      const uint8_t* Cs = smem + L::OFF_X + st * (TILE_M * CB);
      uint8_t* As = smem + L::OFF_A + st * L::A_BYTES;
      const int64_t tile = tile_begin + it;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int rloc = warp * 32 + i * RPI + sub;
        const bool valid = tile * TILE_M + rloc < A.rows;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (valid) raw = *reinterpret_cast<const uint4*>(Cs + rloc * CB + pos * 16);
        const uint32_t* words = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
        for (int cb = 0; cb < VALS / 8; ++cb) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int idx = cb * 8 + e;
            const int byte = idx / PER, sl = idx % PER;
            const uint32_t b = (words[byte >> 2] >> (8 * (byte & 3))) & 0xFFu;
            const int q = (int)((b >> (BITS * (PER - 1 - sl))) & MASK) - OFFSET;
            v[e] = valid ? (float)q : 0.f;
          }
          *reinterpret_cast<uint4*>(As + sw128_off(rloc, pos * VALS + cb * 8, TILE_M)) = pack8<__nv_bfloat16>(v);
        }
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
    cp_async_wait<0>();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(TILE_M, D, true);
      int it = 0;
      for (; it < n_my; ++it) {
        const int st = it % NSTAGE, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NSTAGE) & 1), 0x211)) break;
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x212)) break;
        tc_fence_after();
        const uint32_t a_base = sbase + L::OFF_A + st * L::A_BYTES;
        const uint32_t d_tmem = tmem + (uint32_t)(ac * D);
#pragma unroll
        for (int term = 0; term < 2; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t ka = (uint32_t)((ks >> 2) * (TILE_M * 128) + (ks & 3) * 32);
            const uint32_t kb = (uint32_t)((ks >> 2) * (D * 128) + (ks & 3) * 32);
            umma_f16(d_tmem, desc_sw128(a_base + ka), desc_sw128(sbase + L::OFF_B + term * L::B_TERM + kb),
                     idesc, (term | ks) ? 1u : 0u);
          }
        }
        umma_commit(&empty[st]);
        umma_commit(&accf[ac]);
      }
      if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x213);
    }
    __syncwarp();
  } else {
    const int e = warp - 5;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;
    TOut* out = static_cast<TOut*>(A.out.p[cell]);
    for (int it = 0; it < n_my; ++it) {
      const int ac = it & 1;
      const int64_t orow = (tile_begin + it) * TILE_M + rloc;
      const bool valid = orow < A.rows;
      float tmp[RDM];  // loaded before the wait so the latency overlaps it
#pragma unroll
      for (int r = 0; r < RDM; ++r)
        tmp[r] = (valid && A.rt > 0 && r < A.rd) ? __ldg(A.tmp + ((int64_t)cell * A.rows + orow) * A.rd + r) : 0.f;
      if (!mbar_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x311)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        if (valid) {
          float o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (A.rt > 0) {
              float rec = 0.f;
#pragma unroll
              for (int r = 0; r < RDM; ++r)
                rec = fmaf(tmp[r], ud_s[(c * 32 + j) * RDM + r], rec);
              o[j] = __fadd_rn(rec, v[j]);
            } else {
              o[j] = v[j];
            }
          }
          TOut* dst = out + orow * D + c * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) w[k] = o[q * 8 + k];
            reinterpret_cast<uint4*>(dst)[q] = pack8<TOut>(w);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * D);
  }
}

// B[n][k] = scale[k] * Pi[k][n] split in two bf16 terms, per cell.
__global__ void prep_decode_kernel(const float* __restrict__ proj, CellPtrs scale, int d, uint8_t* out) {
  const int cell = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= d * d) return;
  const int n = e / d, k = e % d;
  const float sk = static_cast<const float*>(scale.p[cell])[k];
  float rest = __fmul_rn(sk, proj[(int64_t)k * d + n]);
  uint8_t* base = out + (size_t)cell * 2 * d * d * 2;
  for (int term = 0; term < 2; ++term) {
    const __nv_bfloat16 v = __float2bfloat16_rn(rest);
    rest -= __bfloat162float(v);
    *reinterpret_cast<__nv_bfloat16*>(base + (size_t)term * d * d * 2 + sw128_off(n, k, d)) = v;
  }
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  return KVC_OK;
}

}  // namespace

// ------------------------------- launchers --------------------------------

bool tc_residual_eligible(int dtype, int d, int rd, const float* proj, int scale_mode) {
  return dtype == KVC_BF16 && (d == 64 || d == 128) && rd <= 4 && proj != nullptr &&
         (scale_mode == KVC_SCALE_CHANNEL || scale_mode == KVC_SCALE_TENSOR);
}

size_t tc_residual_workspace(int n_cells, int64_t rows, int d, int rd) {
  return align256((size_t)3 * d * d * 2) + align256((size_t)n_cells * 2 * d * sizeof(int32_t)) +
         align256((size_t)n_cells * d * rdm_of(rd) * 4) + align256((size_t)n_cells * rows * rd * 4);
}

static int prep_rotation(const float* proj, int d, uint8_t* bops, cudaStream_t st) {
  prep_rotation_kernel<__nv_bfloat16><<<(d * d + 255) / 256, 256, 0, st>>>(proj, d, 3, bops);
  return check_launch("prep_rotation_kernel");
}

static void plan_global(TcResArgs& a, int n_cells, int64_t rows) {
  a.n_cells = n_cells;
  a.tiles_per_cell = ceil_div(rows, TILE_M);
  a.total_tiles = a.tiles_per_cell * n_cells;
  const int64_t ctas = std::min<int64_t>(a.total_tiles, num_sms());
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
}

int tc_residual_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                       const void* const* core, const void* const* u_token, const void* const* u_feature,
                       int rt, int rd, const float* proj, int bits, int symmetric, int scale_mode,
                       int stat_dtype, int arith_dtype, float* const* scale, int32_t* const* zp,
                       uint8_t* const* codes, void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (!workspace || ws_bytes < tc_residual_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core residual: workspace too small");
  TcResArgs a;
  memset(&a, 0, sizeof(a));
  for (int c = 0; c < n_cells; ++c) {
    a.x.p[c] = x[c];
    if (rt > 0) {
      a.core.p[c] = core[c];
      a.ut.p[c] = u_token[c];
      a.ud.p[c] = u_feature[c];
    }
    if (scale) a.scale.p[c] = scale[c];
    if (zp) a.zp.p[c] = zp[c];
    if (codes) a.codes.p[c] = codes[c];
  }
  a.m = m;
  a.t = t;
  a.rows = m * t;
  a.rt = rt;
  a.rd = rd;
  a.bits = bits;
  a.symmetric = symmetric;
  a.scale_mode = scale_mode;
  a.arith_dtype = arith_dtype;
  a.code_bytes = (d * bits + 7) / 8;
  plan_global(a, n_cells, a.rows);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* bops = ws;
  size_t off = align256((size_t)3 * d * d * 2);
  int32_t* mm = reinterpret_cast<int32_t*>(ws + off);
  off += align256((size_t)n_cells * 2 * d * sizeof(int32_t));
  float* ud32 = reinterpret_cast<float*>(ws + off);
  off += align256((size_t)n_cells * d * rdm_of(rd) * 4);
  float* tmp = reinterpret_cast<float*>(ws + off);
  a.bops = bops;
  a.minmax = mm;
  a.tmp = tmp;
  a.ud32 = ud32;
  int rc = prep_rotation(proj, d, bops, st);
  if (rc) return rc;
  if (rt > 0) {
    CellPtrs cp, up, dp;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
      dp.p[c] = u_feature[c];
    }
    const int64_t rows = m * t;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows * rd, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(cp, up, dp, KVC_BF16, KVC_BF16, m, 0, t, rt, rd, d,
                                                              rdm_of(rd), tmp, ud32);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  if (mode == MODE_STATS) {
    minmax_init_kernel<<<(n_cells * 2 * d + 255) / 256, 256, 0, st>>>(mm, n_cells, d);
    if ((rc = check_launch("minmax_init_kernel"))) return rc;
  }
#define KVC_TC_RES(DD, MODEV, RR)                                                              \
  do {                                                                                         \
    auto kern = tc_residual_kernel<__nv_bfloat16, DD, 3, MODEV, RR>;                           \
    const size_t sm = Layout<DD, 3, TILE_M * RR * 4>::BYTES;                                   \
    if ((rc = set_smem(kern, sm))) return rc;                                                  \
    kern<<<grid, NTHREADS, sm, st>>>(a);                                                       \
  } while (0)
#define KVC_TC_RES_R(DD, MODEV)                       \
  do {                                                \
    if (rd <= 1) KVC_TC_RES(DD, MODEV, 1);            \
    else KVC_TC_RES(DD, MODEV, 4);                    \
  } while (0)
  if (mode == MODE_STATS) {
    if (d == 128) KVC_TC_RES_R(128, MODE_STATS);
    else KVC_TC_RES_R(64, MODE_STATS);
  } else {
    if (d == 128) KVC_TC_RES_R(128, MODE_QUANT);
    else KVC_TC_RES_R(64, MODE_QUANT);
  }
#undef KVC_TC_RES_R
#undef KVC_TC_RES
  if ((rc = check_launch("tc_residual_kernel"))) return rc;
  if (mode == MODE_STATS) {
    CellPtrsMut sc, zz;
    for (int c = 0; c < n_cells; ++c) {
      sc.p[c] = scale[c];
      zz.p[c] = zp[c];
    }
    minmax_finalize_kernel<<<n_cells, 128, 0, st>>>(mm, n_cells, d, bits, symmetric, scale_mode, stat_dtype, sc, zz);
    return check_launch("minmax_finalize_kernel");
  }
  return KVC_OK;
}

bool tc_decompress_eligible(int out_dtype, int d, int rd, int bits, int symmetric, int scale_mode,
                            const float* proj) {
  return out_dtype == KVC_BF16 && (d == 64 || d == 128) && rd <= RD_MAX && bits > 0 && symmetric &&
         scale_mode == KVC_SCALE_CHANNEL && proj != nullptr;
}

size_t tc_decompress_workspace(int n_cells, int64_t rows, int d, int rd) {
  return align256((size_t)n_cells * 2 * d * d * 2) + align256((size_t)n_cells * d * rdm_of(rd) * 4) +
         align256((size_t)n_cells * rows * rd * 4);
}

int tc_decompress_launch(int n_cells, const uint8_t* const* codes, const float* const* scale, int bits,
                         const void* const* core, const void* const* u_token, const void* const* u_feature,
                         int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd, const float* proj,
                         int64_t t0, int64_t t1, void* const* out, void* workspace, size_t ws_bytes,
                         cudaStream_t st) {
  if (!workspace || ws_bytes < tc_decompress_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core decompress: workspace too small");
  TcDecArgs a;
  memset(&a, 0, sizeof(a));
  CellPtrs sc;
  for (int c = 0; c < n_cells; ++c) {
    a.codes.p[c] = codes[c];
    sc.p[c] = scale[c];
    a.out.p[c] = out[c];
    if (rt > 0) {
      a.core.p[c] = core[c];
      a.ut.p[c] = u_token[c];
      a.ud.p[c] = u_feature[c];
    }
  }
  a.m = m;
  a.t = t;
  a.t0 = t0;
  a.t1 = t1;
  a.rows = m * (t1 - t0);
  a.tiles_per_cell = ceil_div(a.rows, TILE_M);
  const int64_t per_cell = std::max<int64_t>(1, num_sms() / n_cells);
  const int64_t ctas = std::min<int64_t>(a.tiles_per_cell, per_cell);
  a.tiles_per_cta = (int)ceil_div(a.tiles_per_cell, ctas);
  a.rt = rt;
  a.rd = rd;
  a.bits = bits;
  a.code_bytes = (d * bits + 7) / 8;
  a.factor_dtype = factor_dtype;
  uint8_t* bops = static_cast<uint8_t*>(workspace);
  size_t off = align256((size_t)n_cells * 2 * d * d * 2);
  float* ud32 = reinterpret_cast<float*>(bops + off);
  off += align256((size_t)n_cells * d * rdm_of(rd) * 4);
  float* tmp = reinterpret_cast<float*>(bops + off);
  a.bops = bops;
  a.tmp = tmp;
  a.ud32 = ud32;
  prep_decode_kernel<<<dim3((d * d + 255) / 256, n_cells), 256, 0, st>>>(proj, sc, d, bops);
  int rc = check_launch("prep_decode_kernel");
  if (rc) return rc;
  if (rt > 0) {
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(a.rows * rd, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(a.core, a.ut, a.ud, factor_dtype, KVC_F32, m, t0,
                                                              t1 - t0, rt, rd, d, rdm_of(rd), tmp, ud32);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.tiles_per_cell, a.tiles_per_cta), n_cells);
#define KVC_TC_DEC3(DD, RR, BB)                                             \
  do {                                                                      \
    auto kern = tc_decompress_kernel<__nv_bfloat16, DD, RR, BB>;            \
    using LL = Layout<DD, 2, TILE_M * DD * BB / 8>;                         \
    if ((rc = set_smem(kern, LL::BYTES))) return rc;                        \
    kern<<<grid, NTHREADS, LL::BYTES, st>>>(a);                             \
  } while (0)
#define KVC_TC_DEC(DD, RR)                            \
  do {                                                \
    if (bits == 8) KVC_TC_DEC3(DD, RR, 8);            \
    else if (bits == 4) KVC_TC_DEC3(DD, RR, 4);       \
    else KVC_TC_DEC3(DD, RR, 2);                      \
  } while (0)
  if (d == 128) {
    if (rd <= 1) KVC_TC_DEC(128, 1);
    else if (rd <= 4) KVC_TC_DEC(128, 4);
    else KVC_TC_DEC(128, 16);
  } else {
    if (rd <= 1) KVC_TC_DEC(64, 1);
    else if (rd <= 4) KVC_TC_DEC(64, 4);
    else KVC_TC_DEC(64, 16);
  }
#undef KVC_TC_DEC3
#undef KVC_TC_DEC
  return check_launch("tc_decompress_kernel");
}

int tc_read_device_error(int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tc::g_kvc_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("device error read: ") + cudaGetErrorString(e));
  *out = v;
  int zero = 0;
  cudaMemcpyToSymbol(tc::g_kvc_device_error, &zero, sizeof(int));
  return KVC_OK;
}

}  // namespace kvc
