// Tensor-core (tcgen05 / TMEM, TMA-fed) kernels for the residual encode and
// the fused decode, bf16 caches with head_dim 64 or 128.
//
// Both are persistent, warp-specialised kernels (448 threads, one CTA per
// SM) over 128-row tiles:
//   warp 5     TMA: one thread loads each tile into a 3-stage ring
//   warps 0-3  transform, one row per thread: encode subtracts the Tucker
//              term in place (R = x - recon), decode turns codes into exact
//              bf16 integers in the swizzled operand tile
//   warp 4     one thread issues tcgen05.mma into one of two TMEM
//              accumulators (128 lanes x d fp32 columns each)
//   warps 6-13 epilogue: tcgen05.ld of the accumulator rows, then the
//              per-tile output; two warps per TMEM lane group
//
// Residual encode (kvcompress/compressor/residual.py:201-239):
//   A = R = bf16(x - bf16(recon)) (exact operand), B = the JL matrix Pi
//   split into three bf16 terms (hi + mid + lo = Pi to fp32 precision), so
//   the accumulator holds R Pi^T to fp32 accuracy.  Mode STATS reduces the
//   per-column |max| (symmetric: a running per-thread absmax, one
//   transpose-reduce per cell) or min / max (per tile); mode QUANT divides
//   by the scale, rounds half to even, clamps and packs.
// Decode (kvcompress/compressor/jolt.py:424-463, residual.py:242-288):
//   A = the integer codes (exact in bf16), B = diag(scale) Pi in two bf16
//   terms; the epilogue adds the fp32 Tucker term and writes the tile.
//
// Every mbarrier wait is bounded (kvc_tc.cuh) and warp-uniform: a warp
// whose wait times out leaves its loop as a whole, so the others time out
// in turn and the kernel returns with the error word set.
#include <algorithm>
#include <type_traits>

#include "kvc_common.cuh"
#include "kvc_quant.cuh"
#include "kvc_tc.cuh"
#include "kvc_tma.cuh"

namespace kvc {
namespace {

using namespace tc;

constexpr int TILE_M = 128;
constexpr int NSTAGE = 3;
constexpr int NTHREADS = 448;
constexpr int MMA_WARP = 4;
constexpr int TMA_WARP = 5;
constexpr int EPI_WARP0 = 6;
constexpr int NEPI = 256;  // epilogue threads
constexpr int RD_MAX = 16;

// Quantiser fast path: t = fma(v, fl(1/s), zp) differs from the reference's
// fl(fl(v / s) + zp) by at most 2^-24 (3 |v/s| + 2 |t|) (the reciprocal,
// product and sum roundings against the quotient and sum roundings).  When
// t sits farther than that bound from a half-integer, rint(t) equals the
// reference's rounding; otherwise the exact quotient decides.  When |t| >=
// 257 both clamp to the same code (|qmin|, qmax <= 255).

// 32 codes (low byte of each bq: q + offset in [0, 2^bits)) -> bits words.
__device__ __forceinline__ void pack_codes(const int32_t (&bq)[32], uint32_t (&w)[8], int bits) {
  if (bits == 8) {
#pragma unroll
    for (int b = 0; b < 8; ++b)
      w[b] = __byte_perm(__byte_perm(bq[4 * b], bq[4 * b + 1], 0x0040), __byte_perm(bq[4 * b + 2], bq[4 * b + 3], 0x0040),
                         0x5410);
  } else if (bits == 4) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = ((uint32_t)bq[8 * b + 2 * i] << 4) | ((uint32_t)bq[8 * b + 2 * i + 1] & 0xFu);
      w[b] = __byte_perm(__byte_perm(p[0], p[1], 0x0040), __byte_perm(p[2], p[3], 0x0040), 0x5410);
    }
  } else {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      uint32_t p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = 16 * b + 4 * i;
        p[i] = ((uint32_t)bq[k] << 6) | (((uint32_t)bq[k + 1] & 3u) << 4) | (((uint32_t)bq[k + 2] & 3u) << 2) |
               ((uint32_t)bq[k + 3] & 3u);
      }
      w[b] = __byte_perm(__byte_perm(p[0], p[1], 0x0040), __byte_perm(p[2], p[3], 0x0040), 0x5410);
    }
  }
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// Warp-uniform bounded wait: every lane polls, the warp continues only if
// all lanes saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity, int code) {
  return __all_sync(0xffffffffu, mbar_wait(b, parity, code));
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

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
enum { MODE_STATS = 0, MODE_QUANT = 1 };

template <int D>
struct EncLayout {
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_BYTES = 3 * B_TERM;
  static constexpr uint32_t A_BYTES = TILE_M * D * 2;
  static constexpr uint32_t OFF_A = B_BYTES;
  static constexpr uint32_t OFF_U = OFF_A + NSTAGE * A_BYTES;  // 4 transform warps x D x 4 fp32
  static constexpr uint32_t OFF_UB = OFF_U + 4 * D * 16;        // 4 transform warps x D bf16
  static constexpr uint32_t OFF_SC = OFF_UB + 4 * D * 2;        // 8 epilogue warps x D x (1/s, s, zp)
  static constexpr uint32_t OFF_Q = OFF_SC + 8 * D * 12;       // 8 epilogue warps x 32 lanes x 32 code bytes
  static constexpr uint32_t OFF_BAR = OFF_Q + 8 * 32 * 32;
  static constexpr uint32_t NBAR = 3 * NSTAGE + 4;              // loaded, full, empty, acc full x2, acc empty x2
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;         // + alignment slack
};

struct EncArgs {
  CellPtrs ud, scale, zp;
  CellPtrsMut codes;
  int64_t rows, tiles_per_cell, total_tiles, tiles_per_cta;
  int rt, rd, bits, symmetric, scale_mode, arith_dtype, code_bytes;
  const uint8_t* bops;  // 3 swizzled B tiles of Pi
  int32_t* minmax;      // STATS: [cell][2][d] ordered ints (min, max)
  const float* tmp;     // [cell][row][rdm]: sum_a core[h][a][r] u_token[t][a], rounded to bf16
};

// RDM: 1 (rd == 1, packed bf16x2 residual) or 4 (rd <= 4, fp32 residual).
template <int D, int MODE, bool SYM, int RDM>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_encode_kernel(const __grid_constant__ TmaMaps maps, const __grid_constant__ EncArgs A) {
  using L = EncLayout<D>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NSTAGE;
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
    const uint4* src = reinterpret_cast<const uint4*>(A.bops);
    uint4* dst = reinterpret_cast<uint4*>(smem);
    for (int i = threadIdx.x; i < (int)(L::B_BYTES / 16); i += NTHREADS) dst[i] = src[i];
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&loaded[i], 1);  // TMA issue + transaction bytes
      mbar_init(&full[i], 128);  // transform threads
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
    // ---------------- transform: R = x - recon, one row per thread ----------------
    const int ptid = threadIdx.x;
    float* u32 = reinterpret_cast<float*>(smem + L::OFF_U) + warp * D * 4;               // [j][4]
    uint16_t* ub = reinterpret_cast<uint16_t*>(smem + L::OFF_UB) + warp * D;             // [j]
    int cur_cell = -1;
    auto tmp_of = [&](int it) {
      float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
      if (A.rt <= 0 || it >= n_my) return r;
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      if (row >= A.rows) return r;
      const float* p = A.tmp + ((int64_t)cell * A.rows + row) * RDM;
      if (RDM == 1) r.x = __ldg(p);
      else r = __ldg(reinterpret_cast<const float4*>(p));
      return r;
    };
    float4 tnext = tmp_of(0);
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      const int st = it % NSTAGE;
      const float4 tv = tnext;
      tnext = tmp_of(it + 1);  // issued now, used one tile later
      if (A.rt > 0 && cell != cur_cell) {
        __syncwarp();
        const __nv_bfloat16* ud = static_cast<const __nv_bfloat16*>(A.ud.p[cell]);
        if (RDM == 1) {
          for (int j = lane; j < D; j += 32) ub[j] = reinterpret_cast<const uint16_t*>(ud)[j];
        } else {
          for (int i = lane; i < D * 4; i += 32) {
            const int j = i >> 2, r = i & 3;
            u32[i] = r < A.rd ? __bfloat162float(ud[j * A.rd + r]) : 0.f;
          }
        }
        __syncwarp();
        cur_cell = cell;
      }
      if (!warp_wait(&loaded[st], (uint32_t)((it / NSTAGE) & 1), 0x131)) break;
      if (A.rt > 0 && row < A.rows) {
        uint8_t* As = smem + L::OFF_A + st * L::A_BYTES;
        if (RDM == 1) {
          // rd == 1: recon = bf16(t * u_j) and R = bf16(x - recon), both a
          // single rounding of the exact bf16 product / difference.
          const uint32_t th = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(tv.x));
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(As + sw128_off(ptid, c * 8, TILE_M));
            uint4 x = *slot;
            const uint4 u = u4[c];
            x.x = bf16x2_sub(x.x, bf16x2_mul(t2, u.x));
            x.y = bf16x2_sub(x.y, bf16x2_mul(t2, u.y));
            x.z = bf16x2_sub(x.z, bf16x2_mul(t2, u.z));
            x.w = bf16x2_sub(x.w, bf16x2_mul(t2, u.w));
            *slot = x;
          }
        } else {
          const float4* u4 = reinterpret_cast<const float4*>(u32);
#pragma unroll 2
          for (int c = 0; c < D / 8; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(As + sw128_off(ptid, c * 8, TILE_M));
            float xv[8];
            unpack8<__nv_bfloat16>(*slot, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float4 u = u4[c * 8 + e];
              float rec = tv.x * u.x;
              rec = fmaf(tv.y, u.y, rec);
              rec = fmaf(tv.z, u.z, rec);
              rec = fmaf(tv.w, u.w, rec);
              xv[e] = Elt<__nv_bfloat16>::round(xv[e] - Elt<__nv_bfloat16>::round(rec));
            }
            *slot = pack8<__nv_bfloat16>(xv);
          }
        }
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
  } else if (warp == TMA_WARP) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int it = 0; it < n_my; ++it) {
        const int64_t g = tile_begin + it;
        const int cell = (int)(g / A.tiles_per_cell);
        const int y = (int)((g % A.tiles_per_cell) * TILE_M);
        const int st = it % NSTAGE;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NSTAGE) & 1) ^ 1u, 0x121)) break;
        mbar_expect_tx(&loaded[st], L::A_BYTES);
        const uint32_t dst = sbase + L::OFF_A + st * L::A_BYTES;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * TILE_M * 128, &maps.m[cell], h * 64, y, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(TILE_M, D, true);
      int it = 0;
      for (; it < n_my; ++it) {
        const int st = it % NSTAGE, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NSTAGE) & 1), 0x201)) break;
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x202)) break;
        tc_fence_after();
        const uint32_t a_base = sbase + L::OFF_A + st * L::A_BYTES;
        const uint32_t d_tmem = tmem + (uint32_t)(ac * D);
#pragma unroll
        for (int term = 0; term < 3; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t ka = (uint32_t)((ks >> 2) * (TILE_M * 128) + (ks & 3) * 32);
            const uint32_t kb = (uint32_t)((ks >> 2) * (D * 128) + (ks & 3) * 32);
            umma_f16(d_tmem, desc_sw128(a_base + ka), desc_sw128(sbase + term * L::B_TERM + kb), idesc,
                     (term | ks) ? 1u : 0u);
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
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;  // 32-column chunks per warp
    float* inv_s = reinterpret_cast<float*>(smem + L::OFF_SC) + e * 3 * D;
    float* s_s = inv_s + D;
    float* zp_s = s_s + D;
    uint8_t* qstage = smem + L::OFF_Q + e * 32 * 32;
    float run[NCH][32];  // STATS, SYM: running |max| of this thread's row position
    float rmax[NCH], rmin[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      rmax[c] = -__int_as_float(0x7f800000);
      rmin[c] = __int_as_float(0x7f800000);
#pragma unroll
      for (int j = 0; j < 32; ++j) run[c][j] = 0.f;
    }
    int qmin, qmax;
    qrange(A.bits > 0 ? A.bits : 8, A.symmetric, qmin, qmax);
    const int offset = A.symmetric ? (1 << (A.bits - 1)) : 0;
    const bool fast = A.scale_mode != KVC_SCALE_TENSOR || A.arith_dtype == KVC_F32;
    const int ad = A.scale_mode == KVC_SCALE_TENSOR ? A.arith_dtype : KVC_F32;
    // bound on |t - fl(fl(v / s) + zp)| of the fast path: 2^-24 (3 |v/s| + 2 |t|);
    // symmetric |t| < 257 (beyond it both clamp): 4.6e-5 < 2^-14; asymmetric
    // with |zp| <= 512: 1.7e-4 < 2^-12
    const float guard = SYM ? 0.5f - 1.0f / 16384.0f : 0.5f - 1.0f / 4096.0f;
    const float magic = 12582912.0f + (float)offset;  // 1.5 * 2^23 + offset
    const int lo_bits = 0x4B400000 + offset + qmin, hi_bits = 0x4B400000 + offset + qmax;
    uint32_t fastc = 0;
    auto flush_stats = [&](int cell) {
      int32_t* mm = A.minmax + (int64_t)cell * 2 * D;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int col = (half * NCH + c) * 32 + lane;
        if (SYM) {
          const float am = transpose_reduce32<true>(run[c]);
          atomicMin(&mm[col], ordered_bits(-am));
          atomicMax(&mm[D + col], ordered_bits(am));
#pragma unroll
          for (int j = 0; j < 32; ++j) run[c][j] = 0.f;
        } else {
          atomicMin(&mm[col], ordered_bits(rmin[c]));
          atomicMax(&mm[D + col], ordered_bits(rmax[c]));
          rmax[c] = -__int_as_float(0x7f800000);
          rmin[c] = __int_as_float(0x7f800000);
        }
      }
    };
    int cur_cell = -1;
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      if (cell != cur_cell) {
        if (MODE == MODE_STATS && cur_cell >= 0) flush_stats(cur_cell);
        if (MODE == MODE_QUANT) {
          __syncwarp();
          const float* sc = static_cast<const float*>(A.scale.p[cell]);
          const int32_t* zz = static_cast<const int32_t*>(A.zp.p[cell]);
          for (int j = lane; j < D; j += 32) {
            const int jj = A.scale_mode == KVC_SCALE_CHANNEL ? j : 0;
            s_s[j] = sc[jj];
            inv_s[j] = __fdiv_rn(1.0f, sc[jj]);
            zp_s[j] = (float)zz[jj];
          }
          __syncwarp();
          // the fast path's error bound needs |v / s| < 769: |zp| <= 512
          fastc = 0;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            const int c = half * NCH + cc;
            if (__all_sync(0xffffffffu, fabsf(zp_s[c * 32 + lane]) <= 512.f) && fast) fastc |= 1u << cc;
          }
        }
        cur_cell = cell;
      }
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x301)) break;
      tc_fence_after();
      const int64_t row = tile * TILE_M + rloc;
      const bool valid = row < A.rows;
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        if (MODE == MODE_STATS) {
          if (SYM) {
            // rows past the end hold R = 0 and cannot raise |max|
#pragma unroll
            for (int j = 0; j < 32; ++j) run[cc][j] = fmaxf(run[cc][j], fabsf(v[j]));
          } else {
            float w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              w[j] = valid ? v[j] : __int_as_float(0x7f800000);
              v[j] = valid ? v[j] : -__int_as_float(0x7f800000);
            }
            rmax[cc] = fmaxf(rmax[cc], transpose_reduce32<true>(v));
            rmin[cc] = fminf(rmin[cc], transpose_reduce32<false>(w));
          }
        } else {
          // codes (low byte of bq = q + offset) of this row's 32 columns
          int32_t bq[32];
          bool slow = false;
          const bool fast_c = (fastc >> cc) & 1u;
          if (fast_c) {
            // t = v / s + zp by reciprocal, rounded by adding 1.5 * 2^23 +
            // offset: the float bits of y are 0x4B400000 + offset + rint(t)
            const uint64_t* inv2 = reinterpret_cast<const uint64_t*>(inv_s + c * 32);
            const uint64_t* zp2 = reinterpret_cast<const uint64_t*>(zp_s + c * 32);
            const uint64_t M2 = f2_pack(magic, magic), NM2 = f2_pack(-magic, -magic);
            const uint64_t NEG1 = f2_pack(-1.f, -1.f);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint64_t v2 = f2_pack(v[j], v[j + 1]);
              const uint64_t t2 = SYM ? f2_mul(v2, inv2[j / 2]) : f2_fma(v2, inv2[j / 2], zp2[j / 2]);
              const uint64_t y2 = f2_add(t2, M2);
              const uint64_t d2 = f2_fma(f2_add(y2, NM2), NEG1, t2);  // t - rint(t)
              float d0, d1, y0, y1;
              f2_unpack(d2, d0, d1);
              f2_unpack(y2, y0, y1);
              slow |= (fabsf(d0) > guard) | (fabsf(d1) > guard);
              bq[j] = min(max(__float_as_int(y0), lo_bits), hi_bits);
              bq[j + 1] = min(max(__float_as_int(y1), lo_bits), hi_bits);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              bq[j] = quantize_one(v[j], s_s[c * 32 + j], (int32_t)zp_s[c * 32 + j], qmin, qmax, ad) + offset;
          }
          uint32_t w[8];
          pack_codes(bq, w, A.bits);
          if (__any_sync(0xffffffffu, slow && valid)) {
            // near a rounding tie the exact quotient decides: reload each
            // column from TMEM, redo the fast-path test, patch flagged codes
            uint8_t* slot = qstage + lane * 32;
#pragma unroll
            for (int b = 0; b < 8; ++b)
              if (b < A.bits) reinterpret_cast<uint32_t*>(slot)[b] = w[b];
#pragma unroll 1
            for (int j = 0; j < 32; ++j) {
              const float vj = tmem_ld1(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32 + j));
              if (valid && slow) {
                const float tq = SYM ? __fmul_rn(vj, inv_s[c * 32 + j]) : fmaf(vj, inv_s[c * 32 + j], zp_s[c * 32 + j]);
                const float rq = __fadd_rn(__fadd_rn(tq, magic), -magic);
                if (fabsf(__fadd_rn(tq, -rq)) > guard) {
                  const float re = rintf(__fadd_rn(__fdiv_rn(vj, s_s[c * 32 + j]), zp_s[c * 32 + j]));
                  const uint32_t code = (uint32_t)((int)fminf(fmaxf(re, (float)qmin), (float)qmax) + offset);
                  if (A.bits == 8) {
                    slot[j] = (uint8_t)code;
                  } else if (A.bits == 4) {
                    const int sh = (j & 1) ? 0 : 4;
                    slot[j >> 1] = (uint8_t)((slot[j >> 1] & ~(0xF << sh)) | ((code & 0xF) << sh));
                  } else {
                    const int sh = 6 - 2 * (j & 3);
                    slot[j >> 2] = (uint8_t)((slot[j >> 2] & ~(3 << sh)) | ((code & 3) << sh));
                  }
                }
              }
            }
#pragma unroll
            for (int b = 0; b < 8; ++b)
              if (b < A.bits) w[b] = reinterpret_cast<uint32_t*>(slot)[b];
          }
          if (valid) {
            uint8_t* dst = static_cast<uint8_t*>(A.codes.p[cell]) + row * A.code_bytes + c * 4 * A.bits;
            if (A.bits == 8) {
              reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
              reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else if (A.bits == 4) {
              *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
              *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (MODE == MODE_STATS && cur_cell >= 0) flush_stats(cur_cell);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * D);
  }
}

// Per-row Tucker term for the tensor-core kernels, padded to rdm columns:
//   tmp[cell][row][r] = sum_a core[h][a][r] * u_token[t][a]   (rows of [t0, t1))
// rounded to `round_dt` (the encode rounds it to the cell dtype like the
// reference's einsum intermediate; the decode keeps fp32).
__global__ void tucker_rows_kernel(CellPtrs core, CellPtrs ut, int fdt, int round_dt_, int64_t m, int64_t t0,
                                   int64_t tl, int rt, int rd, int rdm, float* tmp) {
  const int cell = blockIdx.y;
  const int64_t rows = m * tl;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows * rdm;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / rdm;
    const int r = (int)(idx % rdm);
    float acc = 0.f;
    if (r < rd) {
      const int64_t h = row / tl, t = t0 + row % tl;
      for (int a = 0; a < rt; ++a)
        acc = fmaf(load_dt(core.p[cell], (h * rt + a) * rd + r, fdt), load_dt(ut.p[cell], t * rt + a, fdt), acc);
      acc = round_dt(acc, round_dt_);
    }
    tmp[(int64_t)cell * rows * rdm + idx] = acc;
  }
}

int rdm_enc(int rd) { return rd <= 1 ? 1 : 4; }
int rdm_dec(int rd) { return rd <= 1 ? 1 : (rd <= 4 ? 4 : 16); }

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

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

// Pi split into three bf16 terms, laid out as swizzled K-major B tiles:
// B[n][k] = Pi[n][k] (D = R Pi^T).
__global__ void prep_rotation_kernel(const float* __restrict__ proj, int d, uint8_t* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= d * d) return;
  const int n = e / d, k = e % d;
  float rest = proj[e];
  for (int term = 0; term < 3; ++term) {
    const __nv_bfloat16 v = __float2bfloat16_rn(rest);
    rest -= __bfloat162float(v);
    *reinterpret_cast<__nv_bfloat16*>(out + (size_t)term * d * d * 2 + sw128_off(n, k, d)) = v;
  }
}

// ------------------------------------------------------------------------
// decode
// ------------------------------------------------------------------------
template <int D, int CB>
struct DecLayout {
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_BYTES = 2 * B_TERM;
  static constexpr uint32_t A_BYTES = TILE_M * D * 2;
  static constexpr uint32_t C_BYTES = TILE_M * CB;
  static constexpr uint32_t OFF_A = B_BYTES;
  static constexpr uint32_t OFF_C = OFF_A + NSTAGE * A_BYTES;
  static constexpr uint32_t OFF_UD = OFF_C + NSTAGE * C_BYTES;  // D x RD_MAX fp32
  static constexpr uint32_t OFF_BAR = OFF_UD + D * RD_MAX * 4;
  static constexpr uint32_t NBAR = 3 * NSTAGE + 4;
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

struct DecArgsTc {
  CellPtrs ud;
  CellPtrsMut out;
  int64_t m, t0, tl, rows_out, tiles_per_cell;
  int tb_per_head, tiles_per_cta;
  int rt, rd, factor_dtype;
  const uint8_t* bops;  // per cell: 2 swizzled B tiles of diag(scale) Pi
  const float* tmp;     // [cell][out row][rdm] fp32 Tucker row term
};

template <int D, int RDM, int BITS>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_decode_kernel(const __grid_constant__ TmaMaps maps, const __grid_constant__ DecArgsTc A) {
  constexpr int CB = D * BITS / 8;  // code bytes per row
  using L = DecLayout<D, CB>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NSTAGE;
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  float* ud_s = reinterpret_cast<float*>(smem + L::OFF_UD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cell = blockIdx.y;
  const int64_t tile_begin = (int64_t)blockIdx.x * A.tiles_per_cta;
  const int64_t tile_end = tile_begin + A.tiles_per_cta < A.tiles_per_cell ? tile_begin + A.tiles_per_cta
                                                                         : A.tiles_per_cell;
  const int n_my = (int)(tile_end > tile_begin ? tile_end - tile_begin : 0);
  {
    const uint4* src = reinterpret_cast<const uint4*>(A.bops + (size_t)cell * L::B_BYTES);
    uint4* dst = reinterpret_cast<uint4*>(smem);
    for (int i = threadIdx.x; i < (int)(L::B_BYTES / 16); i += NTHREADS) dst[i] = src[i];
  }
  if (A.rt > 0)
    for (int i = threadIdx.x; i < D * RDM; i += NTHREADS) {
      const int j = i / RDM, r = i % RDM;
      ud_s[i] = r < A.rd ? load_dt(A.ud.p[cell], (int64_t)j * A.rd + r, A.factor_dtype) : 0.f;
    }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&loaded[i], 1);
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
    // codes (dense rows of CB bytes) -> exact integers in bf16 -> swizzled A tile
    constexpr int LPR = CB / 16 > 0 ? CB / 16 : 1;  // lanes per row, 16 code bytes each
    constexpr int RPI = 32 / LPR;                   // rows per warp iteration
    constexpr int NIT = 32 / RPI;
    constexpr int PER = 8 / BITS;     // codes per byte
    constexpr int VALS = 16 * PER;    // values per lane
    static_assert(CB % 16 == 0, "code rows must be whole 16-byte chunks");
    const int pos = lane % LPR, sub = lane / LPR;
    // a code byte b placed in the mantissa of 2^23 reads 2^23 + b; subtracting
    // 2^23 + offset leaves the signed code exactly
    const float bias = 8388608.0f + (float)(1 << (BITS - 1));
    const uint64_t NB2 = f2_pack(-bias, -bias);
    for (int it = 0; it < n_my; ++it) {
      const int st = it % NSTAGE;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NSTAGE) & 1), 0x141)) break;
      const uint8_t* Cs = smem + L::OFF_C + st * L::C_BYTES;
      uint8_t* As = smem + L::OFF_A + st * L::A_BYTES;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int rloc = warp * 32 + i * RPI + sub;
        const uint4 raw = *reinterpret_cast<const uint4*>(Cs + rloc * CB + pos * 16);
        const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o[VALS / 2];  // bf16 pairs in value order
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          uint32_t pl[PER];  // plane p: the code at bit offset BITS*(PER-1-p) of every byte
#pragma unroll
          for (int pp = 0; pp < PER; ++pp)
            pl[pp] = (words[wi] >> (BITS * (PER - 1 - pp))) & ((uint32_t)((1 << BITS) - 1) * 0x01010101u);
#pragma unroll
          for (int k = 0; k < 4 * PER; k += 2) {
            const int b0 = k / PER, p0 = k % PER, b1 = (k + 1) / PER, p1 = (k + 1) % PER;
            const float f0 = __uint_as_float(__byte_perm(pl[p0], 0x4B000000u, 0x7540 | b0));
            const float f1 = __uint_as_float(__byte_perm(pl[p1], 0x4B000000u, 0x7540 | b1));
            float q0, q1;
            f2_unpack(f2_add(f2_pack(f0, f1), NB2), q0, q1);
            const __nv_bfloat162 h = __floats2bfloat162_rn(q0, q1);
            o[(wi * 4 * PER + k) / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
#pragma unroll
        for (int cb = 0; cb < VALS / 8; ++cb)
          *reinterpret_cast<uint4*>(As + sw128_off(rloc, pos * VALS + cb * 8, TILE_M)) =
              make_uint4(o[4 * cb], o[4 * cb + 1], o[4 * cb + 2], o[4 * cb + 3]);
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      for (int it = 0; it < n_my; ++it) {
        const int64_t tile = tile_begin + it;
        const int h = (int)(tile / A.tb_per_head);
        const int tok = (int)(A.t0 + (tile % A.tb_per_head) * TILE_M);
        const int st = it % NSTAGE;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NSTAGE) & 1) ^ 1u, 0x151)) break;
        mbar_expect_tx(&loaded[st], L::C_BYTES);
        tma_load_3d(sbase + L::OFF_C + st * L::C_BYTES, &maps.m[cell], 0, tok, h, &loaded[st]);
      }
    }
    __syncwarp();
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
            umma_f16(d_tmem, desc_sw128(a_base + ka), desc_sw128(sbase + term * L::B_TERM + kb), idesc,
                     (term | ks) ? 1u : 0u);
          }
        }
        umma_commit(&empty[st]);
        umma_commit(&accf[ac]);
      }
      if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x213);
    }
    __syncwarp();
  } else {
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(A.out.p[cell]);
    for (int it = 0; it < n_my; ++it) {
      const int ac = it & 1;
      const int64_t tile = tile_begin + it;
      const int64_t h = tile / A.tb_per_head;
      const int64_t i_tok = (tile % A.tb_per_head) * TILE_M + rloc;  // token within [t0, t1)
      const bool valid = i_tok < A.tl;
      const int64_t orow = h * A.tl + i_tok;
      float tmp[RDM];  // loaded before the wait so the latency overlaps it
#pragma unroll
      for (int r = 0; r < RDM; ++r)
        tmp[r] = (valid && A.rt > 0) ? __ldg(A.tmp + ((int64_t)cell * A.rows_out + orow) * RDM + r) : 0.f;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x311)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        if (valid) {
          uint32_t o[16];  // bf16 pairs
          if (A.rt > 0 && RDM == 1) {
            // out = bf16(fl(t * u_j) + v_j): the reference adds the fp32 Tucker
            // reconstruction to the fp32 decoded residual
            const uint64_t t2 = f2_pack(tmp[0], tmp[0]);
            const uint64_t* u2 = reinterpret_cast<const uint64_t*>(ud_s + c * 32);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float o0, o1;
              f2_unpack(f2_add(f2_mul(t2, u2[j / 2]), f2_pack(v[j], v[j + 1])), o0, o1);
              const __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1);
              o[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float oo[2];
#pragma unroll
              for (int x = 0; x < 2; ++x) {
                if (A.rt > 0) {
                  float rec = 0.f;
#pragma unroll
                  for (int r = 0; r < RDM; ++r) rec = fmaf(tmp[r], ud_s[(c * 32 + j + x) * RDM + r], rec);
                  oo[x] = __fadd_rn(rec, v[j + x]);
                } else {
                  oo[x] = v[j + x];
                }
              }
              const __nv_bfloat162 h = __floats2bfloat162_rn(oo[0], oo[1]);
              o[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
            }
          }
          uint4* dst = reinterpret_cast<uint4*>(out + orow * D + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
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
         align256((size_t)n_cells * rows * rdm_enc(rd) * 4);
}

int tc_residual_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                       const void* const* core, const void* const* u_token, const void* const* u_feature,
                       int rt, int rd, const float* proj, int bits, int symmetric, int scale_mode,
                       int stat_dtype, int arith_dtype, float* const* scale, int32_t* const* zp,
                       uint8_t* const* codes, void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (!workspace || ws_bytes < tc_residual_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core residual: workspace too small");
  const int64_t rows = m * t;
  if (rows >= (1LL << 31)) return fail(KVC_ERR_SHAPE, "tensor-core residual: more than 2^31 rows per cell");
  TmaMaps maps;  // copied into the launch parameters
  EncArgs a;
  memset(&a, 0, sizeof(a));
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)d * 2};
    const uint32_t box[2] = {64u, (uint32_t)TILE_M};
    if ((rc = encode_tma(&maps.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (rt > 0) a.ud.p[c] = u_feature[c];
    if (scale) a.scale.p[c] = scale[c];
    if (zp) a.zp.p[c] = zp[c];
    if (codes) a.codes.p[c] = codes[c];
  }
  a.rows = rows;
  a.rt = rt;
  a.rd = rd;
  a.bits = bits;
  a.symmetric = symmetric;
  a.scale_mode = scale_mode;
  a.arith_dtype = arith_dtype;
  a.code_bytes = (d * bits + 7) / 8;
  a.tiles_per_cell = ceil_div(rows, TILE_M);
  a.total_tiles = a.tiles_per_cell * n_cells;
  const int64_t ctas = std::min<int64_t>(a.total_tiles, num_sms());
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  const int rdm = rdm_enc(rd);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* bops = ws;
  size_t off = align256((size_t)3 * d * d * 2);
  int32_t* mm = reinterpret_cast<int32_t*>(ws + off);
  off += align256((size_t)n_cells * 2 * d * sizeof(int32_t));
  float* tmp = reinterpret_cast<float*>(ws + off);
  a.bops = bops;
  a.minmax = mm;
  a.tmp = tmp;
  prep_rotation_kernel<<<(d * d + 255) / 256, 256, 0, st>>>(proj, d, bops);
  if ((rc = check_launch("prep_rotation_kernel"))) return rc;
  if (rt > 0) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows * rdm, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(cp, up, KVC_BF16, KVC_BF16, m, 0, t, rt, rd, rdm,
                                                              tmp);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  if (mode == 0) {
    minmax_init_kernel<<<(n_cells * 2 * d + 255) / 256, 256, 0, st>>>(mm, n_cells, d);
    if ((rc = check_launch("minmax_init_kernel"))) return rc;
  }
#define KVC_TC_ENC(DD, MODEV, SYMV, RR)                        \
  do {                                                         \
    auto kern = tc_encode_kernel<DD, MODEV, SYMV, RR>;         \
    if ((rc = set_smem(kern, EncLayout<DD>::BYTES))) return rc; \
    kern<<<grid, NTHREADS, EncLayout<DD>::BYTES, st>>>(maps, a); \
  } while (0)
#define KVC_TC_ENC_R(DD, MODEV, SYMV)            \
  do {                                           \
    if (rdm == 1) KVC_TC_ENC(DD, MODEV, SYMV, 1); \
    else KVC_TC_ENC(DD, MODEV, SYMV, 4);         \
  } while (0)
  const bool sym = symmetric != 0;
  if (mode == 0) {
    if (d == 128) {
      if (sym) KVC_TC_ENC_R(128, MODE_STATS, true);
      else KVC_TC_ENC_R(128, MODE_STATS, false);
    } else {
      if (sym) KVC_TC_ENC_R(64, MODE_STATS, true);
      else KVC_TC_ENC_R(64, MODE_STATS, false);
    }
  } else {
    if (d == 128) {
      if (sym) KVC_TC_ENC_R(128, MODE_QUANT, true);
      else KVC_TC_ENC_R(128, MODE_QUANT, false);
    } else {
      if (sym) KVC_TC_ENC_R(64, MODE_QUANT, true);
      else KVC_TC_ENC_R(64, MODE_QUANT, false);
    }
  }
#undef KVC_TC_ENC_R
#undef KVC_TC_ENC
  if ((rc = check_launch("tc_encode_kernel"))) return rc;
  if (mode == 0) {
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
  return out_dtype == KVC_BF16 && (d == 64 || d == 128) && rd <= RD_MAX && bits > 0 && d * bits / 8 >= 16 &&
         symmetric && scale_mode == KVC_SCALE_CHANNEL && proj != nullptr;
}

size_t tc_decompress_workspace(int n_cells, int64_t rows, int d, int rd) {
  return align256((size_t)n_cells * 2 * d * d * 2) + align256((size_t)n_cells * rows * rdm_dec(rd) * 4);
}

int tc_decompress_launch(int n_cells, const uint8_t* const* codes, const float* const* scale, int bits,
                         const void* const* core, const void* const* u_token, const void* const* u_feature,
                         int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd, const float* proj,
                         int64_t t0, int64_t t1, void* const* out, void* workspace, size_t ws_bytes,
                         cudaStream_t st) {
  if (!workspace || ws_bytes < tc_decompress_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core decompress: workspace too small");
  if (t >= (1LL << 31) || m >= (1LL << 31)) return fail(KVC_ERR_SHAPE, "tensor-core decompress: shape too large");
  TmaMaps maps;
  DecArgsTc a;
  memset(&a, 0, sizeof(a));
  CellPtrs sc;
  const int cb = d * bits / 8;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[3] = {(uint64_t)cb, (uint64_t)t, (uint64_t)m};
    const uint64_t strides[2] = {(uint64_t)cb, (uint64_t)cb * t};
    const uint32_t box[3] = {(uint32_t)cb, (uint32_t)TILE_M, 1u};
    if ((rc = encode_tma(&maps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, codes[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    sc.p[c] = scale[c];
    a.out.p[c] = out[c];
    if (rt > 0) a.ud.p[c] = u_feature[c];
  }
  a.m = m;
  a.t0 = t0;
  a.tl = t1 - t0;
  a.rows_out = m * a.tl;
  a.tb_per_head = (int)ceil_div(a.tl, TILE_M);
  a.tiles_per_cell = m * a.tb_per_head;
  const int64_t per_cell = std::max<int64_t>(1, num_sms() / n_cells);
  const int64_t ctas = std::min<int64_t>(a.tiles_per_cell, per_cell);
  a.tiles_per_cta = (int)ceil_div(a.tiles_per_cell, ctas);
  a.rt = rt;
  a.rd = rd;
  a.factor_dtype = factor_dtype;
  const int rdm = rdm_dec(rd);
  uint8_t* bops = static_cast<uint8_t*>(workspace);
  float* tmp = reinterpret_cast<float*>(bops + align256((size_t)n_cells * 2 * d * d * 2));
  a.bops = bops;
  a.tmp = tmp;
  prep_decode_kernel<<<dim3((d * d + 255) / 256, n_cells), 256, 0, st>>>(proj, sc, d, bops);
  if ((rc = check_launch("prep_decode_kernel"))) return rc;
  if (rt > 0) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(a.rows_out * rdm, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(cp, up, factor_dtype, KVC_F32, m, t0, a.tl, rt, rd,
                                                              rdm, tmp);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.tiles_per_cell, a.tiles_per_cta), n_cells);
#define KVC_TC_DEC3(DD, RR, BB)                                      \
  do {                                                               \
    auto kern = tc_decode_kernel<DD, RR, BB>;                        \
    using LL = DecLayout<DD, DD * BB / 8>;                           \
    if ((rc = set_smem(kern, LL::BYTES))) return rc;                 \
    kern<<<grid, NTHREADS, LL::BYTES, st>>>(maps, a);                \
  } while (0)
#define KVC_TC_DEC(DD, RR)                      \
  do {                                          \
    if (bits == 8) KVC_TC_DEC3(DD, RR, 8);      \
    else if (bits == 4) KVC_TC_DEC3(DD, RR, 4); \
    else KVC_TC_DEC3(DD, RR, 2);                \
  } while (0)
  if (d == 128) {
    if (rdm == 1) KVC_TC_DEC(128, 1);
    else if (rdm == 4) KVC_TC_DEC(128, 4);
    else KVC_TC_DEC(128, 16);
  } else {
    // d = 64: 2-bit rows are 16 bytes, the smallest TMA row
    if (rdm == 1) KVC_TC_DEC(64, 1);
    else if (rdm == 4) KVC_TC_DEC(64, 4);
    else KVC_TC_DEC(64, 16);
  }
#undef KVC_TC_DEC3
#undef KVC_TC_DEC
  return check_launch("tc_decode_kernel");
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
