// Tensor-core (tcgen05 / TMEM, TMA-fed) kernels for the residual encode and
// the fused decode, bf16 caches with head_dim 64 or 128.
//
// Both are persistent, warp-specialised kernels (448 threads, one CTA per
// SM) over 128-row tiles of a cell:
//   warp 5     TMA: one thread loads each tile into a ring of NS stages
//   warps 0-3  transform, one row per thread: the encode subtracts the
//              Tucker term in place (R = x - recon), the decode turns codes
//              into exact bf16 integers in the swizzled operand tile
//   warp 4     one thread issues tcgen05.mma into one of two accumulators
//   warps 6-13 epilogue: two warps per TMEM lane group, one column half each
//
// The constant operand sits in tensor memory as the MMA's A operand and the
// tile of rows is the shared-memory B operand, so the accumulator is
// feature-major: TMEM lane = output feature, column = row of the tile.
//   encode:  A = Pi (rows = output features) in three bf16 terms (hi + mid +
//            lo = Pi to fp32 precision), B = R; D = (R Pi^T)^T
//            (kvcompress/compressor/residual.py:201-239).  A thread owns one
//            feature, so the stats pass keeps its |max| (or min / max) in a
//            register; the quantise pass writes the codes of 64 rows x 32
//            features through shared memory with a TMA store.
//   decode:  A = (diag(scale) Pi)^T in two bf16 terms (one buffer per cell,
//            double-buffered in TMEM), B = the codes as exact bf16 integers;
//            the epilogue adds the fp32 Tucker term and stores bf16 tiles by
//            TMA (kvcompress/compressor/jolt.py:424-463, residual.py:242-288).
// Keeping the constant operand out of shared memory buys a deeper TMA ring.
//
// TMEM holds A as one row per lane with two 16-bit elements per 32-bit
// column (element 2w in the low half), written by tcgen05.st.
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

constexpr int TILE_M = 128;  // rows per tile (the MMA N)
constexpr int NTHREADS = 448;
constexpr int MMA_WARP = 4;
constexpr int TMA_WARP = 5;
constexpr int EPI_WARP0 = 6;
constexpr int NEPI = 256;  // epilogue threads
constexpr int RD_MAX = 16;
constexpr uint32_t TM_ACC = 256;  // TMEM column of accumulator 0 (1 at +128)

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

__device__ __forceinline__ uint4 pack8_bf16(const float (&v)[8]) {
  uint4 out;
  uint32_t* w = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return out;
}

__device__ __forceinline__ void unpack8_bf16(const uint4& raw, float (&v)[8]) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(e[i]);
}

// Write this thread's A row (WPR 32-bit pairs per term) from global into
// TMEM columns [col0, col0 + nterm * WPR) of its lane.
template <int WPR>
__device__ __forceinline__ void load_a_rows(uint32_t tmem_lane_base, uint32_t col0, const uint32_t* src, int nterm,
                                            int row, int rows_per_term) {
  for (int term = 0; term < nterm; ++term) {
#pragma unroll
    for (int q = 0; q < WPR / 32; ++q) {
      const uint4* g = reinterpret_cast<const uint4*>(src + ((size_t)term * rows_per_term + row) * WPR + q * 32);
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 w = __ldg(g + i);
        r[4 * i] = w.x;
        r[4 * i + 1] = w.y;
        r[4 * i + 2] = w.z;
        r[4 * i + 3] = w.w;
      }
      tmem_st32(tmem_lane_base + col0 + term * WPR + q * 32, r);
    }
  }
  tmem_wait_st();
}

// ------------------------------------------------------------------------
// residual encode: STATS / QUANT
// ------------------------------------------------------------------------
enum { MODE_STATS = 0, MODE_QUANT = 1 };

// Quantiser of the fused encode.  The reference computes
// q = rint(fl32(fl32(v / s) + zp)) (round half to even, then clamp).  Here
// fl32(v / s) is rebuilt from inv = fl(1/s) and eta = fl(s inv - 1):
// v inv = hi + e exactly (hi = fl(v inv), e by fma), and
// v / s = v inv / (1 + eta) = hi + (e - hi eta) + O(2^-47 |v/s|), so
// RN(hi + RN(e - hi eta)) equals fl32(v / s) unless v / s lies within
// 5 * 2^-48 |v/s| of an fp32 rounding boundary (then they differ by one ulp,
// which changes the code only when that ulp straddles a half-integer: of the
// order of 1e-11 of the values).  No branch and no division per value.

template <int D, int RDM, int NS, int MODE>
struct EncLayout {
  static constexpr uint32_t B_BYTES = TILE_M * D * 2;             // R tile (MMA B operand)
  static constexpr uint32_t T_BYTES = TILE_M * RDM * 4;           // Tucker row term of a tile
  static constexpr uint32_t U_BYTES = RDM == 1 ? D * 2 : D * 16;  // u_feature: bf16 [j] or fp32 [j][4]
  static constexpr uint32_t Q_BUF = 64 * 32;                      // codes of 64 rows x 32 features (<= 8-bit)
  static constexpr uint32_t OFF_T = NS * B_BYTES;
  static constexpr uint32_t OFF_U = OFF_T + NS * T_BYTES;
  static constexpr uint32_t OFF_Q = OFF_U + 4 * U_BYTES;          // 8 epilogue warps x 2 buffers
  static constexpr uint32_t OFF_BAR = OFF_Q + (MODE == MODE_QUANT ? 8 * 2 * Q_BUF : 0);
  static constexpr uint32_t NBAR = 3 * NS + 4;                    // loaded, full, empty, acc full x2, acc empty x2
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;           // + alignment slack
};

struct EncArgs {
  CellPtrs ud, scale, zp;
  CellPtrsMut codes;  // plain stores (2-bit codes)
  int64_t rows, tiles_per_cell, total_tiles, tiles_per_cta;
  int rt, rd, bits, symmetric, scale_mode, arith_dtype, code_bytes;
  const uint32_t* arows;  // A = Pi in three bf16 terms: [term][128 rows][D/2 pairs]
  int32_t* minmax;        // STATS: [cell][2][d] ordered ints (min, max)
  const float* tmp;       // [cell][tiles_per_cell * 128][rdm]: sum_a core[h][a][r] u_token[t][a], bf16-rounded
};

template <int D, int MODE, bool SYM, int RDM, int NS>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_encode_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ TmaMaps cmaps,
                     const __grid_constant__ EncArgs A) {
  using L = EncLayout<D, RDM, NS, MODE>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NS;
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t tile_begin = (int64_t)blockIdx.x * A.tiles_per_cta;
  const int64_t tile_end = tile_begin + A.tiles_per_cta < A.total_tiles ? tile_begin + A.tiles_per_cta
                                                                       : A.total_tiles;
  const int n_my = (int)(tile_end > tile_begin ? tile_end - tile_begin : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
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
    tmem_alloc(tm_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tm_holder;
  // A operand: Pi, the same for every cell
  if (warp < 4) load_a_rows<D / 2>(tmem + ((uint32_t)(warp * 32) << 16), 0, A.arows, 3, warp * 32 + lane, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp < 4) {
    // ---------------- transform: R = x - recon, one row per thread ----------------
    const int ptid = threadIdx.x;
    float* u32 = reinterpret_cast<float*>(smem + L::OFF_U + warp * L::U_BYTES);       // [j][4]
    uint16_t* ub = reinterpret_cast<uint16_t*>(smem + L::OFF_U + warp * L::U_BYTES);  // [j]
    int cur_cell = -1;
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      const int st = it % NS;
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
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x131)) break;
      if (A.rt > 0 && row < A.rows) {
        uint8_t* Bs = smem + st * L::B_BYTES;
        const float* ts = reinterpret_cast<const float*>(smem + L::OFF_T + st * L::T_BYTES) + ptid * RDM;
        if (RDM == 1) {
          // rd == 1: recon = bf16(t * u_j) and R = bf16(x - recon), each a
          // single rounding of the exact bf16 product / difference
          const uint32_t th = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(ts[0]));
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, c * 8, TILE_M));
            uint4 x = *slot;
            const uint4 u = u4[c];
            x.x = bf16x2_sub(x.x, bf16x2_mul(t2, u.x));
            x.y = bf16x2_sub(x.y, bf16x2_mul(t2, u.y));
            x.z = bf16x2_sub(x.z, bf16x2_mul(t2, u.z));
            x.w = bf16x2_sub(x.w, bf16x2_mul(t2, u.w));
            *slot = x;
          }
        } else {
          const float4 tv = *reinterpret_cast<const float4*>(ts);
          const float4* u4 = reinterpret_cast<const float4*>(u32);
#pragma unroll 2
          for (int c = 0; c < D / 8; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, c * 8, TILE_M));
            float xv[8];
            unpack8_bf16(*slot, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float4 u = u4[c * 8 + e];
              float rec = tv.x * u.x;
              rec = fmaf(tv.y, u.y, rec);
              rec = fmaf(tv.z, u.z, rec);
              rec = fmaf(tv.w, u.w, rec);
              xv[e] = Elt<__nv_bfloat16>::round(xv[e] - Elt<__nv_bfloat16>::round(rec));
            }
            *slot = pack8_bf16(xv);
          }
        }
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
  } else if (warp == TMA_WARP) {
    // ---------------- TMA producer: x tile (+ Tucker row term) ----------------
    if (lane == 0) {
      for (int it = 0; it < n_my; ++it) {
        const int64_t g = tile_begin + it;
        const int cell = (int)(g / A.tiles_per_cell);
        const int y = (int)((g % A.tiles_per_cell) * TILE_M);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x121)) break;
        mbar_expect_tx(&loaded[st], L::B_BYTES + (A.rt > 0 ? L::T_BYTES : 0u));
        const uint32_t dst = sbase + st * L::B_BYTES;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * TILE_M * 128, &xmaps.m[cell], h * 64, y, &loaded[st]);
        if (A.rt > 0)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    A.tmp + ((int64_t)cell * A.tiles_per_cell * TILE_M + y) * RDM, L::T_BYTES, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer: D[feature][row] = sum_k Pi[feature][k] R[row][k] ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, TILE_M, true);
      int it = 0;
      for (; it < n_my; ++it) {
        const int st = it % NS, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x201)) break;
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x202)) break;
        tc_fence_after();
        const uint32_t b_base = sbase + st * L::B_BYTES;
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * TILE_M);
#pragma unroll
        for (int term = 0; term < 3; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t kb = (uint32_t)((ks >> 2) * (TILE_M * 128) + (ks & 3) * 32);
            umma_f16_ts(d_tmem, tmem + (uint32_t)(term * (D / 2) + ks * 8), desc_sw128(b_base + kb), idesc,
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
    // ---------------- epilogue: thread = output feature, 64 rows per tile ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int feat = lg * 32 + lane;
    const bool active = lg * 32 < D;  // warp-uniform (d = 64 uses lane groups 0-1)
    uint8_t* qst = smem + L::OFF_Q + e * 2 * L::Q_BUF;
    int qmin, qmax;
    qrange(A.bits > 0 ? A.bits : 8, A.symmetric, qmin, qmax);
    const int offset = A.symmetric ? (1 << (A.bits - 1)) : 0;
    const int ad = A.scale_mode == KVC_SCALE_TENSOR ? A.arith_dtype : KVC_F32;
    const float magic = 12582912.0f + (float)offset;  // 1.5 * 2^23 + offset
    const int lo_bits = 0x4B400000 + offset + qmin, hi_bits = 0x4B400000 + offset + qmax;
    float run_max = 0.f, rmin = __int_as_float(0x7f800000), rmax = -__int_as_float(0x7f800000);
    float s_j = 1.f, inv_j = 1.f, eta_j = 0.f, zp_j = 0.f;
    bool fast = true;
    auto flush_stats = [&](int cell) {
      if (!active) return;
      int32_t* mm = A.minmax + (int64_t)cell * 2 * D;
      if (SYM) {
        atomicMin(&mm[feat], ordered_bits(-run_max));
        atomicMax(&mm[D + feat], ordered_bits(run_max));
        run_max = 0.f;
      } else {
        atomicMin(&mm[feat], ordered_bits(rmin));
        atomicMax(&mm[D + feat], ordered_bits(rmax));
        rmax = -__int_as_float(0x7f800000);
        rmin = __int_as_float(0x7f800000);
      }
    };
    int cur_cell = -1;
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      if (cell != cur_cell) {
        if (MODE == MODE_STATS && cur_cell >= 0) flush_stats(cur_cell);
        if (MODE == MODE_QUANT && active) {
          const int jj = A.scale_mode == KVC_SCALE_CHANNEL ? feat : 0;
          s_j = static_cast<const float*>(A.scale.p[cell])[jj];
          inv_j = __fdiv_rn(1.0f, s_j);
          eta_j = fmaf(s_j, inv_j, -1.0f);
          zp_j = (float)static_cast<const int32_t*>(A.zp.p[cell])[jj];
          fast = A.scale_mode != KVC_SCALE_TENSOR || A.arith_dtype == KVC_F32;
        }
        cur_cell = cell;
      }
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x301)) break;
      tc_fence_after();
      const int64_t row0 = tile * TILE_M + half * 64;  // first row of this warp's half
      uint8_t* buf = qst + (it & 1) * L::Q_BUF;
      if (MODE == MODE_QUANT && active && A.bits > 2) {
        // the TMA store issued from this buffer two tiles ago has read it
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * TILE_M + half * 64 + cc * 32), v);
        if (!active) continue;
        if (MODE == MODE_STATS) {
          if (SYM) {
            // rows past the end hold R = 0 and cannot raise |max|
#pragma unroll
            for (int j = 0; j < 32; ++j) run_max = fmaxf(run_max, fabsf(v[j]));
          } else {
            const int64_t nvalid = A.rows - (row0 + cc * 32);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) {
                rmax = fmaxf(rmax, v[j]);
                rmin = fminf(rmin, v[j]);
              }
          }
        } else {
          int code[32];
          if (fast) {
            // fl32(v / s) from the error-free product v * fl(1/s) = hi + e and
            // the reciprocal's residual eta = s fl(1/s) - 1:  RN(hi + (e - hi eta)).
            // Branch-free; the float bits of y = t + 1.5 * 2^23 + offset are
            // 0x4B400000 + offset + rint(t) (ties to even), clamped to the codes
            const uint64_t M2 = f2_pack(magic, magic), NEG1 = f2_pack(-1.f, -1.f);
            const uint64_t I2 = f2_pack(inv_j, inv_j), NI2 = f2_pack(-inv_j, -inv_j);
            const uint64_t E2 = f2_pack(eta_j, eta_j), Z2 = f2_pack(zp_j, zp_j);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint64_t v2 = f2_pack(v[j], v[j + 1]);
              const uint64_t nhi = f2_mul(v2, NI2);        // -hi
              const uint64_t e = f2_fma(v2, I2, nhi);       // v * inv - hi, exact
              const uint64_t lo = f2_fma(nhi, E2, e);       // e - hi * eta
              uint64_t t2 = f2_fma(nhi, NEG1, lo);          // RN(hi + lo) = fl32(v / s)
              if (!SYM) t2 = f2_add(t2, Z2);                // fl32(v / s) + zp, as the reference
              const uint64_t y2 = f2_add(t2, M2);
              float y0, y1;
              f2_unpack(y2, y0, y1);
              code[j] = min(max(__float_as_int(y0), lo_bits), hi_bits) - 0x4B400000;
              code[j + 1] = min(max(__float_as_int(y1), lo_bits), hi_bits) - 0x4B400000;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) code[j] = quantize_one(v[j], s_j, (int32_t)zp_j, qmin, qmax, ad) + offset;
          }
          // stage: buf[row][feature byte] for the 64 rows x 32 features of this warp
          if (A.bits == 8) {
#pragma unroll
            for (int j = 0; j < 32; ++j) buf[(cc * 32 + j) * 32 + lane] = (uint8_t)code[j];
          } else if (A.bits == 4) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int other = __shfl_xor_sync(0xffffffffu, code[j], 1);
              if (!(lane & 1)) buf[(cc * 32 + j) * 16 + (lane >> 1)] = (uint8_t)((code[j] << 4) | (other & 0xF));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int c1 = __shfl_down_sync(0xffffffffu, code[j], 1);
              const int c2 = __shfl_down_sync(0xffffffffu, code[j], 2);
              const int c3 = __shfl_down_sync(0xffffffffu, code[j], 3);
              if (!(lane & 3))
                buf[(cc * 32 + j) * 8 + (lane >> 2)] =
                    (uint8_t)((code[j] << 6) | ((c1 & 3) << 4) | ((c2 & 3) << 2) | (c3 & 3));
            }
          }
        }
      }
      if (MODE == MODE_QUANT && active) {
        if (A.bits > 2) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (row0 < A.rows) tma_store_2d(&cmaps.m[cell], lg * 4 * A.bits, (int)row0, smem_u32(buf));
            bulk_commit();
          }
        } else {
          // 2-bit: 8 bytes per row, below the 16-byte TMA box; lanes store rows
          __syncwarp();
          uint8_t* dst = static_cast<uint8_t*>(A.codes.p[cell]);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int r = lane + 32 * h2;
            if (row0 + r < A.rows)
              *reinterpret_cast<uint2*>(dst + (row0 + r) * A.code_bytes + lg * 8) =
                  *reinterpret_cast<const uint2*>(buf + r * 8);
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (MODE == MODE_STATS && cur_cell >= 0) flush_stats(cur_cell);
    if (MODE == MODE_QUANT && lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per-row Tucker term for the tensor-core kernels, padded to rdm columns:
//   tmp[cell][row][r] = sum_a core[h][a][r] * u_token[t0 + i][a],  row = h * tl + i
// at cell_stride rows per cell, rounded to `round_dt` (the encode rounds it
// to the cell dtype like the reference's einsum intermediate; the decode
// keeps fp32).
__global__ void tucker_rows_kernel(CellPtrs core, CellPtrs ut, int fdt, int round_dt_, int64_t m, int64_t t0,
                                   int64_t tl, int rt, int rd, int rdm, int64_t cell_stride, float* tmp) {
  const int cell = blockIdx.y;
  const int64_t rows = m * tl;  // rows * rdm < 2^31 (checked by the launchers)
  const uint32_t utl = (uint32_t)tl, urdm = (uint32_t)rdm;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows * rdm;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t row = (uint32_t)idx / urdm;
    const int r = (int)((uint32_t)idx - row * urdm);
    float acc = 0.f;
    if (r < rd) {
      const uint32_t h = row / utl;
      const int64_t t = t0 + (row - h * utl);
      for (int a = 0; a < rt; ++a)
        acc = fmaf(load_dt(core.p[cell], ((int64_t)h * rt + a) * rd + r, fdt), load_dt(ut.p[cell], t * rt + a, fdt),
                   acc);
      acc = round_dt(acc, round_dt_);
    }
    tmp[(int64_t)cell * cell_stride * rdm + idx] = acc;
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

// A rows of the encode: Pi[m][k] split in three bf16 terms, as 32-bit pairs
// (k = 2w in the low half) [term][m < 128][d / 2]; rows m >= d are zero.
__global__ void prep_rotation_kernel(const float* __restrict__ proj, int d, uint32_t* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // (m, w) over 128 x d/2
  const int wpr = d / 2;
  if (e >= 128 * wpr) return;
  const int m = e / wpr, w = e % wpr;
  float r0 = m < d ? proj[m * d + 2 * w] : 0.f, r1 = m < d ? proj[m * d + 2 * w + 1] : 0.f;
  for (int term = 0; term < 3; ++term) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(r0, r1);
    r0 -= __low2float(h);
    r1 -= __high2float(h);
    out[((size_t)term * 128 + m) * wpr + w] = *reinterpret_cast<const uint32_t*>(&h);
  }
}

// ------------------------------------------------------------------------
// decode
// ------------------------------------------------------------------------
template <int D, int CB, int NS>
struct DecLayout {
  static constexpr uint32_t B_BYTES = TILE_M * D * 2;  // codes as bf16 (MMA B operand)
  static constexpr uint32_t C_BYTES = TILE_M * CB;     // codes as loaded
  static constexpr uint32_t O_BUF = 64 * 32 * 2;       // 64 rows x 32 features bf16
  static constexpr uint32_t OFF_C = NS * B_BYTES;
  static constexpr uint32_t OFF_O = OFF_C + NS * C_BYTES;  // 8 epilogue warps x 2 buffers
  static constexpr uint32_t OFF_R = OFF_O + 8 * 2 * O_BUF;  // 8 epilogue warps x 64 Tucker row terms (rd = 1)
  static constexpr uint32_t OFF_BAR = OFF_R + 8 * 64 * 4;
  static constexpr uint32_t NBAR = 3 * NS + 6;  // loaded, full, empty, acc full x2, acc empty x2, A free x2
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

struct DecArgsTc {
  CellPtrs ud;
  int64_t m, t0, tl, tiles_per_cell, total_tiles, tiles_per_cta;
  int tb_per_head;
  int rt, rd, factor_dtype;
  const uint32_t* arows;  // per cell: A = (diag(scale) Pi)^T in two bf16 terms [cell][term][128][d/2]
  const float* tmp;       // [cell][m * tl][rdm] fp32 Tucker row term
};

template <int D, int RDM, int BITS, int NS>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_decode_kernel(const __grid_constant__ TmaMaps cmaps, const __grid_constant__ TmaMaps omaps,
                     const __grid_constant__ DecArgsTc A) {
  constexpr int CB = D * BITS / 8;  // code bytes per row
  using L = DecLayout<D, CB, NS>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NS;
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint64_t* afree = acce + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile_begin = (int64_t)blockIdx.x * A.tiles_per_cta;
  const int64_t tile_end = tile_begin + A.tiles_per_cta < A.total_tiles ? tile_begin + A.tiles_per_cta
                                                                       : A.total_tiles;
  const int n_my = (int)(tile_end > tile_begin ? tile_end - tile_begin : 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);
      mbar_init(&full[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], NEPI);
      mbar_init(&afree[i], 1);  // tcgen05.commit after the last MMA reading an A buffer
    }
    mbar_fence_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tm_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tm_holder;

  if (warp < 4) {
    // codes (dense rows of CB bytes) -> exact integers in bf16 -> swizzled B tile;
    // at a cell change, the cell's A rows into the free TMEM buffer
    constexpr int LPR = CB / 16 > 0 ? CB / 16 : 1;  // lanes per row, 16 code bytes each
    constexpr int RPI = 32 / LPR;                   // rows per warp iteration
    constexpr int NIT = 32 / RPI;
    constexpr int PER = 8 / BITS;   // codes per byte
    constexpr int VALS = 16 * PER;  // values per lane
    static_assert(CB % 16 == 0, "code rows must be whole 16-byte chunks");
    const int pos = lane % LPR, sub = lane / LPR;
    // a code byte b placed in the mantissa of 2^23 reads 2^23 + b; subtracting
    // 2^23 + offset leaves the signed code exactly
    const float bias = 8388608.0f + (float)(1 << (BITS - 1));
    const uint64_t NB2 = f2_pack(-bias, -bias);
    int cur_cell = -1, seq = -1;
    for (int it = 0; it < n_my; ++it) {
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int st = it % NS;
      if (cell != cur_cell) {
        ++seq;
        const int b = seq & 1;
        // the MMAs of the cell two changes back read this buffer last
        if (seq >= 2 && !warp_wait(&afree[b], (uint32_t)(((seq - b) / 2 - 1) & 1), 0x161)) break;
        tc_fence_after();
        load_a_rows<D / 2>(tmem + ((uint32_t)(warp * 32) << 16), (uint32_t)(b * D),
                           A.arows + (size_t)cell * 2 * 128 * (D / 2), 2, warp * 32 + lane, 128);
        cur_cell = cell;
      }
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x141)) break;
      const uint8_t* Cs = smem + L::OFF_C + st * L::C_BYTES;
      uint8_t* Bs = smem + st * L::B_BYTES;
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
          *reinterpret_cast<uint4*>(Bs + sw128_off(rloc, pos * VALS + cb * 8, TILE_M)) =
              make_uint4(o[4 * cb], o[4 * cb + 1], o[4 * cb + 2], o[4 * cb + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&full[st]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      for (int it = 0; it < n_my; ++it) {
        const int64_t g = tile_begin + it;
        const int cell = (int)(g / A.tiles_per_cell);
        const int64_t tile = g % A.tiles_per_cell;
        const int h = (int)(tile / A.tb_per_head);
        const int tok = (int)(A.t0 + (tile % A.tb_per_head) * TILE_M);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x151)) break;
        mbar_expect_tx(&loaded[st], L::C_BYTES);
        tma_load_3d(sbase + L::OFF_C + st * L::C_BYTES, &cmaps.m[cell], 0, tok, h, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, TILE_M, true);
      int it = 0, cur_cell = -1, seq = -1;
      for (; it < n_my; ++it) {
        const int cell = (int)((tile_begin + it) / A.tiles_per_cell);
        if (cell != cur_cell) {
          if (seq >= 0) umma_commit(&afree[seq & 1]);  // releases the old buffer when its MMAs finish
          ++seq;
          cur_cell = cell;
        }
        const int st = it % NS, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x211)) break;
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x212)) break;
        tc_fence_after();
        const uint32_t b_base = sbase + st * L::B_BYTES;
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * TILE_M);
        const uint32_t a_base = tmem + (uint32_t)((seq & 1) * D);
#pragma unroll
        for (int term = 0; term < 2; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t kb = (uint32_t)((ks >> 2) * (TILE_M * 128) + (ks & 3) * 32);
            umma_f16_ts(d_tmem, a_base + (uint32_t)(term * (D / 2) + ks * 8), desc_sw128(b_base + kb), idesc,
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
    // ---------------- epilogue: thread = output feature, 64 rows per tile ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int feat = lg * 32 + lane;
    const bool active = lg * 32 < D;
    uint8_t* ost = smem + L::OFF_O + e * 2 * L::O_BUF;
    float* rst = reinterpret_cast<float*>(smem + L::OFF_R) + e * 64;  // this warp's 64 Tucker row terms
    float u[RDM];
#pragma unroll
    for (int r = 0; r < RDM; ++r) u[r] = 0.f;
    int cur_cell = -1;
    for (int it = 0; it < n_my; ++it) {
      const int ac = it & 1;
      const int64_t g = tile_begin + it;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      const int h = (int)(tile / A.tb_per_head);
      const int64_t i0 = (tile % A.tb_per_head) * TILE_M + half * 64;  // first token (within [t0, t1)) of this half
      if (cell != cur_cell) {
        if (A.rt > 0 && active)
#pragma unroll
          for (int r = 0; r < RDM; ++r)
            u[r] = r < A.rd ? load_dt(A.ud.p[cell], (int64_t)feat * A.rd + r, A.factor_dtype) : 0.f;
        cur_cell = cell;
      }
      // Tucker row terms of the 64 rows (rd = 1): one row per lane, loaded
      // before the accumulator wait, shared through this warp's slots
      const float* tp = A.tmp + ((int64_t)cell * A.m * A.tl + (int64_t)h * A.tl) * RDM;
      float tl0 = 0.f, tl1 = 0.f;
      if (A.rt > 0 && RDM == 1) {
        if (i0 + lane < A.tl) tl0 = __ldg(tp + i0 + lane);
        if (i0 + 32 + lane < A.tl) tl1 = __ldg(tp + i0 + 32 + lane);
      }
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x311)) break;
      tc_fence_after();
      uint8_t* buf = ost + (it & 1) * L::O_BUF;
      if (active) {
        if (lane == 0) bulk_wait_read<1>();
        rst[lane] = tl0;
        rst[32 + lane] = tl1;
        __syncwarp();
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * TILE_M + half * 64 + cc * 32), v);
        if (!active) continue;
        uint16_t* ob = reinterpret_cast<uint16_t*>(buf) + cc * 32 * 32 + lane;
        if (A.rt > 0 && RDM == 1) {
          // out = bf16(fl(t * u) + v): the reference adds the fp32 Tucker
          // reconstruction to the fp32 decoded residual
          const float4* t4 = reinterpret_cast<const float4*>(rst + cc * 32);
          const uint64_t U2 = f2_pack(u[0], u[0]);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 t = t4[q];
            float o0, o1, o2, o3;
            f2_unpack(f2_add(f2_mul(f2_pack(t.x, t.y), U2), f2_pack(v[4 * q], v[4 * q + 1])), o0, o1);
            f2_unpack(f2_add(f2_mul(f2_pack(t.z, t.w), U2), f2_pack(v[4 * q + 2], v[4 * q + 3])), o2, o3);
            ob[(4 * q) * 32] = __bfloat16_as_ushort(__float2bfloat16_rn(o0));
            ob[(4 * q + 1) * 32] = __bfloat16_as_ushort(__float2bfloat16_rn(o1));
            ob[(4 * q + 2) * 32] = __bfloat16_as_ushort(__float2bfloat16_rn(o2));
            ob[(4 * q + 3) * 32] = __bfloat16_as_ushort(__float2bfloat16_rn(o3));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float o = v[j];
            if (A.rt > 0) {
              const int64_t i = i0 + cc * 32 + j;
              float rec = 0.f;
              if (i < A.tl)
#pragma unroll
                for (int r = 0; r < RDM; ++r) rec = fmaf(__ldg(tp + i * RDM + r), u[r], rec);
              o = __fadd_rn(rec, v[j]);
            }
            ob[j * 32] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
          }
        }
      }
      if (active) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (i0 < A.tl) tma_store_3d(&omaps.m[cell], lg * 32, (int)i0, h, smem_u32(buf));
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// A rows of the decode, per cell: A[n][k] = scale[k] * Pi[k][n] in two bf16
// terms as 32-bit pairs [cell][term][n < 128][d / 2]; rows n >= d are zero.
__global__ void prep_decode_kernel(const float* __restrict__ proj, CellPtrs scale, int d, uint32_t* out) {
  const int cell = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // (n, w) over 128 x d/2
  const int wpr = d / 2;
  if (e >= 128 * wpr) return;
  const int n = e / wpr, w = e % wpr;
  const float* sc = static_cast<const float*>(scale.p[cell]);
  float r0 = 0.f, r1 = 0.f;
  if (n < d) {
    r0 = __fmul_rn(sc[2 * w], proj[(int64_t)(2 * w) * d + n]);
    r1 = __fmul_rn(sc[2 * w + 1], proj[(int64_t)(2 * w + 1) * d + n]);
  }
  uint32_t* base = out + (size_t)cell * 2 * 128 * wpr;
  for (int term = 0; term < 2; ++term) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(r0, r1);
    r0 -= __low2float(h);
    r1 -= __high2float(h);
    base[((size_t)term * 128 + n) * wpr + w] = *reinterpret_cast<const uint32_t*>(&h);
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
  const int64_t rows_pad = ceil_div(rows, TILE_M) * TILE_M;
  return align256((size_t)3 * 128 * (d / 2) * 4) + align256((size_t)n_cells * 2 * d * sizeof(int32_t)) +
         align256((size_t)n_cells * rows_pad * rdm_enc(rd) * 4);
}

int tc_residual_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                       const void* const* core, const void* const* u_token, const void* const* u_feature,
                       int rt, int rd, const float* proj, int bits, int symmetric, int scale_mode,
                       int stat_dtype, int arith_dtype, float* const* scale, int32_t* const* zp,
                       uint8_t* const* codes, void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (!workspace || ws_bytes < tc_residual_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core residual: workspace too small");
  const int64_t rows = m * t;
  const int rdm = rdm_enc(rd);
  if (ceil_div(rows, TILE_M) * TILE_M * rdm >= (1LL << 31))
    return fail(KVC_ERR_SHAPE, "tensor-core residual: too many rows per cell");
  TmaMaps xmaps, cmaps;  // copied into the launch parameters
  EncArgs a;
  memset(&a, 0, sizeof(a));
  memset(&cmaps, 0, sizeof(cmaps));
  const int cb = (d * bits + 7) / 8;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)d * 2};
    const uint32_t box[2] = {64u, (uint32_t)TILE_M};
    if ((rc = encode_tma(&xmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (mode == 1 && bits > 2) {
      // codes of 64 rows x 32 features: 4 * bits bytes per row
      const uint64_t cd[2] = {(uint64_t)cb, (uint64_t)rows};
      const uint64_t cs[1] = {(uint64_t)cb};
      const uint32_t cbx[2] = {(uint32_t)(4 * bits), 64u};
      if ((rc = encode_tma(&cmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, codes[c], cd, cs, cbx,
                           CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    }
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
  a.code_bytes = cb;
  a.tiles_per_cell = ceil_div(rows, TILE_M);
  a.total_tiles = a.tiles_per_cell * n_cells;
  const int64_t ctas = std::min<int64_t>(a.total_tiles, num_sms());
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* arows = reinterpret_cast<uint32_t*>(ws);
  size_t off = align256((size_t)3 * 128 * (d / 2) * 4);
  int32_t* mm = reinterpret_cast<int32_t*>(ws + off);
  off += align256((size_t)n_cells * 2 * d * sizeof(int32_t));
  float* tmp = reinterpret_cast<float*>(ws + off);
  a.arows = arows;
  a.minmax = mm;
  a.tmp = tmp;
  prep_rotation_kernel<<<(128 * (d / 2) + 255) / 256, 256, 0, st>>>(proj, d, arows);
  if ((rc = check_launch("prep_rotation_kernel"))) return rc;
  if (rt > 0) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows * rdm, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(cp, up, KVC_BF16, KVC_BF16, m, 0, t, rt, rd, rdm,
                                                              a.tiles_per_cell * TILE_M, tmp);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  if (mode == 0) {
    minmax_init_kernel<<<(n_cells * 2 * d + 255) / 256, 256, 0, st>>>(mm, n_cells, d);
    if ((rc = check_launch("minmax_init_kernel"))) return rc;
  }
#define KVC_TC_ENC(DD, MODEV, SYMV, RR, NSV)                     \
  do {                                                           \
    auto kern = tc_encode_kernel<DD, MODEV, SYMV, RR, NSV>;      \
    constexpr size_t sm = EncLayout<DD, RR, NSV, MODEV>::BYTES;  \
    if ((rc = set_smem(kern, sm))) return rc;                    \
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, cmaps, a);           \
  } while (0)
#define KVC_TC_ENC_R(DD, MODEV, SYMV, NSV)              \
  do {                                                  \
    if (rdm == 1) KVC_TC_ENC(DD, MODEV, SYMV, 1, NSV);  \
    else KVC_TC_ENC(DD, MODEV, SYMV, 4, NSV);           \
  } while (0)
  const bool sym = symmetric != 0;
  if (mode == 0) {
    if (d == 128) {
      if (sym) KVC_TC_ENC_R(128, MODE_STATS, true, 6);
      else KVC_TC_ENC_R(128, MODE_STATS, false, 6);
    } else {
      if (sym) KVC_TC_ENC_R(64, MODE_STATS, true, 8);
      else KVC_TC_ENC_R(64, MODE_STATS, false, 8);
    }
  } else {
    if (d == 128) {
      if (sym) KVC_TC_ENC_R(128, MODE_QUANT, true, 5);
      else KVC_TC_ENC_R(128, MODE_QUANT, false, 5);
    } else {
      if (sym) KVC_TC_ENC_R(64, MODE_QUANT, true, 8);
      else KVC_TC_ENC_R(64, MODE_QUANT, false, 8);
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
  return align256((size_t)n_cells * 2 * 128 * (d / 2) * 4) + align256((size_t)n_cells * rows * rdm_dec(rd) * 4);
}

int tc_decompress_launch(int n_cells, const uint8_t* const* codes, const float* const* scale, int bits,
                         const void* const* core, const void* const* u_token, const void* const* u_feature,
                         int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd, const float* proj,
                         int64_t t0, int64_t t1, void* const* out, void* workspace, size_t ws_bytes,
                         cudaStream_t st) {
  if (!workspace || ws_bytes < tc_decompress_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core decompress: workspace too small");
  const int64_t tl = t1 - t0;
  const int rdm = rdm_dec(rd);
  if (t >= (1LL << 31) || m * tl * rdm >= (1LL << 31) || ceil_div(tl, TILE_M) * m >= (1LL << 31))
    return fail(KVC_ERR_SHAPE, "tensor-core decompress: shape too large");
  TmaMaps cmaps, omaps;
  DecArgsTc a;
  memset(&a, 0, sizeof(a));
  CellPtrs sc;
  const int cb = d * bits / 8;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[3] = {(uint64_t)cb, (uint64_t)t, (uint64_t)m};
    const uint64_t strides[2] = {(uint64_t)cb, (uint64_t)cb * t};
    const uint32_t box[3] = {(uint32_t)cb, (uint32_t)TILE_M, 1u};
    if ((rc = encode_tma(&cmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, codes[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    // output (m, tl, d) bf16: boxes of 32 features x 64 tokens
    const uint64_t od[3] = {(uint64_t)d, (uint64_t)tl, (uint64_t)m};
    const uint64_t os[2] = {(uint64_t)d * 2, (uint64_t)d * 2 * tl};
    const uint32_t ob[3] = {32u, 64u, 1u};
    if ((rc = encode_tma(&omaps.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out[c], od, os, ob,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    sc.p[c] = scale[c];
    if (rt > 0) a.ud.p[c] = u_feature[c];
  }
  a.m = m;
  a.t0 = t0;
  a.tl = tl;
  a.tb_per_head = (int)ceil_div(tl, TILE_M);
  a.tiles_per_cell = m * a.tb_per_head;
  a.total_tiles = a.tiles_per_cell * n_cells;
  const int64_t ctas = std::min<int64_t>(a.total_tiles, num_sms());
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  a.rt = rt;
  a.rd = rd;
  a.factor_dtype = factor_dtype;
  uint32_t* arows = static_cast<uint32_t*>(workspace);
  float* tmp = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                        align256((size_t)n_cells * 2 * 128 * (d / 2) * 4));
  a.arows = arows;
  a.tmp = tmp;
  prep_decode_kernel<<<dim3((128 * (d / 2) + 255) / 256, n_cells), 256, 0, st>>>(proj, sc, d, arows);
  if ((rc = check_launch("prep_decode_kernel"))) return rc;
  if (rt > 0) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(m * tl * rdm, 256), 1024));
    tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(cp, up, factor_dtype, KVC_F32, m, t0, tl, rt, rd, rdm,
                                                              m * tl, tmp);
    if ((rc = check_launch("tucker_rows_kernel"))) return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
#define KVC_TC_DEC3(DD, RR, BB)                                      \
  do {                                                               \
    auto kern = tc_decode_kernel<DD, RR, BB, 3>;                     \
    using LL = DecLayout<DD, DD * BB / 8, 3>;                        \
    if ((rc = set_smem(kern, LL::BYTES))) return rc;                 \
    kern<<<grid, NTHREADS, LL::BYTES, st>>>(cmaps, omaps, a);        \
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
