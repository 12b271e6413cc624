// Tensor-core (tcgen05 / TMEM, TMA-fed) kernels for the residual encode and
// the fused decode, bf16 caches with head_dim 64 or 128 and fp32 caches with
// head_dim 64 (tc_enc32_kernel; the decode's fp32 output mode).
//
// All three are persistent, warp-specialised kernels (448 threads, one CTA
// per SM) over 128-row tiles of a cell:
//   warp 5     TMA: one thread loads each tile into a ring of NS stages
//   warps 0-3  transform, one row per thread
//   warp 4     one thread issues tcgen05.mma into one of two accumulators
//   warps 6-13 epilogue: two warps per TMEM lane group, one half each
//
// Stats pass (tc_stats_kernel), feature-major: A = Pi (rows = output
// features) in three bf16 terms (hi + mid + lo = Pi to fp32 precision) sits
// in TMEM, B = R = x - recon is the shared-memory tile, so TMEM lane = output
// feature and a thread keeps its feature's |max| (or min / max) in a register
// (kvcompress/compressor/residual.py:201-239).
//
// Quantise pass (tc_quant_kernel) and decode (tc_decode_kernel), row-major:
// the transform writes the tile's rows into a TMEM A buffer (double-buffered)
// with tcgen05.st and frees its TMA stage at once; the constant operand is
// the shared-memory B image.  TMEM lane = row, so an epilogue thread owns the
// contiguous outputs of one row and stores them with 16-byte stores, with no
// staging through shared memory.
//   quantise: B = Pi in three bf16 terms; codes packed in registers.
//   decode:   A = the codes as exact bf16 integers, B = diag(scale) Pi of the
//             cell in two bf16 terms (bulk-loaded at each cell change); the
//             epilogue adds the fp32 Tucker term and rounds to bf16
//             (kvcompress/compressor/jolt.py:424-463, residual.py:242-288).
//
// TMEM holds an A tile as one row per lane with two 16-bit elements per
// 32-bit column (element 2w in the low half).
//
// Every mbarrier wait is bounded (kvc_tc.cuh) and warp-uniform: a warp
// whose wait times out leaves its loop as a whole, so the others time out
// in turn and the kernel returns with the error word set.
#include <algorithm>
#include <type_traits>

#include "kvc_common.cuh"
#include "kvc_plan.cuh"
#include "kvc_quant.cuh"
#include "kvc_sched.cuh"
#include "kvc_tc.cuh"
#include "kvc_tma.cuh"

namespace kvc {
int kernel_policy();
namespace {

using namespace tc;

constexpr int TILE_M = 128;  // rows per tile (the MMA N)
constexpr int NTHREADS = 448;
constexpr int MMA_WARP = 4;
constexpr int TMA_WARP = 5;
constexpr int EPI_WARP0 = 6;
constexpr int NEPI = 256;  // epilogue threads
// the stats pass: transform warps 0-3 and 10-13 (two per TMEM lane group,
// one feature half each), epilogue warps 6-9
constexpr int STATS_XF_WARP1 = 10;
constexpr int RD_MAX = 16;
constexpr uint32_t TM_ACC = 256;  // TMEM column of accumulator 0 (1 at +128)
constexpr int CORE_MAX = 64;      // heads per cell whose row terms the encode forms in the kernel

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

// A row's RDM Tucker row terms from shared memory into registers.
template <int RDM>
__device__ __forceinline__ void load_row_terms(const float* ts, float (&tv)[RDM]) {
#pragma unroll
  for (int g = 0; g < RDM / 4; ++g) {
    const float4 t4 = reinterpret_cast<const float4*>(ts)[g];
    tv[4 * g] = t4.x;
    tv[4 * g + 1] = t4.y;
    tv[4 * g + 2] = t4.z;
    tv[4 * g + 3] = t4.w;
  }
}

// The Tucker reconstruction of one element before its bf16 rounding:
// sum_r t[r] u[r] in the order r = 0, 1, .. (the fp32 order of the SIMT
// residual), u the feature's RDM entries of u_feature.
template <int RDM>
__device__ __forceinline__ float recon_dot(const float (&tv)[RDM], const float4* u) {
  float4 q = u[0];
  float rec = tv[0] * q.x;
  rec = fmaf(tv[1], q.y, rec);
  rec = fmaf(tv[2], q.z, rec);
  rec = fmaf(tv[3], q.w, rec);
#pragma unroll
  for (int g = 1; g < RDM / 4; ++g) {
    q = u[g];
    rec = fmaf(tv[4 * g], q.x, rec);
    rec = fmaf(tv[4 * g + 1], q.y, rec);
    rec = fmaf(tv[4 * g + 2], q.z, rec);
    rec = fmaf(tv[4 * g + 3], q.w, rec);
  }
  return rec;
}

// ------------------------------------------------------------------------
// residual encode, stats pass: feature-major, one thread per output feature
// ------------------------------------------------------------------------

template <int D, int RDM, int NS, bool F16 = false>
struct StatsLayout {
  static constexpr int NTERM = F16 ? 2 : 3;                       // terms of Pi in TMEM
  static constexpr uint32_t B_BYTES = TILE_M * D * 2;             // R tile (MMA B operand)
  static constexpr uint32_t T_BYTES = TILE_M * RDM * 4;           // Tucker row term of a tile
  static constexpr uint32_t U_BYTES = RDM == 1 ? D : D * RDM * 2;  // per transform warp, its D/2 features of
                                                              // u_feature: bf16 [j] or fp32 [j][4]
  static constexpr uint32_t OFF_T = NS * B_BYTES;
  static constexpr uint32_t OFF_U = OFF_T + NS * T_BYTES;
  static constexpr uint32_t OFF_CORE = OFF_U + 8 * U_BYTES;  // per transform warp: core[h] of the cell
  static constexpr uint32_t OFF_RING = OFF_CORE + 8 * CORE_MAX * 4;  // tile ids drawn by the producer
  static constexpr uint32_t OFF_TE = OFF_RING + sched::RING * 4;          // fp16 mode: E of each tile (ring)
  static constexpr uint32_t OFF_WM = OFF_TE + (F16 ? sched::RING * 4 : 0);  // fp16 mode: [2][8] warp maxima
  static constexpr uint32_t OFF_BAR = OFF_WM + (F16 ? 64 : 0);
  // loaded, full, empty, acc full x2, acc empty x2 (+ fp16 mode: tile max x2)
  static constexpr uint32_t NBAR = 3 * NS + 4 + (F16 ? 2 : 0);
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
  // rows_direct (rt = rd = 1, T a multiple of 128, at most CORE_MAX heads,
  // 16-byte aligned u_token): a tile's row terms bf16(core[h] * u_token[t])
  // are formed in the kernel from a 256-byte bulk copy of u_token and the
  // cell's core[] kept in shared memory, instead of from tmp
  CellPtrs core, ut;
  int64_t t_tok;  // tokens per head
  int rows_direct;
  // STATS: [cell] the float bits of max |R| (atomicMax; for the fp16
  // quantise mode); QUANT (fp16 mode): [cell][1 + d] = 2^E (R's scale), then
  // per output feature n the epilogue's factor 2^-(E + G_n)
  uint32_t* rmax;
  const float* fscale;
  // STATS (fp16 mode): G_n of the A rows Pi[n][.] * 2^G_n
  const int32_t* gexp;
  // STATS (fp16 mode): [cell] E, R's scale 2^E from a bound on |R| known
  // before the pass (stats_bound_kernel), or NULL: per 128-row tile
  const int32_t* sexp;
};

// Bits of the bf16 Tucker term of a tile's row ptid (rd = 1): from the
// stage's row-term window, or (rows_direct) bf16(core[h] * u_token[t]) from
// the stage's u_token copy and the warp's core[] table, the exact bf16
// product rounded once as the row-term kernel rounds it.  row0: the tile's
// first row in the cell.
__device__ __forceinline__ uint32_t enc_row_term(const EncArgs& A, const uint8_t* tslot, const float* cs, int ptid,
                                                 int64_t row0) {
  // rows of a cell stay below 2^31 (checked by the launcher): 32-bit division
  const float v = A.rows_direct ? cs[(uint32_t)row0 / (uint32_t)A.t_tok] * load_dt(tslot, ptid, KVC_BF16)
                                : reinterpret_cast<const float*>(tslot)[ptid];
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

template <int D, bool SYM, int RDM, int NS, bool F16 = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_stats_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ EncArgs A) {
  static_assert(!F16 || RDM == 1, "the fp16 mode takes rank-1 row terms");
  using L = StatsLayout<D, RDM, NS, F16>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NS;
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint64_t* tbar = acce + 2;  // fp16 mode: the transform warps' maxima of a tile are in
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  int32_t* texp = reinterpret_cast<int32_t*>(smem + L::OFF_TE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);  // TMA issue + transaction bytes
      mbar_init(&full[i], 256);  // transform threads
      mbar_init(&empty[i], 1);   // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);     // tcgen05.commit
      mbar_init(&acce[i], 128);   // epilogue threads
      if (F16) mbar_init(&tbar[i], 8);  // one arrive per transform warp
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
  if (warp < 4) load_a_rows<D / 2>(tmem + ((uint32_t)(warp * 32) << 16), 0, A.arows, L::NTERM, warp * 32 + lane, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp < 4 || warp >= STATS_XF_WARP1) {
    // ---------------- transform: R = x - recon, in place, one row per thread ----------------
    // two warps per row block: warp w takes rows (w % 4) * 32.. and feature half `part`
    constexpr int HF = D / 2, HC = HF / 8;  // features and 16-byte chunks per part
    const int lgw = warp & 3, part = warp < 4 ? 0 : 1;
    const int ptid = lgw * 32 + lane;
    float* u32 = reinterpret_cast<float*>(smem + L::OFF_U + (part * 4 + lgw) * L::U_BYTES);       // [j][4]
    uint16_t* ub = reinterpret_cast<uint16_t*>(smem + L::OFF_U + (part * 4 + lgw) * L::U_BYTES);  // [j]
    float* cs = reinterpret_cast<float*>(smem + L::OFF_CORE) + (part * 4 + lgw) * CORE_MAX;     // [h]
    int cur_cell = -1;
    int ecell = 0;  // fp16 mode with a per-cell bound: E of the cell
    for (int it = 0;; ++it) {
      const int st = it % NS;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x131)) break;
      const int32_t g = sched::ring_get(ring, it);
      if (g < 0) {  // no more tiles: pass the end on to the MMA thread
        mbar_arrive(&full[st]);
        break;
      }
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      if (A.rt > 0 && cell != cur_cell) {
        __syncwarp();
        const __nv_bfloat16* ud = static_cast<const __nv_bfloat16*>(A.ud.p[cell]);
        if (RDM == 1) {
          for (int j = lane; j < HF; j += 32) ub[j] = reinterpret_cast<const uint16_t*>(ud)[part * HF + j];
        } else {
          for (int i = lane; i < HF * RDM; i += 32) {
            const int j = i / RDM, r = i % RDM;
            u32[i] = r < A.rd ? __bfloat162float(ud[(part * HF + j) * A.rd + r]) : 0.f;
          }
        }
        if (A.rows_direct)
          for (int j = lane; j < (int)(A.rows / A.t_tok); j += 32) cs[j] = load_dt(A.core.p[cell], j, KVC_BF16);
        if (F16 && A.sexp) ecell = A.sexp[cell];
        __syncwarp();
        cur_cell = cell;
      }
      if constexpr (F16) {
        if (A.sexp) {
          // R * 2^E with E of the cell (its bound puts |R| 2^E below 2^14):
          // no agreement between the warps is needed
          uint8_t* Bs = smem + st * L::B_BYTES;
          uint32_t mh = 0u;  // max of the bf16 magnitude bits (both halves)
          if (row < A.rows) {
            const uint32_t th = enc_row_term(A, smem + L::OFF_T + st * L::T_BYTES, cs, ptid, row - ptid);
            const uint32_t t2 = th | (th << 16);
            const uint4* u4 = reinterpret_cast<const uint4*>(ub);
            const int e1 = min(max(ecell, -100), 100), e2 = ecell - e1;
            const uint32_t f1 = (uint32_t)(e1 + 127) << 7, f2 = (uint32_t)(e2 + 127) << 7;
            const uint32_t p1 = f1 | (f1 << 16), p2 = f2 | (f2 << 16);
#pragma unroll
            for (int c = 0; c < HC; ++c) {
              uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
              const uint4 x = *slot;
              const uint4 u = u4[c];
              uint32_t w[4] = {bf16x2_sub(x.x, bf16x2_mul(t2, u.x)), bf16x2_sub(x.y, bf16x2_mul(t2, u.y)),
                               bf16x2_sub(x.z, bf16x2_mul(t2, u.z)), bf16x2_sub(x.w, bf16x2_mul(t2, u.w))};
              mh = __vmaxu2(mh, __vmaxu2(__vmaxu2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                         __vmaxu2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu)));
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint32_t v = bf16x2_mul(w[i], p1);
                if (e2 != 0) v = bf16x2_mul(v, p2);
                const __half2 h2 = __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
                w[i] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              *slot = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          const uint32_t wm = __reduce_max_sync(0xffffffffu, max(mh & 0xFFFFu, mh >> 16));
          if (lane == 0 && A.rmax && wm) atomicMax(A.rmax + cell, wm << 16);
          if (warp == 0 && lane == 0) *reinterpret_cast<volatile int32_t*>(&texp[it % sched::RING]) = ecell;
          fence_async_smem();
          mbar_arrive(&full[st]);
          continue;
        }
        // fp16 mode: this thread's half row of R stays in registers until the
        // tile's max |R| is known; then R * 2^E, E putting that max in
        // [2^13, 2^14), goes to the B tile in fp16: exact for every bf16
        // value above 2^-14 of the scaled range (smaller ones are below the
        // fp32 resolution of the rotated values).  Rows past the end stay 0.
        uint8_t* Bs = smem + st * L::B_BYTES;
        const bool valid = row < A.rows;  // the launcher takes this mode with rt > 0 only
        uint32_t r[HC * 4];
        uint32_t mh = 0u;  // max of the bf16 magnitude bits (both halves)
        if (valid) {
          const uint32_t th = enc_row_term(A, smem + L::OFF_T + st * L::T_BYTES, cs, ptid, row - ptid);
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            const uint4 x = *reinterpret_cast<const uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
            const uint4 u = u4[c];
            r[4 * c] = bf16x2_sub(x.x, bf16x2_mul(t2, u.x));
            r[4 * c + 1] = bf16x2_sub(x.y, bf16x2_mul(t2, u.y));
            r[4 * c + 2] = bf16x2_sub(x.z, bf16x2_mul(t2, u.z));
            r[4 * c + 3] = bf16x2_sub(x.w, bf16x2_mul(t2, u.w));
            mh = __vmaxu2(mh, __vmaxu2(__vmaxu2(r[4 * c] & 0x7FFF7FFFu, r[4 * c + 1] & 0x7FFF7FFFu),
                                       __vmaxu2(r[4 * c + 2] & 0x7FFF7FFFu, r[4 * c + 3] & 0x7FFF7FFFu)));
          }
        }
        const uint32_t wm = __reduce_max_sync(0xffffffffu, max(mh & 0xFFFFu, mh >> 16));
        uint32_t* wmax = reinterpret_cast<uint32_t*>(smem + L::OFF_WM) + (it & 1) * 8;
        if (lane == 0) {
          wmax[part * 4 + lgw] = wm;
          if (A.rmax && wm) atomicMax(A.rmax + cell, wm << 16);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tbar[it & 1]);
        if (!warp_wait(&tbar[it & 1], (uint32_t)((it >> 1) & 1), 0x132)) break;
        uint32_t tmx = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) tmx = max(tmx, wmax[i]);
        // tmx: bf16 magnitude bits of the tile's max |R| (a subnormal max
        // counts as 2^-126); E in [-114, 139]
        const int E = tmx ? 13 - max((int)(tmx >> 7) - 127, -126) : 0;
        if (warp == 0 && lane == 0) *reinterpret_cast<volatile int32_t*>(&texp[it % sched::RING]) = E;
        if (valid) {
          // 2^E as two bf16 factors (each product exact)
          const int e1 = min(max(E, -100), 100), e2 = E - e1;
          const uint32_t f1 = (uint32_t)(e1 + 127) << 7, f2 = (uint32_t)(e2 + 127) << 7;
          const uint32_t p1 = f1 | (f1 << 16), p2 = f2 | (f2 << 16);
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            uint32_t h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t w = bf16x2_mul(r[4 * c + i], p1);
              if (e2 != 0) w = bf16x2_mul(w, p2);
              const __half2 h2 = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
              h[i] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M)) =
                make_uint4(h[0], h[1], h[2], h[3]);
          }
        }
        fence_async_smem();
        mbar_arrive(&full[st]);
        continue;
      }
      uint32_t rm = 0u;  // float bits of this thread's max |R| (monotonic for non-negative floats)
      if (A.rt > 0 && row < A.rows) {
        uint8_t* Bs = smem + st * L::B_BYTES;
        const float* ts = reinterpret_cast<const float*>(smem + L::OFF_T + st * L::T_BYTES) + ptid * RDM;
        if (RDM == 1) {
          // rd == 1: recon = bf16(t * u_j) and R = bf16(x - recon), each a
          // single rounding of the exact bf16 product / difference
          const uint32_t th = enc_row_term(A, smem + L::OFF_T + st * L::T_BYTES, cs, ptid, row - ptid);
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
          uint32_t mh = 0u;  // max of the bf16 magnitude bits (both halves)
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
            uint4 x = *slot;
            const uint4 u = u4[c];
            x.x = bf16x2_sub(x.x, bf16x2_mul(t2, u.x));
            x.y = bf16x2_sub(x.y, bf16x2_mul(t2, u.y));
            x.z = bf16x2_sub(x.z, bf16x2_mul(t2, u.z));
            x.w = bf16x2_sub(x.w, bf16x2_mul(t2, u.w));
            *slot = x;
            mh = __vmaxu2(mh, __vmaxu2(__vmaxu2(x.x & 0x7FFF7FFFu, x.y & 0x7FFF7FFFu),
                                       __vmaxu2(x.z & 0x7FFF7FFFu, x.w & 0x7FFF7FFFu)));
          }
          rm = max(mh & 0xFFFFu, mh >> 16) << 16;
        } else {
          float tv[RDM];
          load_row_terms<RDM>(ts, tv);
          const float4* u4 = reinterpret_cast<const float4*>(u32);
#pragma unroll 2
          for (int c = 0; c < HC; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
            float xv[8];
            unpack8_bf16(*slot, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float rec = recon_dot<RDM>(tv, u4 + (c * 8 + e) * (RDM / 4));
              xv[e] = Elt<__nv_bfloat16>::round(xv[e] - Elt<__nv_bfloat16>::round(rec));
              rm = max(rm, __float_as_uint(fabsf(xv[e])));
            }
            *slot = pack8_bf16(xv);
          }
        }
      }
      if (A.rmax) {
        const uint32_t wm = __reduce_max_sync(0xffffffffu, rm);
        if (lane == 0 && wm) atomicMax(A.rmax + cell, wm);
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
  } else if (warp == TMA_WARP) {
    // ---------------- TMA producer: x tile (+ Tucker row term) ----------------
    if (lane == 0) {
      sched::Cursor cur(A.tiles_per_cta, A.total_tiles);
      for (int it = 0;; ++it) {
        const int64_t g = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)g);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x121)) break;
        if (g < 0) {  // the end: a plain arrive completes the stage with no bytes
          mbar_arrive(&loaded[st]);
          break;
        }
        const int cell = (int)(g / A.tiles_per_cell);
        const int y = (int)((g % A.tiles_per_cell) * TILE_M);
        mbar_expect_tx(&loaded[st], L::B_BYTES + (A.rt > 0 ? (A.rows_direct ? TILE_M * 2u : L::T_BYTES) : 0u));
        const uint32_t dst = sbase + st * L::B_BYTES;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * TILE_M * 128, &xmaps.m[cell], h * 64, y, &loaded[st]);
        if (A.rt > 0 && A.rows_direct)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    static_cast<const uint8_t*>(A.ut.p[cell]) + ((uint32_t)y % (uint32_t)A.t_tok) * 2u, TILE_M * 2u,
                    &loaded[st]);
        else if (A.rt > 0)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    A.tmp + ((int64_t)cell * A.tiles_per_cell * TILE_M + y) * RDM, L::T_BYTES, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer: D[feature][row] = sum_k Pi[feature][k] R[row][k] ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, TILE_M, !F16);
      int it = 0;
      bool ended = false;
      for (;; ++it) {
        const int st = it % NS, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x201)) break;
        const int32_t g = sched::ring_get(ring, it);
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x202)) break;
        if (g < 0) {  // the end: the epilogue learns it from the same accumulator barrier
          umma_commit(&accf[ac]);
          ended = true;
          break;
        }
        tc_fence_after();
        const uint32_t b_base = sbase + st * L::B_BYTES;
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * TILE_M);
#pragma unroll
        for (int term = 0; term < L::NTERM; ++term) {
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
      if (ended) mbar_wait(&accf[it & 1], (uint32_t)(it >> 1) & 1u, 0x203);
      else if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x203);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: thread = output feature, the tile's 128 rows ----------------
    // (warps 6-9, one per TMEM lane group)
    const int lg = warp & 3;
    const int feat = lg * 32 + lane;
    const bool active = lg * 32 < D;  // warp-uniform (d = 64 uses lane groups 0-1)
    float run_max = 0.f, rmin = __int_as_float(0x7f800000), rmax = -__int_as_float(0x7f800000);
    const int gn = F16 && active ? A.gexp[feat] : 0;  // fp16 mode: the accumulators hold R~ * 2^(E + G_n)
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
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x301)) break;
      const int32_t g = sched::ring_get(ring, it);
      if (g < 0) break;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      if (cell != cur_cell) {
        if (cur_cell >= 0) flush_stats(cur_cell);
        cur_cell = cell;
      }
      tc_fence_after();
      const int64_t row0 = tile * TILE_M;
      // fp16 mode: the tile's extremes in its scaled units, then exactly
      // rescaled (2^-(E + G_n))
      float t_abs = 0.f, t_min = __int_as_float(0x7f800000), t_max = -__int_as_float(0x7f800000);
      float& a_max = F16 ? t_abs : run_max;
      float& a_lo = F16 ? t_min : rmin;
      float& a_hi = F16 ? t_max : rmax;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * TILE_M + cc * 32), v);
        if (!active) continue;
        if (SYM) {
          // rows past the end hold R = 0 and cannot raise |max|
#pragma unroll
          for (int j = 0; j < 32; ++j) a_max = fmaxf(a_max, fabsf(v[j]));
        } else {
          const int64_t nvalid = A.rows - (row0 + cc * 32);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nvalid) {
              a_hi = fmaxf(a_hi, v[j]);
              a_lo = fminf(a_lo, v[j]);
            }
        }
      }
      if (F16 && active) {
        const int sh = -(*reinterpret_cast<const volatile int32_t*>(&texp[it % sched::RING]) + gn);
        if (SYM) {
          run_max = fmaxf(run_max, ldexpf(t_abs, sh));
        } else {
          rmax = fmaxf(rmax, ldexpf(t_max, sh));  // ldexpf keeps +-inf (an empty tile)
          rmin = fminf(rmin, ldexpf(t_min, sh));
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (cur_cell >= 0) flush_stats(cur_cell);
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

// The same row terms as one GEMM per head (u_token rows times core[h]) for
// larger rt: tiles of TR tokens x RDM columns, the rank axis in chunks of 32
// staged in shared memory; each thread accumulates CW columns of one token
// over a in order, the fmaf chain of tucker_rows_kernel, so both give the
// same bits.
template <int RDM>
__global__ void __launch_bounds__(256) tucker_rows_tiled_kernel(CellPtrs core, CellPtrs ut, int fdt, int round_dt_,
                                                                int64_t m, int64_t t0, int64_t tl, int rt, int rd,
                                                                int64_t cell_stride, float* tmp) {
  constexpr int CW = RDM >= 4 ? 4 : 1;  // columns per thread
  constexpr int RG = RDM / CW;          // column groups
  constexpr int TR = 256 / RG;          // tokens per tile
  constexpr int KA = 32;                // rank chunk
  __shared__ float us[TR][KA + 1];
  __shared__ __align__(16) float cs[KA][RDM];
  const int cell = blockIdx.y;
  const int ti = threadIdx.x / RG, g = threadIdx.x % RG;
  const int64_t per_head = (tl + TR - 1) / TR;
  for (int64_t tile = blockIdx.x; tile < m * per_head; tile += gridDim.x) {
    const int64_t h = tile / per_head, i0 = (tile - h * per_head) * TR;
    float acc[CW];
#pragma unroll
    for (int q = 0; q < CW; ++q) acc[q] = 0.f;
    for (int a0 = 0; a0 < rt; a0 += KA) {
      const int ka = min(KA, rt - a0);
      __syncthreads();  // the previous chunk is consumed
      for (int e = threadIdx.x; e < TR * KA; e += blockDim.x) {
        const int ii = e / KA, aa = e % KA;
        us[ii][aa] = (aa < ka && i0 + ii < tl) ? load_dt(ut.p[cell], (t0 + i0 + ii) * rt + a0 + aa, fdt) : 0.f;
      }
      for (int e = threadIdx.x; e < KA * RDM; e += blockDim.x) {
        const int aa = e / RDM, r = e % RDM;
        cs[aa][r] = (aa < ka && r < rd) ? load_dt(core.p[cell], (h * rt + a0 + aa) * rd + r, fdt) : 0.f;
      }
      __syncthreads();
      for (int aa = 0; aa < ka; ++aa) {
        const float u = us[ti][aa];
#pragma unroll
        for (int q = 0; q < CW; ++q) acc[q] = fmaf(cs[aa][g * CW + q], u, acc[q]);
      }
    }
    if (i0 + ti < tl) {
      float* o = tmp + ((int64_t)cell * cell_stride + h * tl + i0 + ti) * RDM + g * CW;
#pragma unroll
      for (int q = 0; q < CW; ++q) o[q] = g * CW + q < rd ? round_dt(acc[q], round_dt_) : 0.f;
    }
  }
}

int rdm_enc(int rd) { return rd <= 1 ? 1 : (rd <= 4 ? 4 : 16); }
int rdm_dec(int rd) { return rd <= 1 ? 1 : (rd <= 4 ? 4 : 16); }

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr int kMaxCtas = 1024;  // grid cap of the persistent kernels
constexpr int ROWTERM_TILED_RT = 8;  // rt from which the row terms take the tiled kernel

// tmp[cell][row][rdm] (cell_stride rows per cell) = the Tucker row terms of
// rows h * tl + i, tokens t0 + i (rdm 1, 4 or 16).
int row_terms_launch(const CellPtrs& core, const CellPtrs& ut, int n_cells, int fdt, int round_dt_, int64_t m,
                     int64_t t0, int64_t tl, int rt, int rd, int rdm, int64_t cell_stride, float* tmp,
                     cudaStream_t st) {
  if (rt >= ROWTERM_TILED_RT && (rdm == 1 || rdm == 4 || rdm == 16)) {
    const int rg = rdm >= 4 ? rdm / 4 : 1, tr = 256 / rg;
    const int64_t tiles = m * ((tl + tr - 1) / tr);
    const dim3 grid((unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, 8 * num_sms())), n_cells);
    if (rdm == 1)
      tucker_rows_tiled_kernel<1><<<grid, 256, 0, st>>>(core, ut, fdt, round_dt_, m, t0, tl, rt, rd, cell_stride, tmp);
    else if (rdm == 4)
      tucker_rows_tiled_kernel<4><<<grid, 256, 0, st>>>(core, ut, fdt, round_dt_, m, t0, tl, rt, rd, cell_stride, tmp);
    else
      tucker_rows_tiled_kernel<16><<<grid, 256, 0, st>>>(core, ut, fdt, round_dt_, m, t0, tl, rt, rd, cell_stride,
                                                         tmp);
    return check_launch("tucker_rows_tiled_kernel");
  }
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(m * tl * rdm, 256), 1024));
  tucker_rows_kernel<<<dim3(blocks, n_cells), 256, 0, st>>>(core, ut, fdt, round_dt_, m, t0, tl, rt, rd, rdm,
                                                            cell_stride, tmp);
  return check_launch("tucker_rows_kernel");
}

// min / max arrays to their identities (ordered ints of +inf / -inf).
__global__ void minmax_init_kernel(int32_t* mm, int n_cells, int d, uint32_t* rmax) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (rmax && i < n_cells) rmax[i] = 0u;
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

// E of each cell for the fp16 stats pass, from bounds known before it:
// |x| <= sqrt(max_j G_jj) (G the cell's feature Gram x^T x) and |recon| <=
// rt max|core| max|u_token| max|u_feature|, with a 10% margin for the
// roundings of the Gram and of the bf16 products; E = 13 - ilogb(bound), so
// |R| 2^E < 2^14.  A loose bound costs nothing: fp16 keeps every value
// exact down to 2^-14 of the scaled range.  One block per cell.
__global__ void stats_bound_kernel(const double* __restrict__ gram, int64_t gstride, int d, CellPtrs core,
                                   CellPtrs ut, CellPtrs ud, int64_t ncore, int64_t nut, int nud, int rt,
                                   int32_t* sexp) {
  __shared__ double red[4][32];
  const int cell = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const double* G = gram + cell * gstride;
  double m[4] = {0.0, 0.0, 0.0, 0.0};
  for (int i = threadIdx.x; i < d; i += blockDim.x) m[0] = fmax(m[0], G[(int64_t)i * d + i]);
  for (int64_t i = threadIdx.x; i < ncore; i += blockDim.x)
    m[1] = fmax(m[1], fabs((double)load_dt(core.p[cell], i, KVC_BF16)));
  for (int64_t i = threadIdx.x; i < nut; i += blockDim.x) m[2] = fmax(m[2], fabs((double)load_dt(ut.p[cell], i, KVC_BF16)));
  for (int i = threadIdx.x; i < nud; i += blockDim.x) m[3] = fmax(m[3], fabs((double)load_dt(ud.p[cell], i, KVC_BF16)));
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m[q] = fmax(m[q], __shfl_xor_sync(0xffffffffu, m[q], o));
    if (lane == 0) red[q][w] = m[q];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double r[4] = {0.0, 0.0, 0.0, 0.0};
    for (int q = 0; q < 4; ++q)
      for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) r[q] = fmax(r[q], red[q][i]);
    const double b = 1.1 * (sqrt(r[0]) + (double)rt * r[1] * r[2] * r[3]);
    int E = 0;
    if (b > 0.0 && isfinite(b)) E = 13 - ilogb(b);
    sexp[cell] = min(max(E, -200), 200);
  }
}

// A rows of the fp16 stats pass: Pi[m][k] * 2^G_m in two fp16 terms (hi +
// lo: 22 bits of each entry), G_m = 13 - ilogb(max_k |Pi[m][k]|), as 32-bit
// pairs [term][m < 128][d / 2]; gexp[m] = G_m.  One block of d / 2 threads
// per row m.
__global__ void prep_rotation16_kernel(const float* __restrict__ proj, int d, uint32_t* out, int32_t* gexp) {
  __shared__ float red[32];
  const int m = blockIdx.x, w = threadIdx.x, wpr = d / 2;
  const float r0 = m < d ? proj[m * d + 2 * w] : 0.f, r1 = m < d ? proj[m * d + 2 * w + 1] : 0.f;
  float mx = fmaxf(fabsf(r0), fabsf(r1));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((w & 31) == 0) red[w >> 5] = mx;
  __syncthreads();
  mx = 0.f;
  for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) mx = fmaxf(mx, red[i]);
  const int G = (mx > 0.f && isfinite(mx)) ? 13 - ilogbf(mx) : 0;
  const float b0 = ldexpf(r0, G), b1 = ldexpf(r1, G);
  const __half2 hi = __floats2half2_rn(b0, b1);
  const __half2 lo = __floats2half2_rn(b0 - __low2float(hi), b1 - __high2float(hi));
  out[(size_t)m * wpr + w] = *reinterpret_cast<const uint32_t*>(&hi);
  out[((size_t)128 + m) * wpr + w] = *reinterpret_cast<const uint32_t*>(&lo);
  if (w == 0) gexp[m] = G;
}

// B images of the quantise pass, per cell: B[n][k] = Pi[n][k] / s_n in three
// bf16 terms (hi + mid + lo, fp32 precision), swizzled K-major
// [cell][term][n][k], so that the MMA yields R~ / s directly (fold = 0 keeps
// Pi itself, for the per-tensor scales quantised in a 16-bit dtype).
__global__ void prep_quant_b_kernel(const float* __restrict__ proj, CellPtrs scale, int per_feature, int fold,
                                    int d, uint8_t* out) {
  const int cell = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= d * d) return;
  const int n = e / d, k = e % d;
  float rest = proj[e];
  if (fold) rest = __fdiv_rn(rest, static_cast<const float*>(scale.p[cell])[per_feature ? n : 0]);
  uint8_t* base = out + (size_t)cell * 3 * d * d * 2;
  for (int term = 0; term < 3; ++term) {
    const __nv_bfloat16 v = __float2bfloat16_rn(rest);
    rest -= __bfloat162float(v);
    *reinterpret_cast<__nv_bfloat16*>(base + (size_t)term * d * d * 2 + sw128_off(n, k, d)) = v;
  }
}

// The fp16 form of those B images (the quantise pass's fp16 mode, d = 128,
// per-channel scales, Tucker factors present).  Two fp16 terms hold a 22-bit
// split of Pi[n][k] / s_n * 2^G_n, G_n putting the row's largest magnitude
// in [2^13, 2^14); the rows R enter the MMA as fp16 scaled by 2^E, E from the
// cell's max |R| (the stats pass) the same way.  Both scalings are exact
// powers of two and fp16 x fp16 products are exact in fp32, so the
// epilogue's factor 2^-(E + G_n) gives R~ / s with an error below 2^-21 of
// the largest term.  One block per (row n, cell), one thread per k.
// rowfmt: the terms as TMEM A rows [cell][term][n < 128][d] (the
// feature-major pass) instead of swizzled B images.
__global__ void prep_quant_b16_kernel(const float* __restrict__ proj, CellPtrs scale,
                                      const uint32_t* __restrict__ rmax, int d, uint8_t* out, float* fscale,
                                      int rowfmt) {
  __shared__ float red[32];
  const int cell = blockIdx.y, n = blockIdx.x, k = threadIdx.x;
  const float v = k < d ? __fdiv_rn(proj[n * d + k], static_cast<const float*>(scale.p[cell])[n]) : 0.f;
  float m = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((k & 31) == 0) red[k >> 5] = m;
  __syncthreads();
  m = 0.f;
  for (int w = 0; w < (int)(blockDim.x + 31) / 32; ++w) m = fmaxf(m, red[w]);
  const int G = (m > 0.f && isfinite(m)) ? 13 - ilogbf(m) : 0;
  const float rm = __uint_as_float(rmax[cell]);
  const int E = (rm > 0.f && isfinite(rm)) ? 13 - ilogbf(rm) : 0;
  if (k < d) {
    const float b = ldexpf(v, G);
    const __half hi = __float2half_rn(b);
    const __half lo = __float2half_rn(b - __half2float(hi));
    uint8_t* base = out + (size_t)cell * 3 * d * d * 2;
    if (rowfmt) {
      __half* rows = reinterpret_cast<__half*>(base);
      rows[(size_t)n * d + k] = hi;
      rows[((size_t)128 + n) * d + k] = lo;
    } else {
      *reinterpret_cast<__half*>(base + sw128_off(n, k, d)) = hi;
      *reinterpret_cast<__half*>(base + (size_t)d * d * 2 + sw128_off(n, k, d)) = lo;
    }
  }
  if (k == 0) {
    fscale[(size_t)cell * (1 + d) + 1 + n] = ldexpf(1.f, -(E + G));
    if (n == 0) fscale[(size_t)cell * (1 + d)] = ldexpf(1.f, E);
  }
}

// Quantiser of the fused encode.  The reference computes
// q = rint(fl32(fl32(v / s) + zp)) (round half to even, then clamp), v the
// fp32 rotated residual.  Here 1/s is folded into the B image (Pi / s in
// three bf16 terms), so the accumulator already holds v / s to fp32
// precision; the epilogue adds zp and rounds with the magic constant: the
// float bits of y = t + 1.5 * 2^23 + offset are 0x4B400000 + offset + rint(t)
// (ties to even), clamped to the code range.  The per-tensor scale with a
// 16-bit arithmetic dtype keeps Pi unscaled and quantises each value with
// the reference's own steps (quantize_one).
// ------------------------------------------------------------------------
// quantise pass, row-major: A = R in TMEM (one row per lane), B = Pi in
// shared memory; thread = row in the epilogue, codes stored directly
// ------------------------------------------------------------------------
template <int D, int RDM, int NS, bool F16 = false>
struct QuantLayout {
  static constexpr int NTERM = F16 ? 2 : 3;
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_BYTES = NTERM * B_TERM;             // Pi / s of the cell in NTERM terms
  static constexpr uint32_t X_BYTES = TILE_M * D * 2;             // x tile (TMA, SWIZZLE_128B)
  static constexpr uint32_t T_BYTES = TILE_M * RDM * 4;           // Tucker row term of a tile
  static constexpr uint32_t U_BYTES = RDM == 1 ? D * 2 : D * 16;  // u_feature: bf16 [j] or fp32 [j][4]
  static constexpr uint32_t S_BYTES = (D / 2) * 4;                // per epilogue warp: zp of its D/2 features
  static constexpr uint32_t Q_BYTES = 32 * (D / 2);                // per epilogue warp: codes of 32 rows x D/2
  static constexpr uint32_t OFF_X = B_BYTES;
  static constexpr uint32_t OFF_Q = OFF_X + NS * X_BYTES;         // 1024-aligned (swizzled staging)
  static constexpr uint32_t OFF_T = OFF_Q + 8 * Q_BYTES;
  static constexpr uint32_t OFF_U = OFF_T + NS * T_BYTES;
  static constexpr uint32_t OFF_S = OFF_U + 4 * U_BYTES;
  static constexpr uint32_t OFF_C = OFF_S + 8 * S_BYTES;       // fp16 mode, per epilogue warp: 2^-(E + G_n)
  static constexpr uint32_t OFF_CORE = OFF_C + (F16 ? 8 * S_BYTES : 0);  // per transform warp: core[h] of the cell
  static constexpr uint32_t OFF_RING = OFF_CORE + 4 * CORE_MAX * 4;  // tile ids drawn by the producer
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t NBAR = 2 * NS + 2 * 2 + 4 + 2;  // loaded, empty, A full/free x2, acc full/empty x2, B free/ready
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

template <int D, bool SYM, int RDM, int NS, bool F16, int BITS>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_quant_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ TmaMaps cmaps,
                    const __grid_constant__ EncArgs A, const uint8_t* bimg) {
  static_assert(!F16 || RDM == 1, "the fp16 mode takes rank-1 row terms");
  static_assert(BITS == 2 || BITS == 4 || BITS == 8, "codes of 2, 4 or 8 bits");
  using L = QuantLayout<D, RDM, NS, F16>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  constexpr uint32_t ACOLS = D / 2;  // TMEM columns of one A buffer (bf16 pairs)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = loaded + NS;
  uint64_t* afull = empty + NS;
  uint64_t* afree = afull + 2;
  uint64_t* accf = afree + 2;
  uint64_t* acce = accf + 2;
  uint64_t* bfree = acce + 2;    // MMA: the last MMA of a cell has read B
  uint64_t* bready = bfree + 1;  // TMA: the next cell's B has arrived
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);  // TMA issue + transaction bytes
      mbar_init(&empty[i], 128);  // transform threads, once the tile is in registers
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&afull[i], 128);  // transform threads, after their TMEM stores
      mbar_init(&afree[i], 1);    // tcgen05.commit
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], NEPI);
    }
    mbar_init(bfree, 1);
    mbar_init(bready, 1);
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
    // ---------------- transform: R = x - recon of one row into a TMEM A buffer ----------------
    const int ptid = threadIdx.x;
    float* u32 = reinterpret_cast<float*>(smem + L::OFF_U + warp * L::U_BYTES);       // [j][4]
    uint16_t* ub = reinterpret_cast<uint16_t*>(smem + L::OFF_U + warp * L::U_BYTES);  // [j]
    float* cs = reinterpret_cast<float*>(smem + L::OFF_CORE) + warp * CORE_MAX;      // [h]
    int cur_cell = -1;
    float es = 1.f;  // fp16 mode: 2^E of the cell
    for (int it = 0;; ++it) {
      const int st = it % NS, b = it & 1;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x171)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) {  // no more tiles: pass the end on to the MMA thread
        if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x172)) break;
        mbar_arrive(&afull[b]);
        break;
      }
      const int cell = (int)(tile / A.tiles_per_cell);
      const int64_t row = (tile % A.tiles_per_cell) * TILE_M + ptid;
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
        if (A.rows_direct)
          for (int j = lane; j < (int)(A.rows / A.t_tok); j += 32) cs[j] = load_dt(A.core.p[cell], j, KVC_BF16);
        if (F16) es = A.fscale[(size_t)cell * (1 + D)];
        __syncwarp();
        cur_cell = cell;
      }
      const uint8_t* Xs = smem + L::OFF_X + st * L::X_BYTES;
      const bool sub = A.rt > 0 && row < A.rows;
      const uint32_t tm_row = tmem + ((uint32_t)(warp * 32) << 16) + b * ACOLS;
      if (RDM == 1) {
        // the whole row and its Tucker term in registers first, so the x
        // stage goes back to the producer before the arithmetic and before
        // this warp waits for its A buffer
        uint32_t r[D / 2];
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const uint4 x = *reinterpret_cast<const uint4*>(Xs + sw128_off(ptid, c * 8, TILE_M));
          r[4 * c] = x.x;
          r[4 * c + 1] = x.y;
          r[4 * c + 2] = x.z;
          r[4 * c + 3] = x.w;
        }
        const uint32_t th = sub ? enc_row_term(A, smem + L::OFF_T + st * L::T_BYTES, cs, ptid, row - ptid) : 0u;
        mbar_arrive(&empty[st]);  // the x stage is no longer needed
        if (sub) {
          // rd == 1: recon = bf16(t * u_j) and R = bf16(x - recon), each a
          // single rounding of the exact bf16 product / difference
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            const uint4 u = u4[c];
            r[4 * c] = bf16x2_sub(r[4 * c], bf16x2_mul(t2, u.x));
            r[4 * c + 1] = bf16x2_sub(r[4 * c + 1], bf16x2_mul(t2, u.y));
            r[4 * c + 2] = bf16x2_sub(r[4 * c + 2], bf16x2_mul(t2, u.z));
            r[4 * c + 3] = bf16x2_sub(r[4 * c + 3], bf16x2_mul(t2, u.w));
          }
        }
        if constexpr (F16) {
          // R * 2^E in fp16: exact for every bf16 value down to 2^-14 of the
          // scaled range (smaller ones are negligible against the step)
#pragma unroll
          for (int i = 0; i < D / 2; ++i) {
            const float lo = __uint_as_float(r[i] << 16) * es, hi = __uint_as_float(r[i] & 0xFFFF0000u) * es;
            const __half2 h2 = __floats2half2_rn(lo, hi);
            r[i] = *reinterpret_cast<const uint32_t*>(&h2);
          }
        }
        // the MMAs of tile it - 2 read this A buffer last
        if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x172)) break;
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < (int)ACOLS / 32; ++q) {
          uint32_t part[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) part[i] = r[q * 32 + i];
          tmem_st32(tm_row + q * 32, part);
        }
      } else {
        // rd > 1: 64 features at a time (register pressure); the A buffer
        // must be free before the first store
        if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x172)) break;
        tc_fence_after();
        const float4 tv = sub ? *reinterpret_cast<const float4*>(smem + L::OFF_T + st * L::T_BYTES + ptid * 16)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4* u4 = reinterpret_cast<const float4*>(u32);
#pragma unroll
        for (int q = 0; q < (int)ACOLS / 32; ++q) {
          uint32_t part[32];
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const int c = q * 8 + c8;
            const uint4 raw = *reinterpret_cast<const uint4*>(Xs + sw128_off(ptid, c * 8, TILE_M));
            float xv[8];
            unpack8_bf16(raw, xv);
            if (sub) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float4 u = u4[c * 8 + e];
                float rec = tv.x * u.x;
                rec = fmaf(tv.y, u.y, rec);
                rec = fmaf(tv.z, u.z, rec);
                rec = fmaf(tv.w, u.w, rec);
                xv[e] = Elt<__nv_bfloat16>::round(xv[e] - Elt<__nv_bfloat16>::round(rec));
              }
            }
            const uint4 w = pack8_bf16(xv);
            part[4 * c8] = w.x;
            part[4 * c8 + 1] = w.y;
            part[4 * c8 + 2] = w.z;
            part[4 * c8 + 3] = w.w;
          }
          tmem_st32(tm_row + q * 32, part);
        }
        mbar_arrive(&empty[st]);  // the x stage is no longer needed
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull[b]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      sched::Cursor cur(A.tiles_per_cta, A.total_tiles);
      for (int it = 0;; ++it) {
        const int64_t tile = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)tile);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x173)) break;
        if (tile < 0) {  // the end: a plain arrive completes the stage with no bytes
          mbar_arrive(&loaded[st]);
          break;
        }
        const int cell = (int)(tile / A.tiles_per_cell);
        const int y = (int)((tile % A.tiles_per_cell) * TILE_M);
        mbar_expect_tx(&loaded[st], L::X_BYTES + (A.rt > 0 ? (A.rows_direct ? TILE_M * 2u : L::T_BYTES) : 0u));
        const uint32_t dst = sbase + L::OFF_X + st * L::X_BYTES;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * TILE_M * 128, &xmaps.m[cell], h * 64, y, &loaded[st]);
        if (A.rt > 0 && A.rows_direct)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    static_cast<const uint8_t*>(A.ut.p[cell]) + ((uint32_t)y % (uint32_t)A.t_tok) * 2u, TILE_M * 2u,
                    &loaded[st]);
        else if (A.rt > 0)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    A.tmp + ((int64_t)cell * A.tiles_per_cell * TILE_M + y) * RDM, L::T_BYTES, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // D[row][feature] = sum_k R[row][k] (Pi / s)[feature][k]
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(TILE_M, D, !F16);
      int it = 0, cur_cell = -1, nb = 0;
      bool ended = false;
      for (;; ++it) {
        const int b = it & 1, ac = it & 1;
        if (!mbar_wait(&afull[b], (uint32_t)((it >> 1) & 1), 0x271)) break;
        const int32_t tile = sched::ring_get(ring, it);
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x272)) break;
        if (tile < 0) {  // the end: the epilogue learns it from the same accumulator barrier
          umma_commit(&accf[ac]);
          ended = true;
          break;
        }
        const int cell = (int)(tile / A.tiles_per_cell);
        if (cell != cur_cell) {
          // Pi / s of the new cell: after this thread's MMAs on the old one
          if (cur_cell >= 0) {
            umma_commit(bfree);
            if (!mbar_wait(bfree, (uint32_t)((nb - 1) & 1), 0x274)) break;
          }
          mbar_expect_tx(bready, L::B_BYTES);
#pragma unroll
          for (int term = 0; term < L::NTERM; ++term)
            bulk_load(sbase + term * L::B_TERM, bimg + (size_t)cell * 3 * L::B_TERM + term * L::B_TERM, L::B_TERM,
                      bready);
          if (!mbar_wait(bready, (uint32_t)(nb & 1), 0x275)) break;
          ++nb;
          cur_cell = cell;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * D);
#pragma unroll
        for (int term = 0; term < L::NTERM; ++term) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t kb = (uint32_t)((ks >> 2) * (D * 128) + (ks & 3) * 32);
            umma_f16_ts(d_tmem, tmem + b * ACOLS + (uint32_t)(ks * 8), desc_sw128(sbase + term * L::B_TERM + kb),
                        idesc, (term | ks) ? 1u : 0u);
          }
        }
        umma_commit(&afree[b]);
        umma_commit(&accf[ac]);
      }
      // do not leave while MMAs that write TMEM are still in flight
      if (ended) mbar_wait(&accf[it & 1], (uint32_t)(it >> 1) & 1u, 0x273);
      else if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x273);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: thread = row, D/2 features per warp ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;  // 32-feature chunks per warp
    float* zpf = reinterpret_cast<float*>(smem + L::OFF_S + e * L::S_BYTES);  // [feature]: zp
    float* cf = reinterpret_cast<float*>(smem + L::OFF_C + e * L::S_BYTES);   // fp16 mode: 2^-(E + G_n)
    // codes of this warp's half row: cbw bytes.  From 16 bytes up they are
    // staged as [32 rows][cbw] in shared memory with the swizzle of that
    // width (16-byte chunk j of row r at j ^ ((r * cbw / 128) mod (cbw / 16)),
    // conflict-free) and leave by one TMA store of whole rows; 8-byte half
    // rows (d = 64, 2 bits) are stored directly.
    uint8_t* stg = smem + L::OFF_Q + e * L::Q_BYTES;
    constexpr int cbw = (D / 2) * BITS / 8;
    constexpr bool tma_out = cbw >= 16;
    const int swz = tma_out ? ((lane * cbw) >> 7) & (cbw / 16 - 1) : 0;
    uint8_t* srow = stg + lane * cbw;
    int qmin, qmax;
    qrange(BITS, SYM ? 1 : 0, qmin, qmax);
    constexpr int offset = SYM ? (1 << (BITS - 1)) : 0;
    const int ad = A.scale_mode == KVC_SCALE_TENSOR ? A.arith_dtype : KVC_F32;
    const bool fast = A.scale_mode != KVC_SCALE_TENSOR || A.arith_dtype == KVC_F32;
    const float magic = 12582912.0f + (float)offset;  // 1.5 * 2^23 + offset
    const int lo_bits = 0x4B400000 + offset + qmin, hi_bits = 0x4B400000 + offset + qmax;
    float s_t = 1.f;  // per-tensor scale and zero point (the unfolded path)
    int32_t zp_t = 0;
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x371)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) break;
      const int cell = (int)(tile / A.tiles_per_cell);
      const int64_t row = (tile % A.tiles_per_cell) * TILE_M + rloc;
      if (cell != cur_cell) {
        const int32_t* zz = static_cast<const int32_t*>(A.zp.p[cell]);
        if (!SYM) {
          __syncwarp();
          for (int jl = lane; jl < D / 2; jl += 32)
            zpf[jl] = (float)zz[A.scale_mode == KVC_SCALE_CHANNEL ? half * (D / 2) + jl : 0];
          __syncwarp();
        }
        if (F16) {
          __syncwarp();
          for (int jl = lane; jl < D / 2; jl += 32) cf[jl] = A.fscale[(size_t)cell * (1 + D) + 1 + half * (D / 2) + jl];
          __syncwarp();
        }
        s_t = static_cast<const float*>(A.scale.p[cell])[0];
        zp_t = zz[0];
        cur_cell = cell;
      }
      tc_fence_after();
      if (tma_out) {
        // the previous tile's store has read the staging rows
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      }
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;  // global 32-feature chunk
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        int code[32];
        if (fast) {
          // v holds R~ / s: add zp, round half to even with the magic
          // constant and clamp on the float bits
          const uint64_t M2 = f2_pack(magic, magic);
          const uint64_t* z2 = reinterpret_cast<const uint64_t*>(zpf + cc * 32);
          const uint64_t* c2 = reinterpret_cast<const uint64_t*>(cf + cc * 32);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            uint64_t t2 = f2_pack(v[j], v[j + 1]);
            if (F16) t2 = f2_mul(t2, c2[j / 2]);  // exact: powers of two
            if (!SYM) t2 = f2_add(t2, z2[j / 2]);
            float y0, y1;
            f2_unpack(f2_add(t2, M2), y0, y1);
            code[j] = min(max(__float_as_int(y0), lo_bits), hi_bits);
            code[j + 1] = min(max(__float_as_int(y1), lo_bits), hi_bits);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) code[j] = quantize_one(v[j], s_t, zp_t, qmin, qmax, ad) + offset;
        }
        // low byte of each code is (q + offset) & 0xFF
        if constexpr (BITS == 8) {
          uint32_t w[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            w[q] = __byte_perm(__byte_perm(code[4 * q], code[4 * q + 1], 0x0040),
                               __byte_perm(code[4 * q + 2], code[4 * q + 3], 0x0040), 0x5410);
          const int j = cc * 2;  // 16-byte chunks of the staged half row
          *reinterpret_cast<uint4*>(srow + ((j ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(srow + (((j + 1) ^ swz) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        } else if constexpr (BITS == 4) {
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t pb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              pb[i] = ((uint32_t)code[8 * q + 2 * i] << 4) | ((uint32_t)code[8 * q + 2 * i + 1] & 0xFu);
            w[q] = __byte_perm(__byte_perm(pb[0], pb[1], 0x0040), __byte_perm(pb[2], pb[3], 0x0040), 0x5410);
          }
          *reinterpret_cast<uint4*>(srow + ((cc ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
          uint32_t w[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint32_t pb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int k = 16 * q + 4 * i;
              pb[i] = ((uint32_t)code[k] << 6) | (((uint32_t)code[k + 1] & 3u) << 4) |
                      (((uint32_t)code[k + 2] & 3u) << 2) | ((uint32_t)code[k + 3] & 3u);
            }
            w[q] = __byte_perm(__byte_perm(pb[0], pb[1], 0x0040), __byte_perm(pb[2], pb[3], 0x0040), 0x5410);
          }
          if constexpr (tma_out) {
            // 8 bytes per 32 features: chunk cc / 2, half cc % 2
            *reinterpret_cast<uint2*>(srow + (((cc >> 1) ^ swz) << 4) + (cc & 1) * 8) = make_uint2(w[0], w[1]);
          } else if (row < A.rows) {
            uint8_t* dst = static_cast<uint8_t*>(A.codes.p[cell]) + row * A.code_bytes + c * 8;
            *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
          }
        }
      }
      if (tma_out) {
        fence_async_smem();
        __syncwarp();
        const int64_t row0 = (tile % A.tiles_per_cell) * TILE_M + lg * 32;
        if (lane == 0) {
          if (row0 < A.rows) tma_store_2d(&cmaps.m[cell], half * cbw, (int)row0, smem_u32(stg));
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
    }
    if (lane == 0) bulk_wait<0>();  // shared memory outlives the stores
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------
// fp32 cells with head_dim 64, both encode passes, row-major: A = R in three
// bf16 terms in TMEM (R0 = bf16(R), R1 = bf16(R - R0), R2 = bf16(R - R0 -
// R1): their sum is R to 2^-27 of |R|), B = Pi (stats) or Pi / s (quantise)
// in three bf16 terms in shared memory.  The six products R_i P_j with
// i + j <= 2 accumulate in fp32 (each of the three left out is below 2^-26
// of the leading one), so the accumulator holds the rotated residual
// (x - recon) Pi^T to fp32 accuracy (kvcompress/compressor/residual.py:
// 201-239).  A 64-float row is 256 bytes, so an x tile is the 32 KB of a
// bf16 row of 128: two 128-byte SWIZZLE_128B boxes of 32 floats.
//   stats:    each epilogue thread keeps its 32 features' extremes over the
//             rows it sees in registers; at a cell change the warp merges
//             them (a reduce-scatter over the lanes, lane = feature) into the
//             cell's ordered-int min / max;
//   quantise: the epilogue of tc_quant_kernel (codes of the magic-constant
//             rounding, staged and stored by TMA from 16-byte half rows).
// ------------------------------------------------------------------------
template <int RDM, int NS>
struct Enc32Layout {
  static constexpr int D = 64;
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_BYTES = 3 * B_TERM;    // Pi or Pi / s of the cell in three bf16 terms
  static constexpr uint32_t X_BYTES = TILE_M * D * 4;  // fp32 x tile (TMA, two SWIZZLE_128B boxes)
  static constexpr uint32_t T_BYTES = TILE_M * RDM * 4;  // Tucker row terms of a tile
  static constexpr uint32_t U_BYTES = D * RDM * 4;       // per transform warp: u_feature fp32 [j][RDM]
  static constexpr uint32_t S_BYTES = (D / 2) * 4;       // per epilogue warp: zp of its D/2 features
  static constexpr uint32_t Q_BYTES = 32 * (D / 2);      // per epilogue warp: codes of 32 rows x D/2 (8-bit)
  static constexpr uint32_t OFF_X = B_BYTES;             // 1024-aligned
  static constexpr uint32_t OFF_Q = OFF_X + NS * X_BYTES;  // 1024-aligned (swizzled staging)
  static constexpr uint32_t OFF_T = OFF_Q + 8 * Q_BYTES;
  static constexpr uint32_t OFF_U = OFF_T + NS * T_BYTES;
  static constexpr uint32_t OFF_S = OFF_U + 4 * U_BYTES;
  static constexpr uint32_t OFF_RING = OFF_S + 8 * S_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t NBAR = 2 * NS + 2 * 2 + 4 + 2;  // loaded, empty, A full/free x2, acc x2 x2, B free/ready
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

// The lanes' v[0..31] reduced over the warp by min or max, lane l ending
// with the result for index l (five exchange steps, 31 shuffles).
template <bool MAX>
__device__ __forceinline__ float lane_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = up ? v[i] : v[i + s];
      const float keep = up ? v[i + s] : v[i];
      const float got = __shfl_xor_sync(0xffffffffu, send, s);
      v[i] = MAX ? fmaxf(keep, got) : fminf(keep, got);
    }
  }
  return v[0];
}

template <bool STATS, bool SYM, int RDM, int NS, int BITS>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_enc32_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ TmaMaps cmaps,
                    const __grid_constant__ EncArgs A, const uint8_t* bimg) {
  static_assert(BITS == 2 || BITS == 4 || BITS == 8, "codes of 2, 4 or 8 bits");
  static_assert(RDM == 1 || RDM == 4, "up to four feature-rank terms a row");
  constexpr int D = 64;
  using L = Enc32Layout<RDM, NS>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  constexpr uint32_t TCOLS = D / 2;      // TMEM columns of one bf16 term of a row
  constexpr uint32_t ACOLS = 3 * TCOLS;  // one A buffer: the three terms
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = loaded + NS;
  uint64_t* afull = empty + NS;
  uint64_t* afree = afull + 2;
  uint64_t* accf = afree + 2;
  uint64_t* acce = accf + 2;
  uint64_t* bfree = acce + 2;
  uint64_t* bready = bfree + 1;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);
      mbar_init(&empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&afull[i], 128);
      mbar_init(&afree[i], 1);
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], NEPI);
    }
    mbar_init(bfree, 1);
    mbar_init(bready, 1);
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
    // ---------------- transform: R = x - recon of one row, three bf16 terms into a TMEM A buffer ----------------
    const int ptid = threadIdx.x;
    float* us = reinterpret_cast<float*>(smem + L::OFF_U + warp * L::U_BYTES);  // [j][RDM]
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int st = it % NS, b = it & 1;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x1A1)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) {  // no more tiles: pass the end on to the MMA thread
        if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x1A2)) break;
        mbar_arrive(&afull[b]);
        break;
      }
      const int cell = (int)(tile / A.tiles_per_cell);
      const int64_t row = (tile % A.tiles_per_cell) * TILE_M + ptid;
      if (A.rt > 0 && cell != cur_cell) {
        __syncwarp();
        const float* ud = static_cast<const float*>(A.ud.p[cell]);
        for (int i = lane; i < D * RDM; i += 32) {
          const int j = i / RDM, r = i % RDM;
          us[i] = r < A.rd ? ud[j * A.rd + r] : 0.f;
        }
        __syncwarp();
        cur_cell = cell;
      }
      const uint8_t* Xs = smem + L::OFF_X + st * L::X_BYTES;
      const bool sub = A.rt > 0 && row < A.rows;
      // the row and its row terms in registers, then the stage goes back
      float xv[D];
#pragma unroll
      for (int c = 0; c < D / 4; ++c) {
        // floats 4c .. 4c + 3 are the 16 bytes of bf16 columns 8c .. 8c + 7
        const uint4 raw = *reinterpret_cast<const uint4*>(Xs + sw128_off(ptid, c * 8, TILE_M));
        xv[4 * c] = __uint_as_float(raw.x);
        xv[4 * c + 1] = __uint_as_float(raw.y);
        xv[4 * c + 2] = __uint_as_float(raw.z);
        xv[4 * c + 3] = __uint_as_float(raw.w);
      }
      float tv[RDM];
      if (sub) {
        const float* ts = reinterpret_cast<const float*>(smem + L::OFF_T + st * L::T_BYTES) + ptid * RDM;
        if constexpr (RDM == 1) tv[0] = ts[0];
        else load_row_terms<RDM>(ts, tv);
      }
      mbar_arrive(&empty[st]);  // the x stage is no longer needed
      if (sub) {
        // recon in the fp32 order of the SIMT residual, then R = x - recon
#pragma unroll
        for (int j = 0; j < D; ++j) {
          float rec;
          if constexpr (RDM == 1) rec = tv[0] * us[j];
          else rec = recon_dot<RDM>(tv, reinterpret_cast<const float4*>(us + j * RDM));
          xv[j] = xv[j] - rec;
        }
      }
      // the MMAs of tile it - 2 read this A buffer last
      if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x1A2)) break;
      tc_fence_after();
      const uint32_t tm_row = tmem + ((uint32_t)(warp * 32) << 16) + b * ACOLS;
#pragma unroll
      for (int term = 0; term < 3; ++term) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(xv[2 * i], xv[2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&h);
          if (term < 2) {  // what the term leaves, exact in fp32
            xv[2 * i] -= __low2float(h);
            xv[2 * i + 1] -= __high2float(h);
          }
        }
        tmem_st32(tm_row + term * TCOLS, w);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull[b]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      sched::Cursor cur(A.tiles_per_cta, A.total_tiles);
      for (int it = 0;; ++it) {
        const int64_t tile = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)tile);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x1A3)) break;
        if (tile < 0) {  // the end: a plain arrive completes the stage with no bytes
          mbar_arrive(&loaded[st]);
          break;
        }
        const int cell = (int)(tile / A.tiles_per_cell);
        const int y = (int)((tile % A.tiles_per_cell) * TILE_M);
        mbar_expect_tx(&loaded[st], L::X_BYTES + (A.rt > 0 ? L::T_BYTES : 0u));
        const uint32_t dst = sbase + L::OFF_X + st * L::X_BYTES;
        tma_load_2d(dst, &xmaps.m[cell], 0, y, &loaded[st]);
        tma_load_2d(dst + TILE_M * 128, &xmaps.m[cell], 32, y, &loaded[st]);
        if (A.rt > 0)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    A.tmp + ((int64_t)cell * A.tiles_per_cell * TILE_M + y) * RDM, L::T_BYTES, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // D[row][feature] = sum_k R[row][k] B[feature][k], the six term pairs
    // smallest first
    if (lane == 0) {
      constexpr int PA[6] = {1, 0, 2, 1, 0, 0}, PB[6] = {1, 2, 0, 0, 1, 0};
      const uint32_t idesc = idesc_f16(TILE_M, D, true);
      int it = 0, cur_cell = -1, nb = 0;
      bool ended = false;
      for (;; ++it) {
        const int b = it & 1, ac = it & 1;
        if (!mbar_wait(&afull[b], (uint32_t)((it >> 1) & 1), 0x2A1)) break;
        const int32_t tile = sched::ring_get(ring, it);
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x2A2)) break;
        if (tile < 0) {  // the end: the epilogue learns it from the same accumulator barrier
          umma_commit(&accf[ac]);
          ended = true;
          break;
        }
        const int cell = (int)(tile / A.tiles_per_cell);
        // stats: one image of Pi for every cell; quantise: Pi / s per cell
        if (STATS ? cur_cell < 0 : cell != cur_cell) {
          if (cur_cell >= 0) {
            umma_commit(bfree);
            if (!mbar_wait(bfree, (uint32_t)((nb - 1) & 1), 0x2A4)) break;
          }
          mbar_expect_tx(bready, L::B_BYTES);
          bulk_load(sbase, bimg + (STATS ? (size_t)0 : (size_t)cell * L::B_BYTES), L::B_BYTES, bready);
          if (!mbar_wait(bready, (uint32_t)(nb & 1), 0x2A5)) break;
          ++nb;
        }
        cur_cell = cell;
        tc_fence_after();
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * D);
#pragma unroll
        for (int p = 0; p < 6; ++p) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_f16_ts(d_tmem, tmem + b * ACOLS + PA[p] * TCOLS + (uint32_t)(ks * 8),
                        desc_sw128(sbase + PB[p] * L::B_TERM + (uint32_t)(ks * 32)), idesc, (p | ks) ? 1u : 0u);
        }
        umma_commit(&afree[b]);
        umma_commit(&accf[ac]);
      }
      // do not leave while MMAs that write TMEM are still in flight
      if (ended) mbar_wait(&accf[it & 1], (uint32_t)(it >> 1) & 1u, 0x2A3);
      else if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x2A3);
    }
    __syncwarp();
  } else if (STATS) {
    // ---------------- stats epilogue: thread = row, 32 features per warp ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    float lo[32], hi[32];  // SYM: hi = max |v|
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      lo[j] = __int_as_float(0x7f800000);
      hi[j] = SYM ? 0.f : -__int_as_float(0x7f800000);
    }
    auto flush = [&](int cell) {
      int32_t* mm = A.minmax + (int64_t)cell * 2 * D;
      const int f = half * 32 + lane;
      const float mx = lane_reduce_scatter32<true>(hi, lane);
      if (SYM) {
        atomicMin(&mm[f], ordered_bits(-mx));
        atomicMax(&mm[D + f], ordered_bits(mx));
      } else {
        const float mn = lane_reduce_scatter32<false>(lo, lane);
        atomicMin(&mm[f], ordered_bits(mn));
        atomicMax(&mm[D + f], ordered_bits(mx));
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        lo[j] = __int_as_float(0x7f800000);
        hi[j] = SYM ? 0.f : -__int_as_float(0x7f800000);
      }
    };
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x3A1)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) break;
      const int cell = (int)(tile / A.tiles_per_cell);
      const int64_t row = (tile % A.tiles_per_cell) * TILE_M + rloc;
      if (cell != cur_cell) {
        if (cur_cell >= 0) flush(cur_cell);
        cur_cell = cell;
      }
      tc_fence_after();
      float v[32];
      tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + half * 32), v);
      tc_fence_before();
      mbar_arrive(&acce[ac]);
      if (row < A.rows) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (SYM) {
            hi[j] = fmaxf(hi[j], fabsf(v[j]));
          } else {
            lo[j] = fminf(lo[j], v[j]);
            hi[j] = fmaxf(hi[j], v[j]);
          }
        }
      }
    }
    if (cur_cell >= 0) flush(cur_cell);
    __syncwarp();
  } else {
    // ---------------- quantise epilogue: thread = row, 32 features per warp ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    float* zpf = reinterpret_cast<float*>(smem + L::OFF_S + e * L::S_BYTES);  // [feature]: zp
    uint8_t* stg = smem + L::OFF_Q + e * L::Q_BYTES;
    constexpr int cbw = (D / 2) * BITS / 8;  // code bytes of a half row: 32, 16 or 8
    constexpr bool tma_out = cbw >= 16;
    const int swz = tma_out ? ((lane * cbw) >> 7) & (cbw / 16 - 1) : 0;
    uint8_t* srow = stg + lane * cbw;
    int qmin, qmax;
    qrange(BITS, SYM ? 1 : 0, qmin, qmax);
    constexpr int offset = SYM ? (1 << (BITS - 1)) : 0;
    const int ad = A.scale_mode == KVC_SCALE_TENSOR ? A.arith_dtype : KVC_F32;
    const bool fast = A.scale_mode != KVC_SCALE_TENSOR || A.arith_dtype == KVC_F32;
    const float magic = 12582912.0f + (float)offset;  // 1.5 * 2^23 + offset
    const int lo_bits = 0x4B400000 + offset + qmin, hi_bits = 0x4B400000 + offset + qmax;
    float s_t = 1.f;
    int32_t zp_t = 0;
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x3A2)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) break;
      const int cell = (int)(tile / A.tiles_per_cell);
      const int64_t row = (tile % A.tiles_per_cell) * TILE_M + rloc;
      if (cell != cur_cell) {
        const int32_t* zz = static_cast<const int32_t*>(A.zp.p[cell]);
        if (!SYM) {
          __syncwarp();
          for (int jl = lane; jl < D / 2; jl += 32)
            zpf[jl] = (float)zz[A.scale_mode == KVC_SCALE_CHANNEL ? half * (D / 2) + jl : 0];
          __syncwarp();
        }
        s_t = static_cast<const float*>(A.scale.p[cell])[0];
        zp_t = zz[0];
        cur_cell = cell;
      }
      tc_fence_after();
      if (tma_out) {
        // the previous tile's store has read the staging rows
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      }
      float v[32];
      tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + half * 32), v);
      tc_fence_before();
      mbar_arrive(&acce[ac]);
      int code[32];
      if (fast) {
        // v holds R~ / s: add zp, round half to even with the magic constant
        // and clamp on the float bits
        const uint64_t M2 = f2_pack(magic, magic);
        const uint64_t* z2 = reinterpret_cast<const uint64_t*>(zpf);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          uint64_t t2 = f2_pack(v[j], v[j + 1]);
          if (!SYM) t2 = f2_add(t2, z2[j / 2]);
          float y0, y1;
          f2_unpack(f2_add(t2, M2), y0, y1);
          code[j] = min(max(__float_as_int(y0), lo_bits), hi_bits);
          code[j + 1] = min(max(__float_as_int(y1), lo_bits), hi_bits);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) code[j] = quantize_one(v[j], s_t, zp_t, qmin, qmax, ad) + offset;
      }
      // low byte of each code is (q + offset) & 0xFF
      if constexpr (BITS == 8) {
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          w[q] = __byte_perm(__byte_perm(code[4 * q], code[4 * q + 1], 0x0040),
                             __byte_perm(code[4 * q + 2], code[4 * q + 3], 0x0040), 0x5410);
        *reinterpret_cast<uint4*>(srow + ((0 ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(srow + ((1 ^ swz) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
      } else if constexpr (BITS == 4) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pb[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pb[i] = ((uint32_t)code[8 * q + 2 * i] << 4) | ((uint32_t)code[8 * q + 2 * i + 1] & 0xFu);
          w[q] = __byte_perm(__byte_perm(pb[0], pb[1], 0x0040), __byte_perm(pb[2], pb[3], 0x0040), 0x5410);
        }
        *reinterpret_cast<uint4*>(srow) = make_uint4(w[0], w[1], w[2], w[3]);
      } else {
        uint32_t w[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t pb[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = 16 * q + 4 * i;
            pb[i] = ((uint32_t)code[k] << 6) | (((uint32_t)code[k + 1] & 3u) << 4) |
                    (((uint32_t)code[k + 2] & 3u) << 2) | ((uint32_t)code[k + 3] & 3u);
          }
          w[q] = __byte_perm(__byte_perm(pb[0], pb[1], 0x0040), __byte_perm(pb[2], pb[3], 0x0040), 0x5410);
        }
        if (row < A.rows) {
          uint8_t* dst = static_cast<uint8_t*>(A.codes.p[cell]) + row * A.code_bytes + half * 8;
          *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
        }
      }
      if (tma_out) {
        fence_async_smem();
        __syncwarp();
        const int64_t row0 = (tile % A.tiles_per_cell) * TILE_M + lg * 32;
        if (lane == 0) {
          if (row0 < A.rows) tma_store_2d(&cmaps.m[cell], half * cbw, (int)row0, smem_u32(stg));
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();  // shared memory outlives the stores
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------
// quantise pass, feature-major (d = 128, 8- and 4-bit codes): A = Pi / s of
// the cell in three bf16 terms in TMEM (192 columns; the transform warps
// reload them when the tile stream enters a new cell, after the MMAs of the
// previous tile have completed), B = R in place in the TMA stage as in the
// stats pass.  Shared memory then holds five x stages instead of the row-
// major pass's three next to its 96 KB B image.  TMEM lane = output feature:
// an epilogue thread quantises its feature's values of the tile's rows and
// writes the code byte of each row (4-bit: even lanes, the byte of the
// feature pair) into its warp's [128 rows][CBW] staging block, which the
// warp stores by TMA (two staging buffers a warp).
// ------------------------------------------------------------------------
template <int RDM, int NS>
struct QuantFmLayout {
  static constexpr int D = 128;
  static constexpr uint32_t B_BYTES = TILE_M * D * 2;         // x stage = R tile (MMA B operand)
  static constexpr uint32_t T_BYTES = TILE_M * RDM * 4;       // Tucker row term of a tile
  static constexpr uint32_t U_BYTES = RDM == 1 ? D : D * RDM * 2;  // per transform warp, as the stats pass
  static constexpr uint32_t Q_BYTES = TILE_M * 32;            // per epilogue warp and buffer: 128 rows x 32 bytes
  static constexpr uint32_t OFF_Q = NS * B_BYTES;
  static constexpr uint32_t OFF_T = OFF_Q + 4 * 2 * Q_BYTES;
  static constexpr uint32_t OFF_U = OFF_T + NS * T_BYTES;
  static constexpr uint32_t OFF_CORE = OFF_U + 8 * U_BYTES;  // per transform warp: core[h] of the cell
  static constexpr uint32_t OFF_RING = OFF_CORE + 8 * CORE_MAX * 4;
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t NBAR = 3 * NS + 4;  // loaded, full, empty, acc full x2, acc empty x2
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

// A rows of the feature-major quantise pass, per cell: Pi[n][k] / s_n
// (s_0 for per-tensor scales) split in three bf16 terms, as 32-bit pairs
// [cell][term][n < 128][d / 2] (k = 2w in the low half): the same values as
// the row-major pass's B images.
__global__ void prep_quant_arows_kernel(const float* __restrict__ proj, CellPtrs scale, int per_feature, int d,
                                        uint32_t* out) {
  const int cell = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // (n, w) over d x d/2
  const int wpr = d / 2;
  if (e >= d * wpr) return;
  const int n = e / wpr, w = e % wpr;
  const float s = static_cast<const float*>(scale.p[cell])[per_feature ? n : 0];
  float r0 = __fdiv_rn(proj[n * d + 2 * w], s), r1 = __fdiv_rn(proj[n * d + 2 * w + 1], s);
  uint32_t* base = out + (size_t)cell * 3 * 128 * wpr;
  for (int term = 0; term < 3; ++term) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(r0, r1);
    r0 -= __low2float(h);
    r1 -= __high2float(h);
    base[((size_t)term * 128 + n) * wpr + w] = *reinterpret_cast<const uint32_t*>(&h);
  }
}

// F16 (kernel policy 2, after the stats pass): A = (Pi / s) 2^G_n in two
// fp16 terms, R enters as fp16 scaled by 2^E of the cell, and the epilogue
// takes the exact factor 2^-(E + G_n) of its feature (the row-major pass's
// fp16 mode, prep_quant_b16_kernel).
template <bool SYM, int RDM, int NS, int BITS, bool F16 = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_quantfm_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ TmaMaps cmaps,
                      const __grid_constant__ EncArgs A, const uint32_t* arows) {
  constexpr int D = 128;
  constexpr int NTERM = F16 ? 2 : 3;
  static_assert(!F16 || RDM == 1, "the fp16 mode takes rank-1 row terms");
  using L = QuantFmLayout<RDM, NS>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  static_assert(BITS == 8 || BITS == 4, "feature-major codes of 8 or 4 bits");
  constexpr int CBW = 32 * BITS / 8;  // code bytes of a warp's 32 features in a row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = loaded + NS;
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);  // TMA issue + transaction bytes
      mbar_init(&full[i], 256);  // transform threads
      mbar_init(&empty[i], 1);   // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);    // tcgen05.commit
      mbar_init(&acce[i], 128);  // epilogue threads
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

  if (warp < 4 || warp >= STATS_XF_WARP1) {
    // ---------------- transform: R = x - recon, in place, one row per thread ----------------
    constexpr int HF = D / 2, HC = HF / 8;
    const int lgw = warp & 3, part = warp < 4 ? 0 : 1;
    const int ptid = lgw * 32 + lane;
    float* u32 = reinterpret_cast<float*>(smem + L::OFF_U + (part * 4 + lgw) * L::U_BYTES);       // [j][4]
    uint16_t* ub = reinterpret_cast<uint16_t*>(smem + L::OFF_U + (part * 4 + lgw) * L::U_BYTES);  // [j]
    float* cs = reinterpret_cast<float*>(smem + L::OFF_CORE) + (part * 4 + lgw) * CORE_MAX;     // [h]
    int cur_cell = -1;
    float es = 1.f;  // fp16 mode: 2^E of the cell
    for (int it = 0;; ++it) {
      const int st = it % NS;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x181)) break;
      const int32_t g = sched::ring_get(ring, it);
      if (g < 0) {  // no more tiles: pass the end on to the MMA thread
        mbar_arrive(&full[st]);
        break;
      }
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row = (g % A.tiles_per_cell) * TILE_M + ptid;
      if (cell != cur_cell) {
        if (warp < 4) {
          // Pi / s of the new cell into TMEM, once the MMAs of the previous
          // tile (the last ones to read the old terms) have completed
          if (it > 0 && !warp_wait(&empty[(it - 1) % NS], (uint32_t)(((it - 1) / NS) & 1), 0x182)) break;
          tc_fence_after();
          load_a_rows<D / 2>(tmem + ((uint32_t)(warp * 32) << 16), 0, arows + (size_t)cell * 3 * 128 * (D / 2),
                             NTERM, warp * 32 + lane, 128);
          tc_fence_before();
        }
        if (A.rt > 0) {
          __syncwarp();
          const __nv_bfloat16* ud = static_cast<const __nv_bfloat16*>(A.ud.p[cell]);
          if (RDM == 1) {
            for (int j = lane; j < HF; j += 32) ub[j] = reinterpret_cast<const uint16_t*>(ud)[part * HF + j];
          } else {
            for (int i = lane; i < HF * RDM; i += 32) {
              const int j = i / RDM, r = i % RDM;
              u32[i] = r < A.rd ? __bfloat162float(ud[(part * HF + j) * A.rd + r]) : 0.f;
            }
          }
          if (A.rows_direct)
            for (int j = lane; j < (int)(A.rows / A.t_tok); j += 32) cs[j] = load_dt(A.core.p[cell], j, KVC_BF16);
          __syncwarp();
        }
        if (F16) es = A.fscale[(size_t)cell * (1 + D)];
        cur_cell = cell;
      }
      if (A.rt > 0 && row < A.rows) {
        uint8_t* Bs = smem + st * L::B_BYTES;
        if (RDM == 1) {
          const uint32_t th = enc_row_term(A, smem + L::OFF_T + st * L::T_BYTES, cs, ptid, row - ptid);
          const uint32_t t2 = th | (th << 16);
          const uint4* u4 = reinterpret_cast<const uint4*>(ub);
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
            uint4 x = *slot;
            const uint4 u = u4[c];
            uint32_t w[4] = {bf16x2_sub(x.x, bf16x2_mul(t2, u.x)), bf16x2_sub(x.y, bf16x2_mul(t2, u.y)),
                             bf16x2_sub(x.z, bf16x2_mul(t2, u.z)), bf16x2_sub(x.w, bf16x2_mul(t2, u.w))};
            if constexpr (F16) {
              // R * 2^E in fp16: exact for every bf16 value down to 2^-14 of
              // the scaled range
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const __half2 h2 =
                    __floats2half2_rn(__uint_as_float(w[i] << 16) * es, __uint_as_float(w[i] & 0xFFFF0000u) * es);
                w[i] = *reinterpret_cast<const uint32_t*>(&h2);
              }
            }
            *slot = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float tv[RDM];
          load_row_terms<RDM>(reinterpret_cast<const float*>(smem + L::OFF_T + st * L::T_BYTES) + ptid * RDM, tv);
          const float4* u4 = reinterpret_cast<const float4*>(u32);
#pragma unroll 2
          for (int c = 0; c < HC; ++c) {
            uint4* slot = reinterpret_cast<uint4*>(Bs + sw128_off(ptid, (part * HC + c) * 8, TILE_M));
            float xv[8];
            unpack8_bf16(*slot, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float rec = recon_dot<RDM>(tv, u4 + (c * 8 + e) * (RDM / 4));
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
      sched::Cursor cur(A.tiles_per_cta, A.total_tiles);
      for (int it = 0;; ++it) {
        const int64_t g = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)g);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x183)) break;
        if (g < 0) {
          mbar_arrive(&loaded[st]);
          break;
        }
        const int cell = (int)(g / A.tiles_per_cell);
        const int y = (int)((g % A.tiles_per_cell) * TILE_M);
        mbar_expect_tx(&loaded[st], L::B_BYTES + (A.rt > 0 ? (A.rows_direct ? TILE_M * 2u : L::T_BYTES) : 0u));
        const uint32_t dst = sbase + st * L::B_BYTES;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * TILE_M * 128, &xmaps.m[cell], h * 64, y, &loaded[st]);
        if (A.rt > 0 && A.rows_direct)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    static_cast<const uint8_t*>(A.ut.p[cell]) + ((uint32_t)y % (uint32_t)A.t_tok) * 2u, TILE_M * 2u,
                    &loaded[st]);
        else if (A.rt > 0)
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    A.tmp + ((int64_t)cell * A.tiles_per_cell * TILE_M + y) * RDM, L::T_BYTES, &loaded[st]);
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer: D[feature][row] = sum_k (Pi / s)[feature][k] R[row][k] ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, TILE_M, !F16);
      int it = 0;
      bool ended = false;
      for (;; ++it) {
        const int st = it % NS, ac = it & 1;
        if (!mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x284)) break;
        const int32_t g = sched::ring_get(ring, it);
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x285)) break;
        if (g < 0) {
          umma_commit(&accf[ac]);
          ended = true;
          break;
        }
        tc_fence_after();
        const uint32_t b_base = sbase + st * L::B_BYTES;
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * TILE_M);
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
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
      if (ended) mbar_wait(&accf[it & 1], (uint32_t)(it >> 1) & 1u, 0x286);
      else if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x286);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: thread = output feature, codes of the tile's 128 rows ----------------
    // (warps 6-9, one per TMEM lane group)
    const int lg = warp & 3;
    const int feat = lg * 32 + lane;
    int qmin, qmax;
    qrange(BITS, SYM ? 1 : 0, qmin, qmax);
    constexpr int offset = SYM ? (1 << (BITS - 1)) : 0;
    const float magic = 12582912.0f + (float)offset;  // 1.5 * 2^23 + offset
    const int lo_bits = 0x4B400000 + offset + qmin, hi_bits = 0x4B400000 + offset + qmax;
    const uint64_t M2 = f2_pack(magic, magic);
    uint64_t z2 = 0, c2 = 0;
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x381)) break;
      const int32_t g = sched::ring_get(ring, it);
      if (g < 0) break;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t row0 = (g % A.tiles_per_cell) * TILE_M;
      if (cell != cur_cell) {
        if (!SYM) {
          const int32_t* zz = static_cast<const int32_t*>(A.zp.p[cell]);
          const float zf = (float)zz[A.scale_mode == KVC_SCALE_CHANNEL ? feat : 0];
          z2 = f2_pack(zf, zf);
        }
        if (F16) {
          const float cf = A.fscale[(size_t)cell * (1 + D) + 1 + feat];
          c2 = f2_pack(cf, cf);
        }
      }
      cur_cell = cell;
      uint8_t* stg = smem + L::OFF_Q + (lg * 2 + (it & 1)) * L::Q_BYTES;
      // the store issued from this buffer two tiles ago has read it
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * TILE_M + cc * 32), v);
        int code[32];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          uint64_t t2 = f2_pack(v[j], v[j + 1]);
          if (F16) t2 = f2_mul(t2, c2);  // exact: powers of two
          if (!SYM) t2 = f2_add(t2, z2);
          float y0, y1;
          f2_unpack(f2_add(t2, M2), y0, y1);
          code[j] = min(max(__float_as_int(y0), lo_bits), hi_bits);
          code[j + 1] = min(max(__float_as_int(y1), lo_bits), hi_bits);
        }
        uint8_t* rows8 = stg + cc * 32 * CBW;
        if constexpr (BITS == 8) {
#pragma unroll
          for (int j = 0; j < 32; ++j) rows8[j * CBW + lane] = (uint8_t)code[j];
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int nbr = __shfl_down_sync(0xffffffffu, code[j], 1);
            if (!(lane & 1)) rows8[j * CBW + (lane >> 1)] = (uint8_t)((code[j] << 4) | (nbr & 0xF));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (row0 < A.rows) tma_store_2d(&cmaps.m[cell], lg * CBW, (int)row0, smem_u32(stg));
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait<0>();  // shared memory outlives the stores
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------
// decode, row-major: A = the codes as exact bf16 integers in TMEM (one row
// per lane), B = diag(scale) Pi of the cell in shared memory (reloaded at a
// cell change), thread = row in the epilogue, bf16 rows stored directly
// ------------------------------------------------------------------------
// rd = 1: the Tucker term t_row * u_feature is one more K-step of the MMA
// (A: t split hi + mid + lo, B: u split hi + lo, every pairing once), so the
// epilogue only rounds; rd > 1 adds it in the epilogue.
// fp32 output (O32, d = 64): diag(scale) Pi in three bf16 terms and the
// Tucker term added in fp32 by the epilogue for every rd (the reference adds
// the fp32 reconstruction to the fp32 residual, jolt.py:424-463).
template <int D, int CB, int RDM, int NS, bool O32 = false>
struct DecLayout {
  static constexpr bool FOLD = RDM == 1 && !O32;
  static constexpr int NTB = O32 ? 3 : 2;                  // terms of diag(scale) Pi
  static constexpr uint32_t B_TERM = D * D * 2;
  static constexpr uint32_t B_TUCKER = FOLD ? D * 128 : 0;  // the extra K block (SW128, 16 of 64 used)
  static constexpr uint32_t B_BYTES = NTB * B_TERM + B_TUCKER;  // diag(scale) Pi (+ u_feature)
  static constexpr uint32_t C_BYTES = TILE_M * CB;    // codes as loaded (dense rows)
  static constexpr uint32_t U_BYTES = FOLD ? 0 : (D / 2) * RDM * 4;  // per epilogue warp: u_feature of its features
  static constexpr uint32_t ROW_BYTES = O32 ? 2 * D : D;   // one row's D/2 outputs
  static constexpr uint32_t O_BYTES = 32 * ROW_BYTES;      // per epilogue warp: 32 rows x D/2 outputs
  // rd = 1: the tile's Tucker terms, bulk-copied from the 16-byte boundary at
  // or below the first row (up to 3 floats early), 132 floats
  static constexpr uint32_t T_BYTES = FOLD ? (TILE_M + 4) * 4 : 0;
  static constexpr uint32_t OFF_C = B_BYTES;
  static constexpr uint32_t OFF_O = OFF_C + NS * C_BYTES;  // 1024-aligned (swizzled staging)
  static constexpr uint32_t OFF_U = OFF_O + 8 * O_BYTES;
  static constexpr uint32_t OFF_T = OFF_U + 8 * U_BYTES;
  static constexpr uint32_t OFF_RING = OFF_T + NS * T_BYTES;  // tile ids drawn by the producer
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t NBAR = 2 * NS + 2 * 2 + 4 + 2;  // loaded, empty, A full/free x2, acc x2 x2, B free/ready
  static constexpr uint32_t OFF_TM = OFF_BAR + NBAR * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

// Deepest codes ring (at most 8 stages) whose layout fits the 227 KB.
template <int D, int CB, int RDM, bool O32 = false, int NS = 8>
struct DecStages {
  static constexpr int value =
      DecLayout<D, CB, RDM, NS, O32>::BYTES <= 227 * 1024 ? NS : DecStages<D, CB, RDM, O32, NS - 1>::value;
};
template <int D, int CB, int RDM, bool O32>
struct DecStages<D, CB, RDM, O32, 2> {
  static constexpr int value = 2;
};

struct DecArgsTc {
  CellPtrs ud;
  CellPtrs core, ut;  // rows_direct: the rank-1 factors the row terms come from
  CellPtrsMut out;
  int64_t m, t0, tl, tiles_per_cell, total_tiles, tiles_per_cta;
  int tb_per_head;
  int rt, rd, factor_dtype;
  // rt = rd = 1, 2-byte factors, 128-token head blocks, 16-byte aligned
  // u_token rows: each tile's row terms core[h] * u_token[t] are formed in
  // the kernel from a 256-byte bulk copy of u_token (no row-term kernel)
  int rows_direct;
  const uint8_t* bimg;  // per cell: two swizzled B images of diag(scale) Pi (+ the u_feature block)
  const float* tmp;     // [cell][m * tl][rdm] fp32 Tucker row term (+ 132 floats of slack at the end)
};

template <int D, int RDM, int BITS, int NS, bool O32 = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_decode_kernel(const __grid_constant__ TmaMaps cmaps, const __grid_constant__ TmaMaps omaps,
                     const __grid_constant__ DecArgsTc A) {
  constexpr int CB = D * BITS / 8;  // code bytes per row
  using L = DecLayout<D, CB, RDM, NS, O32>;
  static_assert(L::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  static_assert(CB % 16 == 0, "code rows must be whole 16-byte chunks");
  // a run launched as a programmatic dependent of this one may start at once:
  // it reads nothing this one writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr bool FOLD = L::FOLD;
  // TMEM columns of one A buffer: D / 2 (+ 8 for the Tucker K-step, padded
  // so both buffers start on a 32-column boundary)
  constexpr uint32_t ACOLS = D / 2 + (FOLD ? 32 : 0);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = loaded + NS;
  uint64_t* afull = empty + NS;
  uint64_t* afree = afull + 2;
  uint64_t* accf = afree + 2;
  uint64_t* acce = accf + 2;
  uint64_t* bfree = acce + 2;    // the MMAs on the old cell's B are done
  uint64_t* bready = bfree + 1;  // the new cell's B has arrived
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + L::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&loaded[i], 1);
      mbar_init(&empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&afull[i], 128);
      mbar_init(&afree[i], 1);
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], NEPI);
    }
    mbar_init(bfree, 1);
    mbar_init(bready, 1);
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
    // ---------------- transform: codes of one row -> exact bf16 integers in a TMEM A buffer ----------------
    const int ptid = threadIdx.x;
    constexpr int NCH16 = CB / 16;  // 16-byte chunks per row
    constexpr int PER = 8 / BITS;   // codes per byte
    // a code byte b placed in the mantissa of 2^23 reads 2^23 + b; subtracting
    // 2^23 + offset leaves the signed code exactly
    const float bias = 8388608.0f + (float)(1 << (BITS - 1));
    const uint64_t NB2 = f2_pack(-bias, -bias);
    for (int it = 0;; ++it) {
      const int st = it % NS, b = it & 1;
      if (!warp_wait(&loaded[st], (uint32_t)((it / NS) & 1), 0x181)) break;
      const int32_t tile = sched::ring_get(ring, it);
      if (tile < 0) {  // no more tiles: pass the end on to the MMA thread
        if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x182)) break;
        mbar_arrive(&afull[b]);
        break;
      }
      float tv = 0.f;  // this row's Tucker term (rd = 1)
      if (FOLD && A.rt > 0) {
        const int64_t tc = tile % A.tiles_per_cell;
        const int64_t i_tok = (tc % A.tb_per_head) * TILE_M + ptid;
        const int64_t base = (int64_t)(tile / A.tiles_per_cell) * A.m * A.tl + (tc / A.tb_per_head) * A.tl +
                             (tc % A.tb_per_head) * TILE_M;
        if (A.rows_direct) {
          // core[h] * u_token[t]: the exact fp32 product of two 2-byte values,
          // the row term the row-term kernel would have written
          const int h = (int)(tc / A.tb_per_head);
          tv = load_dt(A.core.p[tile / A.tiles_per_cell], h, A.factor_dtype) *
               load_dt(smem + L::OFF_T + st * L::T_BYTES, ptid, A.factor_dtype);
        } else if (i_tok < A.tl) {
          tv = reinterpret_cast<const float*>(smem + L::OFF_T + st * L::T_BYTES)[(base & 3) + ptid];
        }
      }
      const uint8_t* Cs = smem + L::OFF_C + st * L::C_BYTES + ptid * CB;
      // the stage is written by TMA with the swizzle of its row width (32,
      // 64 or 128 B): 16-byte chunk c of row r sits at c ^ ((r * CB / 128) mod
      // (CB / 16)), which spreads the 8 rows of a quarter-warp over the banks
      const int swz = (ptid * CB >> 7) & (NCH16 - 1);
      uint32_t r[D / 2];
#pragma unroll
      for (int c = 0; c < NCH16; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(Cs + ((c ^ swz) << 4));
        const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
        // chunk c holds values [c * 16 * PER, (c + 1) * 16 * PER): 8 * PER bf16 pairs
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
            r[(c * 16 * PER + wi * 4 * PER + k) / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
      }
      mbar_arrive(&empty[st]);  // the codes stage is no longer needed
      if (it >= 2 && !warp_wait(&afree[b], (uint32_t)(((it - 2) >> 1) & 1), 0x182)) break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < D / 64; ++q) {
        uint32_t part[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) part[i] = r[q * 32 + i];
        tmem_st32(tmem + ((uint32_t)(warp * 32) << 16) + b * ACOLS + q * 32, part);
      }
      if (FOLD) {
        // K positions 0-5 of the extra step: (hi, mid, lo, hi, mid, lo) of t
        const __nv_bfloat16 th = __float2bfloat16_rn(tv);
        const float r1 = tv - __bfloat162float(th);
        const __nv_bfloat16 tm = __float2bfloat16_rn(r1);
        const __nv_bfloat16 tlo = __float2bfloat16_rn(r1 - __bfloat162float(tm));
        const uint32_t h = __bfloat16_as_ushort(th), mi = __bfloat16_as_ushort(tm), lo = __bfloat16_as_ushort(tlo);
        const uint32_t ext[8] = {h | (mi << 16), lo | (h << 16), mi | (lo << 16), 0u, 0u, 0u, 0u, 0u};
        tmem_st8(tmem + ((uint32_t)(warp * 32) << 16) + b * ACOLS + D / 2, ext);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull[b]);
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      sched::Cursor cur(A.tiles_per_cta, A.total_tiles);
      for (int it = 0;; ++it) {
        const int64_t g = sched::next_tile(cur);
        sched::ring_put(ring, it, (int32_t)g);
        const int st = it % NS;
        if (!mbar_wait(&empty[st], (uint32_t)((it / NS) & 1) ^ 1u, 0x192)) break;
        if (g < 0) {  // the end: a plain arrive completes the stage with no bytes
          mbar_arrive(&loaded[st]);
          break;
        }
        const int cell = (int)(g / A.tiles_per_cell);
        const int64_t tile = g % A.tiles_per_cell;
        const int h = (int)(tile / A.tb_per_head);
        const int64_t i0 = (tile % A.tb_per_head) * TILE_M;
        const bool tload = FOLD && A.rt > 0;
        const uint32_t tbytes = !tload ? 0u : A.rows_direct ? TILE_M * 2u : L::T_BYTES;
        mbar_expect_tx(&loaded[st], L::C_BYTES + tbytes);
        tma_load_3d(sbase + L::OFF_C + st * L::C_BYTES, &cmaps.m[cell], 0, (int)(A.t0 + i0), h, &loaded[st]);
        if (tload && A.rows_direct) {
          // u_token of the tile's 128 tokens (t0 + i0 .. + 127), 256 bytes
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES,
                    static_cast<const uint8_t*>(A.ut.p[cell]) + (A.t0 + i0) * 2, TILE_M * 2u, &loaded[st]);
        } else if (tload) {
          const int64_t base = (int64_t)cell * A.m * A.tl + (int64_t)h * A.tl + i0;
          bulk_load(sbase + L::OFF_T + st * L::T_BYTES, A.tmp + (base & ~(int64_t)3), L::T_BYTES, &loaded[st]);
        }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // D[row][n] = sum_k q[row][k] scale[k] Pi[k][n]
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(TILE_M, D, true);
      int it = 0, cur_cell = -1, nb = 0;
      bool ended = false;
      for (;; ++it) {
        const int b = it & 1, ac = it & 1;
        if (!mbar_wait(&afull[b], (uint32_t)((it >> 1) & 1), 0x292)) break;
        const int32_t g = sched::ring_get(ring, it);
        if (!mbar_wait(&acce[ac], (uint32_t)((it >> 1) & 1) ^ 1u, 0x293)) break;
        if (g < 0) {  // the end: the epilogue learns it from the same accumulator barrier
          umma_commit(&accf[ac]);
          ended = true;
          break;
        }
        const int cell = (int)(g / A.tiles_per_cell);
        if (cell != cur_cell) {
          // diag(scale) Pi of the new cell: after this thread's MMAs on the old one
          if (cur_cell >= 0) {
            umma_commit(bfree);
            if (!mbar_wait(bfree, (uint32_t)((nb - 1) & 1), 0x291)) break;
          }
          mbar_expect_tx(bready, L::B_BYTES);
          const uint8_t* src = A.bimg + (size_t)cell * L::B_BYTES;
#pragma unroll
          for (int term = 0; term < L::NTB; ++term)
            bulk_load(sbase + term * L::B_TERM, src + term * L::B_TERM, L::B_TERM, bready);
          if (FOLD) bulk_load(sbase + 2 * L::B_TERM, src + 2 * L::B_TERM, L::B_TUCKER, bready);
          if (!mbar_wait(bready, (uint32_t)(nb & 1), 0x295)) break;
          ++nb;
          cur_cell = cell;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + TM_ACC + (uint32_t)(ac * D);
        // the smaller terms first
#pragma unroll
        for (int tt = 0; tt < L::NTB; ++tt) {
          const int term = L::NTB - 1 - tt;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t kb = (uint32_t)((ks >> 2) * (D * 128) + (ks & 3) * 32);
            umma_f16_ts(d_tmem, tmem + b * ACOLS + (uint32_t)(ks * 8), desc_sw128(sbase + term * L::B_TERM + kb),
                        idesc, (tt | ks) ? 1u : 0u);
          }
        }
        if (FOLD)  // + t_row * u_feature: K positions 0-5 of the extra block
          umma_f16_ts(d_tmem, tmem + b * ACOLS + (uint32_t)(D / 2), desc_sw128(sbase + 2 * L::B_TERM), idesc, 1u);
        umma_commit(&afree[b]);
        umma_commit(&accf[ac]);
      }
      if (ended) mbar_wait(&accf[it & 1], (uint32_t)(it >> 1) & 1u, 0x294);
      else if (it > 0) mbar_wait(&accf[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, 0x294);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: thread = row, D/2 features per warp ----------------
    const int e = warp - EPI_WARP0;
    const int lg = warp & 3;
    const int half = e >> 2;
    const int rloc = lg * 32 + lane;
    constexpr int NCH = D / 64;
    float* us = reinterpret_cast<float*>(smem + L::OFF_U + e * L::U_BYTES);  // [feature][RDM]
    // the warp's 32 rows x D/2 outputs (ROW_BYTES a row) are staged with the
    // swizzle of that width (16-byte chunk j of row r at j ^ ((r * ROW_BYTES /
    // 128) mod (ROW_BYTES / 16)), conflict-free) and leave by one TMA store
    constexpr int RB = (int)L::ROW_BYTES;
    uint8_t* stg = smem + L::OFF_O + e * L::O_BYTES;
    const int swz = ((lane * RB) >> 7) & (RB / 16 - 1);
    uint8_t* srow = stg + lane * RB;
    int cur_cell = -1;
    for (int it = 0;; ++it) {
      const int ac = it & 1;
      if (!warp_wait(&accf[ac], (uint32_t)((it >> 1) & 1), 0x391)) break;
      const int32_t g = sched::ring_get(ring, it);
      if (g < 0) break;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t tile = g % A.tiles_per_cell;
      const int64_t h = tile / A.tb_per_head;
      const int64_t i_tok = (tile % A.tb_per_head) * TILE_M + rloc;  // token within [t0, t1)
      const bool valid = i_tok < A.tl;
      const int64_t orow = h * A.tl + i_tok;  // row of the Tucker term
      if (!FOLD && cell != cur_cell) {
        __syncwarp();
        if (A.rt > 0)
          for (int i = lane; i < (D / 2) * RDM; i += 32) {
            const int jl = i / RDM, r = i % RDM;
            us[i] = r < A.rd ? load_dt(A.ud.p[cell], (int64_t)(half * (D / 2) + jl) * A.rd + r, A.factor_dtype)
                             : 0.f;
          }
        __syncwarp();
        cur_cell = cell;
      }
      float tv[RDM];  // this row's Tucker term (rd > 1), loaded before the wait
#pragma unroll
      for (int r = 0; r < RDM; ++r)
        tv[r] = (!FOLD && valid && A.rt > 0) ? __ldg(A.tmp + ((int64_t)cell * A.m * A.tl + orow) * RDM + r) : 0.f;
      tc_fence_after();
      // the previous tile's store has read the staging rows
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int c = half * NCH + cc;
        float v[32];
        tmem_ld32(tmem + TM_ACC + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ac * D + c * 32), v);
        uint32_t o[16];
        if constexpr (O32) {
          float oo[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (A.rt > 0) {
              const int f = cc * 32 + j;
              float rec = 0.f;
              if (RDM == 1) {
                rec = tv[0] * us[f];
              } else {
                const float4* u4 = reinterpret_cast<const float4*>(us + f * RDM);
#pragma unroll
                for (int r4 = 0; r4 < RDM / 4; ++r4) {
                  const float4 u = u4[r4];
                  rec = fmaf(tv[4 * r4], u.x, rec);
                  rec = fmaf(tv[4 * r4 + 1], u.y, rec);
                  rec = fmaf(tv[4 * r4 + 2], u.z, rec);
                  rec = fmaf(tv[4 * r4 + 3], u.w, rec);
                }
              }
              oo[j] = __fadd_rn(rec, v[j]);
            } else {
              oo[j] = v[j];
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(srow + (((cc * 8 + q) ^ swz) << 4)) =
                make_float4(oo[4 * q], oo[4 * q + 1], oo[4 * q + 2], oo[4 * q + 3]);
          continue;
        }
        if (FOLD) {
          // the accumulator already holds residual + Tucker term
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const __nv_bfloat162 hh = __floats2bfloat162_rn(v[j], v[j + 1]);
            o[j / 2] = *reinterpret_cast<const uint32_t*>(&hh);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float oo[2];
#pragma unroll
            for (int x = 0; x < 2; ++x) {
              if (A.rt > 0) {
                const int f = cc * 32 + j + x;
                float rec = 0.f;
                if (RDM == 1) {
                  rec = tv[0] * us[f];
                } else {
                  const float4* u4 = reinterpret_cast<const float4*>(us + f * RDM);
#pragma unroll
                  for (int r4 = 0; r4 < RDM / 4; ++r4) {
                    const float4 u = u4[r4];
                    rec = fmaf(tv[4 * r4], u.x, rec);
                    rec = fmaf(tv[4 * r4 + 1], u.y, rec);
                    rec = fmaf(tv[4 * r4 + 2], u.z, rec);
                    rec = fmaf(tv[4 * r4 + 3], u.w, rec);
                  }
                }
                oo[x] = __fadd_rn(rec, v[j + x]);
              } else {
                oo[x] = v[j + x];
              }
            }
            const __nv_bfloat162 hh = __floats2bfloat162_rn(oo[0], oo[1]);
            o[j / 2] = *reinterpret_cast<const uint32_t*>(&hh);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(srow + (((cc * 4 + q) ^ swz) << 4)) =
              make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
      tc_fence_before();
      mbar_arrive(&acce[ac]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        // rows at or past tl are clipped by the store
        const int i0 = (int)((tile % A.tb_per_head) * TILE_M + lg * 32);
        tma_store_3d(&omaps.m[cell], half * (D / 2), i0, (int)h, smem_u32(stg));
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait<0>();  // shared memory outlives the stores
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// B images of the decode, per cell: B[n][k] = scale[k] * Pi[k][n] in two
// bf16 terms (three for fp32 output), swizzled K-major [cell][term] (D[row][n] = sum_k q[row][k] B[n][k]),
// then (rd = 1) the Tucker block B[n][k] for k < 64: u_feature[n] split
// hi + lo at k = 0-2 and 3-5 (the A side holds t_row split hi + mid + lo
// twice), zero elsewhere; zero throughout when there is no Tucker term.
__global__ void prep_decode_kernel(const float* __restrict__ proj, CellPtrs scale, CellPtrs ufeat, int fdt,
                                   int tucker_block, int nterm, int d, uint8_t* out) {
  const int cell = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t per_cell = (size_t)nterm * d * d * 2 + (tucker_block ? (size_t)d * 128 : 0);
  uint8_t* base = out + (size_t)cell * per_cell;
  if (e < d * d) {
    const int n = e / d, k = e % d;
    const float sk = static_cast<const float*>(scale.p[cell])[k];
    float rest = __fmul_rn(sk, proj[(int64_t)k * d + n]);
    for (int term = 0; term < nterm; ++term) {
      const __nv_bfloat16 v = __float2bfloat16_rn(rest);
      rest -= __bfloat162float(v);
      *reinterpret_cast<__nv_bfloat16*>(base + (size_t)term * d * d * 2 + sw128_off(n, k, d)) = v;
    }
  } else if (tucker_block && e < d * d + d * 64) {
    const int n = (e - d * d) / 64, k = (e - d * d) % 64;
    float v = 0.f;
    if (k < 6 && ufeat.p[cell]) {
      const float u = load_dt(ufeat.p[cell], n, fdt);
      const float hi = __bfloat162float(__float2bfloat16_rn(u));
      v = k < 3 ? hi : u - hi;
    }
    *reinterpret_cast<__nv_bfloat16*>(base + (size_t)2 * d * d * 2 + sw128_off(n, k, d)) = __float2bfloat16_rn(v);
  }
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  return KVC_OK;
}

}  // namespace

// Row terms of the SIMT residual passes: tmp[cell][row][stride] (rows = m * t
// per cell) rounded to the cell dtype, as the reference's einsum intermediate.
int simt_row_terms(const void* const* core, const void* const* ut, int n_cells, int dtype, int64_t m, int64_t t,
                   int rt, int rd, int stride, float* tmp, cudaStream_t st) {
  CellPtrs cp, up;
  for (int c = 0; c < n_cells; ++c) {
    cp.p[c] = core[c];
    up.p[c] = ut[c];
  }
  return row_terms_launch(cp, up, n_cells, dtype, dtype, m, 0, t, rt, rd, stride, m * t, tmp, st);
}

// ------------------------------- launchers --------------------------------

// bf16 cells: rd up to 4 for d = 64 and 128, up to 16 for d = 128 (the
// quantise pass then needs its feature-major form: tc_quant_fm_eligible);
// fp32 cells: d = 64, rd up to 4 (tc_enc32_kernel).
bool tc_residual_eligible(int dtype, int d, int rd, const float* proj, int scale_mode) {
  const bool shape = dtype == KVC_BF16 ? (d == 64 || d == 128) && (rd <= 4 || (rd <= 16 && d == 128))
                                       : dtype == KVC_F32 && d == 64 && rd <= 4;
  return shape && proj != nullptr && (scale_mode == KVC_SCALE_CHANNEL || scale_mode == KVC_SCALE_TENSOR);
}

bool tc_quant_fm_eligible(int d, int bits, int scale_mode, int arith_dtype) {
  return kernel_policy() != 3 && d == 128 && (bits == 8 || bits == 4) &&
         (scale_mode != KVC_SCALE_TENSOR || arith_dtype == KVC_F32);
}

size_t tc_residual_workspace(int n_cells, int64_t rows, int d, int rd) {
  const int64_t rows_pad = ceil_div(rows, TILE_M) * TILE_M;
  return align256((size_t)3 * 128 * (d / 2) * 4) + align256((size_t)n_cells * 2 * d * sizeof(int32_t)) +
         align256((size_t)n_cells * rows_pad * rdm_enc(rd) * 4) + align256((size_t)n_cells * 3 * d * d * 2) +
         align256((size_t)n_cells * 4) + align256((size_t)n_cells * (1 + d) * 4) + align256((size_t)128 * 4) +
         align256((size_t)n_cells * 4);
}

// The Tucker row terms a stats launch left in its workspace, per host thread:
// a quantise launch on the same workspace, cells and factors may use them
// instead of recomputing them when its caller allows it
// (tc_reuse_tucker_rows: kvc_compress, whose quantise call follows its stats
// call on the same stream with nothing in between).
struct RowsKey {
  const void* ws;
  int n_cells, rdm;
  int64_t rows;
  const void* core0;
  const void* ut0;
};
static thread_local RowsKey tl_rows_key = {nullptr, 0, 0, 0, nullptr, nullptr};
static thread_local bool tl_rows_reuse = false;

void tc_reuse_tucker_rows(bool allow) { tl_rows_reuse = allow; }

// The feature Gram of the cells of the next stats launch on this host thread
// (kvc_compress, whose Gram is still intact then): it bounds |R| per cell
// for the fp16 stats pass.  NULL: none.
static thread_local const double* tl_stats_gram = nullptr;
static thread_local int64_t tl_stats_gram_stride = 0;
void tc_stats_gram_bound(const double* gram, int64_t stride) {
  tl_stats_gram = gram;
  tl_stats_gram_stride = stride;
}

// One quantise launch, the code width as a template argument (the epilogue's
// packing and store path fixed at compile time).
template <int D, bool SYM, int RDM, int NS, bool F16, int BITS>
int launch_quant_bits(dim3 grid, cudaStream_t st, const TmaMaps& xmaps, const TmaMaps& cmaps, const EncArgs& a,
                      const uint8_t* bimg) {
  auto kern = tc_quant_kernel<D, SYM, RDM, NS, F16, BITS>;
  constexpr size_t sm = QuantLayout<D, RDM, NS, F16>::BYTES;
  int rc;
  if ((rc = set_smem(kern, sm))) return rc;
  kern<<<grid, NTHREADS, sm, st>>>(xmaps, cmaps, a, bimg);
  return KVC_OK;
}
template <int D, bool SYM, int RDM, int NS, bool F16>
int launch_quant(int bits, dim3 grid, cudaStream_t st, const TmaMaps& xmaps, const TmaMaps& cmaps, const EncArgs& a,
                 const uint8_t* bimg) {
  switch (bits) {
    case 8: return launch_quant_bits<D, SYM, RDM, NS, F16, 8>(grid, st, xmaps, cmaps, a, bimg);
    case 4: return launch_quant_bits<D, SYM, RDM, NS, F16, 4>(grid, st, xmaps, cmaps, a, bimg);
    case 2: return launch_quant_bits<D, SYM, RDM, NS, F16, 2>(grid, st, xmaps, cmaps, a, bimg);
    default: return fail(KVC_ERR_ARG, "tensor-core quantise: bits must be 2, 4 or 8");
  }
}

constexpr int QFM_NS = 5;  // x stages of the feature-major quantise pass
template <bool SYM, int RDM, bool F16 = false>
int launch_quantfm(int bits, dim3 grid, cudaStream_t st, const TmaMaps& xmaps, const TmaMaps& cmaps, const EncArgs& a,
                   const uint32_t* arows) {
  // 16 row terms a row: fewer stages for the larger row-term and u_feature tables
  constexpr int NSQ = RDM == 16 ? 3 : QFM_NS;
  constexpr size_t sm = QuantFmLayout<RDM, NSQ>::BYTES;
  int rc;
  if (bits == 8) {
    auto kern = tc_quantfm_kernel<SYM, RDM, NSQ, 8, F16>;
    if ((rc = set_smem(kern, sm))) return rc;
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, cmaps, a, arows);
  } else {
    auto kern = tc_quantfm_kernel<SYM, RDM, NSQ, 4, F16>;
    if ((rc = set_smem(kern, sm))) return rc;
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, cmaps, a, arows);
  }
  return KVC_OK;
}

template <bool STATS, bool SYM, int RDM>
int launch_enc32(int bits, dim3 grid, cudaStream_t st, const TmaMaps& xmaps, const TmaMaps& cmaps, const EncArgs& a,
                 const uint8_t* bimg) {
  constexpr int NS = 5;
  constexpr size_t sm = Enc32Layout<RDM, NS>::BYTES;
  int rc;
#define KVC_ENC32(BB)                                                  \
  do {                                                                 \
    auto kern = tc_enc32_kernel<STATS, SYM, RDM, NS, BB>;              \
    if ((rc = set_smem(kern, sm))) return rc;                          \
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, cmaps, a, bimg);           \
  } while (0)
  if constexpr (STATS) {
    KVC_ENC32(8);  // the code width does not enter the stats pass
  } else {
    if (bits == 8) KVC_ENC32(8);
    else if (bits == 4) KVC_ENC32(4);
    else if (bits == 2) KVC_ENC32(2);
    else return fail(KVC_ERR_ARG, "tensor-core quantise: bits must be 2, 4 or 8");
  }
#undef KVC_ENC32
  return check_launch(STATS ? "tc_enc32_kernel (stats)" : "tc_enc32_kernel (quantise)");
}

// Both encode passes of fp32 cells with head_dim 64 (tc_enc32_kernel); the
// workspace is carved as for the bf16 passes.
static int tc_residual_f32_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d,
                           const void* const* core, const void* const* u_token, const void* const* u_feature,
                           int rt, int rd, const float* proj, int bits, int symmetric, int scale_mode,
                           int stat_dtype, int arith_dtype, float* const* scale, int32_t* const* zp,
                           uint8_t* const* codes, void* workspace, cudaStream_t st) {
  const int64_t rows = m * t;
  const int rdm = rdm_enc(rd);
  TmaMaps xmaps, cmaps;
  EncArgs a;
  memset(&a, 0, sizeof(a));
  memset(&cmaps, 0, sizeof(cmaps));
  const int cbw = (d / 2) * bits / 8;
  const int cb = (d * bits + 7) / 8;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    // rows of 64 floats: two boxes of 32 floats (128 bytes) x 128 rows
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)d * 4};
    const uint32_t box[2] = {32u, (uint32_t)TILE_M};
    if ((rc = encode_tma(&xmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, x[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (mode == 1 && cbw >= 16) {
      const uint64_t cd[2] = {(uint64_t)cb, (uint64_t)rows};
      const uint64_t cs[1] = {(uint64_t)cb};
      const uint32_t cbx[2] = {(uint32_t)cbw, 32u};
      const CUtensorMapSwizzle sw = cbw == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
      if ((rc = encode_tma(&cmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, codes[c], cd, cs, cbx, sw))) return rc;
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
  const int64_t ctas = std::min<int64_t>(std::min<int64_t>(a.total_tiles, num_sms()), kMaxCtas);
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  size_t off = align256((size_t)3 * 128 * (d / 2) * 4);
  int32_t* mm = reinterpret_cast<int32_t*>(ws + off);
  off += align256((size_t)n_cells * 2 * d * sizeof(int32_t));
  float* tmp = reinterpret_cast<float*>(ws + off);
  off += align256((size_t)n_cells * a.tiles_per_cell * TILE_M * rdm * 4);
  uint8_t* bimg = ws + off;  // n_cells x 3 x d x d bf16
  a.minmax = mm;
  a.tmp = tmp;
  const RowsKey key = {workspace, n_cells, rdm, rows, rt > 0 ? core[0] : nullptr, rt > 0 ? u_token[0] : nullptr};
  const bool after_stats = mode == 1 && tl_rows_reuse && tl_rows_key.ws == key.ws &&
                           tl_rows_key.n_cells == key.n_cells && tl_rows_key.rdm == key.rdm &&
                           tl_rows_key.rows == key.rows && tl_rows_key.core0 == key.core0 &&
                           tl_rows_key.ut0 == key.ut0;
  tl_rows_key = RowsKey{nullptr, 0, 0, 0, nullptr, nullptr};
  CellPtrs sp;
  for (int c = 0; c < n_cells; ++c) sp.p[c] = scale ? scale[c] : nullptr;
  if (mode == 0) {
    // Pi in three terms, one image for every cell
    prep_quant_b_kernel<<<dim3((d * d + 255) / 256, 1), 256, 0, st>>>(proj, sp, 0, 0, d, bimg);
    if ((rc = check_launch("prep_quant_b_kernel"))) return rc;
  } else {
    const int fold = scale_mode != KVC_SCALE_TENSOR || arith_dtype == KVC_F32;
    prep_quant_b_kernel<<<dim3((d * d + 255) / 256, n_cells), 256, 0, st>>>(
        proj, sp, scale_mode == KVC_SCALE_CHANNEL, fold, d, bimg);
    if ((rc = check_launch("prep_quant_b_kernel"))) return rc;
  }
  if (rt > 0 && !after_stats) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    if ((rc = row_terms_launch(cp, up, n_cells, KVC_F32, KVC_F32, m, 0, t, rt, rd, rdm, a.tiles_per_cell * TILE_M,
                               tmp, st)))
      return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  const bool sym = symmetric != 0;
  if (mode == 0) {
    minmax_init_kernel<<<(n_cells * 2 * d + 255) / 256, 256, 0, st>>>(mm, n_cells, d, nullptr);
    if ((rc = check_launch("minmax_init_kernel"))) return rc;
    if (sym) rc = rdm == 1 ? launch_enc32<true, true, 1>(bits, grid, st, xmaps, cmaps, a, bimg)
                           : launch_enc32<true, true, 4>(bits, grid, st, xmaps, cmaps, a, bimg);
    else rc = rdm == 1 ? launch_enc32<true, false, 1>(bits, grid, st, xmaps, cmaps, a, bimg)
                       : launch_enc32<true, false, 4>(bits, grid, st, xmaps, cmaps, a, bimg);
    if (rc) return rc;
    CellPtrsMut sc, zz;
    for (int c = 0; c < n_cells; ++c) {
      sc.p[c] = scale[c];
      zz.p[c] = zp[c];
    }
    minmax_finalize_kernel<<<n_cells, 128, 0, st>>>(mm, n_cells, d, bits, symmetric, scale_mode, stat_dtype, sc, zz);
    if ((rc = check_launch("minmax_finalize_kernel"))) return rc;
    tl_rows_key = key;  // the row terms stay in the workspace for a following quantise launch
    return KVC_OK;
  }
  if (sym) rc = rdm == 1 ? launch_enc32<false, true, 1>(bits, grid, st, xmaps, cmaps, a, bimg)
                         : launch_enc32<false, true, 4>(bits, grid, st, xmaps, cmaps, a, bimg);
  else rc = rdm == 1 ? launch_enc32<false, false, 1>(bits, grid, st, xmaps, cmaps, a, bimg)
                     : launch_enc32<false, false, 4>(bits, grid, st, xmaps, cmaps, a, bimg);
  return rc;
}

int tc_residual_launch(int mode, int n_cells, const void* const* x, int64_t m, int64_t t, int d, int dtype,
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
  if (dtype == KVC_F32) {
    if (d != 64 || rdm > 4) return fail(KVC_ERR_UNSUPPORTED, "tensor-core residual: fp32 cells need d = 64, rd <= 4");
    return tc_residual_f32_launch(mode, n_cells, x, m, t, d, core, u_token, u_feature, rt, rd, proj, bits, symmetric,
                                  scale_mode, stat_dtype, arith_dtype, scale, zp, codes, workspace, st);
  }
  if (dtype != KVC_BF16) return fail(KVC_ERR_DTYPE, "tensor-core residual: bf16 or fp32 cells");
  TmaMaps xmaps, cmaps;  // copied into the launch parameters
  EncArgs a;
  memset(&a, 0, sizeof(a));
  memset(&cmaps, 0, sizeof(cmaps));
  const int cbw = (d / 2) * bits / 8;  // code bytes of half a row (one epilogue warp)
  const int cb = (d * bits + 7) / 8;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)d * 2};
    const uint32_t box[2] = {64u, (uint32_t)TILE_M};
    if ((rc = encode_tma(&xmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x[c], dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (mode == 1 && cbw >= 16) {
      // codes of 32 rows x half a row, swizzled by the half-row width
      const uint64_t cd[2] = {(uint64_t)cb, (uint64_t)rows};
      const uint64_t cs[1] = {(uint64_t)cb};
      const uint32_t cbx[2] = {(uint32_t)cbw, 32u};
      const CUtensorMapSwizzle sw = cbw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                    : cbw == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
      if ((rc = encode_tma(&cmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, codes[c], cd, cs, cbx, sw))) return rc;
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
  const int64_t ctas = std::min<int64_t>(std::min<int64_t>(a.total_tiles, num_sms()), kMaxCtas);
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* arows = reinterpret_cast<uint32_t*>(ws);
  size_t off = align256((size_t)3 * 128 * (d / 2) * 4);
  int32_t* mm = reinterpret_cast<int32_t*>(ws + off);
  off += align256((size_t)n_cells * 2 * d * sizeof(int32_t));
  float* tmp = reinterpret_cast<float*>(ws + off);
  off += align256((size_t)n_cells * a.tiles_per_cell * TILE_M * rdm * 4);
  uint8_t* bimg = ws + off;  // quantise: n_cells x 3 x d x d 16-bit
  off += align256((size_t)n_cells * 3 * d * d * 2);
  uint32_t* rmax = reinterpret_cast<uint32_t*>(ws + off);  // stats: max |R| per cell
  off += align256((size_t)n_cells * 4);
  float* fscale = reinterpret_cast<float*>(ws + off);  // fp16 quantise: 2^E, 2^-(E + G_n) per cell
  off += align256((size_t)n_cells * (1 + d) * 4);
  int32_t* gexp = reinterpret_cast<int32_t*>(ws + off);  // fp16 stats: G_n per A row
  off += align256((size_t)128 * 4);
  int32_t* sexp = reinterpret_cast<int32_t*>(ws + off);  // fp16 stats: E per cell (bounded |R|)
  a.gexp = gexp;
  a.arows = arows;
  a.minmax = mm;
  a.tmp = tmp;
  a.rmax = mode == 0 ? rmax : nullptr;
  // the stats pass takes Pi as TMEM rows, the quantise pass Pi / s of each
  // cell as shared-memory B images
  // policy 2: the stats pass in two fp16 terms of Pi (rank-1 row terms,
  // d = 128), a third fewer MMAs than three bf16 terms.  R's power of two
  // is per cell where the feature Gram bounds |R| (inside kvc_compress),
  // else per 128-row tile (agreed between the transform warps).  Not the
  // default: in the compress pipeline on B200 both forms measured slower
  // than the bf16 pass (the conversion makes the transform the critical
  // path; the bf16 pass is held by its MMAs only a little longer)
  const bool gram_bound = tl_stats_gram != nullptr && mode == 0 && rd == 1;
  const bool f16s = mode == 0 && d == 128 && rdm == 1 && rt > 0 && kernel_policy() == 2;
  if (f16s && gram_bound) {
    CellPtrs cp, up, dp;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
      dp.p[c] = u_feature[c];
    }
    stats_bound_kernel<<<n_cells, 256, 0, st>>>(tl_stats_gram, tl_stats_gram_stride, d, cp, up, dp, m * rt, t * rt, d,
                                                rt, sexp);
    if ((rc = check_launch("stats_bound_kernel"))) return rc;
    a.sexp = sexp;
  }
  if (f16s) {
    prep_rotation16_kernel<<<128, d / 2, 0, st>>>(proj, d, arows, gexp);
    if ((rc = check_launch("prep_rotation16_kernel"))) return rc;
  } else if (mode == 0) {
    prep_rotation_kernel<<<(128 * (d / 2) + 255) / 256, 256, 0, st>>>(proj, d, arows);
    if ((rc = check_launch("prep_rotation_kernel"))) return rc;
  }
  const RowsKey key = {workspace, n_cells, rdm, rows, rt > 0 ? core[0] : nullptr, rt > 0 ? u_token[0] : nullptr};
  // the stats launch just before on this workspace and these cells left
  // max |R| per cell: the quantise pass may take its fp16 mode
  const bool after_stats = mode == 1 && tl_rows_reuse && tl_rows_key.ws == key.ws &&
                           tl_rows_key.n_cells == key.n_cells && tl_rows_key.rdm == key.rdm &&
                           tl_rows_key.rows == key.rows && tl_rows_key.core0 == key.core0 &&
                           tl_rows_key.ut0 == key.ut0;
  // the quantise pass's fp16 mode (after a stats launch on these cells,
  // which leaves max |R| per cell): by default with the feature-major pass
  // (measured faster), with either pass under policy 2
  const int pol = kernel_policy();
  const bool fm = mode == 1 && tc_quant_fm_eligible(d, bits, scale_mode, arith_dtype);
  if (mode == 1 && rdm == 16 && !fm)
    return fail(KVC_ERR_UNSUPPORTED, "tensor-core quantise: rd > 4 needs d = 128 and 8- or 4-bit codes");
  const bool f16_ok = after_stats && d == 128 && rdm == 1 && rt > 0 && scale_mode == KVC_SCALE_CHANNEL;
  const bool f16 = f16_ok && ((pol == 0 && fm) || pol == 2);
  bool direct = rt == 1 && rd == 1 && t % TILE_M == 0 && m <= CORE_MAX;
  for (int c = 0; c < n_cells && direct; ++c) direct = (reinterpret_cast<uintptr_t>(u_token[c]) & 15u) == 0;
  a.rows_direct = direct ? 1 : 0;
  a.t_tok = t;
  if (direct) {
    for (int c = 0; c < n_cells; ++c) {
      a.core.p[c] = core[c];
      a.ut.p[c] = u_token[c];
    }
  }
  const bool rows_ready = direct || after_stats;
  tl_rows_key = RowsKey{nullptr, 0, 0, 0, nullptr, nullptr};
  // the feature-major quantise pass (d = 128, 8- / 4-bit codes, the
  // quantiser's fast path); policy 3 keeps the row-major one for comparison
  TmaMaps fmaps;
  if (fm) {
    memset(&fmaps, 0, sizeof(fmaps));
    const uint32_t fbw = (uint32_t)(32 * bits / 8);  // code bytes of 32 features
    for (int c = 0; c < n_cells; ++c) {
      const uint64_t cd[2] = {(uint64_t)cb, (uint64_t)rows};
      const uint64_t cst[1] = {(uint64_t)cb};
      const uint32_t cbx[2] = {fbw, (uint32_t)TILE_M};
      if ((rc = encode_tma(&fmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, codes[c], cd, cst, cbx,
                           CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    }
  }
  if (mode == 1) {
    CellPtrs sp;
    for (int c = 0; c < n_cells; ++c) sp.p[c] = scale[c];
    if (fm && !f16) {
      prep_quant_arows_kernel<<<dim3((d * (d / 2) + 255) / 256, n_cells), 256, 0, st>>>(
          proj, sp, scale_mode == KVC_SCALE_CHANNEL, d, reinterpret_cast<uint32_t*>(bimg));
      if ((rc = check_launch("prep_quant_arows_kernel"))) return rc;
    } else if (f16) {
      prep_quant_b16_kernel<<<dim3(d, n_cells), d, 0, st>>>(proj, sp, rmax, d, bimg, fscale, fm ? 1 : 0);
      if ((rc = check_launch("prep_quant_b16_kernel"))) return rc;
      a.fscale = fscale;
    } else {
      const int fold = scale_mode != KVC_SCALE_TENSOR || arith_dtype == KVC_F32;
      prep_quant_b_kernel<<<dim3((d * d + 255) / 256, n_cells), 256, 0, st>>>(
          proj, sp, scale_mode == KVC_SCALE_CHANNEL, fold, d, bimg);
      if ((rc = check_launch("prep_quant_b_kernel"))) return rc;
    }
  }
  if (rt > 0 && !rows_ready) {
    CellPtrs cp, up;
    for (int c = 0; c < n_cells; ++c) {
      cp.p[c] = core[c];
      up.p[c] = u_token[c];
    }
    if ((rc = row_terms_launch(cp, up, n_cells, KVC_BF16, KVC_BF16, m, 0, t, rt, rd, rdm, a.tiles_per_cell * TILE_M,
                               tmp, st)))
      return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  if (mode == 0) {
    minmax_init_kernel<<<(n_cells * 2 * d + 255) / 256, 256, 0, st>>>(mm, n_cells, d, rmax);
    if ((rc = check_launch("minmax_init_kernel"))) return rc;
  }
#define KVC_TC_STATS(DD, SYMV, RR, NSV)                 \
  do {                                                  \
    auto kern = tc_stats_kernel<DD, SYMV, RR, NSV>;     \
    constexpr size_t sm = StatsLayout<DD, RR, NSV>::BYTES; \
    if ((rc = set_smem(kern, sm))) return rc;           \
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, a);         \
  } while (0)
#define KVC_TC_STATS16(SYMV)                                 \
  do {                                                       \
    auto kern = tc_stats_kernel<128, SYMV, 1, 6, true>;      \
    constexpr size_t sm = StatsLayout<128, 1, 6, true>::BYTES; \
    if ((rc = set_smem(kern, sm))) return rc;                \
    kern<<<grid, NTHREADS, sm, st>>>(xmaps, a);              \
  } while (0)
#define KVC_TC_QUANT(DD, SYMV, RR, NSV)                                                          \
  do {                                                                                           \
    if ((rc = launch_quant<DD, SYMV, RR, NSV, false>(bits, grid, st, xmaps, cmaps, a, bimg))) return rc; \
  } while (0)
#define KVC_TC_QUANT16(SYMV)                                                                     \
  do {                                                                                           \
    if ((rc = launch_quant<128, SYMV, 1, 4, true>(bits, grid, st, xmaps, cmaps, a, bimg))) return rc; \
  } while (0)
#define KVC_TC_ENC_R(WHICH, DD, SYMV, NSV)     \
  do {                                         \
    if (rdm == 1) WHICH(DD, SYMV, 1, NSV);     \
    else WHICH(DD, SYMV, 4, NSV);              \
  } while (0)
  const bool sym = symmetric != 0;
  if (mode == 0) {
    if (f16s) {
      if (sym) KVC_TC_STATS16(true);
      else KVC_TC_STATS16(false);
    } else if (d == 128 && rdm == 16) {
      if (sym) KVC_TC_STATS(128, true, 16, 4);
      else KVC_TC_STATS(128, false, 16, 4);
    } else if (d == 128) {
      if (sym) KVC_TC_ENC_R(KVC_TC_STATS, 128, true, 6);
      else KVC_TC_ENC_R(KVC_TC_STATS, 128, false, 6);
    } else {
      if (sym) KVC_TC_ENC_R(KVC_TC_STATS, 64, true, 8);
      else KVC_TC_ENC_R(KVC_TC_STATS, 64, false, 8);
    }
  } else {
    if (fm) {
      const uint32_t* ar = reinterpret_cast<const uint32_t*>(bimg);
      if (f16) {
        if (sym) rc = launch_quantfm<true, 1, true>(bits, grid, st, xmaps, fmaps, a, ar);
        else rc = launch_quantfm<false, 1, true>(bits, grid, st, xmaps, fmaps, a, ar);
      } else if (rdm == 1) {
        if (sym) rc = launch_quantfm<true, 1>(bits, grid, st, xmaps, fmaps, a, ar);
        else rc = launch_quantfm<false, 1>(bits, grid, st, xmaps, fmaps, a, ar);
      } else if (rdm == 16) {
        if (sym) rc = launch_quantfm<true, 16>(bits, grid, st, xmaps, fmaps, a, ar);
        else rc = launch_quantfm<false, 16>(bits, grid, st, xmaps, fmaps, a, ar);
      } else {
        if (sym) rc = launch_quantfm<true, 4>(bits, grid, st, xmaps, fmaps, a, ar);
        else rc = launch_quantfm<false, 4>(bits, grid, st, xmaps, fmaps, a, ar);
      }
      if (rc) return rc;
    } else if (f16) {
      // two fp16 terms of Pi / s (64 KB) leave room for a fourth x stage
      if (sym) KVC_TC_QUANT16(true);
      else KVC_TC_QUANT16(false);
    } else if (d == 128) {
      if (sym) KVC_TC_ENC_R(KVC_TC_QUANT, 128, true, 3);
      else KVC_TC_ENC_R(KVC_TC_QUANT, 128, false, 3);
    } else {
      if (sym) KVC_TC_ENC_R(KVC_TC_QUANT, 64, true, 6);
      else KVC_TC_ENC_R(KVC_TC_QUANT, 64, false, 6);
    }
  }
#undef KVC_TC_ENC_R
#undef KVC_TC_QUANT16
#undef KVC_TC_QUANT
#undef KVC_TC_STATS16
#undef KVC_TC_STATS
  if ((rc = check_launch(mode == 0 ? "tc_stats_kernel" : "tc_quant_kernel"))) return rc;
  if (mode == 0) {
    CellPtrsMut sc, zz;
    for (int c = 0; c < n_cells; ++c) {
      sc.p[c] = scale[c];
      zz.p[c] = zp[c];
    }
    minmax_finalize_kernel<<<n_cells, 128, 0, st>>>(mm, n_cells, d, bits, symmetric, scale_mode, stat_dtype, sc, zz);
    if ((rc = check_launch("minmax_finalize_kernel"))) return rc;
    tl_rows_key = key;  // the row terms stay in the workspace for a following quantise launch
  }
  return KVC_OK;
}

bool tc_decompress_eligible(int out_dtype, int d, int rd, int bits, int symmetric, int scale_mode,
                            const float* proj) {
  const bool out_ok = out_dtype == KVC_BF16 ? (d == 64 || d == 128) : out_dtype == KVC_F32 && d == 64;
  return out_ok && rd <= RD_MAX && bits > 0 && d * bits / 8 >= 16 && symmetric && scale_mode == KVC_SCALE_CHANNEL &&
         proj != nullptr;
}

// Bytes of one cell's decode B image: bf16 output two terms (+ the Tucker
// block at rd = 1), fp32 output three terms.
size_t dec_bimg_cell_bytes(int d, int rd, bool o32) {
  return o32 ? (size_t)6 * d * d : (size_t)4 * d * d + (rdm_dec(rd) == 1 ? (size_t)128 * d : 0);
}

size_t tc_decompress_workspace(int n_cells, int64_t rows, int d, int rd) {
  // d = 64 may decode to fp32 (three terms)
  const size_t cellb = std::max(dec_bimg_cell_bytes(d, rd, false), d == 64 ? dec_bimg_cell_bytes(d, rd, true) : 0);
  return align256((size_t)n_cells * cellb) + align256((size_t)n_cells * rows * rdm_dec(rd) * 4 + 132 * 4);
}

// A decode plan holds what does not depend on the token range: the codes'
// tensor maps, the factor pointers and, in its workspace, each cell's B image
// (built once by prep_decode_kernel).  Runs then decode any [t0, t1) with the
// Tucker-term kernel and the decode kernel only.
int tc_decode_plan_init(TcDecodePlan* p, int n_cells, const uint8_t* const* codes, const float* const* scale,
                        int bits, const void* const* core, const void* const* u_token,
                        const void* const* u_feature, int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd,
                        const float* proj, int out_dtype, void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (out_dtype != KVC_BF16 && !(out_dtype == KVC_F32 && d == 64))
    return fail(KVC_ERR_UNSUPPORTED, "tensor-core decompress: bf16 output, or fp32 output at d = 64");
  if (!workspace || ws_bytes < tc_decompress_workspace(n_cells, m * t, d, rd))
    return fail(KVC_ERR_WORKSPACE, "tensor-core decompress: workspace too small");
  if (t >= (1LL << 31) || m * t * rdm_dec(rd) >= (1LL << 31) || ceil_div(t, TILE_M) * m >= (1LL << 31))
    return fail(KVC_ERR_SHAPE, "tensor-core decompress: shape too large");
  memset(p, 0, sizeof(*p));
  p->n_cells = n_cells;
  p->d = d;
  p->bits = bits;
  p->rt = rt;
  p->rd = rd;
  p->factor_dtype = factor_dtype;
  p->out_dtype = out_dtype;
  p->m = m;
  p->t = t;
  const int cb = d * bits / 8;
  CellPtrs sc, uf;
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[3] = {(uint64_t)cb, (uint64_t)t, (uint64_t)m};
    const uint64_t strides[2] = {(uint64_t)cb, (uint64_t)cb * t};
    const uint32_t box[3] = {(uint32_t)cb, (uint32_t)TILE_M, 1u};
    // rows of 32 / 64 / 128 B take the swizzle of their width (the kernel
    // reads chunk c of row r at c ^ ((r * cb / 128) mod (cb / 16)))
    const CUtensorMapSwizzle swz = cb == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : cb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : cb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE;
    if ((rc = encode_tma(&p->cmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, codes[c], dims, strides, box, swz)))
      return rc;
    sc.p[c] = scale[c];
    uf.p[c] = rt > 0 ? u_feature[c] : nullptr;
    if (rt > 0) {
      p->core.p[c] = core[c];
      p->ut.p[c] = u_token[c];
      p->ud.p[c] = u_feature[c];
    }
  }
  const bool o32 = out_dtype == KVC_F32;
  const int tucker_block = rdm_dec(rd) == 1 && !o32;
  p->bimg = static_cast<uint8_t*>(workspace);
  p->tmp = reinterpret_cast<float*>(p->bimg + align256((size_t)n_cells * dec_bimg_cell_bytes(d, rd, o32)));
  prep_decode_kernel<<<dim3((d * d + d * 64 + 255) / 256, n_cells), 256, 0, st>>>(
      proj, sc, uf, factor_dtype, tucker_block, o32 ? 3 : 2, d, p->bimg);
  return check_launch("prep_decode_kernel");
}

int tc_decode_plan_run(const TcDecodePlan* p, int64_t t0, int64_t t1, void* const* out, cudaStream_t st) {
  const int n_cells = p->n_cells, d = p->d, bits = p->bits, rt = p->rt, rd = p->rd;
  const int64_t m = p->m, t = p->t;
  if (t0 < 0 || t1 > t || t0 >= t1) return fail(KVC_ERR_SHAPE, "tensor-core decompress: bad token range");
  const int64_t tl = t1 - t0;
  const int rdm = rdm_dec(rd);
  TmaMaps omaps;
  DecArgsTc a;
  memset(&a, 0, sizeof(a));
  int rc;
  for (int c = 0; c < n_cells; ++c) {
    if (!out[c] || (reinterpret_cast<uintptr_t>(out[c]) & 15u))
      return fail(KVC_ERR_ALIGN, "tensor-core decompress: output not 16-byte aligned");
    // output (m, tl, d): boxes of d/2 features x 32 tokens, swizzled by their
    // rows (bf16: d bytes; fp32 at d = 64: 128 bytes)
    const bool o32 = p->out_dtype == KVC_F32;
    const int esz = o32 ? 4 : 2;
    const uint64_t od[3] = {(uint64_t)d, (uint64_t)tl, (uint64_t)m};
    const uint64_t os[2] = {(uint64_t)d * esz, (uint64_t)d * esz * tl};
    const uint32_t ob[3] = {(uint32_t)(d / 2), 32u, 1u};
    if ((rc = encode_tma(&omaps.m[c], o32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                         out[c], od, os, ob,
                         (d == 128 || o32) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
    a.out.p[c] = out[c];
    if (rt > 0) a.ud.p[c] = p->ud.p[c];
  }
  a.m = m;
  a.t0 = t0;
  a.tl = tl;
  a.tb_per_head = (int)ceil_div(tl, TILE_M);
  a.tiles_per_cell = m * a.tb_per_head;
  a.total_tiles = a.tiles_per_cell * n_cells;
  const int64_t ctas = std::min<int64_t>(std::min<int64_t>(a.total_tiles, num_sms()), kMaxCtas);
  a.tiles_per_cta = ceil_div(a.total_tiles, ctas);
  a.rt = rt;
  a.rd = rd;
  a.factor_dtype = p->factor_dtype;
  a.bimg = p->bimg;
  a.tmp = p->tmp;
  // (fp32 output adds the row terms in its epilogue, from the row-term kernel)
  bool direct = rt == 1 && rd == 1 && (p->factor_dtype == KVC_F16 || p->factor_dtype == KVC_BF16) &&
                tl % TILE_M == 0 && t0 % 8 == 0 && p->out_dtype != KVC_F32;
  for (int c = 0; c < n_cells && direct; ++c)
    direct = (reinterpret_cast<uintptr_t>(p->ut.p[c]) & 15u) == 0;
  a.rows_direct = direct ? 1 : 0;
  if (direct) {
    for (int c = 0; c < n_cells; ++c) {
      a.core.p[c] = p->core.p[c];
      a.ut.p[c] = p->ut.p[c];
    }
  }
  if (rt > 0 && !direct) {
    if ((rc = row_terms_launch(p->core, p->ut, n_cells, p->factor_dtype, KVC_F32, m, t0, tl, rt, rd, rdm, m * tl,
                               p->tmp, st)))
      return rc;
  }
  const dim3 grid((unsigned)ceil_div(a.total_tiles, a.tiles_per_cta));
  const TmaMaps& cmaps = p->cmaps;
  // Inside stream capture (DecodeStream.capture: every block decodes into its
  // own outputs, with nothing else between the decodes), a run with rank-1
  // factors (no row-term scratch shared between runs) is launched as a
  // programmatic dependent of the run before it: consecutive runs are
  // independent, so this run's CTAs start on the SMs the previous one's
  // finishing CTAs free (its kernel lets dependents launch at once).  Only
  // for layouts of more than half an SM's shared memory: one CTA per SM, so
  // two runs never share an SM's tensor memory.
  bool pdl = false;
  if (direct) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    pdl = cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusActive;
  }
#define KVC_TC_DEC3(DD, RR, BB)                                                        \
  do {                                                                                 \
    constexpr int NSD = DecStages<DD, DD * BB / 8, RR>::value;                         \
    auto kern = tc_decode_kernel<DD, RR, BB, NSD>;                                     \
    using LL = DecLayout<DD, DD * BB / 8, RR, NSD>;                                    \
    if ((rc = set_smem(kern, LL::BYTES))) return rc;                                   \
    if (pdl && LL::BYTES > 116 * 1024) {                                               \
      cudaLaunchConfig_t cfg = {};                                                     \
      cfg.gridDim = grid;                                                              \
      cfg.blockDim = dim3(NTHREADS);                                                   \
      cfg.dynamicSmemBytes = LL::BYTES;                                                \
      cfg.stream = st;                                                                 \
      cudaLaunchAttribute attr[1];                                                     \
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                 \
      attr[0].val.programmaticStreamSerializationAllowed = 1;                          \
      cfg.attrs = attr;                                                                \
      cfg.numAttrs = 1;                                                                \
      const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, cmaps, omaps, a);          \
      if (le != cudaSuccess)                                                           \
        return fail(KVC_ERR_LAUNCH, std::string("tc_decode_kernel: ") + cudaGetErrorString(le)); \
    } else {                                                                           \
      kern<<<grid, NTHREADS, LL::BYTES, st>>>(cmaps, omaps, a);                        \
    }                                                                                  \
  } while (0)
#define KVC_TC_DEC(DD, RR)                      \
  do {                                          \
    if (bits == 8) KVC_TC_DEC3(DD, RR, 8);      \
    else if (bits == 4) KVC_TC_DEC3(DD, RR, 4); \
    else KVC_TC_DEC3(DD, RR, 2);                \
  } while (0)
#define KVC_TC_DEC32_3(RR, BB)                                                 \
  do {                                                                         \
    constexpr int NSD = DecStages<64, 64 * BB / 8, RR, true>::value;           \
    auto kern = tc_decode_kernel<64, RR, BB, NSD, true>;                       \
    using LL = DecLayout<64, 64 * BB / 8, RR, NSD, true>;                      \
    if ((rc = set_smem(kern, LL::BYTES))) return rc;                           \
    kern<<<grid, NTHREADS, LL::BYTES, st>>>(cmaps, omaps, a);                  \
  } while (0)
#define KVC_TC_DEC32(RR)                         \
  do {                                           \
    if (bits == 8) KVC_TC_DEC32_3(RR, 8);        \
    else if (bits == 4) KVC_TC_DEC32_3(RR, 4);   \
    else KVC_TC_DEC32_3(RR, 2);                  \
  } while (0)
  if (p->out_dtype == KVC_F32) {
    // d = 64 (checked when the plan was made)
    if (rdm == 1) KVC_TC_DEC32(1);
    else if (rdm == 4) KVC_TC_DEC32(4);
    else KVC_TC_DEC32(16);
  } else if (d == 128) {
    if (rdm == 1) KVC_TC_DEC(128, 1);
    else if (rdm == 4) KVC_TC_DEC(128, 4);
    else KVC_TC_DEC(128, 16);
  } else {
    // d = 64: 2-bit rows are 16 bytes, the smallest TMA row
    if (rdm == 1) KVC_TC_DEC(64, 1);
    else if (rdm == 4) KVC_TC_DEC(64, 4);
    else KVC_TC_DEC(64, 16);
  }
#undef KVC_TC_DEC32
#undef KVC_TC_DEC32_3
#undef KVC_TC_DEC3
#undef KVC_TC_DEC
  return check_launch("tc_decode_kernel");
}

int tc_decompress_launch(int n_cells, const uint8_t* const* codes, const float* const* scale, int bits,
                         const void* const* core, const void* const* u_token, const void* const* u_feature,
                         int factor_dtype, int64_t m, int64_t t, int d, int rt, int rd, const float* proj,
                         int64_t t0, int64_t t1, int out_dtype, void* const* out, void* workspace, size_t ws_bytes,
                         cudaStream_t st) {
  TcDecodePlan plan;
  int rc = tc_decode_plan_init(&plan, n_cells, codes, scale, bits, core, u_token, u_feature, factor_dtype, m, t, d,
                               rt, rd, proj, out_dtype, workspace, ws_bytes, st);
  if (rc) return rc;
  return tc_decode_plan_run(&plan, t0, t1, out, st);
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
