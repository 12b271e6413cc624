// Tensor-core feature-mode Gram + sketch: one pass over bf16 cells with
// head_dim 128 computes, per cell,
//   G = x^T x (128 x 128) and Y = x^T Omega (128 x k), k <= 32,
// the quantities the reference's randomised SVD extracts with five passes
// over the unfolding (kvcompress/compressor/svd.py:259-265, 289).
//
// Operands: an x tile of 128 rows staged by cp.async in the SWIZZLE_128B
// layout is at the same time the MN-major A operand (x^T: M = feature,
// K = row) and the MN-major B operand (x: N = feature); products of bf16
// values are exact and accumulate in fp32 in TMEM.  Omega (fp32) is staged
// per row, split in place into bf16 hi / lo (columns 0..31 / 32..63 of a
// 64-column MN-major B tile), so Y carries ~16 mantissa bits of Omega.
//
// Work: the global (cell, tile) list is cut into one contiguous segment per
// CTA; a CTA flushes its TMEM accumulator (two buffers) to a per-(cell,
// segment) fp32 partial whenever the cell changes or its range ends, and a
// second kernel sums the segments of each cell in order in fp64.  Results
// are bit-reproducible for a given batch of cells.
//
// Warps 0-3 produce (cp.async, 4 stages), warp 4 issues tcgen05.mma,
// warps 5-8 drain accumulators.  Every mbarrier wait is bounded.
#include <algorithm>

#include "kvc_common.cuh"
#include "kvc_tc.cuh"

namespace kvc {
namespace {

using namespace tc;

constexpr int D = 128;        // head_dim handled here
constexpr int TILE = 128;     // rows per tile (the MMA K extent of 8 K-steps)
constexpr int NY = 64;        // Omega columns (hi 0..31, lo 32..63)
constexpr int NACC = D + NY;  // accumulator columns: [G | Y]
constexpr int NS = 4;         // pipeline stages
constexpr int NTH = 288;

struct GLayout {
  static constexpr uint32_t X_BYTES = TILE * D * 2;   // 32 KB
  static constexpr uint32_t O_BYTES = TILE * NY * 2;  // 16 KB
  static constexpr uint32_t STAGE = X_BYTES + O_BYTES;
  static constexpr uint32_t OFF_BAR = NS * STAGE;
  static constexpr uint32_t OFF_TM = OFF_BAR + (2 * NS + 4) * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

struct GramArgs {
  CellPtrs x;
  const float* omega;  // rows x k, shared by every cell
  int k;
  int64_t rows, tiles_per_cell, total_tiles, tpc;
  int max_slots;
  float* partial;      // [cell][slot][D][NACC]
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// MN-major SWIZZLE_128B descriptor: LBO = stride between 64-element MN
// groups, SBO = stride between 8-row K groups.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__host__ __device__ inline int64_t seg_lo(int64_t cell, int64_t tiles_per_cell, int64_t tpc) {
  return cell * tiles_per_cell / tpc;
}
__host__ __device__ inline int64_t seg_hi(int64_t cell, int64_t tiles_per_cell, int64_t tpc) {
  return ((cell + 1) * tiles_per_cell - 1) / tpc;
}

__global__ void __launch_bounds__(NTH, 1) tc_gram_kernel(GramArgs A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GLayout::OFF_BAR);
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + GLayout::OFF_TM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t_begin = (int64_t)blockIdx.x * A.tpc;
  const int64_t t_end = t_begin + A.tpc < A.total_tiles ? t_begin + A.tpc : A.total_tiles;
  const int n_my = (int)(t_end > t_begin ? t_end - t_begin : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 128);
    }
    mbar_fence_init();
  }
  if (warp == 4) {
    tmem_alloc(tm_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tm_holder;

  if (warp < 4) {
    // ---------------- producers ----------------
    const int ptid = threadIdx.x;        // 0..127: x chunk owner, and Omega row owner
    const int chunk = ptid & 15;         // x: 16 chunks of 8 features per row
    const int rsub = ptid >> 4;          // x: rows rsub, rsub + 8, ...
    bool ok = true;
    auto issue = [&](int j) {
      const int64_t g = t_begin + j;
      const int cell = (int)(g / A.tiles_per_cell);
      const int64_t r0 = (g % A.tiles_per_cell) * TILE;
      const int st = j % NS;
      if (!mbar_wait(&empty[st], (uint32_t)((j / NS) & 1) ^ 1u, 0x401)) return false;
      const uint32_t xs = sbase + st * GLayout::STAGE;
      const uint32_t os = xs + GLayout::X_BYTES;
      const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(A.x.p[cell]);
#pragma unroll
      for (int i = 0; i < TILE / 8; ++i) {
        const int r = rsub + 8 * i;
        const int64_t row = r0 + r;
        if (row < A.rows) cp_async16(xs + sw128_off(r, chunk * 8, TILE), x + row * D + chunk * 8);
      }
      const int64_t orow = r0 + ptid;
      if (orow < A.rows)
        for (int c = 0; c < A.k; ++c)
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(os + ptid * 128 + c * 4),
                       "l"(A.omega + orow * A.k + c)
                       : "memory");
      return true;
    };
    for (int j = 0; j < NS - 1; ++j) {
      if (ok && j < n_my) ok = issue(j);
      cp_async_commit();
    }
    for (int it = 0; it < n_my && ok; ++it) {
      const int jn = it + NS - 1;
      if (jn < n_my) ok = issue(jn);
      cp_async_commit();
      if (!ok) break;
      cp_async_wait<NS - 1>();
      const int st = it % NS;
      uint8_t* xs = smem + st * GLayout::STAGE;
      uint8_t* os = xs + GLayout::X_BYTES;
      const int64_t g = t_begin + it;
      const int64_t r0 = (g % A.tiles_per_cell) * TILE;
      // zero the x rows past the end of the cell
      if (r0 + TILE > A.rows) {
#pragma unroll
        for (int i = 0; i < TILE / 8; ++i) {
          const int r = rsub + 8 * i;
          if (r0 + r >= A.rows)
            *reinterpret_cast<uint4*>(xs + sw128_off(r, chunk * 8, TILE)) = make_uint4(0, 0, 0, 0);
        }
      }
      // Omega row ptid: fp32 (staged linearly in this row's 128 bytes) -> bf16 hi / lo, swizzled in place
      {
        float v[32];
        const bool valid = r0 + ptid < A.rows;
        const float* src = reinterpret_cast<const float*>(os + ptid * 128);
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = (valid && c < A.k) ? src[c] : 0.f;
        uint16_t hi[32], lo[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const __nv_bfloat16 h = __float2bfloat16_rn(v[c]);
          const __nv_bfloat16 l = __float2bfloat16_rn(v[c] - __bfloat162float(h));
          hi[c] = *reinterpret_cast<const uint16_t*>(&h);
          lo[c] = *reinterpret_cast<const uint16_t*>(&l);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint16_t* s16 = q < 4 ? hi + 8 * q : lo + 8 * (q - 4);
          uint4 w;
          w.x = s16[0] | (uint32_t)s16[1] << 16;
          w.y = s16[2] | (uint32_t)s16[3] << 16;
          w.z = s16[4] | (uint32_t)s16[5] << 16;
          w.w = s16[6] | (uint32_t)s16[7] << 16;
          *reinterpret_cast<uint4*>(os + sw128_off(ptid, q * 8, TILE)) = w;
        }
      }
      fence_async_smem();
      mbar_arrive(&full[st]);
    }
    cp_async_wait<0>();
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // A = x^T and B = x, both MN-major; D[feature][feature / omega column]
      const uint32_t id_g = idesc_f16(D, D, true) | (1u << 15) | (1u << 16);
      const uint32_t id_y = idesc_f16(D, NY, true) | (1u << 15) | (1u << 16);
      int cur_cell = -1, seg = -1, it = 0;
      bool first = true;
      for (; it < n_my; ++it) {
        const int64_t g = t_begin + it;
        const int cell = (int)(g / A.tiles_per_cell);
        if (cell != cur_cell) {
          if (cur_cell >= 0) umma_commit(&accf[seg & 1]);  // close the previous segment
          cur_cell = cell;
          ++seg;
          if (!mbar_wait(&acce[seg & 1], (uint32_t)((seg >> 1) & 1) ^ 1u, 0x402)) break;
          tc_fence_after();
          first = true;
        }
        const int st = it % NS;
        if (!mbar_wait(&full[st], (uint32_t)((it / NS) & 1), 0x403)) break;
        tc_fence_after();
        const uint32_t xs = sbase + st * GLayout::STAGE;
        const uint32_t os = xs + GLayout::X_BYTES;
        const uint32_t acc = tmem + (uint32_t)((seg & 1) * 256);
#pragma unroll
        for (int ks = 0; ks < TILE / 16; ++ks) {
          const uint64_t da = desc_mn_sw128(xs + ks * 2048, TILE * 128);
          const uint64_t dy = desc_mn_sw128(os + ks * 2048, TILE * 128);
          const uint32_t accumulate = (first && ks == 0) ? 0u : 1u;
          umma_f16(acc, da, da, id_g, accumulate);
          umma_f16(acc + D, da, dy, id_y, accumulate);
        }
        first = false;
        umma_commit(&empty[st]);
      }
      if (cur_cell >= 0 && it == n_my) umma_commit(&accf[seg & 1]);
      if (seg >= 0) mbar_wait(&accf[seg & 1], (uint32_t)((seg >> 1) & 1), 0x404);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: flush one segment's accumulator ----------------
    const int lg = warp & 3;
    const int feat = lg * 32 + lane;
    int cur_cell = -1, seg = -1;
    for (int it = 0; it <= n_my; ++it) {
      const int cell = it < n_my ? (int)((t_begin + it) / A.tiles_per_cell) : -2;
      if (cell == cur_cell) continue;
      if (cur_cell >= 0) {
        if (!mbar_wait(&accf[seg & 1], (uint32_t)((seg >> 1) & 1), 0x405)) break;
        tc_fence_after();
        const int slot = (int)(blockIdx.x - seg_lo(cur_cell, A.tiles_per_cell, A.tpc));
        float* dst = A.partial + (((int64_t)cur_cell * A.max_slots + slot) * D + feat) * NACC;
#pragma unroll
        for (int c = 0; c < NACC / 32; ++c) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)((seg & 1) * 256 + c * 32), v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(dst + c * 32)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        tc_fence_before();
        mbar_arrive(&acce[seg & 1]);
      }
      if (cell < 0) break;
      cur_cell = cell;
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Sum the segments of each cell in order (fp64) into [G | Y | trace].
__global__ void tc_gram_reduce_kernel(const float* __restrict__ partial, int n_cells, int64_t tiles_per_cell,
                                      int64_t tpc, int max_slots, int k, double* __restrict__ out,
                                      int64_t stride) {
  const int64_t total = (int64_t)n_cells * D * (D + k);
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int cell = (int)(idx / ((int64_t)D * (D + k)));
    const int64_t e = idx % ((int64_t)D * (D + k));
    const int i = (int)(e / (D + k)), j = (int)(e % (D + k));
    const int nseg = (int)(seg_hi(cell, tiles_per_cell, tpc) - seg_lo(cell, tiles_per_cell, tpc) + 1);
    const float* base = partial + ((int64_t)cell * max_slots * D + i) * NACC;
    double s = 0.0;
    if (j < D) {
      for (int sl = 0; sl < nseg; ++sl) s += (double)base[(int64_t)sl * D * NACC + j];
      out[cell * stride + (int64_t)i * D + j] = s;
    } else {
      const int jj = j - D;
      for (int sl = 0; sl < nseg; ++sl)
        s += (double)base[(int64_t)sl * D * NACC + D + jj] + (double)base[(int64_t)sl * D * NACC + D + 32 + jj];
      out[cell * stride + (int64_t)D * D + (int64_t)i * k + jj] = s;
    }
  }
}

struct GPlan {
  int64_t tiles_per_cell, total, tpc;
  int ctas, max_slots;
};

GPlan gplan(int n_cells, int64_t rows) {
  GPlan p;
  p.tiles_per_cell = ceil_div(rows, TILE);
  p.total = p.tiles_per_cell * n_cells;
  p.tpc = std::max<int64_t>(1, ceil_div(p.total, num_sms()));
  p.ctas = (int)ceil_div(p.total, p.tpc);
  int ms = 1;
  for (int c = 0; c < n_cells; ++c)
    ms = std::max<int>(ms, (int)(seg_hi(c, p.tiles_per_cell, p.tpc) - seg_lo(c, p.tiles_per_cell, p.tpc) + 1));
  p.max_slots = ms;
  return p;
}

}  // namespace

bool tc_gram_eligible(int dtype, int p, int k) { return dtype == KVC_BF16 && p == D && k <= 32; }

size_t tc_gram_workspace(int n_cells, int64_t rows) {
  GPlan p = gplan(n_cells, rows);
  return (size_t)n_cells * p.max_slots * D * NACC * sizeof(float);
}

int tc_gram_launch(int n_cells, const void* const* a, int64_t rows, const float* omega, int k, double* out,
                   void* workspace, size_t ws_bytes, cudaStream_t st) {
  GPlan p = gplan(n_cells, rows);
  if (!workspace || ws_bytes < (size_t)n_cells * p.max_slots * D * NACC * sizeof(float))
    return fail(KVC_ERR_WORKSPACE, "tensor-core gram: workspace too small");
  GramArgs g;
  memset(&g, 0, sizeof(g));
  for (int c = 0; c < n_cells; ++c) g.x.p[c] = a[c];
  g.omega = omega;
  g.k = k;
  g.rows = rows;
  g.tiles_per_cell = p.tiles_per_cell;
  g.total_tiles = p.total;
  g.tpc = p.tpc;
  g.max_slots = p.max_slots;
  g.partial = static_cast<float*>(workspace);
  cudaError_t e = cudaFuncSetAttribute(tc_gram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)GLayout::BYTES);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  tc_gram_kernel<<<p.ctas, NTH, GLayout::BYTES, st>>>(g);
  int rc = check_launch("tc_gram_kernel");
  if (rc) return rc;
  const int64_t stride = (int64_t)D * D + (int64_t)D * k + 1;
  const int64_t total = (int64_t)n_cells * D * (D + k);
  const int blocks = (int)std::min<int64_t>(ceil_div(total, 256), 8 * num_sms());
  tc_gram_reduce_kernel<<<blocks, 256, 0, st>>>(g.partial, n_cells, p.tiles_per_cell, p.tpc, p.max_slots, k, out,
                                                stride);
  return check_launch("tc_gram_reduce_kernel");
}

}  // namespace kvc
