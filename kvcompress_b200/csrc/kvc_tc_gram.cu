// Tensor-core feature-mode Gram + sketch: one pass over bf16 cells with
// head_dim 128 computes, per cell,
//   G = x^T x (128 x 128) and Y = x^T Omega (128 x k), k <= 32,
// the quantities the reference's randomised SVD extracts with five passes
// over the unfolding (kvcompress/compressor/svd.py:259-265, 289).
//
// Operands: an x tile of 128 rows loaded by TMA in the SWIZZLE_128B layout
// (two 64-column boxes) is at the same time the MN-major A operand (x^T: M = feature,
// K = row) and the MN-major B operand (x: N = feature); products of bf16
// values are exact and accumulate in fp32 in TMEM.  Omega (fp32) is split
// once by a small kernel into bf16 hi / lo (columns 0..NY/2-1 / NY/2..NY-1 of
// an NY-column MN-major B tile), so Y carries ~16 mantissa bits of Omega.
// NY = 32 (SWIZZLE_64B rows) for k <= 16, which leaves room for five stages;
// NY = 64 (SWIZZLE_128B) with four stages up to k = 32.
//
// Work: every cell is cut into segments of a fixed number of tiles that
// depends on the row count only; CTAs take contiguous runs of segments in an
// order that runs the cells fastest (every cell shares Omega), keep
// one segment's sum in a TMEM accumulator (two buffers, so the flush of one
// overlaps the next), flush it to a per-segment fp32 partial, and a second
// kernel sums the segments of each cell in order in fp64.  The result of a
// cell is therefore bit-identical however many cells share the launch.
//
// Warp 0 loads tiles by TMA (4 or 5 stages, rows past the end of a cell read
// as zeros), warp 1 issues tcgen05.mma, warps 2-5 drain accumulators.  Every
// mbarrier wait is bounded.
#include <algorithm>

#include "kvc_common.cuh"
#include "kvc_sched.cuh"
#include "kvc_tc.cuh"
#include "kvc_tma.cuh"

namespace kvc {
namespace {

using namespace tc;

constexpr int D = 128;        // head_dim handled here
constexpr int TILE = 128;     // rows per tile (the MMA K extent of 8 K-steps)
constexpr int NTH = 192;      // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int TMA_WARP = 0;
constexpr int MMA_WARP = 1;
constexpr int EPI_WARP0 = 2;

// NY Omega columns (hi, then lo), NS pipeline stages
template <int NY, int NS>
struct GLayout {
  static constexpr int NACC = D + NY;                 // accumulator columns: [G | Y]
  static constexpr uint32_t X_BYTES = TILE * D * 2;   // 32 KB
  static constexpr uint32_t O_BYTES = TILE * NY * 2;  // 8 or 16 KB
  static constexpr uint32_t O_ROW = NY * 2;           // bytes per Omega row: the swizzle span
  static constexpr uint32_t STAGE = X_BYTES + O_BYTES;
  static constexpr uint32_t OFF_RING = NS * STAGE;  // segment ids drawn by the producer
  static constexpr uint32_t OFF_BAR = OFF_RING + sched::RING * 4;
  static constexpr uint32_t OFF_TM = OFF_BAR + (2 * NS + 4) * 8;
  static constexpr uint32_t BYTES = OFF_TM + 16 + 1024;
};

struct GramArgs {
  int k;
  int64_t rows, tiles_per_cell;
  int64_t seg_tiles, segs_per_cell, total_segs;
  float* partial;  // [segment][D][NACC]
};

// Tiles in segment s (the last segment of a cell may be short).
__device__ __forceinline__ int seg_len(const GramArgs& A, int64_t s) {
  const int64_t first = (s % A.segs_per_cell) * A.seg_tiles;
  return (int)(A.tiles_per_cell - first < A.seg_tiles ? A.tiles_per_cell - first : A.seg_tiles);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// MN-major swizzled descriptor: rows of SPAN bytes (128: SWIZZLE_128B, 64:
// SWIZZLE_64B), LBO = stride between MN groups of one row's elements, SBO =
// stride between 8-row K groups (8 rows x SPAN bytes).
template <int SPAN>
__device__ __forceinline__ uint64_t desc_mn_sw(uint32_t saddr, uint32_t lbo) {
  static_assert(SPAN == 128 || SPAN == 64, "128- or 64-byte swizzle");
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((8 * SPAN) >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(SPAN == 128 ? 2 : 4) << 61;
  return d;
}

// Work unit: one segment (seg_tiles consecutive tiles of a cell), summed
// into its own fp32 partial, so the sums do not depend on which CTA made
// them; each CTA takes a contiguous range of segments (kvc_sched.cuh).
template <int NY, int NS>
__global__ void __launch_bounds__(NTH, 1)
    tc_gram_kernel(const __grid_constant__ TmaMaps xmaps, const __grid_constant__ CUtensorMap omap,
                   const __grid_constant__ GramArgs A) {
  using GLayout = kvc::GLayout<NY, NS>;
  constexpr int NACC = GLayout::NACC;
  static_assert(GLayout::BYTES <= 227 * 1024, "shared-memory layout above the 227 KB per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GLayout::OFF_BAR);
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  uint64_t* acce = accf + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(smem + GLayout::OFF_TM);
  int32_t* ring = reinterpret_cast<int32_t*>(smem + GLayout::OFF_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);   // TMA issue + transaction bytes
      mbar_init(&empty[i], 1);  // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 128);
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

  if (warp == TMA_WARP) {
    // ---------------- TMA producer: x tile (two 64-column boxes) + Omega tile ----------------
    if (lane == 0) {
      sched::Cursor cur((A.total_segs + gridDim.x - 1) / gridDim.x, A.total_segs);
      int j = 0;  // stage uses so far
      const int64_t n_cells = A.total_segs / A.segs_per_cell;
      for (int si = 0;; ++si) {
        // the schedule runs the cells fastest (g = segment * n_cells + cell),
        // so a CTA takes one row range of every cell in turn and reads that
        // range of Omega from L2 after the first cell; the id published is
        // the segment's own (cell-major: its partial slot and its rows)
        const int64_t g = sched::next_tile(cur);
        const int64_t sg = g < 0 ? -1 : (g % n_cells) * A.segs_per_cell + g / n_cells;
        sched::ring_put(ring, si, (int32_t)sg);
        if (sg < 0) {  // the end, through the next stage with no bytes
          const int st = j % NS;
          if (mbar_wait(&empty[st], (uint32_t)((j / NS) & 1) ^ 1u, 0x401)) mbar_arrive(&full[st]);
          break;
        }
        const int cell = (int)(sg / A.segs_per_cell);
        const int64_t t0 = (sg % A.segs_per_cell) * A.seg_tiles;
        const int n = seg_len(A, sg);
        bool ok = true;
        for (int t = 0; t < n; ++t, ++j) {
          const int st = j % NS;
          if (!mbar_wait(&empty[st], (uint32_t)((j / NS) & 1) ^ 1u, 0x401)) {
            ok = false;
            break;
          }
          const int y = (int)((t0 + t) * TILE);
          mbar_expect_tx(&full[st], GLayout::STAGE);
          const uint32_t xs = sbase + st * GLayout::STAGE;
          tma_load_2d(xs, &xmaps.m[cell], 0, y, &full[st]);
          tma_load_2d(xs + TILE * 128, &xmaps.m[cell], 64, y, &full[st]);
          tma_load_2d(xs + GLayout::X_BYTES, &omap, 0, y, &full[st]);
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // A = x^T and B = x, both MN-major; D[feature][feature / omega column]
      const uint32_t id_g = idesc_f16(D, D, true) | (1u << 15) | (1u << 16);
      const uint32_t id_y = idesc_f16(D, NY, true) | (1u << 15) | (1u << 16);
      int j = 0, si = 0;
      bool ok = true;
      for (;; ++si) {
        // the segment's first stage (or the end marker) orders the ring read
        if (!mbar_wait(&full[j % NS], (uint32_t)((j / NS) & 1), 0x403)) {
          ok = false;
          break;
        }
        const int32_t sg = sched::ring_get(ring, si);
        if (!mbar_wait(&acce[si & 1], (uint32_t)((si >> 1) & 1) ^ 1u, 0x402)) {
          ok = false;
          break;
        }
        if (sg < 0) {  // the end: the epilogue learns it from the same accumulator barrier
          umma_commit(&accf[si & 1]);
          break;
        }
        tc_fence_after();
        const int n = seg_len(A, sg);
        const uint32_t acc = tmem + (uint32_t)((si & 1) * 256);
        for (int t = 0; t < n && ok; ++t, ++j) {
          const int st = j % NS;
          if (t > 0 && !mbar_wait(&full[st], (uint32_t)((j / NS) & 1), 0x403)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xs = sbase + st * GLayout::STAGE;
          const uint32_t os = xs + GLayout::X_BYTES;
#pragma unroll
          for (int ks = 0; ks < TILE / 16; ++ks) {
            const uint64_t da = desc_mn_sw<128>(xs + ks * 2048, TILE * 128);
            const uint64_t dy = desc_mn_sw<GLayout::O_ROW>(os + ks * 16 * GLayout::O_ROW, TILE * GLayout::O_ROW);
            const uint32_t accumulate = (t == 0 && ks == 0) ? 0u : 1u;
            umma_f16(acc, da, da, id_g, accumulate);
            umma_f16(acc + D, da, dy, id_y, accumulate);
          }
          umma_commit(&empty[st]);
        }
        if (!ok) break;
        umma_commit(&accf[si & 1]);
      }
      // do not leave while MMAs that write TMEM are still in flight
      if (ok) mbar_wait(&accf[si & 1], (uint32_t)((si >> 1) & 1), 0x404);
    }
    __syncwarp();
  } else if (warp >= EPI_WARP0) {
    // ---------------- epilogue: flush one segment's accumulator ----------------
    const int lg = warp & 3;
    const int feat = lg * 32 + lane;
    for (int si = 0;; ++si) {
      if (!__all_sync(0xffffffffu, mbar_wait(&accf[si & 1], (uint32_t)((si >> 1) & 1), 0x405))) break;
      const int32_t sg = sched::ring_get(ring, si);
      if (sg < 0) break;
      tc_fence_after();
      float* dst = A.partial + ((int64_t)sg * D + feat) * NACC;
#pragma unroll
      for (int c = 0; c < NACC / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)((si & 1) * 256 + c * 32), v);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          reinterpret_cast<float4*>(dst + c * 32)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
      tc_fence_before();
      mbar_arrive(&acce[si & 1]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Omega (rows x k fp32) -> rows x ny bf16: hi = bf16(w) in columns
// [0, ny/2), lo = bf16(w - hi) in [ny/2, ny).
__global__ void omega_pad_kernel(const float* __restrict__ omega, int64_t rows, int k, int ny, uint8_t* out) {
  const int half = ny / 2;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows * half;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / half;
    const int c = (int)(idx % half);
    const float w = c < k ? omega[r * k + c] : 0.f;
    const __nv_bfloat16 h = __float2bfloat16_rn(w);
    const __nv_bfloat16 l = __float2bfloat16_rn(w - __bfloat162float(h));
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out + r * (ny * 2));
    o[c] = h;
    o[half + c] = l;
  }
}

// Sum the segments of each cell in order (fp64) into [G | Y | trace].
template <int NY>
__global__ void tc_gram_reduce_kernel(const float* __restrict__ partial, int n_cells, int64_t segs_per_cell,
                                      int k, double* __restrict__ out, int64_t stride) {
  constexpr int NACC = D + NY;
  const int64_t total = (int64_t)n_cells * D * (D + k);
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int cell = (int)(idx / ((int64_t)D * (D + k)));
    const int64_t e = idx % ((int64_t)D * (D + k));
    const int i = (int)(e / (D + k)), j = (int)(e % (D + k));
    const int nseg = (int)segs_per_cell;
    const float* base = partial + ((int64_t)cell * segs_per_cell * D + i) * NACC;
    double s = 0.0;
    if (j < D) {
      for (int sl = 0; sl < nseg; ++sl) s += (double)base[(int64_t)sl * D * NACC + j];
      out[cell * stride + (int64_t)i * D + j] = s;
    } else {
      const int jj = j - D;
      for (int sl = 0; sl < nseg; ++sl)
        s += (double)base[(int64_t)sl * D * NACC + D + jj] + (double)base[(int64_t)sl * D * NACC + D + NY / 2 + jj];
      out[cell * stride + (int64_t)D * D + (int64_t)i * k + jj] = s;
    }
  }
}

struct GPlan {
  int64_t tiles_per_cell, seg_tiles, segs_per_cell, total_segs;
  int ctas;
};

// The segment length depends on the row count only (about 16 segments per
// cell, 4..128 tiles each), never on how many cells share the launch.  Each
// segment costs a flush of its 128 x (128 + NY) fp32 sums and their read in
// the reduce: at 128 tiles that is 2.5% of the segment's x bytes (10% at
// 32), while 128 segments a cell still split a launch of many cells evenly
// over the SMs.
GPlan gplan(int n_cells, int64_t rows) {
  GPlan p;
  p.tiles_per_cell = ceil_div(rows, TILE);
  p.seg_tiles = std::min<int64_t>(p.tiles_per_cell, std::min<int64_t>(128, std::max<int64_t>(4, ceil_div(p.tiles_per_cell, 16))));
  p.segs_per_cell = ceil_div(p.tiles_per_cell, p.seg_tiles);
  p.total_segs = p.segs_per_cell * n_cells;
  p.ctas = (int)std::min<int64_t>(std::min<int64_t>(p.total_segs, num_sms()), 1024);
  return p;
}

}  // namespace

bool tc_gram_eligible(int dtype, int p, int k) { return dtype == KVC_BF16 && p == D && k <= 32; }

// workspace sized for the wider Omega tile (NY = 64), whichever the launch uses
constexpr int NY_MAX = 64;

static size_t partial_bytes(int n_cells, const GPlan& p) {
  (void)n_cells;
  return ((size_t)p.total_segs * D * (D + NY_MAX) * sizeof(float) + 255) & ~(size_t)255;
}

static size_t opad_bytes(int64_t rows) { return ((size_t)rows * NY_MAX * 2 + 255) & ~(size_t)255; }

size_t tc_gram_workspace(int n_cells, int64_t rows) {
  GPlan p = gplan(n_cells, rows);
  return partial_bytes(n_cells, p) + opad_bytes(rows);
}

template <int NY, int NS>
static int tc_gram_run(int n_cells, const void* const* a, int64_t rows, const float* omega, int k, double* out,
                       const GPlan& p, void* workspace, cudaStream_t st) {
  using L = GLayout<NY, NS>;
  GramArgs g;
  memset(&g, 0, sizeof(g));
  uint8_t* opad = static_cast<uint8_t*>(workspace) + partial_bytes(n_cells, p);
  g.k = k;
  {
    const int blocks = (int)std::min<int64_t>(ceil_div(rows * (NY / 2), 256), 16LL * num_sms());
    omega_pad_kernel<<<blocks, 256, 0, st>>>(omega, rows, k, NY, opad);
    int rc0 = check_launch("omega_pad_kernel");
    if (rc0) return rc0;
  }
  // the tensor maps are encoded while the padding kernel runs
  TmaMaps xmaps;
  CUtensorMap omap;
  int rc1;
  for (int c = 0; c < n_cells; ++c) {
    const uint64_t dims[2] = {(uint64_t)D, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)D * 2};
    const uint32_t box[2] = {64u, (uint32_t)TILE};
    if ((rc1 = encode_tma(&xmaps.m[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a[c], dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc1;
  }
  {
    const uint64_t dims[2] = {(uint64_t)NY, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)NY * 2};
    const uint32_t box[2] = {(uint32_t)NY, (uint32_t)TILE};
    if ((rc1 = encode_tma(&omap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, opad, dims, strides, box,
                          NY == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc1;
  }
  g.rows = rows;
  g.tiles_per_cell = p.tiles_per_cell;
  g.seg_tiles = p.seg_tiles;
  g.segs_per_cell = p.segs_per_cell;
  g.total_segs = p.total_segs;
  g.partial = static_cast<float*>(workspace);
  cudaError_t e = cudaFuncSetAttribute(tc_gram_kernel<NY, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)L::BYTES);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  tc_gram_kernel<NY, NS><<<p.ctas, NTH, L::BYTES, st>>>(xmaps, omap, g);
  int rc = check_launch("tc_gram_kernel");
  if (rc) return rc;
  const int64_t stride = (int64_t)D * D + (int64_t)D * k + 1;
  const int64_t total = (int64_t)n_cells * D * (D + k);
  const int blocks = (int)std::min<int64_t>(ceil_div(total, 256), 8 * num_sms());
  tc_gram_reduce_kernel<NY><<<blocks, 256, 0, st>>>(g.partial, n_cells, p.segs_per_cell, k, out, stride);
  return check_launch("tc_gram_reduce_kernel");
}

int tc_gram_launch(int n_cells, const void* const* a, int64_t rows, const float* omega, int k, double* out,
                   void* workspace, size_t ws_bytes, cudaStream_t st) {
  GPlan p = gplan(n_cells, rows);
  if (!workspace || ws_bytes < tc_gram_workspace(n_cells, rows))
    return fail(KVC_ERR_WORKSPACE, "tensor-core gram: workspace too small");
  if (rows >= (1LL << 31)) return fail(KVC_ERR_SHAPE, "tensor-core gram: more than 2^31 rows per cell");
  // Omega rows of 32 columns (hi / lo of k <= 16) leave room for a fifth stage
  if (k <= 16) return tc_gram_run<32, 5>(n_cells, a, rows, omega, k, out, p, workspace, st);
  return tc_gram_run<64, 4>(n_cells, a, rows, omega, k, out, p, workspace, st);
}

int tc_gram_read_device_error(int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tc::g_kvc_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("device error read: ") + cudaGetErrorString(e));
  *out = v;
  int zero = 0;
  cudaMemcpyToSymbol(tc::g_kvc_device_error, &zero, sizeof(int));
  return KVC_OK;
}

}  // namespace kvc
