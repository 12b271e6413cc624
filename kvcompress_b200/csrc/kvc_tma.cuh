// Tensor Memory Accelerator (TMA) helpers: tiled tensor maps built on the
// host, bulk tensor loads into shared memory that complete on an mbarrier.
//
// Rules the callers keep: the innermost box coordinate x times the element
// size is a multiple of 16 bytes (x is 0 or a multiple of 64 bf16 elements
// here); global bases are 16-byte aligned and row strides multiples of 16
// bytes (checked when the map is encoded); every load fills the issuing
// CTA's own shared memory only.  Rows outside the tensor read as zeros.
#pragma once

#include <cuda.h>

#include "kvc_common.cuh"
#include "kvc_tc.cuh"

namespace kvc {

// Maps for every cell of a launch, passed as one __grid_constant__ kernel
// parameter (KVC_MAX_CELLS x 128 bytes).
struct TmaMaps {
  CUtensorMap m[KVC_MAX_CELLS];
};

// Encode a row-major tensor [dims[rank-1]] ... [dims[0]] (dims[0] innermost,
// in elements) with byte strides strides[i] of dimension i+1, box box[i].
// Returns KVC_OK or KVC_ERR_ALIGN / KVC_ERR_LAUNCH with kvc_last_error set.
int encode_tma(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle);

namespace tc {

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// 2-D tile load: box at (x = column, y = row) of map into shared dst.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 3-D tile load: box at (x, y, z).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(m), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Tile stores shared -> global (bulk async group of the issuing thread).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(m), "r"(x),
               "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, int x, int y, int z, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(m), "r"(x),
               "r"(y), "r"(z), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed groups still read their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace tc
}  // namespace kvc
