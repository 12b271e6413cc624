// Host side of the TMA helpers: cuTensorMapEncodeTiled, looked up through
// the runtime's driver entry-point query so that the library does not link
// against libcuda (it still loads on machines without a driver).
#include <mutex>

#include <cudaTypedefs.h>

#include "kvc_tma.cuh"

namespace kvc {
namespace {

std::once_flag g_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
cudaError_t g_lookup = cudaSuccess;

void lookup() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  g_lookup = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (g_lookup == cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

int encode_tma(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  std::call_once(g_once, lookup);
  if (!g_encode)
    return fail(KVC_ERR_LAUNCH, std::string("cuTensorMapEncodeTiled unavailable: ") + cudaGetErrorString(g_lookup));
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(KVC_ERR_ALIGN, "TMA base not 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16 != 0) return fail(KVC_ERR_ALIGN, "TMA row stride not a multiple of 16 bytes");
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) gs[i] = strides[i];
  }
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KVC_ERR_LAUNCH, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return KVC_OK;
}

}  // namespace kvc
