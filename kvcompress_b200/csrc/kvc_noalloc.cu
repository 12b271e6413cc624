// kvc_decompress_noalloc: the fused decode of kvc_decompress with its scratch
// in a fixed device array of this library instead of a caller workspace.
//
// Who needs it: a caller that cannot hand over device memory.  One example is
// a host runtime that binds the C ABI directly (ctypes, cgo, JNI) and owns no
// device allocator.  Another is a serving engine that plans device memory at
// start-up and allows no allocation on its decode path.  For them,
// kvc_decompress's workspace contract means a cudaMalloc of their own.
//
// Scratch: g_noalloc_scratch, KVC_NOALLOC_SCRATCH_BYTES (8 MiB) per device,
// allocated with the module.  Its address is looked up with
// cudaGetSymbolAddress once per device and CUDA context, on the first call
// on that device (again after the device's context was destroyed and made
// anew, e.g. after cudaDeviceReset: the old address would point into a
// context that no longer exists); that lookup may load the module, so make
// the first call on each device before any stream capture.  Only decodes that
// take the tensor-core kernel use scratch: those whose scratch
// (kvc_decompress_workspace_bytes) exceeds the array are rejected with
// KVC_ERR_WORKSPACE; layouts that kvc_decompress decodes with its SIMT kernel
// use none and have no size limit.  Nothing is allocated: no cudaMalloc /
// cudaFree and no allocating library call.
//
// Nothing in the scratch has to start at zero: every byte the decode reads is
// written earlier in the same call, on the same stream (operand tiles,
// u_feature as float, the per-row Tucker term).  There is one array per
// device, so two calls whose work overlaps in time on the device (different
// streams, or different host threads) race on it; calls on one stream are
// ordered and safe.
#include <cuda.h>

#include <mutex>

#include "kvc_common.cuh"

extern "C" size_t kvc_decompress_workspace_bytes(int n_cells, int64_t rows, int d, int rd);
extern "C" int kvc_decompress(int n_cells, const uint8_t* const* codes, const float* const* scale,
                              const int32_t* const* zp, int bits, int symmetric, int scale_mode,
                              int group_size, const void* const* core, const void* const* u_token,
                              const void* const* u_feature, int factor_dtype, int64_t m, int64_t t,
                              int d, int rt, int rd, const float* proj, int64_t t0, int64_t t1,
                              int out_dtype, void* const* out, void* workspace, size_t ws_bytes,
                              void* stream);

namespace kvc {
int kernel_policy();
bool tc_decompress_eligible(int out_dtype, int d, int rd, int bits, int symmetric, int scale_mode,
                            const float* proj);
namespace {

constexpr size_t kScratchBytes = (size_t)KVC_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
// per device: the context the address was looked up in, and the address
CUcontext g_scratch_ctx[kMaxDevices];
void* g_scratch_addr[kMaxDevices];

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link the driver library itself, so it loads on machines without one)
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;

CUcontext current_context() {
  if (!g_ctx_get_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return nullptr;
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of the scratch array on the current device.
int scratch_address(void** addr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(KVC_ERR_ARG, "kvc_decompress_noalloc: device ordinal out of range");
  // the thread's current context; NULL before the runtime made one current
  // (then the lookup below makes the device's primary context current)
  std::lock_guard<std::mutex> lock(g_mu);
  CUcontext ctx = current_context();
  if (!g_scratch_addr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(KVC_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    ctx = current_context();
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *addr = g_scratch_addr[dev];
  return KVC_OK;
}

}  // namespace
}  // namespace kvc

using namespace kvc;

extern "C" int kvc_decompress_noalloc(int n_cells, const uint8_t* const* codes, const float* const* scale,
                                      const int32_t* const* zp, int bits, int symmetric, int scale_mode,
                                      int group_size, const void* const* core, const void* const* u_token,
                                      const void* const* u_feature, int factor_dtype, int64_t m, int64_t t,
                                      int d, int rt, int rd, const float* proj, int64_t t0, int64_t t1,
                                      int out_dtype, void* const* out, void* stream) {
  if (n_cells <= 0 || n_cells > KVC_MAX_CELLS) return fail(KVC_ERR_ARG, "kvc_decompress_noalloc: bad n_cells");
  if (m <= 0 || t <= 0 || d <= 0 || rd < 0) return fail(KVC_ERR_SHAPE, "kvc_decompress_noalloc: bad shape");
  // only the tensor-core decode reads the workspace; the SIMT decode of the
  // other layouts ignores it, so its size is no limit there
  if (kernel_policy() != 1 && tc_decompress_eligible(out_dtype, d, rd, bits, symmetric, scale_mode, proj)) {
    const size_t need = kvc_decompress_workspace_bytes(n_cells, m * t, d, rd);
    if (need > kScratchBytes)
      return fail(KVC_ERR_WORKSPACE, "kvc_decompress_noalloc: needs " + std::to_string(need) +
                                         " bytes of scratch, above the fixed " + std::to_string(kScratchBytes));
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return kvc_decompress(n_cells, codes, scale, zp, bits, symmetric, scale_mode, group_size, core, u_token,
                        u_feature, factor_dtype, m, t, d, rt, rd, proj, t0, t1, out_dtype, out, scratch,
                        kScratchBytes, stream);
}
