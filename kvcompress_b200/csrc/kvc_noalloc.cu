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
// cudaGetSymbolAddress once per device, on the first call on that device;
// that lookup may load the module, so make the first call on each device
// before any stream capture.  Sizes whose decode scratch
// (kvc_decompress_workspace_bytes) exceeds the array are rejected with
// KVC_ERR_WORKSPACE.  Nothing is allocated: no cudaMalloc / cudaFree and no
// allocating library call.
//
// Nothing in the scratch has to start at zero: every byte the decode reads is
// written earlier in the same call, on the same stream (operand tiles,
// u_feature as float, the per-row Tucker term).  There is one array per
// device, so two calls whose work overlaps in time on the device (different
// streams, or different host threads) race on it; calls on one stream are
// ordered and safe.
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
namespace {

constexpr size_t kScratchBytes = (size_t)KVC_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices];  // per device, looked up once

// Device address of the scratch array on the current device.
int scratch_address(void** addr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(KVC_ERR_ARG, "kvc_decompress_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(KVC_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
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
  const size_t need = kvc_decompress_workspace_bytes(n_cells, m * t, d, rd);
  if (need > kScratchBytes)
    return fail(KVC_ERR_WORKSPACE, "kvc_decompress_noalloc: needs " + std::to_string(need) +
                                       " bytes of scratch, above the fixed " + std::to_string(kScratchBytes));
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return kvc_decompress(n_cells, codes, scale, zp, bits, symmetric, scale_mode, group_size, core, u_token,
                        u_feature, factor_dtype, m, t, d, rt, rd, proj, t0, t1, out_dtype, out, scratch,
                        kScratchBytes, stream);
}
