// Error state and device queries shared by every entry point.
#include <cstring>
#include <string>

#include "kvc_common.cuh"

namespace kvc {

static thread_local std::string g_last_error;
// kernels this host thread launched through the library (every launch is
// followed by check_launch)
static thread_local unsigned long long g_launches = 0;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(KVC_ERR_LAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  ++g_launches;
  return KVC_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace kvc

extern "C" const char* kvc_last_error(void) { return kvc::g_last_error.c_str(); }

extern "C" int kvc_abi_version(void) { return 1; }

extern "C" unsigned long long kvc_launch_count(void) { return kvc::g_launches; }
