// C-ABI bookkeeping: version, status strings, last CUDA error.
#include <atomic>

#include "common.cuh"

#include <cstdlib>
#include <cstring>

namespace vq2 {
static std::atomic<int> g_last_cuda_error{0};
void set_last_cuda_error(cudaError_t e) { g_last_cuda_error.store(static_cast<int>(e)); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VQ2_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

bool moe_fused_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VQ2_MOE_FUSED");  // A/B switch for the native paged step
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int v = cache[dev & 63].load();
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (v <= 0) v = 148;
    cache[dev & 63].store(v);
  }
  return v;
}
}  // namespace vq2

extern "C" int vq2_abi_version(void) { return 2; }

extern "C" int vq2_last_cuda_error(void) { return vq2::g_last_cuda_error.load(); }

extern "C" const char* vq2_status_string(int status) {
  switch (status) {
    case VQ2_OK: return "ok";
    case VQ2_ERR_SHAPE: return "unsupported or inconsistent shape";
    case VQ2_ERR_DTYPE: return "unsupported dtype";
    case VQ2_ERR_ALIGN: return "misaligned pointer or stride";
    case VQ2_ERR_LAUNCH: return "CUDA launch/runtime error";
    case VQ2_ERR_TIMEOUT: return "device-side wait timed out";
    case VQ2_ERR_ARG: return "null pointer or bad argument";
    default: return "unknown status";
  }
}
