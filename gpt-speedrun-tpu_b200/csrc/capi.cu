// Library-level entry points: version, status strings, device error flags.
#include "common.cuh"
#include "gemm.cuh"

#include <atomic>

namespace gptb200 {
int attention_read_error(int clear);
int embed_read_error(int clear);
int optim_read_error(int clear);
static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace gptb200

extern "C" uint64_t gptb200_launch_count(void) {
  return gptb200::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* gptb200_version(void) { return "gptb200 0.1.0 (sm_100a)"; }

extern "C" const char* gptb200_status_string(int status) {
  switch (status) {
    case GPTB200_OK: return "ok";
    case GPTB200_EINVAL: return "invalid argument";
    case GPTB200_ESHAPE: return "unsupported shape or alignment";
    case GPTB200_EUNSUPPORTED: return "unsupported option combination";
    case GPTB200_EDEVICE: return "a kernel reported a device-side error";
    case GPTB200_ERANGE: return "token id outside the vocabulary";
    case GPTB200_ETOOLARGE: return "size exceeds the fixed scratch of this allocation-free entry point";
    default:
      if (status < 0) return cudaGetErrorString(static_cast<cudaError_t>(-status));
      return "unknown status";
  }
}

extern "C" int gptb200_device_error_flags(int clear) {
  cudaDeviceSynchronize();
  int f = 0;
  if (gptb200::gemm_read_error(clear)) f |= GPTB200_DEVERR_GEMM;
  if (gptb200::attention_read_error(clear)) f |= GPTB200_DEVERR_ATTENTION;
  if (gptb200::embed_read_error(clear)) f |= GPTB200_DEVERR_TOKEN_RANGE;
  if (gptb200::optim_read_error(clear)) f |= GPTB200_DEVERR_NONFINITE;
  return f;
}

extern "C" int gptb200_device_error(int clear) {
  return gptb200_device_error_flags(clear) ? GPTB200_EDEVICE : GPTB200_OK;
}
