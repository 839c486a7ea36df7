// Error reporting and version entry points of the C ABI.
#include <cstdlib>
#include <string>
#include "runtime.cuh"

namespace fb {
static thread_local std::string g_last_error;

int set_error(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int cuda_error(cudaError_t e, const char *where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return FB_ERR_CUDA;
}
}  // namespace fb

extern "C" const char *fb_last_error(void) { return fb::g_last_error.c_str(); }

extern "C" const char *fb_version(void) { return "fast_b200 0.1 (sm_100a)"; }

namespace fb {
bool pdl_enabled() {
  static const bool on = getenv("FB_NO_PDL") == nullptr;
  return on;
}
}  // namespace fb
