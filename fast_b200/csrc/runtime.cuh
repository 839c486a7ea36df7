// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <string>
#include "common.cuh"

namespace fb {
// Records a message for fb_last_error() and returns `code`.
int set_error(int code, const std::string &msg);
// Same, for a failed CUDA call.
int cuda_error(cudaError_t e, const char *where);
}  // namespace fb

#define FB_TRY_CUDA(x)                                              \
  do {                                                              \
    cudaError_t _e = (x);                                           \
    if (_e != cudaSuccess) return fb::cuda_error(_e, #x);           \
  } while (0)

#define FB_LAUNCHED(name)                                           \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return fb::cuda_error(_e, name);         \
  } while (0)
