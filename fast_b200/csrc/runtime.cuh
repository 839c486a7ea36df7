// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <string>
#include <utility>
#include "common.cuh"

namespace fb {
// Records a message for fb_last_error() and returns `code`.
int set_error(int code, const std::string &msg);
// Same, for a failed CUDA call.
int cuda_error(cudaError_t e, const char *where);

// Programmatic dependent launch.  The kernels of a training step are launched
// with it: a kernel may be scheduled while its predecessor in the stream is
// still finishing, which hides the launch gap between the ~50 short kernels of
// a step.  Every kernel launched this way starts with pdl_enter(), which waits
// until the predecessor grid has completed and its writes are visible, then
// lets the next kernel be scheduled.  FB_NO_PDL in the environment turns the
// attribute off (plain stream order).
bool pdl_enabled();

// Projection GEMMs on the tensor cores (gemm_tc.cu).  fb_gemm_group sends every
// problem tc_problem_ok accepts there unless FB_GEMM=ffma is set in the
// environment (then the CUDA-core kernels of gemm_pipe.cu run everything).
bool tc_enabled();
bool tc_problem_ok(const fb_gemm_problem &p);
int64_t tc_ws_floats(const fb_gemm_problem &p);   // TN partial sums, floats
int tc_group(const fb_gemm_problem *const *probs, float *const *ws, int n, cudaStream_t stream);

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
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
