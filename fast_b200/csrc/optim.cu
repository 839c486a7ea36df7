// Adam over one flat parameter buffer (torch.optim.Adam, weight_decay 0,
// amsgrad off; the reference trains with it, train.py:128):
//   m = b1 m + (1 - b1) g,  v = b2 v + (1 - b2) g^2,  t = t + 1,
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// One launch.  The step count t lives on the device (CUDA-graph replays
// advance it): every CTA reads the old value, and the last CTA to finish
// stores t + 1, so no CTA can see a half-advanced count.
#include <algorithm>
#include "runtime.cuh"

namespace {

__global__ void k_adam(float *__restrict__ p, const float *__restrict__ g, float *__restrict__ m, float *__restrict__ v,
                       int64_t n, float lr, float b1, float b2, float eps, int64_t *step, uint32_t *done) {
  fb::pdl_enter();
  const int64_t t = *step + 1;
  const float bc1 = 1.f - powf(b1, (float)t), bc2 = 1.f - powf(b2, (float)t);
  const float step_size = lr / bc1, inv_sqrt_bc2 = 1.f / sqrtf(bc2);
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 gg = reinterpret_cast<const float4 *>(g)[i];
    float4 mm = reinterpret_cast<float4 *>(m)[i];
    float4 vv = reinterpret_cast<float4 *>(v)[i];
    float4 pp = reinterpret_cast<float4 *>(p)[i];
    float *gf = &gg.x, *mf = &mm.x, *vf = &vv.x, *pf = &pp.x;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      mf[c] = b1 * mf[c] + (1.f - b1) * gf[c];
      vf[c] = b2 * vf[c] + (1.f - b2) * gf[c] * gf[c];
      pf[c] -= step_size * mf[c] / (sqrtf(vf[c]) * inv_sqrt_bc2 + eps);
    }
    reinterpret_cast<float4 *>(m)[i] = mm;
    reinterpret_cast<float4 *>(v)[i] = vv;
    reinterpret_cast<float4 *>(p)[i] = pp;
  }
  for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    m[i] = b1 * m[i] + (1.f - b1) * g[i];
    v[i] = b2 * v[i] + (1.f - b2) * g[i] * g[i];
    p[i] -= step_size * m[i] / (sqrtf(v[i]) * inv_sqrt_bc2 + eps);
  }
  // the last CTA out publishes the new step count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *step = t;
      *done = 0;
    }
  }
}

}  // namespace

extern "C" int fb_adam_step(float *p, const float *g, float *m, float *v, int64_t n, float lr, float beta1,
                            float beta2, float eps, int64_t *step, uint32_t *done, cudaStream_t stream) {
  if (!p || !g || !m || !v || !step || !done || n < 0)
    return fb::set_error(FB_ERR_ARG, "adam_step: bad argument");
  if (((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
        reinterpret_cast<uintptr_t>(v)) & 15u) != 0)
    return fb::set_error(FB_ERR_ARG, "adam_step: buffers must be 16-byte aligned");
  const int64_t need = (n / 4 + 255) / 256;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, 148 * 4));
  FB_TRY_CUDA(fb::launch(k_adam, grid, 256, 0, stream, p, g, m, v, n, lr, beta1, beta2, eps, step, done));
  FB_LAUNCHED("k_adam");
  return FB_OK;
}
