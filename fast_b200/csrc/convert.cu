// fp32 -> bf16 block copies for the bf16 precision mode: the per-step bf16
// copies of the projection weights (each column segment placed at an
// 8-element boundary of the copy, matching the bf16 projection rows) and
// the fp32 activations that feed a bf16 GEMM (the attention output, the
// layer-tail gradient, the query gradient).  Round to nearest even.  One
// launch covers a list of jobs: blockIdx.y is the job, blocks stride its
// rows, a thread converts 4 columns.
#include <cuda_bf16.h>
#include <cstring>
#include "runtime.cuh"

namespace {

struct CastArgs {
  fb_cast_job job[FB_CAST_MAX_JOBS];
  int n;
};
static_assert(sizeof(CastArgs) <= 4096, "kernel parameters of k_cast_bf16 exceed 4 KB");

__device__ __forceinline__ uint32_t pack2(float x, float y) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t *>(&v);
}

__global__ void __launch_bounds__(256) k_cast_bf16(const __grid_constant__ CastArgs a) {
  fb::pdl_enter();
  if ((int)blockIdx.y >= a.n) return;
  const fb_cast_job &j = a.job[blockIdx.y];
  const int64_t rows = j.rows_dev ? min((int64_t)(*j.rows_dev), j.rows) : j.rows;
  const int cols = j.cols;
  const int q4 = (cols + 3) >> 2;            // 4-column groups per row
  const bool vec = (cols & 3) == 0 && (j.lds & 3) == 0 && (j.ldd & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(j.src) & 15) == 0 && (reinterpret_cast<uintptr_t>(j.dst) & 7) == 0;
  const int64_t total = rows * q4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / q4;
    const int c = (int)(i - r * q4) * 4;
    const float *s = j.src + r * j.lds + c;
    uint16_t *d = j.dst + r * j.ldd + c;
    if (vec) {
      const float4 v = __ldg(reinterpret_cast<const float4 *>(s));
      *reinterpret_cast<uint2 *>(d) = make_uint2(pack2(v.x, v.y), pack2(v.z, v.w));
    } else {
      for (int e = 0; e < 4 && c + e < cols; ++e) d[e] = (uint16_t)(pack2(__ldg(s + e), 0.f) & 0xFFFFu);
    }
  }
}

// splitmix64's finaliser (Steele, Lea & Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014): a counter-based hash.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// Seeded N(0, 1) values as bf16, two per thread by the Box-Muller transform
// of two 24-bit uniforms hashed from (seed, element index); columns >= cols
// of each ldd-wide row are zeros.
__global__ void __launch_bounds__(256) k_fill_normal_bf16(uint16_t *dst, int64_t rows, int cols, int64_t ldd,
                                                          uint64_t seed) {
  const int64_t half = ldd >> 1;
  const int64_t total = rows * half;
  const uint64_t key = mix64(seed + 0x9e3779b97f4a7c15ull);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / half;
    const int c = (int)(i - r * half) * 2;
    float z0 = 0.f, z1 = 0.f;
    if (c < cols) {
      const uint64_t h = mix64(key ^ (uint64_t)i);
      const float u1 = ((float)(h >> 40) + 1.f) * (1.f / 16777216.f);          // (0, 1]
      const float u2 = (float)((h >> 16) & 0xFFFFFFu) * (1.f / 16777216.f);    // [0, 1)
      const float rad = sqrtf(-2.f * logf(u1));
      float sn, cs;
      sincospif(2.f * u2, &sn, &cs);
      z0 = rad * cs;
      z1 = c + 1 < cols ? rad * sn : 0.f;
    }
    reinterpret_cast<uint32_t *>(dst + r * ldd)[c >> 1] = pack2(z0, z1);
  }
}

}  // namespace

extern "C" int fb_fill_normal_bf16(uint16_t *dst, int64_t rows, int cols, int64_t ldd, uint64_t seed,
                                   cudaStream_t stream) {
  if (!dst || rows < 0 || cols < 0 || ldd < cols || ldd % 2 || (reinterpret_cast<uintptr_t>(dst) & 3))
    return fb::set_error(FB_ERR_ARG, "fill_normal_bf16: bad argument");
  if (rows == 0 || ldd == 0) return FB_OK;
  const int64_t total = rows * (ldd / 2);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 148 * 16));
  FB_TRY_CUDA(fb::launch(k_fill_normal_bf16, grid, 256, 0, stream, dst, rows, cols, ldd, seed));
  FB_LAUNCHED("k_fill_normal_bf16");
  return FB_OK;
}

extern "C" int fb_cast_bf16(const fb_cast_job *jobs, int n, cudaStream_t stream) {
  if (n < 0 || n > FB_CAST_MAX_JOBS || (n > 0 && !jobs))
    return fb::set_error(FB_ERR_ARG, "cast_bf16: between 0 and FB_CAST_MAX_JOBS jobs");
  CastArgs a;
  std::memset(&a, 0, sizeof(a));
  int64_t most = 0;
  for (int i = 0; i < n; ++i) {
    const fb_cast_job &j = jobs[i];
    if (j.rows < 0 || j.cols < 0 || (j.rows > 0 && j.cols > 0 && (!j.src || !j.dst || j.lds < j.cols || j.ldd < j.cols)))
      return fb::set_error(FB_ERR_ARG, "cast_bf16: bad job " + std::to_string(i));
    a.job[a.n++] = j;
    most = std::max<int64_t>(most, j.rows * ((j.cols + 3) / 4));
  }
  if (a.n == 0 || most == 0) return FB_OK;
  const int gx = (int)std::max<int64_t>(1, std::min<int64_t>((most + 255) / 256, 148 * 8));
  FB_TRY_CUDA(fb::launch(k_cast_bf16, dim3(gx, a.n), 256, 0, stream, a));
  FB_LAUNCHED("k_cast_bf16");
  return FB_OK;
}
