// Shared device helpers for the fast_b200 kernels (sm_100a only).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "../../include/fast_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "fast_b200 kernels are written for sm_100a only"
#endif

#define FB_CHECK_LAUNCH()                                   \
  do {                                                      \
    cudaError_t _e = cudaGetLastError();                    \
    if (_e != cudaSuccess) return FB_ERR_CUDA;              \
  } while (0)

#define FB_CHECK_CUDA(x)                                    \
  do {                                                      \
    cudaError_t _e = (x);                                   \
    if (_e != cudaSuccess) return FB_ERR_CUDA;              \
  } while (0)

namespace fb {

constexpr int kWarp = 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011).  Constants are
// the ones published with the algorithm.
struct Philox4 {
  uint32_t v[4];
};

__device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                 uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0 = __umulhi(M0, c0), lo0 = M0 * c0;
    uint32_t hi1 = __umulhi(M1, c2), lo1 = M1 * c2;
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n1 = lo1;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    uint32_t n3 = lo0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += W0; k1 += W1;
  }
  Philox4 r;
  r.v[0] = c0; r.v[1] = c1; r.v[2] = c2; r.v[3] = c3;
  return r;
}

// Block-wide exclusive scan of a pair of ints (blockDim.x multiple of 32,
// at most 1024).  `smem` must hold 2*32 ints.  Returns the block totals.
__device__ __forceinline__ int2 block_excl_scan2(int a, int b, int &ea, int &eb, int *smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int ta = __shfl_up_sync(0xffffffffu, ia, o);
    int tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += ta; ib += tb; }
  }
  if (lane == 31) { smem[wid] = ia; smem[32 + wid] = ib; }
  __syncthreads();
  if (wid == 0) {
    int va = lane < nw ? smem[lane] : 0;
    int vb = lane < nw ? smem[32 + lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int ta = __shfl_up_sync(0xffffffffu, va, o);
      int tb = __shfl_up_sync(0xffffffffu, vb, o);
      if (lane >= o) { va += ta; vb += tb; }
    }
    smem[lane] = va;       // inclusive per-warp prefix
    smem[32 + lane] = vb;
  }
  __syncthreads();
  int wa = wid > 0 ? smem[wid - 1] : 0;
  int wb = wid > 0 ? smem[32 + wid - 1] : 0;
  ea = wa + ia - a;
  eb = wb + ib - b;
  int2 tot = make_int2(smem[nw - 1], smem[32 + nw - 1]);
  __syncthreads();
  return tot;
}

// Number of partial sums a split reduction over n rows uses: one per
// rows_min rows, between 1 and max_parts.  Kernels launched for a capacity
// recompute it from the true row count on the device, so the partition and
// the summation order, and with them the rounded result, depend on n only.
__host__ __device__ __forceinline__ int split_parts(int64_t n, int64_t rows_min, int64_t max_parts) {
  int64_t p = (n + rows_min - 1) / rows_min;
  if (p > max_parts) p = max_parts;
  if (p < 1) p = 1;
  return (int)p;
}

// Splits of a weight-gradient reduction over n rows: split_parts, raised to
// at least one split per kTnRowsMax rows so that the running sum of a split
// stays short (its rounding error grows with its length).  A function of n
// alone, like split_parts.
constexpr int64_t kTnRowsMax = 8192;
__host__ __device__ __forceinline__ int tn_parts(int64_t n, int64_t rows_min, int64_t max_parts) {
  const int p = split_parts(n, rows_min, max_parts);
  const int64_t q = (n + kTnRowsMax - 1) / kTnRowsMax;
  return q > p ? (int)q : p;
}

// First statement of every kernel launched with fb::launch(): wait for the
// previous grid in the stream (its writes visible), then allow the next one
// to be scheduled.  Both are no-ops for a kernel launched without the
// programmatic-dependency attribute.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace fb
