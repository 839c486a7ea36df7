// Legacy fastAgg segment operators with the reference's names and argument
// meaning, computing the true results (NoneBone/FAST
// getFastAgg/cuda_operators: edge_softmax.cu K1-K4, aggregate_acc_kernel.cu
// K7/K8, aggregate_shd_kernel.cu K9/K10, utils.cu).  One warp per segment,
// fixed reduction order; only the scatter of arbitrary (unsorted) edge lists
// uses float atomics, as the reference does.
#include <atomic>
#include <algorithm>
#include <cfloat>
#include "runtime.cuh"

namespace {

__global__ void k_edge_softmax_fwd(const int32_t *__restrict__ indptr, int64_t n_seg, const float *__restrict__ x,
                                   int heads, float *__restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t s = wg; s < n_seg; s += nw) {
    const int beg = indptr[s], end = indptr[s + 1];
    for (int h = 0; h < heads; ++h) {
      float m = -FLT_MAX;
      for (int e = beg + lane; e < end; e += 32) m = fmaxf(m, x[(int64_t)e * heads + h]);
      m = fb::warp_max(m);
      float sum = 0.f;
      for (int e = beg + lane; e < end; e += 32) sum += expf(x[(int64_t)e * heads + h] - m);
      float inv = 1.f / fb::warp_sum(sum);
      for (int e = beg + lane; e < end; e += 32) y[(int64_t)e * heads + h] = expf(x[(int64_t)e * heads + h] - m) * inv;
    }
  }
}

__global__ void k_edge_softmax_bwd(const int32_t *__restrict__ indptr, int64_t n_seg, const float *__restrict__ dy,
                                   const float *__restrict__ y, int heads, float *__restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t s = wg; s < n_seg; s += nw) {
    const int beg = indptr[s], end = indptr[s + 1];
    for (int h = 0; h < heads; ++h) {
      float acc = 0.f;
      for (int e = beg + lane; e < end; e += 32) acc = fmaf(y[(int64_t)e * heads + h], dy[(int64_t)e * heads + h], acc);
      acc = fb::warp_sum(acc);
      for (int e = beg + lane; e < end; e += 32) {
        int64_t o = (int64_t)e * heads + h;
        dx[o] = y[o] * (dy[o] - acc);
      }
    }
  }
}

__global__ void k_scatter_rows(const int64_t *__restrict__ dst_idx, const int64_t *__restrict__ src_idx,
                               int64_t n_edges, const float *__restrict__ v, int64_t n_v, int dim,
                               float *__restrict__ out, int64_t n_out, int32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t e = wg; e < n_edges; e += nw) {
    int64_t d = dst_idx[e], s = src_idx[e];
    if (d < 0 || d >= n_out || s < 0 || s >= n_v) { if (lane == 0) atomicOr(err, 1); continue; }
    for (int c = lane; c < dim; c += 32) atomicAdd(out + d * dim + c, v[s * dim + c]);
  }
}

__global__ void k_segment_rows(const int32_t *__restrict__ indptr, int64_t n_seg, const int64_t *__restrict__ row,
                               const int64_t *__restrict__ col, const float *__restrict__ v, int64_t n_v, int dim,
                               float *__restrict__ out, int64_t n_out, int32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t s = wg; s < n_seg; s += nw) {
    const int beg = indptr[s], end = indptr[s + 1];
    if (end <= beg) continue;
    const int64_t d = row[beg];
    if (d < 0 || d >= n_out) { if (lane == 0) atomicOr(err, 1); continue; }
    for (int c = lane; c < dim; c += 32) {
      float acc = 0.f;
      for (int e = beg; e < end; ++e) {
        int64_t sidx = col[e];
        if (sidx >= 0 && sidx < n_v) acc += v[sidx * dim + c];
      }
      out[d * dim + c] = acc;
    }
  }
}

__global__ void __launch_bounds__(256) k_xsum_part(const int32_t *__restrict__ in, int64_t n, int2 *part) {
  __shared__ int sm[64];
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int v = i < n ? in[i] : 0;
  int ea, eb;
  int2 t = fb::block_excl_scan2(v, 0, ea, eb, sm);
  if (threadIdx.x == 0) part[blockIdx.x] = t;
}

__global__ void __launch_bounds__(1024) k_xsum_scan(int2 *part, int nparts, int32_t *out, int64_t n) {
  __shared__ int sm[64];
  int run = 0;
  for (int base = 0; base < nparts; base += blockDim.x) {
    int i = base + threadIdx.x;
    int v = i < nparts ? part[i].x : 0;
    int ea, eb;
    int2 t = fb::block_excl_scan2(v, 0, ea, eb, sm);
    if (i < nparts) part[i].x = run + ea;
    run += t.x;
  }
  if (threadIdx.x == 0) out[n] = run;
}

__global__ void __launch_bounds__(256) k_xsum_write(const int32_t *__restrict__ in, int64_t n, const int2 *part,
                                                    int32_t *out) {
  __shared__ int sm[64];
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int v = i < n ? in[i] : 0;
  int ea, eb;
  fb::block_excl_scan2(v, 0, ea, eb, sm);
  if (i < n) out[i] = part[blockIdx.x].x + ea;
}

__global__ void k_count_ids(const int32_t *__restrict__ ids, int64_t n, int32_t *deg, int64_t n_ids, int32_t *err) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int32_t v = ids[i];
  if (v < 0 || v >= n_ids) { atomicOr(err, 1); return; }
  atomicAdd(deg + v, 1);
}

__global__ void __launch_bounds__(256) k_balanced_mask(const int32_t *__restrict__ ptr, int64_t n_seg, int threshold,
                                                       int32_t *__restrict__ mask) {
  __shared__ int sm[64];
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int d = i < n_seg ? ptr[i + 1] - ptr[i] : 0;
  int ea, eb;
  fb::block_excl_scan2(d, 0, ea, eb, sm);
  if (i < n_seg) {
    int after = ea + d, before = ea;
    mask[i] = (after / threshold > before / threshold) ? 1 : 0;
  }
}

int seg_grid(int64_t n_seg) {
  int64_t need = (n_seg + 7) / 8;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, 148 * 16));
}

int32_t *err_word() {
  static int32_t *w[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!w[dev]) {
    cudaMalloc(&w[dev], 4);
    cudaMemset(w[dev], 0, 4);
  }
  return w[dev];
}

}  // namespace

extern "C" int fb_edge_softmax_fwd(const int32_t *indptr, int64_t n_seg, const float *x, int heads, float *y,
                                   cudaStream_t stream) {
  if (!indptr || n_seg < 0 || heads < 1 || (!x && n_seg) || (!y && n_seg))
    return fb::set_error(FB_ERR_ARG, "edge_softmax_fwd: bad argument");
  if (n_seg == 0) return FB_OK;
  k_edge_softmax_fwd<<<seg_grid(n_seg), 256, 0, stream>>>(indptr, n_seg, x, heads, y);
  FB_LAUNCHED("k_edge_softmax_fwd");
  return FB_OK;
}

extern "C" int fb_edge_softmax_bwd(const int32_t *indptr, int64_t n_seg, const float *dy, const float *y, int heads,
                                   float *dx, cudaStream_t stream) {
  if (!indptr || n_seg < 0 || heads < 1 || (n_seg && (!dy || !y || !dx)))
    return fb::set_error(FB_ERR_ARG, "edge_softmax_bwd: bad argument");
  if (n_seg == 0) return FB_OK;
  k_edge_softmax_bwd<<<seg_grid(n_seg), 256, 0, stream>>>(indptr, n_seg, dy, y, heads, dx);
  FB_LAUNCHED("k_edge_softmax_bwd");
  return FB_OK;
}

extern "C" int fb_scatter_rows(const int64_t *dst_idx, const int64_t *src_idx, int64_t n_edges, const float *v,
                               int64_t n_v, int dim, float *out, int64_t n_out, cudaStream_t stream) {
  if (n_edges < 0 || dim < 1 || (n_edges && (!dst_idx || !src_idx || !v || !out)))
    return fb::set_error(FB_ERR_ARG, "scatter_rows: bad argument");
  if (n_edges == 0) return FB_OK;
  k_scatter_rows<<<seg_grid(n_edges), 256, 0, stream>>>(dst_idx, src_idx, n_edges, v, n_v, dim, out, n_out,
                                                       err_word());
  FB_LAUNCHED("k_scatter_rows");
  return FB_OK;
}

extern "C" int fb_segment_rows(const int32_t *indptr, int64_t n_seg, const int64_t *row, const int64_t *col,
                               const float *v, int64_t n_v, int dim, float *out, int64_t n_out,
                               cudaStream_t stream) {
  if (n_seg < 0 || dim < 1 || (n_seg && (!indptr || !row || !col || !v || !out)))
    return fb::set_error(FB_ERR_ARG, "segment_rows: bad argument");
  if (n_seg == 0) return FB_OK;
  k_segment_rows<<<seg_grid(n_seg), 256, 0, stream>>>(indptr, n_seg, row, col, v, n_v, dim, out, n_out,
                                                     err_word());
  FB_LAUNCHED("k_segment_rows");
  return FB_OK;
}

extern "C" size_t fb_exclusive_sum_ws_bytes(int64_t n) {
  return sizeof(int2) * (size_t)std::max<int64_t>(1, (n + 255) / 256);
}

extern "C" int fb_exclusive_sum(const int32_t *in, int64_t n, int32_t *out, void *ws, cudaStream_t stream) {
  if (n < 0 || !out || !ws || (n && !in)) return fb::set_error(FB_ERR_ARG, "exclusive_sum: bad argument");
  const int nb = (int)std::max<int64_t>(1, (n + 255) / 256);
  int2 *part = static_cast<int2 *>(ws);
  k_xsum_part<<<nb, 256, 0, stream>>>(in, n, part);
  FB_LAUNCHED("k_xsum_part");
  k_xsum_scan<<<1, 1024, 0, stream>>>(part, nb, out, n);
  FB_LAUNCHED("k_xsum_scan");
  k_xsum_write<<<nb, 256, 0, stream>>>(in, n, part, out);
  FB_LAUNCHED("k_xsum_write");
  return FB_OK;
}

extern "C" int fb_count_ids(const int32_t *ids, int64_t n, int32_t *deg, int64_t n_ids, cudaStream_t stream) {
  if (n < 0 || n_ids < 0 || (n && (!ids || !deg))) return fb::set_error(FB_ERR_ARG, "count_ids: bad argument");
  if (n == 0) return FB_OK;
  k_count_ids<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(ids, n, deg, n_ids, err_word());
  FB_LAUNCHED("k_count_ids");
  return FB_OK;
}

extern "C" int fb_balanced_mask(const int32_t *ptr, int64_t n_ptr, int threshold, int32_t *mask, cudaStream_t stream) {
  if (n_ptr < 1 || threshold < 1 || !ptr || (n_ptr > 1 && !mask))
    return fb::set_error(FB_ERR_ARG, "balanced_mask: bad argument");
  const int64_t n_seg = n_ptr - 1;
  if (n_seg == 0) return FB_OK;
  k_balanced_mask<<<(unsigned)((n_seg + 255) / 256), 256, 0, stream>>>(ptr, n_seg, threshold, mask);
  FB_LAUNCHED("k_balanced_mask");
  return FB_OK;
}

// ---- exclusive sum without any allocation ------------------------------------
// Some callers cannot allocate device memory: a host that hands the library a
// fixed memory budget and owns every allocation itself (an embedding runtime
// with its own pool), or a latency-critical loop where a cudaMalloc would
// synchronise the device.  They still need the scan's per-chunk partial sums
// somewhere.  They live in this file-scope array: one int2 per 256-element
// chunk, 4096 chunks (32 KiB), so at most 4096 * 256 = 1,048,576 elements per
// call.  Every GPU that loads the library holds the array until the process
// exits.  All calls share it and it keeps the last call's contents: the first
// kernel overwrites every chunk entry a call uses before anything reads it, so
// nothing needs clearing, but two calls whose kernels overlap on the GPU
// (different streams, no ordering) corrupt each other's results.
namespace {
constexpr int64_t kStaticScanChunks = 4096;
constexpr int kMaxDevices = 64;
// The array's device address per device, from cudaGetSymbolAddress on the
// first call there.  Atomic, so that host threads making their first calls at
// the same time do not race on the cache (both store the same address).  The
// address belongs to the device's primary context: after a cudaDeviceReset the
// process must not call this entry point on that device again.
std::atomic<int2 *> g_static_scan_scratch[kMaxDevices];
}  // namespace

static __device__ __align__(256) int2 g_scan_scratch[kStaticScanChunks];

extern "C" int fb_exclusive_sum_noalloc(const int32_t *in, int64_t n, int32_t *out, cudaStream_t stream) {
  if (n < 0 || !out || (n && !in)) return fb::set_error(FB_ERR_ARG, "exclusive_sum_noalloc: bad argument");
  if (n > kStaticScanChunks * 256)
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "exclusive_sum_noalloc: at most 1048576 elements (4096 chunks of 256) per call");
  int dev = 0;
  FB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fb::set_error(FB_ERR_UNSUPPORTED, "exclusive_sum_noalloc: device index >= 64");
  int2 *part = g_static_scan_scratch[dev].load(std::memory_order_acquire);
  if (!part) {
    // one-time set-up on this device: the host-side symbol is not a device
    // address, so ask the runtime for the array's address on the current device
    void *p = nullptr;
    FB_TRY_CUDA(cudaGetSymbolAddress(&p, g_scan_scratch));
    part = static_cast<int2 *>(p);
    g_static_scan_scratch[dev].store(part, std::memory_order_release);
  }
  const int nb = (int)std::max<int64_t>(1, (n + 255) / 256);
  k_xsum_part<<<nb, 256, 0, stream>>>(in, n, part);
  FB_LAUNCHED("k_xsum_part");
  k_xsum_scan<<<1, 1024, 0, stream>>>(part, nb, out, n);
  FB_LAUNCHED("k_xsum_scan");
  k_xsum_write<<<nb, 256, 0, stream>>>(in, n, part, out);
  FB_LAUNCHED("k_xsum_write");
  return FB_OK;
}
