// Feature rows split between HBM and page-locked host memory: the B200 form of
// the reference's slim feature cache (fast_util/slimCache.py:184-403).  The
// reference keeps the hot rows of the node / edge feature tables on the GPU
// (init_cache, fresh_cache) and, per batch, copies the rest from the CPU table
// with torch.index_select(...).to(device) (trans2Device, :261-403): a host
// gather, a host-to-device copy and a device scatter, with the host in the
// loop.  Here the gather is one kernel: a row whose slot map entry is >= 0 is
// read from the device table, any other row straight from the host table,
// which sits in page-locked memory that the GPU addresses directly (its device
// address from fb_host_rows_device_pointer), so the step needs no host round
// trip.  Rows are copied as they are (fp32 or
// bf16 bits), one warp per row, 16 bytes per lane where rows allow.
#include "runtime.cuh"

namespace {

constexpr int kRowsPerCtaFc = 8;   // warps per CTA

template <int E, bool VEC>
__global__ void __launch_bounds__(32 * kRowsPerCtaFc) k_gather_tiered(
    const int32_t *__restrict__ ids, int64_t n, const int32_t *n_dev, const int32_t *__restrict__ slot_of,
    int64_t n_rows_total, const uint8_t *__restrict__ dev_rows, int64_t ld_dev, int64_t n_dev_rows,
    const uint8_t *host_rows, int64_t ld_host, int d, uint8_t *__restrict__ out, int64_t ld_out,
    unsigned long long *misses, int32_t *err) {
  fb::pdl_enter();
  const int64_t nn = n_dev ? min((int64_t)(*n_dev), n) : n;
  const int lane = threadIdx.x & 31;
  const int64_t bytes = (int64_t)d * E;
  unsigned long long missed = 0;           // rows this warp read from the host table
  for (int64_t r = (int64_t)blockIdx.x * kRowsPerCtaFc + (threadIdx.x >> 5); r < nn;
       r += (int64_t)gridDim.x * kRowsPerCtaFc) {
    const int id = __ldg(ids + r);
    uint8_t *dst = out + r * ld_out * E;
    const uint8_t *src = nullptr;
    if (id >= 0 && id < n_rows_total) {
      const int slot = __ldg(slot_of + id);
      if (slot >= 0 && slot < n_dev_rows) {
        src = dev_rows + (int64_t)slot * ld_dev * E;
      } else {
        src = host_rows + (int64_t)id * ld_host * E;
        ++missed;
      }
    } else if (lane == 0 && err) {
      atomicOr(err, 1);                    // an id outside the table: its row is written as zeros
    }
    if (VEC) {
      const int64_t nv = bytes >> 4;
      for (int64_t c = lane; c < nv; c += 32) {
        const uint4 v = src ? reinterpret_cast<const uint4 *>(src)[c] : make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4 *>(dst)[c] = v;
      }
    } else {
      for (int64_t c = lane; c < d; c += 32) {
        if (E == 4) {
          reinterpret_cast<uint32_t *>(dst)[c] = src ? reinterpret_cast<const uint32_t *>(src)[c] : 0u;
        } else {
          reinterpret_cast<uint16_t *>(dst)[c] = src ? reinterpret_cast<const uint16_t *>(src)[c] : (uint16_t)0;
        }
      }
    }
  }
  if (lane == 0 && misses && missed) atomicAdd(misses, missed);
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fb_gather_rows_tiered(const int32_t *ids, int64_t n, const int32_t *n_dev, const int32_t *slot_of,
                                     int64_t n_rows_total, const void *dev_rows, int64_t ld_dev, int64_t n_dev_rows,
                                     const void *host_rows, int64_t ld_host, int d, int elem_bytes, void *out,
                                     int64_t ld_out, unsigned long long *misses, int32_t *err, cudaStream_t stream) {
  if (n < 0 || d < 1 || (elem_bytes != 2 && elem_bytes != 4) || !out || ld_out < d || n_rows_total < 0 ||
      n_dev_rows < 0 || (n > 0 && (!ids || !slot_of)) || (n_dev_rows > 0 && (!dev_rows || ld_dev < d)) ||
      (n_rows_total > 0 && (!host_rows || ld_host < d)))
    return fb::set_error(FB_ERR_ARG, "gather_rows_tiered: bad argument");
  if (n == 0) return FB_OK;
  const auto row_ok = [&](const void *p, int64_t ld) { return !p || (al16(p) && (ld * elem_bytes) % 16 == 0); };
  const bool vec = ((int64_t)d * elem_bytes) % 16 == 0 && row_ok(dev_rows, ld_dev) && row_ok(host_rows, ld_host) &&
                   row_ok(out, ld_out);
  const int64_t need = (n + kRowsPerCtaFc - 1) / kRowsPerCtaFc;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, 148 * 16));
  const auto *dr = static_cast<const uint8_t *>(dev_rows);
  const auto *hr = static_cast<const uint8_t *>(host_rows);
  auto *o = static_cast<uint8_t *>(out);
  if (elem_bytes == 4) {
    if (vec) {
      FB_TRY_CUDA(fb::launch(k_gather_tiered<4, true>, grid, 32 * kRowsPerCtaFc, 0, stream, ids, n, n_dev, slot_of,
                             n_rows_total, dr, ld_dev, n_dev_rows, hr, ld_host, d, o, ld_out, misses, err));
    } else {
      FB_TRY_CUDA(fb::launch(k_gather_tiered<4, false>, grid, 32 * kRowsPerCtaFc, 0, stream, ids, n, n_dev, slot_of,
                             n_rows_total, dr, ld_dev, n_dev_rows, hr, ld_host, d, o, ld_out, misses, err));
    }
  } else {
    if (vec) {
      FB_TRY_CUDA(fb::launch(k_gather_tiered<2, true>, grid, 32 * kRowsPerCtaFc, 0, stream, ids, n, n_dev, slot_of,
                             n_rows_total, dr, ld_dev, n_dev_rows, hr, ld_host, d, o, ld_out, misses, err));
    } else {
      FB_TRY_CUDA(fb::launch(k_gather_tiered<2, false>, grid, 32 * kRowsPerCtaFc, 0, stream, ids, n, n_dev, slot_of,
                             n_rows_total, dr, ld_dev, n_dev_rows, hr, ld_host, d, o, ld_out, misses, err));
    }
  }
  FB_LAUNCHED("k_gather_tiered");
  return FB_OK;
}

extern "C" int fb_host_rows_device_pointer(const void *host, void **dev) {
  if (!host || !dev) return fb::set_error(FB_ERR_ARG, "host_rows_device_pointer: bad argument");
  // fails (instead of letting a kernel fault later) when the memory is not page-locked and mapped
  void *p = nullptr;
  FB_TRY_CUDA(cudaHostGetDevicePointer(&p, const_cast<void *>(host), 0));
  *dev = p;
  return FB_OK;
}
