// Feature gather fused with the cos time encoding, and its backward.
//
// Reference: prepare_input gathers node_feats[ID] / edge_feats[eID] on the
// host and copies them over PCIe (utils.py:126-196); TimeEncode computes
// cos(Linear(1, d)(dt)) (layers.py:8-29); the attention layer concatenates
// [h_src | f | time] as the K/V projection input (layers.py:157-164).
// Here one kernel reads the device-resident tables and writes the
// concatenated projection rows directly.
//
// Rounding: torch's CPU Linear(1, d) produces w*dt + b with one rounding
// (a fused multiply-add); with dt up to ~1e8 the argument of cos is large and
// a second rounding changes the feature by O(1), so the kernel uses fmaf.
// The backward needs sin of fp32 arguments up to 1e8 radians and beyond (real
// timestamps).  The library's double sin handles them exactly but is bound by
// the fp64 rate (~100 operations per call).  sin_big() reduces the argument
// by pi/2 itself (Cody & Waite: a three-float split of pi/2 in fp32 below
// 2^22, a two-double split up to 2^28) and evaluates the Taylor series of sin
// and cos on |r| <= 0.96 in fp32 (degrees 11 and 10: truncation below
// 1.3e-9).  The forward keeps cosf, which measured faster in its wide gather.
#include <cuda_bf16.h>
#include "runtime.cuh"

namespace {

constexpr int kRowsPerCta = 8;

template <bool VEC>
__device__ __forceinline__ void copy_seg(const float *__restrict__ src, float *__restrict__ dst, int n, int lane) {
  if (VEC) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int c = lane; c < (n >> 2); c += 32) d4[c] = __ldg(s4 + c);
  } else {
    for (int c = lane; c < n; c += 32) dst[c] = __ldg(src + c);
  }
}

struct GatherArgs {
  const float *h; int64_t ldh; const int32_t *h_idx; int64_t h_off; const int32_t *h_off_dev; int dn;
  const float *f; int64_t ldf; const int32_t *f_idx; int de;
  const float *dt, *w, *b; int dtime;
  float *A; int64_t lda; int64_t n_rows; const int32_t *n_rows_dev;
};

// Batched form for 16-byte rows: a warp takes NB rows at a time, loads
// their ids (one lane each), then issues every 16-byte load of the batch's
// source rows before any store, so NB rows are in flight per warp instead
// of one.  NCH 16-byte chunks per lane cover a source row of up to
// 128 NCH floats.  (Eight rows in flight measured slower than four.)
constexpr int kBatch = 4;                     // rows per batch of the bf16 gather
constexpr int kMaxChunks = 4;                 // 16-byte chunks per lane per source row

template <int NB, int NCH>
__device__ __forceinline__ void gather_rows(const float *__restrict__ src, int64_t ld, const int64_t (&row)[NB],
                                            int nb, int nq, float *__restrict__ out0, int64_t lda, int lane) {
  float4 v[NB][NCH];
#pragma unroll
  for (int i = 0; i < NB; ++i)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int q = lane + 32 * c;
      v[i][c] = (i < nb && q < nq) ? __ldg(reinterpret_cast<const float4 *>(src + row[i] * ld) + q)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
  for (int i = 0; i < NB; ++i)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int q = lane + 32 * c;
      if (i < nb && q < nq) reinterpret_cast<float4 *>(out0 + i * lda)[q] = v[i][c];
    }
}

template <int NB, int NCH>
__global__ void __launch_bounds__(32 * kRowsPerCta) k_gather_time_encode_batched(GatherArgs a) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t n = a.n_rows_dev ? min((int64_t)(*a.n_rows_dev), a.n_rows) : a.n_rows;
  const int64_t h_off = a.h_off + (a.h_off_dev ? (int64_t)(*a.h_off_dev) : 0);
  const int64_t step = (int64_t)gridDim.x * kRowsPerCta * NB;
  for (int64_t r0 = ((int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5)) * NB; r0 < n; r0 += step) {
    const int nb = (int)min((int64_t)NB, n - r0);
    // ids and times of the batch: lane i loads row r0 + i's, then broadcast
    int64_t hid = 0, fid = 0;
    float tt = 0.f;
    if (lane < nb) {
      const int64_t r = r0 + lane;
      hid = a.h_idx ? (int64_t)a.h_idx[r] : r + h_off;
      fid = a.f_idx ? (int64_t)a.f_idx[r] : r;
      tt = a.dt ? a.dt[r] : 0.f;
    }
    int64_t hr[NB], fr[NB];
    float t[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      hr[i] = __shfl_sync(0xffffffffu, hid, i);
      fr[i] = __shfl_sync(0xffffffffu, fid, i);
      t[i] = __shfl_sync(0xffffffffu, tt, i);
    }
    float *out0 = a.A + r0 * a.lda;
    if (a.dn > 0) gather_rows<NB, NCH>(a.h, a.ldh, hr, nb, a.dn / 4, out0, a.lda, lane);
    if (a.de > 0) gather_rows<NB, NCH>(a.f, a.ldf, fr, nb, a.de / 4, out0 + a.dn, a.lda, lane);
    if (a.dtime > 0) {
      // the time-encoding block in 16-byte stores when dtime % 4 == 0 and w, b
      // are 16-byte aligned (the row offset dn + de is a multiple of 4 here)
      if ((a.dtime & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.w) | reinterpret_cast<uintptr_t>(a.b)) & 15) == 0) {
        for (int c4 = lane; c4 < (a.dtime >> 2); c4 += 32) {
          const float4 wc = __ldg(reinterpret_cast<const float4 *>(a.w) + c4);
          const float4 bc = __ldg(reinterpret_cast<const float4 *>(a.b) + c4);
#pragma unroll
          for (int i = 0; i < NB; ++i)
            if (i < nb)
              reinterpret_cast<float4 *>(out0 + i * a.lda + a.dn + a.de)[c4] =
                  make_float4(cosf(fmaf(t[i], wc.x, bc.x)), cosf(fmaf(t[i], wc.y, bc.y)),
                              cosf(fmaf(t[i], wc.z, bc.z)), cosf(fmaf(t[i], wc.w, bc.w)));
        }
      } else {
        for (int c = lane; c < a.dtime; c += 32) {
          const float wc = __ldg(a.w + c), bc = __ldg(a.b + c);
#pragma unroll
          for (int i = 0; i < NB; ++i)
            if (i < nb) out0[i * a.lda + a.dn + a.de + c] = cosf(fmaf(t[i], wc, bc));
        }
      }
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(32 * kRowsPerCta) k_gather_time_encode(GatherArgs a) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t n = a.n_rows_dev ? min((int64_t)(*a.n_rows_dev), a.n_rows) : a.n_rows;
  const int64_t h_off = a.h_off + (a.h_off_dev ? (int64_t)(*a.h_off_dev) : 0);
  for (int64_t r = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5); r < n;
       r += (int64_t)gridDim.x * kRowsPerCta) {
    float *out = a.A + r * a.lda;
    if (a.dn > 0) {
      const int64_t hr = a.h_idx ? (int64_t)a.h_idx[r] : r + h_off;
      copy_seg<VEC>(a.h + hr * a.ldh, out, a.dn, lane);
    }
    if (a.de > 0) {
      const int64_t fr = a.f_idx ? (int64_t)a.f_idx[r] : r;
      copy_seg<VEC>(a.f + fr * a.ldf, out + a.dn, a.de, lane);
    }
    if (a.dtime > 0) {
      const float t = a.dt ? a.dt[r] : 0.f;
      float *o = out + a.dn + a.de;
      for (int c = lane; c < a.dtime; c += 32) o[c] = cosf(fmaf(t, __ldg(a.w + c), __ldg(a.b + c)));
    }
  }
}

// bf16 projection rows for the bf16 precision mode: [h | f | cos(w dt + b)]
// with each segment starting at a multiple of 8 columns (16 bytes), so that
// every segment of the row -- and the matching column block of the bf16
// weight copy -- is a valid TMA box origin.  bf16 sources (feature tables)
// are copied as 16-byte words, rows padded with zeros to a multiple of 8
// columns, so the gap after a segment is copied as zeros; fp32 sources (a
// layer's output) are rounded to nearest even and the gap is written as
// zeros.  A warp takes kBatch rows and issues all loads of a segment before
// its stores, as k_gather_time_encode_batched does.
struct GatherBfArgs {
  const void *h; int h_bf; int64_t ldh; const int32_t *h_idx; int64_t h_off; const int32_t *h_off_dev; int dn;
  const void *f; int f_bf; int64_t ldf; const int32_t *f_idx; int de;
  const float *dt, *w, *b; int dtime;
  uint16_t *A; int64_t lda; int f_at, t_at; int64_t n_rows; const int32_t *n_rows_dev;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float x, float y) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// One source segment of kBatch rows into the bf16 row block at out0.
__device__ __forceinline__ void gather_seg_bf16(const void *src, int is_bf, int64_t ld, const int64_t (&row)[kBatch],
                                                int nb, int d, uint16_t *__restrict__ out0, int64_t lda, int lane) {
  if (is_bf) {
    const int nq = (d + 7) >> 3;             // 16-byte words of the zero-padded row
    uint4 v[kBatch][kMaxChunks];
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int q = lane + 32 * c;
        v[i][c] = (i < nb && q < nq)
                      ? __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + row[i] * ld) + q)
                      : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int q = lane + 32 * c;
        if (i < nb && q < nq) reinterpret_cast<uint4 *>(out0 + i * lda)[q] = v[i][c];
      }
  } else {
    const int nq = d >> 2;                   // float4 words (d % 4 == 0)
    float4 v[kBatch][kMaxChunks];
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int q = lane + 32 * c;
        v[i][c] = (i < nb && q < nq)
                      ? __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(src) + row[i] * ld) + q)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int q = lane + 32 * c;
        if (i < nb && q < nq)
          reinterpret_cast<uint2 *>(out0 + i * lda)[q] =
              make_uint2(pack_bf16x2(v[i][c].x, v[i][c].y), pack_bf16x2(v[i][c].z, v[i][c].w));
      }
      if (i < nb && lane == 0 && (d & 7)) reinterpret_cast<uint2 *>(out0 + i * lda)[nq] = make_uint2(0u, 0u);
    }
  }
}

__global__ void __launch_bounds__(32 * kRowsPerCta) k_gather_time_encode_bf16(GatherBfArgs a) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t n = a.n_rows_dev ? min((int64_t)(*a.n_rows_dev), a.n_rows) : a.n_rows;
  const int64_t h_off = a.h_off + (a.h_off_dev ? (int64_t)(*a.h_off_dev) : 0);
  const int64_t step = (int64_t)gridDim.x * kRowsPerCta * kBatch;
  for (int64_t r0 = ((int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5)) * kBatch; r0 < n; r0 += step) {
    const int nb = (int)min((int64_t)kBatch, n - r0);
    int64_t hid = 0, fid = 0;
    float tt = 0.f;
    if (lane < nb) {
      const int64_t r = r0 + lane;
      hid = a.h_idx ? (int64_t)a.h_idx[r] : r + h_off;
      fid = a.f_idx ? (int64_t)a.f_idx[r] : r;
      tt = a.dt ? a.dt[r] : 0.f;
    }
    int64_t hr[kBatch], fr[kBatch];
    float t[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      hr[i] = __shfl_sync(0xffffffffu, hid, i);
      fr[i] = __shfl_sync(0xffffffffu, fid, i);
      t[i] = __shfl_sync(0xffffffffu, tt, i);
    }
    uint16_t *out0 = a.A + r0 * a.lda;
    if (a.dn > 0) gather_seg_bf16(a.h, a.h_bf, a.ldh, hr, nb, a.dn, out0, a.lda, lane);
    if (a.de > 0) gather_seg_bf16(a.f, a.f_bf, a.ldf, fr, nb, a.de, out0 + a.f_at, a.lda, lane);
    if (a.dtime > 0) {
      for (int c = 2 * lane; c < a.dtime; c += 64) {
        const bool two = c + 1 < a.dtime;
        const float w0 = __ldg(a.w + c), b0 = __ldg(a.b + c);
        const float w1 = two ? __ldg(a.w + c + 1) : 0.f, b1 = two ? __ldg(a.b + c + 1) : 0.f;
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (i >= nb) continue;
          const float x0 = cosf(fmaf(t[i], w0, b0));
          uint16_t *o = out0 + i * a.lda + a.t_at + c;
          if (two) {
            *reinterpret_cast<uint32_t *>(o) = pack_bf16x2(x0, cosf(fmaf(t[i], w1, b1)));
          } else {
            *o = (uint16_t)(pack_bf16x2(x0, 0.f) & 0xFFFFu);
          }
        }
      }
    }
  }
}

// +-sin(r) or +-cos(r) for the quadrant q (mod 4) of an argument reduced to
// r, |r| <= 0.96: sin(r + q pi/2).  Taylor series of sin and cos (degrees 11
// and 10, coefficients 1/n!; truncation below 1.3e-9 on that interval).
__device__ __forceinline__ float sin_quadrant(float r, int q) {
  const float r2 = r * r;
  const float sr = fmaf(r2 * r, fmaf(r2, fmaf(r2, fmaf(r2, fmaf(r2, -1.f / 39916800.f, 1.f / 362880.f), -1.f / 5040.f),
                                                1.f / 120.f), -1.f / 6.f), r);
  const float cr = fmaf(r2, fmaf(r2, fmaf(r2, fmaf(r2, fmaf(r2, -1.f / 3628800.f, 1.f / 40320.f), -1.f / 720.f),
                                                1.f / 24.f), -0.5f), 1.f);
  const float v = (q & 1) ? cr : sr;
  return (q & 2) ? -v : v;
}

// sin(x) for |x| >= 2^22: below 2^28, Cody & Waite's reduction in double with
// pi/2 split into a 30-bit head and a 53-bit tail (|pi/2 - head - tail| <
// 2e-26): x - k head is exact (a multiple of 2^-29 below 1 in magnitude, for
// k < 2^28), the tail's fma rounds once, so r is off by < 1e-17; from 2^28 on
// the library's double sin.  Kept out of line: arguments this large are rare
// (w dt beyond 4.2e6 rad).
__device__ __noinline__ float sin_far(float x) {
  if (fabsf(x) >= 268435456.f) return (float)sin((double)x);
  const double xd = (double)x;
  const double kd = rint(xd * 0x1.45f306dc9c883p-1);               // nearest multiple of pi/2
  const float r = (float)fma(-kd, -0x1.de973dcb3b39ap-31, fma(-kd, 0x1.921fb548p+0, xd));
  return sin_quadrant(r, (int)((long long)kd & 3));
}

// sin(x) for a float x, to about 2 ulp of the double result.  |x| < 2^22 (every
// argument of a time encoding but the rare far ones): Cody & Waite's reduction
// in fp32 ("Software Manual for the Elementary Functions", 1980), with pi/2
// split into three floats C1 = fl(pi/2), C2 = fl(pi/2 - C1), C3 = fl(pi/2 -
// C1 - C2) (computed from Machin's series; |pi/2 - C1 - C2 - C3| < 1.1e-23).
// k = rint(x fl(2/pi)) comes from adding 1.5 2^23 (the float's last mantissa
// bits are then k, so k mod 4 is read from them); fl(2/pi) is 2.6e-8 below
// 2/pi, so |x 2/pi - k| <= 0.61 and |r| <= 0.96.  The first fma x - k C1 is
// exact (for |x| >= 1, x and k C1 are multiples of 2^-23 and the result is
// below 2 in magnitude; for |x| < 1, k is 0 or +-1 and Sterbenz's lemma
// applies), the next two round once each, so r carries about one ulp of its
// own plus 2^-45.  No double arithmetic, no conversion, and no divergence
// between lanes of a warp whose arguments differ in size.
__device__ __forceinline__ float sin_big(float x) {
  if (!(fabsf(x) < 4194304.f)) return isnan(x) ? x : sin_far(x);
  const float s = fmaf(x, 0x1.45f306p-1f, 12582912.f);   // 1.5 2^23 + k
  const float k = __fsub_rn(s, 12582912.f);
  float r = fmaf(-k, 0x1.921fb6p+0f, x);
  r = fmaf(-k, -0x1.777a5cp-25f, r);
  r = fmaf(-k, -0x1.ee59dap-50f, r);
  return sin_quadrant(r, __float_as_int(s));
}

constexpr int64_t kTeRowsPerCta = 64;
constexpr int64_t kTeMaxParts = 592;   // two waves of two 800-thread CTAs per SM at most

// Time-encoding backward, stage 1: CTA (x = 32-column tile, y = row chunk)
// with 8 warps striding over the chunk's rows, lanes over columns; the warps'
// sums are combined in shared memory in a fixed order.
// g as fp32, or as bf16 bits (the bf16 projection mode's time-encoding input
// gradient); either is summed in fp32
__device__ __forceinline__ float te_g(const float *p) { return __ldg(p); }
__device__ __forceinline__ float te_g(const uint16_t *p) { return __uint_as_float((uint32_t)__ldg(p) << 16); }

template <typename T>
__global__ void __launch_bounds__(256) k_te_bwd_part(const T *__restrict__ g, int64_t ldg,
                                                     const float *__restrict__ dt, const float *__restrict__ w,
                                                     const float *__restrict__ b, int dtime, int64_t n_rows,
                                                     const int32_t *n_rows_dev, float *__restrict__ part) {
  fb::pdl_enter();
  __shared__ float sw_s[8][32], sb_s[8][32];
  const int64_t n = n_rows_dev ? min((int64_t)(*n_rows_dev), n_rows) : n_rows;
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int parts = fb::split_parts(n, kTeRowsPerCta, kTeMaxParts);
  if ((int)blockIdx.y >= parts) return;
  const int64_t per = (n + parts - 1) / parts;
  const int64_t r0 = (int64_t)blockIdx.y * per;
  const int64_t r1 = min(n, r0 + per);
  float sw = 0.f, sb = 0.f;
  if (c < dtime) {
    const float wc = __ldg(w + c), bc = __ldg(b + c);
    int64_t r = r0 + wp;
    // eight rows' loads in flight per iteration; rows still summed in order
    for (; r + 56 < r1; r += 64) {
      float tv[8], gv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        tv[u] = __ldg(dt + r + 8 * u);
        gv[u] = te_g(g + (r + 8 * u) * ldg + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float gs = -sin_big(fmaf(tv[u], wc, bc)) * gv[u];
        sw = fmaf(gs, tv[u], sw);
        sb += gs;
      }
    }
    for (; r < r1; r += 8) {
      const float t = __ldg(dt + r);
      const float gs = -sin_big(fmaf(t, wc, bc)) * te_g(g + r * ldg + c);
      sw = fmaf(gs, t, sw);
      sb += gs;
    }
  }
  sw_s[wp][lane] = sw;
  sb_s[wp][lane] = sb;
  __syncthreads();
  if (wp == 0 && c < dtime) {
    float aw = 0.f, ab = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { aw += sw_s[i][lane]; ab += sb_s[i][lane]; }
    part[((int64_t)blockIdx.y * 2 + 0) * dtime + c] = aw;
    part[((int64_t)blockIdx.y * 2 + 1) * dtime + c] = ab;
  }
}

// Stage 1 for dtime <= 512: one CTA per row chunk covers every column, thread
// t on column t % dtime and row group t / dtime (kTeGroups groups striding
// over the chunk's rows, eight rows' loads in flight), so no lane idles on a
// partial 32-column block; the groups' sums are combined in a fixed order.
constexpr int kTeGroups = 8;
constexpr int kTeColsMax = 512;

template <typename T>
__global__ void __launch_bounds__(1024) k_te_bwd_rows(const T *__restrict__ g, int64_t ldg,
                                                      const float *__restrict__ dt, const float *__restrict__ w,
                                                      const float *__restrict__ b, int dtime, int groups,
                                                      int64_t n_rows, const int32_t *n_rows_dev,
                                                      float *__restrict__ part) {
  fb::pdl_enter();
  __shared__ float sw_s[kTeGroups * kTeColsMax / 2], sb_s[kTeGroups * kTeColsMax / 2];
  const int64_t n = n_rows_dev ? min((int64_t)(*n_rows_dev), n_rows) : n_rows;
  const int parts = fb::split_parts(n, kTeRowsPerCta, kTeMaxParts);
  if ((int)blockIdx.y >= parts) return;
  const int c = threadIdx.x % dtime, grp = threadIdx.x / dtime;
  const bool live = grp < groups;
  const int64_t per = (n + parts - 1) / parts;
  const int64_t r0 = (int64_t)blockIdx.y * per;
  const int64_t r1 = min(n, r0 + per);
  float sw = 0.f, sb = 0.f;
  if (live) {
    const float wc = __ldg(w + c), bc = __ldg(b + c);
    const int G = groups;
    int64_t r = r0 + grp;
    for (; r + 7 * G < r1; r += 8 * G) {
      float tv[8], gv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        tv[u] = __ldg(dt + r + u * G);
        gv[u] = te_g(g + (r + u * G) * ldg + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float gs = -sin_big(fmaf(tv[u], wc, bc)) * gv[u];
        sw = fmaf(gs, tv[u], sw);
        sb += gs;
      }
    }
    for (; r < r1; r += G) {
      const float t = __ldg(dt + r);
      const float gs = -sin_big(fmaf(t, wc, bc)) * te_g(g + r * ldg + c);
      sw = fmaf(gs, t, sw);
      sb += gs;
    }
    sw_s[grp * dtime + c] = sw;
    sb_s[grp * dtime + c] = sb;
  }
  __syncthreads();
  if (grp == 0) {
    float aw = 0.f, ab = 0.f;
    for (int i = 0; i < groups; ++i) { aw += sw_s[i * dtime + c]; ab += sb_s[i * dtime + c]; }
    part[((int64_t)blockIdx.y * 2 + 0) * dtime + c] = aw;
    part[((int64_t)blockIdx.y * 2 + 1) * dtime + c] = ab;
  }
}

// Stage 1 for dtime <= 512 with V-column-aligned rows (V = 2 or 4): as
// k_te_bwd_rows, but thread t owns the V adjacent columns V (t % (dtime/V)) ..
// +V-1 -- one 4- to 16-byte load of g and one load of dt per V elements -- in
// CTAs of at most 512 threads (two per SM), and the row groups' sums are
// combined in a fixed order.
__device__ __forceinline__ void te_gv(const float *p, float (&o)[2]) {
  const float2 v = __ldg(reinterpret_cast<const float2 *>(p));
  o[0] = v.x, o[1] = v.y;
}
__device__ __forceinline__ void te_gv(const float *p, float (&o)[4]) {
  const float4 v = __ldg(reinterpret_cast<const float4 *>(p));
  o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
}
__device__ __forceinline__ void te_gv(const uint16_t *p, float (&o)[2]) {
  const uint32_t u = __ldg(reinterpret_cast<const uint32_t *>(p));
  o[0] = __uint_as_float(u << 16), o[1] = __uint_as_float(u & 0xFFFF0000u);
}
__device__ __forceinline__ void te_gv(const uint16_t *p, float (&o)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
  o[0] = __uint_as_float(u.x << 16), o[1] = __uint_as_float(u.x & 0xFFFF0000u);
  o[2] = __uint_as_float(u.y << 16), o[3] = __uint_as_float(u.y & 0xFFFF0000u);
}

constexpr int kTeVecThreads = 512;

template <typename T, int V>
__global__ void __launch_bounds__(kTeVecThreads, 2) k_te_bwd_vec(const T *__restrict__ g, int64_t ldg,
                                                                 const float *__restrict__ dt,
                                                                 const float *__restrict__ w,
                                                                 const float *__restrict__ b, int dtime, int groups,
                                                                 int64_t n_rows, const int32_t *n_rows_dev,
                                                                 float *__restrict__ part) {
  fb::pdl_enter();
  // groups * dtime / V <= kTeVecThreads
  __shared__ float sw_s[kTeVecThreads * V], sb_s[kTeVecThreads * V];
  const int64_t n = n_rows_dev ? min((int64_t)(*n_rows_dev), n_rows) : n_rows;
  const int parts = fb::split_parts(n, kTeRowsPerCta, kTeMaxParts);
  if ((int)blockIdx.y >= parts) return;
  const int nt = dtime / V;
  const int c = V * (threadIdx.x % nt), grp = threadIdx.x / nt;
  const bool live = grp < groups;
  const int64_t per = (n + parts - 1) / parts;
  const int64_t r0 = (int64_t)blockIdx.y * per;
  const int64_t r1 = min(n, r0 + per);
  float sw[V], sb[V];
#pragma unroll
  for (int v = 0; v < V; ++v) sw[v] = sb[v] = 0.f;
  if (live) {
    float wv[V], bv[V];
#pragma unroll
    for (int v = 0; v < V; ++v) wv[v] = __ldg(w + c + v), bv[v] = __ldg(b + c + v);
    const int G = groups;
    const T *gp = g + (r0 + grp) * ldg + c;
    const int64_t gstep = (int64_t)G * ldg;
    int64_t r = r0 + grp;
    for (; r + 3 * G < r1; r += 4 * G, gp += 4 * gstep) {
      float tv[4], gv[4][V];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        tv[u] = __ldg(dt + r + u * G);
        te_gv(gp + u * gstep, gv[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const float gs = -sin_big(fmaf(tv[u], wv[v], bv[v])) * gv[u][v];
          sw[v] = fmaf(gs, tv[u], sw[v]);
          sb[v] += gs;
        }
      }
    }
    for (; r < r1; r += G, gp += gstep) {
      const float t = __ldg(dt + r);
      float gg[V];
      te_gv(gp, gg);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float gs = -sin_big(fmaf(t, wv[v], bv[v])) * gg[v];
        sw[v] = fmaf(gs, t, sw[v]);
        sb[v] += gs;
      }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      sw_s[grp * dtime + c + v] = sw[v];
      sb_s[grp * dtime + c + v] = sb[v];
    }
  }
  __syncthreads();
  if (grp == 0) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float aw = 0.f, ab = 0.f;
      for (int i = 0; i < groups; ++i) { aw += sw_s[i * dtime + c + v]; ab += sb_s[i * dtime + c + v]; }
      part[((int64_t)blockIdx.y * 2 + 0) * dtime + c + v] = aw;
      part[((int64_t)blockIdx.y * 2 + 1) * dtime + c + v] = ab;
    }
  }
}

// Stage 2: one warp per column sums the partials, lanes striding over them,
// then a fixed shuffle tree (deterministic).
__global__ void k_te_bwd_reduce(const float *__restrict__ part, int64_t n_rows, const int32_t *n_rows_dev, int dtime,
                                float *dw, float *db) {
  fb::pdl_enter();
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (c >= dtime) return;
  const int64_t n = n_rows_dev ? min((int64_t)(*n_rows_dev), n_rows) : n_rows;
  const int nparts = fb::split_parts(n, kTeRowsPerCta, kTeMaxParts);
  float sw = 0.f, sb = 0.f;
  for (int p = lane; p < nparts; p += 32) {
    sw += part[((int64_t)p * 2 + 0) * dtime + c];
    sb += part[((int64_t)p * 2 + 1) * dtime + c];
  }
  sw = fb::warp_sum(sw);
  sb = fb::warp_sum(sb);
  if (lane == 0) {
    dw[c] += sw;
    db[c] += sb;
  }
}

inline int te_parts(int64_t n) { return fb::split_parts(n, kTeRowsPerCta, kTeMaxParts); }

inline bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fb_gather_time_encode(const float *h, int64_t ldh, const int32_t *h_idx, int64_t h_off,
                                     const int32_t *h_off_dev, int dn,
                                     const float *f, int64_t ldf, const int32_t *f_idx, int de, const float *dt,
                                     const float *w, const float *b, int dtime, float *A, int64_t lda,
                                     int64_t n_rows, const int32_t *n_rows_dev, cudaStream_t stream) {
  if (!A || n_rows < 0 || dn < 0 || de < 0 || dtime < 0 || lda < dn + de + dtime || (dn > 0 && !h) ||
      (de > 0 && !f) || (dtime > 0 && (!w || !b)))
    return fb::set_error(FB_ERR_ARG, "gather_time_encode: bad argument");
  if (n_rows == 0) return FB_OK;
  GatherArgs a{h, ldh, h_idx, h_off, h_off_dev, dn, f, ldf, f_idx, de, dt, w, b, dtime, A, lda, n_rows, n_rows_dev};
  const bool vec = (dn % 4 == 0) && (de % 4 == 0) && (lda % 4 == 0) && (ldh % 4 == 0 || dn == 0) &&
                   (ldf % 4 == 0 || de == 0) && a16(A) && (dn == 0 || a16(h)) && (de == 0 || a16(f));
  int64_t need = (n_rows + kRowsPerCta - 1) / kRowsPerCta;
  int grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, 148 * 16));
  if (vec && dn <= 4 * 32 * kMaxChunks && de <= 4 * 32 * kMaxChunks) {
    // four rows in flight per warp; source rows of <= 256 floats take two
    // 16-byte chunks a lane, wider ones (<= 512) four
    const bool narrow = dn <= 4 * 32 * 2 && de <= 4 * 32 * 2;
    const int nb = 4;
    const int64_t need_b = (n_rows + kRowsPerCta * nb - 1) / (kRowsPerCta * nb);
    const int grid_b = (int)std::max<int64_t>(1, std::min<int64_t>(need_b, 148 * 16));
    if (narrow) {
      FB_TRY_CUDA(fb::launch(k_gather_time_encode_batched<4, 2>, grid_b, 32 * kRowsPerCta, 0, stream, a));
    } else {
      FB_TRY_CUDA(fb::launch(k_gather_time_encode_batched<4, 4>, grid_b, 32 * kRowsPerCta, 0, stream, a));
    }
  } else if (vec) {
    FB_TRY_CUDA(fb::launch(k_gather_time_encode<true>, grid, 32 * kRowsPerCta, 0, stream, a));
  } else {
    FB_TRY_CUDA(fb::launch(k_gather_time_encode<false>, grid, 32 * kRowsPerCta, 0, stream, a));
  }
  FB_LAUNCHED("k_gather_time_encode");
  return FB_OK;
}

extern "C" int fb_gather_time_encode_bf16(const void *h, int h_bf16, int64_t ldh, const int32_t *h_idx, int64_t h_off,
                                          const int32_t *h_off_dev, int dn, const void *f, int f_bf16, int64_t ldf,
                                          const int32_t *f_idx, int de, const float *dt, const float *w,
                                          const float *b, int dtime, uint16_t *A, int64_t lda, int64_t n_rows,
                                          const int32_t *n_rows_dev, cudaStream_t stream) {
  const int f_at = (dn + 7) / 8 * 8, t_at = f_at + (de + 7) / 8 * 8;
  const auto src_ok = [](const void *p, int bf, int64_t ld, int d) {
    return bf ? (a16(p) && ld % 8 == 0 && ld >= (d + 7) / 8 * 8) : (a16(p) && ld % 4 == 0 && d % 4 == 0 && ld >= d);
  };
  if (!A || !a16(A) || lda % 8 || n_rows < 0 || dn < 0 || de < 0 || dtime < 0 || lda < t_at + dtime ||
      (dn > 0 && (!h || !src_ok(h, h_bf16, ldh, dn))) || (de > 0 && (!f || !src_ok(f, f_bf16, ldf, de))) ||
      (dtime > 0 && (!w || !b)) || dn > 8 * 32 * kMaxChunks || de > 8 * 32 * kMaxChunks ||
      (!h_bf16 && dn > 4 * 32 * kMaxChunks) || (!f_bf16 && de > 4 * 32 * kMaxChunks))
    return fb::set_error(FB_ERR_ARG, "gather_time_encode_bf16: bad argument (alignment, widths or pitch)");
  if (n_rows == 0) return FB_OK;
  GatherBfArgs a{h, h_bf16, ldh, h_idx, h_off, h_off_dev, dn, f, f_bf16, ldf, f_idx, de, dt, w, b, dtime,
                 A, lda, f_at, t_at, n_rows, n_rows_dev};
  const int64_t need = (n_rows + kRowsPerCta * kBatch - 1) / (kRowsPerCta * kBatch);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, 148 * 16));
  FB_TRY_CUDA(fb::launch(k_gather_time_encode_bf16, grid, 32 * kRowsPerCta, 0, stream, a));
  FB_LAUNCHED("k_gather_time_encode_bf16");
  return FB_OK;
}

extern "C" size_t fb_time_encode_bwd_ws_bytes(int64_t n_rows, int dtime) {
  const int64_t parts = te_parts(n_rows);
  return (size_t)(parts * 2 * std::max(dtime, 1)) * sizeof(float);
}

namespace {

template <typename T>
int te_bwd(const T *g, int64_t ldg, const float *dt, const float *w, const float *b,
           int dtime, int64_t n_rows, const int32_t *n_rows_dev, float *dw, float *db, void *ws,
           cudaStream_t stream) {
  if (!g || !dt || !w || !b || !dw || !db || !ws || dtime < 1 || n_rows < 0)
    return fb::set_error(FB_ERR_ARG, "time_encode_bwd: bad argument");
  // launched for n_rows (a capacity when n_rows_dev is given); the kernels
  // take the partition from the true count
  const int parts = te_parts(n_rows);
  float *part = static_cast<float *>(ws);
  // V adjacent columns per thread, the widest of 4 and 2 that dtime, the
  // pitch and the alignment of g allow (FB_TE_BWD_VEC=1/2/4 forces one
  // column per thread / at most V; FB_TE_BWD_GROUPS caps the row groups)
  static const int vec_env = getenv("FB_TE_BWD_VEC") ? atoi(getenv("FB_TE_BWD_VEC")) : 4;
  static const int gcap = getenv("FB_TE_BWD_GROUPS") ? std::max(1, atoi(getenv("FB_TE_BWD_GROUPS"))) : 1 << 20;
  const auto fits = [&](int V) {
    return vec_env >= V && dtime % V == 0 && dtime <= kTeColsMax && ldg % V == 0 &&
           reinterpret_cast<uintptr_t>(g) % (sizeof(T) * V) == 0;
  };
  const int V = fits(4) ? 4 : fits(2) ? 2 : 1;
  if (V > 1) {
    // groups of dtime / V threads: as many as fit kTeVecThreads threads
    const int nt = dtime / V;
    const int groups = std::max(1, std::min(gcap, kTeVecThreads / nt));
    const int threads = (groups * nt + 31) / 32 * 32;
    if (V == 4) {
      FB_TRY_CUDA(fb::launch(k_te_bwd_vec<T, 4>, dim3(1, parts), threads, 0, stream, g, ldg, dt, w, b, dtime, groups,
                             n_rows, n_rows_dev, part));
    } else {
      FB_TRY_CUDA(fb::launch(k_te_bwd_vec<T, 2>, dim3(1, parts), threads, 0, stream, g, ldg, dt, w, b, dtime, groups,
                             n_rows, n_rows_dev, part));
    }
    FB_LAUNCHED("k_te_bwd_vec");
  } else if (dtime <= kTeColsMax) {
    // groups of dtime threads: as many as fit 1024 threads, at most kTeGroups
    const int groups = std::max(1, std::min(kTeGroups, 1024 / dtime));
    const int threads = (groups * dtime + 31) / 32 * 32;
    FB_TRY_CUDA(fb::launch(k_te_bwd_rows<T>, dim3(1, parts), threads, 0, stream, g, ldg, dt, w, b, dtime, groups,
                           n_rows, n_rows_dev, part));
    FB_LAUNCHED("k_te_bwd_rows");
  } else {
    dim3 grid((dtime + 31) / 32, parts);
    FB_TRY_CUDA(fb::launch(k_te_bwd_part<T>, grid, 256, 0, stream, g, ldg, dt, w, b, dtime, n_rows, n_rows_dev, part));
    FB_LAUNCHED("k_te_bwd_part");
  }
  FB_TRY_CUDA(fb::launch(k_te_bwd_reduce, (dtime * 32 + 255) / 256, 256, 0, stream, part, n_rows, n_rows_dev, dtime, dw, db));
  FB_LAUNCHED("k_te_bwd_reduce");
  return FB_OK;
}

}  // namespace

extern "C" int fb_time_encode_bwd(const float *g, int64_t ldg, const float *dt, const float *w, const float *b,
                                  int dtime, int64_t n_rows, const int32_t *n_rows_dev, float *dw, float *db,
                                  void *ws, cudaStream_t stream) {
  return te_bwd(g, ldg, dt, w, b, dtime, n_rows, n_rows_dev, dw, db, ws, stream);
}

extern "C" int fb_time_encode_bwd_bf16(const uint16_t *g, int64_t ldg, const float *dt, const float *w,
                                       const float *b, int dtime, int64_t n_rows, const int32_t *n_rows_dev,
                                       float *dw, float *db, void *ws, cudaStream_t stream) {
  return te_bwd(g, ldg, dt, w, b, dtime, n_rows, n_rows_dev, dw, db, ws, stream);
}
