// Fused temporal attention over destination segments, one warp per
// destination row, plus the legacy fastAgg segment operators.
//
// Reference semantics (NoneBone/FAST):
//   logits  LeakyReLU_0.2(sum_d Q.K)           layers.py:165-173
//   softmax per destination (dgl edge_softmax) layers.py:188-192, edge_softmax.cu:255-293
//   dropout on att, V*att, scatter-sum          layers.py:198-222
//   backward                                    efficientGOP.py:80-131 (true gradient)
//
// Memory plan per destination row j with edges [rptr[j], rptr[j+1]):
//   forward reads q_j once, each K row once (pass 1) and each V row once
//   (pass 3), writes att[e, :] and agg_j.  Backward reads q_j, dagg_j, each
//   V row (pass 1) and K row (pass 2) once, writes dV, dK rows and dq_j.
// Rows are 16-byte vectors spread over the lanes, so every K/V row is one
// fully coalesced warp load.  Reductions stay inside the warp: no atomics,
// results are bit-identical run to run.
#include <cfloat>
#include <cstdlib>
#include <cuda_bf16.h>
#include "runtime.cuh"

namespace {

constexpr int kWarpsPerCta = 8;
// Segments are short (fan-out ~10), so a warp's work is a chain of a few
// dependent loads; resident warps hide that latency.  Rows of <= 128 floats
// fit 3 CTAs (24 warps) per SM; wider rows need the registers of 2.
template <int NV>
struct MinCtas {
  static constexpr int value = NV <= 1 ? 3 : 2;
};
constexpr int kMaxHeads = 4;
constexpr int kStash = 64;  // edges whose per-head values a warp keeps in shared memory

struct RowGeom {
  int nv4;   // float4 vectors per row
  int dh;    // features per head
  int heads;
};

// Head index of each of the 4 components of the lane's t-th vector.
template <int NV>
__device__ __forceinline__ void lane_heads(const RowGeom &g, int lane, int hsel[NV][4]) {
#pragma unroll
  for (int t = 0; t < NV; ++t)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int idx = 4 * (lane + 32 * t) + c;
      hsel[t][c] = (lane + 32 * t < g.nv4) ? idx / g.dh : kMaxHeads;
    }
}

template <int NV>
__device__ __forceinline__ void load_row(const float *__restrict__ p, const RowGeom &g, int lane, float4 r[NV]) {
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    int v = lane + 32 * t;
    r[t] = (v < g.nv4) ? __ldg(reinterpret_cast<const float4 *>(p) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int NV>
__device__ __forceinline__ void store_row(float *__restrict__ p, const RowGeom &g, int lane, const float4 r[NV]) {
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    int v = lane + 32 * t;
    if (v < g.nv4) reinterpret_cast<float4 *>(p)[v] = r[t];
  }
}

// Four consecutive gradient values at element offset off of p: fp32, or
// bf16 when bf (p then holds bf16 bit patterns).
__device__ __forceinline__ void put4(float *p, int64_t off, float4 v, int bf) {
  if (bf) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    *reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(p) + off) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
  } else {
    *reinterpret_cast<float4 *>(p + off) = v;
  }
}

template <int NV>
__device__ __forceinline__ void store_grad_row(float *__restrict__ p, int64_t row_off, const RowGeom &g, int lane,
                                               const float4 r[NV], int bf) {
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    int v = lane + 32 * t;
    if (v < g.nv4) put4(p, row_off + 4 * v, r[t], bf);
  }
}

__device__ __forceinline__ float comp(const float4 &v, int c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

__device__ __forceinline__ float pick(const float (&a)[kMaxHeads], int h) {
  return h == 0 ? a[0] : (h == 1 ? a[1] : (h == 2 ? a[2] : (h == 3 ? a[3] : 0.f)));
}

// Per-head dot products of two rows, reduced over the warp (all lanes get them).
template <int NV>
__device__ __forceinline__ void head_dots(const float4 a[NV], const float4 b[NV], const int hsel[NV][4], int heads,
                                          float (&out)[kMaxHeads]) {
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h) out[h] = 0.f;
#pragma unroll
  for (int t = 0; t < NV; ++t)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float p = comp(a[t], c) * comp(b[t], c);
      int h = hsel[t][c];
#pragma unroll
      for (int hh = 0; hh < kMaxHeads; ++hh)
        if (h == hh) out[hh] += p;
    }
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h)
    if (h < heads) out[h] = fb::warp_sum(out[h]);
}

__device__ __forceinline__ float leaky(float z, float slope) { return z > 0.f ? z : z * slope; }

// Dropout keep-scale of (edge, head): 0 or 1/(1-p).  The keep decision comes
// from explicit uniforms when given (kept when u > p, as the reference mask
// test does), else from Philox(seed, offset; edge) so the backward pass can
// regenerate it without storing a mask.
__device__ __forceinline__ void drop_scale(int64_t e, int heads, float p, uint64_t seed, uint64_t offset,
                                           const float *mask_u, float (&s)[kMaxHeads]) {
  if (p <= 0.f) {
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) s[h] = 1.f;
    return;
  }
  const float inv = 1.f / (1.f - p);
  if (mask_u) {
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) s[h] = (h < heads && mask_u[e * heads + h] > p) ? inv : 0.f;
    return;
  }
  fb::Philox4 r = fb::philox4x32_10((uint32_t)e, (uint32_t)(e >> 32), (uint32_t)offset, (uint32_t)(offset >> 32),
                                    (uint32_t)seed, (uint32_t)(seed >> 32));
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h) {
    float u = (float)(r.v[h] >> 8) * (1.0f / 16777216.0f);
    s[h] = (h < heads && u >= p) ? inv : 0.f;
  }
}

struct AttnArgs {
  const float *q; int64_t ldq;
  const float *k, *v; int64_t ldkv;
  const int32_t *rptr; int64_t n_dst; const int32_t *n_dst_dev;
  int heads, dim;
  float slope, drop_p; uint64_t seed, offset;
  const uint64_t *offset_dev;  // optional: dropout stream offset read on the device (graph replays)
  const float *att; float *att_out;
  float *agg; int64_t ldagg;
  const float *x;          // optional pre-activation logits [E, heads] replacing q.k
  const float *mask_u;     // optional dropout uniforms [E, heads]
  const int64_t *seg_row;  // optional: segment s owns output row seg_row[rptr[s]]
  int64_t n_out;           // rows of agg / dagg when seg_row is given (others are skipped)
  float *dx;               // optional gradient of the pre-activation logits
  const float *dagg; int64_t lddagg;
  float *dq, *dk, *dv; int64_t lddkv;
  int kv_bf16;             // dk / dv are bf16 (bit patterns, round to nearest even)
  int kv_in_bf16;          // k / v are bf16 rows (bulk-copy kernels only)
  int agg_bf16;            // agg is bf16 (bulk-copy kernels only): the next product's bf16 operand
  int dq_bf16; int64_t lddq;  // dq is bf16 at lddq elements per row (bulk-copy kernels only)
};

// Output (or incoming gradient) row of segment j: j itself, or the row named
// by seg_row at the segment's first edge (legacy cntE segments).
__device__ __forceinline__ int64_t seg_out_row(const AttnArgs &a, int64_t j, int beg, int end) {
  if (!a.seg_row) return j;
  if (end <= beg) return -1;
  const int64_t r = a.seg_row[beg];
  return (r >= 0 && r < a.n_out) ? r : -1;
}

// Edges handled per chunk: all of a chunk's K (or V) rows are loaded before
// any of them is reduced, so the row loads overlap instead of serialising.
template <int NV>
struct Chunk {
  static constexpr int value = NV <= 1 ? 4 : (NV == 2 ? 2 : 1);
};

template <int NV>
__global__ void __launch_bounds__(32 * kWarpsPerCta, MinCtas<NV>::value) k_attn_fwd(AttnArgs a) {
  __shared__ float stash[kWarpsPerCta][kStash][kMaxHeads];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  RowGeom g{a.dim / 4, a.dim / a.heads, a.heads};
  int hsel[NV][4];
  lane_heads<NV>(g, lane, hsel);
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  if (a.n_dst_dev && !a.seg_row) {
    // rows past the device-side count: zeros, so fixed-size consumers stay finite
    const float4 z[NV] = {};
    for (int64_t j = n_dst + (int64_t)blockIdx.x * kWarpsPerCta + w; j < a.n_dst;
         j += (int64_t)gridDim.x * kWarpsPerCta)
      store_row<NV>(a.agg + j * a.ldagg, g, lane, z);
  }
  for (int64_t j = (int64_t)blockIdx.x * kWarpsPerCta + w; j < n_dst; j += (int64_t)gridDim.x * kWarpsPerCta) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    const int64_t orow = seg_out_row(a, j, beg, end);
    float4 acc[NV];
#pragma unroll
    for (int t = 0; t < NV; ++t) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (end > beg) {
      float4 q[NV];
      if (!a.x) load_row<NV>(a.q + j * a.ldq, g, lane, q);
      float m[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) m[h] = -FLT_MAX;
      // pass 1: activated logits (stashed), running max
      constexpr int CH = Chunk<NV>::value;
      for (int e0 = beg; e0 < end; e0 += CH) {
        float4 kr[CH][NV];
        if (!a.x) {
#pragma unroll
          for (int c = 0; c < CH; ++c)
            if (e0 + c < end) load_row<NV>(a.k + (int64_t)(e0 + c) * a.ldkv, g, lane, kr[c]);
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int e = e0 + c;
          if (e >= end) break;
          float z[kMaxHeads];
          if (a.x) {
#pragma unroll
            for (int h = 0; h < kMaxHeads; ++h) z[h] = (h < a.heads) ? __ldg(a.x + (int64_t)e * a.heads + h) : 0.f;
          } else {
            head_dots<NV>(q, kr[c], hsel, a.heads, z);
          }
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h) {
            z[h] = leaky(z[h], a.slope);
            m[h] = fmaxf(m[h], z[h]);
          }
          const int i = e - beg;
          if (lane < a.heads) {
            if (i < kStash) stash[w][i][lane] = pick(z, lane);
            else a.att_out[(int64_t)e * a.heads + lane] = pick(z, lane);
          }
        }
      }
      __syncwarp();
      // pass 2: softmax denominators
      float ssum[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) ssum[h] = 0.f;
      for (int e = beg + lane; e < end; e += 32) {
        const int i = e - beg;
#pragma unroll
        for (int h = 0; h < kMaxHeads; ++h)
          if (h < a.heads) {
            float l = (i < kStash) ? stash[w][i][h] : a.att_out[(int64_t)e * a.heads + h];
            ssum[h] += expf(l - m[h]);
          }
      }
      float inv[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) inv[h] = (h < a.heads) ? 1.f / fb::warp_sum(ssum[h]) : 0.f;
      __syncwarp();
      // pass 3: probabilities, dropout, weighted sum of V
      for (int e0 = beg; e0 < end; e0 += CH) {
        float4 vr[CH][NV];
#pragma unroll
        for (int c = 0; c < CH; ++c)
          if (e0 + c < end) load_row<NV>(a.v + (int64_t)(e0 + c) * a.ldkv, g, lane, vr[c]);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int e = e0 + c;
          if (e >= end) break;
          const int i = e - beg;
          float y[kMaxHeads], ds[kMaxHeads];
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h) {
            float l = (h < a.heads) ? ((i < kStash) ? stash[w][i][h] : a.att_out[(int64_t)e * a.heads + h]) : 0.f;
            y[h] = (h < a.heads) ? expf(l - m[h]) * inv[h] : 0.f;
          }
          __syncwarp();
          if (lane < a.heads) a.att_out[(int64_t)e * a.heads + lane] = pick(y, lane);
          drop_scale(e, a.heads, a.drop_p, a.seed, doff, a.mask_u, ds);
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h) y[h] *= ds[h];
#pragma unroll
          for (int t = 0; t < NV; ++t) {
            acc[t].x = fmaf(pick(y, hsel[t][0]), vr[c][t].x, acc[t].x);
            acc[t].y = fmaf(pick(y, hsel[t][1]), vr[c][t].y, acc[t].y);
            acc[t].z = fmaf(pick(y, hsel[t][2]), vr[c][t].z, acc[t].z);
            acc[t].w = fmaf(pick(y, hsel[t][3]), vr[c][t].w, acc[t].w);
          }
        }
      }
    }
    if (orow >= 0) store_row<NV>(a.agg + orow * a.ldagg, g, lane, acc);
    __syncwarp();
  }
}

template <int NV>
__global__ void __launch_bounds__(32 * kWarpsPerCta, MinCtas<NV>::value) k_attn_bwd(AttnArgs a) {
  __shared__ float stash[kWarpsPerCta][kStash][kMaxHeads];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  RowGeom g{a.dim / 4, a.dim / a.heads, a.heads};
  int hsel[NV][4];
  lane_heads<NV>(g, lane, hsel);
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const bool need_dl = (a.dq != nullptr) || (a.dk != nullptr) || (a.dx != nullptr);
  for (int64_t j = (int64_t)blockIdx.x * kWarpsPerCta + w; j < n_dst; j += (int64_t)gridDim.x * kWarpsPerCta) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    const int64_t irow = seg_out_row(a, j, beg, end);
    float4 dqa[NV];
#pragma unroll
    for (int t = 0; t < NV; ++t) dqa[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (end > beg && irow >= 0) {
      float4 da[NV], q[NV];
      load_row<NV>(a.dagg + irow * a.lddagg, g, lane, da);
      if (!a.x) load_row<NV>(a.q + j * a.ldq, g, lane, q);
      float sdot[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) sdot[h] = 0.f;
      // pass 1: dL/d(att) through dropout, dV, and sum_e y * dL/dy per head
      constexpr int CH = Chunk<NV>::value;
      for (int e0 = beg; e0 < end; e0 += CH) {
        float4 vr[CH][NV];
#pragma unroll
        for (int c = 0; c < CH; ++c)
          if (e0 + c < end) load_row<NV>(a.v + (int64_t)(e0 + c) * a.ldkv, g, lane, vr[c]);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int e = e0 + c;
          if (e >= end) break;
          float datt[kMaxHeads], ds[kMaxHeads], y[kMaxHeads];
          head_dots<NV>(da, vr[c], hsel, a.heads, datt);
          drop_scale(e, a.heads, a.drop_p, a.seed, doff, a.mask_u, ds);
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h) {
            y[h] = (h < a.heads) ? __ldg(a.att + (int64_t)e * a.heads + h) : 0.f;
            datt[h] *= ds[h];
            sdot[h] = fmaf(y[h], datt[h], sdot[h]);
          }
          const int i = e - beg;
          if (i < kStash && lane < a.heads) stash[w][i][lane] = pick(datt, lane);
          if (a.dv) {
            float4 o[NV];
#pragma unroll
            for (int t = 0; t < NV; ++t) {
              o[t].x = pick(y, hsel[t][0]) * pick(ds, hsel[t][0]) * da[t].x;
              o[t].y = pick(y, hsel[t][1]) * pick(ds, hsel[t][1]) * da[t].y;
              o[t].z = pick(y, hsel[t][2]) * pick(ds, hsel[t][2]) * da[t].z;
              o[t].w = pick(y, hsel[t][3]) * pick(ds, hsel[t][3]) * da[t].w;
            }
            store_grad_row<NV>(a.dv, (int64_t)e * a.lddkv, g, lane, o, a.kv_bf16);
          }
        }
      }
      __syncwarp();
      if (need_dl) {
        // pass 2: softmax and LeakyReLU backward, dK rows, dq accumulation
        for (int e0 = beg; e0 < end; e0 += CH) {
        float4 krc[CH][NV];
        if (!a.x) {
#pragma unroll
          for (int c = 0; c < CH; ++c)
            if (e0 + c < end) load_row<NV>(a.k + (int64_t)(e0 + c) * a.ldkv, g, lane, krc[c]);
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int e = e0 + c;
          if (e >= end) break;
          const int i = e - beg;
          float dy[kMaxHeads];
          if (i < kStash) {
#pragma unroll
            for (int h = 0; h < kMaxHeads; ++h) dy[h] = (h < a.heads) ? stash[w][i][h] : 0.f;
          } else {
            float4 vr[NV];
            float ds[kMaxHeads];
            load_row<NV>(a.v + (int64_t)e * a.ldkv, g, lane, vr);
            head_dots<NV>(da, vr, hsel, a.heads, dy);
            drop_scale(e, a.heads, a.drop_p, a.seed, doff, a.mask_u, ds);
#pragma unroll
            for (int h = 0; h < kMaxHeads; ++h) dy[h] *= ds[h];
          }
          float z[kMaxHeads], dz[kMaxHeads];
          const float4 *kr = krc[c];
          if (a.x) {
#pragma unroll
            for (int h = 0; h < kMaxHeads; ++h) z[h] = (h < a.heads) ? __ldg(a.x + (int64_t)e * a.heads + h) : 0.f;
          } else {
            head_dots<NV>(q, krc[c], hsel, a.heads, z);
          }
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h) {
            const float y = (h < a.heads) ? __ldg(a.att + (int64_t)e * a.heads + h) : 0.f;
            const float dl = y * (dy[h] - sdot[h]);
            dz[h] = z[h] > 0.f ? dl : dl * a.slope;
          }
          if (a.dx && lane < a.heads) a.dx[(int64_t)e * a.heads + lane] = pick(dz, lane);
          if (!a.x) {
            if (a.dk) {
              float4 o[NV];
#pragma unroll
              for (int t = 0; t < NV; ++t) {
                o[t].x = pick(dz, hsel[t][0]) * q[t].x;
                o[t].y = pick(dz, hsel[t][1]) * q[t].y;
                o[t].z = pick(dz, hsel[t][2]) * q[t].z;
                o[t].w = pick(dz, hsel[t][3]) * q[t].w;
              }
              store_grad_row<NV>(a.dk, (int64_t)e * a.lddkv, g, lane, o, a.kv_bf16);
            }
#pragma unroll
            for (int t = 0; t < NV; ++t) {
              dqa[t].x = fmaf(pick(dz, hsel[t][0]), kr[t].x, dqa[t].x);
              dqa[t].y = fmaf(pick(dz, hsel[t][1]), kr[t].y, dqa[t].y);
              dqa[t].z = fmaf(pick(dz, hsel[t][2]), kr[t].z, dqa[t].z);
              dqa[t].w = fmaf(pick(dz, hsel[t][3]), kr[t].w, dqa[t].w);
            }
          }
        }
        }
      }
    }
    if (a.dq) store_row<NV>(a.dq + j * (int64_t)a.dim, g, lane, dqa);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Edge-parallel kernels (rows of <= 128 floats, logits from q.k, even
// per-head width).  Per destination a warp works in groups of up to 32 edges:
//   * dot products are lane-per-edge: lane c reads edge c's K (or V) row in
//     16-byte chunks and multiplies it with q (or dagg) staged in shared
//     memory once per head, masked to that head's features, so one warp
//     instruction advances up to 32 edges and no shuffle reduction is needed;
//   * softmax statistics are warp reductions over the group's lanes;
//   * row outputs (agg, dK, dV, dq) are lane-per-feature: lane t owns the
//     16-byte chunk t of the row, and each edge's per-head weights are
//     broadcast from the edge's lane.
// With an even per-head width, features 4t, 4t+1 share one head (hA) and
// 4t+2, 4t+3 another (hB).

constexpr int kEdgeGroup = 32;

template <int HP>
__device__ __forceinline__ float hv(const float (&a)[HP], int h) {
  float r = a[0];
#pragma unroll
  for (int i = 1; i < HP; ++i)
    if (h == i) r = a[i];
  return r;
}

// Philox keep scales of edge e for every head (the decisions of drop_scale()).
template <int HP>
__device__ __forceinline__ void keep_heads(const AttnArgs &a, uint64_t doff, int64_t e, bool valid, float inv_keep,
                                           float (&k)[HP]) {
  if (!valid) {
#pragma unroll
    for (int h = 0; h < HP; ++h) k[h] = 0.f;
    return;
  }
  if (a.drop_p <= 0.f) {
#pragma unroll
    for (int h = 0; h < HP; ++h) k[h] = 1.f;
    return;
  }
  if (a.mask_u) {
#pragma unroll
    for (int h = 0; h < HP; ++h) k[h] = (h < a.heads && a.mask_u[e * a.heads + h] > a.drop_p) ? inv_keep : 0.f;
    return;
  }
  fb::Philox4 r = fb::philox4x32_10((uint32_t)e, (uint32_t)(e >> 32), (uint32_t)doff, (uint32_t)(doff >> 32),
                                    (uint32_t)a.seed, (uint32_t)(a.seed >> 32));
#pragma unroll
  for (int h = 0; h < HP; ++h) k[h] = ((float)(r.v[h] >> 8) * (1.0f / 16777216.0f) >= a.drop_p) ? inv_keep : 0.f;
}

// Stages x (one row, nq chunks) into sm[h][t], masked to head h's features.
template <int HP>
__device__ __forceinline__ void stage_masked(float4 (*sm)[32], const float *x, int nq, int dh, int lane) {
  if (lane < nq) {
    const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + lane);
    const int hA = (4 * lane) / dh, hB = (4 * lane + 2) / dh;
#pragma unroll
    for (int h = 0; h < HP; ++h)
      sm[h][lane] = make_float4(hA == h ? v.x : 0.f, hA == h ? v.y : 0.f, hB == h ? v.z : 0.f, hB == h ? v.w : 0.f);
  }
}

// Lane-per-edge: out[h] = sum_t sm[h][t] . row[t] over the row's nq chunks.
template <int HP>
__device__ __forceinline__ void row_dots(const float *row, const float4 (*sm)[32], int nq, float (&out)[HP]) {
#pragma unroll
  for (int h = 0; h < HP; ++h) out[h] = 0.f;
  const float4 *r4 = reinterpret_cast<const float4 *>(row);
#pragma unroll 5
  for (int t = 0; t < nq; ++t) {
    const float4 k = __ldg(r4 + t);
#pragma unroll
    for (int h = 0; h < HP; ++h) {
      const float4 m = sm[h][t];
      out[h] = fmaf(m.x, k.x, fmaf(m.y, k.y, fmaf(m.z, k.z, fmaf(m.w, k.w, out[h]))));
    }
  }
}

template <int HP>
__global__ void __launch_bounds__(32 * kWarpsPerCta, 4) k_attn_fwd_s(AttnArgs a) {
  __shared__ float4 qm[kWarpsPerCta][HP][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.n_dst_dev) {
    for (int64_t j = n_dst + (int64_t)blockIdx.x * kWarpsPerCta + w; j < a.n_dst;
         j += (int64_t)gridDim.x * kWarpsPerCta)
      if (live) reinterpret_cast<float4 *>(a.agg + j * a.ldagg)[lane] = zero4;
  }
  for (int64_t j = (int64_t)blockIdx.x * kWarpsPerCta + w; j < n_dst; j += (int64_t)gridDim.x * kWarpsPerCta) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 acc = zero4;
    if (end > beg) {
      __syncwarp();
      stage_masked<HP>(qm[w], a.q + j * a.ldq, nq, dh, lane);
      __syncwarp();
      const bool one = end - beg <= kEdgeGroup;
      float m[HP], ssum[HP], ex[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) { m[h] = -FLT_MAX; ssum[h] = 0.f; ex[h] = 0.f; }
      for (int g0 = beg; g0 < end; g0 += kEdgeGroup) {
        const int n = min(kEdgeGroup, end - g0);
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float z[HP];
        if (valid) row_dots<HP>(a.k + e * a.ldkv, qm[w], nq, z);
        float kp[HP];
        keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
        float wt[HP], sc[HP];
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool ok = valid && h < a.heads;
          const float zz = ok ? leaky(z[h], a.slope) : -FLT_MAX;
          if (!one && ok) a.att_out[e * a.heads + h] = zz;          // raw; normalised below
          const float mn = fmaxf(m[h], fb::warp_max(zz));
          sc[h] = (m[h] == -FLT_MAX) ? 0.f : expf(m[h] - mn);
          m[h] = mn;
          ex[h] = ok ? expf(zz - mn) : 0.f;
          ssum[h] = ssum[h] * sc[h] + fb::warp_sum(ex[h]);
          wt[h] = ex[h] * kp[h];
        }
        const float sa = hv<HP>(sc, hA), sb = hv<HP>(sc, hB);
        acc.x *= sa; acc.y *= sa; acc.z *= sb; acc.w *= sb;
        // lane-per-feature weighted sum of the group's V rows
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          float wc[HP];
#pragma unroll
          for (int h = 0; h < HP; ++h) wc[h] = __shfl_sync(0xffffffffu, wt[h], c);
          const float wa = hv<HP>(wc, hA), wb = hv<HP>(wc, hB);
          const float4 v = live ? __ldg(reinterpret_cast<const float4 *>(a.v + (int64_t)(g0 + c) * a.ldkv) + lane)
                                : zero4;
          acc.x = fmaf(wa, v.x, acc.x);
          acc.y = fmaf(wa, v.y, acc.y);
          acc.z = fmaf(wb, v.z, acc.z);
          acc.w = fmaf(wb, v.w, acc.w);
        }
      }
      float inv[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) inv[h] = h < a.heads ? 1.f / ssum[h] : 0.f;
      const float ia = hv<HP>(inv, hA), ib = hv<HP>(inv, hB);
      acc.x *= ia; acc.y *= ia; acc.z *= ib; acc.w *= ib;
      if (one) {
        if (lane < end - beg)
#pragma unroll
          for (int h = 0; h < HP; ++h)
            if (h < a.heads) a.att_out[(int64_t)(beg + lane) * a.heads + h] = ex[h] * inv[h];
      } else {
        __syncwarp();
        for (int t = lane; t < (end - beg) * a.heads; t += 32) {
          const int h = t % a.heads;
          float *pz = a.att_out + (int64_t)beg * a.heads + t;
          *pz = expf(*pz - hv<HP>(m, h)) * hv<HP>(inv, h);
        }
      }
    }
    if (live) put4(a.agg, j * a.ldagg + 4 * lane, acc, a.agg_bf16);
  }
}

template <int HP>
__global__ void __launch_bounds__(32 * kWarpsPerCta, 4) k_attn_bwd_s(AttnArgs a) {
  __shared__ float4 qm[kWarpsPerCta][HP][32];
  __shared__ float4 dm[kWarpsPerCta][HP][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t j = (int64_t)blockIdx.x * kWarpsPerCta + w; j < n_dst; j += (int64_t)gridDim.x * kWarpsPerCta) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 dq = zero4;
    if (end > beg) {
      __syncwarp();
      stage_masked<HP>(qm[w], a.q + j * a.ldq, nq, dh, lane);
      stage_masked<HP>(dm[w], a.dagg + j * a.lddagg, nq, dh, lane);
      __syncwarp();
      const float4 q4 = live ? __ldg(reinterpret_cast<const float4 *>(a.q + j * a.ldq) + lane) : zero4;
      const float4 da4 = live ? __ldg(reinterpret_cast<const float4 *>(a.dagg + j * a.lddagg) + lane) : zero4;
      const bool one = end - beg <= kEdgeGroup;
      // pass 1: dL/dy through dropout (lane per edge), sum_e y dL/dy per head, dV rows
      float sd[HP], dl1[HP], y1[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) { sd[h] = 0.f; dl1[h] = 0.f; y1[h] = 0.f; }
      for (int g0 = beg; g0 < end; g0 += kEdgeGroup) {
        const int n = min(kEdgeGroup, end - g0);
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float d[HP], kp[HP], yk[HP];
        if (valid) row_dots<HP>(a.v + e * a.ldkv, dm[w], nq, d);
        keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool ok = valid && h < a.heads;
          const float y = ok ? __ldg(a.att + e * a.heads + h) : 0.f;
          const float dl = ok ? d[h] * kp[h] : 0.f;
          sd[h] += fb::warp_sum(y * dl);
          dl1[h] = dl;
          y1[h] = y;
          yk[h] = y * kp[h];
        }
        if (a.dv) {
#pragma unroll 4
          for (int c = 0; c < n; ++c) {
            float yc[HP];
#pragma unroll
            for (int h = 0; h < HP; ++h) yc[h] = __shfl_sync(0xffffffffu, yk[h], c);
            const float ya = hv<HP>(yc, hA), yb = hv<HP>(yc, hB);
            if (live)
              put4(a.dv, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(ya * da4.x, ya * da4.y, yb * da4.z, yb * da4.w), a.kv_bf16);
          }
        }
      }
      // pass 2: logits again (lane per edge), LeakyReLU and softmax backward,
      // dK rows and dq (lane per feature)
      for (int g0 = beg; g0 < end; g0 += kEdgeGroup) {
        const int n = min(kEdgeGroup, end - g0);
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float z[HP], dl[HP], y[HP], dz[HP];
        if (valid) row_dots<HP>(a.k + e * a.ldkv, qm[w], nq, z);
        if (one) {
#pragma unroll
          for (int h = 0; h < HP; ++h) { dl[h] = dl1[h]; y[h] = y1[h]; }
        } else {
          float d[HP], kp[HP];
          if (valid) row_dots<HP>(a.v + e * a.ldkv, dm[w], nq, d);
          keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
#pragma unroll
          for (int h = 0; h < HP; ++h) {
            const bool ok = valid && h < a.heads;
            y[h] = ok ? __ldg(a.att + e * a.heads + h) : 0.f;
            dl[h] = ok ? d[h] * kp[h] : 0.f;
          }
        }
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool ok = valid && h < a.heads;
          const float g = y[h] * (dl[h] - sd[h]);
          dz[h] = ok ? (z[h] > 0.f ? g : g * a.slope) : 0.f;
        }
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          float zc[HP];
#pragma unroll
          for (int h = 0; h < HP; ++h) zc[h] = __shfl_sync(0xffffffffu, dz[h], c);
          const float za = hv<HP>(zc, hA), zb = hv<HP>(zc, hB);
          if (live) {
            const float4 k = __ldg(reinterpret_cast<const float4 *>(a.k + (int64_t)(g0 + c) * a.ldkv) + lane);
            if (a.dk)
              put4(a.dk, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(za * q4.x, za * q4.y, zb * q4.z, zb * q4.w), a.kv_bf16);
            dq.x = fmaf(za, k.x, dq.x);
            dq.y = fmaf(za, k.y, dq.y);
            dq.z = fmaf(zb, k.z, dq.z);
            dq.w = fmaf(zb, k.w, dq.w);
          }
        }
      }
    }
    if (a.dq && live) reinterpret_cast<float4 *>(a.dq + j * (int64_t)a.dim)[lane] = dq;
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy variants of the edge-parallel kernels, for the interleaved K|V
// layout (V = K + dim, row stride 2 dim): a destination's edges are
// consecutive rows, so a group's K and V rows are one contiguous block that a
// single TMA bulk copy (cp.async.bulk, completion on an mbarrier, no
// multicast) moves into the warp's shared-memory slot.  The whole group's
// bytes are then in flight at once, where the register-fed kernels kept a few
// 16-byte loads per lane in flight; K is read from DRAM once in the backward.
// Every mbarrier wait is bounded: past the bound the warp records bit 2 in
// g_attn_err (fb_attn_error), waits once more (bounded) for its copy, and
// stops.

constexpr int kBulkGroup = 12;                         // edges per copy
constexpr int kBulkWarps = 4;                          // warps (destination slots) per CTA
constexpr long long kBulkWaitCycles = 4000000000LL;    // ~2 s at 1.9 GHz
__device__ int g_attn_err;

__device__ __forceinline__ uint32_t sm_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t *bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_addr(bar)) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(sm_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Lane 0: announce `bytes` and start the copy of [src, src + bytes) into dst.
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_addr(bar)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   sm_addr(dst)),
               "l"(src), "r"(bytes), "r"(sm_addr(bar))
               : "memory");
}
// Whole warp: true once the copy of this phase landed, warp-uniformly; false
// (error recorded, one more bounded wait done) when it did not in time.
__device__ __forceinline__ bool bulk_wait(uint64_t *bar, uint32_t parity) {
  long long t0 = clock64();
  bool ok = true;
  while (!bar_try_wait(bar, parity)) {
    if (clock64() - t0 > kBulkWaitCycles) { ok = false; break; }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) {
    if ((threadIdx.x & 31) == 0) atomicOr(&g_attn_err, 2);
    t0 = clock64();
    while (!bar_try_wait(bar, parity) && clock64() - t0 < kBulkWaitCycles) {
    }
  }
  return ok;
}
// Orders the warp's earlier generic reads of its slot before the next copy.
__device__ __forceinline__ void slot_release() {
  __syncwarp();
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Four consecutive features (float4 index q) of row `row` of a warp's slot:
// fp32 rows, or bf16 rows (BF) widened to fp32.
template <bool BF>
__device__ __forceinline__ float4 slot4(const unsigned char *slot, int row, int rowf, int q) {
  if (BF) {
    const uint2 u = reinterpret_cast<const uint2 *>(slot + (size_t)row * rowf * 2)[q];
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xFFFF0000u));
  }
  return reinterpret_cast<const float4 *>(slot + (size_t)row * rowf * 4)[q];
}

// Lane-per-edge dot products of slot row `row` (features from float4 index
// q0) against the masked rows in shared memory.
template <int HP, bool BF>
__device__ __forceinline__ void row_dots_sm(const unsigned char *slot, int row, int rowf, int q0,
                                            const float4 (*sm)[32], int nq, float (&out)[HP]) {
#pragma unroll
  for (int h = 0; h < HP; ++h) out[h] = 0.f;
#pragma unroll 5
  for (int t = 0; t < nq; ++t) {
    const float4 k = slot4<BF>(slot, row, rowf, q0 + t);
#pragma unroll
    for (int h = 0; h < HP; ++h) {
      const float4 m = sm[h][t];
      out[h] = fmaf(m.x, k.x, fmaf(m.y, k.y, fmaf(m.z, k.z, fmaf(m.w, k.w, out[h]))));
    }
  }
}

template <int HP, bool BF>
__global__ void __launch_bounds__(32 * kBulkWarps) k_attn_fwd_b(AttnArgs a) {
  fb::pdl_enter();
  extern __shared__ __align__(128) unsigned char smraw[];
  __shared__ uint64_t bar[kBulkWarps];
  constexpr int kEsz = BF ? 2 : 4;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rowf = (int)a.ldkv;
  unsigned char *slot = smraw + (size_t)w * kBulkGroup * rowf * kEsz;
  const unsigned char *kbase = reinterpret_cast<const unsigned char *>(a.k);
  float4 (*qm)[32] =
      reinterpret_cast<float4 (*)[32]>(smraw + (size_t)kBulkWarps * kBulkGroup * rowf * kEsz) + (size_t)w * HP;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane == 0) bar_init(&bar[w]);
  __syncwarp();
  uint32_t phase = 0;
  if (a.n_dst_dev) {
    for (int64_t j = n_dst + (int64_t)blockIdx.x * kBulkWarps + w; j < a.n_dst;
         j += (int64_t)gridDim.x * kBulkWarps)
      if (live) put4(a.agg, j * a.ldagg + 4 * lane, zero4, a.agg_bf16);
  }
  for (int64_t j = (int64_t)blockIdx.x * kBulkWarps + w; j < n_dst; j += (int64_t)gridDim.x * kBulkWarps) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 acc = zero4;
    if (end > beg) {
      slot_release();
      stage_masked<HP>(qm, a.q + j * a.ldq, nq, dh, lane);
      const bool one = end - beg <= kBulkGroup;
      float m[HP], ssum[HP], ex[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) { m[h] = -FLT_MAX; ssum[h] = 0.f; ex[h] = 0.f; }
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        slot_release();
        if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
        const bool ok = bulk_wait(&bar[w], phase);
        phase ^= 1u;
        if (!ok) return;
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float z[HP];
        if (valid) row_dots_sm<HP, BF>(slot, lane, rowf, 0, qm, nq, z);
        float kp[HP];
        keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
        float wt[HP], sc[HP];
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool okh = valid && h < a.heads;
          const float zz = okh ? leaky(z[h], a.slope) : -FLT_MAX;
          if (!one && okh) a.att_out[e * a.heads + h] = zz;          // raw; normalised below
          const float mn = fmaxf(m[h], fb::warp_max(zz));
          sc[h] = (m[h] == -FLT_MAX) ? 0.f : expf(m[h] - mn);
          m[h] = mn;
          ex[h] = okh ? expf(zz - mn) : 0.f;
          ssum[h] = ssum[h] * sc[h] + fb::warp_sum(ex[h]);
          wt[h] = ex[h] * kp[h];
        }
        const float sa = hv<HP>(sc, hA), sb = hv<HP>(sc, hB);
        acc.x *= sa; acc.y *= sa; acc.z *= sb; acc.w *= sb;
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          float wc[HP];
#pragma unroll
          for (int h = 0; h < HP; ++h) wc[h] = __shfl_sync(0xffffffffu, wt[h], c);
          const float wa = hv<HP>(wc, hA), wb = hv<HP>(wc, hB);
          const float4 v = live ? slot4<BF>(slot, c, rowf, (a.dim >> 2) + lane) : zero4;
          acc.x = fmaf(wa, v.x, acc.x);
          acc.y = fmaf(wa, v.y, acc.y);
          acc.z = fmaf(wb, v.z, acc.z);
          acc.w = fmaf(wb, v.w, acc.w);
        }
      }
      float inv[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) inv[h] = h < a.heads ? 1.f / ssum[h] : 0.f;
      const float ia = hv<HP>(inv, hA), ib = hv<HP>(inv, hB);
      acc.x *= ia; acc.y *= ia; acc.z *= ib; acc.w *= ib;
      if (one) {
        if (lane < end - beg)
#pragma unroll
          for (int h = 0; h < HP; ++h)
            if (h < a.heads) a.att_out[(int64_t)(beg + lane) * a.heads + h] = ex[h] * inv[h];
      } else {
        __syncwarp();
        for (int t = lane; t < (end - beg) * a.heads; t += 32) {
          const int h = t % a.heads;
          float *pz = a.att_out + (int64_t)beg * a.heads + t;
          *pz = expf(*pz - hv<HP>(m, h)) * hv<HP>(inv, h);
        }
      }
    }
    if (live) put4(a.agg, j * a.ldagg + 4 * lane, acc, a.agg_bf16);
  }
}

template <int HP, bool BF>
__global__ void __launch_bounds__(32 * kBulkWarps) k_attn_bwd_b(AttnArgs a) {
  fb::pdl_enter();
  extern __shared__ __align__(128) unsigned char smraw[];
  __shared__ uint64_t bar[kBulkWarps];
  constexpr int kEsz = BF ? 2 : 4;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rowf = (int)a.ldkv;
  unsigned char *slot = smraw + (size_t)w * kBulkGroup * rowf * kEsz;
  const unsigned char *kbase = reinterpret_cast<const unsigned char *>(a.k);
  float4 (*qm)[32] =
      reinterpret_cast<float4 (*)[32]>(smraw + (size_t)kBulkWarps * kBulkGroup * rowf * kEsz) + (size_t)w * 2 * HP;
  float4 (*dm)[32] = qm + HP;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane == 0) bar_init(&bar[w]);
  __syncwarp();
  uint32_t phase = 0;
  for (int64_t j = (int64_t)blockIdx.x * kBulkWarps + w; j < n_dst; j += (int64_t)gridDim.x * kBulkWarps) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 dq = zero4;
    if (end > beg) {
      slot_release();
      stage_masked<HP>(qm, a.q + j * a.ldq, nq, dh, lane);
      stage_masked<HP>(dm, a.dagg + j * a.lddagg, nq, dh, lane);
      const float4 q4 = live ? __ldg(reinterpret_cast<const float4 *>(a.q + j * a.ldq) + lane) : zero4;
      const float4 da4 = live ? __ldg(reinterpret_cast<const float4 *>(a.dagg + j * a.lddagg) + lane) : zero4;
      const bool one = end - beg <= kBulkGroup;
      // pass 1: dL/dy through dropout (lane per edge, V rows), sum_e y dL/dy per head, dV rows
      float sd[HP], dl1[HP], y1[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) { sd[h] = 0.f; dl1[h] = 0.f; y1[h] = 0.f; }
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        slot_release();
        if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
        const bool ok = bulk_wait(&bar[w], phase);
        phase ^= 1u;
        if (!ok) return;
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float d[HP], kp[HP], yk[HP];
        if (valid) row_dots_sm<HP, BF>(slot, lane, rowf, a.dim >> 2, dm, nq, d);
        keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool okh = valid && h < a.heads;
          const float y = okh ? __ldg(a.att + e * a.heads + h) : 0.f;
          const float dl = okh ? d[h] * kp[h] : 0.f;
          sd[h] += fb::warp_sum(y * dl);
          dl1[h] = dl;
          y1[h] = y;
          yk[h] = y * kp[h];
        }
        if (a.dv) {
#pragma unroll 4
          for (int c = 0; c < n; ++c) {
            float yc[HP];
#pragma unroll
            for (int h = 0; h < HP; ++h) yc[h] = __shfl_sync(0xffffffffu, yk[h], c);
            const float ya = hv<HP>(yc, hA), yb = hv<HP>(yc, hB);
            if (live)
              put4(a.dv, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(ya * da4.x, ya * da4.y, yb * da4.z, yb * da4.w), a.kv_bf16);
          }
        }
      }
      // pass 2: logits again (lane per edge, K rows), LeakyReLU and softmax
      // backward, dK rows and dq (lane per feature); a single group is still
      // in the slot
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        if (!one) {
          slot_release();
          if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
          const bool ok = bulk_wait(&bar[w], phase);
          phase ^= 1u;
          if (!ok) return;
        }
        const bool valid = lane < n;
        const int64_t e = g0 + lane;
        float z[HP], dl[HP], y[HP], dz[HP];
        if (valid) row_dots_sm<HP, BF>(slot, lane, rowf, 0, qm, nq, z);
        if (one) {
#pragma unroll
          for (int h = 0; h < HP; ++h) { dl[h] = dl1[h]; y[h] = y1[h]; }
        } else {
          float d[HP], kp[HP];
          if (valid) row_dots_sm<HP, BF>(slot, lane, rowf, a.dim >> 2, dm, nq, d);
          keep_heads<HP>(a, doff, e, valid, inv_keep, kp);
#pragma unroll
          for (int h = 0; h < HP; ++h) {
            const bool okh = valid && h < a.heads;
            y[h] = okh ? __ldg(a.att + e * a.heads + h) : 0.f;
            dl[h] = okh ? d[h] * kp[h] : 0.f;
          }
        }
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          const bool okh = valid && h < a.heads;
          const float g = y[h] * (dl[h] - sd[h]);
          dz[h] = okh ? (z[h] > 0.f ? g : g * a.slope) : 0.f;
        }
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          float zc[HP];
#pragma unroll
          for (int h = 0; h < HP; ++h) zc[h] = __shfl_sync(0xffffffffu, dz[h], c);
          const float za = hv<HP>(zc, hA), zb = hv<HP>(zc, hB);
          if (live) {
            const float4 k = slot4<BF>(slot, c, rowf, lane);
            if (a.dk)
              put4(a.dk, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(za * q4.x, za * q4.y, zb * q4.z, zb * q4.w), a.kv_bf16);
            dq.x = fmaf(za, k.x, dq.x);
            dq.y = fmaf(za, k.y, dq.y);
            dq.z = fmaf(zb, k.z, dq.z);
            dq.w = fmaf(zb, k.w, dq.w);
          }
        }
      }
    }
    if (a.dq && live) put4(a.dq, j * (a.dq_bf16 ? a.lddq : (int64_t)a.dim) + 4 * lane, dq, a.dq_bf16);
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy kernels with lane-per-(edge, head) dot products, for 1 or 2
// heads: lane l holds edge l / HP of the group and head l % HP, and takes the
// dot product over that head's dh features only (the other kernels give every
// lane all heads over all features, with queries masked per head), so a group
// of up to 12 edges keeps 12 * HP lanes busy instead of 12.  Softmax
// statistics are reductions over the lanes of one head; the row outputs stay
// lane-per-feature, each taking its edge's weight from lane c * HP + head.

// sum over t < dh/2 of q[2t] row[2t] + q[2t+1] row[2t+1]: the row is slot row i
// from element f0 (fp32, or bf16 widened), q a float array in shared memory.
template <bool BF>
__device__ __forceinline__ float head_dot(const unsigned char *slot, int i, int rowf, int f0, const float *q, int dh) {
  float acc = 0.f;
  if (BF) {
    const uint32_t *r = reinterpret_cast<const uint32_t *>(slot + ((size_t)i * rowf + f0) * 2);
    const float2 *q2 = reinterpret_cast<const float2 *>(q);
#pragma unroll 5
    for (int t = 0; t < dh / 2; ++t) {
      const uint32_t u = r[t];
      const float2 qq = q2[t];
      acc = fmaf(qq.x, __uint_as_float(u << 16), fmaf(qq.y, __uint_as_float(u & 0xFFFF0000u), acc));
    }
  } else {
    const float2 *r = reinterpret_cast<const float2 *>(slot + ((size_t)i * rowf + f0) * 4);
    const float2 *q2 = reinterpret_cast<const float2 *>(q);
#pragma unroll 5
    for (int t = 0; t < dh / 2; ++t) {
      const float2 k = r[t];
      const float2 qq = q2[t];
      acc = fmaf(qq.x, k.x, fmaf(qq.y, k.y, acc));
    }
  }
  return acc;
}

// Reductions over the lanes of one head (lanes l, l + HP, l + 2 HP, ...).
template <int HP>
__device__ __forceinline__ float head_max(float v) {
#pragma unroll
  for (int o = HP; o < 32; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int HP>
__device__ __forceinline__ float head_sum(float v) {
#pragma unroll
  for (int o = HP; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Dropout keep scale of (edge e, head h): drop_scale()'s decision.
__device__ __forceinline__ float keep1(const AttnArgs &a, uint64_t doff, int64_t e, int h, float inv_keep) {
  if (a.drop_p <= 0.f) return 1.f;
  if (a.mask_u) return a.mask_u[e * a.heads + h] > a.drop_p ? inv_keep : 0.f;
  const fb::Philox4 r = fb::philox4x32_10((uint32_t)e, (uint32_t)(e >> 32), (uint32_t)doff, (uint32_t)(doff >> 32),
                                          (uint32_t)a.seed, (uint32_t)(a.seed >> 32));
  const uint32_t w = h == 0 ? r.v[0] : (h == 1 ? r.v[1] : (h == 2 ? r.v[2] : r.v[3]));
  return ((float)(w >> 8) * (1.0f / 16777216.0f) >= a.drop_p) ? inv_keep : 0.f;
}

// Stages one row of dim floats into a warp's shared-memory array.
__device__ __forceinline__ void stage_row(float *dst, const float *x, int nq, int lane) {
  if (lane < nq) reinterpret_cast<float4 *>(dst)[lane] = __ldg(reinterpret_cast<const float4 *>(x) + lane);
}

template <int HP, bool BF>
__global__ void __launch_bounds__(32 * kBulkWarps) k_attn_fwd_h(AttnArgs a) {
  static_assert(HP == 1 || HP == 2, "lane-per-(edge, head) kernels take 1 or 2 heads");
  fb::pdl_enter();
  extern __shared__ __align__(128) unsigned char smraw[];
  __shared__ uint64_t bar[kBulkWarps];
  constexpr int kEsz = BF ? 2 : 4;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rowf = (int)a.ldkv;
  unsigned char *slot = smraw + (size_t)w * kBulkGroup * rowf * kEsz;
  const unsigned char *kbase = reinterpret_cast<const unsigned char *>(a.k);
  float *qs = reinterpret_cast<float *>(smraw + (size_t)kBulkWarps * kBulkGroup * rowf * kEsz) + (size_t)w * 128;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const int li = lane / HP, lh = lane % HP;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane == 0) bar_init(&bar[w]);
  __syncwarp();
  uint32_t phase = 0;
  if (a.n_dst_dev) {
    for (int64_t j = n_dst + (int64_t)blockIdx.x * kBulkWarps + w; j < a.n_dst;
         j += (int64_t)gridDim.x * kBulkWarps)
      if (live) put4(a.agg, j * a.ldagg + 4 * lane, zero4, a.agg_bf16);
  }
  for (int64_t j = (int64_t)blockIdx.x * kBulkWarps + w; j < n_dst; j += (int64_t)gridDim.x * kBulkWarps) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 acc = zero4;
    if (end > beg) {
      slot_release();
      stage_row(qs, a.q + j * a.ldq, nq, lane);
      const bool one = end - beg <= kBulkGroup;
      float m = -FLT_MAX, ssum = 0.f, ex = 0.f;       // this lane's head
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        slot_release();
        if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
        const bool ok = bulk_wait(&bar[w], phase);
        phase ^= 1u;
        if (!ok) return;
        __syncwarp();
        const bool vl = li < n && lh < a.heads;
        const int64_t e = g0 + li;
        const float z = vl ? head_dot<BF>(slot, li, rowf, lh * dh, qs + lh * dh, dh) : 0.f;
        const float kp = vl ? keep1(a, doff, e, lh, inv_keep) : 0.f;
        const float zz = vl ? leaky(z, a.slope) : -FLT_MAX;
        if (!one && vl) a.att_out[e * a.heads + lh] = zz;          // raw; normalised below
        const float mn = fmaxf(m, head_max<HP>(zz));
        const float sc = (m == -FLT_MAX) ? 0.f : expf(m - mn);
        m = mn;
        ex = vl ? expf(zz - mn) : 0.f;
        ssum = ssum * sc + head_sum<HP>(ex);
        const float wt = ex * kp;
        const float sa = __shfl_sync(0xffffffffu, sc, hA), sb = __shfl_sync(0xffffffffu, sc, hB);
        acc.x *= sa; acc.y *= sa; acc.z *= sb; acc.w *= sb;
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          const float wa = __shfl_sync(0xffffffffu, wt, c * HP + hA);
          const float wb = __shfl_sync(0xffffffffu, wt, c * HP + hB);
          const float4 v = live ? slot4<BF>(slot, c, rowf, (a.dim >> 2) + lane) : zero4;
          acc.x = fmaf(wa, v.x, acc.x);
          acc.y = fmaf(wa, v.y, acc.y);
          acc.z = fmaf(wb, v.z, acc.z);
          acc.w = fmaf(wb, v.w, acc.w);
        }
      }
      const float inv = 1.f / ssum;                   // lanes of a live head
      const float ia = __shfl_sync(0xffffffffu, inv, hA), ib = __shfl_sync(0xffffffffu, inv, hB);
      acc.x *= ia; acc.y *= ia; acc.z *= ib; acc.w *= ib;
      if (one) {
        if (li < end - beg && lh < a.heads) a.att_out[(int64_t)(beg + li) * a.heads + lh] = ex * inv;
      } else {
        float mh[HP], ih[HP];
#pragma unroll
        for (int h = 0; h < HP; ++h) {
          mh[h] = __shfl_sync(0xffffffffu, m, h);
          ih[h] = __shfl_sync(0xffffffffu, inv, h);
        }
        __syncwarp();
        for (int t = lane; t < (end - beg) * a.heads; t += 32) {
          const int h = t % a.heads;
          float *pz = a.att_out + (int64_t)beg * a.heads + t;
          *pz = expf(*pz - hv<HP>(mh, h)) * hv<HP>(ih, h);
        }
      }
    }
    if (live) put4(a.agg, j * a.ldagg + 4 * lane, acc, a.agg_bf16);
  }
}

template <int HP, bool BF>
__global__ void __launch_bounds__(32 * kBulkWarps) k_attn_bwd_h(AttnArgs a) {
  static_assert(HP == 1 || HP == 2, "lane-per-(edge, head) kernels take 1 or 2 heads");
  fb::pdl_enter();
  extern __shared__ __align__(128) unsigned char smraw[];
  __shared__ uint64_t bar[kBulkWarps];
  constexpr int kEsz = BF ? 2 : 4;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rowf = (int)a.ldkv;
  unsigned char *slot = smraw + (size_t)w * kBulkGroup * rowf * kEsz;
  const unsigned char *kbase = reinterpret_cast<const unsigned char *>(a.k);
  float *qs = reinterpret_cast<float *>(smraw + (size_t)kBulkWarps * kBulkGroup * rowf * kEsz) + (size_t)w * 256;
  float *ds = qs + 128;
  const int64_t n_dst = a.n_dst_dev ? min((int64_t)(*a.n_dst_dev), a.n_dst) : a.n_dst;
  const int nq = a.dim / 4, dh = a.dim / a.heads;
  const bool live = lane < nq;
  const int hA = live ? (4 * lane) / dh : 0, hB = live ? (4 * lane + 2) / dh : 0;
  const int li = lane / HP, lh = lane % HP;
  const uint64_t doff = a.offset_dev ? *a.offset_dev : a.offset;
  const float inv_keep = a.drop_p > 0.f ? 1.f / (1.f - a.drop_p) : 1.f;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane == 0) bar_init(&bar[w]);
  __syncwarp();
  uint32_t phase = 0;
  for (int64_t j = (int64_t)blockIdx.x * kBulkWarps + w; j < n_dst; j += (int64_t)gridDim.x * kBulkWarps) {
    const int beg = a.rptr[j], end = a.rptr[j + 1];
    float4 dq = zero4;
    if (end > beg) {
      slot_release();
      stage_row(qs, a.q + j * a.ldq, nq, lane);
      stage_row(ds, a.dagg + j * a.lddagg, nq, lane);
      const float4 q4 = live ? __ldg(reinterpret_cast<const float4 *>(a.q + j * a.ldq) + lane) : zero4;
      const float4 da4 = live ? __ldg(reinterpret_cast<const float4 *>(a.dagg + j * a.lddagg) + lane) : zero4;
      const bool one = end - beg <= kBulkGroup;
      // pass 1 (lane per edge and head): dL/dy through dropout from the V rows,
      // sum_e y dL/dy of the lane's head; dV rows lane-per-feature
      float sd = 0.f, dl1 = 0.f, y1 = 0.f;
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        slot_release();
        if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
        const bool ok = bulk_wait(&bar[w], phase);
        phase ^= 1u;
        if (!ok) return;
        __syncwarp();
        const bool vl = li < n && lh < a.heads;
        const int64_t e = g0 + li;
        const float d = vl ? head_dot<BF>(slot, li, rowf, a.dim + lh * dh, ds + lh * dh, dh) : 0.f;
        const float kp = vl ? keep1(a, doff, e, lh, inv_keep) : 0.f;
        const float y = vl ? __ldg(a.att + e * a.heads + lh) : 0.f;
        const float dl = d * kp;
        sd += head_sum<HP>(y * dl);
        dl1 = dl;
        y1 = y;
        const float yk = y * kp;
        if (a.dv) {
#pragma unroll 4
          for (int c = 0; c < n; ++c) {
            const float ya = __shfl_sync(0xffffffffu, yk, c * HP + hA);
            const float yb = __shfl_sync(0xffffffffu, yk, c * HP + hB);
            if (live)
              put4(a.dv, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(ya * da4.x, ya * da4.y, yb * da4.z, yb * da4.w), a.kv_bf16);
          }
        }
      }
      // pass 2: the logits again from the K rows, LeakyReLU and softmax
      // backward per (edge, head), dK rows and dq lane-per-feature; a single
      // group is still in the slot
      for (int g0 = beg; g0 < end; g0 += kBulkGroup) {
        const int n = min(kBulkGroup, end - g0);
        if (!one) {
          slot_release();
          if (lane == 0) bulk_copy(slot, kbase + (int64_t)g0 * a.ldkv * kEsz, (uint32_t)(n * rowf * kEsz), &bar[w]);
          const bool ok = bulk_wait(&bar[w], phase);
          phase ^= 1u;
          if (!ok) return;
          __syncwarp();
        }
        const bool vl = li < n && lh < a.heads;
        const int64_t e = g0 + li;
        const float z = vl ? head_dot<BF>(slot, li, rowf, lh * dh, qs + lh * dh, dh) : 0.f;
        float dl = dl1, y = y1;
        if (!one) {
          const float d = vl ? head_dot<BF>(slot, li, rowf, a.dim + lh * dh, ds + lh * dh, dh) : 0.f;
          dl = d * (vl ? keep1(a, doff, e, lh, inv_keep) : 0.f);
          y = vl ? __ldg(a.att + e * a.heads + lh) : 0.f;
        }
        const float g = y * (dl - sd);
        const float dz = vl ? (z > 0.f ? g : g * a.slope) : 0.f;
#pragma unroll 4
        for (int c = 0; c < n; ++c) {
          const float za = __shfl_sync(0xffffffffu, dz, c * HP + hA);
          const float zb = __shfl_sync(0xffffffffu, dz, c * HP + hB);
          if (live) {
            const float4 k = slot4<BF>(slot, c, rowf, lane);
            if (a.dk)
              put4(a.dk, (int64_t)(g0 + c) * a.lddkv + 4 * lane,
                   make_float4(za * q4.x, za * q4.y, zb * q4.z, zb * q4.w), a.kv_bf16);
            dq.x = fmaf(za, k.x, dq.x);
            dq.y = fmaf(za, k.y, dq.y);
            dq.z = fmaf(zb, k.z, dq.z);
            dq.w = fmaf(zb, k.w, dq.w);
          }
        }
      }
    }
    if (a.dq && live) put4(a.dq, j * (a.dq_bf16 ? a.lddq : (int64_t)a.dim) + 4 * lane, dq, a.dq_bf16);
  }
}

int attn_grid(int64_t n_dst) {
  static int sms_of[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int &sms = sms_of[dev & 63];
  if (sms == 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
  int64_t need = (n_dst + kWarpsPerCta - 1) / kWarpsPerCta;
  int64_t cap = (int64_t)sms * 8;  // grid-stride beyond a few waves of resident CTAs
  return (int)std::max<int64_t>(1, std::min(need, cap));
}

bool aligned16(const void *p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_attn(const AttnArgs &a, bool bwd) {
  if (a.dim <= 0 || a.dim % 4 || a.dim > 512 || a.heads < 1 || a.heads > kMaxHeads || a.dim % a.heads)
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "attention: need dim % 4 == 0, dim <= 512, 1 <= heads <= 4, dim % heads == 0");
  if ((!a.x && (!a.q || !a.k)) || !a.v || !a.rptr || a.n_dst < 0 || a.ldkv % 4 || a.ldq % 4 || a.ldkv < 0 ||
      a.ldq < 0)
    return fb::set_error(FB_ERR_ARG, "attention: bad pointer or leading dimension (multiples of 4 floats)");
  // bf16 K|V rows are read whole from k (v = k + dim elements need not be 16-byte aligned)
  if (!aligned16(a.q) || !aligned16(a.k) || (!a.kv_in_bf16 && !aligned16(a.v)) || (a.kv_in_bf16 && a.ldkv % 8))
    return fb::set_error(FB_ERR_ARG, "attention: q/k/v must be 16-byte aligned");
  if (!(a.drop_p >= 0.f && a.drop_p < 1.f)) return fb::set_error(FB_ERR_ARG, "attention: dropout p must be in [0, 1)");
  if (!bwd) {
    if (!a.att_out || !a.agg || a.ldagg % 4 || (!a.agg_bf16 && !aligned16(a.agg)))
      return fb::set_error(FB_ERR_ARG, "attn_fwd: bad att/agg output");
  } else {
    // fp32 gradient rows are stored as 16-byte words, bf16 ones as 8-byte words
    const uintptr_t kv_mask = a.kv_bf16 ? 7u : 15u;
    const bool kv_ok = ((reinterpret_cast<uintptr_t>(a.dk) | reinterpret_cast<uintptr_t>(a.dv)) & kv_mask) == 0;
    if (!a.att || !a.dagg || a.lddagg % 4 || !aligned16(a.dagg) || a.lddkv % 4 || !kv_ok ||
        (!a.dq_bf16 && !aligned16(a.dq)))
      return fb::set_error(FB_ERR_ARG, "attn_bwd: bad gradient buffers");
  }
  return FB_OK;
}

// The edge-parallel kernels take rows of <= 128 floats with logits from q.k,
// an even per-head width, one output row per segment, and (backward) no
// pre-activation gradient output.
// FB_GENERIC_ATTN in the environment forces the general kernels.
bool short_path(const AttnArgs &a) {
  static const bool generic = getenv("FB_GENERIC_ATTN") != nullptr;
  return !generic && a.dim <= 128 && !a.x && !a.seg_row && !a.dx && a.heads != 3 && (a.dim / a.heads) % 2 == 0;
}

// Bulk-copy kernels: the edge-parallel shapes with the interleaved K|V rows.
bool bulk_path(const AttnArgs &a) {
  static const bool off = getenv("FB_NO_BULK_ATTN") != nullptr;
  const size_t esz = a.kv_in_bf16 ? 2 : 4;
  const bool interleaved = reinterpret_cast<const char *>(a.v) == reinterpret_cast<const char *>(a.k) + a.dim * esz;
  return (!off || a.kv_in_bf16) && short_path(a) && interleaved && a.ldkv == 2 * a.dim;
}

size_t bulk_smem(const AttnArgs &a, int hp, bool bwd) {
  const size_t esz = a.kv_in_bf16 ? 2 : 4;
  // the masked-query kernels stage hp rows of 32 float4 per staged vector;
  // the lane-per-(edge, head) kernels (hp <= 2) one row of 128 floats
  const size_t per = hp <= 2 ? 128 * 4 : (size_t)hp * 32 * 16;
  return (size_t)kBulkWarps * ((size_t)kBulkGroup * a.ldkv * esz + (bwd ? 2 : 1) * per);
}

int bulk_grid(int64_t n_dst) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n_dst + kBulkWarps - 1) / kBulkWarps, (int64_t)148 * 16));
}

// Opts a kernel into `bytes` of dynamic shared memory once per device.
template <typename K>
int allow_smem(K kernel, size_t bytes, int slot) {
  static size_t done[24][64] = {};
  int dev = 0;
  FB_TRY_CUDA(cudaGetDevice(&dev));
  size_t &d = done[slot % 24][dev & 63];
  if (d < bytes) {
    FB_TRY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    d = bytes;
  }
  return FB_OK;
}

template <int HP, bool BF>
int launch_bulk_t(const AttnArgs &a, bool bwd, cudaStream_t stream) {
  const size_t sm = bulk_smem(a, HP, bwd);
  const int grid = bulk_grid(a.n_dst);
  const int slot = (HP == 1 ? 0 : (HP == 2 ? 1 : 2)) + (bwd ? 3 : 0) + (BF ? 6 : 0);
  int rc;
  if constexpr (HP <= 2) {
    // lane-per-(edge, head) dot products (FB_MASKED_ATTN selects the masked-query kernels)
    static const bool masked = getenv("FB_MASKED_ATTN") != nullptr;
    if (!masked) {
      if (bwd) {
        if ((rc = allow_smem(k_attn_bwd_h<HP, BF>, sm, slot))) return rc;
        FB_TRY_CUDA(fb::launch(k_attn_bwd_h<HP, BF>, grid, 32 * kBulkWarps, sm, stream, a));
        FB_LAUNCHED("k_attn_bwd_h");
      } else {
        if ((rc = allow_smem(k_attn_fwd_h<HP, BF>, sm, slot))) return rc;
        FB_TRY_CUDA(fb::launch(k_attn_fwd_h<HP, BF>, grid, 32 * kBulkWarps, sm, stream, a));
        FB_LAUNCHED("k_attn_fwd_h");
      }
      return FB_OK;
    }
  }
  const size_t smm = (size_t)kBulkWarps * ((size_t)kBulkGroup * a.ldkv * (BF ? 2 : 4) + (bwd ? 2 : 1) *
                                           (size_t)HP * 32 * 16);
  if (bwd) {
    if ((rc = allow_smem(k_attn_bwd_b<HP, BF>, smm, slot + 12))) return rc;
    FB_TRY_CUDA(fb::launch(k_attn_bwd_b<HP, BF>, grid, 32 * kBulkWarps, smm, stream, a));
    FB_LAUNCHED("k_attn_bwd_b");
  } else {
    if ((rc = allow_smem(k_attn_fwd_b<HP, BF>, smm, slot + 12))) return rc;
    FB_TRY_CUDA(fb::launch(k_attn_fwd_b<HP, BF>, grid, 32 * kBulkWarps, smm, stream, a));
    FB_LAUNCHED("k_attn_fwd_b");
  }
  return FB_OK;
}

template <int HP>
int launch_bulk(const AttnArgs &a, bool bwd, cudaStream_t stream) {
  return a.kv_in_bf16 ? launch_bulk_t<HP, true>(a, bwd, stream) : launch_bulk_t<HP, false>(a, bwd, stream);
}

int launch_fwd(const AttnArgs &a, cudaStream_t stream) {
  int rc = check_attn(a, false);
  if (rc) return rc;
  if ((a.kv_in_bf16 || a.agg_bf16 || a.dq_bf16) && !bulk_path(a))
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "attention: bf16 K|V rows and bf16 outputs need interleaved rows [E, 2 dim], dim <= 128");
  if ((a.agg_bf16 && ((reinterpret_cast<uintptr_t>(a.agg) & 7u) || a.ldagg % 4)) ||
      (a.dq_bf16 && a.dq && ((reinterpret_cast<uintptr_t>(a.dq) & 7u) || a.lddq % 4 || a.lddq < a.dim)))
    return fb::set_error(FB_ERR_ARG, "attention: bf16 outputs need 8-byte aligned rows, pitch a multiple of 4");
  if (a.n_dst == 0) return FB_OK;
  const int grid = attn_grid(a.n_dst), nv = (a.dim / 4 + 31) / 32;
  if (bulk_path(a)) {
    if (a.heads == 1) return launch_bulk<1>(a, false, stream);
    if (a.heads == 2) return launch_bulk<2>(a, false, stream);
    return launch_bulk<4>(a, false, stream);
  }
  if (short_path(a)) {
    if (a.heads == 1) k_attn_fwd_s<1><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    else if (a.heads == 2) k_attn_fwd_s<2><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    else k_attn_fwd_s<4><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    FB_LAUNCHED("k_attn_fwd_s");
    return FB_OK;
  }
  switch (nv) {
    case 1: k_attn_fwd<1><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    case 2: k_attn_fwd<2><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    case 3: k_attn_fwd<3><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    default: k_attn_fwd<4><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
  }
  FB_LAUNCHED("k_attn_fwd");
  return FB_OK;
}

int launch_bwd(const AttnArgs &a, cudaStream_t stream) {
  int rc = check_attn(a, true);
  if (rc) return rc;
  if ((a.kv_in_bf16 || a.agg_bf16 || a.dq_bf16) && !bulk_path(a))
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "attention: bf16 K|V rows and bf16 outputs need interleaved rows [E, 2 dim], dim <= 128");
  if ((a.agg_bf16 && ((reinterpret_cast<uintptr_t>(a.agg) & 7u) || a.ldagg % 4)) ||
      (a.dq_bf16 && a.dq && ((reinterpret_cast<uintptr_t>(a.dq) & 7u) || a.lddq % 4 || a.lddq < a.dim)))
    return fb::set_error(FB_ERR_ARG, "attention: bf16 outputs need 8-byte aligned rows, pitch a multiple of 4");
  if (a.n_dst == 0) return FB_OK;
  const int grid = attn_grid(a.n_dst), nv = (a.dim / 4 + 31) / 32;
  if (bulk_path(a)) {
    if (a.heads == 1) return launch_bulk<1>(a, true, stream);
    if (a.heads == 2) return launch_bulk<2>(a, true, stream);
    return launch_bulk<4>(a, true, stream);
  }
  if (short_path(a)) {
    if (a.heads == 1) k_attn_bwd_s<1><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    else if (a.heads == 2) k_attn_bwd_s<2><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    else k_attn_bwd_s<4><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a);
    FB_LAUNCHED("k_attn_bwd_s");
    return FB_OK;
  }
  switch (nv) {
    case 1: k_attn_bwd<1><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    case 2: k_attn_bwd<2><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    case 3: k_attn_bwd<3><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
    default: k_attn_bwd<4><<<grid, 32 * kWarpsPerCta, 0, stream>>>(a); break;
  }
  FB_LAUNCHED("k_attn_bwd");
  return FB_OK;
}

__global__ void k_dropout_scale(int64_t E, int heads, float p, uint64_t seed, uint64_t offset, float *out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  float s[kMaxHeads];
  drop_scale(e, heads, p, seed, offset, nullptr, s);
  for (int h = 0; h < heads; ++h) out[e * heads + h] = s[h];
}

}  // namespace

extern "C" int fb_attn_error(int *flags, int clear) {
  if (!flags) return fb::set_error(FB_ERR_ARG, "attn_error: null flags");
  FB_TRY_CUDA(cudaMemcpyFromSymbol(flags, g_attn_err, sizeof(int)));
  if (clear) {
    const int zero = 0;
    FB_TRY_CUDA(cudaMemcpyToSymbol(g_attn_err, &zero, sizeof(int)));
  }
  return FB_OK;
}

extern "C" int fb_dropout_scale(int64_t n_edges, int heads, float drop_p, uint64_t seed, uint64_t offset, float *out,
                                cudaStream_t stream) {
  if (n_edges < 0 || heads < 1 || heads > kMaxHeads || !(drop_p >= 0.f && drop_p < 1.f) || (n_edges && !out))
    return fb::set_error(FB_ERR_ARG, "dropout_scale: bad argument");
  if (n_edges == 0) return FB_OK;
  k_dropout_scale<<<(unsigned)((n_edges + 255) / 256), 256, 0, stream>>>(n_edges, heads, drop_p, seed, offset, out);
  FB_LAUNCHED("k_dropout_scale");
  return FB_OK;
}

extern "C" int fb_attn_fwd(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                           const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                           float slope, float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                           float *att, float *agg, int64_t ldagg, cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.k = k; a.v = v; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att_out = att; a.agg = agg; a.ldagg = ldagg;
  return launch_fwd(a, stream);
}

extern "C" int fb_attn_bwd(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                           const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                           float slope, float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                           const float *att, const float *dagg, int64_t lddagg, float *dq, float *dk, float *dv,
                           int64_t lddkv, cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.k = k; a.v = v; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att = att; a.dagg = dagg; a.lddagg = lddagg; a.dq = dq; a.dk = dk; a.dv = dv; a.lddkv = lddkv;
  return launch_bwd(a, stream);
}

// fb_attn_bwd with dk / dv written as bf16 (round to nearest even): the K|V
// gradient that feeds the bf16 projection GEMMs.  lddkv % 4 == 0.
extern "C" int fb_attn_bwd_bf16kv(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                                  const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                                  float slope, float drop_p, uint64_t seed, uint64_t offset,
                                  const uint64_t *offset_dev, const float *att, const float *dagg, int64_t lddagg,
                                  float *dq, uint16_t *dk, uint16_t *dv, int64_t lddkv, cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.k = k; a.v = v; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att = att; a.dagg = dagg; a.lddagg = lddagg; a.dq = dq; a.lddkv = lddkv;
  a.dk = reinterpret_cast<float *>(dk);
  a.dv = reinterpret_cast<float *>(dv);
  a.kv_bf16 = 1;
  return launch_bwd(a, stream);
}

// The attention forward on bf16 K|V rows kv[E, ldkv] (K in the first dim
// columns, V in the next dim): the K|V projection's bf16 output in the bf16
// projection mode.  Softmax, dropout and the weighted sum run in fp32.
extern "C" int fb_attn_fwd_kvbf16(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv,
                                  const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                                  float slope, float drop_p, uint64_t seed, uint64_t offset,
                                  const uint64_t *offset_dev, float *att, float *agg, int64_t ldagg,
                                  cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.k = reinterpret_cast<const float *>(kv);
  a.v = reinterpret_cast<const float *>(kv + dim);
  a.kv_in_bf16 = 1;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att_out = att; a.agg = agg; a.ldagg = ldagg;
  return launch_fwd(a, stream);
}

// Its backward: reads the bf16 K|V rows, writes dq fp32 and dK|dV as bf16
// rows dkv[E, lddkv] in the same interleaved layout.
extern "C" int fb_attn_bwd_kvbf16(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv,
                                  const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                                  float slope, float drop_p, uint64_t seed, uint64_t offset,
                                  const uint64_t *offset_dev, const float *att, const float *dagg, int64_t lddagg,
                                  float *dq, uint16_t *dkv, int64_t lddkv, cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.k = reinterpret_cast<const float *>(kv);
  a.v = reinterpret_cast<const float *>(kv + dim);
  a.kv_in_bf16 = 1;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att = att; a.dagg = dagg; a.lddagg = lddagg; a.dq = dq; a.lddkv = lddkv;
  a.dk = reinterpret_cast<float *>(dkv);
  a.dv = reinterpret_cast<float *>(dkv + dim);
  a.kv_bf16 = 1;
  return launch_bwd(a, stream);
}

// fb_attn_fwd_kvbf16 with agg written as bf16 (round to nearest even) at
// ldagg elements per row: the aggregate is only the w_out product's bf16
// operand in the bf16 projection mode.
extern "C" int fb_attn_fwd_kvbf16_bf16out(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv,
                                          const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads,
                                          int dim, float slope, float drop_p, uint64_t seed, uint64_t offset,
                                          const uint64_t *offset_dev, float *att, uint16_t *agg, int64_t ldagg,
                                          cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.k = reinterpret_cast<const float *>(kv);
  a.v = reinterpret_cast<const float *>(kv + dim);
  a.kv_in_bf16 = 1;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att_out = att; a.agg = reinterpret_cast<float *>(agg); a.ldagg = ldagg; a.agg_bf16 = 1;
  return launch_fwd(a, stream);
}

// fb_attn_bwd_kvbf16 with dq written as bf16 at lddq elements per row: dq is
// only the bf16 operand of the Q-side gradient products.
extern "C" int fb_attn_bwd_kvbf16_bf16dq(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv,
                                         const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads,
                                         int dim, float slope, float drop_p, uint64_t seed, uint64_t offset,
                                         const uint64_t *offset_dev, const float *att, const float *dagg,
                                         int64_t lddagg, uint16_t *dq, int64_t lddq, uint16_t *dkv, int64_t lddkv,
                                         cudaStream_t stream) {
  AttnArgs a{};
  a.offset_dev = offset_dev;
  a.q = q; a.ldq = ldq; a.ldkv = ldkv; a.rptr = rptr; a.n_dst = n_dst; a.n_dst_dev = n_dst_dev;
  a.k = reinterpret_cast<const float *>(kv);
  a.v = reinterpret_cast<const float *>(kv + dim);
  a.kv_in_bf16 = 1;
  a.heads = heads; a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.seed = seed; a.offset = offset;
  a.att = att; a.dagg = dagg; a.lddagg = lddagg; a.lddkv = lddkv;
  a.dq = reinterpret_cast<float *>(dq); a.dq_bf16 = 1; a.lddq = lddq;
  a.dk = reinterpret_cast<float *>(dkv);
  a.dv = reinterpret_cast<float *>(dkv + dim);
  a.kv_bf16 = 1;
  return launch_bwd(a, stream);
}

extern "C" int fb_attn_logits_fwd(const float *x, const float *v, int64_t ldv, const int32_t *indptr, int64_t n_seg,
                                  const int64_t *seg_row, int64_t n_out, int heads, int dim, float slope,
                                  float drop_p, const float *mask_u, float *att, float *agg, cudaStream_t stream) {
  AttnArgs a{};
  a.n_out = n_out;
  a.x = x; a.v = v; a.ldkv = ldv; a.rptr = indptr; a.n_dst = n_seg; a.seg_row = seg_row; a.heads = heads;
  a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.mask_u = mask_u; a.att_out = att; a.agg = agg; a.ldagg = dim;
  if (!x) return fb::set_error(FB_ERR_ARG, "attn_logits_fwd: x is required");
  return launch_fwd(a, stream);
}

extern "C" int fb_attn_logits_bwd(const float *x, const float *v, int64_t ldv, const int32_t *indptr, int64_t n_seg,
                                  const int64_t *seg_row, int64_t n_out, int heads, int dim, float slope,
                                  float drop_p, const float *mask_u, const float *att, const float *dagg, float *dx,
                                  float *dv, cudaStream_t stream) {
  AttnArgs a{};
  a.n_out = n_out;
  a.x = x; a.v = v; a.ldkv = ldv; a.rptr = indptr; a.n_dst = n_seg; a.seg_row = seg_row; a.heads = heads;
  a.dim = dim; a.slope = slope; a.drop_p = drop_p; a.mask_u = mask_u; a.att = att; a.dagg = dagg; a.lddagg = dim;
  a.dx = dx; a.dv = dv; a.lddkv = ldv;
  if (!x) return fb::set_error(FB_ERR_ARG, "attn_logits_bwd: x is required");
  return launch_bwd(a, stream);
}
