// Temporal neighbour sampler on the device: the stateful time pointers,
// most-recent-k and uniform-k sampling, COO/CSR block construction and eid
// dedup, all on one CUDA stream without host round trips.
//
// Reference: NoneBone/FAST getSamplerCore/sampler_core.cpp
//   update_ts_ptr   :133-157   pointer scan          -> k_update_ptr (binary search + atomicMax)
//   sample_layer    :458-595   per-root window/pick  -> k_sample_count + k_sample_write
//   combine_coo     :185-456   concat / cntE / dedup -> scan offsets, rptr/cntE, k_dedup_*
//   sample          :597-712   layer/history driver  -> fb_sampler_sample
//
// Layout per block (all device, int32 unless noted): row/col/eid[E], then
// ts/dts(float)/nodes[R+E] with the R roots first, rptr[R+1] over every root,
// cntE[S+1] over non-empty roots, dims[8] = {R, E, S, R+E, n_uni}.
#include <algorithm>
#include <climits>
#include <vector>
#include "runtime.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kErrRootRange = 1;

struct BlockBuf {
  int32_t *row = nullptr, *col = nullptr, *eid = nullptr, *nodes = nullptr;
  int32_t *rptr = nullptr, *cntE = nullptr, *uniE = nullptr, *invE = nullptr, *nbr = nullptr;
  float *ts = nullptr, *dts = nullptr, *dte = nullptr;
  int64_t cap_roots = 0, cap_edges = 0;
};

// First index in [lo, hi) with ts[i] > v (std::upper_bound on a sorted run).
__device__ __forceinline__ int upper_bound_dev(const float *__restrict__ ts, int lo, int hi, float v) {
  while (lo < hi) {
    int mid = lo + ((hi - lo) >> 1);
    if (v < __ldg(ts + mid)) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// A group of kGroup lanes works on one root: the time-window search probes
// kGroup positions per round (a (kGroup+1)-ary search) and each lane takes
// one candidate pick, so a root costs a few dependent memory latencies
// instead of one per search step and per pick.
constexpr int kGroup = 16;
constexpr int kRootsPerCta = kThreads / kGroup;

struct Lanes {
  int gl;          // lane within the group
  unsigned mask;   // the group's lanes in the warp
  int shift;       // bit offset of the group in a warp ballot
};

__device__ __forceinline__ Lanes group_lanes() {
  const int lane = threadIdx.x & 31;
  Lanes L;
  L.gl = lane & (kGroup - 1);
  L.shift = lane & ~(kGroup - 1);
  L.mask = ((1u << kGroup) - 1) << L.shift;
  return L;
}

// The group's ballot of pred, bit i = lane i of the group.
__device__ __forceinline__ unsigned group_ballot(bool pred, const Lanes &L) {
  return (__ballot_sync(L.mask, pred) >> L.shift) & ((1u << kGroup) - 1);
}

// upper_bound_dev by the lanes of a group (same result in every lane).
__device__ __forceinline__ int upper_bound_group(const float *__restrict__ ts, int lo, int hi, float v,
                                                 const Lanes &L) {
  while (hi - lo > kGroup) {
    const int len = hi - lo;
    const int q = lo + (int)(((int64_t)(L.gl + 1) * len) / (kGroup + 1));
    const unsigned b = group_ballot(v < __ldg(ts + q), L);   // probes ascend, so b is 0..0 1..1
    const int t = b ? __ffs(b) - 1 : kGroup;                  // first probe with ts > v
    const int q_before = __shfl_sync(L.mask, q, t > 0 ? t - 1 : 0, kGroup);
    const int q_at = __shfl_sync(L.mask, q, t < kGroup ? t : kGroup - 1, kGroup);
    if (t > 0) lo = q_before + 1;
    if (t < kGroup) hi = q_at;
  }
  const int i = lo + L.gl;
  const unsigned b = group_ballot(i < hi && v < __ldg(ts + i), L);
  return b ? lo + __ffs(b) - 1 : hi;
}

struct SampleArgs {
  const int32_t *indptr, *indices, *eid;
  const float *ts;
  int64_t n_nodes;
  const int32_t *ptr_s, *ptr_e;  // pointer slots (nh-1-i) and (nh-i)
  const int32_t *roots;
  const float *rts;
  int64_t R_host;
  const int32_t *R_dev;
  int use_ptr, num_history, neighs, recent, prop_time;
  float wd, offset;
  uint32_t key0, key1, slot;
  const uint32_t *call_dev;  // sampler step counter (device)
  int32_t *err;
  int32_t *pick;             // staging: the kept edge indices of root j at pick[j * neighs + i]
};

__device__ __forceinline__ int64_t num_roots(const SampleArgs &a) {
  return a.R_dev ? (int64_t)(*a.R_dev) : a.R_host;
}

// The window [s, e] of one root (sampler_core.cpp:522-552), by its group.
__device__ __forceinline__ void root_window(const SampleArgs &a, int n, float nts, int &s, int &e, const Lanes &L) {
  if (a.use_ptr) {
    s = a.ptr_s[n];
    e = a.ptr_e[n];
  } else if (a.num_history == 1) {
    s = a.indptr[n];
    int ub = upper_bound_group(a.ts, a.indptr[n], a.indptr[n + 1], nts, L);
    e = max(ub - 1, s);
  } else {
    int lo = a.indptr[n], hi = a.indptr[n + 1];
    int ub = upper_bound_group(a.ts, lo, hi, __fsub_rn(__fadd_rn(nts, a.offset), a.wd), L);
    s = max(ub - 1, lo);
    int ub2 = upper_bound_group(a.ts, lo, hi, __fadd_rn(nts, a.offset), L);
    e = max(ub2 - 1, s);
  }
}

// Uniform pick number i of root j: s + floor(u * (e - s + 1)), u the
// (i % 4)-th word of Philox(j, i / 4; step, slot).
__device__ __forceinline__ int uniform_pick_u(uint32_t u, int s, int e) {
  const uint32_t span = (uint32_t)(e - s + 1);
  return s + (int)(((uint64_t)u * (uint64_t)span) >> 32);
}

// The kept neighbours of root j in the reference order, one candidate per
// lane: store(rank, k) for each kept edge k; returns the kept count (the same
// in every lane of the group).
template <typename F>
__device__ __forceinline__ int group_picks(const SampleArgs &a, int64_t j, int n, float nts, const Lanes &L,
                                           F store) {
  int s, e;
  root_window(a, n, nts, s, e, L);
  const float keep_thr = __fsub_rn(__fadd_rn(nts, a.offset), 1e-7f);
  const unsigned below = (1u << L.gl) - 1;
  int c = 0;
  if (a.recent || (e - s < a.neighs)) {
    // candidates k = e, e - 1, ..., lo + 1
    const int lo = max(s, e - a.neighs);
    for (int base = 0; base < e - lo; base += kGroup) {
      const int k = e - base - L.gl;
      const bool keep = base + L.gl < e - lo && __ldg(a.ts + k) < keep_thr;
      const unsigned b = group_ballot(keep, L);
      if (keep) store(c + __popc(b & below), k);
      c += __popc(b);
    }
  } else {
    const uint32_t step = *a.call_dev;
    for (int base = 0; base < a.neighs; base += kGroup) {
      const int i = base + L.gl;
      bool keep = false;
      int k = 0;
      if (i < a.neighs) {
        const fb::Philox4 r = fb::philox4x32_10((uint32_t)j, (uint32_t)(i >> 2), step, a.slot, a.key0, a.key1);
        const int w = i & 3;
        const uint32_t u = w == 0 ? r.v[0] : (w == 1 ? r.v[1] : (w == 2 ? r.v[2] : r.v[3]));
        k = uniform_pick_u(u, s, e);
        keep = __ldg(a.ts + k) < keep_thr;
      }
      const unsigned b = group_ballot(keep, L);
      if (keep) store(c + __popc(b & below), k);
      c += __popc(b);
    }
  }
  return c;
}

__global__ void k_bump_call(uint32_t *call) {
  fb::pdl_enter(); *call += 1; }

__global__ void k_set_call(uint32_t *call, uint32_t v) { *call = v; }

__global__ void k_reset(const int32_t *__restrict__ indptr, int32_t *__restrict__ ptr, int64_t n_nodes,
                        int nslots) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_nodes) return;
  int32_t v = indptr[i];
  for (int s = 0; s < nslots; ++s) ptr[s * n_nodes + i] = v;
}

// update_ts_ptr (sampler_core.cpp:133-157).  With per-node time-sorted
// edges the reference scan leaves ptr = max(ptr, ub - 1), ub = first edge with
// ts > root_ts + offset - 1e-7f; a max is order independent, so every root
// applies its candidate with one atomicMax instead of a per-node lock.
// One group of kGroup lanes per root.
__global__ void k_update_ptr(const int32_t *__restrict__ indptr, const float *__restrict__ ts,
                             int64_t n_nodes, int32_t *__restrict__ ptr, const int32_t *__restrict__ roots,
                             const float *__restrict__ rts, int64_t R_host, const int32_t *R_dev,
                             float offset, int32_t *err) {
  fb::pdl_enter();
  const Lanes L = group_lanes();
  const int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / kGroup;
  const int64_t R = R_dev ? (int64_t)(*R_dev) : R_host;
  if (j >= R) return;                       // whole groups leave together
  const int n = roots[j];
  if (n < 0 || n >= n_nodes) {
    if (L.gl == 0) atomicOr(err, kErrRootRange);
    return;
  }
  const int beg = indptr[n], end = indptr[n + 1];
  if (end <= beg) return;
  const float thr = __fsub_rn(__fadd_rn(rts[j], offset), 1e-7f);
  const int ub = upper_bound_group(ts, beg, end, thr, L);
  if (L.gl == 0 && ub > beg) atomicMax(ptr + n, ub - 1);
}

// Pass 1: kept-edge count per root, its picks staged for pass 3, plus per-CTA
// partial sums (edges, non-empty rows).
__global__ void __launch_bounds__(kThreads) k_sample_count(SampleArgs a, int32_t *__restrict__ cnt,
                                                           int2 *__restrict__ part) {
  fb::pdl_enter();
  __shared__ int sm[64];
  const Lanes L = group_lanes();
  const int64_t j = (int64_t)blockIdx.x * kRootsPerCta + threadIdx.x / kGroup;
  const int64_t R = num_roots(a);
  int c = 0;
  if (j < R) {
    const int n = a.roots[j];
    if (n >= 0 && n < a.n_nodes) {
      int32_t *pk = a.pick + j * a.neighs;
      c = group_picks(a, j, n, a.rts[j], L, [&](int rank, int k) { pk[rank] = k; });
    } else if (L.gl == 0) {
      atomicOr(a.err, kErrRootRange);
    }
    if (L.gl == 0) cnt[j] = c;
  }
  const int lead = L.gl == 0 ? c : 0;         // one value per root
  int ea, eb;
  int2 tot = fb::block_excl_scan2(lead, lead > 0 ? 1 : 0, ea, eb, sm);
  if (threadIdx.x == 0) part[blockIdx.x] = tot;
}

// Pass 2: one CTA turns the partial sums into exclusive CTA offsets and
// publishes the block dims; it also writes the closing entries of rptr/cntE.
__global__ void __launch_bounds__(1024) k_scan_parts(int2 *__restrict__ part, int nparts, int64_t R_host,
                                                     const int32_t *R_dev, int32_t *__restrict__ dims,
                                                     int32_t *__restrict__ rptr, int32_t *__restrict__ cntE) {
  fb::pdl_enter();
  __shared__ int sm[64];
  int runA = 0, runB = 0;
  for (int base = 0; base < nparts; base += blockDim.x) {
    int i = base + threadIdx.x;
    int2 v = i < nparts ? part[i] : make_int2(0, 0);
    int ea, eb;
    int2 tot = fb::block_excl_scan2(v.x, v.y, ea, eb, sm);
    if (i < nparts) part[i] = make_int2(runA + ea, runB + eb);
    runA += tot.x;
    runB += tot.y;
  }
  if (threadIdx.x == 0) {
    int R = R_dev ? *R_dev : (int)R_host;
    dims[0] = R;
    dims[1] = runA;
    dims[2] = runB;
    dims[3] = R + runA;
    dims[4] = 0;
    rptr[R] = runA;
    if (runA > 0) cntE[runB] = runA;
  }
}

// Pass 3: offsets from the CTA scan, then the COO/CSR writes of the staged picks.
__global__ void __launch_bounds__(kThreads) k_sample_write(SampleArgs a, const int32_t *__restrict__ cnt,
                                                           const int2 *__restrict__ part,
                                                           int32_t *__restrict__ row, int32_t *__restrict__ col,
                                                           int32_t *__restrict__ eid_out, float *__restrict__ ts_out,
                                                           float *__restrict__ dts_out, int32_t *__restrict__ nodes_out,
                                                           int32_t *__restrict__ rptr, int32_t *__restrict__ cntE,
                                                           float *__restrict__ dte, int32_t *__restrict__ nbr) {
  fb::pdl_enter();
  __shared__ int sm[64];
  const Lanes L = group_lanes();
  const int64_t j = (int64_t)blockIdx.x * kRootsPerCta + threadIdx.x / kGroup;
  const int64_t R = num_roots(a);
  const int c = (j < R) ? cnt[j] : 0;
  const int lead = L.gl == 0 ? c : 0;
  int ea, eb;
  fb::block_excl_scan2(lead, lead > 0 ? 1 : 0, ea, eb, sm);
  ea = __shfl_sync(0xffffffffu, ea, L.shift);   // the root's offsets, from its group's first lane
  eb = __shfl_sync(0xffffffffu, eb, L.shift);
  if (j >= R) return;
  const int2 base = part[blockIdx.x];
  const int off = base.x + ea;
  const int seg = base.y + eb;
  const int n = a.roots[j];
  const float nts = a.rts[j];
  if (L.gl == 0) {
    ts_out[j] = nts;
    dts_out[j] = 0.f;
    nodes_out[j] = n;
    rptr[j] = off;
    if (c > 0) cntE[seg] = off;
  }
  if (n < 0 || n >= a.n_nodes) return;
  const int32_t *pk = a.pick + j * a.neighs;   // the count pass's picks, in the reference order
  for (int i = L.gl; i < c; i += kGroup) {
    const int t = off + i;
    const int k = pk[i];
    const float tk = __ldg(a.ts + k);
    const float d = __fsub_rn(nts, tk);
    const int32_t nb = __ldg(a.indices + k);
    row[t] = (int32_t)j;
    col[t] = (int32_t)(R + t);
    eid_out[t] = __ldg(a.eid + k);
    ts_out[R + t] = a.prop_time ? nts : tk;
    dts_out[R + t] = d;
    nodes_out[R + t] = nb;
    dte[t] = d;
    nbr[t] = nb;
  }
}

// ---- eid dedup (combine_coo :414-451), first-appearance order -------------
__global__ void k_dedup_init(int32_t *keys, int32_t *minpos, int64_t cap) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < cap) { keys[i] = -1; minpos[i] = INT_MAX; }
}

__device__ __forceinline__ uint32_t hash_eid(int32_t k) { return (uint32_t)k * 2654435761u; }

__global__ void k_dedup_insert(const int32_t *__restrict__ eid, const int32_t *dims, int32_t *keys,
                               int32_t *minpos, int32_t *slot, uint32_t mask) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dims[1]) return;
  int32_t k = eid[i];
  uint32_t h = hash_eid(k) & mask;
  // Linear probing; the table holds at least 2x the edges, so a free or
  // matching slot is always found within `mask + 1` probes.
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    int32_t prev = atomicCAS(keys + h, -1, k);
    if (prev == -1 || prev == k) {
      atomicMin(minpos + h, (int32_t)i);
      slot[i] = (int32_t)h;
      return;
    }
    h = (h + 1) & mask;
  }
}

__global__ void __launch_bounds__(kThreads) k_dedup_count(const int32_t *dims, const int32_t *minpos,
                                                          const int32_t *slot, int2 *part) {
  __shared__ int sm[64];
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int first = (i < dims[1]) ? (minpos[slot[i]] == (int32_t)i) : 0;
  int ea, eb;
  int2 tot = fb::block_excl_scan2(first, 0, ea, eb, sm);
  if (threadIdx.x == 0) part[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024) k_dedup_scan(int2 *part, int nparts, int32_t *dims) {
  __shared__ int sm[64];
  int run = 0;
  for (int base = 0; base < nparts; base += blockDim.x) {
    int i = base + threadIdx.x;
    int v = i < nparts ? part[i].x : 0;
    int ea, eb;
    int2 tot = fb::block_excl_scan2(v, 0, ea, eb, sm);
    if (i < nparts) part[i].x = run + ea;
    run += tot.x;
  }
  if (threadIdx.x == 0) dims[4] = run;
}

__global__ void __launch_bounds__(kThreads) k_dedup_emit(const int32_t *__restrict__ eid, const int32_t *dims,
                                                         const int32_t *minpos, const int32_t *slot,
                                                         const int2 *part, int32_t *uidx, int32_t *uniE) {
  __shared__ int sm[64];
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int E = dims[1];
  int first = (i < E) ? (minpos[slot[i]] == (int32_t)i) : 0;
  int ea, eb;
  fb::block_excl_scan2(first, 0, ea, eb, sm);
  if (i < E && first) {
    int u = part[blockIdx.x].x + ea;
    uidx[i] = u;
    uniE[u] = eid[i];
  }
}

__global__ void k_dedup_inv(const int32_t *dims, const int32_t *minpos, const int32_t *slot,
                            const int32_t *uidx, int32_t *invE) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dims[1]) return;
  invE[i] = uidx[minpos[slot[i]]];
}

inline int nblk(int64_t n, int t = kThreads) { return (int)std::max<int64_t>(1, (n + t - 1) / t); }

}  // namespace

struct fb_sampler {
  int device = 0;
  int64_t n_nodes = 0, n_edges = 0;
  int32_t *indptr = nullptr, *indices = nullptr, *eid = nullptr;
  float *ts = nullptr;
  bool owns_graph = false;
  int num_layers = 0, num_history = 1;
  std::vector<int> neigh;
  bool recent = true, prop_time = false;
  float wd = 0.f;
  uint64_t seed = 0, call_index = 0;
  int32_t *ts_ptr = nullptr;   // (num_history + 1) slots x n_nodes
  std::vector<BlockBuf> blocks;
  int32_t *dims = nullptr;     // 8 per block
  int32_t *err = nullptr;
  uint32_t *call_dev = nullptr;
  int32_t *roots_in = nullptr;
  float *rts_in = nullptr;
  int64_t cap_r0 = 0;
  int32_t *ws_cnt = nullptr;
  int2 *ws_part = nullptr;
  int32_t *ws_pick = nullptr;  // staged picks of the block being sampled
  int64_t ws_cap_roots = 0;
  int32_t *dd_keys = nullptr, *dd_minpos = nullptr, *dd_slot = nullptr, *dd_uidx = nullptr;
  int2 *dd_part = nullptr;
  int64_t dd_cap_edges = 0, dd_table = 0;
  // data-parallel shards: the global batch's blocks of every layer whose nodes
  // advance a later layer's pointers, and their workspace
  std::vector<BlockBuf> gblocks;
  int32_t *gdims = nullptr;    // 8 per global block
  int32_t *gws_cnt = nullptr, *gws_pick = nullptr;
  int2 *gws_part = nullptr;
  int64_t cap_g0 = 0;
  bool sampled = false;
};

namespace {

void free_block(BlockBuf &b) {
  int32_t *ip[] = {b.row, b.col, b.eid, b.nodes, b.rptr, b.cntE, b.uniE, b.invE, b.nbr};
  for (auto p : ip) if (p) cudaFree(p);
  if (b.ts) cudaFree(b.ts);
  if (b.dts) cudaFree(b.dts);
  if (b.dte) cudaFree(b.dte);
  b = BlockBuf();
}

int alloc_block(BlockBuf &b, int64_t cr, int64_t ce) {
  free_block(b);
  const int64_t ce1 = std::max<int64_t>(ce, 1), cn = cr + ce1;
  FB_TRY_CUDA(cudaMalloc(&b.row, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.col, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.eid, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.uniE, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.invE, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.nbr, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.dte, ce1 * 4));
  FB_TRY_CUDA(cudaMalloc(&b.nodes, cn * 4));
  FB_TRY_CUDA(cudaMalloc(&b.ts, cn * 4));
  FB_TRY_CUDA(cudaMalloc(&b.dts, cn * 4));
  FB_TRY_CUDA(cudaMalloc(&b.rptr, (cr + 1) * 4));
  FB_TRY_CUDA(cudaMalloc(&b.cntE, (cr + 1) * 4));
  b.cap_roots = cr;
  b.cap_edges = ce;
  return FB_OK;
}

// Capacity of every block for r0 layer-0 roots.
void block_caps(const fb_sampler *s, int64_t r0, std::vector<int64_t> &cr, std::vector<int64_t> &ce) {
  const int nh = s->num_history;
  cr.assign(s->num_layers * nh, 0);
  ce.assign(s->num_layers * nh, 0);
  int64_t roots = r0;
  for (int l = 0; l < s->num_layers; ++l) {
    int64_t edges = roots * (int64_t)std::max(0, s->neigh[l]);
    for (int h = 0; h < nh; ++h) { cr[l * nh + h] = roots; ce[l * nh + h] = edges; }
    roots += edges;
  }
}

int ensure_capacity(fb_sampler *s, int64_t r0) {
  if (r0 <= s->cap_r0 && !s->blocks.empty()) return FB_OK;
  FB_TRY_CUDA(cudaDeviceSynchronize());
  std::vector<int64_t> cr, ce;
  block_caps(s, r0, cr, ce);
  int64_t max_roots = 0, total = 0;
  for (size_t i = 0; i < cr.size(); ++i) {
    max_roots = std::max(max_roots, cr[i]);
    total += cr[i] + ce[i];
  }
  if (total > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "sampler: block sizes exceed int32 indexing");
  s->blocks.resize(cr.size());
  for (size_t i = 0; i < cr.size(); ++i) {
    int rc = alloc_block(s->blocks[i], cr[i], ce[i]);
    if (rc) return rc;
  }
  if (s->roots_in) cudaFree(s->roots_in);
  if (s->rts_in) cudaFree(s->rts_in);
  FB_TRY_CUDA(cudaMalloc(&s->roots_in, std::max<int64_t>(r0, 1) * 4));
  FB_TRY_CUDA(cudaMalloc(&s->rts_in, std::max<int64_t>(r0, 1) * 4));
  if (s->ws_cnt) cudaFree(s->ws_cnt);
  if (s->ws_part) cudaFree(s->ws_part);
  if (s->ws_pick) cudaFree(s->ws_pick);
  int64_t max_pick = 1;
  for (size_t i = 0; i < cr.size(); ++i)
    max_pick = std::max<int64_t>(max_pick, cr[i] * std::max(0, s->neigh[i / s->num_history]));
  FB_TRY_CUDA(cudaMalloc(&s->ws_cnt, std::max<int64_t>(max_roots, 1) * 4));
  FB_TRY_CUDA(cudaMalloc(&s->ws_part, nblk(max_roots, kRootsPerCta) * sizeof(int2)));
  FB_TRY_CUDA(cudaMalloc(&s->ws_pick, max_pick * 4));
  s->ws_cap_roots = max_roots;
  s->cap_r0 = r0;
  return FB_OK;
}

// Workspace of one block's count / scan / write passes.
struct LayerWork {
  int32_t *cnt;
  int2 *part;
  int32_t *pick;
};

int run_block(fb_sampler *s, BlockBuf &b, int32_t *dims, const LayerWork &w, int bidx, const int32_t *roots,
              const float *rts, int64_t R_host, const int32_t *R_dev, int64_t R_cap, int use_ptr, int hist_i,
              int neighs, float offset, cudaStream_t st) {
  const int nh = s->num_history;
  SampleArgs a;
  a.indptr = s->indptr; a.indices = s->indices; a.eid = s->eid; a.ts = s->ts;
  a.n_nodes = s->n_nodes;
  a.ptr_s = s->ts_ptr + (int64_t)(nh - 1 - hist_i) * s->n_nodes;
  a.ptr_e = s->ts_ptr + (int64_t)(nh - hist_i) * s->n_nodes;
  a.roots = roots; a.rts = rts; a.R_host = R_host; a.R_dev = R_dev;
  a.use_ptr = use_ptr; a.num_history = nh; a.neighs = neighs;
  a.recent = s->recent; a.prop_time = s->prop_time;
  a.wd = s->wd; a.offset = offset;
  a.key0 = (uint32_t)s->seed; a.key1 = (uint32_t)(s->seed >> 32);
  a.call_dev = s->call_dev; a.slot = (uint32_t)bidx;
  a.err = s->err;
  a.pick = w.pick;
  const int nb = nblk(R_cap, kRootsPerCta);
  FB_TRY_CUDA(fb::launch(k_sample_count, nb, kThreads, 0, st, a, w.cnt, w.part));
  FB_LAUNCHED("k_sample_count");
  FB_TRY_CUDA(fb::launch(k_scan_parts, 1, 1024, 0, st, w.part, nb, R_host, R_dev, dims, b.rptr, b.cntE));
  FB_LAUNCHED("k_scan_parts");
  FB_TRY_CUDA(fb::launch(k_sample_write, nb, kThreads, 0, st, a, w.cnt, w.part, b.row, b.col, b.eid, b.ts, b.dts,
                                          b.nodes, b.rptr, b.cntE, b.dte, b.nbr));
  FB_LAUNCHED("k_sample_write");
  return FB_OK;
}

int run_layer_slot(fb_sampler *s, int bidx, const int32_t *roots, const float *rts, int64_t R_host,
                   const int32_t *R_dev, int64_t R_cap, int use_ptr, int hist_i, int neighs, float offset,
                   cudaStream_t st) {
  const LayerWork w{s->ws_cnt, s->ws_part, s->ws_pick};
  return run_block(s, s->blocks[bidx], s->dims + 8 * bidx, w, bidx, roots, rts, R_host, R_dev, R_cap, use_ptr,
                   hist_i, neighs, offset, st);
}

// A layer after the first advances the pointers with the previous layer's
// nodes when it samples with them (sampler_core.cpp:700-706).
bool layer_uses_ptr(const fb_sampler *s, int l) {
  return l == 0 || (s->prop_time && s->num_history == 1) || s->recent;
}

// Global blocks of the layers whose nodes advance a later layer's pointers:
// layer l < L-1 when layer l+1 uses them.  g0 = global roots.
int ensure_global_capacity(fb_sampler *s, int64_t g0) {
  int nglob = 0;
  for (int l = 0; l + 1 < s->num_layers; ++l)
    if (layer_uses_ptr(s, l + 1)) nglob = l + 1;
  if (nglob == 0) return FB_OK;
  if (g0 <= s->cap_g0 && (int)s->gblocks.size() >= nglob) return FB_OK;
  FB_TRY_CUDA(cudaDeviceSynchronize());
  for (auto &b : s->gblocks) free_block(b);
  void *ps[] = {s->gdims, s->gws_cnt, s->gws_pick, s->gws_part};
  for (auto p : ps) if (p) cudaFree(p);
  s->gblocks.assign(nglob, BlockBuf());
  int64_t roots = g0, max_roots = 1, max_pick = 1;
  for (int l = 0; l < nglob; ++l) {
    const int64_t edges = roots * (int64_t)std::max(0, s->neigh[l]);
    if (roots + edges > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "sampler: global blocks exceed int32");
    int rc = alloc_block(s->gblocks[l], roots, edges);
    if (rc) return rc;
    max_roots = std::max(max_roots, roots);
    max_pick = std::max(max_pick, edges);
    roots += edges;
  }
  FB_TRY_CUDA(cudaMalloc(&s->gdims, 8 * 4 * nglob));
  FB_TRY_CUDA(cudaMemset(s->gdims, 0, 8 * 4 * nglob));
  FB_TRY_CUDA(cudaMalloc(&s->gws_cnt, max_roots * 4));
  FB_TRY_CUDA(cudaMalloc(&s->gws_part, nblk(max_roots, kRootsPerCta) * sizeof(int2)));
  FB_TRY_CUDA(cudaMalloc(&s->gws_pick, max_pick * 4));
  s->cap_g0 = g0;
  return FB_OK;
}

}  // namespace

extern "C" int fb_sampler_create(const int32_t *indptr, const int32_t *indices, const int32_t *eid,
                                 const float *ts, int64_t n_nodes, int64_t n_edges, int graph_on_device,
                                 int num_layers, const int32_t *num_neighbors, int recent, int prop_time,
                                 int num_history, float window_duration, uint64_t seed, fb_sampler **out) {
  if (!out || !indptr || (n_edges > 0 && (!indices || !eid || !ts)) || n_nodes < 0 || n_edges < 0 ||
      num_layers < 1 || num_history < 1 || !num_neighbors)
    return fb::set_error(FB_ERR_ARG, "fb_sampler_create: bad argument");
  if (n_edges >= INT32_MAX || n_nodes >= INT32_MAX)
    return fb::set_error(FB_ERR_UNSUPPORTED, "fb_sampler_create: graph exceeds int32 ids");
  auto *s = new fb_sampler();
  FB_TRY_CUDA(cudaGetDevice(&s->device));
  s->n_nodes = n_nodes; s->n_edges = n_edges;
  s->num_layers = num_layers; s->num_history = num_history;
  s->neigh.assign(num_neighbors, num_neighbors + num_layers);
  s->recent = recent != 0; s->prop_time = prop_time != 0;
  s->wd = window_duration; s->seed = seed;
  if (graph_on_device) {
    s->indptr = const_cast<int32_t *>(indptr);
    s->indices = const_cast<int32_t *>(indices);
    s->eid = const_cast<int32_t *>(eid);
    s->ts = const_cast<float *>(ts);
    s->owns_graph = false;
  } else {
    const int64_t e1 = std::max<int64_t>(n_edges, 1);
    FB_TRY_CUDA(cudaMalloc(&s->indptr, (n_nodes + 1) * 4));
    FB_TRY_CUDA(cudaMalloc(&s->indices, e1 * 4));
    FB_TRY_CUDA(cudaMalloc(&s->eid, e1 * 4));
    FB_TRY_CUDA(cudaMalloc(&s->ts, e1 * 4));
    FB_TRY_CUDA(cudaMemcpy(s->indptr, indptr, (n_nodes + 1) * 4, cudaMemcpyHostToDevice));
    if (n_edges > 0) {
      FB_TRY_CUDA(cudaMemcpy(s->indices, indices, n_edges * 4, cudaMemcpyHostToDevice));
      FB_TRY_CUDA(cudaMemcpy(s->eid, eid, n_edges * 4, cudaMemcpyHostToDevice));
      FB_TRY_CUDA(cudaMemcpy(s->ts, ts, n_edges * 4, cudaMemcpyHostToDevice));
    }
    s->owns_graph = true;
  }
  FB_TRY_CUDA(cudaMalloc(&s->ts_ptr, std::max<int64_t>(n_nodes, 1) * 4 * (num_history + 1)));
  FB_TRY_CUDA(cudaMalloc(&s->dims, 8 * 4 * num_layers * num_history));
  FB_TRY_CUDA(cudaMemset(s->dims, 0, 8 * 4 * num_layers * num_history));
  FB_TRY_CUDA(cudaMalloc(&s->err, 4));
  FB_TRY_CUDA(cudaMemset(s->err, 0, 4));
  FB_TRY_CUDA(cudaMalloc(&s->call_dev, 4));
  FB_TRY_CUDA(cudaMemset(s->call_dev, 0, 4));
  *out = s;
  return fb_sampler_reset(s, 0) == FB_OK ? (cudaDeviceSynchronize() == cudaSuccess ? FB_OK : FB_ERR_CUDA)
                                         : FB_ERR_CUDA;
}

extern "C" int fb_sampler_destroy(fb_sampler *s) {
  if (!s) return FB_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(s->device);
  cudaDeviceSynchronize();
  for (auto &b : s->blocks) free_block(b);
  for (auto &b : s->gblocks) free_block(b);
  if (s->owns_graph) {
    cudaFree(s->indptr); cudaFree(s->indices); cudaFree(s->eid); cudaFree(s->ts);
  }
  void *ps[] = {s->ts_ptr, s->dims, s->err, s->call_dev, s->roots_in, s->rts_in, s->ws_cnt, s->ws_part, s->ws_pick,
                s->dd_keys, s->dd_minpos, s->dd_slot, s->dd_uidx, s->dd_part,
                s->gdims, s->gws_cnt, s->gws_pick, s->gws_part};
  for (auto p : ps) if (p) cudaFree(p);
  cudaSetDevice(cur);
  delete s;
  return FB_OK;
}

extern "C" int fb_sampler_reset(fb_sampler *s, cudaStream_t st) {
  if (!s) return fb::set_error(FB_ERR_ARG, "fb_sampler_reset: null sampler");
  if (s->n_nodes == 0) return FB_OK;
  k_reset<<<nblk(s->n_nodes), kThreads, 0, st>>>(s->indptr, s->ts_ptr, s->n_nodes, s->num_history + 1);
  FB_LAUNCHED("k_reset");
  return FB_OK;
}

namespace {

// sample() (sampler_core.cpp:597-712) over this process's roots.  With
// g_roots (data-parallel shards), every pointer update that sample() over the
// global batch would make is made instead of the local one: layer 0 advances
// the pointers with the global roots, and a later layer with the nodes of the
// global batch's previous-layer block, sampled here alongside the local one
// (both read the same pointers).  The local roots are a subset of the global
// ones and a max is idempotent, so the pointers, and every recent-k pick of
// every layer, are those of one process sampling the global batch.
int sample_impl(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots, int roots_on_device,
                const int32_t *g_roots, const float *g_ts, int64_t n_global, cudaStream_t st) {
  int rc = ensure_capacity(s, n_roots);
  if (rc) return rc;
  const bool global = g_roots != nullptr;
  if (global) {
    rc = ensure_global_capacity(s, n_global);
    if (rc) return rc;
  }
  const int32_t *r0 = roots;
  const float *t0 = root_ts;
  if (!roots_on_device && n_roots > 0) {
    FB_TRY_CUDA(cudaMemcpyAsync(s->roots_in, roots, n_roots * 4, cudaMemcpyHostToDevice, st));
    FB_TRY_CUDA(cudaMemcpyAsync(s->rts_in, root_ts, n_roots * 4, cudaMemcpyHostToDevice, st));
    r0 = s->roots_in;
    t0 = s->rts_in;
  }
  const int nh = s->num_history;
  std::vector<int64_t> cr, ce, gcr, gce;
  block_caps(s, n_roots, cr, ce);
  if (global) block_caps(s, n_global, gcr, gce);
  const int nglob = (int)s->gblocks.size();
  for (int l = 0; l < s->num_layers; ++l) {
    const int use_ptr = layer_uses_ptr(s, l) ? 1 : 0;
    const int neighs = s->neigh[l];
    // Roots of the pointer update before the history loop (sampler_core.cpp:464-476).
    const int32_t *ur = r0;
    const float *ut = t0;
    const int32_t *uR = nullptr;
    int64_t uR_host = n_roots, ucap = cr[l * nh];
    if (!use_ptr) {
      // no pointer update in this layer (and, sharded, no global block of the layer above)
    } else if (global) {
      // a layer l > 0 that uses the pointers has the global block of layer l - 1
      ur = g_roots; ut = g_ts; uR_host = n_global; ucap = gcr[l * nh];
      if (l > 0) {
        ur = s->gblocks[l - 1].nodes; ut = s->gblocks[l - 1].ts; uR = s->gdims + 8 * (l - 1) + 3;
      }
    } else if (l > 0) {
      const int pb = (l - 1) * nh + nh - 1;
      ur = s->blocks[pb].nodes; ut = s->blocks[pb].ts; uR = s->dims + 8 * pb + 3;
    }
    const int64_t rcap = cr[l * nh];
    if (use_ptr && ucap > 0) {
      FB_TRY_CUDA(fb::launch(k_update_ptr, nblk(ucap * kGroup), kThreads, 0, st, s->indptr, s->ts, s->n_nodes,
                             s->ts_ptr + (int64_t)nh * s->n_nodes, ur, ut, uR_host, uR, 0.f, s->err));
      FB_LAUNCHED("k_update_ptr");
    }
    for (int i = 0; i < nh; ++i) {
      const int32_t *hr = r0;
      const float *ht = t0;
      const int32_t *hR = nullptr;
      if (l > 0) {
        const int pb = (l - 1) * nh + nh - 1 - i;
        hr = s->blocks[pb].nodes; ht = s->blocks[pb].ts; hR = s->dims + 8 * pb + 3;
      }
      const float offset = (float)(-i) * s->wd;
      if (use_ptr && fabsf(s->wd) > 1e-7f && rcap > 0) {
        FB_TRY_CUDA(fb::launch(k_update_ptr, nblk(rcap * kGroup), kThreads, 0, st, s->indptr, s->ts, s->n_nodes,
                                                      s->ts_ptr + (int64_t)(nh - 1 - i) * s->n_nodes, hr, ht,
                                                      n_roots, hR, offset - s->wd, s->err));
        FB_LAUNCHED("k_update_ptr");
      }
      rc = run_layer_slot(s, l * nh + nh - 1 - i, hr, ht, n_roots, hR, rcap, use_ptr, i, neighs, offset, st);
      if (rc) return rc;
    }
    if (global && l < nglob && gcr[l * nh] > 0) {
      // the global batch's block of this layer, for the next layer's pointer update
      const LayerWork w{s->gws_cnt, s->gws_part, s->gws_pick};
      const int32_t *gr = l == 0 ? g_roots : s->gblocks[l - 1].nodes;
      const float *gt = l == 0 ? g_ts : s->gblocks[l - 1].ts;
      const int32_t *gR = l == 0 ? nullptr : s->gdims + 8 * (l - 1) + 3;
      rc = run_block(s, s->gblocks[l], s->gdims + 8 * l, w, l * nh, gr, gt, n_global, gR, gcr[l * nh], use_ptr, 0,
                     neighs, 0.f, st);
      if (rc) return rc;
    }
  }
  FB_TRY_CUDA(fb::launch(k_bump_call, 1, 1, 0, st, s->call_dev));
  FB_LAUNCHED("k_bump_call");
  s->call_index++;
  s->sampled = true;
  return FB_OK;
}

}  // namespace

extern "C" int fb_sampler_sample(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                                 int roots_on_device, cudaStream_t st) {
  if (!s || n_roots < 0 || (n_roots > 0 && (!roots || !root_ts)))
    return fb::set_error(FB_ERR_ARG, "fb_sampler_sample: bad argument");
  return sample_impl(s, roots, root_ts, n_roots, roots_on_device, nullptr, nullptr, 0, st);
}

extern "C" int fb_sampler_sample_shard(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                                       const int32_t *global_roots, const float *global_ts, int64_t n_global,
                                       cudaStream_t st) {
  if (!s || n_roots < 0 || n_global < n_roots || (n_roots > 0 && (!roots || !root_ts)) ||
      (n_global > 0 && (!global_roots || !global_ts)))
    return fb::set_error(FB_ERR_ARG, "fb_sampler_sample_shard: bad argument");
  if (s->num_history != 1 || fabsf(s->wd) > 1e-7f)
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "fb_sampler_sample_shard: sharded sampling supports num_history 1 without a window");
  if (n_global == 0) return sample_impl(s, roots, root_ts, n_roots, 1, nullptr, nullptr, 0, st);
  return sample_impl(s, roots, root_ts, n_roots, 1, global_roots, global_ts, n_global, st);
}

extern "C" int fb_sampler_update_pointers(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                                          cudaStream_t st) {
  if (!s || n_roots < 0 || (n_roots > 0 && (!roots || !root_ts)))
    return fb::set_error(FB_ERR_ARG, "fb_sampler_update_pointers: bad argument");
  if (n_roots == 0) return FB_OK;
  // the first layer's pointer updates of sample(), for these roots only
  const int nh = s->num_history;
  FB_TRY_CUDA(fb::launch(k_update_ptr, nblk(n_roots * kGroup), kThreads, 0, st, s->indptr, s->ts, s->n_nodes, s->ts_ptr + (int64_t)nh * s->n_nodes,
                                                    roots, root_ts, n_roots, nullptr, 0.f, s->err));
  FB_LAUNCHED("k_update_ptr");
  for (int i = 0; i < nh; ++i) {
    const float offset = (float)(-i) * s->wd;
    if (fabsf(s->wd) > 1e-7f) {
      FB_TRY_CUDA(fb::launch(k_update_ptr, nblk(n_roots * kGroup), kThreads, 0, st, s->indptr, s->ts, s->n_nodes,
                                                        s->ts_ptr + (int64_t)(nh - 1 - i) * s->n_nodes, roots,
                                                        root_ts, n_roots, nullptr, offset - s->wd, s->err));
      FB_LAUNCHED("k_update_ptr");
    }
  }
  return FB_OK;
}

extern "C" int fb_sampler_num_blocks(const fb_sampler *s) {
  return s ? s->num_layers * s->num_history : 0;
}

extern "C" int fb_sampler_block(const fb_sampler *s, int i, fb_block_view *out) {
  if (!s || !out || i < 0 || i >= (int)s->blocks.size())
    return fb::set_error(FB_ERR_ARG, "fb_sampler_block: bad block index (sample() first)");
  const BlockBuf &b = s->blocks[i];
  out->row = b.row; out->col = b.col; out->eid = b.eid;
  out->ts = b.ts; out->dts = b.dts; out->nodes = b.nodes;
  out->rptr = b.rptr; out->cntE = b.cntE; out->uniE = b.uniE; out->invE = b.invE;
  out->dte = b.dte; out->nbr = b.nbr;
  out->dims = s->dims + 8 * i;
  out->max_roots = b.cap_roots;
  out->max_edges = b.cap_edges;
  return FB_OK;
}

extern "C" int fb_sampler_dims(fb_sampler *s, int32_t *host_dims, cudaStream_t st) {
  if (!s || !host_dims) return fb::set_error(FB_ERR_ARG, "fb_sampler_dims: bad argument");
  const int nb = s->num_layers * s->num_history;
  int32_t err = 0;
  FB_TRY_CUDA(cudaMemcpyAsync(host_dims, s->dims, 8 * 4 * nb, cudaMemcpyDeviceToHost, st));
  FB_TRY_CUDA(cudaMemcpyAsync(&err, s->err, 4, cudaMemcpyDeviceToHost, st));
  FB_TRY_CUDA(cudaStreamSynchronize(st));
  if (err & kErrRootRange) {
    cudaMemsetAsync(s->err, 0, 4, st);
    return fb::set_error(FB_ERR_ARG, "sampler: a root node id is outside [0, num_nodes)");
  }
  return FB_OK;
}

extern "C" int fb_sampler_set_call_index(fb_sampler *s, uint64_t call_index) {
  if (!s) return fb::set_error(FB_ERR_ARG, "fb_sampler_set_call_index: null sampler");
  s->call_index = call_index;
  k_set_call<<<1, 1>>>(s->call_dev, (uint32_t)call_index);
  FB_LAUNCHED("k_set_call");
  FB_TRY_CUDA(cudaDeviceSynchronize());
  return FB_OK;
}

extern "C" int fb_sampler_dedup(fb_sampler *s, int i, cudaStream_t st) {
  if (!s || i < 0 || i >= (int)s->blocks.size())
    return fb::set_error(FB_ERR_ARG, "fb_sampler_dedup: bad block index");
  BlockBuf &b = s->blocks[i];
  const int64_t ce = std::max<int64_t>(b.cap_edges, 1);
  if (ce > s->dd_cap_edges) {
    FB_TRY_CUDA(cudaStreamSynchronize(st));
    void *ps[] = {s->dd_keys, s->dd_minpos, s->dd_slot, s->dd_uidx, s->dd_part};
    for (auto p : ps) if (p) cudaFree(p);
    int64_t table = 1;
    while (table < 2 * ce) table <<= 1;
    FB_TRY_CUDA(cudaMalloc(&s->dd_keys, table * 4));
    FB_TRY_CUDA(cudaMalloc(&s->dd_minpos, table * 4));
    FB_TRY_CUDA(cudaMalloc(&s->dd_slot, ce * 4));
    FB_TRY_CUDA(cudaMalloc(&s->dd_uidx, ce * 4));
    FB_TRY_CUDA(cudaMalloc(&s->dd_part, nblk(ce) * sizeof(int2)));
    s->dd_cap_edges = ce;
    s->dd_table = table;
  }
  // The table must be at least twice the edge count of this block.
  int64_t table = 1;
  while (table < 2 * ce) table <<= 1;
  int32_t *dims = s->dims + 8 * i;
  const int nb = nblk(ce);
  k_dedup_init<<<nblk(table), kThreads, 0, st>>>(s->dd_keys, s->dd_minpos, table);
  FB_LAUNCHED("k_dedup_init");
  k_dedup_insert<<<nb, kThreads, 0, st>>>(b.eid, dims, s->dd_keys, s->dd_minpos, s->dd_slot, (uint32_t)(table - 1));
  FB_LAUNCHED("k_dedup_insert");
  k_dedup_count<<<nb, kThreads, 0, st>>>(dims, s->dd_minpos, s->dd_slot, s->dd_part);
  FB_LAUNCHED("k_dedup_count");
  k_dedup_scan<<<1, 1024, 0, st>>>(s->dd_part, nb, dims);
  FB_LAUNCHED("k_dedup_scan");
  k_dedup_emit<<<nb, kThreads, 0, st>>>(b.eid, dims, s->dd_minpos, s->dd_slot, s->dd_part, s->dd_uidx, b.uniE);
  FB_LAUNCHED("k_dedup_emit");
  k_dedup_inv<<<nb, kThreads, 0, st>>>(dims, s->dd_minpos, s->dd_slot, s->dd_uidx, b.invE);
  FB_LAUNCHED("k_dedup_inv");
  return FB_OK;
}
