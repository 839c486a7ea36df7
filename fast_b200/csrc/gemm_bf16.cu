// bf16 projection GEMMs on the tcgen05 tensor cores: kind::f16 MMAs with
// bf16 operands and fp32 accumulation in tensor memory, grouped like the
// fp32 ones of gemm_tc.cu (independent NT / NN / TN problems of one
// dependency level share one persistent launch).
//
//   NT: C[m, n] (+)= sum_k A[m, k] B[n, k] + bias[n]     A, B K-major
//   NN: C[m, n] (+)= sum_k A[m, k] B[k, n] + bias[n]     A K-major, B MN-major
//   TN: P[s][n, k] = sum_{m in split s} G[m, n] X[m, k]  G, X MN-major; a
//       ones column of X at k = K gives the bias gradient; k_bf_reduce sums
//       the splits in a fixed order into C (+ C) and db (+ db).  With column
//       segments of X (a weight gradient over a bf16 projection row whose
//       segments sit at 8-column boundaries) the tile roles swap: X's columns
//       run along the MMA's M side and G's (few) columns along N, so X
//       streams through once instead of once per 128 columns of G; the bias
//       gradient comes from a ones column on the M side, and the reduce
//       writes P transposed through the segment map, skipping the gaps.
//   NT / NN may take A as [A | A2] concatenated along K (k1 % 8 == 0).
//   Gathered operand (NT's A, or the segmented TN's X): the rows are not read
//   from one matrix but gathered per 64-column segment from up to three bf16
//   sources -- node-feature rows by node id, edge-feature rows by edge id
//   (16-byte cp.async copies from every producer lane, written in the
//   swizzled layout and counted on the stage's barrier through
//   cp.async.mbarrier.arrive), and a matrix read row by row by TMA (the time
//   encoding) -- so the
//   projection rows of a block are never written to memory.
//
// Operands are bf16 in global memory and reach the tensor cores untouched:
// TMA moves 64-element (128-byte) rows with the 128-byte swizzle, K-major
// tiles as [rows][64 k] boxes and MN-major tiles as [64 k][64 mn] boxes side
// by side, and the MMA reads them through K-major or MN-major descriptors.
// There is no conversion pass, so a slice costs one TMA write and one MMA
// read of shared memory.  A tile accumulates its whole reduction range in
// one of two TMEM accumulators (up to 256 columns each) while the epilogue
// drains the other.
//
// CTA = 12 warps:
//   warp 0      TMA producer (lane 0; every lane issues row gathers)
//   warp 1      TMEM allocator; the MMA issuer (one elected lane); for TN
//               slices it clears the rows outside the split (rows past the
//               device-side count hold stale data) and writes the ones column
//   warps 4..11 epilogue: two warps per TMEM lane quadrant, alternate
//               32-column blocks, rows staged through shared memory so each
//               store instruction writes 32 consecutive columns of one row
// Every wait is bounded: past the limit the CTA records an error, stops
// issuing work, drains what it already issued (again bounded), frees its
// tensor memory and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>
#include "runtime.cuh"
#include "tc_common.cuh"

namespace {

using namespace fbtc;

constexpr int BM = 128;                      // MMA M = TMEM lanes
constexpr int BK = 64;                       // reduction slice: 64 bf16 = one 128-byte swizzle row
constexpr int kStagesN = 4;                  // stages of the standard variant (48 KB each)
constexpr int kStagesW = 3;                  // of the wide variant (64 KB each)
constexpr int kMaxBn = 256;
constexpr int kMaxBf = 7;                    // problems per launch (parameters under 4 KB)
constexpr int kAOp = BM * BK * 2;            // 16 KB
constexpr int kBOp = kMaxBn * BK * 2;        // 32 KB
// Wide variant (launches holding a segmented TN): such a TN item covers 2 BM
// columns of X with two MMAs per K step sharing the staged G slice, so the A
// area of a stage holds four MN-major boxes.
template <bool W> __host__ __device__ constexpr int a_bytes() { return W ? 2 * kAOp : kAOp; }
template <bool W> __host__ __device__ constexpr int stages() { return W ? kStagesW : kStagesN; }
template <bool W> __host__ __device__ constexpr int stage_bytes() { return a_bytes<W>() + kBOp; }
constexpr int kBox = BK * 128;               // one MN-major box: BK rows of 64 elements
constexpr int kEpiWarps = 8;
constexpr int kStagePitch = 33;              // epilogue staging rows (floats; odd: no bank conflicts)
constexpr int kStageWarp = 32 * kStagePitch * 4;
constexpr int kBarBytes = 256;
template <bool W> __host__ __device__ constexpr int smem_bytes() {
  return 1024 + stages<W>() * stage_bytes<W>() + kBarBytes + kEpiWarps * kStageWarp;
}
static_assert(smem_bytes<false>() <= 232448 && smem_bytes<true>() <= 232448,
              "shared memory of k_bf_group exceeds 227 KB");
constexpr int kTmemCols = 512;               // two accumulators of up to 256 columns
constexpr int kAccStride = 256;
constexpr int64_t kTnRowsMin = 512;          // TN: rows per split, at least (FB_TN_ROWS_MIN overrides)
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpEpi0 = 4;

constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;

enum : int { kNT = 0, kNN = 1, kTN = 2 };

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor (128-byte swizzle), tile base 1024-byte
// aligned.  K-major: rows of 128 B (64 k), 8-row groups 1024 B apart (SBO);
// a K step of 16 advances the start by 32 B.  MN-major: [64 k][64 mn] boxes
// side by side along MN (LBO = one box), 8-row k groups 1024 B apart (SBO);
// a K step of 16 advances the start by 2 KB.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, bool mn) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(mn ? (kBox >> 4) : 1) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

struct BfProb {
  CUtensorMap ta, ta2, tb;   // A (TN: G), A2, B (TN: X); gathered A: segments 0, 1 in ta, ta2
  CUtensorMap tg;            // gathered A: segment 2
  // TN: P is [N rows][Kp cols] in the tiling's own orientation; ones = 1:
  // the ones column is B's column K, 2: it is A's column N - 1 (swapped form)
  int kind, a_mn, b_mn, k1, K, N, Kp, bn, rt, nt, ones, accumulate, db_accumulate, max_splits;
  int swap, ktot, nseg, seg_at[3], seg_len[3], seg_to[3];
  int c_bf16;                // NT / NN: C holds bf16 (round to nearest even), written, not accumulated
  int wide;                  // segmented TN in a wide launch: items of 2 BM rows (X columns)
  int rows_min;                            // TN: rows per split, at least
  int gat, g_nseg, g_end[3], g_rows[3];   // A of the tiling gathered (see fb_bf16_row_gather)
  const int32_t *g_idx[3];
  const uint16_t *g_tab[3];                 // gathered segments' sources (16-byte cp.async copies)
  int64_t g_ld[3];
  int g_cols[3];
  const float *add;                         // NT / NN: + add[add_idx[m] * ld_add + n] in the epilogue
  const int32_t *add_idx;
  int64_t ld_add;
  int add_rows;
  uint32_t idesc;
  int64_t M;
  const int32_t *M_dev;
  const float *bias;
  float *C;
  int64_t ldc;
  float *db, *P;
};

struct BfArgs {
  BfProb p[kMaxBf];
  int n;
  int gat_any;                              // a problem has a gathered operand (cp.async row copies)
  int red_start[kMaxBf + 1];
  int32_t *err;
};
// Large kernel parameters (CUDA 12.1+, up to 32,764 bytes on sm_70 and later).
static_assert(sizeof(BfArgs) <= 32764, "kernel parameters of k_bf_group exceed 32 KB");

// Segment of a gathered operand holding column c (g_nseg when past the last).
__device__ __forceinline__ int gseg(const BfProb &q, int c) {
  int s = 0;
  while (s < q.g_nseg && c >= q.g_end[s]) ++s;
  return s;
}
__device__ __forceinline__ int gstart(const BfProb &q, int s) { return s ? q.g_end[s - 1] : 0; }
__device__ __forceinline__ const CUtensorMap *gmap(const BfProb &q, int s) {
  return s == 0 ? &q.ta : (s == 1 ? &q.ta2 : &q.tg);
}
// Source row of operand row r in gathered segment s (rows past `valid`, and
// indices outside the table, read row 0 / are clamped: those rows never
// reach an output).
__device__ __forceinline__ int grow(const BfProb &q, int s, int64_t r, int64_t valid) {
  if (r >= valid) return 0;
  const int v = __ldg(q.g_idx[s] + r);
  return min(max(v, 0), q.g_rows[s] - 1);
}

struct Item {
  int p, z, nk, nk1, c0;
  int64_t r0, s0, s1;
};

__device__ __forceinline__ Item decode(const BfArgs &a, const int *st, const long long *sm, const long long *sper,
                                       int i) {
  Item it;
  int p = 0;
  while (p + 1 < a.n && i >= st[p + 1]) ++p;
  const BfProb &q = a.p[p];
  int l = i - st[p];
  it.p = p;
  if (q.kind == kTN) {
    const int per_z = q.rt * q.nt;
    it.z = l / per_z;
    l -= it.z * per_z;
    it.r0 = (int64_t)(l / q.nt) * (q.wide ? 2 * BM : BM);
    it.c0 = (l % q.nt) * q.bn;
    it.s0 = (int64_t)it.z * sper[p];
    it.s1 = min((int64_t)sm[p], it.s0 + (int64_t)sper[p]);
    it.nk1 = 0;
    it.nk = it.s1 > it.s0 ? (int)((it.s1 - it.s0 + BK - 1) / BK) : 1;   // an empty split writes zeros
  } else {
    it.z = 0;
    it.r0 = (int64_t)(l / q.nt) * BM;
    it.c0 = (l % q.nt) * q.bn;
    it.s0 = it.s1 = 0;
    it.nk1 = (q.k1 + BK - 1) / BK;
    it.nk = it.nk1 + (q.K - q.k1 + BK - 1) / BK;
  }
  return it;
}

// TN slice fix-up by the MMA warp: rows >= valid of every MN-major box (A's
// two, B's nbox) are cleared -- they lie past the split or past the
// device-side row count, where memory may hold anything -- and column
// `onescol` of B (or `onescol_a` of A) is set to 1 for the rows that count.
// In a 128-byte swizzled row, 16-byte chunk c sits at position c ^ (row & 7).
__device__ __forceinline__ void set_ones(uint8_t *box0, int col, int valid, int lane) {
  uint8_t *base = box0 + (col >> 6) * kBox;
  const int c = col & 63;
  for (int r = lane; r < valid; r += 32)
    *reinterpret_cast<uint16_t *>(base + r * 128 + (((c >> 3) ^ (r & 7)) << 4) + (c & 7) * 2) = 0x3F80u;
}

__device__ __forceinline__ void fix_tn_slice(uint8_t *a, uint8_t *b, int nbox, int valid, int onescol, int onescol_a,
                                             int lane, int clear_a = 0, int na = 2) {
  // A boxes that nothing loaded (past a gathered operand's last segment): zeros
  for (int bx = 0; bx < 2; ++bx)
    if (clear_a & (1 << bx))
      for (int t = lane; t < kBox / 16; t += 32) reinterpret_cast<uint4 *>(a + bx * kBox)[t] = make_uint4(0u, 0u, 0u, 0u);
  if (valid < BK) {
    const int per_box = (BK - valid) * 8;    // 16-byte words to clear per box
    for (int t = lane; t < (na + nbox) * per_box; t += 32) {
      const int bx = t / per_box, e = t - bx * per_box;
      uint8_t *base = bx < na ? a + bx * kBox : b + (bx - na) * kBox;
      reinterpret_cast<uint4 *>(base + valid * 128)[e] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if (onescol >= 0) set_ones(b, onescol, valid, lane);
  if (onescol_a >= 0) set_ones(a, onescol_a, valid, lane);
}

// 64 columns (128 bytes) from column `col` of 32 U gathered rows into a
// 128-byte-swizzled box (16-byte chunk c of box row r at r * 128 + ((c ^ (r &
// 7)) << 4)), by cp.async: lane l copies box rows l + 32 u, source row
// idx[u]; columns at or past `cols` are zero-filled.
template <int U>
__device__ __forceinline__ void gather_box(uint8_t *box, const uint16_t *tab, int64_t ld, int col, int cols,
                                           const int (&idx)[U], int lane) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int r = lane + 32 * u;
    const uint16_t *src = tab + (int64_t)idx[u] * ld + col;
    uint8_t *dst = box + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int nb = min(max(2 * (cols - col - 8 * c), 0), 16);
      cp_async16(dst + ((c ^ (r & 7)) << 4), nb ? src + 8 * c : tab, (uint32_t)nb);
    }
  }
}

template <bool W>
__global__ void __launch_bounds__(kThreads, 1) k_bf_group(const __grid_constant__ BfArgs a) {
  constexpr int kStages = stages<W>(), kStage = stage_bytes<W>(), kAOpS = a_bytes<W>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  auto sA = [&](int s) { return smem + s * kStage; };
  auto sB = [&](int s) { return smem + s * kStage + kAOpS; };
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * kStage);
  uint64_t *full = bars, *empty = bars + kStages;
  uint64_t *accf = bars + 2 * kStages, *acce = bars + 2 * kStages + 2, *drain = bars + 2 * kStages + 4;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * kStages + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int32_t *err = a.err;
  __shared__ int s_start[kMaxBf + 1];
  __shared__ long long s_m[kMaxBf], s_per[kMaxBf];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // with gathered rows every producer lane arrives (after its copies), else lane 0
      mbar_init(full + s, a.gat_any ? 32 : 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, kEpiWarps * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kWarpProducer && lane < a.n) {
    const BfProb &q = a.p[lane];
    prefetch_map(&q.ta);
    if (q.kind != kTN && q.k1 < q.K) prefetch_map(&q.ta2);
    prefetch_map(&q.tb);
  }
  if (warp == kWarpMma) tmem_alloc(tmem_holder, kTmemCols);

  fb::pdl_enter();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int p = 0; p < a.n; ++p) {
      const BfProb &q = a.p[p];
      int64_t M = q.M_dev ? min((int64_t)(*q.M_dev), q.M) : q.M;
      M = max(M, (int64_t)0);
      s_m[p] = M;
      s_start[p] = acc;
      if (q.kind == kTN) {
        const int ns = fb::tn_parts(M, q.rows_min, q.max_splits);
        s_per[p] = ((M + ns - 1) / ns + BK - 1) / BK * BK;
        acc += q.rt * q.nt * ns;
      } else {
        s_per[p] = 0;
        acc += (int)((M + BM - 1) / BM) * q.nt;
      }
    }
    s_start[a.n] = acc;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int total = s_start[a.n];
  if ((int)blockIdx.x >= total) {
    if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
    return;
  }

  if (warp == kWarpProducer) {
    // every lane waits for a stage to be free, issues its gathered-row copies
    // (if any) and arrives; lane 0 arms the barrier with the byte count of the
    // tiled (TMA) copies and issues them
    uint32_t g = 0;
    bool stop = false;
    for (int i = blockIdx.x; i < total && !stop; i += gridDim.x) {
      const Item it = decode(a, s_start, s_m, s_per, i);
      const BfProb &q = a.p[it.p];
      const bool tn = q.kind == kTN, bmn = q.b_mn != 0, gat = q.gat != 0;
      const int bn = q.bn, k1 = q.k1, c0 = it.c0;
      const int r0 = (int)it.r0;
      // Gathered rows are copied by every lane with cp.async (gather_box): the
      // source row of tile row lane + 32 u sits in this lane's register u.  NT:
      // ix[segment][u] for the item's 128 rows.  TN: the two X boxes' 64 rows
      // of a slice, in two register sets used by alternate slices, so a set's
      // index loads are issued two slices ahead of the copies that use them.
      int ix[3][4];
      if (gat && !tn) {
#pragma unroll
        for (int sg = 0; sg < 3; ++sg)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            ix[sg][u] = (sg < q.g_nseg && q.g_idx[sg]) ? grow(q, sg, (int64_t)r0 + lane + 32 * u, s_m[it.p]) : 0;
      }
      int gsg[2] = {0, 0};
      bool gidx[2] = {false, false};
      int nxa[2][2] = {{0, 0}, {0, 0}}, nxb[2][2] = {{0, 0}, {0, 0}};
      auto load_nx = [&](int jj, int (&o)[2][2]) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int u = 0; u < 2; ++u)
            o[t][u] = (gidx[t] && jj < it.nk) ? grow(q, gsg[t], it.s0 + (int64_t)BK * jj + lane + 32 * u, it.s1) : 0;
      };
      if (gat && tn) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          gsg[t] = gseg(q, r0 + 64 * t);
          gidx[t] = gsg[t] < q.g_nseg && q.g_idx[gsg[t]] != nullptr;
        }
        load_nx(0, nxa);
        load_nx(1, nxb);
      }
      const bool wide = q.wide != 0;
      // bytes the TMA copies of a stage bring (gathered boxes arrive through cp.async)
      uint32_t bytes = (uint32_t)((wide ? 2 * kAOp : kAOp) + bn * BK * 2);
      if (gat && tn) {
        for (int t = 0; t < 2; ++t)
          if (gsg[t] >= q.g_nseg || gidx[t]) bytes -= kBox;  // cleared (past the last segment) or gathered
      }
      // slice j of the item into the next stage; false: the pipeline stopped
      auto slice = [&](int j, const int (&nx)[2][2]) -> bool {
        const int s = g % kStages;
        int ok = 1;
        if (lane == 0 && g >= kStages && !mbar_wait(empty + s, ((g / kStages) - 1) & 1, abort_flag, err)) ok = 0;
        if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
        __syncwarp();                                        // the stage is free for every lane's copies
        const int kb = j < it.nk1 ? BK * j : k1 + BK * (j - it.nk1);
        const int my = (int)it.s0 + BK * j;
        bool tiled_a = true;                                 // lane 0 issues A by TMA
        if (gat && !tn) {
          const int sg = gseg(q, kb);                        // kb < K: a segment
          if (q.g_idx[sg]) {
            tiled_a = false;
            int cur[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) cur[u] = sg == 0 ? ix[0][u] : (sg == 1 ? ix[1][u] : ix[2][u]);
            gather_box<4>(sA(s), q.g_tab[sg], q.g_ld[sg], kb - gstart(q, sg), q.g_cols[sg], cur, lane);
            cp_async_arrive(full + s);
          }
        } else if (gat) {
          bool any = false;
#pragma unroll
          for (int t = 0; t < 2; ++t)
            if (gidx[t]) {
              any = true;
              gather_box<2>(sA(s) + t * kBox, q.g_tab[gsg[t]], q.g_ld[gsg[t]], r0 + 64 * t - gstart(q, gsg[t]),
                            q.g_cols[gsg[t]], nx[t], lane);
            }
          if (any) cp_async_arrive(full + s);
        }
        // with gathered rows in the launch every lane arrives on the stage's
        // barrier (lane 0 with the TMA byte count), each after its cp.async
        // arrival: the phase completes when the tiled copies and every lane's
        // gathered copies have landed
        if (a.gat_any && lane != 0) mbar_arrive(full + s);
        if (lane == 0) {
          mbar_expect_tx(full + s, tiled_a ? bytes : bytes - kAOp);
          if (gat && tn) {
            for (int t = 0; t < 2; ++t)
              if (gsg[t] < q.g_nseg && !gidx[t])
                tma_load_2d(sA(s) + t * kBox, gmap(q, gsg[t]), full + s, r0 + 64 * t - gstart(q, gsg[t]), my);
          } else if (gat) {
            if (tiled_a) {
              const int sg = gseg(q, kb);
              tma_load_2d(sA(s), gmap(q, sg), full + s, kb - gstart(q, sg), r0);
            }
          } else if (tn) {
            for (int t = 0; t < (wide ? 4 : 2); ++t) tma_load_2d(sA(s) + t * kBox, &q.ta, full + s, r0 + 64 * t, my);
          } else if (j < it.nk1) {
            tma_load_2d(sA(s), &q.ta, full + s, BK * j, r0);
          } else {
            tma_load_2d(sA(s), &q.ta2, full + s, BK * (j - it.nk1), r0);
          }
          if (!bmn) {
            tma_load_2d(sB(s), &q.tb, full + s, kb, c0);
          } else {
            const int y = tn ? my : kb;
            for (int t = 0; t < bn / 64; ++t) tma_load_2d(sB(s) + t * kBox, &q.tb, full + s, c0 + 64 * t, y);
          }
        }
        __syncwarp();
        ++g;
        return true;
      };
      if (!(gat && tn)) {
        for (int j = 0; j < it.nk; ++j)
          if (!slice(j, nxa)) {
            stop = true;
            break;
          }
      } else {
        for (int j = 0; j < it.nk; j += 2) {
          if (!slice(j, nxa)) {
            stop = true;
            break;
          }
          load_nx(j + 2, nxa);
          if (j + 1 < it.nk) {
            if (!slice(j + 1, nxb)) {
              stop = true;
              break;
            }
            load_nx(j + 3, nxb);
          }
        }
      }
    }
    if (lane == 0 && *abort_flag) {
      // let the copies already issued land before the CTA's memory goes away
      for (uint32_t h = g > (uint32_t)kStages ? g - kStages : 0; h < g; ++h) mbar_drain(full + h % kStages, (h / kStages) & 1);
    }
  } else if (warp == kWarpMma) {
    uint32_t g = 0, used[2] = {0u, 0u};
    int nxt = 0;
    bool stop = false;
    for (int i = blockIdx.x; i < total && !stop; i += gridDim.x) {
      const Item it = decode(a, s_start, s_m, s_per, i);
      const BfProb &q = a.p[it.p];
      const bool tn = q.kind == kTN, amn = q.a_mn != 0, bmn = q.b_mn != 0;
      const bool wide = q.wide != 0;
      const uint32_t idesc = q.idesc;
      const int nbox = q.bn / 64;
      const int onescol = (tn && q.ones == 1 && q.K >= it.c0 && q.K < it.c0 + q.bn) ? q.K - it.c0 : -1;
      const int64_t ones_row = (int64_t)q.ktot - it.r0;      // swapped form: A's ones column in this tile
      const int onescol_a = (tn && q.ones == 2 && ones_row >= 0 && ones_row < (wide ? 2 * BM : BM)) ? (int)ones_row
                                                                                                   : -1;
      int clear_a = 0;                                        // gathered X: boxes past the last segment
      if (tn && q.gat)
        for (int t = 0; t < 2; ++t)
          if (gseg(q, (int)it.r0 + 64 * t) >= q.g_nseg) clear_a |= 1 << t;
      const uint64_t adv_a = amn ? (2048 >> 4) : 2, adv_b = bmn ? (2048 >> 4) : 2;   // one K step of 16
      // accumulators of this item: the next one in turn, or both (wide)
      const int b = wide ? 0 : nxt;
      if (!wide) nxt ^= 1;
      bool free_ok = true;
      for (int bb = b; bb <= (wide ? 1 : b); ++bb)
        if (used[bb] >= 1 && !mbar_wait(acce + bb, (used[bb] - 1) & 1, abort_flag, err)) free_ok = false;
      if (!free_ok) break;
      const uint32_t d = tmem + (uint32_t)(b * kAccStride);
      for (int j = 0; j < it.nk; ++j) {
        const int s = g % kStages;
        if (!mbar_wait(full + s, (g / kStages) & 1, abort_flag, err)) {
          stop = true;
          break;
        }
        if (tn) {
          const int64_t left = it.s1 - (it.s0 + (int64_t)BK * j);
          const int valid = left <= 0 ? 0 : (left >= BK ? BK : (int)left);
          if (valid < BK || onescol >= 0 || onescol_a >= 0 || clear_a) {
            fix_tn_slice(sA(s), sB(s), nbox, valid, onescol, onescol_a, lane, clear_a, wide ? 4 : 2);
            fence_async_smem();
          }
          __syncwarp();
        }
        if (lane == 0) {
          tc_fence_after();
          const uint64_t ad = sdesc(smem_u32(sA(s)), amn), bd = sdesc(smem_u32(sB(s)), bmn);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(d, ad + kk * adv_a, bd + kk * adv_b, idesc, (j | kk) != 0 ? 1u : 0u);
          if (wide) {
            // X columns BM .. 2 BM of the item: the other accumulator, the same G slice
            const uint64_t ad1 = sdesc(smem_u32(sA(s) + 2 * kBox), amn);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_bf16(d + kAccStride, ad1 + kk * adv_a, bd + kk * adv_b, idesc, (j | kk) != 0 ? 1u : 0u);
          }
          umma_commit(empty + s);
          if (j == it.nk - 1) {
            umma_commit(accf + b);
            if (wide) umma_commit(accf + 1);
          }
        }
        __syncwarp();
        ++g;
      }
      if (!stop) {
        ++used[b];
        if (wide) ++used[1];
      }
    }
    if (lane == 0) {
      // every MMA this warp issued must be complete before TMEM is freed
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
    __syncwarp();
  } else if (warp >= kWarpEpi0) {
    const int e = warp - kWarpEpi0;
    const int qd = warp & 3;                 // TMEM lane quadrant this warp may read
    const int half = e >> 2;
    const uint32_t tlane = (uint32_t)(qd * 32) << 16;
    float *stg = reinterpret_cast<float *>(smem + kStages * kStage + kBarBytes + e * kStageWarp);
    uint32_t used[2] = {0u, 0u};
    int nxt = 0;
    bool quit = false;
    for (int i = blockIdx.x; i < total && !quit; i += gridDim.x) {
      const Item it = decode(a, s_start, s_m, s_per, i);
      const BfProb &q = a.p[it.p];
      const bool wide = q.wide != 0;
      const int b0 = wide ? 0 : nxt;
      if (!wide) nxt ^= 1;
     for (int b = b0; b <= (wide ? 1 : b0); ++b) {
      if (!__all_sync(0xffffffffu, mbar_wait(accf + b, used[b] & 1, abort_flag, err) ? 1 : 0)) {
        quit = true;
        break;
      }
      tc_fence_after();
      const uint32_t t = tmem + tlane + (uint32_t)(b * kAccStride);
      // the problem's fields in registers (read through the parameter
      // pointer they would be reloaded after every store)
      const int bn = q.bn;
      const bool tn = q.kind == kTN;
      const int64_t rows = tn ? (int64_t)q.N : (int64_t)s_m[it.p];
      const int ncols = tn ? q.Kp : q.N;
      const int64_t ld = tn ? (int64_t)q.Kp : q.ldc;
      float *const out = tn ? q.P + (int64_t)it.z * q.N * q.Kp : q.C;
      const float *const bias = tn ? nullptr : q.bias;
      const bool accum = !tn && q.accumulate;
      const bool c16 = q.c_bf16 != 0;
      const float *const add = tn ? nullptr : q.add;
      const int32_t *const add_idx = q.add_idx;
      const int64_t ld_add = q.ld_add;
      const int add_rows = q.add_rows;
      const int64_t row0 = it.r0 + (wide ? (int64_t)b * BM : 0) + qd * 32;
      const int nrows = rows - row0 < 32 ? (int)max(rows - row0, (int64_t)0) : 32;
      // add table: lane r adds the (clamped) table row of output row row0 + r
      const int add_row = (add && lane < nrows) ? min(max(__ldg(add_idx + row0 + lane), 0), add_rows - 1) : 0;
#pragma unroll 1
      for (int c0 = 32 * half; c0 < bn; c0 += 64) {
        uint32_t r[32];
        tmem_ld32(t + c0, r);
        if (add && lane < nrows) {
          // + this lane's row of the add table (the lane holds one output row's
          // 32 columns here), read as 16-byte words
          const int cb = it.c0 + c0;
          const float *src = add + (int64_t)add_row * ld_add + cb;
          if (cb + 32 <= ncols) {
#pragma unroll
            for (int k4 = 0; k4 < 8; ++k4) {
              const float4 v = __ldg(reinterpret_cast<const float4 *>(src) + k4);
              r[4 * k4 + 0] = __float_as_uint(__uint_as_float(r[4 * k4 + 0]) + v.x);
              r[4 * k4 + 1] = __float_as_uint(__uint_as_float(r[4 * k4 + 1]) + v.y);
              r[4 * k4 + 2] = __float_as_uint(__uint_as_float(r[4 * k4 + 2]) + v.z);
              r[4 * k4 + 3] = __float_as_uint(__uint_as_float(r[4 * k4 + 3]) + v.w);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (cb + k < ncols) r[k] = __float_as_uint(__uint_as_float(r[k]) + __ldg(src + k));
          }
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 32; ++k) stg[lane * kStagePitch + k] = __uint_as_float(r[k]);
        __syncwarp();
        const int col = it.c0 + c0 + lane;
        if (c16 && c0 + lane < bn && col < ncols) {
          const float bv = bias ? bias[col] : 0.f;
          uint16_t *o = reinterpret_cast<uint16_t *>(out) + row0 * ld + col;
          const float *sv = stg + lane;
#pragma unroll 8
          for (int rr = 0; rr < nrows; ++rr) {
            const __nv_bfloat16 hv = __float2bfloat16_rn(sv[rr * kStagePitch] + bv);
            o[rr * ld] = *reinterpret_cast<const uint16_t *>(&hv);
          }
        } else if (c0 + lane < bn && col < ncols) {
          const float bv = bias ? bias[col] : 0.f;
          float *o = out + row0 * ld + col;
          const float *sv = stg + lane;
          if (nrows == 32) {
            if (accum) {
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr) o[rr * ld] += sv[rr * kStagePitch] + bv;
            } else {
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr) o[rr * ld] = sv[rr * kStagePitch] + bv;
            }
          } else {
            for (int rr = 0; rr < nrows; ++rr) {
              const float v = sv[rr * kStagePitch] + bv;
              o[rr * ld] = accum ? o[rr * ld] + v : v;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acce + b);
      ++used[b];
     }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
}

// Sums the TN partials of every TN problem of the launch (fixed split order)
// into C (+ C) and, for the ones column, db (+ db).
__global__ void k_bf_reduce(const __grid_constant__ BfArgs a) {
  fb::pdl_enter();
  int p = -1;
  for (int i = 0; i < a.n; ++i)
    if (a.p[i].kind == kTN && (int)blockIdx.x >= a.red_start[i] && (int)blockIdx.x < a.red_start[i + 1]) p = i;
  if (p < 0) return;
  const BfProb &q = a.p[p];
  const int64_t i = (int64_t)(blockIdx.x - a.red_start[p]) * blockDim.x + threadIdx.x;
  if (i >= (int64_t)q.N * q.Kp) return;
  int64_t M = q.M_dev ? min((int64_t)(*q.M_dev), q.M) : q.M;
  M = max(M, (int64_t)0);
  const int ns = fb::tn_parts(M, q.rows_min, q.max_splits);
  const int n = (int)(i / q.Kp), k = (int)(i % q.Kp);
  const int64_t stride = (int64_t)q.N * q.Kp;
  const float *part = q.P + i;
  float s = 0.f;
  int z = 0;
  for (; z + 8 <= ns; z += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = part[(int64_t)(z + u) * stride];
#pragma unroll
    for (int u = 0; u < 8; ++u) s += v[u];
  }
  for (; z < ns; ++z) s += part[(int64_t)z * stride];
  if (q.swap) {
    // P row n = column n of X, P column k = column k of G: C[k, map(n)], db[k]
    float *c;
    int acc;
    if (q.ones == 2 && n == q.ktot) {
      c = q.db + k;
      acc = q.db_accumulate;
    } else {
      int col = -1;
      for (int g = 0; g < q.nseg; ++g)
        if (n >= q.seg_at[g] && n < q.seg_at[g] + q.seg_len[g]) col = q.seg_to[g] + (n - q.seg_at[g]);
      if (col < 0) return;                   // a gap between segments
      c = q.C + (int64_t)k * q.ldc + col;
      acc = q.accumulate;
    }
    *c = acc ? (*c + s) : s;
    return;
  }
  float *c = (k < q.K) ? q.C + (int64_t)n * q.ldc + k : q.db + n;
  const int acc = (k < q.K) ? q.accumulate : q.db_accumulate;
  *c = acc ? (*c + s) : s;
}

// Row-major bf16 [rows, cols] with leading dimension ld (elements), boxes of
// 64 columns x box_rows rows, 128-byte swizzle; reads past the extents
// return zeros.
int make_map(CUtensorMap *m, const uint16_t *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fb::set_error(FB_ERR_CUDA, "gemm_bf16: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fb::set_error(FB_ERR_ARG, "gemm_bf16: tensor map rejected (alignment or stride)");
  return FB_OK;
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tile width along the MMA N dimension.  K-major B: a multiple of 16 up to
// 256, as even as the tiles allow.  MN-major B: whole 64-column boxes, the
// width that wastes the fewest columns counting a per-tile cost.
int bn_kmajor(int N) {
  const int t = (N + kMaxBn - 1) / kMaxBn, w = (N + t - 1) / t;
  return (w + 15) / 16 * 16;
}
int bn_mnmajor(int N) {
  int best = 256, cost = (N + 255) / 256 * (256 + 32);
  for (int w : {192, 128, 64}) {
    const int c = (N + w - 1) / w * (w + 32);
    if (c < cost) cost = c, best = w;
  }
  return best;
}

uint32_t idesc_bf16(int bn, int a_mn, int b_mn) {
  // D fp32, A and B bf16, dense; N >> 3 at bit 17, M >> 4 at bit 24
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// TN tiling: rows x cols of P (the swapped form when X comes in segments).
// Segmented TN with a bias gradient: the X column that carries the ones (its
// row of P is the bias gradient) -- the first column outside every segment
// (a gap between or after the segments, overwritten in shared memory), or K,
// one row past the operand, when the segments leave no gap.
int tn_ones_row(const fb_gemm_bf16_problem &p) {
  for (int c = 0; c < p.K; ++c) {
    bool in = false;
    for (int g = 0; g < p.nseg && !in; ++g) in = c >= p.seg_at[g] && c < p.seg_at[g] + p.seg_len[g];
    if (!in) return c;
  }
  return p.K;
}

void tn_dims(const fb_gemm_bf16_problem &p, int &rows, int &cols) {
  if (p.nseg > 0) {
    rows = p.db ? std::max(p.K, tn_ones_row(p) + 1) : p.K;
    cols = p.N;
  } else {
    rows = p.N;
    cols = p.K + (p.db ? 1 : 0);
  }
}

// Segmented TN problems on materialised rows run wide (items of 2 BM rows).
bool tn_wide(const fb_gemm_bf16_problem &p) {
  static const bool off = getenv("FB_TN_NARROW") != nullptr;
  return !off && p.kind == FB_GEMM_TN && p.nseg > 0 && !p.gather;
}

int tn_rows_min() {
  static const int v = [] {
    const char *e = getenv("FB_TN_ROWS_MIN");
    const int x = e ? atoi(e) : 0;
    return x >= 64 ? x : (int)kTnRowsMin;
  }();
  return v;
}

int tn_split_waves() {
  static const int v = [] {
    const char *e = getenv("FB_TN_SPLIT_WAVES");
    const int x = e ? atoi(e) : 0;
    return x >= 1 && x <= 8 ? x : 1;
  }();
  return v;
}

int tn_splits_max(const fb_gemm_bf16_problem &p) {
  int rows, cols;
  tn_dims(p, rows, cols);
  const int tr = tn_wide(p) ? 2 * BM : BM;
  const int tiles = ((rows + tr - 1) / tr) * ((cols + bn_mnmajor(cols) - 1) / bn_mnmajor(cols));
  return std::max(1, tn_split_waves() * num_sms() / std::max(tiles, 1));
}

int64_t slices_per_item(const fb_gemm_bf16_problem &p) {
  if (p.kind == FB_GEMM_TN) {
    const int ns = fb::tn_parts(p.M, tn_rows_min(), tn_splits_max(p));
    return ((p.M + ns - 1) / ns + BK - 1) / BK;
  }
  const int k1 = (p.A2 && p.k1 < p.K) ? p.k1 : p.K;
  return (k1 + BK - 1) / BK + (p.K - k1 + BK - 1) / BK;
}

// A gathered operand: 1..3 segments on 64-column boundaries, 16-byte aligned
// sources with leading dimensions that are multiples of 8, K = the last end.
bool gather_ok(const fb_bf16_row_gather &g, int K) {
  if (g.nseg < 1 || g.nseg > 3) return false;
  int prev = 0;
  for (int s = 0; s < g.nseg; ++s) {
    if (g.end[s] <= prev || g.end[s] % BK) return false;
    if (!g.tab[s] || !al16(g.tab[s]) || g.tab_ld[s] % 8 || g.tab_cols[s] < 1 || g.tab_ld[s] < g.tab_cols[s] ||
        g.tab_rows[s] < 1 || g.tab_rows[s] > INT32_MAX)
      return false;
    prev = g.end[s];
  }
  return prev == K;
}

bool problem_ok(const fb_gemm_bf16_problem &p) {
  if (p.kind < FB_GEMM_NT || p.kind > FB_GEMM_TN) return false;
  if (p.M < 0 || p.M > (int64_t)1 << 30 || p.N < 1 || p.K < 1) return false;
  if (p.add && (p.kind == FB_GEMM_TN || !p.add_idx || p.ld_add < p.N || p.ld_add % 4 || !al16(p.add) ||
                p.add_rows < 1 || p.add_rows > INT32_MAX))
    return false;
  if (p.gather) {
    if (!gather_ok(*p.gather, p.K)) return false;
    if (p.kind == FB_GEMM_NT) {
      if (p.A2 || !p.B || !al16(p.B) || p.ldb % 8 || p.ldb < p.K || !p.C || p.ldc < p.N) return false;
      return !(p.c_bf16 && p.accumulate);
    }
    if (p.kind != FB_GEMM_TN || p.nseg < 1 || p.nseg > 3 || !p.A || !al16(p.A) || p.lda % 8 || p.lda < p.N ||
        !p.C || p.c_bf16)
      return false;
    int end = 0;
    for (int g = 0; g < p.nseg; ++g) {
      if (p.seg_len[g] < 1 || p.seg_at[g] < end || p.seg_to[g] < 0 || p.seg_to[g] + p.seg_len[g] > p.ldc) return false;
      end = p.seg_at[g] + p.seg_len[g];
    }
    return end <= p.K;
  }
  if (!p.A || !al16(p.A) || p.lda % 8 || !p.B || !al16(p.B) || p.ldb % 8) return false;
  if (p.kind == FB_GEMM_TN) {
    if (p.c_bf16 || p.nseg < 0 || p.nseg > 3 || p.lda < p.N || p.ldb < p.K || !p.C) return false;
    if (p.nseg == 0) return p.ldc >= p.K;
    int end = 0;
    for (int g = 0; g < p.nseg; ++g) {
      if (p.seg_len[g] < 1 || p.seg_at[g] < end || p.seg_to[g] < 0 || p.seg_to[g] + p.seg_len[g] > p.ldc) return false;
      end = p.seg_at[g] + p.seg_len[g];
    }
    return end <= p.K;
  }
  if (!p.C || p.ldc < p.N || p.ldb < (p.kind == FB_GEMM_NT ? p.K : p.N)) return false;
  if (p.c_bf16 && p.accumulate) return false;
  if (p.A2 && p.k1 < p.K) {
    const int ka = p.ka > 0 ? p.ka : p.k1;
    return p.k1 >= 8 && p.k1 % 8 == 0 && ka <= p.k1 && p.lda >= ka && al16(p.A2) && p.lda2 % 8 == 0 &&
           p.lda2 >= p.K - p.k1;
  }
  return p.lda >= p.K;
}

int64_t ws_floats(const fb_gemm_bf16_problem &p) {
  if (p.kind != FB_GEMM_TN || p.M < 1) return 0;
  int rows, cols;
  tn_dims(p, rows, cols);
  const int64_t ns = fb::tn_parts(p.M, tn_rows_min(), tn_splits_max(p));
  return (ns * (int64_t)rows * cols + 63) / 64 * 64;
}

// A gathered operand: tensor maps with `box_rows`-row boxes for the segments
// read row by row; the segments read by row index are copied with cp.async
// from their source pointers.
int gather_maps(BfProb &q, const fb_bf16_row_gather &g, int box_rows) {
  q.gat = 1;
  q.g_nseg = g.nseg;
  CUtensorMap *maps[3] = {&q.ta, &q.ta2, &q.tg};
  for (int s = 0; s < g.nseg; ++s) {
    q.g_end[s] = g.end[s];
    q.g_rows[s] = (int)g.tab_rows[s];
    q.g_idx[s] = g.idx[s];
    q.g_tab[s] = static_cast<const uint16_t *>(g.tab[s]);
    q.g_ld[s] = g.tab_ld[s];
    q.g_cols[s] = (int)g.tab_cols[s];
    if (g.idx[s]) continue;
    const int rc = make_map(maps[s], g.tab[s], g.tab_rows[s], g.tab_cols[s], g.tab_ld[s], box_rows);
    if (rc) return rc;
  }
  return FB_OK;
}

int build_prob(BfProb &q, const fb_gemm_bf16_problem &p, float *ws) {
  std::memset(&q, 0, sizeof(q));
  q.kind = p.kind;
  q.rows_min = tn_rows_min();
  q.add = p.add;
  q.add_idx = p.add_idx;
  q.ld_add = p.ld_add;
  q.add_rows = (int)p.add_rows;
  q.M = p.M;
  q.M_dev = p.M_dev;
  q.N = p.N;
  q.K = p.K;
  q.accumulate = p.accumulate;
  q.C = p.C;
  q.ldc = p.ldc;
  int rc;
  if (p.kind == FB_GEMM_TN && p.nseg > 0) {
    // swapped form: the tile's rows are X's columns (+ the ones row), its
    // columns are G's; A of the tiling is X, B is G
    q.swap = 1;
    q.a_mn = q.b_mn = 1;
    q.ktot = p.db ? tn_ones_row(p) : p.K;
    q.ones = p.db ? 2 : 0;
    q.N = std::max(p.K, q.ktot + (p.db ? 1 : 0));
    q.K = p.N;
    q.Kp = p.N;
    q.bn = bn_mnmajor(q.Kp);
    q.wide = tn_wide(p) ? 1 : 0;
    q.rt = (q.N + (q.wide ? 2 * BM : BM) - 1) / (q.wide ? 2 * BM : BM);
    q.nt = (q.Kp + q.bn - 1) / q.bn;
    q.db = p.db;
    q.db_accumulate = p.db_accumulate;
    q.P = ws;
    q.max_splits = tn_splits_max(p);
    q.nseg = p.nseg;
    for (int g = 0; g < p.nseg; ++g) {
      q.seg_at[g] = p.seg_at[g];
      q.seg_len[g] = p.seg_len[g];
      q.seg_to[g] = p.seg_to[g];
    }
    if (p.gather) {
      if ((rc = gather_maps(q, *p.gather, BK))) return rc;
    } else if ((rc = make_map(&q.ta, p.B, p.M, p.K, p.ldb, BK))) {
      return rc;
    }
    if ((rc = make_map(&q.tb, p.A, p.M, p.N, p.lda, BK))) return rc;
  } else if (p.kind == FB_GEMM_TN) {
    q.a_mn = q.b_mn = 1;
    q.ones = p.db ? 1 : 0;
    q.Kp = p.K + q.ones;
    q.bn = bn_mnmajor(q.Kp);
    q.rt = (p.N + BM - 1) / BM;
    q.nt = (q.Kp + q.bn - 1) / q.bn;
    q.db = p.db;
    q.db_accumulate = p.db_accumulate;
    q.P = ws;
    q.max_splits = tn_splits_max(p);
    if ((rc = make_map(&q.ta, p.A, p.M, p.N, p.lda, BK))) return rc;
    if ((rc = make_map(&q.tb, p.B, p.M, p.K, p.ldb, BK))) return rc;
  } else {
    const bool two = p.A2 && p.k1 < p.K;
    q.k1 = two ? p.k1 : p.K;
    q.bias = p.bias;
    q.c_bf16 = p.c_bf16;
    q.a_mn = 0;
    q.b_mn = p.kind == FB_GEMM_NN ? 1 : 0;
    q.bn = q.b_mn ? bn_mnmajor(p.N) : bn_kmajor(p.N);
    q.nt = (p.N + q.bn - 1) / q.bn;
    const int ka = two ? (p.ka > 0 ? p.ka : p.k1) : p.K;
    if (p.gather) {
      if ((rc = gather_maps(q, *p.gather, BM))) return rc;
    } else {
      if ((rc = make_map(&q.ta, p.A, p.M, ka, p.lda, BM))) return rc;
      if (two && (rc = make_map(&q.ta2, p.A2, p.M, p.K - p.k1, p.lda2, BM))) return rc;
    }
    if (q.b_mn) rc = make_map(&q.tb, p.B, p.K, p.N, p.ldb, BK);
    else rc = make_map(&q.tb, p.B, p.N, p.K, p.ldb, q.bn);
    if (rc) return rc;
  }
  q.idesc = idesc_bf16(q.bn, q.a_mn, q.b_mn);
  return FB_OK;
}

int launch_group(const std::vector<const fb_gemm_bf16_problem *> &probs, const std::vector<float *> &ws,
                 cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FB_TRY_CUDA(cudaFuncSetAttribute(k_bf_group<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     smem_bytes<false>()));
    FB_TRY_CUDA(cudaFuncSetAttribute(k_bf_group<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     smem_bytes<true>()));
    attr_set[dev & 63] = true;
  }
  BfArgs a;
  std::memset(&a, 0, sizeof(a));
  a.err = err_word();
  int64_t items = 0;
  int red = 0;
  for (size_t i = 0; i < probs.size(); ++i) {
    BfProb &q = a.p[a.n];
    const int rc = build_prob(q, *probs[i], ws[i]);
    if (rc) return rc;
    a.red_start[a.n] = red;
    a.gat_any |= q.gat;
    if (q.kind == kTN) {
      items += (int64_t)q.rt * q.nt * fb::tn_parts(q.M, q.rows_min, q.max_splits);
      red += (int)(((int64_t)q.N * q.Kp + 255) / 256);
    } else {
      items += (q.M + BM - 1) / BM * q.nt;
    }
    a.n++;
  }
  a.red_start[a.n] = red;
  if (items == 0) return FB_OK;
  const int grid = (int)std::min<int64_t>(items, num_sms());
  bool wide = false;
  for (int i = 0; i < a.n; ++i) wide = wide || a.p[i].wide;
  if (wide) {
    FB_TRY_CUDA(fb::launch(k_bf_group<true>, grid, kThreads, smem_bytes<true>(), stream, a));
  } else {
    FB_TRY_CUDA(fb::launch(k_bf_group<false>, grid, kThreads, smem_bytes<false>(), stream, a));
  }
  FB_LAUNCHED("k_bf_group");
  if (red > 0) {
    FB_TRY_CUDA(fb::launch(k_bf_reduce, red, 256, 0, stream, a));
    FB_LAUNCHED("k_bf_reduce");
  }
  return FB_OK;
}

}  // namespace

extern "C" size_t fb_gemm_bf16_group_ws_bytes(const fb_gemm_bf16_problem *probs, int n) {
  size_t total = 0;
  for (int i = 0; i < n; ++i) total += (size_t)ws_floats(probs[i]) * sizeof(float);
  return total + 256;
}

// Runs the problems (at most kMaxBf per launch, longest work items first).
extern "C" int fb_gemm_bf16_group(const fb_gemm_bf16_problem *probs, int n, void *ws, size_t ws_bytes,
                                  cudaStream_t stream) {
  if (n < 0 || (n > 0 && !probs)) return fb::set_error(FB_ERR_ARG, "gemm_bf16_group: bad problem list");
  if (!encode_fn()) return fb::set_error(FB_ERR_CUDA, "gemm_bf16_group: cuTensorMapEncodeTiled unavailable");
  std::vector<int> live;
  std::vector<float *> pws(n, nullptr);
  size_t need = 0;
  for (int i = 0; i < n; ++i) {
    if (!problem_ok(probs[i]))
      return fb::set_error(FB_ERR_UNSUPPORTED,
                           "gemm_bf16_group: problem " + std::to_string(i) +
                               " needs 16-byte aligned operands with leading dimensions (and k1) multiples of 8");
    if (probs[i].M == 0) continue;
    const size_t w = (size_t)ws_floats(probs[i]) * sizeof(float);
    if (w) {
      pws[i] = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + need);
      need += w;
    }
    live.push_back(i);
  }
  if (need > 0 && (!ws || ws_bytes < need)) return fb::set_error(FB_ERR_ARG, "gemm_bf16_group: workspace too small");
  std::stable_sort(live.begin(), live.end(),
                   [&](int x, int y) { return slices_per_item(probs[x]) > slices_per_item(probs[y]); });
  for (size_t s = 0; s < live.size(); s += kMaxBf) {
    std::vector<const fb_gemm_bf16_problem *> part;
    std::vector<float *> w;
    for (size_t i = s; i < std::min(live.size(), s + kMaxBf); ++i) {
      part.push_back(&probs[live[i]]);
      w.push_back(pws[live[i]]);
    }
    const int rc = launch_group(part, w, stream);
    if (rc) return rc;
  }
  return FB_OK;
}
