// fp32 projection GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a),
// grouped: independent NT / NN / TN problems of one dependency level share one
// persistent launch (one CTA per SM looping over 128 x bn output tiles).
//
//   NT: C[m, n] (+)= sum_k A[m, k] B[n, k] + bias[n]     A, B K-major
//   NN: C[m, n] (+)= sum_k A[m, k] B[k, n] + bias[n]     A K-major, B MN-major
//   TN: P[s][n, k] = sum_{m in split s} G[m, n] X[m, k]  G, X MN-major; a ones
//       column of X at k = K gives the bias gradient; k_tc_reduce sums the
//       splits in a fixed order into C (+ C) and db (+ db)
//   NT / NN may take A as [A | A2] concatenated along K.
//
// Operands are moved by TMA exactly as they lie in memory: K-major tiles as
// [rows][32 k] boxes with the 128-byte swizzle (16-byte chunks), MN-major
// tiles as [32 k][32 mn] boxes side by side with the 128-byte swizzle of
// 32-byte chunks (the one shared-memory layout the tensor cores accept for
// MN-major 32-bit operands), and the MMA reads them through K-major or
// MN-major descriptors, so no operand is transposed by software.
//
// fp32 accuracy from TF32 tensor-core products with the split of Ootomo &
// Yokota ("Recovering single precision accuracy from Tensor Cores while
// surpassing the FP32 theoretical peak performance", IJHPCA 2022): every
// operand x is written as hi + lo with hi = x rounded to TF32 and lo = the
// residual x - hi (exact in fp32) rounded to TF32, and
//   A B ~= A_lo B_hi + A_hi B_lo + A_hi B_hi,
// three kind::tf32 MMAs accumulating in fp32 in tensor memory.
//
// CTA = 10 warps:
//   warp 0      TMA producer: raw A/B slices -> shared memory
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 2..5  split each slice into hi (in place) + lo; zero the rows of a
//               TN slice outside its split; write the ones column
//   warps 6..9  per slice, add the slice's TMEM accumulator into fp32
//               registers (one output row per thread); per tile, the store
// Stages are handed over with mbarriers: full (TMA bytes landed) -> conv
// (split written, made visible to the async proxy) -> empty (tcgen05.commit
// once the MMAs reading the stage are done); the two slice accumulators with
// accf (committed) / acce (promoted).  The slice counter runs on across the
// tiles of a CTA, so the next tile's loads and MMAs overlap the last tile's
// promotion and store.  Every wait is bounded: past the limit the CTA records
// an error, stops issuing work, drains what it already issued (again
// bounded), frees its tensor memory and exits.
//
// Every TMA load here is issued by one CTA for its own shared memory.
#include <cuda.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>
#include "runtime.cuh"
#include "tc_common.cuh"

namespace fbtc {

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
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

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

}  // namespace fbtc

namespace {

using namespace fbtc;

constexpr int BM = 128;                      // MMA M: tile rows = TMEM lanes
constexpr int BK = 32;                       // reduction slice: 32 fp32 = one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kMaxTc = 7;                    // problems per launch (keeps the parameters under 4 KB)
constexpr int kOpBytes = BM * BK * 4;        // one operand slice, at most 128 x 32 fp32
constexpr int kStage = 4 * kOpBytes;         // A hi | A lo | B hi | B lo
constexpr int kStagePitch = 33;             // epilogue staging rows (floats; odd: no bank conflicts)
constexpr int kStageWarp = 32 * kStagePitch * 4;
constexpr int kSmem = 1024 + kStages * kStage + 128 + 4 * kStageWarp;
constexpr int kTmemCols = 512;               // two slice accumulators + the running sum, 128 columns each
constexpr int kAccStride = 128;
constexpr int kRunCol = 256;                 // TMEM column of the fp32 running sum
constexpr int64_t kTnRowsMin = 256;          // TN: rows per split, at least


enum : int { kNT = 0, kNN = 1, kTN = 2 };

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor, tile base 1024-byte aligned.
//   K-major (SWIZZLE_128B, 16-byte chunks): rows of 128 B (32 k), 8-row
//     groups 1024 B apart (SBO); a K step of 8 fp32 advances the start by 32 B.
//   MN-major (SWIZZLE_128B with 32-byte atoms): boxes of [32 k][32 mn] (4 KB)
//     side by side along MN (LBO 4 KB), 4-row k groups 512 B apart (SBO); a K
//     step of 8 advances the start by 1 KB.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, bool mn) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);                  // start address
  d |= (uint64_t)(mn ? (4096 >> 4) : 1) << 16;               // leading byte offset
  d |= (uint64_t)((mn ? 512 : 1024) >> 4) << 32;             // stride byte offset
  d |= (uint64_t)1 << 46;                                    // descriptor version (sm_100)
  d |= (uint64_t)(mn ? 1 : 2) << 61;                         // SWIZZLE_128B_BASE32B / SWIZZLE_128B
  return d;
}

// Round to TF32's 10 explicit mantissa bits, to nearest with ties away from
// zero, by integer arithmetic on the fp32 bit pattern: add half of the 13
// dropped bits, then clear them (a carry into the exponent rounds up to the
// next binade).  Two integer operations instead of a conversion instruction,
// which the split would otherwise issue 16 times per 4 elements.
__device__ __forceinline__ float to_tf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// x = hi + lo with hi = tf32(x) and lo = tf32(x - hi) (x - hi is exact in fp32).
__device__ __forceinline__ void split_tf32(const float4 v, float4 &h, float4 &l) {
  h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
  l = make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
}

__device__ __forceinline__ void set_lane(float4 &v, int e, float x) {
  if (e == 0) v.x = x;
  else if (e == 1) v.y = x;
  else if (e == 2) v.z = x;
  else v.w = x;
}

struct TcProb {
  CUtensorMap ta, ta2, tb;   // A (TN: G), A2, B (TN: X)
  int kind, a_mn, b_mn, b_synth;
  int k1, K, N, Kp, bn, rt, nt;
  int ones, accumulate, db_accumulate, max_splits;
  uint32_t idesc;
  int64_t M;
  const int32_t *M_dev;
  const float *bias;
  float *C;
  int64_t ldc;
  float *db, *P;
};

struct TcArgs {
  TcProb p[kMaxTc];
  int n;
  int red_start[kMaxTc + 1];
  int32_t *err;
};
static_assert(sizeof(TcArgs) <= 4096, "kernel parameters of k_tc_group exceed 4 KB");

// One work item: a 128 x bn output tile of problem p (TN: of split z).
struct Item {
  int p, z, nk, nk1, c0;
  int64_t r0, s0, s1;
};

__device__ __forceinline__ Item decode(const TcArgs &a, const int *st, const long long *sm, const long long *sper,
                                       int i) {
  Item it;
  int p = 0;
  while (p + 1 < a.n && i >= st[p + 1]) ++p;
  const TcProb &q = a.p[p];
  int l = i - st[p];
  it.p = p;
  if (q.kind == kTN) {
    const int per_z = q.rt * q.nt;
    it.z = l / per_z;
    l -= it.z * per_z;
    it.r0 = (int64_t)(l / q.nt) * BM;
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

// Warp roles of the 16-warp CTA (warps 2 and 3 only join the final barrier;
// the epilogue warps 12..15 reach TMEM lane quadrants 0..3).
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpConv0 = 4, kWarpEpi0 = 12;
constexpr int kConvThreads = (kWarpEpi0 - kWarpConv0) * 32;   // 256
constexpr int kThreadsTc = 512;

// The tensor-core accumulator adds with truncation; summing a whole K range in
// it loses ~10x more than fp32.  So each 32-wide K slice is accumulated alone
// (small correction products first, hi*hi last) in one of two TMEM buffers,
// and the promotion warps add the finished slice into an fp32 running sum
// (kept in TMEM, read and written back by the same thread) with
// round-to-nearest while the tensor cores fill the other buffer.
__global__ void __launch_bounds__(kThreadsTc, 1) k_tc_group(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned tile base, derived from the shared array itself so the
  // compiler keeps every tile access in the shared address space
  uint8_t *smem = align1024(smem_raw);
  auto sA = [&](int s) { return smem + s * kStage; };
  auto sAlo = [&](int s) { return smem + s * kStage + kOpBytes; };
  auto sB = [&](int s) { return smem + s * kStage + 2 * kOpBytes; };
  auto sBlo = [&](int s) { return smem + s * kStage + 3 * kOpBytes; };
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * kStage);
  uint64_t *full = bars, *conv = bars + kStages, *empty = bars + 2 * kStages;
  uint64_t *accf = bars + 3 * kStages, *acce = bars + 3 * kStages + 2, *drain = bars + 3 * kStages + 4;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * kStages + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int32_t *err = a.err;
  __shared__ int s_start[kMaxTc + 1];
  __shared__ long long s_m[kMaxTc], s_per[kMaxTc];

  // Setup that reads nothing the previous kernel writes (barriers, tensor
  // memory, tensor-map prefetch) runs before the dependency wait, so under
  // programmatic dependent launch it overlaps the previous kernel's tail.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(conv + s, kConvThreads);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kWarpProducer && lane < a.n) {
    const TcProb &q = a.p[lane];
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&q.ta)) : "memory");
    if (q.kind != kTN && q.k1 < q.K)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&q.ta2)) : "memory");
    if (!q.b_synth) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&q.tb)) : "memory");
  }
  if (warp == kWarpMma) tmem_alloc(tmem_holder, kTmemCols);

  fb::pdl_enter();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int p = 0; p < a.n; ++p) {
      const TcProb &q = a.p[p];
      int64_t M = q.M_dev ? min((int64_t)(*q.M_dev), q.M) : q.M;
      M = max(M, (int64_t)0);
      s_m[p] = M;
      s_start[p] = acc;
      if (q.kind == kTN) {
        const int ns = fb::tn_parts(M, kTnRowsMin, q.max_splits);
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
  if ((int)blockIdx.x >= total) {         // nothing for this CTA at the device-side sizes
    if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
    return;
  }

  if (warp == kWarpProducer) {
    if (lane == 0) {
      uint32_t g = 0;
      bool stop = false;
      for (int i = blockIdx.x; i < total && !stop; i += gridDim.x) {
        const Item it = decode(a, s_start, s_m, s_per, i);
        const TcProb &q = a.p[it.p];
        const bool tn = q.kind == kTN, synth = q.b_synth != 0, bmn = q.b_mn != 0;
        const int bn = q.bn, k1 = q.k1;
        const uint32_t bytes = kOpBytes + (synth ? 0u : (uint32_t)(bn * BK * 4));
        const int r0 = (int)it.r0;
        for (int j = 0; j < it.nk; ++j) {
          const int s = g % kStages;
          if (g >= kStages && !mbar_wait(empty + s, ((g / kStages) - 1) & 1, abort_flag, err)) {
            stop = true;
            break;
          }
          mbar_expect_tx(full + s, bytes);
          // reduction coordinate of this slice in B (NT / NN) and in A, B (TN)
          const int kb = j < it.nk1 ? BK * j : k1 + BK * (j - it.nk1);
          const int my = (int)it.s0 + BK * j;
          if (tn) {
#pragma unroll
            for (int t = 0; t < BM / 32; ++t) tma_load_2d(sA(s) + t * 4096, &q.ta, full + s, r0 + 32 * t, my);
          } else if (j < it.nk1) {
            tma_load_2d(sA(s), &q.ta, full + s, BK * j, r0);
          } else {
            tma_load_2d(sA(s), &q.ta2, full + s, BK * (j - it.nk1), r0);
          }
          if (!synth) {
            if (!bmn) {
              tma_load_2d(sB(s), &q.tb, full + s, kb, it.c0);
            } else {
              const int y = tn ? my : kb;
              for (int t = 0; t < bn / 32; ++t) tma_load_2d(sB(s) + t * 4096, &q.tb, full + s, it.c0 + 32 * t, y);
            }
          }
          ++g;
        }
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA's memory goes away
        for (uint32_t h = g > (uint32_t)kStages ? g - kStages : 0; h < g; ++h) {
          const long long t0 = clock64();
          while (!mbar_try_wait(full + h % kStages, (h / kStages) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      uint32_t g = 0;
      bool stop = false;
      for (int i = blockIdx.x; i < total && !stop; i += gridDim.x) {
        const Item it = decode(a, s_start, s_m, s_per, i);
        const TcProb &q = a.p[it.p];
        const uint32_t idesc = q.idesc;
        const bool amn = q.a_mn != 0, bmn = q.b_mn != 0;
        const uint64_t adv_a = amn ? 64 : 2, adv_b = bmn ? 64 : 2;   // one K step of 8, in 16-byte units
        for (int j = 0; j < it.nk; ++j) {
          const int s = g % kStages, b = g & 1;
          if (g >= 2 && !mbar_wait(acce + b, ((g >> 1) - 1) & 1, abort_flag, err)) {
            stop = true;
            break;
          }
          if (!mbar_wait(conv + s, (g / kStages) & 1, abort_flag, err)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(b * kAccStride);
          const uint64_t ah = sdesc_sw128(smem_u32(sA(s)), amn), al = sdesc_sw128(smem_u32(sAlo(s)), amn);
          const uint64_t bh = sdesc_sw128(smem_u32(sB(s)), bmn), bl = sdesc_sw128(smem_u32(sBlo(s)), bmn);
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) umma_tf32(d, al + kk * adv_a, bh + kk * adv_b, idesc, kk != 0);
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) umma_tf32(d, ah + kk * adv_a, bl + kk * adv_b, idesc, 1);
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) umma_tf32(d, ah + kk * adv_a, bh + kk * adv_b, idesc, 1);
          umma_commit(empty + s);
          umma_commit(accf + b);
          ++g;
        }
      }
      // every MMA this thread issued must be complete before TMEM is freed
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
  } else if (warp >= kWarpConv0 && warp < kWarpEpi0) {
    const int ct = threadIdx.x - kWarpConv0 * 32;   // 0..255
    uint32_t g = 0;
    bool stop = false;
    for (int i = blockIdx.x; i < total && !stop; i += gridDim.x) {
      const Item it = decode(a, s_start, s_m, s_per, i);
      const TcProb &q = a.p[it.p];
      const bool tn = q.kind == kTN, synth = q.b_synth != 0;
      const int nb4 = q.bn * BK / 4;
      // TN: the ones column of X, as a column of this tile (-1: not here)
      const int onescol = (q.ones && q.K >= it.c0 && q.K < it.c0 + q.bn) ? q.K - it.c0 : -1;
      const int64_t s1 = it.s1;
      for (int j = 0; j < it.nk; ++j) {
        const int s = g % kStages;
        if (!mbar_wait(full + s, (g / kStages) & 1, abort_flag, err)) {
          stop = true;
          break;
        }
        const int64_t rbase = it.s0 + BK * j;   // TN: row m of box row 0
        // all loads of a half-slice are issued before its stores
        float4 *a4 = reinterpret_cast<float4 *>(sA(s));
        float4 *al4 = reinterpret_cast<float4 *>(sAlo(s));
        constexpr int kPer = BM * BK / 4 / kConvThreads;   // float4 per thread and operand: 4
        float4 v[kPer];
#pragma unroll
        for (int t = 0; t < kPer; ++t) v[t] = a4[ct + kConvThreads * t];
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
          const int idx = ct + kConvThreads * t;
          float4 h, l;
          if (tn && rbase + ((idx >> 3) & 31) >= s1) {
            h = l = make_float4(0.f, 0.f, 0.f, 0.f);
          } else {
            split_tf32(v[t], h, l);
          }
          a4[idx] = h;
          al4[idx] = l;
        }
        float4 *b4 = reinterpret_cast<float4 *>(sB(s));
        float4 *bl4 = reinterpret_cast<float4 *>(sBlo(s));
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
          const int idx = ct + kConvThreads * t;
          v[t] = (!synth && idx < nb4) ? b4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
          const int idx = ct + kConvThreads * t;
          if (idx < nb4) {
            float4 h, l;
            const int row = (idx >> 3) & 31;
            const bool valid = !tn || rbase + row < s1;
            if (!valid) {
              h = l = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
              split_tf32(v[t], h, l);
            }
            if (onescol >= 0 && (idx >> 8) == (onescol >> 5)) {
              // MN-major box: 32-byte chunk p of row `row` holds logical chunk p ^ (row & 3)
              const int c = onescol & 31;
              const int lc = ((((idx & 7) >> 1) ^ (row & 3)) << 1) | (idx & 1);   // logical 16-byte chunk
              if ((c >> 2) == lc) {
                set_lane(h, c & 3, valid ? 1.f : 0.f);
                set_lane(l, c & 3, 0.f);
              }
            }
            b4[idx] = h;
            bl4[idx] = l;
          }
        }
        fence_async_smem();
        mbar_arrive(conv + s);
        ++g;
      }
    }
  } else if (warp >= kWarpEpi0) {
    // promotion + epilogue: warp w owns TMEM lanes 32*(w % 4) .. +31 = one output row per thread
    const int qd = warp & 3;
    const uint32_t tlane = (uint32_t)(qd * 32) << 16;
    const uint32_t run = tmem + tlane + kRunCol;
    float *stg = reinterpret_cast<float *>(smem + kStages * kStage + 128 + qd * kStageWarp);
    uint32_t g = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
      const Item it = decode(a, s_start, s_m, s_per, i);
      const TcProb &q = a.p[it.p];
      const int bn = q.bn;
      for (int j = 0; j < it.nk; ++j) {
        const int b = g & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(accf + b, (g >> 1) & 1, abort_flag, err) ? 1 : 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t t = tmem + tlane + (uint32_t)(b * kAccStride);
#pragma unroll 1
        for (int c0 = 0; c0 < bn; c0 += 32) {
          uint32_t r[32], u[32];
          tmem_ld32(t + c0, r);
          if (j > 0) {
            tmem_ld32(run + c0, u);
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) + __uint_as_float(u[e]));
          }
          tmem_st32(run + c0, r);
        }
        tc_fence_before();
        mbar_arrive(acce + b);
        ++g;
      }
      if (!ok) break;
      // store: per 32-column block, rows through this warp's staging area, so
      // that each store instruction writes one row's 32 consecutive columns.
      // The problem's fields are copied to registers first: read through a
      // pointer into the parameters, they would be reloaded after every store.
      const bool tn = q.kind == kTN;
      const int64_t rows = tn ? (int64_t)q.N : (int64_t)s_m[it.p];
      const int ncols = tn ? q.Kp : q.N;
      const int64_t ld = tn ? (int64_t)q.Kp : q.ldc;
      float *const out = tn ? q.P + (int64_t)it.z * q.N * q.Kp : q.C;
      const float *const bias = tn ? nullptr : q.bias;
      const bool accum = !tn && q.accumulate;
      const int64_t row0 = it.r0 + qd * 32;
      const int nrows = rows - row0 < 32 ? (int)(rows - row0) : 32;
#pragma unroll 1
      for (int c0 = 0; c0 < bn; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(run + c0, r);
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 32; ++e) stg[lane * kStagePitch + e] = __uint_as_float(r[e]);
        __syncwarp();
        const int col = it.c0 + c0 + lane;
        if (c0 + lane < bn && col < ncols) {
          const float bv = bias ? bias[col] : 0.f;
          float *o = out + row0 * ld + col;
          const float *sv = stg + lane;
          if (nrows == 32) {              // unrolled: the staging loads are issued ahead of the stores
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
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
}

// Sums the TN partials of every TN problem of the launch (fixed split order)
// into C (+ C) and, for the ones column, db (+ db).
__global__ void k_tc_reduce(const __grid_constant__ TcArgs a) {
  fb::pdl_enter();
  int p = -1;
  for (int i = 0; i < a.n; ++i)
    if (a.p[i].kind == kTN && (int)blockIdx.x >= a.red_start[i] && (int)blockIdx.x < a.red_start[i + 1]) p = i;
  if (p < 0) return;
  const TcProb &q = a.p[p];
  const int64_t i = (int64_t)(blockIdx.x - a.red_start[p]) * blockDim.x + threadIdx.x;
  if (i >= (int64_t)q.N * q.Kp) return;
  int64_t M = q.M_dev ? min((int64_t)(*q.M_dev), q.M) : q.M;
  M = max(M, (int64_t)0);
  const int ns = fb::tn_parts(M, kTnRowsMin, q.max_splits);
  const int n = (int)(i / q.Kp), k = (int)(i % q.Kp);
  const int64_t stride = (int64_t)q.N * q.Kp;
  const float *part = q.P + i;
  float s = 0.f;
  int z = 0;
  for (; z + 8 <= ns; z += 8) {          // eight loads in flight, added in split order
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = part[(int64_t)(z + u) * stride];
#pragma unroll
    for (int u = 0; u < 8; ++u) s += v[u];
  }
  for (; z < ns; ++z) s += part[(int64_t)z * stride];
  float *c = (k < q.K) ? q.C + (int64_t)n * q.ldc + k : q.db + n;
  const int acc = (k < q.K) ? q.accumulate : q.db_accumulate;
  *c = acc ? (*c + s) : s;
}

// Row-major fp32 [rows, cols] with leading dimension ld, boxes of 32 columns x
// box_rows rows; reads past the extents return zeros.  mn: the 32-byte-atom
// swizzle of MN-major operand tiles, else the 16-byte-chunk 128-byte swizzle.
int make_map(CUtensorMap *m, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows, bool mn) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fb::set_error(FB_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fb::set_error(FB_ERR_ARG, "gemm_tc: tensor map rejected (alignment or stride)");
  return FB_OK;
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tile width along the MMA N dimension.  K-major B: any multiple of 16 up to
// 128, as even as the tiles allow.  MN-major B: whole 32-column boxes, the
// width that wastes the fewest columns counting a per-tile cost.
int bn_kmajor(int N) {
  const int t = (N + 127) / 128, w = (N + t - 1) / t;
  return (w + 15) / 16 * 16;
}
int bn_mnmajor(int N) {
  int best = 128, cost = (N + 127) / 128 * (128 + 16);
  for (int w : {96, 64, 32}) {
    const int c = (N + w - 1) / w * (w + 16);
    if (c < cost) cost = c, best = w;
  }
  return best;
}

uint32_t idesc_tf32(int bn, int a_mn, int b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

int tn_splits_max(const fb_gemm_problem &p) {
  const int Kp = p.K + (p.db ? 1 : 0);
  const int tiles = ((p.N + BM - 1) / BM) * ((Kp + bn_mnmajor(Kp) - 1) / bn_mnmajor(Kp));
  return std::max(1, num_sms() / std::max(tiles, 1));
}

// Slices per work item (for ordering the problems, longest first).
int64_t slices_per_item(const fb_gemm_problem &p) {
  if (p.kind == FB_GEMM_TN) {
    const int ns = fb::tn_parts(p.M, kTnRowsMin, tn_splits_max(p));
    return ((p.M + ns - 1) / ns + BK - 1) / BK;
  }
  const int k1 = (p.A2 && p.k1 < p.K) ? p.k1 : p.K;
  return (k1 + BK - 1) / BK + (p.K - k1 + BK - 1) / BK;
}

int build_prob(TcProb &q, const fb_gemm_problem &p, float *ws) {
  std::memset(&q, 0, sizeof(q));
  q.kind = p.kind;
  q.M = p.M;
  q.M_dev = p.M_dev;
  q.N = p.N;
  q.K = p.K;
  q.accumulate = p.accumulate;
  q.C = p.C;
  q.ldc = p.ldc;
  int rc;
  if (p.kind == FB_GEMM_TN) {
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
    q.b_synth = p.K == 0 ? 1 : 0;
    if ((rc = make_map(&q.ta, p.A, p.M, p.N, p.lda, 32, true))) return rc;
    if (!q.b_synth && (rc = make_map(&q.tb, p.B, p.M, p.K, p.ldb, 32, true))) return rc;
  } else {
    const bool two = p.A2 && p.k1 < p.K;
    q.k1 = two ? p.k1 : p.K;
    q.bias = p.bias;
    q.a_mn = 0;
    q.b_mn = p.kind == FB_GEMM_NN ? 1 : 0;
    q.bn = q.b_mn ? bn_mnmajor(p.N) : bn_kmajor(p.N);
    q.nt = (p.N + q.bn - 1) / q.bn;
    if ((rc = make_map(&q.ta, p.A, p.M, q.k1, p.lda, BM, false))) return rc;
    if (two && (rc = make_map(&q.ta2, p.A2, p.M, p.K - p.k1, p.lda2, BM, false))) return rc;
    if (q.b_mn) rc = make_map(&q.tb, p.B, p.K, p.N, p.ldb, 32, true);
    else rc = make_map(&q.tb, p.B, p.N, p.K, p.ldb, q.bn, false);
    if (rc) return rc;
  }
  q.idesc = idesc_tf32(q.bn, q.a_mn, q.b_mn);
  return FB_OK;
}

int launch_group(const std::vector<const fb_gemm_problem *> &probs, const std::vector<float *> &ws,
                 cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    FB_TRY_CUDA(cudaFuncSetAttribute(k_tc_group, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr_set[dev] = true;
  }
  TcArgs a;
  std::memset(&a, 0, sizeof(a));
  a.err = err_word();
  int64_t items = 0;
  int red = 0;
  for (size_t i = 0; i < probs.size(); ++i) {
    TcProb &q = a.p[a.n];
    const int rc = build_prob(q, *probs[i], ws[i]);
    if (rc) return rc;
    a.red_start[a.n] = red;
    if (q.kind == kTN) {
      items += (int64_t)q.rt * q.nt * fb::tn_parts(q.M, kTnRowsMin, q.max_splits);
      red += (int)(((int64_t)q.N * q.Kp + 255) / 256);
    } else {
      items += (q.M + BM - 1) / BM * q.nt;
    }
    a.n++;
  }
  a.red_start[a.n] = red;
  if (items == 0) return FB_OK;
  const int grid = (int)std::min<int64_t>(items, num_sms());
  FB_TRY_CUDA(fb::launch(k_tc_group, grid, kThreadsTc, kSmem, stream, a));
  FB_LAUNCHED("k_tc_group");
  if (red > 0) {
    FB_TRY_CUDA(fb::launch(k_tc_reduce, red, 256, 0, stream, a));
    FB_LAUNCHED("k_tc_reduce");
  }
  return FB_OK;
}

}  // namespace

namespace fb {

bool tc_enabled() {
  const char *v = getenv("FB_GEMM");
  return !(v && std::strcmp(v, "ffma") == 0) && encode_fn() != nullptr;
}

bool tc_problem_ok(const fb_gemm_problem &p) {
  if (p.M < 1 || p.M > (int64_t)1 << 30 || p.N < 1 || p.K < 0) return false;
  if (!p.A || !al16(p.A) || p.lda % 4) return false;
  if (p.kind == FB_GEMM_TN) {
    if (p.K == 0) return p.db != nullptr;
    return p.B && al16(p.B) && p.ldb % 4 == 0;
  }
  if (p.K < 1 || !p.B || !al16(p.B) || p.ldb % 4) return false;
  if (p.A2 && p.k1 < p.K) return p.k1 >= 4 && p.k1 % 4 == 0 && al16(p.A2) && p.lda2 % 4 == 0;
  return true;
}

int64_t tc_ws_floats(const fb_gemm_problem &p) {
  if (p.kind != FB_GEMM_TN || p.M < 1) return 0;
  const int Kp = p.K + (p.db ? 1 : 0);
  const int64_t ns = tn_parts(p.M, kTnRowsMin, tn_splits_max(p));
  return (ns * (int64_t)p.N * Kp + 63) / 64 * 64;
}

// Launches the problems (all tc_problem_ok, M > 0) on the tensor cores, at
// most kMaxTc per launch, longest work items first.  ws[i]: TN partials of
// problem i (tc_ws_floats floats).
int tc_group(const fb_gemm_problem *const *probs, float *const *ws, int n, cudaStream_t stream) {
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int x, int y) { return slices_per_item(*probs[x]) > slices_per_item(*probs[y]); });
  for (int s = 0; s < n; s += kMaxTc) {
    std::vector<const fb_gemm_problem *> part;
    std::vector<float *> pws;
    for (int i = s; i < std::min(n, s + kMaxTc); ++i) {
      part.push_back(probs[order[i]]);
      pws.push_back(ws[order[i]]);
    }
    const int rc = launch_group(part, pws, stream);
    if (rc) return rc;
  }
  return FB_OK;
}

}  // namespace fb

extern "C" int fb_gemm_nt_tc_supported(const float *A, int64_t lda, const float *B, int64_t ldb, int N, int K) {
  fb_gemm_problem p{};
  p.kind = FB_GEMM_NT;
  p.A = A; p.lda = lda; p.B = B; p.ldb = ldb; p.M = 1; p.N = N; p.K = K;
  return fb::tc_problem_ok(p) && encode_fn() != nullptr;
}

extern "C" int fb_gemm_nt_tc(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C,
                             int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K, int accumulate,
                             cudaStream_t stream) {
  if (!C || M < 0 || ldc < N || !fb_gemm_nt_tc_supported(A, lda, B, ldb, N, K))
    return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_nt_tc: needs K, lda, ldb multiples of 4 and 16-byte aligned A, B");
  if (M == 0) return FB_OK;
  fb_gemm_problem p{};
  p.kind = FB_GEMM_NT;
  p.A = A; p.lda = lda; p.B = B; p.ldb = ldb; p.bias = bias; p.C = C; p.ldc = ldc;
  p.M = M; p.M_dev = M_dev; p.N = N; p.K = K; p.accumulate = accumulate;
  const fb_gemm_problem *pp = &p;
  float *ws = nullptr;
  return fb::tc_group(&pp, &ws, 1, stream);
}

extern "C" int fb_gemm_tc_error(int *flags, int clear) {
  if (!flags) return fb::set_error(FB_ERR_ARG, "gemm_tc_error: null");
  int32_t *w = err_word();
  FB_TRY_CUDA(cudaMemcpy(flags, w, 4, cudaMemcpyDeviceToHost));
  if (clear) FB_TRY_CUDA(cudaMemset(w, 0, 4));
  return FB_OK;
}
