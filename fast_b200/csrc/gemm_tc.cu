// fp32 projection GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[m, n] (+)= sum_k A[m, k] B[n, k] + bias[n]        A, B K-major (row-major, k contiguous)
//
// fp32 accuracy from TF32 tensor-core products with the split of Ootomo &
// Yokota ("Recovering single precision accuracy from Tensor Cores while
// surpassing the FP32 theoretical peak performance", IJHPCA 2022): every
// operand x is written as hi + lo with hi = x rounded to TF32 and lo = the
// residual x - hi (exact in fp32) rounded to TF32, and
//   A B ~= A_hi B_hi + A_hi B_lo + A_lo B_hi,
// three kind::tf32 MMAs accumulating in fp32 in tensor memory.
//
// CTA = 10 warps, one 128 x BN output tile (BN <= 128), K in 32-float
// (128-byte) slices:
//   warp 0      TMA producer: raw A/B slices -> SWIZZLE_128B shared memory
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 2..5  split each slice into hi (in place) + lo
//   warps 6..9  per slice, add the slice's TMEM accumulator into fp32
//               registers (one output row per thread); finally bias + store
// Stages are handed over with mbarriers: full (TMA bytes landed) -> conv
// (split written, made visible to the async proxy) -> empty (tcgen05.commit
// once the MMAs reading the stage are done); the two slice accumulators with
// accf (committed) / acce (promoted).  Every wait is bounded: past the limit
// the CTA records an error, stops issuing work, drains what it already issued
// (again bounded), frees its tensor memory and exits.
//
// Every TMA load here is issued by one CTA for its own shared memory.
#include <cuda.h>
#include <algorithm>
#include "runtime.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 32;                       // fp32 per 128-byte swizzle row

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz
constexpr int kErrTimeout = 2;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false when the CTA is aborting (set here on timeout).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int32_t *err) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart, tile base 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);   // start address
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::tf32: fp32 accumulate, TF32 A and B, both K-major.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <int BN>
struct Cfg {
  static constexpr int kStages = 3;
  static constexpr int kTileA = BM * BK * 4;   // bytes of one A slice
  static constexpr int kTileB = BN * BK * 4;
  static constexpr int kStage = 2 * kTileA + 2 * kTileB;   // raw/hi + lo of A and B
  static constexpr int kAccStride = 128;       // TMEM columns between the two slice accumulators
  static constexpr int kTmemCols = 256;
  static constexpr int kSmem = 1024 + kStages * kStage + 64 * 8 + 64;
};

// Round-to-nearest TF32 (low 13 mantissa bits cleared), as a float.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// x = hi + lo with hi = rna_tf32(x) and lo = rna_tf32(x - hi).
__device__ __forceinline__ void split_tf32(const float4 v, float4 &h, float4 &l) {
  h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
  l = make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
}

// Warp roles of the 10-warp CTA.
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpConv0 = 2, kWarpEpi0 = 6;
constexpr int kThreadsTc = 320;

// The tensor-core accumulator adds with truncation; summing a whole K range in
// it loses ~10x more than fp32.  So each 32-wide K slice is accumulated alone
// (small correction products first, hi*hi last) in one of two TMEM buffers,
// and the promotion warps add the finished slice into fp32 registers with
// round-to-nearest while the tensor cores fill the other buffer.
template <int BN>
__global__ void __launch_bounds__(kThreadsTc, 1)
    k_gemm_nt_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const float *__restrict__ bias, float *__restrict__ C, int64_t ldc, int64_t M_host,
                 const int32_t *M_dev, int N, int K, int accumulate, int32_t *err) {
  using CF = Cfg<BN>;
  constexpr int S = CF::kStages;
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  if (m0 >= M) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sA = [&](int s) { return smem + s * CF::kStage; };
  auto sAlo = [&](int s) { return smem + s * CF::kStage + CF::kTileA; };
  auto sB = [&](int s) { return smem + s * CF::kStage + 2 * CF::kTileA; };
  auto sBlo = [&](int s) { return smem + s * CF::kStage + 2 * CF::kTileA + CF::kTileB; };
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * CF::kStage);
  uint64_t *full = bars, *conv = bars + S, *empty = bars + 2 * S;
  uint64_t *accf = bars + 3 * S, *acce = bars + 3 * S + 2, *drain = bars + 3 * S + 4;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * S + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(conv + s, 128);
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
  if (warp == kWarpMma) tmem_alloc(tmem_holder, CF::kTmemCols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int nk = (K + BK - 1) / BK;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % S, u = kt / S;
        if (kt >= S && !mbar_wait(empty + s, (u - 1) & 1, abort_flag, err)) break;
        mbar_expect_tx(full + s, CF::kTileA + CF::kTileB);
        tma_load_2d(sA(s), &tmA, full + s, kt * BK, (int)m0);
        tma_load_2d(sB(s), &tmB, full + s, kt * BK, n0);
        ++issued;
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA's memory goes away
        for (int kt = max(0, issued - S); kt < issued; ++kt) {
          const long long t0 = clock64();
          while (!mbar_try_wait(full + kt % S, (kt / S) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32<BN>();
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % S, b = kt & 1;
        if (kt >= 2 && !mbar_wait(acce + b, ((kt >> 1) - 1) & 1, abort_flag, err)) break;
        if (!mbar_wait(conv + s, (kt / S) & 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * CF::kAccStride);
        const uint64_t ah = sdesc_k_sw128(smem_u32(sA(s))), al = sdesc_k_sw128(smem_u32(sAlo(s)));
        const uint64_t bh = sdesc_k_sw128(smem_u32(sB(s))), bl = sdesc_k_sw128(smem_u32(sBlo(s)));
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {   // 8 tf32 = 32 bytes along K per MMA
          const uint64_t adv = (uint64_t)(kk * 32 >> 4);
          umma_tf32(d, al + adv, bh + adv, idesc, kk != 0);
        }
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t adv = (uint64_t)(kk * 32 >> 4);
          umma_tf32(d, ah + adv, bl + adv, idesc, 1);
        }
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t adv = (uint64_t)(kk * 32 >> 4);
          umma_tf32(d, ah + adv, bh + adv, idesc, 1);
        }
        umma_commit(empty + s);
        umma_commit(accf + b);
      }
      // every MMA this thread issued must be complete before TMEM is freed
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
  } else if (warp < kWarpEpi0) {
    const int ct = threadIdx.x - kWarpConv0 * 32;   // 0..127
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % S, u = kt / S;
      if (!mbar_wait(full + s, u & 1, abort_flag, err)) break;
      float4 *a4 = reinterpret_cast<float4 *>(sA(s));
      float4 *al4 = reinterpret_cast<float4 *>(sAlo(s));
#pragma unroll
      for (int i = 0; i < BM * BK / 4 / 128; ++i) {
        const int idx = ct + 128 * i;
        float4 h, l;
        split_tf32(a4[idx], h, l);
        a4[idx] = h;
        al4[idx] = l;
      }
      float4 *b4 = reinterpret_cast<float4 *>(sB(s));
      float4 *bl4 = reinterpret_cast<float4 *>(sBlo(s));
#pragma unroll
      for (int i = 0; i < BN * BK / 4 / 128; ++i) {
        const int idx = ct + 128 * i;
        float4 h, l;
        split_tf32(b4[idx], h, l);
        b4[idx] = h;
        bl4[idx] = l;
      }
      fence_async_smem();
      mbar_arrive(conv + s);
    }
  } else {
    // promotion + epilogue: warp w owns TMEM lanes 32*(w % 4) .. +31 = one output row per thread
    const int q = warp & 3;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    float acc[BN];
#pragma unroll
    for (int c = 0; c < BN; ++c) acc[c] = 0.f;
    bool ok = true;
    for (int kt = 0; kt < nk; ++kt) {
      const int b = kt & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(accf + b, (kt >> 1) & 1, abort_flag, err) ? 1 : 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t = tmem + tlane + (uint32_t)(b * CF::kAccStride);
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(t + c0, r);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[c0 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      mbar_arrive(acce + b);
    }
    const int64_t row = m0 + q * 32 + lane;
    if (ok && row < M) {
      float *crow = C + row * ldc + n0;
      const bool vec = (ldc % 4 == 0) && (n0 % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
#pragma unroll
      for (int c = 0; c < BN; c += 4) {
        const int col = n0 + c;
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = acc[c + t] + ((bias && col + t < N) ? bias[col + t] : 0.f);
        if (vec && col + 3 < N) {
          float4 *p = reinterpret_cast<float4 *>(crow + c);
          if (accumulate) {
            const float4 o = *p;
            v[0] += o.x; v[1] += o.y; v[2] += o.z; v[3] += o.w;
          }
          *p = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t)
            if (col + t < N) crow[c + t] = accumulate ? crow[c + t] + v[t] : v[t];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, CF::kTmemCols);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

// Row-major fp32 [rows, cols] with leading dimension ld, boxes of 32 x box_rows.
int make_map(CUtensorMap *m, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fb::set_error(FB_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fb::set_error(FB_ERR_ARG, "gemm_tc: tensor map rejected (alignment or stride)");
  return FB_OK;
}

int32_t *tc_err_word() {
  static int32_t *w[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!w[dev]) {
    cudaMalloc(&w[dev], 4);
    cudaMemset(w[dev], 0, 4);
  }
  return w[dev];
}

template <int BN>
int launch_tc(const CUtensorMap &ma, const CUtensorMap &mb, const float *bias, float *C, int64_t ldc, int64_t M,
              const int32_t *M_dev, int N, int K, int accumulate, cudaStream_t stream) {
  using CF = Cfg<BN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    FB_TRY_CUDA(cudaFuncSetAttribute(k_gemm_nt_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  k_gemm_nt_tc<BN><<<grid, kThreadsTc, CF::kSmem, stream>>>(ma, mb, bias, C, ldc, M, M_dev, N, K, accumulate,
                                                             tc_err_word());
  FB_LAUNCHED("k_gemm_nt_tc");
  return FB_OK;
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fb_gemm_nt_tc_supported(const float *A, int64_t lda, const float *B, int64_t ldb, int N, int K) {
  return A && B && N >= 1 && N <= 256 && K >= 1 && K % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 && al16(A) &&
         al16(B) && encode_fn() != nullptr;
}

extern "C" int fb_gemm_nt_tc(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C,
                             int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K, int accumulate,
                             cudaStream_t stream) {
  if (!C || M < 0 || ldc < N || !fb_gemm_nt_tc_supported(A, lda, B, ldb, N, K))
    return fb::set_error(FB_ERR_UNSUPPORTED,
                         "gemm_nt_tc: needs N <= 256, K, lda, ldb multiples of 4 and 16-byte aligned A, B");
  if (M == 0) return FB_OK;
  // N tiles of at most 128 columns (two slice accumulators fit TMEM, and the
  // fp32 promotion sums fit the registers of one thread per row)
  const int BNr = N <= 64 ? 64 : (N <= 112 ? 112 : (N <= 128 ? 128 : (N <= 224 ? 112 : 128)));
  CUtensorMap ma, mb;
  int rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, B, N, K, ldb, BNr);
  if (rc) return rc;
  switch (BNr) {
    case 64: return launch_tc<64>(ma, mb, bias, C, ldc, M, M_dev, N, K, accumulate, stream);
    case 112: return launch_tc<112>(ma, mb, bias, C, ldc, M, M_dev, N, K, accumulate, stream);
    default: return launch_tc<128>(ma, mb, bias, C, ldc, M, M_dev, N, K, accumulate, stream);
  }
}

extern "C" int fb_gemm_tc_error(int *flags, int clear) {
  if (!flags) return fb::set_error(FB_ERR_ARG, "gemm_tc_error: null");
  int32_t *w = tc_err_word();
  FB_TRY_CUDA(cudaMemcpy(flags, w, 4, cudaMemcpyDeviceToHost));
  if (clear) FB_TRY_CUDA(cudaMemset(w, 0, 4));
  return FB_OK;
}
