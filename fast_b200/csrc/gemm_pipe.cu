// Pipelined fp32 FFMA GEMMs for the projection path (exact fp32 products,
// fp32 accumulation).  The projection problems of a temporal-attention step
// are small (M ~ 10^3..10^5 rows, N, K ~ 10^2), so they are latency-bound:
// the kernels stream 16-deep slices of both operands into a 4-stage ring of
// shared memory with cp.async (16-byte copies, zero-filled at the edges),
// so three slices are in flight while one is multiplied, and use 64x64 tiles
// so that even ~2k-row problems spread over the SMs.
//
//   NT: C[m, n] = sum_k A[m, k] B[n, k] (+ bias[n]) (+ C)
//   NN: C[m, n] = sum_k A[m, k] B[k, n] (+ bias[n]) (+ C)
//   TN: P[s][n, k] = sum_{m in split s} G[m, n] X[m, k]   (+ a ones column of X at k = K)
//
// Each 16-deep slice is summed into a fresh register tile before it is added
// to the running tile (two-level summation: error grows with the number of
// slices, not of terms).  Shapes must have 16-byte aligned rows (leading
// dimensions and contiguous extents multiples of 4, aligned bases); the
// callers fall back to the register-staged kernels otherwise.
#include <algorithm>
#include "runtime.cuh"

namespace {

constexpr int PM = 64, PN = 64, PK = 16, PS = 4, PT = 128;

__device__ __forceinline__ void cp16(float *smem, const float *gmem, bool pred) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// One operand slice in shared memory.  KC (k-contiguous in global memory):
// [64 output rows][PK + 4]; otherwise (output-contiguous): [PK][64 + 4].
template <bool KC>
struct Tile {
  static constexpr int C = KC ? PK + 4 : PM + 4;
  static constexpr int SZ = KC ? PM * C : PK * C;
};

// Copies the slice of reduction rows/cols [k0, k0 + PK) (< klim) and output
// indices [o0, o0 + 64) (< O).  KC: global op[o * ld + k]; else op[k * ld + o].
template <bool KC>
__device__ __forceinline__ void load_slice(float *sm, const float *g, int64_t ld, int64_t o0, int64_t O, int64_t k0,
                                           int64_t klim, int tid) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int idx = tid + PT * c;                 // 256 chunks of 4 floats
    const int r = KC ? (idx >> 2) : (idx >> 4);
    const int ch = KC ? (idx & 3) : (idx & 15);
    int64_t gr, gc;
    bool ok;
    if (KC) {
      gr = o0 + r; gc = k0 + 4 * ch; ok = gr < O && gc < klim;
    } else {
      gr = k0 + r; gc = o0 + 4 * ch; ok = gr < klim && gc < O;
    }
    cp16(sm + r * Tile<KC>::C + 4 * ch, ok ? g + gr * ld + gc : g, ok);
  }
}

// acc[i][j] += sum over the slice of A(oa_i, k) B(ob_j, k), with
// oa_i = ty*8 + i and ob_j = BKC ? tx + 16 j : tx*4 + j.
template <bool AKC, bool BKC>
__device__ __forceinline__ void slice_fma(float (&acc)[8][4], const float *As, const float *Bs, int ty, int tx) {
  float sl[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) sl[i][j] = 0.f;
#pragma unroll
  for (int kk = 0; kk < PK; kk += 4) {
    float a[8][4], b[4][4];
    if (AKC) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(As + (ty * 8 + i) * Tile<true>::C + kk);
        a[i][0] = v.x; a[i][1] = v.y; a[i][2] = v.z; a[i][3] = v.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v0 = *reinterpret_cast<const float4 *>(As + (kk + q) * Tile<false>::C + ty * 8);
        const float4 v1 = *reinterpret_cast<const float4 *>(As + (kk + q) * Tile<false>::C + ty * 8 + 4);
        a[0][q] = v0.x; a[1][q] = v0.y; a[2][q] = v0.z; a[3][q] = v0.w;
        a[4][q] = v1.x; a[5][q] = v1.y; a[6][q] = v1.z; a[7][q] = v1.w;
      }
    }
    if (BKC) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v = *reinterpret_cast<const float4 *>(Bs + (tx + 16 * j) * Tile<true>::C + kk);
        b[j][0] = v.x; b[j][1] = v.y; b[j][2] = v.z; b[j][3] = v.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = *reinterpret_cast<const float4 *>(Bs + (kk + q) * Tile<false>::C + tx * 4);
        b[0][q] = v.x; b[1][q] = v.y; b[2][q] = v.z; b[3][q] = v.w;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sl[i][j] = fmaf(a[i][q], b[j][q], sl[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] += sl[i][j];
}

struct PGemm {
  const float *A; int64_t lda; const float *B; int64_t ldb; const float *bias; float *C; int64_t ldc;
  int64_t M; const int32_t *M_dev; int N; int K; int accumulate;
};

// NT (BKC = true: B stored [N, K]) and NN (BKC = false: B stored [K, N]).
// Grid: x = N tiles, y strides over M tiles (M may be a device-side count).
template <bool BKC>
__global__ void __launch_bounds__(PT) k_pgemm(PGemm a) {
  __shared__ __align__(16) float As[PS][Tile<true>::SZ];
  __shared__ __align__(16) float Bs[PS][Tile<BKC>::SZ];
  const int64_t M = a.M_dev ? min((int64_t)(*a.M_dev), a.M) : a.M;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t n0 = (int64_t)blockIdx.x * PN;
  const int nk = (a.K + PK - 1) / PK;
  for (int64_t m0 = (int64_t)blockIdx.y * PM; m0 < M; m0 += (int64_t)gridDim.y * PM) {
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll
    for (int s = 0; s < PS - 1; ++s) {
      if (s < nk) {
        load_slice<true>(As[s], a.A, a.lda, m0, M, (int64_t)s * PK, a.K, tid);
        load_slice<BKC>(Bs[s], a.B, a.ldb, n0, a.N, (int64_t)s * PK, a.K, tid);
      }
      cp_commit();
    }
    for (int t = 0; t < nk; ++t) {
      cp_wait<PS - 2>();
      __syncthreads();
      const int tn = t + PS - 1;
      if (tn < nk) {
        load_slice<true>(As[tn % PS], a.A, a.lda, m0, M, (int64_t)tn * PK, a.K, tid);
        load_slice<BKC>(Bs[tn % PS], a.B, a.ldb, n0, a.N, (int64_t)tn * PK, a.K, tid);
      }
      cp_commit();
      slice_fma<true, BKC>(acc, As[t % PS], Bs[t % PS], ty, tx);
    }
    cp_wait<0>();
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t m = m0 + ty * 8 + i;
      if (m >= M) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + (BKC ? tx + 16 * j : tx * 4 + j);
        if (n < a.N) {
          float v = acc[i][j];
          if (a.bias) v += a.bias[n];
          float *c = a.C + m * a.ldc + n;
          *c = a.accumulate ? (*c + v) : v;
        }
      }
    }
  }
}

struct PTn {
  const float *G; int64_t ldg; const float *X; int64_t ldx; float *P; int64_t ldp;
  int64_t M; const int32_t *M_dev; int N; int K; int max_splits; int64_t rows_min; bool ones;
};

// TN partials: grid x = output-column tiles (K, + 1 with the ones column),
// y = N tiles, z = splits of the m reduction (count-determined).
__global__ void __launch_bounds__(PT) k_ptn(PTn a) {
  __shared__ __align__(16) float Gs[PS][Tile<false>::SZ];
  __shared__ __align__(16) float Xs[PS][Tile<false>::SZ];
  const int64_t M = a.M_dev ? min((int64_t)(*a.M_dev), a.M) : a.M;
  const int ns = fb::split_parts(M, a.rows_min, a.max_splits);
  if ((int)blockIdx.z >= ns) return;
  const int64_t per = ((M + ns - 1) / ns + PK - 1) / PK * PK;
  const int64_t s0 = (int64_t)blockIdx.z * per, s1 = min(M, s0 + per);
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t n0 = (int64_t)blockIdx.y * PM, k0 = (int64_t)blockIdx.x * PN;
  const bool fix = a.ones && k0 <= a.K && a.K < k0 + PN;     // this tile holds the ones column
  const int nk = s1 > s0 ? (int)((s1 - s0 + PK - 1) / PK) : 0;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll
  for (int s = 0; s < PS - 1; ++s) {
    if (s < nk) {
      load_slice<false>(Gs[s], a.G, a.ldg, n0, a.N, s0 + (int64_t)s * PK, s1, tid);
      load_slice<false>(Xs[s], a.X, a.ldx, k0, a.K, s0 + (int64_t)s * PK, s1, tid);
    }
    cp_commit();
  }
  for (int t = 0; t < nk; ++t) {
    cp_wait<PS - 2>();
    __syncthreads();
    if (fix) {
      if (tid < PK) Xs[t % PS][tid * Tile<false>::C + (int)(a.K - k0)] = (s0 + (int64_t)t * PK + tid < s1) ? 1.f : 0.f;
      __syncthreads();
    }
    const int tn = t + PS - 1;
    if (tn < nk) {
      load_slice<false>(Gs[tn % PS], a.G, a.ldg, n0, a.N, s0 + (int64_t)tn * PK, s1, tid);
      load_slice<false>(Xs[tn % PS], a.X, a.ldx, k0, a.K, s0 + (int64_t)tn * PK, s1, tid);
    }
    cp_commit();
    slice_fma<false, false>(acc, Gs[t % PS], Xs[t % PS], ty, tx);
  }
  cp_wait<0>();
  const int Kout = a.K + (a.ones ? 1 : 0);
  float *out = a.P + (int64_t)blockIdx.z * a.N * a.ldp;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t n = n0 + ty * 8 + i;
    if (n >= a.N) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + tx * 4 + j;
      if (k < Kout) out[n * a.ldp + k] = acc[i][j];
    }
  }
}

inline bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace fb {

// True when the pipelined kernels can take the shape (16-byte rows).
bool pgemm_ok(const float *A, int64_t lda, const float *B, int64_t ldb, int N, int K, bool b_kn) {
  return a16(A) && a16(B) && lda % 4 == 0 && ldb % 4 == 0 && K % 4 == 0 && (!b_kn || N % 4 == 0);
}

int pgemm_launch(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C, int64_t ldc,
                 int64_t M, const int32_t *M_dev, int N, int K, int accumulate, bool b_kn, cudaStream_t stream) {
  PGemm a{A, lda, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate};
  const int64_t mt = (M + PM - 1) / PM;
  const int nt = (N + PN - 1) / PN;
  dim3 grid(nt, (unsigned)std::min<int64_t>(mt, std::max<int64_t>(1, 148 * 5 / nt)));
  if (b_kn) k_pgemm<false><<<grid, PT, 0, stream>>>(a);
  else k_pgemm<true><<<grid, PT, 0, stream>>>(a);
  FB_LAUNCHED(b_kn ? "k_pgemm_nn" : "k_pgemm_nt");
  return FB_OK;
}

bool ptn_ok(const float *G, int64_t ldg, const float *X, int64_t ldx, int N, int K) {
  return a16(G) && a16(X) && ldg % 4 == 0 && ldx % 4 == 0 && N % 4 == 0 && K % 4 == 0;
}

// Most splits of the m reduction: enough CTAs to cover the SMs ~4 times.
int ptn_max_splits(int N, int Kp) {
  const int64_t tiles = (int64_t)((N + PM - 1) / PM) * ((Kp + PN - 1) / PN);
  return (int)std::max<int64_t>(1, (148 * 4) / std::max<int64_t>(tiles, 1));
}

int ptn_launch(const float *G, int64_t ldg, const float *X, int64_t ldx, float *P, int64_t M, const int32_t *M_dev,
               int N, int K, bool ones, int max_splits, int64_t rows_min, cudaStream_t stream) {
  const int Kp = K + (ones ? 1 : 0);
  PTn a{G, ldg, X, ldx, P, Kp, M, M_dev, N, K, max_splits, rows_min, ones};
  const int ns = fb::split_parts(M, rows_min, max_splits);
  dim3 grid((Kp + PN - 1) / PN, (N + PM - 1) / PM, ns);
  k_ptn<<<grid, PT, 0, stream>>>(a);
  FB_LAUNCHED("k_ptn");
  return FB_OK;
}

}  // namespace fb
