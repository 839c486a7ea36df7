// fp32 projection GEMMs on the CUDA cores (FFMA), exact fp32 arithmetic.
//   NT: C[m,n] = sum_k A[m,k] B[n,k] + bias[n]      (nn.Linear forward / dX)
//   TN: C[n,k] = sum_m G[m,n] X[m,k]                 (nn.Linear weight grad)
// 128x64 CTA tiles, 16-deep k slices staged through shared memory with a
// register prefetch of the next slice, 8x4 outputs per thread.  The TN form
// splits the long m reduction over CTAs and sums the partials in a fixed
// order, so every result is deterministic.
#include <algorithm>
#include "runtime.cuh"

namespace {

constexpr int BM = 128, BN = 64, BK = 16, PAD = 4, NT = 256;

__device__ __forceinline__ void tile_fma(float (&acc)[8][4], const float (*As)[BM + PAD], const float (*Bs)[BN + PAD],
                                         int ty, int tx) {
#pragma unroll
  for (int kk = 0; kk < BK; ++kk) {
    float4 a0 = *reinterpret_cast<const float4 *>(&As[kk][ty * 8]);
    float4 a1 = *reinterpret_cast<const float4 *>(&As[kk][ty * 8 + 4]);
    float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
    float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

__device__ __forceinline__ float4 ld4_guard(const float *p, int64_t row, int64_t nrows, int col, int ncols, int64_t ld,
                                            bool vec) {
  if (row >= nrows) return make_float4(0.f, 0.f, 0.f, 0.f);
  const float *q = p + row * ld + col;
  if (vec && col + 3 < ncols) return __ldg(reinterpret_cast<const float4 *>(q));
  float4 r;
  r.x = (col + 0 < ncols) ? __ldg(q + 0) : 0.f;
  r.y = (col + 1 < ncols) ? __ldg(q + 1) : 0.f;
  r.z = (col + 2 < ncols) ? __ldg(q + 2) : 0.f;
  r.w = (col + 3 < ncols) ? __ldg(q + 3) : 0.f;
  return r;
}

// C[M,N] = A[M,K] * B[N,K]^T       (BKN = false: B stored [N, K])
// C[M,N] = A[M,K] * B[K,N]         (BKN = true:  B stored [K, N])
template <bool BKN>
__global__ void __launch_bounds__(NT) k_gemm_nt(const float *__restrict__ A, int64_t lda, const float *__restrict__ B,
                                                int64_t ldb, const float *__restrict__ bias, float *__restrict__ C,
                                                int64_t ldc, int64_t M_host, const int32_t *M_dev, int N, int K,
                                                int accumulate, bool vecA, bool vecB) {
  __shared__ __align__(16) float As[2][BK][BM + PAD];
  __shared__ __align__(16) float Bs[2][BK][BN + PAD];
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int n0 = blockIdx.x * BN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  for (int64_t m0 = (int64_t)blockIdx.y * BM; m0 < M; m0 += (int64_t)gridDim.y * BM) {
  float acc[8][4] = {};
  // loader coordinates: A 128x16 = 512 float4 (2 per thread), B 64x16 = 256 float4
  const int ar0 = tid >> 2, ac = (tid & 3) * 4;  // rows ar0 and ar0 + 64
  // B [N,K]: 64 rows x 16 k, one float4 along k per thread;
  // B [K,N]: 16 k-rows x 64 n, one float4 along n per thread
  const int br = BKN ? (tid >> 4) : (tid >> 2), bc = BKN ? (tid & 15) * 4 : (tid & 3) * 4;
  float4 ra0, ra1, rb;
  auto load = [&](int k0) {
    ra0 = ld4_guard(A, m0 + ar0, M, k0 + ac, K, lda, vecA);
    ra1 = ld4_guard(A, m0 + ar0 + 64, M, k0 + ac, K, lda, vecA);
    if (BKN) rb = ld4_guard(B, k0 + br, K, n0 + bc, N, ldb, vecB);
    else rb = ld4_guard(B, n0 + br, N, k0 + bc, K, ldb, vecB);
  };
  auto stash = [&](int buf) {
    As[buf][ac + 0][ar0] = ra0.x; As[buf][ac + 1][ar0] = ra0.y;
    As[buf][ac + 2][ar0] = ra0.z; As[buf][ac + 3][ar0] = ra0.w;
    As[buf][ac + 0][ar0 + 64] = ra1.x; As[buf][ac + 1][ar0 + 64] = ra1.y;
    As[buf][ac + 2][ar0 + 64] = ra1.z; As[buf][ac + 3][ar0 + 64] = ra1.w;
    if (BKN) {
      *reinterpret_cast<float4 *>(&Bs[buf][br][bc]) = rb;
    } else {
      Bs[buf][bc + 0][br] = rb.x; Bs[buf][bc + 1][br] = rb.y;
      Bs[buf][bc + 2][br] = rb.z; Bs[buf][bc + 3][br] = rb.w;
    }
  };
  const int nk = (K + BK - 1) / BK;
  load(0);
  stash(0);
  __syncthreads();
  for (int t = 0; t < nk; ++t) {
    const int buf = t & 1;
    if (t + 1 < nk) load((t + 1) * BK);
    tile_fma(acc, As[buf], Bs[buf], ty, tx);
    if (t + 1 < nk) stash(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + ty * 8 + i;
    if (m >= M) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) {
        float v = acc[i][j];
        if (bias) v += bias[n];
        float *c = C + m * ldc + n;
        *c = accumulate ? (*c + v) : v;
      }
    }
  }
  __syncthreads();
  }
}

constexpr int64_t kTnRowsMin = 256;      // rows per TN split, at least
constexpr int64_t kColsumRows = 256;
constexpr int64_t kColsumMaxParts = 148;

// P[split][N][K] = sum_{m in split} G[m,n] X[m,k]
// With ones = true, X carries a virtual column of ones at k = K, so output
// column K of P holds sum_m G[m,n] (the bias gradient).
__global__ void __launch_bounds__(NT) k_gemm_tn(const float *__restrict__ G, int64_t ldg, const float *__restrict__ X,
                                                int64_t ldx, float *__restrict__ P, int64_t ldp, int64_t M_host,
                                                const int32_t *M_dev, int N, int K, int max_splits,
                                                bool vecG, bool vecX, bool ones) {
  __shared__ __align__(16) float Gs[2][BK][BM + PAD];
  __shared__ __align__(16) float Xs[2][BK][BN + PAD];
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int n0 = blockIdx.y * BM, k0 = blockIdx.x * BN;
  // the partition comes from the true row count, not from the launch
  const int ns = fb::tn_parts(M, kTnRowsMin, max_splits);
  if ((int)blockIdx.z >= ns) return;
  const int64_t per = ((M + ns - 1) / ns + BK - 1) / BK * BK;
  const int64_t s0 = (int64_t)blockIdx.z * per;
  const int64_t s1 = min(M, s0 + per);
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float acc[8][4] = {};
  // loader: G slice 16 x 128 (2 float4 per thread), X slice 16 x 64 (1 float4)
  const int gr = tid >> 5, gc = (tid & 31) * 4;  // rows gr and gr + 8
  const int xr = tid >> 4, xc = (tid & 15) * 4;
  float4 rg0, rg1, rx;
  auto load = [&](int64_t m) {
    rg0 = ld4_guard(G, m + gr, s1, n0 + gc, N, ldg, vecG);
    rg1 = ld4_guard(G, m + gr + 8, s1, n0 + gc, N, ldg, vecG);
    rx = ld4_guard(X, m + xr, s1, k0 + xc, K, ldx, vecX);
    if (ones && m + xr < s1) {
      const int j = K - (k0 + xc);
      if (j == 0) rx.x = 1.f;
      else if (j == 1) rx.y = 1.f;
      else if (j == 2) rx.z = 1.f;
      else if (j == 3) rx.w = 1.f;
    }
  };
  auto stash = [&](int buf) {
    *reinterpret_cast<float4 *>(&Gs[buf][gr][gc]) = rg0;
    *reinterpret_cast<float4 *>(&Gs[buf][gr + 8][gc]) = rg1;
    *reinterpret_cast<float4 *>(&Xs[buf][xr][xc]) = rx;
  };
  if (s0 < s1) {
    const int64_t nt = (s1 - s0 + BK - 1) / BK;
    load(s0);
    stash(0);
    __syncthreads();
    for (int64_t t = 0; t < nt; ++t) {
      const int buf = (int)(t & 1);
      if (t + 1 < nt) load(s0 + (t + 1) * BK);
      tile_fma(acc, Gs[buf], Xs[buf], ty, tx);
      if (t + 1 < nt) stash(buf ^ 1);
      __syncthreads();
    }
  }
  float *out = P + (int64_t)blockIdx.z * N * ldp;
  const int Kout = K + (ones ? 1 : 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int n = n0 + ty * 8 + i;
    if (n >= N) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + tx * 4 + j;
      if (k < Kout) out[(int64_t)n * ldp + k] = acc[i][j];
    }
  }
}

// Sums the splits in order.  P rows hold Kp = K (+1 with a bias column)
// values; column K goes to db.
__global__ void k_split_reduce(const float *__restrict__ P, int64_t M_host, const int32_t *M_dev, int max_splits,
                               int N, int K, int Kp, float *__restrict__ C, int64_t ldc, int accumulate,
                               float *__restrict__ db, int db_accumulate) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)N * Kp) return;
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int nsplit = fb::tn_parts(M, kTnRowsMin, max_splits);
  const int n = (int)(i / Kp), k = (int)(i % Kp);
  float s = 0.f;
  for (int p = 0; p < nsplit; ++p) s += P[(int64_t)p * N * Kp + i];
  float *c = (k < K) ? C + (int64_t)n * ldc + k : db + n;
  const int acc = (k < K) ? accumulate : db_accumulate;
  *c = acc ? (*c + s) : s;
}

// Column sums, stage 1: CTA (x = 32-column tile, y = row chunk), 8 warps
// striding over rows, lanes over columns, warp sums combined in fixed order.
__global__ void __launch_bounds__(256) k_colsum_part(const float *__restrict__ G, int64_t ldg, int64_t M_host,
                                                     const int32_t *M_dev, int N, float *__restrict__ part) {
  __shared__ float s_acc[8][32];
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int parts = fb::split_parts(M, kColsumRows, kColsumMaxParts);
  if ((int)blockIdx.y >= parts) return;
  const int64_t per = (M + parts - 1) / parts;
  const int64_t r0 = (int64_t)blockIdx.y * per, r1 = min(M, r0 + per);
  float s = 0.f;
  if (c < N)
    for (int64_t r = r0 + wp; r < r1; r += 8) s += G[r * ldg + c];
  s_acc[wp][lane] = s;
  __syncthreads();
  if (wp == 0 && c < N) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a += s_acc[i][lane];
    part[(int64_t)blockIdx.y * N + c] = a;
  }
}

// One warp per column over the partials, fixed shuffle tree (deterministic).
__global__ void k_colsum_reduce(const float *__restrict__ part, int64_t M_host, const int32_t *M_dev, int N,
                                float *db, int accumulate) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (c >= N) return;
  const int64_t M = M_dev ? min((int64_t)(*M_dev), M_host) : M_host;
  const int nparts = fb::split_parts(M, kColsumRows, kColsumMaxParts);
  float s = 0.f;
  for (int p = lane; p < nparts; p += 32) s += part[(int64_t)p * N + c];
  s = fb::warp_sum(s);
  if (lane == 0) db[c] = accumulate ? db[c] + s : s;
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace fb {
bool pgemm_ok(const float *A, int64_t lda, const float *B, int64_t ldb, int N, int K, bool b_kn);
int pgemm_launch(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C, int64_t ldc,
                 int64_t M, const int32_t *M_dev, int N, int K, int accumulate, bool b_kn, cudaStream_t stream);
bool ptn_ok(const float *G, int64_t ldg, const float *X, int64_t ldx, int N, int K);
int ptn_max_splits(int N, int Kp);
int ptn_launch(const float *G, int64_t ldg, const float *X, int64_t ldx, float *P, int64_t M, const int32_t *M_dev,
               int N, int K, bool ones, int max_splits, int64_t rows_min, cudaStream_t stream);
}  // namespace fb

namespace {

// Most splits of the TN GEMM's m reduction: enough to fill the machine with
// output tiles.  Each split covers at least kTnRowsMin rows.
inline int tn_max_splits(int N, int K) {
  const int64_t tiles = (int64_t)((N + BM - 1) / BM) * ((K + BN - 1) / BN);
  return (int)std::max<int64_t>(1, (148 * 4) / std::max<int64_t>(tiles, 1));
}

inline int colsum_parts(int64_t M) { return fb::split_parts(M, kColsumRows, kColsumMaxParts); }

}  // namespace

extern "C" int fb_gemm_nt(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C,
                          int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K, int accumulate,
                          cudaStream_t stream) {
  if (!A || !B || !C || M < 0 || N < 1 || K < 1 || lda < K || ldb < K || ldc < N)
    return fb::set_error(FB_ERR_ARG, "gemm_nt: bad argument");
  if (M == 0) return FB_OK;
  if (fb::pgemm_ok(A, lda, B, ldb, N, K, false))
    return fb::pgemm_launch(A, lda, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate, false, stream);
  const bool vecA = (lda % 4 == 0) && al16(A), vecB = (ldb % 4 == 0) && al16(B);
  const int64_t mt = (M + BM - 1) / BM;
  const int nt = (N + BN - 1) / BN;
  dim3 grid(nt, (unsigned)std::min<int64_t>(mt, std::max<int64_t>(1, 148 * 4 / nt)));
  k_gemm_nt<false><<<grid, NT, 0, stream>>>(A, lda, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate, vecA, vecB);
  FB_LAUNCHED("k_gemm_nt");
  return FB_OK;
}

extern "C" int fb_gemm_nn(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C,
                          int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K, int accumulate,
                          cudaStream_t stream) {
  if (!A || !B || !C || M < 0 || N < 1 || K < 1 || lda < K || ldb < N || ldc < N)
    return fb::set_error(FB_ERR_ARG, "gemm_nn: bad argument");
  if (M == 0) return FB_OK;
  if (fb::pgemm_ok(A, lda, B, ldb, N, K, true))
    return fb::pgemm_launch(A, lda, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate, true, stream);
  const bool vecA = (lda % 4 == 0) && al16(A), vecB = (ldb % 4 == 0) && al16(B);
  const int64_t mt = (M + BM - 1) / BM;
  const int nt = (N + BN - 1) / BN;
  dim3 grid(nt, (unsigned)std::min<int64_t>(mt, std::max<int64_t>(1, 148 * 4 / nt)));
  k_gemm_nt<true><<<grid, NT, 0, stream>>>(A, lda, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate, vecA, vecB);
  FB_LAUNCHED("k_gemm_nn");
  return FB_OK;
}

extern "C" size_t fb_gemm_tn_ws_bytes(int64_t M, int N, int K) {
  // room for either kernel family, with or without the bias column
  int64_t most = 0;
  for (int Kp = K; Kp <= K + 1; ++Kp) {
    const int64_t a = fb::tn_parts(M, kTnRowsMin, tn_max_splits(N, Kp));
    const int64_t b = fb::tn_parts(M, kTnRowsMin, fb::ptn_max_splits(N, Kp));
    most = std::max(most, std::max(a, b) * (int64_t)N * Kp);
  }
  return (size_t)most * sizeof(float);
}

extern "C" int fb_gemm_tn_bias(const float *G, int64_t ldg, const float *X, int64_t ldx, float *C, int64_t ldc,
                               int64_t M, const int32_t *M_dev, int N, int K, int accumulate, float *db,
                               int db_accumulate, void *ws, cudaStream_t stream) {
  if (!G || !X || !C || !ws || M < 0 || N < 1 || K < 1 || ldg < N || ldx < K || ldc < K)
    return fb::set_error(FB_ERR_ARG, "gemm_tn: bad argument");
  const bool ones = db != nullptr;
  const int Kp = K + (ones ? 1 : 0);
  float *P = static_cast<float *>(ws);
  // launched for M (a capacity when M_dev is given); the kernels take the
  // partition from the true row count
  const bool pipe = fb::ptn_ok(G, ldg, X, ldx, N, K);
  const int max_splits = pipe ? fb::ptn_max_splits(N, Kp) : tn_max_splits(N, Kp);
  if (pipe) {
    const int rc = fb::ptn_launch(G, ldg, X, ldx, P, M, M_dev, N, K, ones, max_splits, kTnRowsMin, stream);
    if (rc != FB_OK) return rc;
  } else {
    const int ns = fb::tn_parts(M, kTnRowsMin, max_splits);
    const bool vecG = (ldg % 4 == 0) && al16(G), vecX = (ldx % 4 == 0) && al16(X);
    dim3 grid((Kp + BN - 1) / BN, (N + BM - 1) / BM, ns);
    k_gemm_tn<<<grid, NT, 0, stream>>>(G, ldg, X, ldx, P, Kp, M, M_dev, N, K, max_splits, vecG, vecX, ones);
    FB_LAUNCHED("k_gemm_tn");
  }
  const int64_t tot = (int64_t)N * Kp;
  k_split_reduce<<<(unsigned)((tot + 255) / 256), 256, 0, stream>>>(P, M, M_dev, max_splits, N, K, Kp, C, ldc,
                                                                      accumulate, db, db_accumulate);
  FB_LAUNCHED("k_split_reduce");
  return FB_OK;
}

extern "C" int fb_gemm_tn(const float *G, int64_t ldg, const float *X, int64_t ldx, float *C, int64_t ldc, int64_t M,
                          const int32_t *M_dev, int N, int K, int accumulate, void *ws, cudaStream_t stream) {
  return fb_gemm_tn_bias(G, ldg, X, ldx, C, ldc, M, M_dev, N, K, accumulate, nullptr, 0, ws, stream);
}

extern "C" size_t fb_colsum_ws_bytes(int64_t M, int N) {
  const int64_t parts = colsum_parts(M);
  return (size_t)(parts * std::max(N, 1)) * sizeof(float);
}

extern "C" int fb_colsum(const float *G, int64_t ldg, float *db, int64_t M, const int32_t *M_dev, int N,
                         int accumulate, void *ws, cudaStream_t stream) {
  if (!G || !db || !ws || M < 0 || N < 1 || ldg < N) return fb::set_error(FB_ERR_ARG, "colsum: bad argument");
  const int parts = colsum_parts(M);
  float *part = static_cast<float *>(ws);
  dim3 grid((N + 31) / 32, parts);
  k_colsum_part<<<grid, 256, 0, stream>>>(G, ldg, M, M_dev, N, part);
  FB_LAUNCHED("k_colsum_part");
  k_colsum_reduce<<<(N * 32 + 255) / 256, 256, 0, stream>>>(part, M, M_dev, N, db, accumulate);
  FB_LAUNCHED("k_colsum_reduce");
  return FB_OK;
}
