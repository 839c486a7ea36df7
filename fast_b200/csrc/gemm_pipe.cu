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
// slices, not of terms); the long TN reductions add a third level, every 16
// slices into a block total.  Shapes must have 16-byte aligned rows (leading
// dimensions and contiguous extents multiples of 4, aligned bases); the
// callers fall back to the register-staged kernels otherwise.
#include <algorithm>
#include <vector>
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

// A operand of NT/NN: A [M, K] row-major, or the concatenation along K of
// A (columns < k1) and A2 (columns >= k1, at A2[m * lda2 + k - k1]).
struct PGemm {
  const float *A; int64_t lda; const float *A2; int64_t lda2; int k1;
  const float *B; int64_t ldb; const float *bias; float *C; int64_t ldc;
  int64_t M; const int32_t *M_dev; int N; int K; int accumulate;
};

__device__ __forceinline__ void load_a_slice(float *sm, const PGemm &a, int64_t m0, int64_t M, int64_t k0, int tid) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int idx = tid + PT * c;
    const int r = idx >> 2, ch = idx & 3;
    const int64_t gr = m0 + r, gc = k0 + 4 * ch;
    const bool ok = gr < M && gc < a.K;
    const float *src = a.A;
    if (ok) src = gc < a.k1 ? a.A + gr * a.lda + gc : a.A2 + gr * a.lda2 + (gc - a.k1);
    cp16(sm + r * Tile<true>::C + 4 * ch, src, ok);
  }
}

// One output tile column (n0) of NT (BKC) / NN, over the m tiles
// m_slot, m_slot + m_slots, ... below the (device-side) row count.
template <bool BKC>
__device__ __forceinline__ void pgemm_body(const PGemm &a, float (*As)[Tile<true>::SZ], float (*Bs)[Tile<true>::SZ],
                                           int64_t n0, int64_t m_slot, int64_t m_slots) {
  const int64_t M = a.M_dev ? min((int64_t)(*a.M_dev), a.M) : a.M;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nk = (a.K + PK - 1) / PK;
  for (int64_t m0 = m_slot * PM; m0 < M; m0 += m_slots * PM) {
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll
    for (int s = 0; s < PS - 1; ++s) {
      if (s < nk) {
        load_a_slice(As[s], a, m0, M, (int64_t)s * PK, tid);
        load_slice<BKC>(Bs[s], a.B, a.ldb, n0, a.N, (int64_t)s * PK, a.K, tid);
      }
      cp_commit();
    }
    for (int t = 0; t < nk; ++t) {
      cp_wait<PS - 2>();
      __syncthreads();
      const int tn = t + PS - 1;
      if (tn < nk) {
        load_a_slice(As[tn % PS], a, m0, M, (int64_t)tn * PK, tid);
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

// NT (BKC = true: B stored [N, K]) and NN (BKC = false: B stored [K, N]).
// Grid: x = N tiles, y strides over M tiles (M may be a device-side count).
template <bool BKC>
__global__ void __launch_bounds__(PT) k_pgemm(PGemm a) {
  __shared__ __align__(16) float As[PS][Tile<true>::SZ];
  __shared__ __align__(16) float Bs[PS][Tile<true>::SZ];
  pgemm_body<BKC>(a, As, Bs, (int64_t)blockIdx.x * PN, blockIdx.y, gridDim.y);
}

struct PTn {
  const float *G; int64_t ldg; const float *X; int64_t ldx; float *P; int64_t ldp;
  int64_t M; const int32_t *M_dev; int N; int K; int max_splits; int64_t rows_min; bool ones;
};

// TN partial tile (k0 output columns, n0 output rows) of split z.
__device__ __forceinline__ void ptn_body(const PTn &a, float (*Gs)[Tile<true>::SZ], float (*Xs)[Tile<true>::SZ],
                                         int64_t k0, int64_t n0, int z) {
  const int64_t M = a.M_dev ? min((int64_t)(*a.M_dev), a.M) : a.M;
  const int ns = fb::tn_parts(M, a.rows_min, a.max_splits);
  if (z >= ns) return;
  const int64_t per = ((M + ns - 1) / ns + PK - 1) / PK * PK;
  const int64_t s0 = (int64_t)z * per, s1 = min(M, s0 + per);
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const bool fix = a.ones && k0 <= a.K && a.K < k0 + PN;     // this tile holds the ones column
  const int nk = s1 > s0 ? (int)((s1 - s0 + PK - 1) / PK) : 0;
  // three-level sum: 16-row slices into acc, acc into tot every 16 slices
  float acc[8][4], tot[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = tot[i][j] = 0.f;
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
    if ((t & 15) == 15) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) tot[i][j] += acc[i][j], acc[i][j] = 0.f;
    }
  }
  cp_wait<0>();
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] += tot[i][j];
  const int Kout = a.K + (a.ones ? 1 : 0);
  float *out = a.P + (int64_t)z * a.N * a.ldp;
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

// TN partials: grid x = output-column tiles (K, + 1 with the ones column),
// y = N tiles, z = splits of the m reduction (count-determined).
__global__ void __launch_bounds__(PT) k_ptn(PTn a) {
  __shared__ __align__(16) float Gs[PS][Tile<true>::SZ];
  __shared__ __align__(16) float Xs[PS][Tile<true>::SZ];
  ptn_body(a, Gs, Xs, (int64_t)blockIdx.x * PN, (int64_t)blockIdx.y * PM, blockIdx.z);
}

// ---------------------------------------------------------------------------
// Grouped launch: independent NT / NN / TN problems share one grid.  CTA b
// belongs to the problem p with start[p] <= b < start[p + 1].

constexpr int kMaxGroup = 12;

struct GroupProb {
  int kind;                    // 0 NT, 1 NN, 2 TN
  PGemm g;                     // NT / NN
  PTn t;                       // TN
  int nt, mslots;              // NT / NN: N tiles, M slots
  int kt, ntn;                 // TN: output-column tiles, N tiles (splits = t.max_splits)
  float *C; int64_t ldc; float *db; int accumulate, db_accumulate;   // TN outputs
};

struct GroupArgs {
  GroupProb p[kMaxGroup];
  int start[kMaxGroup + 1];
  int n;
  int red_start[kMaxGroup + 1];  // TN problems: reduction blocks
};

__global__ void __launch_bounds__(PT) k_gemm_group(const __grid_constant__ GroupArgs ga) {
  fb::pdl_enter();
  __shared__ __align__(16) float As[PS][Tile<true>::SZ];
  __shared__ __align__(16) float Bs[PS][Tile<true>::SZ];
  int p = 0;
  while (p + 1 < ga.n && (int)blockIdx.x >= ga.start[p + 1]) ++p;
  const GroupProb &q = ga.p[p];
  const int local = (int)blockIdx.x - ga.start[p];
  if (q.kind == 2) {
    const int kt = local % q.kt, rest = local / q.kt;
    ptn_body(q.t, As, Bs, (int64_t)kt * PN, (int64_t)(rest % q.ntn) * PM, rest / q.ntn);
  } else {
    const int nt = local % q.nt, ms = local / q.nt;
    if (q.kind == 0) pgemm_body<true>(q.g, As, Bs, (int64_t)nt * PN, ms, q.mslots);
    else pgemm_body<false>(q.g, As, Bs, (int64_t)nt * PN, ms, q.mslots);
  }
}

// Sums the TN partials of every TN problem of the group (fixed order).
__global__ void k_group_reduce(const __grid_constant__ GroupArgs ga) {
  fb::pdl_enter();
  int p = -1;
  for (int i = 0; i < ga.n; ++i)
    if (ga.p[i].kind == 2 && (int)blockIdx.x >= ga.red_start[i] && (int)blockIdx.x < ga.red_start[i + 1]) p = i;
  if (p < 0) return;
  const GroupProb &q = ga.p[p];
  const int64_t i = (int64_t)(blockIdx.x - ga.red_start[p]) * blockDim.x + threadIdx.x;
  const int Kp = q.t.K + (q.t.ones ? 1 : 0);
  if (i >= (int64_t)q.t.N * Kp) return;
  const int64_t M = q.t.M_dev ? min((int64_t)(*q.t.M_dev), q.t.M) : q.t.M;
  const int nsplit = fb::tn_parts(M, q.t.rows_min, q.t.max_splits);
  const int n = (int)(i / Kp), k = (int)(i % Kp);
  float s = 0.f;
  for (int z = 0; z < nsplit; ++z) s += q.t.P[(int64_t)z * q.t.N * Kp + i];
  float *c = (k < q.t.K) ? q.C + (int64_t)n * q.ldc + k : q.db + n;
  const int acc = (k < q.t.K) ? q.accumulate : q.db_accumulate;
  *c = acc ? (*c + s) : s;
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
  PGemm a{A, lda, A, lda, K, B, ldb, bias, C, ldc, M, M_dev, N, K, accumulate};
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
  const int ns = fb::tn_parts(M, rows_min, max_splits);
  dim3 grid((Kp + PN - 1) / PN, (N + PM - 1) / PM, ns);
  k_ptn<<<grid, PT, 0, stream>>>(a);
  FB_LAUNCHED("k_ptn");
  return FB_OK;
}

}  // namespace fb

// ---------------------------------------------------------------------------
// fb_gemm_group: host side.

namespace {

constexpr int64_t kGroupRowsMin = 256;   // TN: rows per split, at least

bool problem_pipelined(const fb_gemm_problem &p) {
  if (p.kind == FB_GEMM_TN) return fb::ptn_ok(p.A, p.lda, p.B ? p.B : p.A, p.B ? p.ldb : p.lda, p.N, p.K);
  const bool two = p.A2 && p.k1 < p.K;
  if (two && (p.k1 % 4 || !a16(p.A2) || p.lda2 % 4)) return false;
  return fb::pgemm_ok(p.A, p.lda, p.B, p.ldb, p.N, p.K, p.kind == FB_GEMM_NN);
}

int64_t tn_ws_floats(const fb_gemm_problem &p) {
  const int Kp = p.K + (p.db ? 1 : 0);
  const int64_t ns = fb::tn_parts(p.M, kGroupRowsMin, fb::ptn_max_splits(p.N, Kp));
  return (ns * (int64_t)p.N * Kp + 63) / 64 * 64;
}

}  // namespace

extern "C" size_t fb_gemm_group_ws_bytes(const fb_gemm_problem *probs, int n) {
  int64_t f = 0;
  for (int i = 0; i < n; ++i)
    if (probs[i].kind == FB_GEMM_TN && probs[i].M > 0) {
      const size_t own = problem_pipelined(probs[i]) ? 0 : fb_gemm_tn_ws_bytes(probs[i].M, probs[i].N, probs[i].K);
      f += std::max({tn_ws_floats(probs[i]), (int64_t)((own + 3) / 4 + 63) / 64 * 64, fb::tc_ws_floats(probs[i])});
    }
  return (size_t)std::max<int64_t>(f, 64) * sizeof(float);
}

extern "C" int fb_gemm_group(const fb_gemm_problem *probs, int n, void *ws, size_t ws_bytes, cudaStream_t stream) {
  if (!probs || n < 0 || (n > 0 && !ws)) return fb::set_error(FB_ERR_ARG, "gemm_group: bad argument");
  if (ws_bytes < fb_gemm_group_ws_bytes(probs, n)) return fb::set_error(FB_ERR_ARG, "gemm_group: workspace too small");
  GroupArgs ga{};
  std::vector<int> single;                 // problems outside the pipelined shapes: launched one by one
  float *wsf = static_cast<float *>(ws);
  int64_t off = 0;
  int tiles = 0, red = 0;
  std::vector<float *> ws_of(n, nullptr);
  const bool use_tc = fb::tc_enabled();
  std::vector<const fb_gemm_problem *> tc;   // problems for the tensor cores
  std::vector<float *> tc_ws;
  for (int i = 0; i < n; ++i) {
    const fb_gemm_problem &p = probs[i];
    if (p.kind < FB_GEMM_NT || p.kind > FB_GEMM_TN || !p.A || !p.C || p.M < 0 || p.N < 1 || p.K < 0 ||
        (p.kind != FB_GEMM_TN && (!p.B || p.K < 1)) || (p.kind == FB_GEMM_TN && p.K > 0 && !p.B))
      return fb::set_error(FB_ERR_ARG, "gemm_group: bad problem");
    if (p.kind == FB_GEMM_TN && p.M > 0) {
      const size_t own = problem_pipelined(p) ? 0 : fb_gemm_tn_ws_bytes(p.M, p.N, p.K);
      ws_of[i] = wsf + off;
      off += std::max({tn_ws_floats(p), (int64_t)((own + 3) / 4 + 63) / 64 * 64, fb::tc_ws_floats(p)});
    }
    if (p.M == 0) {
      if (p.kind == FB_GEMM_TN && !p.accumulate) {   // an empty sum is zero
        for (int r = 0; r < p.N; ++r) FB_TRY_CUDA(cudaMemsetAsync(p.C + (int64_t)r * p.ldc, 0, p.K * 4, stream));
        if (p.db && !p.db_accumulate) FB_TRY_CUDA(cudaMemsetAsync(p.db, 0, p.N * 4, stream));
      }
      continue;
    }
    if (use_tc && fb::tc_problem_ok(p)) {
      tc.push_back(&probs[i]);
      tc_ws.push_back(ws_of[i]);
      continue;
    }
    if (!problem_pipelined(p) || ga.n == kMaxGroup) {
      single.push_back(i);
      continue;
    }
    GroupProb &q = ga.p[ga.n];
    q.kind = p.kind;
    q.accumulate = p.accumulate;
    q.db_accumulate = p.db_accumulate;
    q.C = p.C; q.ldc = p.ldc; q.db = p.db;
    ga.start[ga.n] = tiles;
    if (p.kind == FB_GEMM_TN) {
      const int Kp = p.K + (p.db ? 1 : 0);
      const int ms = fb::ptn_max_splits(p.N, Kp);
      q.t = PTn{p.A, p.lda, p.B ? p.B : p.A, p.B ? p.ldb : p.lda, ws_of[i], Kp, p.M, p.M_dev, p.N, p.K, ms,
                kGroupRowsMin, p.db != nullptr};
      q.kt = (Kp + PN - 1) / PN;
      q.ntn = (p.N + PM - 1) / PM;
      const int ns = fb::tn_parts(p.M, kGroupRowsMin, ms);
      tiles += q.kt * q.ntn * ns;
      ga.red_start[ga.n] = red;
      red += (int)(((int64_t)p.N * Kp + 255) / 256);
    } else {
      const bool two = p.A2 && p.k1 < p.K;
      q.g = PGemm{p.A, p.lda, two ? p.A2 : p.A, two ? p.lda2 : p.lda, two ? p.k1 : p.K, p.B, p.ldb, p.bias, p.C,
                  p.ldc, p.M, p.M_dev, p.N, p.K, p.accumulate};
      q.nt = (p.N + PN - 1) / PN;
      q.mslots = (int)std::min<int64_t>((p.M + PM - 1) / PM, std::max<int64_t>(1, 148 * 5 / q.nt));
      tiles += q.nt * q.mslots;
      ga.red_start[ga.n] = red;
    }
    ga.n++;
  }
  ga.start[ga.n] = tiles;
  ga.red_start[ga.n] = red;
  if (!tc.empty()) {
    const int rc = fb::tc_group(tc.data(), tc_ws.data(), (int)tc.size(), stream);
    if (rc != FB_OK) return rc;
  }
  if (ga.n > 0) {
    FB_TRY_CUDA(fb::launch(k_gemm_group, tiles, PT, 0, stream, ga));
    FB_LAUNCHED("k_gemm_group");
    if (red > 0) {
      FB_TRY_CUDA(fb::launch(k_group_reduce, red, 256, 0, stream, ga));
      FB_LAUNCHED("k_group_reduce");
    }
  }
  for (int i : single) {
    const fb_gemm_problem &p = probs[i];
    int rc;
    if (p.kind == FB_GEMM_TN) {
      rc = fb_gemm_tn_bias(p.A, p.lda, p.B, p.ldb, p.C, p.ldc, p.M, p.M_dev, p.N, p.K, p.accumulate, p.db,
                           p.db_accumulate, ws_of[i], stream);
    } else if (p.A2 && p.k1 < p.K) {
      return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_group: a concatenated A needs 16-byte aligned rows");
    } else if (p.kind == FB_GEMM_NT) {
      rc = fb_gemm_nt(p.A, p.lda, p.B, p.ldb, p.bias, p.C, p.ldc, p.M, p.M_dev, p.N, p.K, p.accumulate, stream);
    } else {
      rc = fb_gemm_nn(p.A, p.lda, p.B, p.ldb, p.bias, p.C, p.ldc, p.M, p.M_dev, p.N, p.K, p.accumulate, stream);
    }
    if (rc != FB_OK) return rc;
  }
  return FB_OK;
}
