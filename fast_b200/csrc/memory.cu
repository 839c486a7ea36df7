// TGN node memory on the device: the memory / mailbox gather of a block's
// source nodes fused with the memory time encoding, the GRU updater's gate
// math (forward and backward; its matrix products run as grouped GEMMs), and
// the mailbox / memory writes after a step.
//
// Reference: NoneBone/FAST memorys.py
//   MailBox.prep_input_mails      :51-73    -> k_mem_gather
//   GRUMemeoryUpdater.forward     :270-304  -> GEMMs + k_gru_fwd / k_gru_bwd
//   MailBox.update_mailbox 'self' :101-142  -> k_last_index + k_write_mail
//   MailBox.update_memory         :84-99    -> k_last_index + k_write_mem
//   TransformerMemoryUpdater      :342-385  -> k_mail_slots_gather, k_add_ln_fwd / k_add_ln_bwd
//                                              (the slot attention and the GEMMs are the shared kernels)
//   MailBox.update_mailbox 'neighbors' (APAN) :143-178 -> k_last_nbr + k_write_nbr
//
// The reference writes duplicates with index assignment (node_memory[nid] =
// memory), where the last occurrence wins on the CPU; here every write list
// first records, per node, the largest occurrence index with a 64-bit
// atomicMax of (generation << 32 | index), then only that occurrence writes.
// The generation counter lives on the device and advances after each write
// pass (the last CTA to finish bumps it), so the per-node tables never need
// clearing and replays inside a CUDA graph stay correct.
#include "runtime.cuh"

namespace {

constexpr int kRowsPerCta = 8;   // one warp per row

// x[r] = [mailbox[nid] | cos(w (ts[r] - mem_ts[nid]) + b)], h0[r] = memory[nid],
// dtm[r] = ts[r] - mem_ts[nid], for rows r < *n_dev (all n rows without it).
__global__ void __launch_bounds__(32 * kRowsPerCta)
    k_mem_gather(const int32_t *__restrict__ nodes, const float *__restrict__ ts, int64_t n, const int32_t *n_dev,
                 const float *__restrict__ memory, int dmem, const float *__restrict__ mem_ts,
                 const float *__restrict__ mailbox, int dmail, const float *__restrict__ w,
                 const float *__restrict__ b, int dtime, float *__restrict__ x, int64_t ldx, float *__restrict__ h0,
                 float *__restrict__ dtm) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  for (int64_t r = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * kRowsPerCta) {
    const int64_t id = nodes[r];
    const float *mrow = memory + id * dmem;
    for (int c = lane; c < dmem; c += 32) h0[r * dmem + c] = __ldg(mrow + c);
    const float *brow = mailbox + id * dmail;
    float *xr = x + r * ldx;
    for (int c = lane; c < dmail; c += 32) xr[c] = __ldg(brow + c);
    const float d = __fsub_rn(ts[r], __ldg(mem_ts + id));
    if (lane == 0 && dtm) dtm[r] = d;
    for (int c = lane; c < dtime; c += 32) xr[dmail + c] = cosf(fmaf(d, __ldg(w + c), __ldg(b + c)));
  }
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.f / (1.f + expf(-v)); }

// GRUCell (torch.nn.GRUCell; gates r, z, n in that order along the 3H axis):
//   r = s(gi_r + gh_r), z = s(gi_z + gh_z), n = tanh(gi_n + r gh_n),
//   h' = (1 - z) n + z h0.
// gi, gh hold the products with their biases; gi is overwritten with (r, z, n)
// for the backward, gh keeps gh_n.
__global__ void k_gru_fwd(float *__restrict__ gi, const float *__restrict__ gh, const float *__restrict__ h0,
                          float *__restrict__ h1, int64_t n, const int32_t *n_dev, int H) {
  fb::pdl_enter();
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  const int64_t total = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int j = (int)(i - r * H);
    float *g = gi + r * 3 * H;
    const float *q = gh + r * 3 * H;
    const float rr = sigmoidf_(g[j] + q[j]);
    const float zz = sigmoidf_(g[H + j] + q[H + j]);
    const float nn = tanhf(fmaf(rr, q[2 * H + j], g[2 * H + j]));
    const float hp = h0[r * H + j];
    h1[r * H + j] = fmaf(zz, hp - nn, nn);
    g[j] = rr;
    g[H + j] = zz;
    g[2 * H + j] = nn;
  }
}

// Backward of k_gru_fwd for dh1: gi <- d(gi) = (dr~, dz~, dn~), gh <- d(gh) =
// (dr~, dz~, dn~ r) with dn~ = dh1 (1 - z)(1 - n^2), dz~ = dh1 (h0 - n) z (1 - z),
// dr~ = dn~ gh_n r (1 - r).  (h0 is the stored memory: no gradient.)
__global__ void k_gru_bwd(float *__restrict__ gi, float *__restrict__ gh, const float *__restrict__ h0,
                          const float *__restrict__ dh1, int64_t ld_dh, int64_t n, const int32_t *n_dev, int H) {
  fb::pdl_enter();
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  const int64_t total = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int j = (int)(i - r * H);
    float *g = gi + r * 3 * H;
    float *q = gh + r * 3 * H;
    const float rr = g[j], zz = g[H + j], nn = g[2 * H + j];
    const float ghn = q[2 * H + j];
    const float d = dh1[r * ld_dh + j];
    const float dn = d * (1.f - zz) * (1.f - nn * nn);
    const float dz = d * (h0[r * H + j] - nn) * zz * (1.f - zz);
    const float dr = dn * ghn * rr * (1.f - rr);
    g[j] = dr;
    g[H + j] = dz;
    g[2 * H + j] = dn;
    q[j] = dr;
    q[H + j] = dz;
    q[2 * H + j] = dn * rr;
  }
}

// ---- last-write-wins scatters ------------------------------------------------
// Mailbox, deliver_to 'self' (memorys.py:106-142): for the n positive edges,
// list entry k = 2i is src_i = roots[i] with mail [h[i] | h[n+i] | f[e0+i]],
// k = 2i + 1 is dst_i = roots[n+i] with [h[n+i] | h[i] | f[e0+i]]; the mail
// time of entry k is root_ts[k] (the reference indexes ts[:2n] with the
// interleaved k).  Memory (memorys.py:84-99): entry k < 2n is roots[k] with
// row h[k] and time root_ts[k].
__device__ __forceinline__ int mail_node(const int32_t *roots, int64_t n, int64_t k) {
  return (k & 1) ? roots[n + (k >> 1)] : roots[k >> 1];
}

__global__ void k_last_index(const int32_t *__restrict__ roots, int64_t n, int interleaved,
                             unsigned long long *__restrict__ last, const uint32_t *__restrict__ gen) {
  fb::pdl_enter();
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= 2 * n) return;
  const int id = interleaved ? mail_node(roots, n, k) : roots[k];
  atomicMax(last + id, ((unsigned long long)(*gen) << 32) | (unsigned long long)k);
}

// The last CTA of a write pass advances the generation.
__device__ __forceinline__ void finish_pass(uint32_t *gen, uint32_t *done) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *gen += 1;
      *done = 0;
    }
  }
}

// One warp per list entry.
__global__ void __launch_bounds__(256)
    k_write_mail(const int32_t *__restrict__ roots, const float *__restrict__ root_ts, int64_t n,
                 const float *__restrict__ h, int64_t ldh, int dmem, const float *__restrict__ f, int64_t ldf, int de,
                 const int64_t *__restrict__ e0_dev, float *__restrict__ mailbox, float *__restrict__ mailbox_ts,
                 int32_t *__restrict__ next_pos, int mailbox_size, const unsigned long long *__restrict__ last, uint32_t *gen, uint32_t *done) {
  fb::pdl_enter();
  const uint32_t g = *gen;
  const int64_t e0 = e0_dev ? *e0_dev : 0;
  const int lane = threadIdx.x & 31;
  const int64_t k = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (k < 2 * n) {
    const int id = mail_node(roots, n, k);
    if (last[id] == (((unsigned long long)g << 32) | (unsigned long long)k)) {
      const int64_t i = k >> 1;
      const int64_t a = (k & 1) ? n + i : i, bb = (k & 1) ? i : n + i;
      const int pos = next_pos[id];
      const int dmail = 2 * dmem + de;
      float *row = mailbox + ((int64_t)id * mailbox_size + pos) * dmail;
      for (int c = lane; c < dmem; c += 32) {
        row[c] = h[a * ldh + c];
        row[dmem + c] = h[bb * ldh + c];
      }
      for (int c = lane; c < de; c += 32) row[2 * dmem + c] = f[(e0 + i) * ldf + c];
      if (lane == 0) {
        mailbox_ts[(int64_t)id * mailbox_size + pos] = root_ts[k];
        if (mailbox_size > 1) next_pos[id] = (pos + 1) % mailbox_size;
      }
    }
  }
  finish_pass(gen, done);
}

__global__ void __launch_bounds__(256)
    k_write_mem(const int32_t *__restrict__ roots, const float *__restrict__ root_ts, int64_t n,
                const float *__restrict__ h, int64_t ldh, int dmem, float *__restrict__ memory,
                float *__restrict__ mem_ts, const unsigned long long *__restrict__ last, uint32_t *gen,
                uint32_t *done) {
  fb::pdl_enter();
  const uint32_t g = *gen;
  const int lane = threadIdx.x & 31;
  const int64_t k = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (k < 2 * n) {
    const int id = roots[k];
    if (last[id] == (((unsigned long long)g << 32) | (unsigned long long)k)) {
      for (int c = lane; c < dmem; c += 32) memory[(int64_t)id * dmem + c] = h[k * ldh + c];
      if (lane == 0) mem_ts[id] = root_ts[k];
    }
  }
  finish_pass(gen, done);
}

// ---- APAN: transformer memory updater over the mailbox slots ----------------
// Row r * S + s of x: [mailbox[id, s] | cos(w (ts[r] - mailbox_ts[id, s]) + b)],
// dts[r * S + s] = ts[r] - mailbox_ts[id, s]; h0[r] = memory[id]  (id = nodes[r]).
__global__ void __launch_bounds__(32 * kRowsPerCta)
    k_mail_slots_gather(const int32_t *__restrict__ nodes, const float *__restrict__ ts, int64_t n,
                        const int32_t *n_dev, const float *__restrict__ memory, int dmem,
                        const float *__restrict__ mailbox, const float *__restrict__ mailbox_ts, int S, int dmail,
                        const float *__restrict__ w, const float *__restrict__ b, int dtime, float *__restrict__ x,
                        int64_t ldx, float *__restrict__ h0, float *__restrict__ dts) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t rows = (n_dev ? min((int64_t)(*n_dev), n) : n) * S;
  for (int64_t q = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5); q < rows;
       q += (int64_t)gridDim.x * kRowsPerCta) {
    const int64_t r = q / S;
    const int s = (int)(q - r * S);
    const int64_t id = nodes[r];
    if (s == 0)
      for (int c = lane; c < dmem; c += 32) h0[r * dmem + c] = __ldg(memory + id * dmem + c);
    const float *mrow = mailbox + (id * S + s) * dmail;
    float *xr = x + q * ldx;
    for (int c = lane; c < dmail; c += 32) xr[c] = __ldg(mrow + c);
    const float d = __fsub_rn(ts[r], __ldg(mailbox_ts + id * S + s));
    if (lane == 0) dts[q] = d;
    for (int c = lane; c < dtime; c += 32) xr[dmail + c] = cosf(fmaf(d, __ldg(w + c), __ldg(b + c)));
  }
}

// out = LayerNorm(x + res) per row (torch.nn.LayerNorm, biased variance);
// keeps the normalised row in xhat and 1 / std in rstd for the backward.
__global__ void __launch_bounds__(256)
    k_add_ln_fwd(const float *__restrict__ x, const float *__restrict__ res, const float *__restrict__ gamma,
                 const float *__restrict__ beta, float eps, float *__restrict__ out, float *__restrict__ xhat,
                 float *__restrict__ rstd, int64_t n, const int32_t *n_dev, int D) {
  fb::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * 8) {
    float sum = 0.f;
    for (int c = lane; c < D; c += 32) sum += x[r * D + c] + res[r * D + c];
    const float mean = fb::warp_sum(sum) / D;
    float var = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float v = x[r * D + c] + res[r * D + c] - mean;
      var = fmaf(v, v, var);
    }
    const float rs = rsqrtf(fb::warp_sum(var) / D + eps);
    for (int c = lane; c < D; c += 32) {
      const float xh = (x[r * D + c] + res[r * D + c] - mean) * rs;
      xhat[r * D + c] = xh;
      out[r * D + c] = fmaf(xh, gamma[c], beta[c]);
    }
    if (lane == 0) rstd[r] = rs;
  }
}

constexpr int64_t kLnRowsMin = 64;

// dx = rstd (g - mean(g) - xhat mean(g xhat)), g = dout gamma; dgamma / dbeta
// partial sums per CTA into part[blockIdx.x][2][D] (reduced by k_col_reduce).
// The rows split into contiguous parts whose number depends on the row count
// only, so capacity-sized and exact launches sum in the same order.
__global__ void __launch_bounds__(256)
    k_add_ln_bwd(const float *__restrict__ dout, const float *__restrict__ xhat, const float *__restrict__ rstd,
                 const float *__restrict__ gamma, float *__restrict__ dx, float *__restrict__ part, int64_t n,
                 const int32_t *n_dev, int D) {
  fb::pdl_enter();
  extern __shared__ float acc[];   // [8 warps][2][D]
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  const int parts = fb::split_parts(rows, kLnRowsMin, gridDim.x);
  if ((int)blockIdx.x >= parts) return;
  for (int c = threadIdx.x; c < 16 * D; c += blockDim.x) acc[c] = 0.f;
  __syncthreads();
  const int64_t per = (rows + parts - 1) / parts;
  const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
  float *ag = acc + wp * 2 * D, *ab = ag + D;
  for (int64_t r = r0 + wp; r < r1; r += 8) {
    float s1 = 0.f, s2 = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float g = dout[r * D + c] * gamma[c];
      s1 += g;
      s2 = fmaf(g, xhat[r * D + c], s2);
    }
    const float m1 = fb::warp_sum(s1) / D, m2 = fb::warp_sum(s2) / D;
    const float rs = rstd[r];
    for (int c = lane; c < D; c += 32) {
      const float go = dout[r * D + c], xh = xhat[r * D + c];
      dx[r * D + c] = rs * (go * gamma[c] - m1 - xh * m2);
      ag[c] = fmaf(go, xh, ag[c]);
      ab[c] += go;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += acc[w * 2 * D + c];
    part[(int64_t)blockIdx.x * 2 * D + c] = t;
  }
}

// dgamma (+)= sum of part[:, 0, :], dbeta (+)= sum of part[:, 1, :] (fixed order).
__global__ void k_col_reduce(const float *__restrict__ part, int max_parts, int64_t n, const int32_t *n_dev, int D,
                             float *dgamma, float *dbeta) {
  fb::pdl_enter();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * D) return;
  const int64_t rows = n_dev ? min((int64_t)(*n_dev), n) : n;
  const int parts = fb::split_parts(rows, kLnRowsMin, max_parts);
  float t = 0.f;
  for (int p = 0; p < parts; ++p) t += part[(int64_t)p * 2 * D + c];
  if (c < D) dgamma[c] += t;
  else dbeta[c - D] += t;
}

// APAN delivery (memorys.py:143-178): list entry k < 2n is root k (its own
// mail), entry 2n + e is nodes[2n + e], the neighbour sampled for edge e,
// which receives the mail of its root row[e].  The mail of root j is
// [h[j] | h[j +- n] | f[e0 + j mod n]] (src roots j < n, dst roots after),
// its time root_ts[j].  Last occurrence wins per node; the winner writes slot
// next_pos[node] and advances it modulo the mailbox size.
__global__ void k_last_nbr(const int32_t *__restrict__ nodes, int64_t n, const int32_t *E_dev, int64_t E_cap,
                           unsigned long long *__restrict__ last, const uint32_t *__restrict__ gen) {
  fb::pdl_enter();
  const int64_t E = E_dev ? min((int64_t)(*E_dev), E_cap) : E_cap;
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= 2 * n + E) return;
  atomicMax(last + nodes[k], ((unsigned long long)(*gen) << 32) | (unsigned long long)k);
}

__global__ void __launch_bounds__(256)
    k_write_nbr(const int32_t *__restrict__ nodes, const int32_t *__restrict__ row, const float *__restrict__ root_ts,
                int64_t n, const int32_t *E_dev, int64_t E_cap, const float *__restrict__ h, int64_t ldh, int dmem,
                const float *__restrict__ f, int64_t ldf, int de, const int64_t *__restrict__ e0_dev,
                float *__restrict__ mailbox, float *__restrict__ mailbox_ts, int32_t *__restrict__ next_pos,
                int mailbox_size, const unsigned long long *__restrict__ last, uint32_t *gen, uint32_t *done) {
  fb::pdl_enter();
  const uint32_t g = *gen;
  const int64_t e0 = e0_dev ? *e0_dev : 0;
  const int64_t E = E_dev ? min((int64_t)(*E_dev), E_cap) : E_cap;
  const int lane = threadIdx.x & 31;
  const int64_t k = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (k < 2 * n + E) {
    const int id = nodes[k];
    if (last[id] == (((unsigned long long)g << 32) | (unsigned long long)k)) {
      const int64_t j = k < 2 * n ? k : (int64_t)row[k - 2 * n];   // root whose mail this is
      const int64_t other = j < n ? j + n : j - n, ei = j < n ? j : j - n;
      const int pos = next_pos[id];
      const int dmail = 2 * dmem + de;
      float *dst = mailbox + ((int64_t)id * mailbox_size + pos) * dmail;
      for (int c = lane; c < dmem; c += 32) {
        dst[c] = h[j * ldh + c];
        dst[dmem + c] = h[other * ldh + c];
      }
      for (int c = lane; c < de; c += 32) dst[2 * dmem + c] = f[(e0 + ei) * ldf + c];
      if (lane == 0) {
        mailbox_ts[(int64_t)id * mailbox_size + pos] = root_ts[j];
        if (mailbox_size > 1) next_pos[id] = (pos + 1) % mailbox_size;
      }
    }
  }
  finish_pass(gen, done);
}

inline int grid_for(int64_t total, int threads) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((total + threads - 1) / threads, 148 * 16));
}

}  // namespace

extern "C" int fb_mem_gather(const int32_t *nodes, const float *ts, int64_t n, const int32_t *n_dev,
                             const float *memory, int dmem, const float *mem_ts, const float *mailbox, int dmail,
                             const float *w, const float *b, int dtime, float *x, int64_t ldx, float *h0, float *dtm,
                             cudaStream_t stream) {
  if (n < 0 || dmem < 0 || dmail < 0 || dtime < 0 || (n > 0 && (!nodes || !ts || !memory || !mem_ts || !x || !h0)) ||
      (dmail > 0 && !mailbox) || (dtime > 0 && (!w || !b)) || ldx < dmail + dtime)
    return fb::set_error(FB_ERR_ARG, "mem_gather: bad argument");
  if (n == 0) return FB_OK;
  const int grid = (int)std::min<int64_t>((n + kRowsPerCta - 1) / kRowsPerCta, 148 * 8);
  FB_TRY_CUDA(fb::launch(k_mem_gather, grid, 32 * kRowsPerCta, 0, stream, nodes, ts, n, n_dev, memory, dmem, mem_ts,
                         mailbox, dmail, w, b, dtime, x, ldx, h0, dtm));
  FB_LAUNCHED("k_mem_gather");
  return FB_OK;
}

extern "C" int fb_gru_fwd(float *gi, const float *gh, const float *h0, float *h1, int64_t n, const int32_t *n_dev,
                          int H, cudaStream_t stream) {
  if (n < 0 || H < 1 || (n > 0 && (!gi || !gh || !h0 || !h1))) return fb::set_error(FB_ERR_ARG, "gru_fwd: bad argument");
  if (n == 0) return FB_OK;
  FB_TRY_CUDA(fb::launch(k_gru_fwd, grid_for(n * H, 256), 256, 0, stream, gi, gh, h0, h1, n, n_dev, H));
  FB_LAUNCHED("k_gru_fwd");
  return FB_OK;
}

extern "C" int fb_gru_bwd(float *gi, float *gh, const float *h0, const float *dh1, int64_t ld_dh, int64_t n,
                          const int32_t *n_dev, int H, cudaStream_t stream) {
  if (n < 0 || H < 1 || ld_dh < H || (n > 0 && (!gi || !gh || !h0 || !dh1)))
    return fb::set_error(FB_ERR_ARG, "gru_bwd: bad argument");
  if (n == 0) return FB_OK;
  FB_TRY_CUDA(fb::launch(k_gru_bwd, grid_for(n * H, 256), 256, 0, stream, gi, gh, h0, dh1, ld_dh, n, n_dev, H));
  FB_LAUNCHED("k_gru_bwd");
  return FB_OK;
}

extern "C" int fb_mailbox_update_self(const int32_t *roots, const float *root_ts, int64_t n, const float *h,
                                      int64_t ldh, int dmem, const float *f, int64_t ldf, int de,
                                      const int64_t *e0_dev, float *mailbox, float *mailbox_ts, int32_t *next_pos, int mailbox_size,
                                      unsigned long long *last, uint32_t *gen, uint32_t *done, cudaStream_t stream) {
  if (n < 0 || dmem < 1 || de < 0 || mailbox_size < 1 || ldh < dmem ||
      (n > 0 && (!roots || !root_ts || !h || !mailbox || !mailbox_ts || !next_pos || !last || !gen || !done)) ||
      (de > 0 && (!f || ldf < de)))
    return fb::set_error(FB_ERR_ARG, "mailbox_update_self: bad argument");
  if (n == 0) return FB_OK;
  FB_TRY_CUDA(fb::launch(k_last_index, (int)((2 * n + 255) / 256), 256, 0, stream, roots, n, 1, last,
                         (const uint32_t *)gen));
  FB_LAUNCHED("k_last_index");
  FB_TRY_CUDA(fb::launch(k_write_mail, (int)((2 * n + 7) / 8), 256, 0, stream, roots, root_ts, n, h, ldh, dmem, f, ldf,
                         de, e0_dev, mailbox, mailbox_ts, next_pos, mailbox_size, (const unsigned long long *)last, gen,
                         done));
  FB_LAUNCHED("k_write_mail");
  return FB_OK;
}

extern "C" int fb_memory_update(const int32_t *roots, const float *root_ts, int64_t n, const float *h, int64_t ldh,
                                int dmem, float *memory, float *mem_ts, unsigned long long *last, uint32_t *gen,
                                uint32_t *done, cudaStream_t stream) {
  if (n < 0 || dmem < 1 || ldh < dmem ||
      (n > 0 && (!roots || !root_ts || !h || !memory || !mem_ts || !last || !gen || !done)))
    return fb::set_error(FB_ERR_ARG, "memory_update: bad argument");
  if (n == 0) return FB_OK;
  FB_TRY_CUDA(fb::launch(k_last_index, (int)((2 * n + 255) / 256), 256, 0, stream, roots, n, 0, last,
                         (const uint32_t *)gen));
  FB_LAUNCHED("k_last_index");
  FB_TRY_CUDA(fb::launch(k_write_mem, (int)((2 * n + 7) / 8), 256, 0, stream, roots, root_ts, n, h, ldh, dmem, memory,
                         mem_ts, (const unsigned long long *)last, gen, done));
  FB_LAUNCHED("k_write_mem");
  return FB_OK;
}

extern "C" int fb_mail_slots_gather(const int32_t *nodes, const float *ts, int64_t n, const int32_t *n_dev,
                                    const float *memory, int dmem, const float *mailbox, const float *mailbox_ts,
                                    int slots, int dmail, const float *w, const float *b, int dtime, float *x,
                                    int64_t ldx, float *h0, float *dts, cudaStream_t stream) {
  if (n < 0 || slots < 1 || dmem < 1 || dmail < 1 || dtime < 0 || ldx < dmail + dtime ||
      (n > 0 && (!nodes || !ts || !memory || !mailbox || !mailbox_ts || !x || !h0 || !dts)) ||
      (dtime > 0 && (!w || !b)))
    return fb::set_error(FB_ERR_ARG, "mail_slots_gather: bad argument");
  if (n == 0) return FB_OK;
  const int grid = (int)std::min<int64_t>((n * slots + kRowsPerCta - 1) / kRowsPerCta, 148 * 8);
  FB_TRY_CUDA(fb::launch(k_mail_slots_gather, grid, 32 * kRowsPerCta, 0, stream, nodes, ts, n, n_dev, memory, dmem,
                         mailbox, mailbox_ts, slots, dmail, w, b, dtime, x, ldx, h0, dts));
  FB_LAUNCHED("k_mail_slots_gather");
  return FB_OK;
}

extern "C" int fb_add_layernorm_fwd(const float *x, const float *res, const float *gamma, const float *beta, float eps,
                                    float *out, float *xhat, float *rstd, int64_t n, const int32_t *n_dev, int D,
                                    cudaStream_t stream) {
  if (n < 0 || D < 1 || (n > 0 && (!x || !res || !gamma || !beta || !out || !xhat || !rstd)))
    return fb::set_error(FB_ERR_ARG, "add_layernorm_fwd: bad argument");
  if (n == 0) return FB_OK;
  const int grid = (int)std::min<int64_t>((n + 7) / 8, 148 * 8);
  FB_TRY_CUDA(fb::launch(k_add_ln_fwd, grid, 256, 0, stream, x, res, gamma, beta, eps, out, xhat, rstd, n, n_dev, D));
  FB_LAUNCHED("k_add_ln_fwd");
  return FB_OK;
}

extern "C" size_t fb_add_layernorm_bwd_ws_bytes(int64_t n, int D) {
  const int64_t parts = std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 148 * 2));
  return (size_t)parts * 2 * (size_t)std::max(D, 1) * sizeof(float);
}

extern "C" int fb_add_layernorm_bwd(const float *dout, const float *xhat, const float *rstd, const float *gamma,
                                    float *dx, float *dgamma, float *dbeta, int64_t n, const int32_t *n_dev, int D,
                                    void *ws, cudaStream_t stream) {
  if (n < 0 || D < 1 || D > 1024 || (n > 0 && (!dout || !xhat || !rstd || !gamma || !dx || !dgamma || !dbeta || !ws)))
    return fb::set_error(FB_ERR_ARG, "add_layernorm_bwd: bad argument");
  if (n == 0) return FB_OK;
  const int parts = (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 148 * 2));
  const size_t smem = (size_t)16 * D * sizeof(float);
  if (smem > 48 * 1024) FB_TRY_CUDA(cudaFuncSetAttribute(k_add_ln_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         (int)smem));
  float *part = static_cast<float *>(ws);
  FB_TRY_CUDA(fb::launch(k_add_ln_bwd, parts, 256, smem, stream, dout, xhat, rstd, gamma, dx, part, n, n_dev, D));
  FB_LAUNCHED("k_add_ln_bwd");
  FB_TRY_CUDA(fb::launch(k_col_reduce, (2 * D + 255) / 256, 256, 0, stream, (const float *)part, parts, n, n_dev, D,
                         dgamma, dbeta));
  FB_LAUNCHED("k_col_reduce");
  return FB_OK;
}

extern "C" int fb_mailbox_update_neighbors(const int32_t *nodes, const int32_t *row, const float *root_ts, int64_t n,
                                           const int32_t *E_dev, int64_t E_cap, const float *h, int64_t ldh, int dmem,
                                           const float *f, int64_t ldf, int de, const int64_t *e0_dev, float *mailbox,
                                           float *mailbox_ts, int32_t *next_pos, int mailbox_size,
                                           unsigned long long *last, uint32_t *gen, uint32_t *done,
                                           cudaStream_t stream) {
  if (n < 0 || E_cap < 0 || dmem < 1 || de < 0 || mailbox_size < 1 || ldh < dmem ||
      (n > 0 && (!nodes || !root_ts || !h || !mailbox || !mailbox_ts || !next_pos || !last || !gen || !done)) ||
      (E_cap > 0 && !row) || (de > 0 && (!f || ldf < de)))
    return fb::set_error(FB_ERR_ARG, "mailbox_update_neighbors: bad argument");
  const int64_t total = 2 * n + E_cap;
  if (total == 0) return FB_OK;
  FB_TRY_CUDA(fb::launch(k_last_nbr, (int)((total + 255) / 256), 256, 0, stream, nodes, n, E_dev, E_cap, last,
                         (const uint32_t *)gen));
  FB_LAUNCHED("k_last_nbr");
  FB_TRY_CUDA(fb::launch(k_write_nbr, (int)((total + 7) / 8), 256, 0, stream, nodes, row, root_ts, n, E_dev, E_cap, h,
                         ldh, dmem, f, ldf, de, e0_dev, mailbox, mailbox_ts, next_pos, mailbox_size,
                         (const unsigned long long *)last, gen, done));
  FB_LAUNCHED("k_write_nbr");
  return FB_OK;
}
