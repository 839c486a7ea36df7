/*
 * fast_b200 -- C ABI of the B200-native temporal-attention hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * launches sm_100a kernels on that stream, never synchronises unless it says
 * so, and returns an fb_status (0 == FB_OK).  Sizes that are only known on
 * the device (edge counts produced by the sampler) can be passed as a device
 * pointer (`*_dev`, may be NULL) together with a host upper bound, so a whole
 * training step can be enqueued without a host round trip.
 *
 * Reference interfaces replaced (paths inside NoneBone/FAST):
 *   ParallelSampler / TemporalGraphBlock   getSamplerCore/sampler_core.cpp:31-712, :1115-1149
 *   fastAgg operators                      getFastAgg/cuda_operators/operators.cpp:606-624
 *   prepare_input + TimeEncode             utils.py:126-196, layers.py:8-29
 *   Q/K/V torch.nn.Linear                  layers.py:91-95, :149-164
 */
#ifndef FAST_B200_H
#define FAST_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FB_OK = 0,
  FB_ERR_ARG = 1,          /* bad pointer / size / layout argument                */
  FB_ERR_CUDA = 2,         /* a CUDA runtime call or kernel launch failed         */
  FB_ERR_UNSUPPORTED = 3,  /* shape outside what the kernels are built for        */
  FB_ERR_NOMEM = 4,        /* device allocation inside a runtime object failed    */
  FB_ERR_STATE = 5         /* object used in the wrong order                      */
} fb_status;

/* Human-readable text of the last error raised on the calling thread. */
const char *fb_last_error(void);
/* Library version string. */
const char *fb_version(void);

/* ------------------------------------------------------------------------- */
/* Temporal neighbour sampler (runtime object).                               */
/* Replaces ParallelSampler (sampler_core.cpp:67-712, bound at :1139-1149).   */
/* ------------------------------------------------------------------------- */
typedef struct fb_sampler fb_sampler;

/* Device view of one sampled block (TemporalGraphBlock, sampler_core.cpp:31-65).
 * Arrays are sized for the block's capacity; `dims` (device, 8 x int32) holds
 * {dim_out (= roots), E, S (non-empty rows), dim_in (= roots + E), n_uni, 0,0,0}.
 *   row[E], col[E], eid[E]            COO in root order (sampler_core.cpp:273-277)
 *   ts[dim_in], dts[dim_in], nodes[dim_in]  roots first, then one entry per edge
 *   rptr[dim_out + 1]                 CSR offsets over ALL roots (empty rows allowed)
 *   cntE[S + 1]                       offsets over non-empty rows only (:384-410)
 *   uniE[n_uni], invE[E]              eid dedup, first-appearance order (:414-451),
 *                                     valid after fb_sampler_dedup()
 *   dte[E], nbr[E]                    copies of dts[R + e] and nodes[R + e] at a
 *                                     fixed base, for launches that must not
 *                                     depend on the device-only root count   */
typedef struct {
  int32_t *row, *col, *eid;
  float *ts, *dts;
  int32_t *nodes, *rptr, *cntE, *uniE, *invE;
  int32_t *dims;
  int64_t max_roots, max_edges;
  float *dte;
  int32_t *nbr;
} fb_block_view;

/* Copies (graph_on_device == 0) or borrows (== 1) the time-sorted CSR
 * indptr[n_nodes+1], indices/eid/ts[n_edges] on the current device.
 * Mirrors the ParallelSampler constructor (sampler_core.cpp:89-114);
 * thread counts of the reference have no meaning here.  `seed` keys the
 * Philox stream used by uniform sampling. */
int fb_sampler_create(const int32_t *indptr, const int32_t *indices, const int32_t *eid,
                      const float *ts, int64_t n_nodes, int64_t n_edges, int graph_on_device,
                      int num_layers, const int32_t *num_neighbors, int recent, int prop_time,
                      int num_history, float window_duration, uint64_t seed, fb_sampler **out);
int fb_sampler_destroy(fb_sampler *s);
/* Rewinds the stateful time pointers (ParallelSampler::reset, :122-131). */
int fb_sampler_reset(fb_sampler *s, cudaStream_t stream);
/* Samples all layers/history slots for n_roots roots (ParallelSampler::sample,
 * :597-712).  roots/root_ts are host arrays when roots_on_device == 0 (copied
 * on `stream`), device arrays otherwise.  May grow the block buffers (which
 * synchronises the device) when n_roots exceeds every earlier call. */
int fb_sampler_sample(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                      int roots_on_device, cudaStream_t stream);
/* Applies the first layer's pointer updates of sample() (update_ts_ptr,
 * :133-157) for device roots without sampling.  It advances the pointers the
 * first layer samples with; data-parallel ranks sample with
 * fb_sampler_sample_shard, which makes every layer's updates. */
int fb_sampler_update_pointers(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                               cudaStream_t stream);
/* sample() of one data-parallel rank's shard (ParallelSampler::sample,
 * :597-712, with update_ts_ptr :133-157 and the per-layer use_ptr rule
 * :700-706).  roots/root_ts (device, n_roots) are this rank's roots, a subset
 * of the global batch global_roots/global_ts (device, n_global).  Every
 * pointer update that one sample() over the global batch makes is made here:
 * layer 0 with the global roots, each later layer that samples with the
 * pointers with the nodes of the global batch's previous-layer block, which
 * this call samples alongside the rank's own.  Every block, of every layer,
 * then holds exactly the picks that one process sampling the global batch
 * makes for these roots (recent-k: bit for bit), and the pointers after the
 * call are that process's.  num_history must be 1 with no window
 * (FB_ERR_UNSUPPORTED otherwise).  Grows its buffers (synchronising the
 * device) when n_global exceeds every earlier call. */
int fb_sampler_sample_shard(fb_sampler *s, const int32_t *roots, const float *root_ts, int64_t n_roots,
                            const int32_t *global_roots, const float *global_ts, int64_t n_global,
                            cudaStream_t stream);
/* Number of blocks from the last sample() (= num_layers * num_history), in
 * the reference's get_ret() order. */
int fb_sampler_num_blocks(const fb_sampler *s);
int fb_sampler_block(const fb_sampler *s, int i, fb_block_view *out);
/* Copies every block's dims to host_dims[8 * num_blocks]; synchronises `stream`. */
int fb_sampler_dims(fb_sampler *s, int32_t *host_dims, cudaStream_t stream);
/* Builds uniE/invE of block i on the device (dims[4] receives n_uni). */
int fb_sampler_dedup(fb_sampler *s, int i, cudaStream_t stream);
/* Sampler step counter that keys uniform draws; set it to replay a batch.
 * The counter lives in device memory and every sample() call advances it on
 * the stream, so a captured CUDA graph draws fresh samples on each replay. */
int fb_sampler_set_call_index(fb_sampler *s, uint64_t call_index);

/* ------------------------------------------------------------------------- */
/* Fused temporal attention: LeakyReLU(q.k) -> per-destination edge softmax  */
/* -> dropout -> weighted aggregate.  Replaces, in one launch, layers.py:165-223
 * = ESM_Function_TGAT (efficientGOP.py:66-78, kernel edge_softmax.cu:255-293)
 * + MA_Function_TGAT (efficientGOP.py:97-113, aggregate_*_kernel.cu).       */
/* ------------------------------------------------------------------------- */
/* q[n_dst, dim] (ldq elements per row; ldq == 0 broadcasts one row),
 * k/v rows of edge e at k + e*ldkv, v + e*ldkv, rptr[n_dst+1] CSR over
 * destinations.  Writes att[E, heads] (softmax before dropout) and
 * agg[n_dst, dim] (zero rows for destinations without edges).  With
 * n_dst_dev, the rows [*n_dst_dev, n_dst) of agg are written as zeros.  dim % 4 == 0,
 * dim <= 512, heads <= 4, dim % heads == 0.  drop_p == 0 disables dropout;
 * otherwise the keep mask is Philox(seed, offset, edge, head), with the
 * offset read from offset_dev when that is not NULL (for graph replays). */
int fb_attn_fwd(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                float slope, float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                float *att, float *agg, int64_t ldagg, cudaStream_t stream);
/* Backward of fb_attn_fwd (efficientGOP.py:80-95,115-131, but with the true
 * gradient).  Writes dq[n_dst, dim] (ld = dim; the segment sum of the
 * per-edge gradient), dk, dv (rows at e*lddkv).  Any of dq/dk/dv may be NULL. */
int fb_attn_bwd(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                float slope, float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                const float *att, const float *dagg, int64_t lddagg, float *dq, float *dk, float *dv,
                int64_t lddkv, cudaStream_t stream);
/* fb_attn_bwd with dk / dv written as bf16 bit patterns (round to nearest
 * even) for the bf16 projection GEMMs; lddkv % 4 == 0. */
int fb_attn_bwd_bf16kv(const float *q, int64_t ldq, const float *k, const float *v, int64_t ldkv,
                       const int32_t *rptr, int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim,
                       float slope, float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                       const float *att, const float *dagg, int64_t lddagg, float *dq, uint16_t *dk, uint16_t *dv,
                       int64_t lddkv, cudaStream_t stream);
/* fb_attn_fwd / fb_attn_bwd_bf16kv on bf16 K|V rows kv[E, ldkv] (K then V,
 * dim columns each, ldkv == 2 dim, ldkv % 8 == 0, dim <= 128): the bf16
 * projection mode, where the K|V projection stores bf16.  Softmax, dropout
 * and the sums run in fp32; the backward writes dq fp32 and dK|dV as bf16
 * rows in the same interleaved layout. */
int fb_attn_fwd_kvbf16(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv, const int32_t *rptr,
                       int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim, float slope, float drop_p,
                       uint64_t seed, uint64_t offset, const uint64_t *offset_dev, float *att, float *agg,
                       int64_t ldagg, cudaStream_t stream);
int fb_attn_bwd_kvbf16(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv, const int32_t *rptr,
                       int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim, float slope, float drop_p,
                       uint64_t seed, uint64_t offset, const uint64_t *offset_dev, const float *att,
                       const float *dagg, int64_t lddagg, float *dq, uint16_t *dkv, int64_t lddkv,
                       cudaStream_t stream);
/* The same two with the row outputs that only feed bf16 products written as
 * bf16 (round to nearest even; rows 8-byte aligned, pitch a multiple of 4):
 * agg [n_dst, ldagg] (the w_out operand, layers.py:213-217) and dq
 * [n_dst, lddq] (the Q-side gradient operand) -- one cast launch less each. */
int fb_attn_fwd_kvbf16_bf16out(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv, const int32_t *rptr,
                               int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim, float slope,
                               float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev, float *att,
                               uint16_t *agg, int64_t ldagg, cudaStream_t stream);
int fb_attn_bwd_kvbf16_bf16dq(const float *q, int64_t ldq, const uint16_t *kv, int64_t ldkv, const int32_t *rptr,
                              int64_t n_dst, const int32_t *n_dst_dev, int heads, int dim, float slope,
                              float drop_p, uint64_t seed, uint64_t offset, const uint64_t *offset_dev,
                              const float *att, const float *dagg, int64_t lddagg, uint16_t *dq, int64_t lddq,
                              uint16_t *dkv, int64_t lddkv, cudaStream_t stream);
/* Sticky error bits of the attention kernels on the current device (2 = a
 * bounded wait for a shared-memory bulk copy timed out and the warp gave up);
 * synchronises; clear resets. */
int fb_attn_error(int *flags, int clear);

/* The dropout multipliers (0 or 1/(1-p)) fb_attn_fwd/bwd apply to edge e,
 * head h for (seed, offset): out[e*heads + h].  For checking and replay. */
int fb_dropout_scale(int64_t n_edges, int heads, float drop_p, uint64_t seed, uint64_t offset, float *out,
                     cudaStream_t stream);
/* Same attention with precomputed pre-activation logits x[E, heads] in place
 * of q.k, V rows at v + e*ldv, segments [indptr[s], indptr[s+1]) over n_seg
 * segments.  seg_row (int64, may be NULL) names the output row of a segment
 * at its first edge, seg_row[indptr[s]] (rows of agg not named are left as
 * they are; ids outside [0, n_out) are skipped); NULL means segment s writes
 * row s.  mask_u (may be NULL) holds
 * dropout uniforms [E, heads], kept when u > drop_p.  agg rows have `dim`
 * floats.  Replaces forward_fused_attn (fused_attention.cu:68-127,203-328). */
int fb_attn_logits_fwd(const float *x, const float *v, int64_t ldv, const int32_t *indptr, int64_t n_seg,
                       const int64_t *seg_row, int64_t n_out, int heads, int dim, float slope, float drop_p,
                       const float *mask_u, float *att, float *agg, cudaStream_t stream);
/* Backward of fb_attn_logits_fwd: dx[E, heads] (gradient of the
 * pre-activation logits, LeakyReLU included) and dv rows at e*ldv.
 * Replaces backward_fused_attn (fused_attention.cu:129-200,330-446). */
int fb_attn_logits_bwd(const float *x, const float *v, int64_t ldv, const int32_t *indptr, int64_t n_seg,
                       const int64_t *seg_row, int64_t n_out, int heads, int dim, float slope, float drop_p,
                       const float *mask_u, const float *att, const float *dagg, float *dx, float *dv,
                       cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* fastAgg legacy operators (operators.cpp:606-624), correct semantics.        */
/* ------------------------------------------------------------------------- */
/* cal_deg (utils.cu:42-79): deg[edges[e]] += 1 for e < n_edges; deg zeroed by caller. */
int fb_count_ids(const int32_t *ids, int64_t n, int32_t *deg, int64_t n_ids, cudaStream_t stream);
/* getBalancedPtr (utils.cu:81-141): for segment i (< n_ptr - 1) with the
 * inclusive prefix P_i of degrees taken within its aligned group of 256
 * segments, mask[i] = (P_i / threshold > (P_i - deg_i) / threshold). */
int fb_balanced_mask(const int32_t *ptr, int64_t n_ptr, int threshold, int32_t *mask, cudaStream_t stream);
/* forward_edge_softmax / forward_csr_edge_softmax (edge_softmax.cu:55-78,178-206):
 * y[e,h] = softmax of x over each segment [indptr[s], indptr[s+1]). */
int fb_edge_softmax_fwd(const int32_t *indptr, int64_t n_seg, const float *x, int heads,
                        float *y, cudaStream_t stream);
/* backward_edge_softmax / backward_csr_edge_softmax (edge_softmax.cu:79-106,207-235):
 * dx = y * (dy - sum_seg(y * dy)). */
int fb_edge_softmax_bwd(const int32_t *indptr, int64_t n_seg, const float *dy, const float *y,
                        int heads, float *dx, cudaStream_t stream);
/* forward_tgat (aggregate_acc_kernel.cu:36-69), over ALL n_edges edges:
 * out[dst_idx[e], :] += v[src_idx[e], :].  `out` must be zeroed by the caller. */
int fb_scatter_rows(const int64_t *dst_idx, const int64_t *src_idx, int64_t n_edges,
                    const float *v, int64_t n_v, int dim, float *out, int64_t n_out,
                    cudaStream_t stream);
/* forward_tgat_shd (aggregate_shd_kernel.cu:37-94): segment sums
 * out[row[indptr[s]], :] = sum_{e in s} v[col[e], :] (deterministic order). */
int fb_segment_rows(const int32_t *indptr, int64_t n_seg, const int64_t *row, const int64_t *col,
                    const float *v, int64_t n_v, int dim, float *out, int64_t n_out,
                    cudaStream_t stream);
/* exclusive_sum (utils.cu:16-40): out[0] = 0, out[i+1] = sum(in[0..i]).
 * `ws` must hold fb_exclusive_sum_ws_bytes(n) bytes. */
size_t fb_exclusive_sum_ws_bytes(int64_t n);
int fb_exclusive_sum(const int32_t *in, int64_t n, int32_t *out, void *ws, cudaStream_t stream);
/* No counterpart in the reference.  fb_exclusive_sum for callers that cannot
 * allocate device memory and so cannot provide `ws`: a host that gives the
 * library a fixed memory budget and owns every allocation itself, or a loop
 * where an allocator call would synchronise the device.  The scratch is a
 * library-owned static device array (32 KiB, held by every GPU that loads the
 * library until exit); n is limited to 1,048,576 and larger n returns
 * FB_ERR_UNSUPPORTED.  It allocates nothing.  Its first call on a device looks
 * up the array's device address (cudaGetSymbolAddress), so make that first
 * call before any stream capture.  All calls share the one array: calls whose
 * kernels can overlap on the GPU (different streams without ordering) race. */
int fb_exclusive_sum_noalloc(const int32_t *in, int64_t n, int32_t *out, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* Feature gather fused with the cos time encoding (utils.py:126-196,         */
/* layers.py:17-29,103-110,157-164).                                           */
/* ------------------------------------------------------------------------- */
/* For every row r < n_rows (n_rows_dev overrides when not NULL):
 *   A[r, 0:dn)          = h[(h_idx ? h_idx[r] : r + h_off), :]
 *   A[r, dn:dn+de)      = f[(f_idx ? f_idx[r] : r), :]
 *   A[r, dn+de:+dtime)  = cos(w * dt[r] + b)          (dt == NULL -> dt = 0)
 * Any block with dn/de/dtime == 0 is skipped.  h_off_dev (may be NULL) adds a
 * device-resident row offset to h_off. */
int fb_gather_time_encode(const float *h, int64_t ldh, const int32_t *h_idx, int64_t h_off,
                          const int32_t *h_off_dev, int dn,
                          const float *f, int64_t ldf, const int32_t *f_idx, int de,
                          const float *dt, const float *w, const float *b, int dtime,
                          float *A, int64_t lda, int64_t n_rows, const int32_t *n_rows_dev,
                          cudaStream_t stream);
/* The bf16 projection rows of the bf16 precision mode: [h | f | cos(w dt + b)]
 * as bf16 with h at column 0, f at column pad8(dn) and the time encoding at
 * pad8(dn) + pad8(de) (pad8: up to a multiple of 8), so that each segment
 * starts on a 16-byte boundary; the gaps are zeros.  h and f are bf16 tables
 * (h_bf16 / f_bf16 = 1; rows 16-byte aligned and padded with zeros to a
 * multiple of 8 columns) or fp32 (dims multiples of 4).  lda % 8 == 0. */
int fb_gather_time_encode_bf16(const void *h, int h_bf16, int64_t ldh, const int32_t *h_idx, int64_t h_off,
                               const int32_t *h_off_dev, int dn, const void *f, int f_bf16, int64_t ldf,
                               const int32_t *f_idx, int de, const float *dt, const float *w, const float *b,
                               int dtime, uint16_t *A, int64_t lda, int64_t n_rows, const int32_t *n_rows_dev,
                               cudaStream_t stream);
/* Gradient of the time encoding (TimeEncode, layers.py:17-29; autograd in the
 * reference): with g = dL/dcos(w*dt+b) (rows at g + r*ldg),
 * dw[j] += sum_r -sin(w_j dt_r + b_j) dt_r g[r,j],  db[j] += sum_r -sin(..) g[r,j].
 * `ws` must hold fb_time_encode_bwd_ws_bytes(n_rows, dtime) bytes. */
size_t fb_time_encode_bwd_ws_bytes(int64_t n_rows, int dtime);
int fb_time_encode_bwd(const float *g, int64_t ldg, const float *dt, const float *w, const float *b,
                       int dtime, int64_t n_rows, const int32_t *n_rows_dev, float *dw, float *db,
                       void *ws, cudaStream_t stream);
/* The same with g as bf16 (raw bits), the bf16 projection mode's time-encoding
 * input gradient; the sums are fp32, and equal fb_time_encode_bwd's on g
 * widened to fp32.  Same workspace. */
int fb_time_encode_bwd_bf16(const uint16_t *g, int64_t ldg, const float *dt, const float *w, const float *b,
                            int dtime, int64_t n_rows, const int32_t *n_rows_dev, float *dw, float *db,
                            void *ws, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* Feature rows split between HBM and page-locked host memory: the slim      */
/* feature cache (slimCache.py:184-403: init_cache, fresh_cache,             */
/* trans2Device :261-403).                                                   */
/* ------------------------------------------------------------------------- */
/* out[r, 0:d) = table row ids[r] for r < n (n_dev overrides when not NULL):
 * from dev_rows[slot_of[ids[r]]] when that slot is in [0, n_dev_rows), else
 * from host_rows[ids[r]] (the full table, read by the GPU from page-locked
 * host memory: pass the address fb_host_rows_device_pointer returns).  Rows
 * are elem_bytes = 4 (fp32) or 2 (bf16) wide elements with leading dimensions
 * in elements.  An id outside [0, n_rows_total) gives a zero row and sets bit
 * 1 of *err (may be NULL); *misses (may be NULL) is increased by the rows read
 * from host memory. */
int fb_gather_rows_tiered(const int32_t *ids, int64_t n, const int32_t *n_dev, const int32_t *slot_of,
                          int64_t n_rows_total, const void *dev_rows, int64_t ld_dev, int64_t n_dev_rows,
                          const void *host_rows, int64_t ld_host, int d, int elem_bytes, void *out, int64_t ld_out,
                          unsigned long long *misses, int32_t *err, cudaStream_t stream);
/* The device address of page-locked, mapped host memory (cudaHostGetDevicePointer);
 * fails for pageable memory. */
int fb_host_rows_device_pointer(const void *host, void **dev);

/* ------------------------------------------------------------------------- */
/* fp32 projection GEMMs (torch.nn.Linear, layers.py:91-95).                  */
/* ------------------------------------------------------------------------- */
/* C[m, n] = sum_k A[m,k] B[n,k] (+ bias[n]) (+ C when accumulate)   "NT"
 * m < M (M_dev overrides), n < N, k < K.  Row-major with leading dims. */
int fb_gemm_nt(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias,
               float *C, int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K,
               int accumulate, cudaStream_t stream);
/* C[m, n] = sum_k A[m,k] B[k,n] (+ bias[n]) (+ C when accumulate)   "NN"
 * B stored [K, N] (ldb >= N): the input gradient dX = dY W of a Linear layer
 * without transposing W. */
int fb_gemm_nn(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias,
               float *C, int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K,
               int accumulate, cudaStream_t stream);
/* Same contract as fb_gemm_nt on the tcgen05 tensor cores: TMA-fed 128 x N
 * tiles, fp32 accuracy from three TF32 products per term (Ootomo & Yokota's
 * hi/lo split, computed in shared memory), accumulation in tensor memory.
 * Needs N <= 256, K, lda, ldb multiples of 4, A and B 16-byte aligned
 * (fb_gemm_nt_tc_supported). */
int fb_gemm_nt_tc_supported(const float *A, int64_t lda, const float *B, int64_t ldb, int N, int K);
int fb_gemm_nt_tc(const float *A, int64_t lda, const float *B, int64_t ldb, const float *bias, float *C,
                  int64_t ldc, int64_t M, const int32_t *M_dev, int N, int K, int accumulate,
                  cudaStream_t stream);
/* Sticky error bits of the tensor-core kernels on the current device (2 = a
 * bounded wait timed out and the CTA gave up); synchronises; clear resets. */
int fb_gemm_tc_error(int *flags, int clear);
/* C[n, k] = sum_m G[m, n] X[m, k]  (+ C when accumulate)              "TN"
 * the weight gradient of a Linear layer; deterministic split over M.
 * `ws` must hold fb_gemm_tn_ws_bytes(M, N, K) bytes. */
size_t fb_gemm_tn_ws_bytes(int64_t M, int N, int K);
int fb_gemm_tn(const float *G, int64_t ldg, const float *X, int64_t ldx, float *C, int64_t ldc,
               int64_t M, const int32_t *M_dev, int N, int K, int accumulate, void *ws,
               cudaStream_t stream);
/* fb_gemm_tn plus the bias gradient in the same pass: db[n] (+)= sum_m G[m, n]
 * (X gets a virtual column of ones).  db_accumulate applies to db alone. */
int fb_gemm_tn_bias(const float *G, int64_t ldg, const float *X, int64_t ldx, float *C, int64_t ldc,
                    int64_t M, const int32_t *M_dev, int N, int K, int accumulate, float *db,
                    int db_accumulate, void *ws, cudaStream_t stream);
/* Grouped launch of independent projection GEMMs (one grid, one split-reduce
 * pass): the GEMMs of one dependency level of a layer (e.g. every product
 * that reads dKV) run concurrently.  Outputs must not overlap.  Problems whose
 * rows are not 16-byte aligned run as single launches.  NT / NN may take A
 * as the concatenation along K of A (columns < k1) and A2 (columns >= k1):
 * torch.cat([agg, h_dst], 1) @ W^T without the copy (layers.py:213-217).
 * TN with K == 0 and db set computes column sums only.  ws:
 * fb_gemm_group_ws_bytes(probs, n) bytes. */
enum { FB_GEMM_NT = 0, FB_GEMM_NN = 1, FB_GEMM_TN = 2 };
typedef struct fb_gemm_problem {
  int kind;
  const float *A; int64_t lda;             /* NT / NN: A [M, K]; TN: G [M, N] */
  const float *A2; int64_t lda2; int k1;   /* NT / NN: columns >= k1 from A2 (NULL: none) */
  const float *B; int64_t ldb;             /* NT: [N, K]; NN: [K, N]; TN: X [M, K] */
  const float *bias;                       /* NT / NN, or NULL */
  float *C; int64_t ldc;                   /* NT / NN: [M, N]; TN: [N, K] */
  int64_t M; const int32_t *M_dev;         /* rows (capacity) and optional device count */
  int N, K;
  int accumulate;
  float *db; int db_accumulate;            /* TN: db[n] (+)= sum_m G[m, n], or NULL */
} fb_gemm_problem;
size_t fb_gemm_group_ws_bytes(const fb_gemm_problem *probs, int n);
int fb_gemm_group(const fb_gemm_problem *probs, int n, void *ws, size_t ws_bytes, cudaStream_t stream);
/* The same groups with bf16 operands (bf16 bit patterns, round-to-nearest-
 * even from fp32) and fp32 accumulation: the projections of the bf16
 * precision mode, on the tcgen05 tensor cores (kind::f16).  Field meanings as
 * in fb_gemm_problem (plus ka); C, bias and db stay fp32.  Every operand 16-byte
 * aligned with a leading dimension (elements) that is a multiple of 8, k1 a
 * multiple of 8, K >= 1 (TN: db via a virtual ones column at k = K).  ws:
 * fb_gemm_bf16_group_ws_bytes(probs, n) bytes. */
/* Rows of a bf16 GEMM operand gathered from up to three sources instead of
 * read from one matrix: the gathers of prepare_input (utils.py:126-196,
 * node_feats[nodes], edge_feats[eid]) and the time encoding (layers.py:17-29)
 * fused into the projection's operand load (TMA row gathers), so the
 * projection rows are never written to memory.  The operand's columns come in
 * nseg (1..3) segments, each starting and ending on a multiple of 64 columns:
 * segment s covers [s ? end[s-1] : 0, end[s]), and its row r is row
 * idx[s][r] (idx[s] NULL: row r) of the bf16 matrix tab[s] (tab_rows[s] rows,
 * tab_cols[s] data columns, leading dimension tab_ld[s], a multiple of 8; tab
 * 16-byte aligned).  Columns past tab_cols[s] read as zeros; row indices are
 * clamped into [0, tab_rows[s]). */
typedef struct fb_bf16_row_gather {
  int nseg;
  int end[3];
  const uint16_t *tab[3];
  int64_t tab_rows[3], tab_ld[3];
  int tab_cols[3];
  const int32_t *idx[3];
} fb_bf16_row_gather;

typedef struct fb_gemm_bf16_problem {
  int kind;
  const uint16_t *A; int64_t lda;
  const uint16_t *A2; int64_t lda2; int k1;
  const uint16_t *B; int64_t ldb;
  const float *bias;
  float *C; int64_t ldc;
  int64_t M; const int32_t *M_dev;
  int N, K;
  int accumulate;
  float *db; int db_accumulate;
  int ka;        /* NT / NN with A2: data columns of A (<= k1; 0 means k1); A's
                    columns [ka, k1) read as zeros, so k1 can round A's width up
                    to the 8-column boundary where A2's block of B starts */
  int nseg;      /* TN only, 0..3: X's columns come in segments -- columns
                    [seg_at[i], seg_at[i] + seg_len[i]) land in C's columns from
                    seg_to[i] (ascending, within [0, K)); columns of X outside
                    them are skipped.  The weight gradient over a bf16
                    projection row in one problem; the kernel then tiles X's
                    columns along the MMA's M side, which reads X once */
  int seg_at[3], seg_len[3], seg_to[3];
  int c_bf16;    /* NT / NN: C is bf16 (bit patterns, round to nearest even; no
                    accumulate) -- the K|V projection feeding the attention's
                    bf16 K|V path */
  const fb_bf16_row_gather *gather;   /* NT (no A2): A's rows, A unused; TN with
                    nseg > 0: X's rows, B unused; K = the last segment's end.
                    NULL: the operand is the matrix */
  const float *add;                   /* NT / NN, or NULL: C[m, n] (+)= ... +
                    add[add_idx[m] * ld_add + n] (an fp32 table of add_rows rows,
                    ld_add >= N; indices clamped into it), added before the bf16
                    rounding -- a product whose input rows repeat a few distinct
                    rows, computed once per row in the table */
  const int32_t *add_idx;
  int64_t ld_add, add_rows;
} fb_gemm_bf16_problem;
size_t fb_gemm_bf16_group_ws_bytes(const fb_gemm_bf16_problem *probs, int n);
int fb_gemm_bf16_group(const fb_gemm_bf16_problem *probs, int n, void *ws, size_t ws_bytes, cudaStream_t stream);
/* fp32 -> bf16 (round to nearest even) block copies, one launch for a list:
 * job i copies src [rows, cols] (leading dimension lds) into dst (ldd); rows
 * at or past *rows_dev are skipped when rows_dev is given.  At most
 * FB_CAST_MAX_JOBS jobs per call.  Used for the bf16 copies of the
 * projection weights (column segments placed at 8-element boundaries) and of
 * fp32 activations that feed bf16 GEMMs. */
enum { FB_CAST_MAX_JOBS = 32 };
typedef struct fb_cast_job {
  const float *src; int64_t lds;
  uint16_t *dst; int64_t ldd;
  int64_t rows; const int32_t *rows_dev;
  int cols; int pad_;
} fb_cast_job;
int fb_cast_bf16(const fb_cast_job *jobs, int n, cudaStream_t stream);
/* Synthetic feature tables on the device: dst[rows, ldd] (bf16) gets seeded
 * N(0, 1) values in columns < cols (Box-Muller over a counter hash of
 * (seed, element)) and zeros in the padding columns.  ldd even. */
int fb_fill_normal_bf16(uint16_t *dst, int64_t rows, int cols, int64_t ldd, uint64_t seed, cudaStream_t stream);
/* db[n] (+)= sum_m G[m, n]; deterministic.  ws: fb_colsum_ws_bytes(M, N). */
size_t fb_colsum_ws_bytes(int64_t M, int N);
int fb_colsum(const float *G, int64_t ldg, float *db, int64_t M, const int32_t *M_dev, int N,
              int accumulate, void *ws, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* Layer tail and edge predictor (layers.py:213-223, layers.py:31-50,        */
/* train.py:205-206).                                                         */
/* ------------------------------------------------------------------------- */
/* y = relu(dropout(z)), out = LayerNorm(y; gamma, beta, eps) per row.  Rows at
 * or past the count (n_rows_dev overrides n_rows) get out = 0, and so do all
 * rows when gate_dev is given and *gate_dev == 0 (a block without edges
 * outputs zeros, layers.py:101-102; the backward then gives dz = 0).  Dropout keeps a
 * value when u >= drop_p, u from Philox keyed by (seed, offset or *offset_dev),
 * or from mask_u [n_rows, dim] when given; kept values scale by 1/(1-p).
 * dim % 4 == 0, dim <= 512, 16-byte aligned rows. */
int fb_layer_tail_fwd(const float *z, int64_t ldz, const float *gamma, const float *beta, float eps,
                      float drop_p, uint64_t seed, uint64_t offset, const int64_t *offset_dev,
                      const float *mask_u, float *y, int64_t ldy, float *out, int64_t ldo, int64_t n_rows,
                      const int32_t *n_rows_dev, const int32_t *gate_dev, int dim, cudaStream_t stream);
/* Backward from dout and the saved y: dz, and dgamma += sum dout*xhat,
 * dbeta += sum dout (deterministic).  ws: fb_layer_tail_bwd_ws_bytes. */
size_t fb_layer_tail_bwd_ws_bytes(int64_t n_rows, int dim);
int fb_layer_tail_bwd(const float *dout, int64_t lddo, const float *y, int64_t ldy, const float *gamma,
                      float eps, float drop_p, float *dz, int64_t lddz, float *dgamma, float *dbeta,
                      int64_t n_rows, const int32_t *n_rows_dev, const int32_t *gate_dev, int dim, void *ws,
                      cudaStream_t stream);
/* EdgePredictor scores and BCE-with-logits loss, forward and backward:
 * S = src_fc(h_src) [B, dim], P = dst_fc([h_pos; h_neg]) [2B, dim];
 * x = relu(S_i + P_.) . w_o + b_o;  *loss = mean bce(x_pos, 1) + mean bce(x_neg, 0);
 * writes dS, dP; dw_o += ..., *db_o += ...; scores [2B] optional.  Deterministic;
 * ws: fb_edge_predictor_loss_ws_bytes(B, dim) bytes. */
size_t fb_edge_predictor_loss_ws_bytes(int64_t B, int dim);
int fb_edge_predictor_loss(const float *S, int64_t lds, const float *P, int64_t ldp, const float *w_o,
                           const float *b_o, int64_t B, int dim, float *loss, float *dS, int64_t ldds,
                           float *dP, int64_t lddp, float *dw_o, float *db_o, float *scores, void *ws,
                           cudaStream_t stream);
/* Q-side gradients that depend on v = sum over rows of dQ only:
 * db_q += v; db_t[c] -= sin(b_t[c]) sum_j v[j] W_q[j, dn + c]; and with qin0
 * (the single shared Q input row) dW_q[j, c] += v[j] qin0[c]. */
int fb_q_time_bwd(const float *v, int D, const float *W_q, int64_t ldwq, int dn, int dtime,
                  const float *b_t, const float *qin0, float *dW_q, int64_t lddwq, float *db_q,
                  float *db_t, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* Optimizer (torch.optim.Adam, train.py:128) over one flat fp32 buffer.      */
/* ------------------------------------------------------------------------- */
/* p, g, m, v: n floats each, 16-byte aligned.  *step (device) is the number of
 * steps taken so far and advances by one per call; *done (device, zero before
 * the first call) is the call's CTA counter and is left at zero. */
int fb_adam_step(float *p, const float *g, float *m, float *v, int64_t n, float lr, float beta1,
                 float beta2, float eps, int64_t *step, uint32_t *done, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* TGN node memory (memorys.py:6-182, 270-304).  Tables live on the device:  */
/* memory [N, dmem], mem_ts [N], mailbox [N, mailbox_size, dmail],           */
/* mailbox_ts [N, mailbox_size], next_pos [N] (int32).                       */
/* ------------------------------------------------------------------------- */
/* MailBox.prep_input_mails (memorys.py:51-73) fused with the time encoding of
 * GRUMemeoryUpdater.forward (memorys.py:286-289): for source rows r < *n_dev
 * (all n without it), id = nodes[r]:
 *   h0[r] = memory[id],  dtm[r] = ts[r] - mem_ts[id] (dtm may be NULL),
 *   x[r]  = [mailbox[id] (dmail = mailbox_size * mail width) | cos(w dtm + b)]. */
int fb_mem_gather(const int32_t *nodes, const float *ts, int64_t n, const int32_t *n_dev,
                  const float *memory, int dmem, const float *mem_ts, const float *mailbox, int dmail,
                  const float *w, const float *b, int dtime, float *x, int64_t ldx, float *h0, float *dtm,
                  cudaStream_t stream);
/* torch.nn.GRUCell gates (the updater of memorys.py:272-304) from the products
 * gi = x W_ih^T + b_ih and gh = h0 W_hh^T + b_hh ([n, 3H], gates r, z, n):
 * writes h1 = (1 - z) n + z h0 and keeps (r, z, n) in gi for fb_gru_bwd. */
int fb_gru_fwd(float *gi, const float *gh, const float *h0, float *h1, int64_t n, const int32_t *n_dev, int H,
               cudaStream_t stream);
/* Backward of fb_gru_fwd for dh1 (row stride ld_dh): overwrites gi with d(gi)
 * and gh with d(gh); h0 (the stored memory) gets no gradient. */
int fb_gru_bwd(float *gi, float *gh, const float *h0, const float *dh1, int64_t ld_dh, int64_t n,
               const int32_t *n_dev, int H, cudaStream_t stream);
/* MailBox.update_mailbox, deliver_to 'self', mail_combine 'last'
 * (memorys.py:101-142): the n positive edges (roots [src | dst | neg], h the
 * updated memory of those roots, f the edge features of the batch's edges
 * e0 .. e0+n-1 with e0 = *e0_dev, a device int64, 0 when NULL) deliver
 * [h_self | h_other | f] to both endpoints; of several
 * mails to one node the last in the reference's interleaved order wins.
 * last [N] (uint64, zero-initialised), gen and done (uint32, gen = 1, done = 0
 * initially) are the write-order bookkeeping, advanced on the device. */
int fb_mailbox_update_self(const int32_t *roots, const float *root_ts, int64_t n, const float *h, int64_t ldh,
                           int dmem, const float *f, int64_t ldf, int de, const int64_t *e0_dev, float *mailbox,
                           float *mailbox_ts, int32_t *next_pos, int mailbox_size, unsigned long long *last,
                           uint32_t *gen, uint32_t *done, cudaStream_t stream);
/* MailBox.update_memory (memorys.py:84-99): memory[roots[k]] = h[k],
 * mem_ts[roots[k]] = root_ts[k] for k < 2n, the last occurrence winning. */
int fb_memory_update(const int32_t *roots, const float *root_ts, int64_t n, const float *h, int64_t ldh, int dmem,
                     float *memory, float *mem_ts, unsigned long long *last, uint32_t *gen, uint32_t *done,
                     cudaStream_t stream);

/* APAN's TransformerMemoryUpdater (memorys.py:342-385) input: for roots r <
 * *n_dev (all n without it), slot s < slots, id = nodes[r]:
 *   x[r * slots + s] = [mailbox[id, s] (dmail) | cos(w (ts[r] - mailbox_ts[id, s]) + b)],
 *   dts[r * slots + s] = ts[r] - mailbox_ts[id, s],  h0[r] = memory[id]. */
int fb_mail_slots_gather(const int32_t *nodes, const float *ts, int64_t n, const int32_t *n_dev,
                         const float *memory, int dmem, const float *mailbox, const float *mailbox_ts, int slots,
                         int dmail, const float *w, const float *b, int dtime, float *x, int64_t ldx, float *h0,
                         float *dts, cudaStream_t stream);
/* out = LayerNorm(x + res; gamma, beta, eps) per row ([n, D], contiguous), the
 * residual step of memorys.py:378-379; xhat [n, D] and rstd [n] are kept for
 * the backward. */
int fb_add_layernorm_fwd(const float *x, const float *res, const float *gamma, const float *beta, float eps,
                         float *out, float *xhat, float *rstd, int64_t n, const int32_t *n_dev, int D,
                         cudaStream_t stream);
/* dx (the gradient of x and of res), dgamma += , dbeta += ; deterministic.
 * D <= 1024; ws: fb_add_layernorm_bwd_ws_bytes(n, D) bytes. */
size_t fb_add_layernorm_bwd_ws_bytes(int64_t n, int D);
int fb_add_layernorm_bwd(const float *dout, const float *xhat, const float *rstd, const float *gamma, float *dx,
                         float *dgamma, float *dbeta, int64_t n, const int32_t *n_dev, int D, void *ws,
                         cudaStream_t stream);
/* MailBox.update_mailbox, deliver_to 'neighbors', mail_combine 'last'
 * (memorys.py:143-178, APAN): nodes [2n + E] are the block's nodes (the 2n
 * positive roots, then the node sampled for each edge), row [E] each edge's
 * root.  Root j receives its own mail [h[j] | h[j +- n] | f[e0 + j mod n]] with
 * time root_ts[j]; the node of edge e receives the mail of root row[e].  Of
 * several mails to one node the last in that list wins; it goes to slot
 * next_pos[node], which then advances modulo mailbox_size.  E = *E_dev when
 * given (E_cap rows allocated).  last / gen / done as fb_mailbox_update_self. */
int fb_mailbox_update_neighbors(const int32_t *nodes, const int32_t *row, const float *root_ts, int64_t n,
                                const int32_t *E_dev, int64_t E_cap, const float *h, int64_t ldh, int dmem,
                                const float *f, int64_t ldf, int de, const int64_t *e0_dev, float *mailbox,
                                float *mailbox_ts, int32_t *next_pos, int mailbox_size, unsigned long long *last,
                                uint32_t *gen, uint32_t *done, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FAST_B200_H */
