/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference temporal
 * sampler, used as the checker for the CUDA sampler.  Only tests/, smoke()
 * and bench.py's cpu_baseline leg load this library; the product never does.
 *
 * Restates NoneBone/FAST getSamplerCore/sampler_core.cpp single-threaded:
 *   orc_reset          <- ParallelSampler::reset            sampler_core.cpp:122-131
 *   orc_update_ptr     <- ParallelSampler::update_ts_ptr    sampler_core.cpp:133-157
 *   orc_sample_window  <- sample_layer per-root body        sampler_core.cpp:517-583
 *                         (+ add_neighbor                   sampler_core.cpp:159-181)
 *   orc_cnt            <- combine_coo cntE (NODE_CNT path)  sampler_core.cpp:384-410
 *   orc_dedup          <- combine_coo uniE/invE             sampler_core.cpp:414-451
 * Uniform sampling draws with libc rand_r seeded with 0, which is what the
 * reference does with one OpenMP thread (loc_seed = tid, :501), so with one
 * reference thread the two agree bit for bit.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void orc_reset(const int32_t *indptr, int32_t *ptr, int64_t n_nodes)
{
    for (int64_t i = 0; i < n_nodes; i++) ptr[i] = indptr[i];
}

/* Forward-only scan from the stored pointer to the last edge whose timestamp
 * is <= root_ts + offset - 1e-7f, exactly as the reference loop does. */
void orc_update_ptr(const int32_t *indptr, const float *ts, int32_t *ptr,
                    const int32_t *roots, const float *root_ts, int64_t R, float offset)
{
    for (int64_t i = 0; i < R; i++) {
        int32_t n = roots[i];
        float thr = root_ts[i] + offset - 1e-7f;
        for (int64_t j = ptr[n]; j < indptr[n + 1]; j++) {
            if (ts[j] > thr) {
                if (j != ptr[n]) ptr[n] = (int32_t)(j - 1);
                break;
            }
            if (j == indptr[n + 1] - 1) ptr[n] = (int32_t)j;
        }
    }
}

/* First index in [lo, hi) whose ts is > v (std::upper_bound). */
static int64_t upper_bound_f(const float *ts, int64_t lo, int64_t hi, float v)
{
    while (lo < hi) {
        int64_t mid = lo + (hi - lo) / 2;
        if (v < ts[mid]) hi = mid; else lo = mid + 1;
    }
    return lo;
}

/*
 * Samples one history slot of one layer for R roots.  Writes the edges in
 * root order into row/col/eid (length E) and the per-edge tail of
 * ts/dts/nodes at offset R (the caller fills the first R entries with the
 * roots).  Returns E.  `state` is the rand_r state (seed 0 == one thread).
 */
int64_t orc_sample_layer(const int32_t *indptr, const int32_t *indices, const int32_t *eidv,
                         const float *ts, const int32_t *ptr_s, const int32_t *ptr_e,
                         int use_ptr, int num_history, float window_duration, float offset,
                         const int32_t *roots, const float *root_ts, int64_t R, int neighs,
                         int recent, int prop_time, unsigned int *state,
                         int32_t *row, int32_t *col, int32_t *eid_out, float *ts_out,
                         float *dts_out, int32_t *nodes_out)
{
    int64_t E = 0;
    for (int64_t j = 0; j < R; j++) {
        int32_t n = roots[j];
        float nts = root_ts[j];
        int64_t s, e;
        if (use_ptr) {
            s = ptr_s[n];
            e = ptr_e[n];
        } else if (num_history == 1) {
            s = indptr[n];
            int64_t ub = upper_bound_f(ts, indptr[n], indptr[n + 1], nts);
            e = ub - 1 > s ? ub - 1 : s;
        } else {
            float lo_t = nts + offset - window_duration;
            int64_t ub = upper_bound_f(ts, indptr[n], indptr[n + 1], lo_t);
            s = ub - 1 > indptr[n] ? ub - 1 : indptr[n];
            int64_t ub2 = upper_bound_f(ts, indptr[n], indptr[n + 1], nts + offset);
            e = ub2 - 1 > s ? ub2 - 1 : s;
        }
        float keep_thr = nts + offset - 1e-7f;
        if (recent || (e - s < neighs)) {
            int64_t lo = (e - neighs) > s ? (e - neighs) : s;
            for (int64_t k = e; k > lo; k--) {
                if (ts[k] < keep_thr) {
                    row[E] = (int32_t)j;
                    col[E] = (int32_t)(R + E);
                    eid_out[E] = eidv[k];
                    ts_out[R + E] = prop_time ? nts : ts[k];
                    dts_out[R + E] = nts - ts[k];
                    nodes_out[R + E] = indices[k];
                    E++;
                }
            }
        } else {
            for (int i = 0; i < neighs; i++) {
                int64_t picked = s + rand_r(state) % (e - s + 1);
                if (ts[picked] < keep_thr) {
                    row[E] = (int32_t)j;
                    col[E] = (int32_t)(R + E);
                    eid_out[E] = eidv[picked];
                    ts_out[R + E] = prop_time ? nts : ts[picked];
                    dts_out[R + E] = nts - ts[picked];
                    nodes_out[R + E] = indices[picked];
                    E++;
                }
            }
        }
    }
    return E;
}

/* cntE: prefix over runs of equal row ids (non-empty rows only); an empty
 * block yields an empty cntE.  Returns the number of entries written. */
int64_t orc_cnt(const int32_t *row, int64_t E, int32_t *cnt)
{
    if (E == 0) return 0;
    int64_t m = 0;
    cnt[m++] = 0;
    for (int64_t i = 1; i < E; i++)
        if (row[i] != row[i - 1]) cnt[m++] = (int32_t)i;
    cnt[m++] = (int32_t)E;
    return m;
}

/* uniE in first-appearance order and invE such that uniE[invE[i]] == eid[i]. */
int64_t orc_dedup(const int32_t *eid, int64_t E, int32_t *uniE, int32_t *invE)
{
    if (E == 0) return 0;
    int64_t cap = 1;
    while (cap < 2 * E) cap <<= 1;
    int32_t *keys = (int32_t *)malloc(sizeof(int32_t) * cap);
    int32_t *vals = (int32_t *)malloc(sizeof(int32_t) * cap);
    for (int64_t i = 0; i < cap; i++) keys[i] = -1;
    int64_t nu = 0;
    for (int64_t i = 0; i < E; i++) {
        uint32_t h = ((uint32_t)eid[i] * 2654435761u) & (uint32_t)(cap - 1);
        for (;;) {
            if (keys[h] == -1) {
                keys[h] = eid[i];
                vals[h] = (int32_t)nu;
                uniE[nu] = eid[i];
                invE[i] = (int32_t)nu;
                nu++;
                break;
            }
            if (keys[h] == eid[i]) { invE[i] = vals[h]; break; }
            h = (h + 1) & (uint32_t)(cap - 1);
        }
    }
    free(keys);
    free(vals);
    return nu;
}
