/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the TRIDENT lossless IVF query path.
 *
 * Nothing in the product (trident_b200/) links, loads or calls this file. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only as the checker.
 *
 * It is a plain-C restatement of the reference algorithm (mazaiying/TRIDENT), written from the
 * reference's behaviour, not copied from it. Each function names the reference lines it follows.
 * Paths are relative to the reference project root.
 *
 *   oracle_l2_ref_order      exact FP32 squared L2 in the reference GPU summation order
 *                            (src/trident_v4_kernels.cu:321-336 chain, :11-17 butterfly; the
 *                            Stage-Z refine at :870-883 uses the identical loop)
 *   oracle_topk_insert       the (distance asc, id asc) insertion rule, :19-39
 *   oracle_probe_select_f64  top-nprobe lists by float64 direct ||q-c||^2, ties to the smaller list id
 *                            (tie rule :117-161; float64 coarse step benchmarks/phase4b_suite.py:191-197)
 *   oracle_ivf_search        exact IVF-Flat top-K over the probed lists
 *                            (benchmarks/phase8_ooc_100m_4080.py:141-204, with the distance above)
 *   oracle_rotate_f64        the PCA rotation (q - mu) R in float64, sequential in k
 *                            (benchmarks/phase4a_suite.py:148-155 applies it to the base rows)
 *   oracle_stage_y_profile   the Stage-Y lower bound (src/trident_v4_kernels.cu:725-780) evaluated
 *                            under each query's final K-th distance: per-pair scanned 32-dim
 *                            blocks and survivors, the counters of :700-704/:774-795
 *
 * Build: oracle/build_oracle.py (gcc, -ffp-contract=off so that no expression is re-associated
 * or fused beyond the explicit fmaf/fma calls).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define ORACLE_VERSION 3

int oracle_version(void) { return ORACLE_VERSION; }

static void set_threads(int nthreads) {
    if (nthreads > 0) omp_set_num_threads(nthreads);
}

int oracle_max_threads(void) { return omp_get_max_threads(); }

/* Exact FP32 squared L2 distance in the reference's GPU order.
 * Lane l of a warp accumulates fmaf over d = 4l + 128k + j (k ascending, j = 0..3) while d+3 < D,
 * then a scalar tail over [d, min(d+4, D)); the 32 lane partials are then combined by the
 * shfl_down butterfly (offsets 16, 8, 4, 2, 1) and lane 0's value is the distance. */
float oracle_l2_ref_order(const float* x, const float* q, int D) {
    float part[32];
    for (int l = 0; l < 32; ++l) {
        float p = 0.0f;
        int d = 4 * l;
        for (; d + 3 < D; d += 128) {
            for (int j = 0; j < 4; ++j) {
                float df = x[d + j] - q[d + j];
                p = fmaf(df, df, p);
            }
        }
        for (int dr = d; dr < d + 4 && dr < D; ++dr) {
            float df = x[dr] - q[dr];
            p = fmaf(df, df, p);
        }
        part[l] = p;
    }
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) part[l] = part[l] + part[l + off];
    return part[0];
}

/* Insert (dv, iv) into the sorted list (d[0..K), id[0..K)) under the total order (d asc, id asc). */
void oracle_topk_insert(float* d, int64_t* id, int K, float dv, int64_t iv) {
    if (dv < d[K - 1] || (dv == d[K - 1] && iv < id[K - 1])) {
        d[K - 1] = dv;
        id[K - 1] = iv;
        for (int j = K - 1; j > 0; --j) {
            if (d[j] < d[j - 1] || (d[j] == d[j - 1] && id[j] < id[j - 1])) {
                float td = d[j - 1]; d[j - 1] = d[j]; d[j] = td;
                int64_t ti = id[j - 1]; id[j - 1] = id[j]; id[j] = ti;
            } else {
                break;
            }
        }
    }
}

/* float64 direct squared distance: the oracle's definition of the coarse distance (the reference
 * fixes no float64 summation order; this one is chosen so that a warp evaluates it in parallel
 * with coalesced loads). Lane l in 0..31 sums fma(df, df, .) over d = l, l + 32, l + 64, ... < D
 * in ascending d from 0.0; the 32 lane sums are then added in order l = 0..31. The GPU's exact
 * re-check evaluates the same expression in the same order. */
double oracle_l2_f64(const float* a, const float* b, int D) {
    double total = 0.0;
    for (int l = 0; l < 32; ++l) {
        double acc = 0.0;
        for (int d = l; d < D; d += 32) {
            double df = (double)a[d] - (double)b[d];
            acc = fma(df, df, acc);
        }
        total = (l == 0) ? acc : total + acc;
    }
    return total;
}

typedef struct { double d; int32_t c; } dc_pair;

static int cmp_dc(const void* a, const void* b) {
    const dc_pair* x = (const dc_pair*)a;
    const dc_pair* y = (const dc_pair*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return (x->c < y->c) ? -1 : (x->c > y->c);
}

/* Top-nprobe lists per query, ascending by (float64 distance, list id). */
int oracle_probe_select_f64(const float* xq, const float* cent, int64_t B, int D, int nlist,
                            int nprobe, int32_t* out_cids, double* out_d, int nthreads) {
    if (nprobe > nlist || nprobe <= 0) return 1;
    set_threads(nthreads);
    int err = 0;
#pragma omp parallel
    {
        dc_pair* buf = (dc_pair*)malloc(sizeof(dc_pair) * (size_t)nlist);
        if (!buf) {
#pragma omp atomic write
            err = 2;
        }
#pragma omp for schedule(dynamic, 4)
        for (int64_t q = 0; q < B; ++q) {
            if (!buf) continue;
            const float* qr = xq + q * (int64_t)D;
            for (int c = 0; c < nlist; ++c) {
                buf[c].d = oracle_l2_f64(qr, cent + (int64_t)c * D, D);
                buf[c].c = c;
            }
            qsort(buf, (size_t)nlist, sizeof(dc_pair), cmp_dc);
            for (int p = 0; p < nprobe; ++p) {
                out_cids[q * nprobe + p] = buf[p].c;
                if (out_d) out_d[q * nprobe + p] = buf[p].d;
            }
        }
        free(buf);
    }
    return err;
}

/* Exact IVF-Flat: for each query, every row of every probed list, distance in reference order,
 * top-K by (d asc, id asc). Lists with id < 0 are skipped. Empty slots stay (+inf, -1). */
int oracle_ivf_search(const float* xq, int64_t B, int D, const int32_t* probe_cids, int nprobe,
                      const int64_t* vec_off, const float* xb_sorted, const int32_t* orig_ids,
                      int K, float* out_d, int64_t* out_i, int nthreads) {
    if (K <= 0) return 1;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t q = 0; q < B; ++q) {
        const float* qr = xq + q * (int64_t)D;
        float* td = out_d + q * K;
        int64_t* ti = out_i + q * K;
        for (int j = 0; j < K; ++j) { td[j] = INFINITY; ti[j] = -1; }
        for (int p = 0; p < nprobe; ++p) {
            int32_t c = probe_cids[q * nprobe + p];
            if (c < 0) continue;
            for (int64_t v = vec_off[c]; v < vec_off[c + 1]; ++v) {
                float dv = oracle_l2_ref_order(xb_sorted + v * (int64_t)D, qr, D);
                oracle_topk_insert(td, ti, K, dv, (int64_t)orig_ids[v]);
            }
        }
    }
    return 0;
}

/* (q - mu) R in float64 with k ascending and fma, rounded to float32 at the end; zero-padded to
 * D_pad columns. R is [D, D] row-major (column d is principal direction d). */
int oracle_rotate_f64(const float* xq, int64_t B, int D, int D_pad, const double* mu,
                      const double* R, float* out, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t q = 0; q < B; ++q) {
        const float* qr = xq + q * (int64_t)D;
        for (int d = 0; d < D_pad; ++d) {
            double acc = 0.0;
            if (d < D) {
                for (int k = 0; k < D; ++k) acc = fma((double)qr[k] - mu[k], R[(int64_t)k * D + d], acc);
            }
            out[q * D_pad + d] = (float)acc;
        }
    }
    return 0;
}

/* Stage-Y profile under the final threshold. For query q and every row x of every probed list,
 * evaluate the blocked lower bound of src/trident_v4_kernels.cu:725-780,
 *   u_d = |code_d * delta_cd + (vmin_cd - qrot_d)|,  l_d = max(u_d - eps_cd, 0),  acc += l_d^2,
 * one 32-dim block at a time, and stop after the first block whose running sum exceeds tau_safe[q].
 * codes are the blocked layout [tiles][num_blocks][T][32] (tile t of list c holds rows
 * vec_off[c] + (t - tile_off[c]) * T + v). Outputs, per query: candidate rows, scanned blocks and
 * survivors (rows whose full-D bound stays <= tau_safe). Per sorted row (optional): the largest
 * number of blocks any query scanned (the bytes model's nb*), plus one when some query kept the row
 * through the full bound (so num_blocks + 1 marks a row that must be read in FP32). */
int oracle_stage_y_profile(int64_t B, int D_pad, int nprobe, const int32_t* probe_cids,
                           const int64_t* vec_off, const int64_t* tile_off, int T,
                           const uint8_t* codes, const float* vmin, const float* delta,
                           const float* eps, const float* qrot, const float* tau_safe,
                           int64_t* out_cand, int64_t* out_blocks, int64_t* out_surv,
                           int32_t* row_max_blocks, int nthreads) {
    set_threads(nthreads);
    const int nb = D_pad / 32;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t q = 0; q < B; ++q) {
        int64_t cand = 0, blocks = 0, surv = 0;
        const float* qr = qrot + q * (int64_t)D_pad;
        const float ts = tau_safe[q];
        for (int p = 0; p < nprobe; ++p) {
            int32_t c = probe_cids[q * nprobe + p];
            if (c < 0) continue;
            const float* vm = vmin + (int64_t)c * D_pad;
            const float* dl = delta + (int64_t)c * D_pad;
            const float* ep = eps + (int64_t)c * D_pad;
            for (int64_t v = vec_off[c]; v < vec_off[c + 1]; ++v) {
                int64_t local = v - vec_off[c];
                int64_t tile = tile_off[c] + local / T;
                int slot = (int)(local % T);
                float acc = 0.0f;
                int used = 0;
                int alive = 1;
                for (int b = 0; b < nb && alive; ++b) {
                    const uint8_t* cb = codes + ((tile * nb + b) * (int64_t)T + slot) * 32;
                    for (int j = 0; j < 32; ++j) {
                        int d = b * 32 + j;
                        float base = vm[d] - qr[d];
                        float u = fabsf(fmaf((float)cb[j], dl[d], base));
                        float l = fmaxf(u - ep[d], 0.0f);
                        acc = fmaf(l, l, acc);
                    }
                    used = b + 1;
                    if (acc > ts) alive = 0;
                }
                cand += 1;
                blocks += used;
                surv += alive;
                if (row_max_blocks) {
                    /* blocks scanned, plus one if the row survived the full bound */
                    const int32_t enc = used + alive;
                    int32_t* slotp = &row_max_blocks[v];
                    int32_t cur;
#pragma omp atomic read
                    cur = *slotp;
                    while (enc > cur) {
                        if (__sync_bool_compare_and_swap(slotp, cur, enc)) break;
#pragma omp atomic read
                        cur = *slotp;
                    }
                }
            }
        }
        out_cand[q] = cand;
        out_blocks[q] = blocks;
        out_surv[q] = surv;
    }
    return 0;
}
