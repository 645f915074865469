// The list scan of the query path: the TRIDENT cascade (Stage X threshold seeding, Stage Y SQ8
// lower-bound early exit, Stage Z exact FP32 refinement, per-query top-K) and the CM-FP32 exact
// scan, plus the top-K merges.
//
// Reference: trident_cluster_major_scan_kernel (src/trident_v4_kernels.cu:530-962, mode 2),
// trident_cm_fp32_scan_kernel (:269-374, mode 10) and trident_merge_topk_kernel (:966-1036).
// The reference runs one CTA per (list, query) pair and relies on L2 to share a list's codes among
// the ~40-60 queries that probe it. On B200 one CTA takes a work item (list c, up to G queries):
// each thread owns one row of a tile, keeps that row's first 32-dim code block in registers, and
// evaluates the lower bound for every query of the item, so a tile's codes cross HBM/L2 once per
// item instead of once per query. The item's queries keep their thresholds in shared memory and
// share them across CTAs through a per-query atomicMin (any CTA's K-th exact distance bounds the
// query's final K-th distance), so pruning tightens as the whole GPU makes progress.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

struct ScanArgs {
    const float* xb;
    const int32_t* oid;
    const int64_t* row_off;
    const int64_t* tile_off;
    const uint8_t* codes;
    const float* vmin;
    const float* delta;
    const float* eps;
    const float* xq;
    const float* qrot;
    const float* qinfo;
    const int4* items;
    const int32_t* n_items;
    int32_t* work_ctr;
    const int32_t* pair_q;
    const int32_t* pair_p;
    uint32_t* tau;
    float* cand_d;
    int32_t* cand_i;
    unsigned long long* stats;
    int D, D_pad, nb, K, nprobe, G;
    float rho;
};

constexpr int kMaxG = 32;

// Prune threshold for a query whose current K-th exact distance is tau: a row is dropped when its
// partial bound exceeds (sqrt(tau (1 + rho)) + sigma)^2. rho covers the float32 accumulation of
// the bound and of the exact distance, sigma the query-side roundings (Minkowski); the final
// factor covers the roundings of this expression.
__device__ __forceinline__ float prune_threshold(float tau, float sigma, float rho) {
    if (!(tau < kInf)) return kInf;
    const float s = sqrtf(tau * (1.0f + rho)) + sigma;
    return s * s * (1.0f + 1e-6f);
}

// Threshold implied by an SQ8 upper bound ub of one row: its exact FP32 distance is at most this.
__device__ __forceinline__ float ub_threshold(float ub, float sigma, float rho) {
    if (!(ub < kInf)) return kInf;
    const float s = sqrtf(ub * (1.0f + 2.0f * rho)) + sigma;
    return s * s * (1.0f + 2.0f * rho) * (1.0f + 1e-6f);
}

// Stage Y on one 32-dim block: acc += sum_d max(|code_d delta_d + (vmin_d - q~_d)| - eps_d, 0)^2
// (reference :750-767). base/dl/ep point at the block's 32 entries in shared memory.
__device__ __forceinline__ float lb_block(const uint4 w0, const uint4 w1, const float* __restrict__ base,
                                          const float* __restrict__ dl, const float* __restrict__ ep, float acc) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 b4 = *reinterpret_cast<const float4*>(base + 4 * i);
        const float4 d4 = *reinterpret_cast<const float4*>(dl + 4 * i);
        const float4 e4 = *reinterpret_cast<const float4*>(ep + 4 * i);
        float l;
        l = fmaxf(fabsf(fmaf(u8f(w[i], 0), d4.x, b4.x)) - e4.x, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(u8f(w[i], 1), d4.y, b4.y)) - e4.y, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(u8f(w[i], 2), d4.z, b4.z)) - e4.z, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(u8f(w[i], 3), d4.w, b4.w)) - e4.w, 0.0f); acc = fmaf(l, l, acc);
    }
    return acc;
}

// SQ8 upper bound on one block: acc += sum_d (|code_d delta_d + (vmin_d - q~_d)| + eps_d)^2
// (the reference's UB seeding, :630-675).
__device__ __forceinline__ float ub_block(const uint4 w0, const uint4 w1, const float* __restrict__ base,
                                          const float* __restrict__ dl, const float* __restrict__ ep, float acc) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 b4 = *reinterpret_cast<const float4*>(base + 4 * i);
        const float4 d4 = *reinterpret_cast<const float4*>(dl + 4 * i);
        const float4 e4 = *reinterpret_cast<const float4*>(ep + 4 * i);
        float a;
        a = fabsf(fmaf(u8f(w[i], 0), d4.x, b4.x)) + e4.x; acc = fmaf(a, a, acc);
        a = fabsf(fmaf(u8f(w[i], 1), d4.y, b4.y)) + e4.y; acc = fmaf(a, a, acc);
        a = fabsf(fmaf(u8f(w[i], 2), d4.z, b4.z)) + e4.z; acc = fmaf(a, a, acc);
        a = fabsf(fmaf(u8f(w[i], 3), d4.w, b4.w)) + e4.w; acc = fmaf(a, a, acc);
    }
    return acc;
}

__device__ __forceinline__ void load_block(const uint8_t* __restrict__ p, uint4& w0, uint4& w1) {
    w0 = __ldg(reinterpret_cast<const uint4*>(p));
    w1 = __ldg(reinterpret_cast<const uint4*>(p + 16));
}

template <int T, int KM, bool LB, bool UB, bool VEC4>
__global__ void __launch_bounds__(T, 512 / T) scan_kernel(const ScanArgs a) {
    constexpr int NW = T / 32;
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = a.G;
    const int D_pad = a.D_pad;
    float* s_base = reinterpret_cast<float*>(smem);
    float* s_dl = s_base + (LB ? G * D_pad : 0);
    float* s_ep = s_dl + (LB ? D_pad : 0);
    float* s_topd = s_ep + (LB ? D_pad : 0);
    int32_t* s_topi = reinterpret_cast<int32_t*>(s_topd + G * KM);
    float* s_sd = reinterpret_cast<float*>(s_topi + G * KM);
    uint16_t* s_sq = reinterpret_cast<uint16_t*>(s_sd + G * T);

    __shared__ int32_t s_qid[kMaxG], s_pp[kMaxG], s_cnt[kMaxG], s_pref[kMaxG + 1];
    __shared__ float s_tau[kMaxG], s_ts[kMaxG], s_sig[kMaxG];
    __shared__ int s_item;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, D = a.D, nb = a.nb;
    unsigned long long st_cand = 0, st_dims = 0, st_surv = 0, st_ins = 0, st_items = 0;

    for (;;) {
        if (tid == 0) s_item = atomicAdd(a.work_ctr, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= *a.n_items) break;
        const int4 item = a.items[it];
        const int c = item.x, pstart = item.y, n = item.z;
        ++st_items;
        if (tid < n) {
            const int q = a.pair_q[pstart + tid];
            s_qid[tid] = q;
            s_pp[tid] = a.pair_p[pstart + tid];
            const float sig = a.qinfo[(int64_t)q * QI_LEN + QI_SIGMA];
            const float tq = ld_volatile_f32(a.tau + q);
            s_sig[tid] = sig;
            s_tau[tid] = tq;
            s_ts[tid] = prune_threshold(tq, sig, a.rho);
            s_cnt[tid] = 0;
        }
        if (LB) {
            for (int d = tid; d < D_pad; d += T) {
                s_dl[d] = __ldg(a.delta + (int64_t)c * D_pad + d);
                s_ep[d] = __ldg(a.eps + (int64_t)c * D_pad + d);
            }
        }
        __syncthreads();
        if (LB) {
            for (int i = tid; i < n * D_pad; i += T) {
                const int j = i / D_pad, d = i - j * D_pad;
                s_base[i] = __ldg(a.vmin + (int64_t)c * D_pad + d) - __ldg(a.qrot + (int64_t)s_qid[j] * D_pad + d);
            }
        }
        for (int i = tid; i < n * KM; i += T) {
            s_topd[i] = kInf;
            s_topi[i] = -1;
        }
        __syncthreads();

        const int64_t r0 = a.row_off[c];
        const int L = (int)(a.row_off[c + 1] - r0);
        const int64_t t0 = a.tile_off[c];
        const int nt = (L + T - 1) / T;

        // ---- Stage X (optional): seed each query's threshold from SQ8 upper bounds of this list
        if (UB) {
            for (int t = 0; t < nt; ++t) {
                const int v = t * T + tid;
                const bool valid = v < L;
                const uint8_t* tp = a.codes + (size_t)(t0 + t) * nb * T * 32;
                for (int j = 0; j < n; ++j) {
                    float ub = kInf;
                    if (valid) {
                        float acc = 0.0f;
                        for (int b = 0; b < nb; ++b) {
                            uint4 w0, w1;
                            load_block(tp + ((size_t)b * T + tid) * 32, w0, w1);
                            acc = ub_block(w0, w1, s_base + j * D_pad + 32 * b, s_dl + 32 * b, s_ep + 32 * b, acc);
                        }
                        ub = acc;
                    }
                    s_sd[j * T + tid] = ub;
                }
                __syncthreads();
                for (int j = warp; j < n; j += NW) {
                    float* ld = s_topd + j * KM;
                    int32_t* li = s_topi + j * KM;
                    for (int k0 = 0; k0 < T; k0 += 32) {
                        const int k = k0 + lane;
                        const float ub = s_sd[j * T + k];
                        list_offer<KM>(ld, li, K, ub < kInf, ub, t * T + k, lane);
                    }
                }
                __syncthreads();
            }
            for (int j = warp; j < n; j += NW) {
                float* ld = s_topd + j * KM;
                int32_t* li = s_topi + j * KM;
                if (lane == 0) {
                    const float seed = ub_threshold(ld[K - 1], s_sig[j], a.rho);
                    float tq = s_tau[j];
                    if (seed < tq) {
                        tq = seed;
                        atomicMin(a.tau + s_qid[j], __float_as_uint(seed));
                    }
                    s_tau[j] = tq;
                    s_ts[j] = prune_threshold(tq, s_sig[j], a.rho);
                }
                __syncwarp();
                list_init<KM>(ld, li, lane);
            }
            __syncthreads();
        }

        for (int t = 0; t < nt; ++t) {
            const int v = t * T + tid;
            const bool valid = v < L;
            const int Lt = min(T, L - t * T);
            int total;
            if (LB) {
                // ---- Stage Y: blocked SQ8 lower bound with warp early exit
                const uint8_t* tp = a.codes + (size_t)(t0 + t) * nb * T * 32;
                uint4 c0 = make_uint4(0, 0, 0, 0), c1 = make_uint4(0, 0, 0, 0);
                if (valid) load_block(tp + (size_t)tid * 32, c0, c1);
                for (int j = 0; j < n; ++j) {
                    const float ts = s_ts[j];
                    const float* bj = s_base + j * D_pad;
                    float acc = lb_block(c0, c1, bj, s_dl, s_ep, 0.0f);
                    bool alive = valid && acc <= ts;
                    int used = 1;
                    for (int b = 1; b < nb; ++b) {
                        if (!__any_sync(TB_FULL, alive)) break;
                        if (alive) {
                            uint4 w0, w1;
                            load_block(tp + ((size_t)b * T + tid) * 32, w0, w1);
                            acc = lb_block(w0, w1, bj + 32 * b, s_dl + 32 * b, s_ep + 32 * b, acc);
                            alive = acc <= ts;
                            used = b + 1;
                        }
                    }
                    if (valid) {
                        st_cand += 1;
                        st_dims += 32u * (unsigned)used;
                        st_surv += alive ? 1u : 0u;
                    }
                    // survivor compaction (ballot / ffs leader / popc rank, reference :796-825)
                    const unsigned m = __ballot_sync(TB_FULL, alive);
                    if (m) {
                        const int leader = __ffs(m) - 1;
                        int pos = 0;
                        if (lane == leader) pos = atomicAdd(&s_cnt[j], __popc(m));
                        pos = __shfl_sync(TB_FULL, pos, leader);
                        if (alive) s_sq[j * T + pos + __popc(m & ((1u << lane) - 1u))] = (uint16_t)tid;
                    }
                }
                __syncthreads();
                if (warp == 0) {
                    int cj = lane < n ? s_cnt[lane] : 0;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int x = __shfl_up_sync(TB_FULL, cj, o);
                        if (lane >= o) cj += x;
                    }
                    s_pref[lane + 1] = cj;
                    if (lane == 0) s_pref[0] = 0;
                }
                __syncthreads();
                total = s_pref[n];
            } else {
                if (valid) st_cand += n, st_surv += n;
                total = n * Lt;
            }

            // ---- Stage Z: one warp per surviving (query, row), exact FP32 in the reference order
            for (int s = warp; s < total; s += NW) {
                int j, k, vv;
                if (LB) {
                    j = 0;
                    while (j + 1 < n && s_pref[j + 1] <= s) ++j;
                    k = s - s_pref[j];
                    vv = s_sq[j * T + k];
                } else {
                    j = s / Lt;
                    k = s - j * Lt;
                    vv = k;
                }
                const float* xr = a.xb + (r0 + (int64_t)t * T + vv) * D;
                const float* qr = a.xq + (int64_t)s_qid[j] * D;
                const float dist = exact_dist_warp<VEC4>(xr, qr, D, lane);
                if (lane == 0) s_sd[j * T + k] = dist;
            }
            __syncthreads();

            // ---- per-query top-K insertion, then threshold exchange
            for (int j = warp; j < n; j += NW) {
                const int cj = LB ? s_cnt[j] : Lt;
                float* ld = s_topd + j * KM;
                int32_t* li = s_topi + j * KM;
                for (int k0 = 0; k0 < cj; k0 += 32) {
                    const int k = k0 + lane;
                    const bool ok = k < cj;
                    const float d = ok ? s_sd[j * T + k] : kInf;
                    const int vv = ok ? (LB ? (int)s_sq[j * T + k] : k) : 0;
                    const int32_t id = ok ? __ldg(a.oid + r0 + (int64_t)t * T + vv) : 0;
                    st_ins += (unsigned)list_offer<KM>(ld, li, K, ok, d, id, lane);
                }
                if (lane == 0) {
                    const float kth = ld[K - 1];
                    const int q = s_qid[j];
                    float tq = s_tau[j];
                    if (kth < tq) {
                        tq = kth;
                        atomicMin(a.tau + q, __float_as_uint(kth));
                    }
                    const float g = ld_volatile_f32(a.tau + q);
                    if (g < tq) tq = g;
                    s_tau[j] = tq;
                    s_ts[j] = prune_threshold(tq, s_sig[j], a.rho);
                    s_cnt[j] = 0;
                }
            }
            __syncthreads();
        }

        // ---- emit this item's per-query lists into the (query, probe) candidate slots
        for (int i = tid; i < n * K; i += T) {
            const int j = i / K, k = i - j * K;
            float d = s_topd[j * KM + k];
            int32_t id = s_topi[j * KM + k];
            if (!(id >= 0 && d <= s_tau[j])) { d = kInf; id = -1; }
            const int64_t slot = ((int64_t)s_qid[j] * a.nprobe + s_pp[j]) * K + k;
            a.cand_d[slot] = d;
            a.cand_i[slot] = id;
        }
        __syncthreads();
    }

    if (a.stats) {
        unsigned long long v[5] = {st_cand, st_dims, st_surv, st_ins, (tid == 0) ? st_items : 0ull};
#pragma unroll
        for (int i = 0; i < 5; ++i) {
            unsigned long long x = v[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(TB_FULL, x, o);
            if (lane == 0 && x) atomicAdd(a.stats + i + (i == 4 ? 1 : 0), x);
        }
    }
}

// ------------------------------------------------------------------------------------------
// Merges
// ------------------------------------------------------------------------------------------
template <int KM>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ cand_d, const int32_t* __restrict__ cand_i,
                                                   int B, int K, int nprobe, int p_lo, int p_hi,
                                                   uint32_t* __restrict__ tau_out, float* __restrict__ out_d,
                                                   int64_t* __restrict__ out_i) {
    __shared__ float ld_all[8][KM];
    __shared__ int32_t li_all[8][KM];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= B) return;
    float* ld = ld_all[warp];
    int32_t* li = li_all[warp];
    list_init<KM>(ld, li, lane);
    __syncwarp();
    const int64_t base = ((int64_t)q * nprobe + p_lo) * K;
    const int n = (p_hi - p_lo) * K;
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        float d = kInf;
        int32_t id = -1;
        if (k < n) { d = cand_d[base + k]; id = cand_i[base + k]; }
        list_offer<KM>(ld, li, K, id >= 0, d, id, lane);
    }
    __syncwarp();
    if (out_d) {
        for (int k = lane; k < K; k += 32) {
            out_d[(int64_t)q * K + k] = ld[k];
            out_i[(int64_t)q * K + k] = (int64_t)li[k];
        }
    }
    // Every value ever stored in tau is the K-th distance of K distinct rows, hence an upper bound
    // of the final K-th distance: keep the smallest.
    if (tau_out && lane == 0) atomicMin(tau_out + q, __float_as_uint(ld[K - 1]));
}

template <int KM>
__global__ void __launch_bounds__(256) merge_shards_kernel(const float* __restrict__ d_in, const int64_t* __restrict__ i_in,
                                                          int R, int B, int K, float* __restrict__ out_d,
                                                          int64_t* __restrict__ out_i) {
    __shared__ float ld_all[8][KM];
    __shared__ int32_t li_all[8][KM];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= B) return;
    float* ld = ld_all[warp];
    int32_t* li = li_all[warp];
    list_init<KM>(ld, li, lane);
    __syncwarp();
    const int n = R * K;
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        float d = kInf;
        int64_t id = -1;
        if (k < n) {
            const int r = k / K, kk = k - r * K;
            d = d_in[((int64_t)r * B + q) * K + kk];
            id = i_in[((int64_t)r * B + q) * K + kk];
        }
        list_offer<KM>(ld, li, K, id >= 0, d, (int32_t)id, lane);
    }
    __syncwarp();
    for (int k = lane; k < K; k += 32) {
        out_d[(int64_t)q * K + k] = ld[k];
        out_i[(int64_t)q * K + k] = (int64_t)li[k];
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
static int km_for(int K) { return K <= 32 ? 32 : 128; }

static size_t scan_smem(const trident_index& idx, int K, int G, bool lb) {
    const int T = idx.tile_size;
    const int KM = km_for(K);
    size_t s = 0;
    if (lb) s += (size_t)(G + 2) * idx.D_pad * sizeof(float);
    s += (size_t)G * KM * (sizeof(float) + sizeof(int32_t));
    s += (size_t)G * T * sizeof(float);
    s += (size_t)G * T * sizeof(uint16_t);
    return s;
}

int scan_group_size(const trident_index& idx, int K) {
    // Two CTAs of 256 rows (or four of 128) per SM: about 100 KB of shared memory each.
    const size_t budget = (idx.tile_size == 256) ? 100 * 1024 : 50 * 1024;
    int G = kMaxG;
    while (G > 1 && scan_smem(idx, K, G, true) > budget) --G;
    return G;
}

template <int T, int KM, bool LB, bool UB, bool VEC4>
static cudaError_t launch_scan_t(const ScanArgs& a, size_t smem, int max_items, cudaStream_t st) {
    auto kern = scan_kernel<T, KM, LB, UB, VEC4>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, T, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    int grid = num_sms() * per_sm;
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    kern<<<grid, T, smem, st>>>(a);
    return cudaGetLastError();
}

template <int T, int KM>
static cudaError_t dispatch_mode(const ScanArgs& a, size_t smem, const ScanLaunch& sl, bool vec4, cudaStream_t st) {
    if (sl.lb) {
        if (sl.ub_seed) {
            return vec4 ? launch_scan_t<T, KM, true, true, true>(a, smem, sl.max_items, st)
                        : launch_scan_t<T, KM, true, true, false>(a, smem, sl.max_items, st);
        }
        return vec4 ? launch_scan_t<T, KM, true, false, true>(a, smem, sl.max_items, st)
                    : launch_scan_t<T, KM, true, false, false>(a, smem, sl.max_items, st);
    }
    return vec4 ? launch_scan_t<T, KM, false, false, true>(a, smem, sl.max_items, st)
                : launch_scan_t<T, KM, false, false, false>(a, smem, sl.max_items, st);
}

cudaError_t launch_scan(const trident_index& idx, const float* xq, const Workspace& ws, const ScanLaunch& sl,
                        unsigned long long* stats, cudaStream_t st) {
    if (sl.max_items <= 0) return cudaSuccess;
    ScanArgs a;
    a.xb = idx.xb_sorted;
    a.oid = idx.orig_ids_sorted;
    a.row_off = idx.list_row_off;
    a.tile_off = idx.list_tile_off;
    a.codes = idx.codes;
    a.vmin = idx.vmin;
    a.delta = idx.delta;
    a.eps = idx.eps;
    a.xq = xq;
    a.qrot = ws.qrot;
    a.qinfo = ws.qinfo;
    a.items = ws.items + sl.item_base;
    a.n_items = ws.ctr + sl.pass;
    a.work_ctr = ws.ctr + 2 + sl.pass;
    a.pair_q = ws.pair_q;
    a.pair_p = ws.pair_p;
    a.tau = ws.tau;
    a.cand_d = ws.cand_d;
    a.cand_i = ws.cand_i;
    a.stats = stats;
    a.D = idx.D;
    a.D_pad = idx.D_pad;
    a.nb = idx.num_blocks;
    a.K = sl.K;
    a.nprobe = sl.nprobe;
    a.G = sl.G;
    a.rho = idx.lb_rel_slack;
    const bool vec4 = (idx.D % 4) == 0 && (((uintptr_t)idx.xb_sorted | (uintptr_t)xq) & 15) == 0;
    const size_t smem = scan_smem(idx, sl.K, sl.G, sl.lb != 0);
    const int KM = km_for(sl.K);
    if (idx.tile_size == 256) {
        return KM == 32 ? dispatch_mode<256, 32>(a, smem, sl, vec4, st) : dispatch_mode<256, 128>(a, smem, sl, vec4, st);
    }
    return KM == 32 ? dispatch_mode<128, 32>(a, smem, sl, vec4, st) : dispatch_mode<128, 128>(a, smem, sl, vec4, st);
}

cudaError_t launch_merge(const Workspace& ws, int B, int K, int nprobe, int p_lo, int p_hi, uint32_t* tau_out,
                         float* out_d, int64_t* out_i, cudaStream_t st) {
    const int grid = (B + 7) / 8;
    if (K <= 32)
        merge_kernel<32><<<grid, 256, 0, st>>>(ws.cand_d, ws.cand_i, B, K, nprobe, p_lo, p_hi, tau_out, out_d, out_i);
    else
        merge_kernel<128><<<grid, 256, 0, st>>>(ws.cand_d, ws.cand_i, B, K, nprobe, p_lo, p_hi, tau_out, out_d, out_i);
    return cudaGetLastError();
}

cudaError_t launch_merge_shards(const float* d_in, const int64_t* i_in, int R, int B, int K, float* out_d,
                                int64_t* out_i, cudaStream_t st) {
    const int grid = (B + 7) / 8;
    if (K <= 32)
        merge_shards_kernel<32><<<grid, 256, 0, st>>>(d_in, i_in, R, B, K, out_d, out_i);
    else
        merge_shards_kernel<128><<<grid, 256, 0, st>>>(d_in, i_in, R, B, K, out_d, out_i);
    return cudaGetLastError();
}

}  // namespace tb
