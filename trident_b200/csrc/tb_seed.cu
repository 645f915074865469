// Stage X as a query-major kernel: each query's threshold starts at the K-th exact distance among
// a few hundred well-chosen rows of its nearest lists, before the list scan starts.
//
// The reference seeds thresholds with a warm-up scan: the p_init nearest lists of every query go
// through the full cascade first and their merged K-th distance becomes tau for the remaining
// probes (src/trident_v4_kernels.cu:1264-1276, :1334-1420). That warm-up pass is expensive on a
// GPU: its work items hold ~3 queries each (B * p_init pairs spread over nlist lists) and start
// with no threshold, so most rows run deep into the bound. Here one CTA per query ranks the rows
// of its p_init nearest lists by the SQ8-reconstructed partial distance over the leading
// kSeedBlocks blocks, refines the S best exactly (the reference's FP32 order, so the distances are
// the ones the final top-K holds) and stores their K-th distance as the query's threshold. The
// S rows are distinct rows of the index, so that value bounds the final K-th distance from above
// whichever rows were picked; the ranking only decides how tight it is. The main scan then covers
// every probe, the warm-up lists included.
#include <cuda_runtime.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

constexpr int kSeedThreads = 256;
constexpr int kSeedRowsMax = 8192;  // rows ranked per query: the first ones of its warm-up lists
constexpr int kSeedBlocks = 1;      // leading 32-dim blocks used for the ranking
constexpr int kSeedListsMax = 8;
constexpr int kSeedBits = 12;       // key bits the selection resolves below the keys' common prefix

struct SeedArgs {
    const float* xb;
    const int64_t* row_off;
    const int64_t* tile_off;
    const uint8_t* codes;
    const float* vmin;
    const float* delta;
    const float* eps;
    const float* xq;
    const float* qrot;
    const float* qinfo;
    const int32_t* probe;
    const int32_t* oid;
    uint32_t* tau;
    float* seed_d;    // optional [B, K]: the K smallest seed values per query, ascending (+inf padded)
    int64_t* seed_i;  // optional [B, K]: their row ids (-1 padded)
    int D, D_pad, nb, T, nlist, nprobe, p_seed, K, S;
    int shard;  // 1: the index holds only some lists; S shrinks with the share of local seed lists
    int ub;     // 1: SQ8 upper bounds of the selected rows instead of exact distances (no row reads)
    float rho;  // the index's relative slack of a float32 bound (lb_rel_slack)
};

// SQ8 upper bound of one 32-dim block: sum_d (|code_d delta_d + (vmin_d - q~_d)| + eps_d)^2, the
// same float32 arithmetic as the scan's upper-bound seeding.
__device__ __forceinline__ float ub_block_global(const uint4 w0, const uint4 w1, const float* __restrict__ vm,
                                                 const float* __restrict__ qr, const float* __restrict__ dl,
                                                 const float* __restrict__ ep) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float acc = 0.0f;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const float4 v4 = __ldg(reinterpret_cast<const float4*>(vm) + g);
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qr) + g);
        const float4 d4 = __ldg(reinterpret_cast<const float4*>(dl) + g);
        const float4 e4 = __ldg(reinterpret_cast<const float4*>(ep) + g);
        const float b[4] = {v4.x - q4.x, v4.y - q4.y, v4.z - q4.z, v4.w - q4.w};
        const float dd[4] = {d4.x, d4.y, d4.z, d4.w};
        const float ee[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float u = fabsf(fmaf(u8f(w[g], k), dd[k], b[k])) + ee[k];
            acc = fmaf(u, u, acc);
        }
    }
    return acc;
}

// Callers alternate between two s_w buffers on consecutive calls: a buffer is written again two calls
// later, after every thread has passed the barrier of the call in between and so has read it.
__device__ __forceinline__ int block_sum(int v, int* s_w) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(TB_FULL, v, o);
    if (lane == 0) s_w[warp] = v;
    __syncthreads();
    int t = 0;
#pragma unroll
    for (int w = 0; w < kSeedThreads / 32; ++w) t += s_w[w];
    return t;
}

template <bool VEC4>
__global__ void __launch_bounds__(kSeedThreads, 4) seed_kernel(const SeedArgs a) {
    __shared__ uint32_t s_key[kSeedRowsMax];
    __shared__ int32_t s_sel[kSeedRowsMax / 32];  // selected row indices (S <= kSeedRowsMax / 32)
    __shared__ float s_dist[kSeedRowsMax / 32];
    __shared__ __align__(16) float s_bq[kSeedListsMax][kSeedBlocks * 32];  // vmin - q~ of each list
    __shared__ __align__(16) float s_dl[kSeedListsMax][kSeedBlocks * 32];  // delta of each list
    __shared__ int32_t s_c[kSeedListsMax];
    __shared__ int32_t s_off[kSeedListsMax + 1];
    __shared__ int32_t s_len[kSeedListsMax];
    __shared__ int64_t s_r0[kSeedListsMax], s_t0[kSeedListsMax];
    __shared__ int s_w[2][kSeedThreads / 32];
    __shared__ uint32_t s_mn[kSeedThreads / 32], s_mx[kSeedThreads / 32];
    __shared__ int s_n, s_valid;

    const int q = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T, nb = a.nb, D_pad = a.D_pad;
    if (tid == 0) s_valid = 0;
    __syncthreads();
    if (tid < kSeedListsMax) {  // the warm-up lists, loaded in parallel
        int c = -1, L = 0;
        if (tid < a.p_seed) {
            c = a.probe[(int64_t)q * a.nprobe + tid];
            if ((unsigned)c < (unsigned)a.nlist) atomicAdd(&s_valid, 1);
            if ((unsigned)c < (unsigned)a.nlist) {
                const int64_t r0 = a.row_off[c];
                L = (int)(a.row_off[c + 1] - r0);
                s_r0[tid] = r0;
                s_t0[tid] = a.tile_off[c];
            }
        }
        s_c[tid] = c;
        s_len[tid] = L;
    }
    __syncthreads();
    if (tid == 0) {  // compact the non-empty lists
        int tot = 0, m = 0;
        for (int p = 0; p < kSeedListsMax; ++p) {
            if (s_len[p] == 0) continue;
            s_c[m] = s_c[p];
            s_r0[m] = s_r0[p];
            s_t0[m] = s_t0[p];
            s_off[m] = tot;
            tot += s_len[p];
            ++m;
        }
        for (int p = m; p <= kSeedListsMax; ++p) s_off[p] = tot;
        s_n = 0;
    }
    __syncthreads();
    const int R = min(s_off[kSeedListsMax], kSeedRowsMax);
    int S = a.S;
    if (a.shard && s_valid > 0) {  // this GPU's share of the seed rows: in proportion to its lists
        int m = 0;
        while (m < kSeedListsMax && s_off[m] < s_off[m + 1]) ++m;
        S = (a.S * m + s_valid - 1) / s_valid;
    }
    S = min(S, R);
    if (a.seed_d) {
        for (int k = tid; k < a.K; k += kSeedThreads) {  // slots beyond this GPU's rows stay empty
            a.seed_d[(int64_t)q * a.K + k] = kInf;
            a.seed_i[(int64_t)q * a.K + k] = -1;
        }
    }
    if (S <= 0) return;
    if (!a.shard && S < a.K) return;  // fewer rows than K: no finite threshold from these lists

    // ---- rank: squared distance of the SQ8 reconstruction over the leading blocks
    const int nbx = min(nb, kSeedBlocks);
    const float* qr = a.qrot + (int64_t)q * D_pad;
    for (int p = 0; p < kSeedListsMax && s_off[p] < s_off[p + 1]; ++p) {
        const int64_t o = (int64_t)s_c[p] * D_pad;
        for (int d = tid; d < nbx * 32; d += kSeedThreads) {
            s_bq[p][d] = a.vmin[o + d] - qr[d];
            s_dl[p][d] = a.delta[o + d];
        }
    }
    __syncthreads();
    // two rows per thread in flight: both rows' codes are loaded before either is evaluated
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int i0 = tid; i0 < R; i0 += 2 * kSeedThreads) {
        uint4 cw[2][kSeedBlocks][2];
        int pp[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = i0 + h * kSeedThreads;
            int p = 0;
            if (i < R) {
                while (i >= s_off[p + 1]) ++p;
                const int r = i - s_off[p];
                const uint8_t* rc = a.codes + ((size_t)(s_t0[p] + r / T) * nb * T + (r % T)) * 32;
#pragma unroll
                for (int b = 0; b < kSeedBlocks; ++b) {
                    if (b < nbx) {
                        cw[h][b][0] = __ldg(reinterpret_cast<const uint4*>(rc + (size_t)b * T * 32));
                        cw[h][b][1] = __ldg(reinterpret_cast<const uint4*>(rc + (size_t)b * T * 32 + 16));
                    }
                }
            }
            pp[h] = p;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = i0 + h * kSeedThreads;
            if (i >= R) break;
            const float4* vm = reinterpret_cast<const float4*>(s_bq[pp[h]]);
            const float4* dl = reinterpret_cast<const float4*>(s_dl[pp[h]]);
            float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < kSeedBlocks; ++b) {
                if (b >= nbx) break;
                const uint32_t w[8] = {cw[h][b][0].x, cw[h][b][0].y, cw[h][b][0].z, cw[h][b][0].w,
                                       cw[h][b][1].x, cw[h][b][1].y, cw[h][b][1].z, cw[h][b][1].w};
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const float4 v = vm[8 * b + g], d = dl[8 * b + g];
                    const float2 e01 = __ffma2_rn(u8f2(w[g], 0), make_float2(d.x, d.y), make_float2(v.x, v.y));
                    const float2 e23 = __ffma2_rn(u8f2(w[g], 2), make_float2(d.z, d.w), make_float2(v.z, v.w));
                    acc = __ffma2_rn(e01, e01, acc);
                    acc = __ffma2_rn(e23, e23, acc);
                }
            }
            const uint32_t key = __float_as_uint(acc.x + acc.y);  // non-negative: the bits order like the values
            s_key[i] = key;
            kmin = min(kmin, key);
            kmax = max(kmax, key);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(TB_FULL, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(TB_FULL, kmax, o));
    }
    if (lane == 0) {
        s_mn[warp] = kmin;
        s_mx[warp] = kmax;
    }
    __syncthreads();

    // ---- select S rows: every key below the bucket [v, v + 2^lo) that holds the S-th smallest key,
    // then enough keys from inside it. The bits above the highest bit in which the smallest and the
    // largest key differ are the same in every key; a bitwise search fixes the next kSeedBits bits.
    // Which keys of the bucket are taken only changes how tight the threshold is: any S distinct rows
    // bound the K-th distance from above.
    uint32_t v = 0xFFFFFFFFu;
    int lo = 0;
    if (S < R) {
        uint32_t mn = s_mn[0], mx = s_mx[0];
#pragma unroll
        for (int w = 1; w < kSeedThreads / 32; ++w) {
            mn = min(mn, s_mn[w]);
            mx = max(mx, s_mx[w]);
        }
        uint32_t pre = mn;  // all keys equal: the bucket is that key
        if (mn != mx) {
            const int hb = 31 - __clz(mn ^ mx);
            lo = max(0, hb + 1 - kSeedBits);
            pre = mn & ~((2u << hb) - 1u);
            for (int bit = hb; bit >= lo; --bit) {
                const uint32_t test = pre | ((1u << bit) - 1u);
                int cnt = 0;
                for (int i = tid; i < R; i += kSeedThreads) cnt += s_key[i] <= test;
                if (block_sum(cnt, s_w[bit & 1]) < S) pre |= 1u << bit;
            }
        }
        v = pre;
    }
    const uint32_t vb = v >> lo;
    for (int i = tid; i < R; i += kSeedThreads) {
        if ((s_key[i] >> lo) < vb || (v == 0xFFFFFFFFu)) {
            const int k = atomicAdd(&s_n, 1);
            if (k < S) s_sel[k] = i;
        }
    }
    __syncthreads();
    // Every thread reads the count before any thread adds to it again: a thread that read it late
    // would skip the branch and its barrier while the others wait inside.
    const int n_below = s_n;
    __syncthreads();
    if (n_below < S) {
        for (int i = tid; i < R; i += kSeedThreads) {
            if ((s_key[i] >> lo) == vb) {
                const int k = atomicAdd(&s_n, 1);
                if (k < S) s_sel[k] = i;
            }
        }
        __syncthreads();
    }

    // ---- refine the selected rows: exact distance (whole warp per row, the reference's summation
    // order), or with ub the SQ8 upper bound over every block (lane b takes blocks b, b + 32, ...)
    const float* xq = a.xq + (int64_t)q * a.D;
    for (int k = warp; k < S; k += kSeedThreads / 32) {
        const int i = s_sel[k];
        int p = 0;
        while (i >= s_off[p + 1]) ++p;
        const int r = i - s_off[p];
        __syncwarp();
        if (lane == 0) s_sel[k] = a.oid[s_r0[p] + r];  // keep the row id for the seed list
        float d;
        if (a.ub) {
            const int64_t o = (int64_t)s_c[p] * D_pad;
            const uint8_t* rc = a.codes + ((size_t)(s_t0[p] + r / T) * nb * T + (r % T)) * 32;
            float part = 0.0f;
            for (int b = lane; b < nb; b += 32) {
                const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(rc + (size_t)b * T * 32));
                const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(rc + (size_t)b * T * 32 + 16));
                part += ub_block_global(w0, w1, a.vmin + o + 32 * b, qr + 32 * b, a.delta + o + 32 * b,
                                        a.eps + o + 32 * b);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(TB_FULL, part, off);
            d = part;
        } else {
            d = exact_dist_warp<VEC4, 4>(a.xb + (s_r0[p] + r) * a.D, xq, a.D, lane);
        }
        if (lane == 0) s_dist[k] = d;
    }
    __syncthreads();

    // ---- the K-th smallest of the S values becomes the query's threshold (an upper bound turns
    // into the largest exact distance it admits)
    for (int k = tid; k < S; k += kSeedThreads) {
        const float d = s_dist[k];
        int rank = 0;
        for (int m = 0; m < S; ++m) {
            const float e = s_dist[m];
            rank += (e < d) || (e == d && m < k);
        }
        if (rank < a.K) {
            const float t = a.ub ? ub_threshold(d, a.qinfo[(int64_t)q * QI_LEN + QI_SIGMA], a.rho) : d;
            if (rank == a.K - 1) atomicMin(a.tau + q, __float_as_uint(t));
            if (a.seed_d) {
                a.seed_d[(int64_t)q * a.K + rank] = t;
                a.seed_i[(int64_t)q * a.K + rank] = s_sel[k];
            }
        }
    }
}

__global__ void fill_inf_kernel(uint32_t* __restrict__ tau, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) tau[i] = __float_as_uint(kInf);
}

cudaError_t launch_fill_inf(uint32_t* tau, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fill_inf_kernel<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, st>>>(tau, n);
    return cudaGetLastError();
}

// tau = +inf for every query; the coarse-stage status each query carries in qinfo[QI_PAD] (written
// by probe selection, possibly on another GPU) is or-ed into the workspace's status word.
__global__ void tau_init_import_status_kernel(uint32_t* __restrict__ tau, const float* __restrict__ qinfo, int B,
                                              int32_t* __restrict__ err) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B; i += gridDim.x * blockDim.x) {
        tau[i] = __float_as_uint(kInf);
        const int32_t s = __float_as_int(qinfo[(int64_t)i * QI_LEN + QI_PAD]);
        if (s != 0) atomicOr(err, s);
    }
}

cudaError_t launch_tau_init_import_status(uint32_t* tau, const float* qinfo, int B, int32_t* err, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    tau_init_import_status_kernel<<<(B + 255) / 256 < 1024 ? (B + 255) / 256 : 1024, 256, 0, st>>>(tau, qinfo, B, err);
    return cudaGetLastError();
}

int seed_rows_for(int K) { return 32 * ((K + 31) / 32) < 64 ? 64 : 32 * ((K + 31) / 32); }

int seed_lists_for(int B, int K, int nprobe) {
    const int p_ref = trident_p_init(TRIDENT_MODE_CASCADE, B, K, nprobe);  // the reference's warm-up count
    int p = nprobe / 8;
    if (p > kSeedListsMax) p = kSeedListsMax;
    if (p < p_ref) p = p_ref;
    return p < nprobe ? p : nprobe;
}

cudaError_t launch_seed(const trident_index& idx, const float* xq, const Workspace& ws, int B, int K, int nprobe,
                        int p_seed, int ub, float* seed_d, int64_t* seed_i, int shard, cudaStream_t st) {
    if (B <= 0 || p_seed <= 0) return cudaSuccess;
    SeedArgs a;
    a.xb = idx.xb_sorted;
    a.row_off = idx.list_row_off;
    a.tile_off = idx.list_tile_off;
    a.codes = idx.codes;
    a.vmin = idx.vmin;
    a.delta = idx.delta;
    a.eps = idx.eps;
    a.xq = xq;
    a.qrot = ws.qrot;
    a.qinfo = ws.qinfo;
    a.probe = ws.probe;
    a.oid = idx.orig_ids_sorted;
    a.tau = ws.tau;
    a.seed_d = seed_d;
    a.seed_i = seed_i;
    a.shard = shard;
    a.D = idx.D;
    a.D_pad = idx.D_pad;
    a.nb = idx.num_blocks;
    a.T = idx.tile_size;
    a.nlist = idx.nlist;
    a.nprobe = nprobe;
    a.p_seed = p_seed < kSeedListsMax ? p_seed : kSeedListsMax;
    a.p_seed = a.p_seed < nprobe ? a.p_seed : nprobe;
    a.K = K;
    a.S = seed_rows_for(K);
    a.ub = ub ? 1 : 0;
    a.rho = idx.lb_rel_slack;
    const bool vec4 = (idx.D % 4) == 0 && (((uintptr_t)idx.xb_sorted | (uintptr_t)xq) & 15) == 0;
    if (vec4)
        seed_kernel<true><<<B, kSeedThreads, 0, st>>>(a);
    else
        seed_kernel<false><<<B, kSeedThreads, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace tb
