// Coarse stage of the query path: PCA rotation of the queries and exact top-nprobe list selection.
//
// The reference runs one cuBLAS FP32 GEMM for both (proj = xq [-2C^T | R] + [||c||^2 | -muR],
// src/trident_v4_kernels.cu:1233-1246) and then selects the nprobe smallest coarse distances per
// query with nprobe rounds of block argmin over an smem copy of the row (:68-162), which cannot
// launch once 4*nlist bytes exceed the smem limit (nlist >~ 58k).
//
// Here:
//  * the rotation runs in float64 (DFMA) and is rounded once to float32, so the rotated query that
//    the Stage-Y bound uses is within half an ulp of (q - mu)R; its norm bound sigma feeds the
//    bound's slack;
//  * the coarse distances are computed approximately (a GEMM with a certified error bound E), a
//    radix select finds the nprobe-th approximate value t, and every list whose approximate value
//    is within t + 2E (+ float64 slack) is re-checked with the exact float64 ||q - c||^2. The exact
//    values are sorted by (distance, list id), so the probe set and its order are exactly the
//    oracle's (ties to the smaller list id, as :122/:131), whatever the GEMM's rounding.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

// ------------------------------------------------------------------------------------------
// Rotation: qrot[j][d] = float((q_j - mu) R[:, d]) in float64 on the FP64 tensor cores
// (mma.sync m8n8k4 f64, DMMA). A CTA computes 64 queries x 128 dims with 8 warps of 32 x 32
// (4 x 4 tiles of 8 x 8); 8-deep k-slices are staged in shared memory in two buffers, the next
// slice loaded into registers while the current one is multiplied. The products accumulate in
// float64 in k order in steps of 4; the error bound folded into sigma, (D + 2) 2^-52 relative to
// sum_k |q_k - mu_k| |R_kd|, holds for any rounding inside a step. The result is rounded once to
// float32.
// ------------------------------------------------------------------------------------------
constexpr int kRM = 64, kRN = 128, kRK = 8;
constexpr int kRAP = kRK + 4;   // padded row of the query slice (conflict-free fragment reads)
constexpr int kRBP = kRN + 8;   // padded row of the R slice

__device__ __forceinline__ void dmma_8x8x4(double& d0, double& d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) rotate_f64_kernel(const float* __restrict__ xq, const double* __restrict__ mu,
                                                        const double* __restrict__ R, int B, int D, int D_pad,
                                                        float* __restrict__ qrot) {
    __shared__ __align__(16) double sA[2][kRM][kRAP];
    __shared__ __align__(16) double sB[2][kRK][kRBP];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = (warp & 1) * 32, wn = (warp >> 1) * 32;  // the warp's 32 x 32 tile
    const int m0 = blockIdx.x * kRM, n0 = blockIdx.y * kRN;
    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
    constexpr int kQA = kRM * kRK / 256, kQB = kRK * kRN / 256;  // staged values per thread
    double rq[kQA], rr[kQB];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int t = 0; t < kQA; ++t) {
            const int i = tid + 256 * t;
            const int r = i / kRK, k = i - r * kRK;
            const int gm = m0 + r, gk = k0 + k;
            rq[t] = (gm < B && gk < D) ? (double)__ldg(xq + (int64_t)gm * D + gk) - __ldg(mu + gk) : 0.0;
        }
#pragma unroll
        for (int t = 0; t < kQB; ++t) {
            const int i = tid + 256 * t;
            const int k = i / kRN, n = i - k * kRN;
            const int gk = k0 + k, gn = n0 + n;
            rr[t] = (gk < D && gn < D) ? __ldg(R + (int64_t)gk * D + gn) : 0.0;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int t = 0; t < kQA; ++t) {
            const int i = tid + 256 * t;
            const int r = i / kRK, k = i - r * kRK;
            sA[buf][r][k] = rq[t];
        }
#pragma unroll
        for (int t = 0; t < kQB; ++t) {
            const int i = tid + 256 * t;
            const int k = i / kRN, n = i - k * kRN;
            sB[buf][k][n] = rr[t];
        }
    };
    // fragments of m8n8k4 (row.col): A[row = lane/4][k = lane%4], B[k = lane%4][col = lane/4],
    // D rows lane/4, columns 2 (lane%4) + {0, 1}
    const int fr = lane >> 2, fk = lane & 3;
    fetch(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < D; k0 += kRK) {
        const bool more = k0 + kRK < D;
        if (more) fetch(k0 + kRK);  // in flight during this slice's DMMAs
#pragma unroll
        for (int ks = 0; ks < kRK; ks += 4) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sA[buf][wm + 8 * i + fr][ks + fk];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = sB[buf][ks + fk][wn + 8 * j + fr];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j][0], acc[i][j][1], a[i], b[j]);
        }
        if (more) {
            stash(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + wm + 8 * i + fr;
        if (gm >= B) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int gn = n0 + wn + 8 * j + 2 * fk + h;
                if (gn < D_pad) qrot[(int64_t)gm * D_pad + gn] = gn < D ? (float)acc[i][j][h] : 0.0f;
            }
    }
}

// Per-query norms (one warp per query): ||q|| for the coarse bound, ||q - mu|| for sigma; the
// query's threshold starts at +inf.
__global__ void __launch_bounds__(256) query_norms_kernel(const float* __restrict__ xq, const double* __restrict__ mu,
                                                         int B, int D, int D_pad, float* __restrict__ qinfo,
                                                         uint32_t* __restrict__ tau) {
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (j >= B) return;
    double s_q = 0.0, s_c = 0.0;
    for (int k = lane; k < D; k += 32) {
        const double v = (double)xq[(int64_t)j * D + k];
        const double w = v - mu[k];
        s_q = fma(v, v, s_q);
        s_c = fma(w, w, s_c);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s_q += __shfl_xor_sync(TB_FULL, s_q, o);
        s_c += __shfl_xor_sync(TB_FULL, s_c, o);
    }
    if (lane == 0) {
        const double qn = sqrt(s_q) * (1.0 + 1e-12);
        const double cn = sqrt(s_c) * (1.0 + 1e-12);
        // sigma: Minkowski slack for the query-side float32 roundings of the bound (3u|q~_d| per
        // dim) plus the float64 rotation error per dim.
        const double u = 5.9604644775390625e-08;  // 2^-24
        const double sigma =
            (3.0001 * u * cn + sqrt((double)D_pad) * (D + 2) * 2.220446049250313e-16 * cn) * (1.0 + 1e-6);
        float* qi = qinfo + (int64_t)j * QI_LEN;
        qi[QI_QNORM] = __double2float_ru(qn);
        qi[QI_SIGMA] = __double2float_ru(sigma);
        qi[QI_CNORM] = __double2float_ru(cn);
        qi[QI_PAD] = 0.0f;
        tau[j] = __float_as_uint(kInf);
    }
}

cudaError_t launch_query_norms(const trident_index& idx, const float* xq, int B, float* qinfo, uint32_t* tau,
                               cudaStream_t st) {
    query_norms_kernel<<<(B + 7) / 8, 256, 0, st>>>(xq, idx.pca_mean, B, idx.D, idx.D_pad, qinfo, tau);
    return cudaGetLastError();
}

cudaError_t launch_rotate_f64(const trident_index& idx, const float* xq, int B, float* qrot, cudaStream_t st) {
    dim3 grid((B + kRM - 1) / kRM, (idx.D_pad + kRN - 1) / kRN);
    rotate_f64_kernel<<<grid, 256, 0, st>>>(xq, idx.pca_mean, idx.pca_rot, B, idx.D, idx.D_pad, qrot);
    return cudaGetLastError();
}

cudaError_t launch_rotate(const trident_index& idx, const float* xq, int B, float* qrot, float* qinfo,
                          uint32_t* tau, cudaStream_t st) {
    cudaError_t e = launch_query_norms(idx, xq, B, qinfo, tau, st);
    if (e != cudaSuccess) return e;
    return launch_rotate_f64(idx, xq, B, qrot, st);
}

// ------------------------------------------------------------------------------------------
// Exact top-nprobe selection, one CTA per query.
// ------------------------------------------------------------------------------------------
constexpr int kSelThreads = 256;
constexpr int kSelNW = kSelThreads / 32;
constexpr int kSelCap = 2048;        // sorted best (<= nprobe <= 1024) + one batch of re-check members
constexpr int kSelSmemKeys = 8192;
constexpr int kSelRegKeys = 4;      // keys per thread held in registers by the threshold search (nlist <= 1024)
constexpr int kSelTileKeys = 16;    // span minima per thread (up to 4096 spans of kCoarseMinSpan lists)

__device__ void bitonic_sort_kc(unsigned long long* key, int32_t* cid, int P) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool up = (i & k) == 0;
                    const unsigned long long a = key[i], b = key[ixj];
                    const int32_t ca = cid[i], cb = cid[ixj];
                    const bool gt = (a > b) || (a == b && ca > cb);
                    if (gt == up) {
                        key[i] = b; key[ixj] = a;
                        cid[i] = cb; cid[ixj] = ca;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int block_sum_sel(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = __reduce_add_sync(TB_FULL, (unsigned)v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int s = 0;
#pragma unroll
    for (int w = 0; w < kSelNW; ++w) s += red[w];
    __syncthreads();
    return s;
}

// The k-th smallest (1-based) of n keys held R per thread in registers (absent keys: all ones), bit
// by bit from the top: bit b of the answer is 0 iff at least k keys are <= (the answer so far with
// bit b = 0 and all lower bits = 1). Padding keys count as <= upper only at upper = 0xFFFFFFFF.
template <int R>
__device__ __forceinline__ uint32_t kth_smallest_key(const uint32_t (&kr)[R], int n, int k, int* red) {
    uint32_t ans = 0;
    const int pad = R * kSelThreads - n;
    for (int b = 31; b >= 0; --b) {
        const uint32_t upper = ans | ((1u << b) - 1u);
        int cnt = 0;
#pragma unroll
        for (int u = 0; u < R; ++u) cnt += kr[u] <= upper;
        cnt = block_sum_sel(cnt, red);
        if (upper == 0xFFFFFFFFu) cnt -= pad;
        if (cnt < k) ans |= (1u << b);
    }
    return ans;
}

// float64 ||q - c||^2 in the oracle's order (oracle_l2_f64): lane l sums d = l, l + 32, ... with
// fma (coalesced 128-byte loads of the centroid row), then the 32 lane sums are added in lane
// order. Every lane returns the total.
__device__ __forceinline__ double l2_f64_warp(const float* __restrict__ qv, const float* __restrict__ cr, int D,
                                              int lane) {
    double acc = 0.0;
    int d = lane;
    for (; d + 96 < D; d += 128) {  // four loads in flight, the same fma order
        const float c0 = __ldg(cr + d), c1 = __ldg(cr + d + 32), c2 = __ldg(cr + d + 64), c3 = __ldg(cr + d + 96);
        double df = (double)qv[d] - (double)c0;
        acc = fma(df, df, acc);
        df = (double)qv[d + 32] - (double)c1;
        acc = fma(df, df, acc);
        df = (double)qv[d + 64] - (double)c2;
        acc = fma(df, df, acc);
        df = (double)qv[d + 96] - (double)c3;
        acc = fma(df, df, acc);
    }
    for (; d < D; d += 32) {
        const double df = (double)qv[d] - (double)__ldg(cr + d);
        acc = fma(df, df, acc);
    }
    double total = __shfl_sync(TB_FULL, acc, 0);
#pragma unroll
    for (int l = 1; l < 32; ++l) total += __shfl_sync(TB_FULL, acc, l);
    return total;
}

// Two rows at once, each in exactly the order of l2_f64_warp (two independent fma chains).
__device__ __forceinline__ void l2_f64_warp2(const float* __restrict__ qv, const float* __restrict__ ca,
                                             const float* __restrict__ cb, int D, int lane, double& ra, double& rb) {
    double aa = 0.0, ab = 0.0;
    int d = lane;
    for (; d + 96 < D; d += 128) {
        float a4[4], b4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            a4[u] = __ldg(ca + d + 32 * u);
            b4[u] = __ldg(cb + d + 32 * u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const double q = (double)qv[d + 32 * u];
            const double da = q - (double)a4[u], db = q - (double)b4[u];
            aa = fma(da, da, aa);
            ab = fma(db, db, ab);
        }
    }
    for (; d < D; d += 32) {
        const double q = (double)qv[d];
        const double da = q - (double)__ldg(ca + d), db = q - (double)__ldg(cb + d);
        aa = fma(da, da, aa);
        ab = fma(db, db, ab);
    }
    double ta = __shfl_sync(TB_FULL, aa, 0), tb = __shfl_sync(TB_FULL, ab, 0);
#pragma unroll
    for (int l = 1; l < 32; ++l) {
        ta += __shfl_sync(TB_FULL, aa, l);
        tb += __shfl_sync(TB_FULL, ab, l);
    }
    ra = ta;
    rb = tb;
}

__global__ void __launch_bounds__(kSelThreads, 4) probe_select_kernel(
    const float* __restrict__ coarse, const float* __restrict__ tilemin, const float* __restrict__ xq,
    const float* __restrict__ cent, float* __restrict__ qinfo, int nlist, int D, int nprobe, float cmax,
    int32_t* __restrict__ probe,
    double* __restrict__ probe_d64, unsigned long long* __restrict__ stats, const int32_t* __restrict__ err) {
    extern __shared__ float sel_smem[];
    float* qv = sel_smem;                                              // [D]
    uint32_t* skeys = reinterpret_cast<uint32_t*>(sel_smem + ((D + 3) & ~3));  // [nlist] when cached
    __shared__ unsigned long long skey[kSelCap];
    __shared__ int32_t scid[kSelCap];
    __shared__ int red[kSelNW];
    __shared__ int s_batch, s_n;
    const int j = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* row = coarse + (int64_t)j * nlist;
    // A coarse GEMM that gave up left this row incomplete: no probe list is selected from it. The
    // status goes into the query's qinfo, which travels with the query in the multi-GPU search.
    const int32_t status = ld_volatile_i32(err);
    if (status != 0) {
        for (int p = tid; p < nprobe; p += blockDim.x) {
            probe[(int64_t)j * nprobe + p] = -1;
            if (probe_d64) probe_d64[(int64_t)j * nprobe + p] = __longlong_as_double(0x7ff8000000000000ll);
        }
        if (tid == 0) qinfo[(int64_t)j * QI_LEN + QI_PAD] = __int_as_float(status);
        return;
    }
    const bool cached = nlist <= kSelSmemKeys;
    for (int d = tid; d < D; d += blockDim.x) qv[d] = xq[(int64_t)j * D + d];
    if (cached) {
#pragma unroll 8
        for (int c = tid; c < nlist; c += blockDim.x) skeys[c] = float_key(__ldg(row + c));
    }
    __syncthreads();

    // 1) t >= the nprobe-th smallest approximate value (equal to it except on the tile-minimum path)
    uint32_t ans = 0;
    const int ntiles = (nlist + kCoarseMinSpan - 1) / kCoarseMinSpan;  // entries of the row-minimum array
    if (nlist <= kSelRegKeys * kSelThreads) {  // exact, this thread's keys in registers
        uint32_t kr[kSelRegKeys];
#pragma unroll
        for (int u = 0; u < kSelRegKeys; ++u) {
            const int c = tid + u * kSelThreads;
            kr[u] = c < nlist ? (cached ? skeys[c] : float_key(__ldg(row + c))) : 0xFFFFFFFFu;
        }
        ans = kth_smallest_key<kSelRegKeys>(kr, nlist, nprobe, red);
    } else if (!cached && tilemin && nprobe <= ntiles && ntiles <= kSelTileKeys * kSelThreads) {
        // An upper bound from the GEMM's row minima over 64-list spans: the nprobe smallest of them are nprobe
        // distinct entries of the row, so the row's nprobe-th smallest value is <= their largest.
        // The member pass below then reads the row once instead of once per bit.
        uint32_t kr[kSelTileKeys];
        const float* tm = tilemin + (int64_t)j * ntiles;
#pragma unroll
        for (int u = 0; u < kSelTileKeys; ++u) {
            const int c = tid + u * kSelThreads;
            kr[u] = c < ntiles ? float_key(__ldg(tm + c)) : 0xFFFFFFFFu;
        }
        ans = kth_smallest_key<kSelTileKeys>(kr, ntiles, nprobe, red);
    } else {  // exact, keys re-read per bit (shared memory when cached)
        for (int b = 31; b >= 0; --b) {
            const uint32_t upper = ans | ((1u << b) - 1u);
            int cnt = 0;
            for (int c = tid; c < nlist; c += blockDim.x) {
                const uint32_t k = cached ? skeys[c] : float_key(__ldg(row + c));
                cnt += k <= upper;
            }
            cnt = block_sum_sel(cnt, red);
            if (cnt < nprobe) ans |= (1u << b);
        }
    }
    const float t = key_float(ans);

    // 2) members: approximate value within the certified band above t
    const float* qi = qinfo + (int64_t)j * QI_LEN;
    const double qn = (double)qi[QI_QNORM];
    const double cm = (double)cmax;
    // error bound of the 3xTF32 tensor-core GEMM (tb_coarse_mma.cu)
    const double E = ((double)(3 * D + 16) * 0x1p-22 + 3.02 * 0x1p-20) * 1.01 * (2.0 * qn * cm + cm * cm);
    const double eta = (double)(D + 2) * 2.220446049250313e-16 * (qn + cm) * (qn + cm);
    const float thr = __double2float_ru((double)t + 2.0 * E + 2.0 * eta);

    int best_n = 0;
    int batch = 0;
    if (tid == 0) s_batch = 0;
    __syncthreads();
    long long members = 0;
    auto process_batch = [&]() {
        // exact float64 distance of each batch member (one warp per member), then sort best + batch
        for (int i = warp; i < batch; i += 2 * kSelNW) {
            const int i2 = i + kSelNW;
            const int c = scid[best_n + i];
            if (i2 < batch) {
                double da, db;
                l2_f64_warp2(qv, cent + (int64_t)c * D, cent + (int64_t)scid[best_n + i2] * D, D, lane, da, db);
                if (lane == 0) {
                    skey[best_n + i] = (unsigned long long)__double_as_longlong(da);
                    skey[best_n + i2] = (unsigned long long)__double_as_longlong(db);
                }
            } else {
                const double d64 = l2_f64_warp(qv, cent + (int64_t)c * D, D, lane);
                if (lane == 0) skey[best_n + i] = (unsigned long long)__double_as_longlong(d64);
            }
        }
        const int n = best_n + batch;
        int P = 1;
        while (P < n) P <<= 1;
        for (int i = n + tid; i < P; i += blockDim.x) { skey[i] = ~0ull; scid[i] = 0x7fffffff; }
        __syncthreads();
        bitonic_sort_kc(skey, scid, P);
        best_n = n < nprobe ? n : nprobe;
        batch = 0;
        if (tid == 0) s_batch = 0;
        __syncthreads();
    };
    // One pass with warp-aggregated appends and no CTA barrier; if the members overflow the buffer,
    // the chunked pass below takes them in batches instead.
    if (tid == 0) s_n = 0;
    __syncthreads();
    auto offer = [&](bool mem, int c) {  // warp-aggregated append of the members among 32 lanes
        const unsigned m = __ballot_sync(TB_FULL, mem);
        if (m) {
            const int leader = __ffs(m) - 1;
            int pos = 0;
            if (lane == leader) pos = atomicAdd(&s_n, __popc(m));
            pos = __shfl_sync(TB_FULL, pos, leader) + __popc(m & ((1u << lane) - 1u));
            if (mem && pos < kSelCap) scid[pos] = c;
        }
    };
    if (!cached && (nlist & 3) == 0 && ((uintptr_t)row & 15) == 0) {
        // the row from global memory: 16-byte loads, four in flight per lane (512 lists per warp step)
        constexpr int kU = 4;
        const float4* row4 = reinterpret_cast<const float4*>(row);
        const int n4 = nlist >> 2;
        for (int b4 = warp * 32 * kU; b4 < n4; b4 += kSelThreads * kU) {  // warp-uniform trip count
            float4 v[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int i4 = b4 + u * 32 + lane;
                v[u] = i4 < n4 ? __ldg(row4 + i4) : make_float4(kInf, kInf, kInf, kInf);
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int c = 4 * (b4 + u * 32 + lane);
                const bool in = c < nlist;  // (nlist % 4 == 0: the whole float4 is in range or none)
                offer(in && v[u].x <= thr, c);
                offer(in && v[u].y <= thr, c + 1);
                offer(in && v[u].z <= thr, c + 2);
                offer(in && v[u].w <= thr, c + 3);
            }
        }
    } else {
        for (int c0 = warp * 32; c0 < nlist; c0 += kSelThreads) {  // warp-uniform trip count
            const int c = c0 + lane;
            offer((c < nlist) && ((cached ? key_float(skeys[c]) : __ldg(row + c)) <= thr), c);
        }
    }
    __syncthreads();
    const int n_fast = s_n;
    if (n_fast <= kSelCap) {
        members = n_fast;
        if (n_fast > 0) {
            batch = n_fast;
            process_batch();
        }
    }
    for (int cs = 0; n_fast > kSelCap && cs < nlist; cs += blockDim.x) {
        const int c = cs + tid;
        const bool mem = (c < nlist) && ((cached ? key_float(skeys[c]) : __ldg(row + c)) <= thr);
        const int chunk = __syncthreads_count(mem);
        if (chunk == 0) continue;
        members += chunk;
        if (best_n + batch + chunk > kSelCap) process_batch();
        const unsigned m = __ballot_sync(TB_FULL, mem);
        if (m) {
            const int leader = __ffs(m) - 1;
            int pos = 0;
            if (lane == leader) pos = atomicAdd(&s_batch, __popc(m));
            pos = __shfl_sync(TB_FULL, pos, leader);
            if (mem) scid[best_n + pos + __popc(m & ((1u << lane) - 1u))] = c;
        }
        __syncthreads();
        batch = s_batch;
        __syncthreads();
    }
    if (batch > 0) process_batch();
    // best_n >= nprobe whenever the row is finite; a non-finite query leaves the tail as -1
    // (skipped by the pair kernels, whose candidate slots then stay empty).
    for (int p = tid; p < nprobe; p += blockDim.x) {
        const bool ok = p < best_n;
        probe[(int64_t)j * nprobe + p] = ok ? scid[p] : -1;
        if (probe_d64) probe_d64[(int64_t)j * nprobe + p] = ok ? __longlong_as_double((long long)skey[p]) : kInf;
    }
    if (stats && tid == 0) atomicAdd(stats + TRIDENT_STAT_COARSE_RECHECK, (unsigned long long)members);
}

cudaError_t launch_probe_select(const trident_index& idx, const float* xq, int B, int nprobe, const float* coarse,
                                const float* tilemin, float* qinfo, int32_t* probe, double* probe_d64,
                                unsigned long long* stats, const int32_t* err, cudaStream_t st) {
    size_t smem = (size_t)((idx.D + 3) & ~3) * sizeof(float);
    if (idx.nlist <= kSelSmemKeys) smem += (size_t)idx.nlist * sizeof(uint32_t);
    cudaError_t e = cudaFuncSetAttribute(probe_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    probe_select_kernel<<<B, kSelThreads, smem, st>>>(coarse, tilemin, xq, idx.centroids, qinfo, idx.nlist, idx.D, nprobe,
                                                      idx.centroid_norm_max, probe, probe_d64, stats, err);
    return cudaGetLastError();
}

}  // namespace tb
