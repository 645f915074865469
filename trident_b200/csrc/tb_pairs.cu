// Cluster-major work lists: (list, query) pairs grouped by list, then split into work items of at
// most G queries.
//
// The reference sorts (cid, qid, dqc) pairs of each pass with one 256-thread CTA per pass and an
// smem histogram of nlist+1 counters (src/trident_v4_kernels.cu:168-263), which serialises 2.5-5M
// pairs at the large configs and cannot launch for nlist >~ 58k. Here the histogram and scatter run
// over the whole GPU with global atomics, one 1024-thread CTA per pass scans the counts, and a
// final kernel emits the items. Pass 0 holds probes p < p_init (the warm-up lists), pass 1 the rest.
// The order of queries inside a list is not deterministic; results do not depend on it.
#include <cuda_runtime.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

// A probe of an empty list (a list another GPU owns, in a sharded index) makes no pair.
__device__ __forceinline__ bool probe_has_rows(int32_t c, int nlist, const int64_t* __restrict__ row_off) {
    return (unsigned)c < (unsigned)nlist && row_off[c + 1] > row_off[c];
}

__global__ void pair_hist_kernel(const int32_t* __restrict__ probe, int64_t total, int nprobe, int p_init, int nlist,
                                 const int64_t* __restrict__ row_off, int32_t* __restrict__ cnt) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(i % nprobe);
        const int s = p >= p_init;
        const int32_t c = probe[i];
        if (probe_has_rows(c, nlist, row_off)) atomicAdd(&cnt[s * nlist + c], 1);
    }
}

// One CTA per pass: exclusive scans of the pair counts and of the per-list item counts
// ceil(cnt / G); cursors start at the pair offsets; ctr[pass] receives the item count.
__global__ void __launch_bounds__(1024) pair_scan_kernel(const int32_t* __restrict__ cnt, int nlist, int G,
                                                        int32_t* __restrict__ off, int32_t* __restrict__ item_off,
                                                        int32_t* __restrict__ cursor, int32_t* __restrict__ ctr) {
    __shared__ int32_t wsum[2][32];
    const int s = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int32_t* c_in = cnt + (int64_t)s * nlist;
    int32_t* o = off + (int64_t)s * (nlist + 1);
    int32_t* io = item_off + (int64_t)s * (nlist + 1);
    int32_t* cur = cursor + (int64_t)s * nlist;
    int32_t run_p = 0, run_i = 0;
    for (int base = 0; base < nlist; base += 1024) {
        const int c = base + tid;
        const int32_t vp = (c < nlist) ? c_in[c] : 0;
        const int32_t vi = (vp + G - 1) / G;
        int32_t sp = vp, si = vi;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t np = __shfl_up_sync(TB_FULL, sp, d);
            const int32_t ni = __shfl_up_sync(TB_FULL, si, d);
            if (lane >= d) { sp += np; si += ni; }
        }
        if (lane == 31) { wsum[0][warp] = sp; wsum[1][warp] = si; }
        __syncthreads();
        if (warp == 0) {
            int32_t wp = wsum[0][lane], wi = wsum[1][lane];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t np = __shfl_up_sync(TB_FULL, wp, d);
                const int32_t ni = __shfl_up_sync(TB_FULL, wi, d);
                if (lane >= d) { wp += np; wi += ni; }
            }
            wsum[0][lane] = wp;
            wsum[1][lane] = wi;
        }
        __syncthreads();
        const int32_t pre_p = (warp > 0 ? wsum[0][warp - 1] : 0) + sp - vp;
        const int32_t pre_i = (warp > 0 ? wsum[1][warp - 1] : 0) + si - vi;
        if (c < nlist) {
            o[c] = run_p + pre_p;
            cur[c] = run_p + pre_p;
            io[c] = run_i + pre_i;
        }
        run_p += wsum[0][31];
        run_i += wsum[1][31];
        __syncthreads();
    }
    if (tid == 0) {
        o[nlist] = run_p;
        io[nlist] = run_i;
        ctr[s] = run_i;
    }
}

__global__ void pair_scatter_kernel(const int32_t* __restrict__ probe, int64_t total, int nprobe, int p_init,
                                    int nlist, const int64_t* __restrict__ row_off, int64_t base1,
                                    int32_t* __restrict__ cursor,
                                    int32_t* __restrict__ pair_q, int32_t* __restrict__ pair_p, int K,
                                    float* __restrict__ cand_d, int32_t* __restrict__ cand_i) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(i % nprobe);
        const int q = (int)(i / nprobe);
        const int s = p >= p_init;
        const int32_t c = probe[i];
        if (!probe_has_rows(c, nlist, row_off)) {  // no rows for this probe: its slots stay empty
            for (int k = 0; k < K; ++k) {
                cand_d[i * K + k] = kInf;
                cand_i[i * K + k] = -1;
            }
            continue;
        }
        const int64_t pos = (s ? base1 : 0) + atomicAdd(&cursor[s * nlist + c], 1);
        pair_q[pos] = q;
        pair_p[pos] = p;
    }
}

// Items (list, first pair, query count) in list order; pass 1's items start at items + base1.
__global__ void item_emit_kernel(const int32_t* __restrict__ cnt, const int32_t* __restrict__ off,
                                 const int32_t* __restrict__ item_off, int nlist, int G, int64_t base1,
                                 int4* __restrict__ items) {
    const int s = blockIdx.y;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < nlist; c += gridDim.x * blockDim.x) {
        const int32_t n = cnt[s * nlist + c];
        if (n == 0) continue;
        const int32_t po = off[s * (nlist + 1) + c];
        const int32_t io = item_off[s * (nlist + 1) + c];
        int4* dst = items + (s ? base1 : 0) + io;
        for (int g = 0; g * G < n; ++g) {
            const int32_t m = min(G, n - g * G);
            dst[g] = make_int4(c, (int)((s ? base1 : 0) + po + g * G), m, 0);
        }
    }
}

cudaError_t launch_pairs(const trident_index& idx, const int32_t* probe, int B, int nprobe, int p_init, int G, int K,
                         const Workspace& ws, cudaStream_t st) {
    const int nlist = idx.nlist;
    const int64_t total = (int64_t)B * nprobe;
    const int64_t base1 = (int64_t)B * p_init;
    cudaError_t e = cudaMemsetAsync(ws.cnt, 0, sizeof(int32_t) * 2 * (size_t)nlist, st);
    if (e != cudaSuccess) return e;
    const int threads = 256;
    int blocks = (int)((total + threads - 1) / threads);
    const int cap = num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    pair_hist_kernel<<<blocks, threads, 0, st>>>(probe, total, nprobe, p_init, nlist, idx.list_row_off, ws.cnt);
    pair_scan_kernel<<<2, 1024, 0, st>>>(ws.cnt, nlist, G, ws.off, ws.item_off, ws.cursor, ws.ctr);
    pair_scatter_kernel<<<blocks, threads, 0, st>>>(probe, total, nprobe, p_init, nlist, idx.list_row_off, base1,
                                                     ws.cursor, ws.pair_q,
                                                     ws.pair_p, K, ws.cand_d, ws.cand_i);
    dim3 g2((nlist + 255) / 256, 2);
    item_emit_kernel<<<g2, 256, 0, st>>>(ws.cnt, ws.off, ws.item_off, nlist, G, base1, ws.items);
    return cudaGetLastError();
}

// ---- longest-processing-time order of the main pass's items. The scan is a persistent kernel that
// takes items from a counter; handing out the expensive items first keeps the last CTAs from
// finishing a big item alone. Cost estimate: (rows + 32) x (queries + 2); bin = 4 log2(cost),
// reversed so that bin 0 is the most expensive. The order inside a bin is arbitrary (atomics);
// results do not depend on it.
__device__ __forceinline__ int lpt_bin(const int4 it, const int64_t* __restrict__ row_off) {
    const unsigned long long L = (unsigned long long)(row_off[it.x + 1] - row_off[it.x]);
    const unsigned long long cost = (L + 32ull) * (unsigned long long)(it.z + 2);
    const int msb = 63 - __clzll((long long)cost);
    const int frac = msb >= 2 ? (int)((cost >> (msb - 2)) & 3ull) : 0;
    const int key = min(kLptBins - 1, 4 * msb + frac);
    return kLptBins - 1 - key;
}

__global__ void lpt_hist_kernel(const int4* __restrict__ items, const int32_t* __restrict__ n_items,
                                const int64_t* __restrict__ row_off, int32_t* __restrict__ hist) {
    const int n = *n_items;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        atomicAdd(&hist[lpt_bin(items[i], row_off)], 1);
}

__global__ void __launch_bounds__(kLptBins) lpt_scan_kernel(int32_t* __restrict__ hist) {
    __shared__ int32_t s[kLptBins];
    const int t = threadIdx.x;
    s[t] = hist[t];
    __syncthreads();
    if (t == 0) {
        int run = 0;
        for (int b = 0; b < kLptBins; ++b) {
            const int c = s[b];
            s[b] = run;
            run += c;
        }
    }
    __syncthreads();
    hist[t] = s[t];  // now the cursor of each bin
}

__global__ void lpt_scatter_kernel(const int4* __restrict__ items, const int32_t* __restrict__ n_items,
                                   const int64_t* __restrict__ row_off, int32_t* __restrict__ cursor,
                                   int4* __restrict__ out) {
    const int n = *n_items;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int4 it = items[i];
        out[atomicAdd(&cursor[lpt_bin(it, row_off)], 1)] = it;
    }
}

cudaError_t launch_item_order(const trident_index& idx, int max_items, const Workspace& ws, cudaStream_t st) {
    if (max_items <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(ws.lpt, 0, kLptBins * sizeof(int32_t), st);
    if (e != cudaSuccess) return e;
    int blocks = (max_items + 255) / 256;
    const int cap = num_sms() * 4;
    if (blocks > cap) blocks = cap;
    lpt_hist_kernel<<<blocks, 256, 0, st>>>(ws.items, ws.ctr + 1, idx.list_row_off, ws.lpt);
    lpt_scan_kernel<<<1, kLptBins, 0, st>>>(ws.lpt);
    lpt_scatter_kernel<<<blocks, 256, 0, st>>>(ws.items, ws.ctr + 1, idx.list_row_off, ws.lpt, ws.items_lpt);
    return cudaGetLastError();
}

}  // namespace tb
