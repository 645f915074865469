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
    int32_t* err;  // status word: TRIDENT_STATUS_LOCK_TIMEOUT if a per-query lock wait gave up
    uint32_t lock_spins;  // limit of that wait (tries)
    int D, D_pad, nb, K, nprobe, G;
    int seed_rows;  // best-ranked rows refined first for queries without a finite threshold (0: off)
    float rho;
};

constexpr int kMaxG = 64;
// Resident scan threads per SM the kernel is compiled for (registers) and sized for (shared memory).
constexpr int kScanThreadsPerSm = 512;

// Stage Y on one 32-dim block: acc += sum_d max(|code_d delta_d + (vmin_d - q~_d)| - eps_d, 0)^2
// (reference :750-767). base/dl/ep point at the block's 32 entries in shared memory. Pairs of dims
// go through packed FFMA2 (each lane of the pair rounds like fmaf); the sum runs as two chains,
// which the float32 slack of the prune test covers like any other order.
__device__ __forceinline__ float lb_block(const uint4 w0, const uint4 w1, const float* __restrict__ base,
                                          const float* __restrict__ dl, const float* __restrict__ ep, float acc) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float2 a2 = make_float2(acc, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 b4 = *reinterpret_cast<const float4*>(base + 4 * i);
        const float4 d4 = *reinterpret_cast<const float4*>(dl + 4 * i);
        const float4 e4 = *reinterpret_cast<const float4*>(ep + 4 * i);
        const float2 u01 = __ffma2_rn(u8f2(w[i], 0), make_float2(d4.x, d4.y), make_float2(b4.x, b4.y));
        const float2 u23 = __ffma2_rn(u8f2(w[i], 2), make_float2(d4.z, d4.w), make_float2(b4.z, b4.w));
        const float2 l01 = make_float2(fmaxf(fabsf(u01.x) - e4.x, 0.0f), fmaxf(fabsf(u01.y) - e4.y, 0.0f));
        const float2 l23 = make_float2(fmaxf(fabsf(u23.x) - e4.z, 0.0f), fmaxf(fabsf(u23.y) - e4.w, 0.0f));
        a2 = __ffma2_rn(l01, l01, a2);
        a2 = __ffma2_rn(l23, l23, a2);
    }
    return a2.x + a2.y;
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

// Float codes of one 32-dim block (exact uint8 -> float) for the register-resident first block.
__device__ __forceinline__ void unpack_block(const uint4 w0, const uint4 w1, float* cf) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) cf[4 * i + k] = u8f(w[i], k);
}

// Stage Y on block 0 whose codes are already floats; base = vmin - q~ is formed from global memory
// with the same float32 subtraction as the shared-memory copies.
__device__ __forceinline__ float lb_block_f(const float* cf, const float* __restrict__ vm, const float* __restrict__ qr,
                                            const float* __restrict__ dl, const float* __restrict__ ep, float acc) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v4 = __ldg(reinterpret_cast<const float4*>(vm) + i);
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qr) + i);
        const float4 b4 = make_float4(v4.x - q4.x, v4.y - q4.y, v4.z - q4.z, v4.w - q4.w);
        const float4 d4 = *reinterpret_cast<const float4*>(dl + 4 * i);
        const float4 e4 = *reinterpret_cast<const float4*>(ep + 4 * i);
        float l;
        l = fmaxf(fabsf(fmaf(cf[4 * i + 0], d4.x, b4.x)) - e4.x, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(cf[4 * i + 1], d4.y, b4.y)) - e4.y, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(cf[4 * i + 2], d4.z, b4.z)) - e4.z, 0.0f); acc = fmaf(l, l, acc);
        l = fmaxf(fabsf(fmaf(cf[4 * i + 3], d4.w, b4.w)) - e4.w, 0.0f); acc = fmaf(l, l, acc);
    }
    return acc;
}

// Stage Y / UB on one block beyond the shared-memory window: base = vmin - q~ is formed in
// registers from global (L1-resident) vmin and q~, with the same float32 subtraction as the
// shared-memory copy, so the bound is identical on both paths.
template <bool UPPER>
__device__ __forceinline__ float bound_block_g(const uint4 w0, const uint4 w1, const float* __restrict__ vm,
                                               const float* __restrict__ qr, const float* __restrict__ dl,
                                               const float* __restrict__ ep, float acc) {
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float2 a2 = make_float2(acc, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v4 = __ldg(reinterpret_cast<const float4*>(vm) + i);
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qr) + i);
        const float4 d4 = *reinterpret_cast<const float4*>(dl + 4 * i);
        const float4 e4 = *reinterpret_cast<const float4*>(ep + 4 * i);
        const float2 u01 = __ffma2_rn(u8f2(w[i], 0), make_float2(d4.x, d4.y), make_float2(v4.x - q4.x, v4.y - q4.y));
        const float2 u23 = __ffma2_rn(u8f2(w[i], 2), make_float2(d4.z, d4.w), make_float2(v4.z - q4.z, v4.w - q4.w));
        float2 l01, l23;
        if (UPPER) {
            l01 = make_float2(fabsf(u01.x) + e4.x, fabsf(u01.y) + e4.y);
            l23 = make_float2(fabsf(u23.x) + e4.z, fabsf(u23.y) + e4.w);
        } else {
            l01 = make_float2(fmaxf(fabsf(u01.x) - e4.x, 0.0f), fmaxf(fabsf(u01.y) - e4.y, 0.0f));
            l23 = make_float2(fmaxf(fabsf(u23.x) - e4.z, 0.0f), fmaxf(fabsf(u23.y) - e4.w, 0.0f));
        }
        a2 = __ffma2_rn(l01, l01, a2);
        a2 = __ffma2_rn(l23, l23, a2);
    }
    return a2.x + a2.y;
}

constexpr float kU32 = 5.9604644775390625e-08f;  // 2^-24
constexpr int kSQS = 68;   // floats per query of scaled block-0/1 bases: 64, +4 (an odd count of 16-byte words)
constexpr int kSIS = 128;  // floats per item of scaled block-0/1 intervals: delta' [64], then eps' [64]
constexpr int kWB = 64;    // per-warp block-1 batch capacity
constexpr int kWQ = 64;    // per-warp deep-queue capacity (<= 31 waiting + 32 new entries)

// One 4-dim group of the scaled bound of block 1: two packed FFMA2 for u' = c * delta' + base', four
// saturating |u'| - eps', two packed FFMA2 into the running pair of partial sums.
__device__ __forceinline__ float2 scaled_group(const float2 c01, const float2 c23, const float4 dd, const float4 bb,
                                               const float4 ee, float2 acc) {
    const float2 u01 = __ffma2_rn(c01, make_float2(dd.x, dd.y), make_float2(bb.x, bb.y));
    const float2 u23 = __ffma2_rn(c23, make_float2(dd.z, dd.w), make_float2(bb.z, bb.w));
    const float l0 = __saturatef(fabsf(u01.x) - ee.x), l1 = __saturatef(fabsf(u01.y) - ee.y);
    const float l2 = __saturatef(fabsf(u23.x) - ee.z), l3 = __saturatef(fabsf(u23.y) - ee.w);
    acc = __ffma2_rn(make_float2(l0, l1), make_float2(l0, l1), acc);
    return __ffma2_rn(make_float2(l2, l3), make_float2(l2, l3), acc);
}

// One 4-dim group of the scaled bound of block 0, whose row terms x'' = c * delta' are formed once per
// row and reused for every query: two packed FADD2 for u' = x'' + base', four saturating |u'| - eps',
// two packed FFMA2 into the running pair of partial sums.
__device__ __forceinline__ float2 scaled_group0(const float4 xd, const float4 bb, const float4 ee, float2 acc) {
    const float2 u01 = __fadd2_rn(make_float2(xd.x, xd.y), make_float2(bb.x, bb.y));
    const float2 u23 = __fadd2_rn(make_float2(xd.z, xd.w), make_float2(bb.z, bb.w));
    const float l0 = __saturatef(fabsf(u01.x) - ee.x), l1 = __saturatef(fabsf(u01.y) - ee.y);
    const float l2 = __saturatef(fabsf(u23.x) - ee.z), l3 = __saturatef(fabsf(u23.y) - ee.w);
    acc = __ffma2_rn(make_float2(l0, l1), make_float2(l0, l1), acc);
    return __ffma2_rn(make_float2(l2, l3), make_float2(l2, l3), acc);
}

constexpr int kNBS = 16;  // blocks [kB0, kNBS) have a per-query base staged in shared memory
constexpr int kBS = 36;  // shared-memory stride of one 32-dim block (floats): 4 banks apart per block
constexpr int kB0 = 2;   // first block with a per-query base in shared memory (blocks 0-1 use the scaled form)
constexpr int kGC = 4;   // queries per CM-FP32 chunk: a chunk adds at most kGC * T survivors
constexpr int kQM = 4;   // survivor-list capacity in units of T entries (>= kGC, >= the seed count)
constexpr int kNBR = 1;  // code blocks a lane loads per deep-queue round (2 and 4 measured slower)
constexpr int kWL = 32 * kQM;  // per-warp level-list capacity: the warps share the survivor list's space
constexpr int kLevelMin = 12;  // a shorter level list continues in the deep queue

// Survivor / deep-queue entry: query slot j (kJBits bits) and list-local row r (the rest).
constexpr int kJBits = kMaxG <= 32 ? 5 : 6;
__device__ __forceinline__ uint32_t pack_jr(int j, int r) { return ((uint32_t)j << (32 - kJBits)) | (uint32_t)r; }
__device__ __forceinline__ int entry_j(uint32_t e) { return (int)(e >> (32 - kJBits)); }
__device__ __forceinline__ int entry_r(uint32_t e) { return (int)(e & ((1u << (32 - kJBits)) - 1u)); }

template <int T, int KM, bool LB, bool UB, bool VEC4>
__global__ void __launch_bounds__(T, kScanThreadsPerSm / T) scan_kernel(const ScanArgs a) {
    constexpr int NW = T / 32;
    constexpr int QCAP = kQM * T;
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = a.G;
    const int D_pad = a.D_pad;
    const int nb = a.nb;
    const int nbs = nb < kNBS ? nb : kNBS;  // staged blocks
    const int nsb = nbs > kB0 ? nbs - kB0 : 0;  // blocks kB0 .. nbs-1 have a per-query base in smem
    // Shared-memory copies of per-dim data keep each 32-dim block kBS floats apart, so lanes at
    // different blocks of the same dims read different banks; a query's row of bases is BWS floats
    // long with BWS / 4 odd, so different queries start in different banks as well.
    const int BWS = nsb * kBS + ((nsb & 1) ? 8 : 4);
    float* s_base = reinterpret_cast<float*>(smem);
    float* s_dl = s_base + (LB ? G * BWS : 0);
    float* s_ep = s_dl + (LB ? nb * kBS : 0);
    float* s_topd = s_ep + (LB ? nb * kBS : 0);
    int32_t* s_topi = reinterpret_cast<int32_t*>(s_topd + G * KM);
    uint32_t* s_sv = reinterpret_cast<uint32_t*>(s_topi + G * KM);  // [QCAP] survivors (j, r)
    float* s_sd = reinterpret_cast<float*>(s_sv + QCAP);            // [QCAP] their exact distances
    float* s_si = s_sd + QCAP;                                          // [kSIS] scaled delta', eps' (LB)
    float* s_sq = s_si + (LB ? kSIS : 0);                               // [G][kSQS] scaled bases (LB)
    float* s_wba = s_sq + (LB ? G * kSQS : 0);                          // [NW][kWB] block-1 batch bounds
    float* s_wqa = s_wba + (LB ? NW * kWB : 0);                         // [NW][kWQ] deep-queue bounds
    uint32_t* s_wqe = reinterpret_cast<uint32_t*>(s_wqa + (LB ? NW * kWQ : 0));  // [NW][kWQ] deep (j, r)
    uint8_t* s_wbl = reinterpret_cast<uint8_t*>(s_wqe + (LB ? NW * kWQ : 0));    // [NW][kWB] batch lanes
    uint8_t* s_wbj = s_wbl + (LB ? NW * kWB : 0);                       // [NW][kWB] batch queries
    uint8_t* s_wqb = s_wbj + (LB ? NW * kWB : 0);                       // [NW][kWQ] deep next block

    __shared__ int32_t s_qid[kMaxG], s_pp[kMaxG], s_seed[kMaxG];
    __shared__ float s_tau[kMaxG], s_ts[kMaxG], s_sig[kMaxG], s_scale[kMaxG], s_s2inv[kMaxG], s_tsp[kMaxG];
    __shared__ int s_item, s_sn, s_chunk, s_lock[kMaxG];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, D = a.D;
    unsigned long long st_cand = 0, st_dims = 0, st_surv = 0, st_ins = 0, st_items = 0;

    // Items are claimed one ahead: thread 0 holds the next item's index in a register, so the claim's
    // atomic round trip overlaps the current item.
    int next_item = tid == 0 ? atomicAdd(a.work_ctr, 1) : 0;
    for (;;) {
        if (tid == 0) {
            s_item = next_item;
            next_item = atomicAdd(a.work_ctr, 1);
            s_sn = 0;
            s_chunk = 0;
        }
        __syncthreads();
        const int it = s_item;
        if (it >= *a.n_items) break;
        const int4 item = a.items[it];
        const int c = item.x, pstart = item.y, n = item.z;
        const int64_t r0 = a.row_off[c];
        const int L = (int)(a.row_off[c + 1] - r0);
        const int64_t t0 = a.tile_off[c];
        const int nt = (L + T - 1) / T;
        const float* vm_c = a.vmin + (int64_t)c * D_pad;
        const uint8_t* codes_c = a.codes + (size_t)t0 * nb * T * 32;
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
            s_seed[tid] = 0;
            s_scale[tid] = 1.0f;
            s_lock[tid] = 0;
        }
        if (LB) {
            const float4* d4 = reinterpret_cast<const float4*>(a.delta + (int64_t)c * D_pad);
            const float4* e4 = reinterpret_cast<const float4*>(a.eps + (int64_t)c * D_pad);
            for (int i = tid; i < D_pad / 4; i += T) {
                const int o = (i >> 3) * (kBS / 4) + (i & 7);
                reinterpret_cast<float4*>(s_dl)[o] = __ldg(d4 + i);
                reinterpret_cast<float4*>(s_ep)[o] = __ldg(e4 + i);
            }
        }
        for (int i = tid; i < n * KM; i += T) {
            s_topd[i] = kInf;
            s_topi[i] = -1;
        }
        __syncthreads();
        if (LB) {
            // base_j = vmin_c - q~_j on the staged blocks, float4 over dims, four loads in flight per thread
            const float4* vm4 = reinterpret_cast<const float4*>(vm_c + 32 * kB0);
            const int per = nsb * 8, tot = n * per;
#pragma unroll 4
            for (int i = tid; i < tot; i += T) {
                const int j = i / per, f = i - j * per;
                const float4 x = __ldg(vm4 + f);
                const float4 y = __ldg(reinterpret_cast<const float4*>(a.qrot + (int64_t)s_qid[j] * D_pad + 32 * kB0) + f);
                reinterpret_cast<float4*>(s_base + j * BWS)[(f >> 3) * (kBS / 4) + (f & 7)] =
                    make_float4(x.x - y.x, x.y - y.y, x.z - y.z, x.w - y.w);
            }
        }
        __syncthreads();

        // ---- Stage Z + per-query top-K insertion over the survivor list, then the threshold exchange
        // of query slots [jlo, jhi) (the slots whose lists hold exact distances only)
        auto refine = [&](int jlo, int jhi) {
            const int sn = s_sn;
            for (int s = warp; s < sn; s += NW) {
                const uint32_t e = s_sv[s];
                const float* xr = a.xb + (r0 + entry_r(e)) * D;
                const float* qr = a.xq + (int64_t)s_qid[entry_j(e)] * D;
                const float dist = exact_dist_warp<VEC4, LB ? 1 : 4>(xr, qr, D, lane);
                if (lane == 0) s_sd[s] = dist;
            }
            __syncthreads();
            for (int j = jlo + warp; j < jhi; j += NW) {
                float* ld = s_topd + j * KM;
                int32_t* li = s_topi + j * KM;
                for (int k0 = 0; k0 < sn; k0 += 32) {
                    const int k = k0 + lane;
                    bool ok = false;
                    float d = kInf;
                    int32_t id = 0;
                    if (k < sn) {
                        const uint32_t e = s_sv[k];
                        if (entry_j(e) == j) {
                            ok = true;
                            d = s_sd[k];
                            id = __ldg(a.oid + r0 + entry_r(e));
                        }
                    }
                    if (__any_sync(TB_FULL, ok)) {
                        const int ins = list_offer<KM>(ld, li, K, ok, d, id, lane);
                        if (lane == 0) st_ins += (unsigned)ins;
                    }
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
                    const float ts = prune_threshold(tq, s_sig[j], a.rho);
                    s_ts[j] = ts;
                    const float sc = s_scale[j];
                    s_tsp[j] = (ts < kInf) ? ts * sc * sc * (1.0f + 64.0f * kU32) : kInf;
                }
            }
            st_surv += (tid == 0) ? (unsigned long long)sn : 0ull;
            __syncthreads();
            if (tid == 0) s_sn = 0;
            __syncthreads();
        };

        // ---- Stage X (optional): seed each query's threshold from SQ8 upper bounds of this list
        if (UB) {
            for (int t = 0; t < nt; ++t) {
                const int v = t * T + tid;
                const bool valid = v < L;
                const uint8_t* tp = codes_c + (size_t)t * nb * T * 32;
                for (int jc = 0; jc < n; jc += kQM) {
                    const int je = min(n, jc + kQM);
                    for (int j = jc; j < je; ++j) {
                        float ub = kInf;
                        if (valid) {
                            const float* qr = a.qrot + (int64_t)s_qid[j] * D_pad;
                            float acc = 0.0f;
                            for (int b = 0; b < nb; ++b) {
                                uint4 w0, w1;
                                load_block(tp + ((size_t)b * T + tid) * 32, w0, w1);
                                acc = (b >= kB0 && b < nbs)
                                          ? ub_block(w0, w1, s_base + j * BWS + kBS * (b - kB0), s_dl + kBS * b,
                                                     s_ep + kBS * b, acc)
                                              : bound_block_g<true>(w0, w1, vm_c + 32 * b, qr + 32 * b,
                                                                    s_dl + kBS * b, s_ep + kBS * b, acc);
                            }
                            ub = acc;
                        }
                        s_sd[(j - jc) * T + tid] = ub;
                    }
                    __syncthreads();
                    for (int j = jc + warp; j < je; j += NW) {
                        float* ld = s_topd + j * KM;
                        int32_t* li = s_topi + j * KM;
                        for (int k0 = 0; k0 < T; k0 += 32) {
                            const int k = k0 + lane;
                            const float ub = s_sd[(j - jc) * T + k];
                            list_offer<KM>(ld, li, K, ub < kInf, ub, t * T + k, lane);
                        }
                    }
                    __syncthreads();
                }
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

        // ---- Stage X (ranked seed): a query that reaches this list without a finite threshold
        // (warm-up pass, or no warm-up at all) first ranks every row of the list by its block-0
        // lower bound, refines the S best rows exactly, and starts from their K-th distance. The
        // normal Stage Y then scans every row; a seed row refined again is not inserted twice.
        if (LB && a.seed_rows > 0) {
            const int S = min(L, a.seed_rows);
            if (tid < n && !(s_tau[tid] < kInf)) s_seed[tid] = S;
            __syncthreads();
            int ns = 0;
            for (int j = 0; j < n; ++j) ns += s_seed[j] ? 1 : 0;
            if (ns > 0 && S > 0) {
                for (int t = 0; t < nt; ++t) {
                    const int v = t * T + tid;
                    float cf[32];
                    {
                        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
                        if (v < L) load_block(codes_c + (size_t)t * nb * T * 32 + (size_t)tid * 32, w0, w1);
                        unpack_block(w0, w1, cf);
                    }
                    for (int jc = 0; jc < n; jc += kQM) {
                        const int je = min(n, jc + kQM);
                        for (int j = jc; j < je; ++j)
                            if (s_seed[j])
                                s_sd[(j - jc) * T + tid] =
                                    v < L ? lb_block_f(cf, vm_c, a.qrot + (int64_t)s_qid[j] * D_pad, s_dl, s_ep, 0.0f) : kInf;
                        __syncthreads();
                        for (int j = jc + warp; j < je; j += NW) {
                            if (!s_seed[j]) continue;
                            float* ld = s_topd + j * KM;
                            int32_t* li = s_topi + j * KM;
                            for (int k0 = 0; k0 < T; k0 += 32) {
                                const int k = k0 + lane;
                                const float lb = s_sd[(j - jc) * T + k];
                                list_offer<KM>(ld, li, S, lb < kInf, lb, t * T + k, lane);
                            }
                        }
                        __syncthreads();
                    }
                }
                // the S best-ranked rows of each seeded query become survivors, refined in groups of
                // queries that fit the survivor list (S <= T <= QCAP); the lists start over
                const int per = QCAP / S;
                for (int jc = 0; jc < n; jc += per) {
                    const int je = min(n, jc + per);
                    for (int j = jc + warp; j < je; j += NW) {
                        if (!s_seed[j]) continue;
                        float* ld = s_topd + j * KM;
                        int32_t* li = s_topi + j * KM;
                        for (int k = lane; k < S; k += 32) {
                            const int32_t r = li[k];
                            if (r >= 0) {
                                const int p = atomicAdd(&s_sn, 1);
                                s_sv[p] = pack_jr(j, r);
                            }
                        }
                        __syncwarp();
                        list_init<KM>(ld, li, lane);
                    }
                    __syncthreads();
                    refine(jc, je);  // later slots still hold their ranking
                }
            }
        }

        // ---- scaled intervals for blocks 0 and 1, one scale for every query of the item:
        // s = 1/sqrt(the item's largest finite prune threshold), so each query's scaled threshold
        // ts_j s^2 stays <= 1. Then l'_d = sat(|c delta_d s + base_jd s| - eps'_d) <= s l_d, where eps'_d
        // adds the float32 roundings of the scaled terms for the largest |base_jd| of the item's
        // queries, and clamping at 1 only lowers the bound (a clamped dim already exceeds every
        // query's scaled threshold). delta' and eps' are the same for every query, so block 0 reads
        // only the query's bases (base' = base s) per query.
        if (LB) {
            const int ndim = min(nb, 2) * 32;
            float tmax = 0.0f;
            bool any = false;
            for (int j = 0; j < n; ++j) {
                const float t = s_ts[j];
                if (t < kInf) {
                    tmax = fmaxf(tmax, t);
                    any = true;
                }
            }
            const float sc = any ? 1.0f / sqrtf(fmaxf(tmax, 1e-30f)) : 1.0f;
            if (tid < n) {
                const float ts = s_ts[tid];
                s_scale[tid] = sc;
                s_s2inv[tid] = (ts < kInf) ? 1.0f / (sc * sc) * (1.0f - 4.0f * kU32) : 1.0f;
                s_tsp[tid] = (ts < kInf) ? ts * sc * sc * (1.0f + 64.0f * kU32) : kInf;
            }
            if (tid < 64) s_si[64 + tid] = 0.0f;  // the largest |base_jd| per dim, as float bits
            __syncthreads();
            // base' = (vmin - q~_j) s with the same float32 subtraction as the staged copies
            const int ng = ndim / 4;
#pragma unroll 2
            for (int i = tid; i < n * ng; i += T) {
                const int j = i / ng, g = i - j * ng;
                const float4 v4 = __ldg(reinterpret_cast<const float4*>(vm_c) + g);
                const float4 q4 = __ldg(reinterpret_cast<const float4*>(a.qrot + (int64_t)s_qid[j] * D_pad) + g);
                const float b[4] = {v4.x - q4.x, v4.y - q4.y, v4.z - q4.z, v4.w - q4.w};
                reinterpret_cast<float4*>(s_sq + j * kSQS)[g] = make_float4(b[0] * sc, b[1] * sc, b[2] * sc, b[3] * sc);
#pragma unroll
                for (int k = 0; k < 4; ++k) atomicMax(reinterpret_cast<int*>(s_si + 64 + 4 * g + k), __float_as_int(fabsf(b[k])));
            }
            __syncthreads();
            // delta' = delta s; eps' covers the roundings of delta', base', c delta' and u' (3u |term| each)
            if (tid < ndim) {
                const int sd = (tid >> 5) * kBS + (tid & 31);
                const float dl = s_dl[sd], ep = s_ep[sd];
                const float bm = s_si[64 + tid];
                s_si[tid] = dl * sc;
                s_si[64 + tid] = (ep * sc + 3.0001f * kU32 * sc * (255.0f * dl + bm)) * (1.0f + 3.0f * kU32);
            }
            __syncthreads();
        }

        if (LB) {
            // ---- Stage Y/Z, warp-independent within the item. Each warp takes 32-row chunks of the list:
            //  * block 0 for every query of the item, full warps, codes as floats in registers;
            //  * rows alive after block 0 are batched per warp; their block 1 runs densely with the
            //    codes shuffled from the owning lane;
            //  * rows alive after block 1 go to the warp's level list, which advances one block at a
            //    time over the chunk when the warp leaves it (blocks 2 .. kNBS-1, codes loaded once
            //    per chunk and block);
            //  * a short level list, and rows past the staged blocks, go to the warp's deep queue,
            //    advanced one block per lane per round (entries at mixed levels);
            //  * a row that survives every block is refined at once by its warp (exact FP32, reference
            //    order) and inserted into its query's top-K under a per-query lock; the query's
            //    threshold tightens immediately for every warp.
            // The CTA synchronises only when the item ends.
            uint8_t* wb_l = s_wbl + warp * kWB;
            uint8_t* wb_j = s_wbj + warp * kWB;
            float* wb_a = s_wba + warp * kWB;
            uint32_t* wq_e = s_wqe + warp * kWQ;
            float* wq_a = s_wqa + warp * kWQ;
            uint8_t* wq_b = s_wqb + warp * kWQ;
            int wq_n = 0;  // warp-uniform deep-queue fill
            // the chunk's level list (rows alive after block 1, then after each further block), in the
            // survivor-list space, which the CTA-wide refinement leaves unused during Stage Y/Z
            float* wl_a = s_sd + warp * kWL;
            uint8_t* wl_l = reinterpret_cast<uint8_t*>(s_sv) + warp * 2 * kWL;
            uint8_t* wl_j = wl_l + kWL;
            int wl_n = 0;  // warp-uniform fill

            // exact distance of list row r for query slot j (whole warp), insertion under the lock
            auto refine_one = [&](int j, int r) {
                const int q = s_qid[j];
                const float gq = lane == 0 ? ld_volatile_f32(a.tau + q) : kInf;  // other CTAs' threshold
                float dist = exact_dist_warp<VEC4>(a.xb + (r0 + r) * D, a.xq + (int64_t)q * D, D, lane);
                dist = __shfl_sync(TB_FULL, dist, 0);
                const int32_t id = __ldg(a.oid + r0 + r);
                int got = 0;
                if (lane == 0) {
                    for (uint32_t spin = 0; spin < a.lock_spins; ++spin) {
                        if (atomicCAS(&s_lock[j], 0, 1) == 0) { got = 1; break; }
                        __nanosleep(64);
                    }
                }
                got = __shfl_sync(TB_FULL, got, 0);
                if (!got) {  // never expected: the holder is a warp of this CTA doing one insertion
                    if (lane == 0) atomicOr(a.err, TRIDENT_STATUS_LOCK_TIMEOUT);
                    return;
                }
                __threadfence_block();
                float* ld = s_topd + j * KM;
                int32_t* li = s_topi + j * KM;
                const int ins = list_offer<KM>(ld, li, K, lane == 0, dist, id, lane);
                if (lane == 0) st_ins += (unsigned)ins;
                if (lane == 0) {
                    st_surv += 1;
                    const float kth = ld[K - 1];
                    const float t_old = s_tau[j];
                    const float tq = fminf(fminf(t_old, kth), gq);
                    if (tq < t_old) {
                        s_tau[j] = tq;
                        const float ts = prune_threshold(tq, s_sig[j], a.rho);
                        s_ts[j] = ts;
                        const float sc = s_scale[j];
                        s_tsp[j] = (ts < kInf) ? ts * sc * sc * (1.0f + 64.0f * kU32) : kInf;
                    }
                    __threadfence_block();
                    atomicExch(&s_lock[j], 0);
                    if (kth < t_old && kth < gq) atomicMin(a.tau + q, __float_as_uint(kth));
                }
                __syncwarp();
            };

            // One round over the first min(wq_n, 32 / g) deep entries with g = 2^lg lanes per entry.
            // Lane `sub` of an entry loads its kNBR blocks b + sub + k g together, then adds their
            // bounds while its own partial stays within the threshold; the group sums the partials.
            // Every term is non-negative, so a lane that stops early already proves the entry dead,
            // and a live entry has accounted for every block it advanced over (up to g kNBR).
            // Steady state runs g = 1 (32 entries, kNBR consecutive blocks each); the drain at the
            // end of an item widens g as the queue empties.
            auto deep_round = [&](int lg) {
                const int g = 1 << lg;
                const int m = min(wq_n, 32 >> lg);
                const int i = lane >> lg, sub = lane & (g - 1);
                const bool has = i < m;
                uint32_t e = 0;
                float acc = 0.0f;
                int b = nb;
                if (has) {
                    e = wq_e[i];
                    acc = wq_a[i];
                    b = wq_b[i];
                }
                const int j = entry_j(e), r = entry_r(e);
                const uint8_t* rowc = codes_c + (size_t)(r / T) * nb * T * 32 + (size_t)(r % T) * 32;
                const float* qr = a.qrot + (int64_t)s_qid[j] * D_pad;
                uint4 w[kNBR][2];
#pragma unroll
                for (int k = 0; k < kNBR; ++k) {
                    const int bb = b + sub + k * g;
                    if (bb < nb) load_block(rowc + (size_t)bb * T * 32, w[k][0], w[k][1]);
                }
                const float ts = s_ts[j];
                float part = sub == 0 ? acc : 0.0f;
#pragma unroll
                for (int k = 0; k < kNBR; ++k) {
                    const int bb = b + sub + k * g;
                    if (bb < nb && part <= ts) {
                        part = bb < nbs ? lb_block(w[k][0], w[k][1], s_base + j * BWS + kBS * (bb - kB0), s_dl + kBS * bb,
                                                   s_ep + kBS * bb, part)
                                        : bound_block_g<false>(w[k][0], w[k][1], vm_c + 32 * bb, qr + 32 * bb,
                                                               s_dl + kBS * bb, s_ep + kBS * bb, part);
                        st_dims += 32u;
                    }
                }
                for (int o = g >> 1; o > 0; o >>= 1) part += __shfl_xor_sync(TB_FULL, part, o);
                const int bn = min(b + g * kNBR, nb);
                const bool lead = has && sub == 0;
                const bool alive = lead && part <= ts;
                const bool done = alive && bn == nb;
                const bool keep = alive && bn < nb;
                const int rest = wq_n - m;
                uint32_t te = 0;
                float ta = 0.0f;
                uint8_t tb = 0;
                if (lane < rest) { te = wq_e[m + lane]; ta = wq_a[m + lane]; tb = wq_b[m + lane]; }
                __syncwarp();
                const unsigned km = __ballot_sync(TB_FULL, keep);
                const int nk = __popc(km);
                if (keep) {
                    const int p = __popc(km & ((1u << lane) - 1u));
                    wq_e[p] = e;
                    wq_a[p] = part;
                    wq_b[p] = (uint8_t)bn;
                }
                if (lane < rest) { wq_e[nk + lane] = te; wq_a[nk + lane] = ta; wq_b[nk + lane] = tb; }
                __syncwarp();
                wq_n = nk + rest;
                unsigned dm = __ballot_sync(TB_FULL, done);
                while (dm) {
                    const int s = __ffs(dm) - 1;
                    dm &= dm - 1;
                    const uint32_t es = __shfl_sync(TB_FULL, e, s);
                    refine_one(entry_j(es), entry_r(es));
                }
            };

            // The warps take the item's 32-row chunks in order as they become free, so a warp whose
            // rows run deep takes fewer chunks (a chunk never crosses a tile: T is a multiple of 32).
            const int nch = (L + 31) / 32;
            for (;;) {
                int ch = 0;
                if (lane == 0) ch = atomicAdd(&s_chunk, 1);
                ch = __shfl_sync(TB_FULL, ch, 0);
                if (ch >= nch) break;
                const int rb = ch * 32;  // first list-local row of the chunk
                const bool valid = rb + lane < L;
                const uint8_t* tp = codes_c + ((size_t)(rb / T) * nb * T + (rb % T)) * 32;
                float cf[32];
                uint4 p0 = make_uint4(0, 0, 0, 0), p1 = make_uint4(0, 0, 0, 0);
                {
                    uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
                    if (valid) {
                        load_block(tp + (size_t)lane * 32, w0, w1);
                        if (nb > 1) load_block(tp + ((size_t)T + lane) * 32, p0, p1);
                    }
                    unpack_block(w0, w1, cf);
                }
                int wcnt = 0;  // warp-uniform fill of this warp's block-1 batch
                // block 1 for the first `cnt` batched entries (codes shuffled from the owning lane)
                auto run_batch = [&](int cnt) {
                    const bool has = lane < cnt;
                    const int r = has ? wb_l[lane] : 0;
                    const int jj = has ? wb_j[lane] : 0;
                    float acc = has ? wb_a[lane] : 0.0f;
                    uint32_t w[8];
                    w[0] = __shfl_sync(TB_FULL, p0.x, r); w[1] = __shfl_sync(TB_FULL, p0.y, r);
                    w[2] = __shfl_sync(TB_FULL, p0.z, r); w[3] = __shfl_sync(TB_FULL, p0.w, r);
                    w[4] = __shfl_sync(TB_FULL, p1.x, r); w[5] = __shfl_sync(TB_FULL, p1.y, r);
                    w[6] = __shfl_sync(TB_FULL, p1.z, r); w[7] = __shfl_sync(TB_FULL, p1.w, r);
                    const float4* D1 = reinterpret_cast<const float4*>(s_si + 32);       // delta' of block 1
                    const float4* E1 = reinterpret_cast<const float4*>(s_si + 64 + 32);  // eps' of block 1
                    const float4* B1 = reinterpret_cast<const float4*>(s_sq + jj * kSQS + 32);
                    float2 a2 = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        a2 = scaled_group(make_float2(u8f(w[g], 0), u8f(w[g], 1)), make_float2(u8f(w[g], 2), u8f(w[g], 3)),
                                          D1[g], B1[g], E1[g], a2);
                    }
                    acc += a2.x + a2.y;
                    const bool alive = has && acc <= s_tsp[jj];
                    if (has) st_dims += 32u;
                    const int row = rb + r;
                    const unsigned m = __ballot_sync(TB_FULL, alive);
                    if (nb <= 2) {
                        unsigned dm = m;
                        while (dm) {
                            const int s = __ffs(dm) - 1;
                            dm &= dm - 1;
                            refine_one(__shfl_sync(TB_FULL, jj, s), __shfl_sync(TB_FULL, row, s));
                        }
                    } else if (m) {
                        const int nm = __popc(m);
                        const int p = __popc(m & ((1u << lane) - 1u));
                        if (wl_n + nm <= kWL) {
                            if (alive) {
                                wl_l[wl_n + p] = (uint8_t)r;
                                wl_j[wl_n + p] = (uint8_t)jj;
                                wl_a[wl_n + p] = acc * s_s2inv[jj];  // back to unscaled units
                            }
                            __syncwarp();
                            wl_n += nm;
                        } else {
                            if (alive) {
                                wq_e[wq_n + p] = pack_jr(jj, row);
                                wq_a[wq_n + p] = acc * s_s2inv[jj];
                                wq_b[wq_n + p] = 2;
                            }
                            __syncwarp();
                            wq_n += nm;
                        }
                    }
                    // move the unprocessed tail [cnt, wcnt) to the front
                    const int rest = wcnt - cnt;
                    uint8_t tl = 0, tj = 0;
                    float ta = 0.0f;
                    if (lane < rest) { tl = wb_l[cnt + lane]; tj = wb_j[cnt + lane]; ta = wb_a[cnt + lane]; }
                    __syncwarp();
                    if (lane < rest) { wb_l[lane] = tl; wb_j[lane] = tj; wb_a[lane] = ta; }
                    __syncwarp();
                    wcnt = rest;
                };
                // block 0's row terms x'' = c * delta', kept in registers for all the item's queries; eps'
                // (the same for every query) is read from shared memory with the query's bases
                float4 xd[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const float4 d4 = reinterpret_cast<const float4*>(s_si)[g];
                    const float2 x01 = __fmul2_rn(make_float2(cf[4 * g], cf[4 * g + 1]), make_float2(d4.x, d4.y));
                    const float2 x23 = __fmul2_rn(make_float2(cf[4 * g + 2], cf[4 * g + 3]), make_float2(d4.z, d4.w));
                    xd[g] = make_float4(x01.x, x01.y, x23.x, x23.y);
                }
                const float4* E0 = reinterpret_cast<const float4*>(s_si + 64);
                for (int j = 0; j < n; ++j) {
                    const float4* Bq = reinterpret_cast<const float4*>(s_sq + j * kSQS);
                    float2 a2 = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int g = 0; g < 8; ++g) a2 = scaled_group0(xd[g], Bq[g], E0[g], a2);
                    const float acc = a2.x + a2.y;
                    const bool alive = valid && acc <= s_tsp[j];
                    const unsigned m = __ballot_sync(TB_FULL, alive);
                    if (!m) continue;
                    if (nb == 1) {
                        unsigned dm = m;
                        while (dm) {
                            const int s = __ffs(dm) - 1;
                            dm &= dm - 1;
                            refine_one(j, rb + s);
                        }
                        continue;
                    }
                    if (alive) {
                        const int p = wcnt + __popc(m & ((1u << lane) - 1u));
                        wb_l[p] = (uint8_t)lane;
                        wb_j[p] = (uint8_t)j;
                        wb_a[p] = acc;
                    }
                    __syncwarp();
                    wcnt += __popc(m);
                    if (wcnt >= 32) {
                        run_batch(32);
                        while (wq_n >= 32) deep_round(0);
                    }
                }
                if (valid) {  // block 0 of this row for every query of the item
                    st_cand += (unsigned)n;
                    st_dims += 32u * (unsigned)n;
                }
                // the chunk's block-1 codes leave the registers: finish this warp's batch
                if (wcnt > 0) run_batch(wcnt);
                while (wq_n >= 32) deep_round(0);  // room for a short level list (< kLevelMin entries)
                // Blocks 2, 3, ... for the chunk's level list, one block at a time: the block's codes of
                // the chunk's 32 rows are loaded once (coalesced) and shuffled from the owning lane, and
                // the list is compacted in place. A short list, and every row past the staged blocks,
                // continues in the deep queue.
                const int b_end = min(nbs, nb - 1);
                int b = 2;
                uint4 n0 = make_uint4(0, 0, 0, 0), n1 = make_uint4(0, 0, 0, 0);
                if (valid && wl_n >= kLevelMin && b < b_end) load_block(tp + ((size_t)b * T + lane) * 32, n0, n1);
                for (; wl_n >= kLevelMin && b < b_end; ++b) {
                    const uint4 c0 = n0, c1 = n1;
                    if (valid && b + 1 < b_end) load_block(tp + ((size_t)(b + 1) * T + lane) * 32, n0, n1);
                    int wn = 0;
                    for (int k0 = 0; k0 < wl_n; k0 += 32) {
                        const bool has = k0 + lane < wl_n;
                        const int r = has ? wl_l[k0 + lane] : 0;
                        const int jj = has ? wl_j[k0 + lane] : 0;
                        float acc = has ? wl_a[k0 + lane] : 0.0f;
                        const uint4 w0 = make_uint4(__shfl_sync(TB_FULL, c0.x, r), __shfl_sync(TB_FULL, c0.y, r),
                                                    __shfl_sync(TB_FULL, c0.z, r), __shfl_sync(TB_FULL, c0.w, r));
                        const uint4 w1 = make_uint4(__shfl_sync(TB_FULL, c1.x, r), __shfl_sync(TB_FULL, c1.y, r),
                                                    __shfl_sync(TB_FULL, c1.z, r), __shfl_sync(TB_FULL, c1.w, r));
                        acc = lb_block(w0, w1, s_base + jj * BWS + kBS * (b - kB0), s_dl + kBS * b, s_ep + kBS * b, acc);
                        if (has) st_dims += 32u;
                        const bool alive = has && acc <= s_ts[jj];
                        const unsigned m = __ballot_sync(TB_FULL, alive);
                        __syncwarp();  // every entry of this batch is read before survivors overwrite
                        if (alive) {
                            const int p = wn + __popc(m & ((1u << lane) - 1u));
                            wl_l[p] = (uint8_t)r;
                            wl_j[p] = (uint8_t)jj;
                            wl_a[p] = acc;
                        }
                        wn += __popc(m);
                        __syncwarp();
                    }
                    wl_n = wn;
                }
                for (int k0 = 0; k0 < wl_n; k0 += 32) {  // the rest continues at block b
                    const int cnt = min(32, wl_n - k0);
                    if (lane < cnt) {
                        wq_e[wq_n + lane] = pack_jr(wl_j[k0 + lane], rb + wl_l[k0 + lane]);
                        wq_a[wq_n + lane] = wl_a[k0 + lane];
                        wq_b[wq_n + lane] = (uint8_t)b;
                    }
                    __syncwarp();
                    wq_n += cnt;
                    while (wq_n >= 32) deep_round(0);
                }
                wl_n = 0;
                while (wq_n >= 32) deep_round(0);
            }
            // drain the deep queue, giving each remaining entry as many lanes as fit
            while (wq_n > 0) {
                int lg = 0;
                while (lg < 5 && (wq_n << (lg + 1)) <= 32) ++lg;
                deep_round(lg);
            }
            __syncthreads();
        } else {
            for (int t = 0; t < nt; ++t) {
                const int v = t * T + tid;
                const bool valid = v < L;
                const int Lt = min(T, L - t * T);
                // ---- CM-FP32: every row of the tile is refined for every query of the item
                if (valid) st_cand += n;
                for (int jc = 0; jc < n; jc += kGC) {
                    if (s_sn > QCAP - kGC * T) refine(0, n);
                    const int je = min(n, jc + kGC);
                    for (int i = tid; i < (je - jc) * Lt; i += T) {
                        const int j = jc + i / Lt, r = t * T + i % Lt;
                        s_sv[s_sn + i] = pack_jr(j, r);
                    }
                    __syncthreads();
                    if (tid == 0) s_sn += (je - jc) * Lt;
                    __syncthreads();
                }
            }
            if (s_sn > 0) refine(0, n);
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
                                                   int64_t* __restrict__ out_i, const int32_t* __restrict__ err) {
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
        // A scan whose bounded lock wait gave up may have dropped a candidate: every result row is
        // then marked (NaN, -2) instead of being returned possibly incomplete.
        const bool bad = ld_volatile_i32(err) != 0;
        for (int k = lane; k < K; k += 32) {
            out_d[(int64_t)q * K + k] = bad ? __int_as_float(0x7fc00000) : ld[k];
            out_i[(int64_t)q * K + k] = bad ? (int64_t)-2 : (int64_t)li[k];
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
    bool bad = false;  // some shard marked this query: a bounded wait gave up there
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        float d = kInf;
        int64_t id = -1;
        if (k < n) {
            const int r = k / K, kk = k - r * K;
            d = d_in[((int64_t)r * B + q) * K + kk];
            id = i_in[((int64_t)r * B + q) * K + kk];
        }
        bad |= id == -2;
        list_offer<KM>(ld, li, K, id >= 0, d, (int32_t)id, lane);
    }
    bad = __any_sync(TB_FULL, bad);
    __syncwarp();
    for (int k = lane; k < K; k += 32) {
        out_d[(int64_t)q * K + k] = bad ? __int_as_float(0x7fc00000) : ld[k];
        out_i[(int64_t)q * K + k] = bad ? (int64_t)-2 : (int64_t)li[k];
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
static int km_for(int K) { return K <= 32 ? 32 : 128; }

static size_t scan_smem(const trident_index& idx, int K, int G, bool lb) {
    const int T = idx.tile_size;
    const int KM = km_for(K);
    const int nbs = idx.num_blocks < kNBS ? idx.num_blocks : kNBS;
    const size_t qcap = (size_t)kQM * T;
    size_t s = 0;
    const int nsb = nbs > kB0 ? nbs - kB0 : 0;
    const size_t bws = (size_t)nsb * kBS + ((nsb & 1) ? 8 : 4);
    if (lb) s += ((size_t)G * bws + 2 * (size_t)idx.num_blocks * kBS) * sizeof(float);  // base, delta, eps
    s += (size_t)G * KM * (sizeof(float) + sizeof(int32_t));                          // top-K lists
    s += qcap * (sizeof(uint32_t) + sizeof(float));                                   // survivors + distances
    if (lb) s += ((size_t)kSIS + (size_t)G * kSQS) * sizeof(float);                  // scaled intervals
    if (lb) s += (size_t)(T / 32) * kWB * (sizeof(float) + 2);                         // block-1 batches
    if (lb) s += (size_t)(T / 32) * kWQ * (sizeof(float) + sizeof(uint32_t) + 1);      // deep queues
    return s;
}

int scan_group_size(const trident_index& idx, int K) {
    // kScanThreadsPerSm / T CTAs share an SM's 228 KB; 4 KB per CTA stay for static shared memory and
    // the per-CTA reserve.
    const size_t ctas = (size_t)(kScanThreadsPerSm / idx.tile_size);
    const size_t budget = (228 * 1024) / ctas - 4 * 1024;
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
    a.items = (sl.pass == 1 ? ws.items_lpt : ws.items) + (sl.pass == 1 ? 0 : sl.item_base);
    a.n_items = ws.ctr + sl.pass;
    a.work_ctr = ws.ctr + 2 + sl.pass;
    a.pair_q = ws.pair_q;
    a.pair_p = ws.pair_p;
    a.tau = ws.tau;
    a.cand_d = ws.cand_d;
    a.cand_i = ws.cand_i;
    a.stats = stats;
    a.err = ws.ctr + kStatusWord;
    a.lock_spins = lock_spin_limit();
    a.D = idx.D;
    a.D_pad = idx.D_pad;
    a.nb = idx.num_blocks;
    a.K = sl.K;
    a.nprobe = sl.nprobe;
    a.G = sl.G;
    a.seed_rows = sl.lb ? 32 * ((sl.K + 31) / 32) : 0;
    if (a.seed_rows > idx.tile_size) a.seed_rows = idx.tile_size;
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
        merge_kernel<32><<<grid, 256, 0, st>>>(ws.cand_d, ws.cand_i, B, K, nprobe, p_lo, p_hi, tau_out, out_d, out_i,
                                                ws.ctr + kStatusWord);
    else
        merge_kernel<128><<<grid, 256, 0, st>>>(ws.cand_d, ws.cand_i, B, K, nprobe, p_lo, p_hi, tau_out, out_d, out_i,
                                                 ws.ctr + kStatusWord);
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
