// Host-side launchers shared between the trident_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "trident_b200.h"

namespace tb {

// Per-query side information written by the rotation kernel. QI_PAD carries the int bits of the
// coarse stage's status (0 = ok) for that query.
enum QInfo { QI_QNORM = 0, QI_SIGMA = 1, QI_CNORM = 2, QI_PAD = 3, QI_LEN = 4 };

// Word of the counter block that holds the search's device-side status (TRIDENT_STATUS_*).
constexpr int kStatusWord = 15;
// Lists per tile of the coarse GEMM, and per entry of its row minima (two entries per tile).
constexpr int kCoarseTileN = 128;
constexpr int kCoarseMinSpan = 64;

// Workspace carve-up for one call (B, K, nprobe); every region is 256-byte aligned. The counter
// block comes first, so the status word sits at the same offset whatever B, K and nprobe are.
struct Workspace {
    float* qrot;        // [B, D_pad]
    float* qinfo;       // [B, QI_LEN]
    float* coarse;      // [B, nlist] approximate ||c||^2 - 2 q.c
    float* tilemin;     // [B, ceil(nlist / kCoarseMinSpan)] minimum of each row over each 64-list span
    float* gsplit;      // coarse_split_bytes(idx, B): TF32 hi/lo splits of queries and centroids
    int32_t* probe;     // [B, nprobe]
    int32_t* cnt;       // [2, nlist]
    int32_t* off;       // [2, nlist + 1]
    int32_t* cursor;    // [2, nlist]
    int32_t* item_off;  // [2, nlist + 1]
    int32_t* pair_q;    // [B * nprobe]
    int32_t* pair_p;    // [B * nprobe]
    int4* items;        // [B * nprobe] in list order
    int4* items_lpt;    // [B * nprobe] the same items, most expensive first
    int32_t* lpt;       // [kLptBins] bin counts, then bin cursors
    uint32_t* tau;      // [B] float bits of each query's current K-th distance
    float* cand_d;      // [B, nprobe, K]
    int32_t* cand_i;    // [B, nprobe, K]
    int32_t* ctr;       // [16] item counts and work counters; ctr[kStatusWord] = status
    size_t bytes;
};

// Process-wide limits of the bounded waits (trident_set_wait_limits).
uint32_t lock_spin_limit();   // per-query insertion lock of the scan
uint32_t mma_wait_limit();    // tensor-core completion (mbarrier) polls of the coarse GEMM

size_t carve_workspace(const trident_index& idx, int B, int K, int nprobe, void* base, Workspace* ws);

// Coarse stage (tb_coarse.cu).
// Per-query norms and sigma into qinfo, tau = +inf (query_norms_kernel), and the float64 rotation
// into qrot (rotate_f64_kernel); launch_rotate runs both on one stream.
cudaError_t launch_query_norms(const trident_index& idx, const float* xq, int B, float* qinfo, uint32_t* tau,
                               cudaStream_t st);
cudaError_t launch_rotate_f64(const trident_index& idx, const float* xq, int B, float* qrot, cudaStream_t st);
cudaError_t launch_rotate(const trident_index& idx, const float* xq, int B, float* qrot, float* qinfo,
                          uint32_t* tau, cudaStream_t st);
// Persistent TMA-fed tcgen05 GEMM (tb_gemm.cu), 3xTF32; sets *err |= TRIDENT_STATUS_MMA_TIMEOUT if a
// bounded wait gave up. tilemin (optional, [B, ceil(nlist / kCoarseMinSpan)]) receives each row's
// minimum over each 64-list span; splits is scratch of coarse_split_bytes(idx, B) bytes for the operands'
// TF32 hi/lo splits.
size_t coarse_split_bytes(const trident_index& idx, int B);
cudaError_t launch_coarse_gemm(const trident_index& idx, const float* xq, int B, float* coarse, float* tilemin,
                               float* splits, int32_t* err, cudaStream_t st);
// The same GEMM with an argmin epilogue (1xTF32): out[i] = argmin_c (cnorm[c] - 2 x_i.c), ties to the
// smaller c. Needs D % 4 == 0 and 16-byte aligned x and cent.
cudaError_t launch_assign(const float* x, int64_t n, int D, const float* cent, const float* cnorm, int nlist,
                          int32_t* out, int32_t* err, cudaStream_t st);
// Exact probe lists. A nonzero *err (the GEMM gave up) marks every probe list -1 (and probe_d64 NaN)
// and is copied into each query's qinfo[QI_PAD], which travels with the query to other GPUs.
// tilemin (optional) lets selection above 8192 lists bound the nprobe-th value without re-reading
// the row per bit.
cudaError_t launch_probe_select(const trident_index& idx, const float* xq, int B, int nprobe, const float* coarse,
                                const float* tilemin, float* qinfo, int32_t* probe, double* probe_d64,
                                unsigned long long* stats, const int32_t* err, cudaStream_t st);

// Pair lists and work items (tb_pairs.cu).
cudaError_t launch_pairs(const trident_index& idx, const int32_t* probe, int B, int nprobe, int p_init, int G, int K,
                         const Workspace& ws, cudaStream_t st);
constexpr int kLptBins = 128;
// Reorders the main pass's items by estimated cost, largest first (longest-processing-time order),
// into ws.items_lpt.
cudaError_t launch_item_order(const trident_index& idx, int max_items, const Workspace& ws, cudaStream_t st);

// tau[0..n) = +inf (float bits), tb_seed.cu.
cudaError_t launch_fill_inf(uint32_t* tau, int n, cudaStream_t st);
// tau[0..B) = +inf, and the status that a query's coarse stage left in qinfo[QI_PAD] (possibly on
// another GPU) is or-ed into *err.
cudaError_t launch_tau_init_import_status(uint32_t* tau, const float* qinfo, int B, int32_t* err, cudaStream_t st);

// Query-major threshold seeding (tb_seed.cu): rank the rows of each query's p_seed nearest lists by
// a partial SQ8 distance, refine the best exactly (or bound them from above with ub) and store the
// K-th value in ws.tau.
int seed_lists_for(int B, int K, int nprobe);
// seed_d/seed_i (optional, [B, K]) receive each query's K smallest seed values and their row ids;
// shard = 1 sizes the refined set by the share of the seed lists this GPU holds.
cudaError_t launch_seed(const trident_index& idx, const float* xq, const Workspace& ws, int B, int K, int nprobe,
                        int p_seed, int ub, float* seed_d, int64_t* seed_i, int shard, cudaStream_t st);

// Scans and merges (tb_scan.cu).
struct ScanLaunch {
    int pass;        // 0: warm-up lists, 1: the rest
    int K;
    int nprobe;
    int G;           // queries per work item
    int lb;          // 1: Stage Y lower bound (cascade), 0: CM-FP32 exact scan
    int ub_seed;     // 1: seed each item's threshold from SQ8 upper bounds first
    int max_items;   // upper bound on the item count of this pass
    int64_t item_base;  // index of this pass's first item in the item array
    int filter;      // 1: Stage Y on the tensor cores (tb_filter.cu) instead of scan_kernel
};
cudaError_t launch_scan(const trident_index& idx, const float* xq, const Workspace& ws, const ScanLaunch& sl,
                        unsigned long long* stats, cudaStream_t st);
int scan_group_size(const trident_index& idx, int K);
// Stage Y on the tensor cores (tb_filter.cu): whether it serves this search, its queries per item,
// and its launch (same items, thresholds and candidate slots as launch_scan).
bool filter_eligible(const trident_index& idx, int K, bool lb, bool ub_items, int64_t pairs);
int filter_group_size(const trident_index& idx, int K);
cudaError_t launch_filter(const trident_index& idx, const float* xq, const Workspace& ws, const ScanLaunch& sl,
                          unsigned long long* stats, cudaStream_t st);
cudaError_t launch_merge(const Workspace& ws, int B, int K, int nprobe, int p_lo, int p_hi, uint32_t* tau_out,
                         float* out_d, int64_t* out_i, cudaStream_t st);
cudaError_t launch_merge_shards(const float* d_in, const int64_t* i_in, int R, int B, int K, float* out_d,
                                int64_t* out_i, cudaStream_t st);

int num_sms();

// Store `msg` as the calling thread's last error (trident_last_error) and return `code`.
int record_error(int code, const char* msg);

}  // namespace tb
