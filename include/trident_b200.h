/*
 * trident_b200 — C ABI of the B200 (sm_100a) TRIDENT lossless IVF query path.
 *
 * The reference exposes this path as one pybind11 call,
 *   launch_trident_v4_search(mode, tile_size, use_l1, per_cluster_sq8, rerank_m, nprobe, xq_orig,
 *                            W_combined, ..., topk_d, topk_i, ..., record_events, warp_refine,
 *                            stats_buf, r_vec_sorted) -> float ms
 * (src/trident_v4_kernels.cu:1172-1217, bound at :1606-1627), called by TridentV4Index.search
 * (benchmarks/phase4a_suite.py:280-342). The entry points below replace that call and its pieces.
 * They take plain pointers and sizes only; the caller owns every buffer (index arrays, workspace,
 * outputs), as in the reference, and no entry point allocates device memory.
 *
 * Conventions shared by every entry point:
 *  - return TRIDENT_OK (0) or a TRIDENT_ERR_* code; trident_last_error() gives the message of the
 *    calling thread's last failure (the reference surfaced no errors at all);
 *  - all work is queued on `stream` (a cudaStream_t; NULL = the legacy default stream) and is
 *    asynchronous, like the reference, which ran on torch's current stream (:1231);
 *  - one workspace must not be used by two searches that overlap in time (the reference's scratch
 *    buffers had the same restriction).
 */
#ifndef TRIDENT_B200_H
#define TRIDENT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRIDENT_ABI_VERSION 2

enum trident_status {
    TRIDENT_OK = 0,
    TRIDENT_ERR_INVALID = 1,     /* bad argument, shape or pointer                      */
    TRIDENT_ERR_WORKSPACE = 2,   /* workspace smaller than trident_workspace_size()     */
    TRIDENT_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed         */
    TRIDENT_ERR_UNSUPPORTED = 4  /* a mode or shape this build does not implement       */
};

/* Search modes; the values are the reference's `mode` argument (:1173). */
enum trident_mode {
    TRIDENT_MODE_AUTO = -1,      /* cost router: CM-FP32 if W < w0 else cascade (phase4a_suite.py:1079) */
    TRIDENT_MODE_CASCADE = 2,    /* K2: Stage X warm-up, Stage Y SQ8 lower bound, Stage Z FP32 refine   */
    TRIDENT_MODE_CM_FP32 = 10    /* exact cluster-major FP32 scan of every probed row                   */
};

/* Index arrays on the device (xb_sorted may instead be mapped pinned host memory: the zero-copy
 * out-of-core mode). They carry the semantics of the reference's SharedClusterStorage and
 * TridentV4Index arrays (phase4a_suite.py:75-255) in a B200 layout:
 *   codes    [total_tiles][num_blocks][tile_size][32] u8: tile t of list c holds rows
 *            list_row_off[c] + (t - list_tile_off[c]) * tile_size + v, 32 dims per block; one
 *            32-dim block of one row is one 32-byte DRAM sector (reference layout:
 *            sq8_packed [tiles][D4][W][32] u32, :189-230);
 *   vmin/delta [nlist][D_pad]: per-list SQ8 interval, codes = clip(round((x~ - vmin)/delta),0,255)
 *            of the float32 PCA-rotated row x~ (phase4a_suite.py:157-179);
 *   eps      [nlist][D_pad]: rigorous per-dim bound on |x~ - (vmin + code*delta)| plus the float32
 *            rounding of the bound's arithmetic (the reference used 0.5001*delta, :179). */
typedef struct trident_index {
    int64_t N;                       /* rows                                             */
    int32_t D;                       /* dimension                                        */
    int32_t D_pad;                   /* ceil(D/32)*32                                    */
    int32_t nlist;                   /* IVF lists                                        */
    int32_t tile_size;               /* rows per tile: 128 or 256                        */
    int32_t num_blocks;              /* D_pad / 32                                       */
    int32_t flags;                   /* TRIDENT_INDEX_* bits, 0 by default                */
    const float*   xb_sorted;        /* [N, D] rows in list order                        */
    const int32_t* orig_ids_sorted;  /* [N] original id of each sorted row               */
    const int64_t* list_row_off;     /* [nlist+1] (reference: cluster_vec_off, int32)    */
    const int64_t* list_tile_off;    /* [nlist+1] (reference: cluster_tile_off)          */
    const uint8_t* codes;            /* blocked SQ8 codes, see above                     */
    const float*   vmin;             /* [nlist, D_pad]                                   */
    const float*   delta;            /* [nlist, D_pad]                                   */
    const float*   eps;              /* [nlist, D_pad]                                   */
    const float*   centroids;        /* [nlist, D]                                       */
    const float*   centroid_norm_sq; /* [nlist] ||c||^2 rounded from float64             */
    const double*  pca_mean;         /* [D]                                              */
    const double*  pca_rot;          /* [D, D] row-major; column d is component d        */
    float centroid_norm_max;         /* max_c ||c||, for the coarse GEMM error bound     */
    float lb_rel_slack;              /* relative slack rho of the Stage-Y prune test     */
    /* Optional [total_tiles * tile_size], in code-slot order (tile t, row v of the tile): the row's
     * sum_d (code_d delta_d)^2 in float64, rounded down to float (0 for empty slots). With it the
     * cascade runs Stage Y on the tensor cores (an 8-bit MMA per 32-dim code block and a bound over
     * all dims at once) when D_pad <= 256 and B * nprobe >= 32768, where it is the faster
     * (or always, with TRIDENT_INDEX_TENSOR_STAGE_Y_ALWAYS); NULL keeps the CUDA-core Stage Y.
     * Results are the same either way. */
    const float*   row_p;
} trident_index;

/* trident_index.flags: run Stage Y on the tensor cores for every cascade search (given row_p),
 * not only where the library's size rule picks it (D_pad <= 256, B * nprobe >= 32768). */
#define TRIDENT_INDEX_TENSOR_STAGE_Y_ALWAYS 1

/* Statistics slots of the optional int64 `stats` array (at least TRIDENT_STATS_LEN entries, zeroed
 * by the caller). Slots 0-3 are the reference's stats_buf counters (:700-704, :774-795, :921-923). */
enum trident_stat_slot {
    TRIDENT_STAT_CANDIDATES = 0,     /* (query, row) pairs entering Stage Y                     */
    TRIDENT_STAT_SCANNED_DIMS = 1,   /* dimensions scanned by Stage Y                           */
    TRIDENT_STAT_SURVIVORS = 2,      /* pairs reaching Stage Z (exact FP32)                     */
    TRIDENT_STAT_INSERTED = 3,       /* refined rows inserted into a per-query top-K            */
    TRIDENT_STAT_COARSE_RECHECK = 4, /* lists re-checked in float64 at the nprobe boundary      */
    TRIDENT_STAT_ITEMS = 5,          /* (list, query-group) work items processed                */
    TRIDENT_STATS_LEN = 8
};

/* Version of this ABI (TRIDENT_ABI_VERSION). */
int trident_version(void);

/* Message of the calling thread's last failed call ("" if none). */
const char* trident_last_error(void);

/* Checks the index descriptor (shapes, tile size, alignment of the row array). */
int trident_index_check(const trident_index* idx);

/* Workspace bytes a search of (B, K, nprobe) needs. Replaces the reference's preallocated
 * scratch tensors (proj_buf ... cand_cnt, phase4a_suite.py:257-278). */
int trident_workspace_size(const trident_index* idx, int32_t B, int32_t K, int32_t nprobe,
                           size_t* bytes);

/* The warm-up split m_warm (p_init) the reference uses for mode 2 (:1264-1276). The search seeds its
 * thresholds from max(p_init, min(8, nprobe / 8)) nearest lists of each query. */
int32_t trident_p_init(int32_t mode, int32_t B, int32_t K, int32_t nprobe);

/* Router thresholds. The reference calibrated W0 = 9e8 on an A100 (phase4a_suite.py:1013-1035,
 * data/phase6/auto_v2.csv). The same rule on a B200 (python -m trident_b200.calibrate: the smallest W
 * at which the cascade is at least as fast as the CM-FP32 scan, over B = 1..1024 on the c1-c3
 * stand-ins) finds the cascade faster at every batch size measured, down to W = 8e5 (c1, B = 1). */
#define TRIDENT_ROUTE_W0_A100 9.0e8
#define TRIDENT_ROUTE_W0_B200 8.0e5

/* The cost router (phase4a_suite.py:1013-1035, 1079): returns TRIDENT_MODE_CM_FP32 when
 * W = B * nprobe * (N / nlist) * D < w0, else TRIDENT_MODE_CASCADE. w0 <= 0 selects
 * TRIDENT_ROUTE_W0_B200. */
int32_t trident_route(const trident_index* idx, int32_t B, int32_t nprobe, double w0);

/* 1 when a cascade search of this shape (mode 2, ub_seed 0 or 1) runs Stage Y on the tensor cores,
 * 0 when it runs the CUDA-core Stage Y (no reference counterpart: the reference has one Stage Y). */
int32_t trident_stage_y_tensor(const trident_index* idx, int32_t B, int32_t K, int32_t nprobe, int32_t ub_seed);

/* The whole query path, replacing launch_trident_v4_search (:1172-1604). The cascade runs as
 * coarse stage -> Stage X seed (each query's threshold from the best rows of its nearest lists,
 * ranked by a partial SQ8 distance) -> one Stage Y/Z scan over every probe -> merge, where the
 * reference ran a warm-up scan over its p_init lists before the main scan.
 *   xq       [B, D] float32 queries on the device;
 *   K        1..100 (the reference supported K = 10 only, :575, :984);
 *   mode     TRIDENT_MODE_{AUTO, CASCADE, CM_FP32};
 *   ub_seed  0: the Stage X seed refines its rows exactly; 1: it bounds them with SQ8 upper bounds
 *            instead, reading no FP32 row (for rows in host memory); 2: as 1, and every scan work
 *            item also seeds from upper bounds (the reference's TRIDENT_UB_SEED, :1262, now an
 *            argument);
 *   out_d    [B, K] float32 squared distances ascending; out_i [B, K] int64 original ids;
 *            ties are broken by the smaller id; missing results are (+inf, -1). Every row
 *            reads (NaN, -2) if a bounded wait inside the coarse GEMM or the scan gave up, since
 *            a probe or a candidate may then be missing (not expected in normal operation; the
 *            call still returns 0 because the check runs on the device after the launch, and
 *            trident_workspace_status reads the reason);
 *   stats    optional int64[TRIDENT_STATS_LEN] accumulated counters (NULL to skip). */
int trident_search(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                   int32_t mode, int32_t ub_seed, void* workspace, size_t workspace_bytes,
                   float* out_d, int64_t* out_i, int64_t* stats, void* stream);

/* Phases timed by trident_search_profiled. */
enum trident_phase {
    TRIDENT_PHASE_COARSE = 0,   /* rotation + coarse GEMM + exact probe selection            */
    TRIDENT_PHASE_PAIRS = 1,    /* cluster-major pair lists and work items                   */
    TRIDENT_PHASE_SEED = 2,     /* Stage X: per-query thresholds from the nearest lists      */
    TRIDENT_PHASE_SCAN = 3,     /* Stage Y/Z (or CM-FP32) over every probed list             */
    TRIDENT_PHASE_MERGE = 4,    /* final top-K merge                                         */
    TRIDENT_PHASES = 5
};

/* trident_search plus CUDA-event timing of each phase (milliseconds, 0 for a phase that did not
 * run), like the reference's record_events (:1291-1296, :1595-1603). It synchronises `stream`
 * before returning. */
int trident_search_profiled(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                            int32_t mode, int32_t ub_seed, void* workspace, size_t workspace_bytes,
                            float* out_d, int64_t* out_i, int64_t* stats, void* stream,
                            float* phase_ms);

/* Number of kernels the library has launched from the calling thread so far. */
int64_t trident_launch_count(void);

/* Device-side status of the last search that used a workspace (no counterpart in the reference,
 * whose kernels had no bounded waits and reported nothing). Every wait inside the kernels is
 * bounded; a wait that gives up records why in a status word of the workspace, and the results it
 * may have spoiled read (NaN, -2) (probe lists: -1). */
enum trident_device_status {
    TRIDENT_STATUS_OK = 0,
    TRIDENT_STATUS_LOCK_TIMEOUT = 1,  /* the scan gave up on a per-query insertion lock         */
    TRIDENT_STATUS_MMA_TIMEOUT = 2    /* the coarse GEMM gave up waiting for its tensor-core MMAs */
};

/* Waits for `stream`, then reads the status word of `workspace` (the buffer last passed to
 * trident_search / trident_coarse / trident_search_prep / _seed / _finish) into *status: a bitwise
 * OR of TRIDENT_STATUS_* values. The word sits at the start of the workspace, so no sizes are
 * needed. In the staged multi-GPU search the status of a query's coarse stage travels with its
 * qinfo row, so finish's workspace reports a GEMM timeout on any rank. */
int trident_workspace_status(const void* workspace, void* stream, int32_t* status);

/* Limits of the bounded waits, process-wide: lock_spins tries of a per-query insertion lock (default
 * 2^22, each followed by a 64 ns sleep) and mma_polls polls of a tensor-core completion barrier
 * (default 2^22). A negative value restores the default. A limit of 0 makes every such wait give
 * up at once, which is how the tests exercise the error path without a GPU fault. */
int trident_set_wait_limits(int64_t lock_spins, int64_t mma_polls);

/* The coarse stage alone (query PCA rotation + exact top-nprobe list selection), replacing the
 * addmm_out + trident_topk_centroids_kernel pair (:1233-1259). probe_cids [B, nprobe] int32 comes
 * out ascending by (float64 ||q - c||^2, list id); probe_d64 [B, nprobe] (optional) holds those
 * float64 distances; qrot [B, D_pad] (optional) the float32-rounded rotated queries. */
int trident_coarse(const trident_index* idx, const float* xq, int32_t B, int32_t nprobe,
                   void* workspace, size_t workspace_bytes, int32_t* probe_cids, double* probe_d64,
                   float* qrot, int64_t* stats, void* stream);

/* Size of the fixed workspace behind trident_search_noalloc, per GPU. */
#define TRIDENT_NOALLOC_WORKSPACE_BYTES (32u * 1024u * 1024u)

/* trident_search for callers that cannot allocate device memory (no counterpart in the
 * reference, whose caller always allocated the scratch tensors). Same arguments and results as
 * trident_search without the workspace: the workspace is a TRIDENT_NOALLOC_WORKSPACE_BYTES array
 * compiled into the library, held by every GPU that loads it until the process exits. Returns
 * TRIDENT_ERR_WORKSPACE when trident_workspace_size(B, K, nprobe) exceeds that size. No call
 * allocates device memory. All calls on a device share the array: calls whose GPU work overlaps in
 * time race and must be serialised by the caller. The first call on each device looks up the
 * array's device address, and the first search from each host thread on each device creates the
 * library's side stream and its four events (as trident_search does); make that first call before
 * capturing a stream. */
int trident_search_noalloc(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                           int32_t mode, int32_t ub_seed, float* out_d, int64_t* out_i, int64_t* stats,
                           void* stream);

/* TRIDENT_NOALLOC_WORKSPACE_BYTES as compiled into the library (for bindings that cannot read the
 * header's macro). */
size_t trident_noalloc_workspace_bytes(void);

/* Index build: the nearest centroid of each row, out[i] = argmin_c (cnorm[c] - 2 x_i.c) (ties to the
 * smaller c), on the tensor cores (TF32 products, the TMA-fed GEMM of the coarse stage with an argmin
 * epilogue). Replaces the reference's faiss assignment (benchmarks/phase4a_suite.py:389-421, the
 * k-means training and list assignment of load_or_train_clustering). The list assignment is an input
 * of the index; searches are exact for whatever assignment they are given, so TF32 rounding near a
 * tie only moves a row between two equally near lists.
 *   x [n, D] and centroids [nlist, D] float32 row-major on the device, 16-byte aligned, D % 4 == 0;
 *   cnorm [nlist] = ||c||^2; out [n] int32; dev_status: one device int32 that receives
 *   TRIDENT_STATUS_MMA_TIMEOUT (or-ed in) if a bounded wait gave up (out is then incomplete). */
int trident_assign(const float* x, int64_t n, int32_t D, const float* centroids, const float* cnorm, int32_t nlist,
                   int32_t* out, int32_t* dev_status, void* stream);

/* Per-query side information of trident_search_prep: [B, TRIDENT_QINFO_LEN] float32 (||q||,
 * the bound's query slack sigma, ||q - mu||, padding). */
#define TRIDENT_QINFO_LEN 4

/* The search in three stages, for list sharding over GPUs (one process per GPU; no counterpart
 * in the reference, which ran on one GPU). Every rank's index holds all centroids and only the
 * rows of its own lists. A batch of B_all queries, B_r of them owned by rank r, is processed as
 * follows:
 *   1. trident_search_prep on the rank's own B_r queries writes their probe lists
 *      [B_r, nprobe], rotated queries [B_r, D_pad] and qinfo [B_r, TRIDENT_QINFO_LEN];
 *   2. the caller all-gathers those and the query vectors into [B_all, ...];
 *   3. trident_search_seed on the whole batch builds the work items for the local lists and
 *      writes each query's K smallest seed values of the local rows, with their row ids, into
 *      seed_d [B_all, K] and seed_i [B_all, K], ascending and padded with (+inf, -1). A GPU
 *      refines a share of the seed rows proportional to the seed lists it holds;
 *   4. the caller gathers the R seed lists, merges them with trident_merge_shards and takes
 *      column K-1 as tau [B_all]. That is the K-th smallest over the distinct rows of all
 *      ranks, so it bounds the final K-th distance;
 *   5. trident_search_finish scans the local lists with those thresholds and writes the
 *      per-query top-K of the local rows, [B_all, K];
 *   6. the caller gathers the R lists and merges them with trident_merge_shards.
 * Steps 3 and 5 must use the same workspace, sized for (B_all, K, nprobe), and the same
 * mode/ub_seed/K/nprobe. A single GPU runs the same stages inside trident_search. */
int trident_search_prep(const trident_index* idx, const float* xq, int32_t B, int32_t nprobe,
                        void* workspace, size_t workspace_bytes, int32_t* probe_out, float* qrot_out,
                        float* qinfo_out, void* stream);
int trident_search_seed(const trident_index* idx, const float* xq_all, int32_t B_all, int32_t K,
                        int32_t nprobe, int32_t mode, int32_t ub_seed, const int32_t* probe,
                        const float* qrot, const float* qinfo, void* workspace, size_t workspace_bytes,
                        float* seed_d, int64_t* seed_i, void* stream);
int trident_search_finish(const trident_index* idx, const float* xq_all, int32_t B_all, int32_t K,
                          int32_t nprobe, int32_t mode, int32_t ub_seed, const float* tau_in,
                          void* workspace, size_t workspace_bytes, float* out_d, int64_t* out_i,
                          int64_t* stats, void* stream);

/* Multi-GPU merge: R per-shard result lists d_in/i_in [R, B, K] (as gathered by an NCCL
 * all-gather) -> the global top-K per query under the (distance, id) order. A query for which any
 * shard reports an id of -2 (a bounded wait gave up there) comes out as (NaN, -2) in every slot. */
int trident_merge_shards(const float* d_in, const int64_t* i_in, int32_t R, int32_t B, int32_t K,
                         float* out_d, int64_t* out_i, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIDENT_B200_H */
