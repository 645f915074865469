// C ABI of trident_b200: argument checks, workspace carve-up and the launch sequence of one search.
//
// Launch sequence of trident_search (all on the caller's stream, asynchronous), replacing
// launch_trident_v4_search (src/trident_v4_kernels.cu:1172-1604):
//   rotate_f64 -> coarse_gemm -> probe_select                   (coarse stage, exact probe set)
//   pair_hist -> pair_scan -> pair_scatter -> item_emit          (cluster-major work items)
//   [pass 0: scan over the p_init nearest lists -> merge -> tau]  (Stage X warm-up)
//   pass 1: scan over the remaining lists -> merge -> out        (Stage Y/Z or CM-FP32)
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <string>

#include "tb_internal.h"
#include "trident_b200.h"

namespace {

thread_local std::string g_err;
thread_local int64_t g_launches = 0;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(TRIDENT_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
}

constexpr int kMaxD = 4096;
constexpr int kMaxK = 100;
constexpr int kMaxNprobe = 1024;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Limits of the bounded waits (trident_set_wait_limits); kernels receive them as arguments.
constexpr uint32_t kDefaultWaitLimit = 1u << 22;
std::atomic<uint32_t> g_lock_spins{kDefaultWaitLimit};
std::atomic<uint32_t> g_mma_polls{kDefaultWaitLimit};

}  // namespace

namespace tb {

static_assert(QI_LEN == TRIDENT_QINFO_LEN, "qinfo layout");

int record_error(int code, const char* msg) { return fail(code, "%s", msg); }

uint32_t lock_spin_limit() { return g_lock_spins.load(std::memory_order_relaxed); }
uint32_t mma_wait_limit() { return g_mma_polls.load(std::memory_order_relaxed); }

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 1;
    }
    return cached[dev];
}

size_t carve_workspace(const trident_index& idx, int B, int K, int nprobe, void* base, Workspace* ws) {
    size_t off = 0;
    char* p = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        void* r = p ? (void*)(p + off) : nullptr;
        off += align256(bytes);
        return r;
    };
    const size_t Bs = (size_t)(B > 0 ? B : 1);
    const size_t pairs = Bs * (size_t)nprobe;
    Workspace w;
    w.ctr = (int32_t*)take(16 * sizeof(int32_t));  // first: the status word's offset is fixed
    w.qrot = (float*)take(Bs * idx.D_pad * sizeof(float));
    w.qinfo = (float*)take(Bs * QI_LEN * sizeof(float));
    w.coarse = (float*)take(Bs * (size_t)idx.nlist * sizeof(float));
    w.tilemin = (float*)take(Bs * (size_t)((idx.nlist + kCoarseMinSpan - 1) / kCoarseMinSpan) * sizeof(float));
    w.gsplit = (float*)take(coarse_split_bytes(idx, (int)Bs));
    w.probe = (int32_t*)take(pairs * sizeof(int32_t));
    w.cnt = (int32_t*)take(2 * (size_t)idx.nlist * sizeof(int32_t));
    w.off = (int32_t*)take(2 * (size_t)(idx.nlist + 1) * sizeof(int32_t));
    w.cursor = (int32_t*)take(2 * (size_t)idx.nlist * sizeof(int32_t));
    w.item_off = (int32_t*)take(2 * (size_t)(idx.nlist + 1) * sizeof(int32_t));
    w.pair_q = (int32_t*)take(pairs * sizeof(int32_t));
    w.pair_p = (int32_t*)take(pairs * sizeof(int32_t));
    w.items = (int4*)take(pairs * sizeof(int4));
    w.items_lpt = (int4*)take(pairs * sizeof(int4));
    w.lpt = (int32_t*)take(kLptBins * sizeof(int32_t));
    w.tau = (uint32_t*)take(Bs * sizeof(uint32_t));
    w.cand_d = (float*)take(pairs * (size_t)K * sizeof(float));
    w.cand_i = (int32_t*)take(pairs * (size_t)K * sizeof(int32_t));
    w.bytes = off;
    if (ws) *ws = w;
    return off;
}

}  // namespace tb

using namespace tb;

extern "C" {

int trident_version(void) { return TRIDENT_ABI_VERSION; }

const char* trident_last_error(void) { return g_err.c_str(); }

int trident_index_check(const trident_index* idx) {
    if (!idx) return fail(TRIDENT_ERR_INVALID, "index descriptor is NULL");
    if (idx->D < 1 || idx->D > kMaxD) return fail(TRIDENT_ERR_UNSUPPORTED, "D=%d outside [1, %d]", idx->D, kMaxD);
    if (idx->D_pad != ((idx->D + 31) / 32) * 32)
        return fail(TRIDENT_ERR_INVALID, "D_pad=%d must be ceil(D/32)*32=%d", idx->D_pad, ((idx->D + 31) / 32) * 32);
    if (idx->num_blocks != idx->D_pad / 32)
        return fail(TRIDENT_ERR_INVALID, "num_blocks=%d must be D_pad/32=%d", idx->num_blocks, idx->D_pad / 32);
    if (idx->nlist < 1) return fail(TRIDENT_ERR_INVALID, "nlist=%d", idx->nlist);
    if (idx->tile_size != 128 && idx->tile_size != 256)
        return fail(TRIDENT_ERR_UNSUPPORTED, "tile_size=%d (supported: 128, 256)", idx->tile_size);
    if (idx->N < 0) return fail(TRIDENT_ERR_INVALID, "N=%lld", (long long)idx->N);
    if (idx->N >= (int64_t)1 << 31) return fail(TRIDENT_ERR_UNSUPPORTED, "N=%lld exceeds int32 row ids", (long long)idx->N);
    const void* ptrs[] = {idx->xb_sorted, idx->orig_ids_sorted, idx->list_row_off, idx->list_tile_off, idx->codes,
                          idx->vmin, idx->delta, idx->eps, idx->centroids, idx->centroid_norm_sq,
                          idx->pca_mean, idx->pca_rot};
    const char* names[] = {"xb_sorted", "orig_ids_sorted", "list_row_off", "list_tile_off", "codes", "vmin",
                           "delta", "eps", "centroids", "centroid_norm_sq", "pca_mean", "pca_rot"};
    for (int i = 0; i < 12; ++i)
        if (!ptrs[i]) return fail(TRIDENT_ERR_INVALID, "index array %s is NULL", names[i]);
    if (((uintptr_t)idx->codes & 15) != 0) return fail(TRIDENT_ERR_INVALID, "codes must be 16-byte aligned");
    if (!(idx->lb_rel_slack > 0.0f) || !(idx->centroid_norm_max >= 0.0f))
        return fail(TRIDENT_ERR_INVALID, "lb_rel_slack / centroid_norm_max not set");
    return TRIDENT_OK;
}

int trident_workspace_size(const trident_index* idx, int32_t B, int32_t K, int32_t nprobe, size_t* bytes) {
    int rc = trident_index_check(idx);
    if (rc) return rc;
    if (!bytes) return fail(TRIDENT_ERR_INVALID, "bytes is NULL");
    if (B < 0 || K < 1 || nprobe < 1) return fail(TRIDENT_ERR_INVALID, "B=%d K=%d nprobe=%d", B, K, nprobe);
    *bytes = carve_workspace(*idx, B, K, nprobe, nullptr, nullptr);
    return TRIDENT_OK;
}

int32_t trident_p_init(int32_t mode, int32_t B, int32_t K, int32_t nprobe) {
    if (mode != TRIDENT_MODE_CASCADE) return 0;
    if (nprobe <= 1) return 0;
    if (B == 1 && K <= 10) return 1;
    if (nprobe <= 16) return 2;
    return 3;
}

int32_t trident_route(const trident_index* idx, int32_t B, int32_t nprobe, double w0) {
    if (!idx || idx->nlist < 1) return TRIDENT_MODE_CASCADE;
    if (!(w0 > 0.0)) w0 = TRIDENT_ROUTE_W0_B200;
    const double W = (double)B * (double)nprobe * ((double)idx->N / (double)idx->nlist) * (double)idx->D;
    return W < w0 ? TRIDENT_MODE_CM_FP32 : TRIDENT_MODE_CASCADE;
}

int32_t trident_stage_y_tensor(const trident_index* idx, int32_t B, int32_t K, int32_t nprobe, int32_t ub_seed) {
    if (!idx || B < 0 || nprobe < 1) return 0;
    return filter_eligible(*idx, K, true, ub_seed == 2, (int64_t)B * nprobe) ? 1 : 0;
}

static int check_search_args(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                             void* workspace, size_t workspace_bytes, Workspace* ws) {
    int rc = trident_index_check(idx);
    if (rc) return rc;
    if (B < 0) return fail(TRIDENT_ERR_INVALID, "B=%d", B);
    if (K < 1 || K > kMaxK) return fail(TRIDENT_ERR_UNSUPPORTED, "K=%d outside [1, %d]", K, kMaxK);
    if (nprobe < 1 || nprobe > idx->nlist || nprobe > kMaxNprobe)
        return fail(TRIDENT_ERR_INVALID, "nprobe=%d outside [1, min(nlist=%d, %d)]", nprobe, idx->nlist, kMaxNprobe);
    if (B > 0 && !xq) return fail(TRIDENT_ERR_INVALID, "xq is NULL");
    if ((size_t)B * (size_t)nprobe >= ((size_t)1 << 31)) return fail(TRIDENT_ERR_UNSUPPORTED, "B*nprobe too large");
    const size_t need = carve_workspace(*idx, B, K, nprobe, workspace, ws);
    if (!workspace || workspace_bytes < need)
        return fail(TRIDENT_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed", workspace_bytes, need);
    if (((uintptr_t)workspace & 255) != 0) return fail(TRIDENT_ERR_INVALID, "workspace must be 256-byte aligned");
    return TRIDENT_OK;
}

#define TB_TRY(expr, where)                        \
    do {                                           \
        cudaError_t _e = (expr);                   \
        if (_e != cudaSuccess) return cuda_fail(_e, where); \
    } while (0)

int trident_coarse(const trident_index* idx, const float* xq, int32_t B, int32_t nprobe, void* workspace,
                   size_t workspace_bytes, int32_t* probe_cids, double* probe_d64, float* qrot, int64_t* stats,
                   void* stream) {
    Workspace ws;
    int rc = check_search_args(idx, xq, B, 1, nprobe, workspace, workspace_bytes, &ws);
    if (rc) return rc;
    if (!probe_cids) return fail(TRIDENT_ERR_INVALID, "probe_cids is NULL");
    if (B == 0) return TRIDENT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    TB_TRY(cudaMemsetAsync(ws.ctr, 0, 16 * sizeof(int32_t), st), "memset counters");
    TB_TRY(launch_rotate(*idx, xq, B, ws.qrot, ws.qinfo, ws.tau, st), "rotate");
    TB_TRY(launch_coarse_gemm(*idx, xq, B, ws.coarse, ws.tilemin, ws.gsplit, ws.ctr + kStatusWord, st), "coarse_gemm");
    TB_TRY(launch_probe_select(*idx, xq, B, nprobe, ws.coarse, ws.tilemin, ws.qinfo, probe_cids, probe_d64,
                               (unsigned long long*)stats, ws.ctr + kStatusWord, st),
           "probe_select");
    g_launches += 4;
    if (qrot)
        TB_TRY(cudaMemcpyAsync(qrot, ws.qrot, (size_t)B * idx->D_pad * sizeof(float), cudaMemcpyDeviceToDevice, st),
               "qrot copy");
    return TRIDENT_OK;
}

// CUDA events around the phases of one search (profiled calls only).
struct PhaseEvents {
    cudaEvent_t ev[TRIDENT_PHASES + 1];
    bool ran[TRIDENT_PHASES];
    bool on = false;
};

// Records the CUDA event at the start of a phase (or the end, TRIDENT_PHASES) of a profiled call.
struct Marker {
    PhaseEvents* pe;
    cudaStream_t st;
    cudaError_t operator()(int phase) const {
        if (!pe) return cudaSuccess;
        if (phase < TRIDENT_PHASES) pe->ran[phase] = true;
        return cudaEventRecord(pe->ev[phase], st);
    }
};

// A second stream (and its fork/join events) per calling thread and device. The float64 rotation
// runs there: the coarse GEMM, the probe selection and the pair lists need only the queries and
// their norms, so the rotation overlaps all of them and is joined before the seed kernel.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;    // around the rotation
    cudaEvent_t fork2 = nullptr, join2 = nullptr;  // around the pair lists and work items
};

static cudaError_t side_stream(SideStream** out) {
    static thread_local SideStream per_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) dev = 0;
    SideStream& ss = per_dev[dev];
    if (!ss.s) {
        if ((e = cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ss.fork2, cudaEventDisableTiming)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ss.join2, cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    *out = &ss;
    return cudaSuccess;
}

// Stage 1 of a search: rotation, coarse GEMM and exact probe selection for B queries, into ws.
static int stage_coarse(const trident_index* idx, const float* xq, int32_t B, int32_t nprobe, const Workspace& ws,
                        unsigned long long* sp, cudaStream_t st) {
    SideStream* ss = nullptr;
    TB_TRY(side_stream(&ss), "side stream");
    TB_TRY(launch_query_norms(*idx, xq, B, ws.qinfo, ws.tau, st), "query norms");
    TB_TRY(cudaEventRecord(ss->fork, st), "fork");
    TB_TRY(cudaStreamWaitEvent(ss->s, ss->fork, 0), "fork");
    TB_TRY(launch_rotate_f64(*idx, xq, B, ws.qrot, ss->s), "rotate");
    TB_TRY(cudaEventRecord(ss->join, ss->s), "join");
    TB_TRY(launch_coarse_gemm(*idx, xq, B, ws.coarse, ws.tilemin, ws.gsplit, ws.ctr + kStatusWord, st), "coarse_gemm");
    TB_TRY(launch_probe_select(*idx, xq, B, nprobe, ws.coarse, ws.tilemin, ws.qinfo, ws.probe, nullptr, sp, ws.ctr + kStatusWord,
                               st),
           "probe_select");
    g_launches += 4;
    return TRIDENT_OK;
}

// The caller's stream waits for the rotation that stage_coarse started on the side stream.
static int join_rotation(cudaStream_t st) {
    SideStream* ss = nullptr;
    TB_TRY(side_stream(&ss), "side stream");
    TB_TRY(cudaStreamWaitEvent(st, ss->join, 0), "join");
    return TRIDENT_OK;
}

// Stage 2: cluster-major work items over every probe with rows, then (cascade) the Stage X seed.
// One pass covers every probe: the reference scans its p_init warm-up lists first to obtain the
// thresholds, here the query-major seed kernel takes that role before the scan starts.
static int stage_seed(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe, bool lb,
                      int32_t ub_seed, const Workspace& ws, cudaStream_t st, const Marker& mark,
                      float* seed_d = nullptr, int64_t* seed_i = nullptr) {
    // The pair lists and work items (side stream) and the seed (caller's stream) both need only the
    // probe lists, so they run side by side; the caller's stream then waits for the items.
    int rc_join = 0;
    SideStream* ss = nullptr;
    TB_TRY(side_stream(&ss), "side stream");
    const int G = filter_eligible(*idx, K, lb, ub_seed == 2, (int64_t)B * nprobe) ? filter_group_size(*idx, K) : scan_group_size(*idx, K);
    TB_TRY(mark(TRIDENT_PHASE_PAIRS), "event");
    TB_TRY(cudaEventRecord(ss->fork2, st), "fork");
    TB_TRY(cudaStreamWaitEvent(ss->s, ss->fork2, 0), "fork");
    TB_TRY(launch_pairs(*idx, ws.probe, B, nprobe, 0, G, K, ws, ss->s), "pairs");
    TB_TRY(launch_item_order(*idx, B * nprobe, ws, ss->s), "item order");
    TB_TRY(cudaEventRecord(ss->join2, ss->s), "join");
    g_launches += 7;
    if ((rc_join = join_rotation(st))) return rc_join;  // qrot is read from here on
    if (lb) {
        TB_TRY(mark(TRIDENT_PHASE_SEED), "event");
        TB_TRY(launch_seed(*idx, xq, ws, B, K, nprobe, seed_lists_for(B, K, nprobe), ub_seed >= 1, seed_d, seed_i,
                           seed_d != nullptr, st),
               "seed");
        g_launches += 1;
    }
    TB_TRY(cudaStreamWaitEvent(st, ss->join2, 0), "join");
    return TRIDENT_OK;
}

// Stage 3: Stage Y/Z (or CM-FP32) over the items, then the per-query merge into the output.
static int stage_scan(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe, bool lb,
                      int32_t ub_seed, const Workspace& ws, float* out_d, int64_t* out_i, unsigned long long* sp,
                      cudaStream_t st, const Marker& mark) {
    ScanLaunch sl;
    sl.K = K;
    sl.nprobe = nprobe;
    sl.filter = filter_eligible(*idx, K, lb, ub_seed == 2, (int64_t)B * nprobe) ? 1 : 0;
    sl.G = sl.filter ? filter_group_size(*idx, K) : scan_group_size(*idx, K);
    sl.lb = lb ? 1 : 0;
    sl.pass = 1;
    sl.ub_seed = (lb && ub_seed == 2) ? 1 : 0;
    sl.max_items = B * nprobe;
    sl.item_base = 0;
    TB_TRY(mark(TRIDENT_PHASE_SCAN), "event");
    if (sl.filter) {
        TB_TRY(launch_filter(*idx, xq, ws, sl, sp, st), "tensor-core stage Y");
    } else {
        TB_TRY(launch_scan(*idx, xq, ws, sl, sp, st), "scan");
    }
    TB_TRY(mark(TRIDENT_PHASE_MERGE), "event");
    TB_TRY(launch_merge(ws, B, K, nprobe, 0, nprobe, nullptr, out_d, out_i, st), "merge");
    g_launches += 2;
    return TRIDENT_OK;
}

static int resolve_mode(const trident_index* idx, int32_t B, int32_t nprobe, int32_t* mode, int32_t ub_seed) {
    if (ub_seed < 0 || ub_seed > 2) return fail(TRIDENT_ERR_INVALID, "ub_seed=%d outside [0, 2]", ub_seed);
    if (*mode == TRIDENT_MODE_AUTO) *mode = trident_route(idx, B, nprobe, 0.0);
    if (*mode != TRIDENT_MODE_CASCADE && *mode != TRIDENT_MODE_CM_FP32)
        return fail(TRIDENT_ERR_UNSUPPORTED, "mode=%d (supported: -1 auto, 2 cascade, 10 CM-FP32)", *mode);
    return TRIDENT_OK;
}

static int search_impl(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe, int32_t mode,
                       int32_t ub_seed, void* workspace, size_t workspace_bytes, float* out_d, int64_t* out_i,
                       int64_t* stats, cudaStream_t st, PhaseEvents* pe) {
    Workspace ws;
    int rc = check_search_args(idx, xq, B, K, nprobe, workspace, workspace_bytes, &ws);
    if (rc) return rc;
    if (B > 0 && (!out_d || !out_i)) return fail(TRIDENT_ERR_INVALID, "out_d / out_i is NULL");
    if ((rc = resolve_mode(idx, B, nprobe, &mode, ub_seed))) return rc;
    if (B == 0) return TRIDENT_OK;
    unsigned long long* sp = (unsigned long long*)stats;
    const bool lb = mode == TRIDENT_MODE_CASCADE;
    const Marker mark{pe, st};
    TB_TRY(mark(TRIDENT_PHASE_COARSE), "event");
    TB_TRY(cudaMemsetAsync(ws.ctr, 0, 16 * sizeof(int32_t), st), "memset counters");
    if ((rc = stage_coarse(idx, xq, B, nprobe, ws, sp, st))) return rc;
    if ((rc = stage_seed(idx, xq, B, K, nprobe, lb, ub_seed, ws, st, mark))) return rc;  // joins the rotation
    if ((rc = stage_scan(idx, xq, B, K, nprobe, lb, ub_seed, ws, out_d, out_i, sp, st, mark))) return rc;
    TB_TRY(mark(TRIDENT_PHASES), "event");
    return TRIDENT_OK;
}

int trident_search(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe, int32_t mode,
                   int32_t ub_seed, void* workspace, size_t workspace_bytes, float* out_d, int64_t* out_i,
                   int64_t* stats, void* stream) {
    return search_impl(idx, xq, B, K, nprobe, mode, ub_seed, workspace, workspace_bytes, out_d, out_i, stats,
                       (cudaStream_t)stream, nullptr);
}

int trident_search_profiled(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                            int32_t mode, int32_t ub_seed, void* workspace, size_t workspace_bytes, float* out_d,
                            int64_t* out_i, int64_t* stats, void* stream, float* phase_ms) {
    if (!phase_ms) return fail(TRIDENT_ERR_INVALID, "phase_ms is NULL");
    cudaStream_t st = (cudaStream_t)stream;
    PhaseEvents pe;
    int created = 0;
    for (; created <= TRIDENT_PHASES; ++created) {
        if (cudaEventCreate(&pe.ev[created]) != cudaSuccess) break;
    }
    for (int i = 0; i < TRIDENT_PHASES; ++i) { pe.ran[i] = false; phase_ms[i] = 0.0f; }
    int rc = TRIDENT_OK;
    if (created <= TRIDENT_PHASES) {
        rc = cuda_fail(cudaGetLastError(), "cudaEventCreate");
    } else {
        rc = search_impl(idx, xq, B, K, nprobe, mode, ub_seed, workspace, workspace_bytes, out_d, out_i, stats, st,
                         &pe);
        if (rc == TRIDENT_OK && B > 0) {
            cudaError_t e = cudaEventSynchronize(pe.ev[TRIDENT_PHASES]);
            if (e != cudaSuccess) rc = cuda_fail(e, "cudaEventSynchronize");
            for (int i = 0; rc == TRIDENT_OK && i < TRIDENT_PHASES; ++i) {
                if (!pe.ran[i]) continue;
                int nxt = i + 1;
                while (nxt < TRIDENT_PHASES && !pe.ran[nxt]) ++nxt;
                float ms = 0.0f;
                e = cudaEventElapsedTime(&ms, pe.ev[i], pe.ev[nxt]);
                if (e != cudaSuccess) rc = cuda_fail(e, "cudaEventElapsedTime");
                phase_ms[i] = ms;
            }
        }
    }
    for (int i = 0; i < created; ++i) cudaEventDestroy(pe.ev[i]);
    return rc;
}

int64_t trident_launch_count(void) { return g_launches; }

int trident_workspace_status(const void* workspace, void* stream, int32_t* status) {
    if (!workspace || !status) return fail(TRIDENT_ERR_INVALID, "workspace / status is NULL");
    if (((uintptr_t)workspace & 255) != 0) return fail(TRIDENT_ERR_INVALID, "workspace must be 256-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    int32_t word = 0;
    // the counter block is the workspace's first region (carve_workspace)
    const int32_t* src = static_cast<const int32_t*>(workspace) + kStatusWord;
    TB_TRY(cudaMemcpyAsync(&word, src, sizeof(int32_t), cudaMemcpyDeviceToHost, st), "status copy");
    TB_TRY(cudaStreamSynchronize(st), "status sync");
    *status = word;
    return TRIDENT_OK;
}

int trident_set_wait_limits(int64_t lock_spins, int64_t mma_polls) {
    constexpr int64_t kMax = 0x7fffffff;
    g_lock_spins.store(lock_spins < 0 ? kDefaultWaitLimit : (uint32_t)(lock_spins > kMax ? kMax : lock_spins));
    g_mma_polls.store(mma_polls < 0 ? kDefaultWaitLimit : (uint32_t)(mma_polls > kMax ? kMax : mma_polls));
    return TRIDENT_OK;
}

int trident_search_prep(const trident_index* idx, const float* xq, int32_t B, int32_t nprobe, void* workspace,
                        size_t workspace_bytes, int32_t* probe_out, float* qrot_out, float* qinfo_out, void* stream) {
    Workspace ws;
    int rc = check_search_args(idx, xq, B, 1, nprobe, workspace, workspace_bytes, &ws);
    if (rc) return rc;
    if (B > 0 && (!probe_out || !qrot_out || !qinfo_out)) return fail(TRIDENT_ERR_INVALID, "an output is NULL");
    if (B == 0) return TRIDENT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    TB_TRY(cudaMemsetAsync(ws.ctr, 0, 16 * sizeof(int32_t), st), "memset counters");
    if ((rc = stage_coarse(idx, xq, B, nprobe, ws, nullptr, st))) return rc;
    if ((rc = join_rotation(st))) return rc;
    TB_TRY(cudaMemcpyAsync(probe_out, ws.probe, (size_t)B * nprobe * sizeof(int32_t), cudaMemcpyDeviceToDevice, st),
           "probe copy");
    TB_TRY(cudaMemcpyAsync(qrot_out, ws.qrot, (size_t)B * idx->D_pad * sizeof(float), cudaMemcpyDeviceToDevice, st),
           "qrot copy");
    TB_TRY(cudaMemcpyAsync(qinfo_out, ws.qinfo, (size_t)B * TRIDENT_QINFO_LEN * sizeof(float),
                           cudaMemcpyDeviceToDevice, st),
           "qinfo copy");
    return TRIDENT_OK;
}

int trident_search_seed(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe, int32_t mode,
                        int32_t ub_seed, const int32_t* probe, const float* qrot, const float* qinfo, void* workspace,
                        size_t workspace_bytes, float* seed_d, int64_t* seed_i, void* stream) {
    Workspace ws;
    int rc = check_search_args(idx, xq, B, K, nprobe, workspace, workspace_bytes, &ws);
    if (rc) return rc;
    if ((rc = resolve_mode(idx, B, nprobe, &mode, ub_seed))) return rc;
    if (B > 0 && (!probe || !qrot || !qinfo || !seed_d || !seed_i))
        return fail(TRIDENT_ERR_INVALID, "an input or seed output is NULL");
    if (B == 0) return TRIDENT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    TB_TRY(cudaMemsetAsync(ws.ctr, 0, 16 * sizeof(int32_t), st), "memset counters");
    TB_TRY(cudaMemcpyAsync(ws.probe, probe, (size_t)B * nprobe * sizeof(int32_t), cudaMemcpyDeviceToDevice, st),
           "probe copy");
    TB_TRY(cudaMemcpyAsync(ws.qrot, qrot, (size_t)B * idx->D_pad * sizeof(float), cudaMemcpyDeviceToDevice, st),
           "qrot copy");
    TB_TRY(cudaMemcpyAsync(ws.qinfo, qinfo, (size_t)B * TRIDENT_QINFO_LEN * sizeof(float), cudaMemcpyDeviceToDevice,
                           st),
           "qinfo copy");
    // tau = +inf; a coarse-stage timeout on any rank reaches this workspace's status word through qinfo
    TB_TRY(launch_tau_init_import_status(ws.tau, ws.qinfo, B, ws.ctr + kStatusWord, st), "tau init");
    g_launches += 1;
    const Marker nomark{nullptr, st};
    if (mode != TRIDENT_MODE_CASCADE) {  // CM-FP32 has no seed: empty lists
        TB_TRY(launch_fill_inf(reinterpret_cast<uint32_t*>(seed_d), B * K, st), "seed fill");
        TB_TRY(cudaMemsetAsync(seed_i, 0xFF, (size_t)B * K * sizeof(int64_t), st), "seed fill");
    }
    return stage_seed(idx, xq, B, K, nprobe, mode == TRIDENT_MODE_CASCADE, ub_seed, ws, st, nomark, seed_d, seed_i);
}

int trident_search_finish(const trident_index* idx, const float* xq, int32_t B, int32_t K, int32_t nprobe,
                          int32_t mode, int32_t ub_seed, const float* tau_in, void* workspace, size_t workspace_bytes,
                          float* out_d, int64_t* out_i, int64_t* stats, void* stream) {
    Workspace ws;
    int rc = check_search_args(idx, xq, B, K, nprobe, workspace, workspace_bytes, &ws);
    if (rc) return rc;
    if ((rc = resolve_mode(idx, B, nprobe, &mode, ub_seed))) return rc;
    if (B > 0 && (!out_d || !out_i)) return fail(TRIDENT_ERR_INVALID, "out_d / out_i is NULL");
    if (B == 0) return TRIDENT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (tau_in)
        TB_TRY(cudaMemcpyAsync(ws.tau, tau_in, (size_t)B * sizeof(float), cudaMemcpyDeviceToDevice, st), "tau copy");
    const Marker nomark{nullptr, st};
    return stage_scan(idx, xq, B, K, nprobe, mode == TRIDENT_MODE_CASCADE, ub_seed, ws, out_d, out_i,
                      (unsigned long long*)stats, st, nomark);
}

int trident_assign(const float* x, int64_t n, int32_t D, const float* centroids, const float* cnorm, int32_t nlist,
                   int32_t* out, int32_t* dev_status, void* stream) {
    if (n < 0 || n >= ((int64_t)1 << 31)) return fail(TRIDENT_ERR_UNSUPPORTED, "n=%lld outside [0, 2^31)", (long long)n);
    if (D < 4 || D > kMaxD || (D % 4) != 0) return fail(TRIDENT_ERR_UNSUPPORTED, "D=%d must be a multiple of 4 in [4, %d]", D, kMaxD);
    if (nlist < 1) return fail(TRIDENT_ERR_INVALID, "nlist=%d", nlist);
    if (n == 0) return TRIDENT_OK;
    if (!x || !centroids || !cnorm || !out || !dev_status) return fail(TRIDENT_ERR_INVALID, "NULL buffer");
    if ((((uintptr_t)x) | ((uintptr_t)centroids)) & 15) return fail(TRIDENT_ERR_INVALID, "x / centroids must be 16-byte aligned");
    cudaError_t e = launch_assign(x, n, D, centroids, cnorm, nlist, out, dev_status, (cudaStream_t)stream);
    if (e == cudaErrorNotSupported) return fail(TRIDENT_ERR_UNSUPPORTED, "tensor maps unavailable for this layout");
    TB_TRY(e, "assign");
    g_launches += 1;
    return TRIDENT_OK;
}

int trident_merge_shards(const float* d_in, const int64_t* i_in, int32_t R, int32_t B, int32_t K, float* out_d,
                         int64_t* out_i, void* stream) {
    if (R < 1 || B < 0 || K < 1 || K > kMaxK) return fail(TRIDENT_ERR_INVALID, "R=%d B=%d K=%d", R, B, K);
    if (B == 0) return TRIDENT_OK;
    if (!d_in || !i_in || !out_d || !out_i) return fail(TRIDENT_ERR_INVALID, "NULL buffer");
    TB_TRY(launch_merge_shards(d_in, i_in, R, B, K, out_d, out_i, (cudaStream_t)stream), "merge_shards");
    return TRIDENT_OK;
}

}  // extern "C"
