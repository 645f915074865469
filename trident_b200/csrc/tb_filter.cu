// Stage Y on the tensor cores: the cascade's lower-bound filter as an 8-bit GEMM per work item.
//
// The reference bounds every (query, row) pair dimension by dimension on the CUDA cores, a 32-dim
// block at a time with early exit (src/trident_v4_kernels.cu:725-780). Here the whole bound of a
// row comes from one tcgen05 integer MMA per 32-dim code block. For list c and query j (all in the
// PCA-rotated space, x^ = vmin + code * delta the dequantised row, q~ the rotated query):
//   b_d = vmin_d - q~_d,  w_d = delta_d b_d,
//   ||x^ - q~||^2 = P_r + 2 sum_d code_d w_d + sum_d b_d^2,  P_r = sum_d (code_d delta_d)^2 (per row,
//   stored at build time rounded down).
// Per item and query, w is split into two signed bytes, w_d = s_j (hi_d + lo_d / 254) + res_d with
// |res_d| <= R_j, so 2 sum_d code_d w_d = (2 s_j / 254) (254 Hi + Lo) + 2 sum_d code_d res_d, where
// Hi = sum code_d hi_d and Lo = sum code_d lo_d are integer dot products of the u8 codes with s8
// weights that tcgen05.mma.kind::i8 accumulates exactly in int32 (A = 128 rows of codes, B = the
// item's queries as N = 2n columns hi, lo). The epilogue evaluates per (row, query)
//   v = (P_r + Bsq_j) + (2 s_j / 254) (254 Hi + Lo)      (D_pad <= 256, so 254 Hi + Lo fits int32;
//                                                         above, 2 s_j Hi + (2 s_j / 254) Lo)
// in float32; v - slack_j is a lower bound of ||x^ - q~||^2, where slack_j covers the quantisation
// residual (2 R_j 255 D_pad) and every float32 rounding (8 u times a bound of each term's size).
// With E_c = ||eps_c||_2 >= ||x~ - x^|| (eps bounds each dim), the triangle inequality gives
// ||x~ - q~|| >= sqrt(v - slack_j) - E_c, so the row is dropped when
//   v > Phi_j = (sqrt(ts_j) + E_c)^2 + slack_j,
// with ts_j the same prune threshold (prune_threshold: tau, the query's sigma, rho) as the
// CUDA-core Stage Y. Survivors are refined at once (exact FP32, the reference's summation order)
// and inserted into the item's per-query top-K under a bounded per-query lock, all of a query's
// survivors among a warp's 32 rows with one lock and one list insertion; a list that fills
// lowers the query's threshold for this CTA (Phi_j) and, through the per-query atomicMin, for the
// whole GPU. At the item's end its lists go to the (query, probe) candidate slots the merge reads,
// exactly like scan_kernel's.
//
// One CTA per SM, persistent over the items (longest first, round robin):
//   warp 0      TMA producer: per 128-row sub-tile of the list and per 32-dim block, one 2-D copy of
//               128 rows x 32 bytes of codes, 32-byte swizzled (the blocked code layout holds a
//               block of a tile's rows contiguously, so no repacking is needed);
//   warp 1      MMA issuer: per sub-tile nb MMAs (K = 32 each) into one of four accumulators;
//   warps 2-13  epilogue: build the next item's B operand (the s8 weights, written in the same
//               swizzled layout) while the MMAs of the current item run, then read each sub-tile's
//               accumulator (3 warps per tensor-memory lane quarter, split over the queries), test
//               the bound and refine the survivors.
// Every wait is bounded. A wait that gives up sets the status word (TRIDENT_STATUS_MMA_TIMEOUT;
// the merge then marks every result), the producer drains its copies, the MMA warp its last
// commit, and the epilogue warps keep meeting their named barriers without further work, so the
// CTA always reaches its end and frees the tensor memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"
#include "tb_tc.cuh"

namespace tb {

bool make_codes_map(CUtensorMap* m, const uint8_t* codes, int64_t rows);  // tb_gemm.cu

namespace {

constexpr int kFM = 128;                       // rows per sub-tile (UMMA M)
constexpr int kFStages = 8;                    // code-block stages
constexpr int kFStageBytes = kFM * 32;         // one 32-dim block of 128 rows
constexpr int kFEpiWarps = 12;                 // three per tensor-memory lane quarter
constexpr int kFParts = kFEpiWarps / 4;        // epilogue warps sharing a lane quarter (split the queries)
constexpr int kFThreads = 64 + 32 * kFEpiWarps;
constexpr int kFMaxG = 64;                     // queries per item
constexpr int kFMaxN = 2 * kFMaxG;             // accumulator columns per sub-tile
constexpr int kFQW = ((kFMaxG + kFParts - 1) / kFParts + 7) / 8 * 8;  // queries per epilogue warp, at most
constexpr int kFAcc = 4;                       // accumulators in tensor memory (the MMAs run up to 3 ahead)
constexpr uint32_t kFTmemCols = kFAcc * kFMaxN; // all 512 columns: one CTA per SM
constexpr int kFSmemLimit = 227 * 1024;
constexpr int kFStatic = 8 * 1024;             // static shared memory and reserve
constexpr double kU = 5.9604644775390625e-08;  // float32 unit roundoff 2^-24
constexpr int kFNarrowDPad = 256;              // up to here 254 Hi + Lo stays within int32
constexpr int kFMaxDPad = 1024;                // beyond 256, Hi and Lo are converted separately
constexpr int64_t kFMinPairs = 32768;          // (query, list) pairs of a search that picks this path

struct FilterArgs {
    const float* xb;
    const int32_t* oid;
    const int64_t* row_off;
    const int64_t* tile_off;
    const float* rowp;
    const float* vmin;
    const float* delta;
    const float* eps;
    const float* xq;
    const float* qrot;
    const float* qinfo;
    const int4* items;
    const int32_t* n_items;
    const int32_t* pair_q;
    const int32_t* pair_p;
    uint32_t* tau;
    float* cand_d;
    int32_t* cand_i;
    unsigned long long* stats;
    int32_t* err;
    uint32_t lock_spins;
    uint32_t polls;
    int D, D_pad, nb, T, K, nprobe, G;
    int b_stride;  // bytes per code block of the B operand (round16(2 G) * 32)
    float rho;
};

__host__ __device__ constexpr int round16(int x) { return (x + 15) & ~15; }

// K-major descriptor of a 32-byte-swizzled operand (rows of 32 bytes, 16-byte half h of row r at
// h ^ ((r / 4) % 2)): stride byte offset 256 between 8-row groups, version 1, layout type 6 =
// SWIZZLE_32B. The operand starts 256-byte aligned.
__device__ __forceinline__ uint64_t desc_sw32(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46) |
           (6ull << 61);
}

// D = S32, A = U8, B = S8, both K-major, M = 128; N >> 3 at bits 17-22.
__device__ __forceinline__ uint32_t idesc_i8(int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kFM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kFEpiWarps * 32) : "memory"); }

// Byte offset of byte k (0..31) of row n in a 32-byte-swizzled operand.
__device__ __forceinline__ int sw32_off(int n, int k) { return n * 32 + ((((k >> 4) ^ (n >> 2)) & 1) << 4) + (k & 15); }

// Smallest float >= x (x finite and >= 0, or +inf).
__device__ __forceinline__ float f32_up(double x) {
    float f = (float)x;
    if ((double)f < x) f = nextafterf(f, kInf);
    return f;
}
// Largest float <= x (x >= 0).
__device__ __forceinline__ float f32_down(double x) {
    float f = (float)x;
    if ((double)f > x) f = nextafterf(f, 0.0f);
    return f;
}

// Phi_j of the header: the float the row's v must exceed to be dropped.
__device__ __forceinline__ float phi_of(float ts, double E, double slack) {
    if (!(ts < kInf)) return kInf;
    const double s = sqrt((double)ts) * (1.0 + 1e-12) + E;
    return f32_up(s * s * (1.0 + 1e-12) + slack);
}

template <int KM, bool VEC4, bool WIDE>
__global__ void __launch_bounds__(kFThreads, 1)
    filter_kernel(const __grid_constant__ CUtensorMap mcodes, const FilterArgs a) {
    extern __shared__ unsigned char f_smem_raw[];
    __shared__ __align__(8) uint64_t full[kFStages], empty[kFStages], tfull[kFAcc], tempty[kFAcc], bfull[2], bempty[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    // per B buffer (the item it was built for): per-query weight constants
    __shared__ float2 s_qc[2][kFMaxG];     // {c_x = 2 s_j / 254 (WIDE: c_hi = 2 s_j), base = Bsq rounded down}
    __shared__ float s_qlo[2][kFMaxG];     // WIDE: c_lo = 2 s_j / 254
    __shared__ double s_slack[2][kFMaxG];  // slack_j
    __shared__ double s_ec[2];             // E_c
    // the item being tested
    __shared__ int32_t s_qid[kFMaxG], s_pp[kFMaxG], s_lock[kFMaxG];
    __shared__ float s_tau[kFMaxG], s_sig[kFMaxG];
    __shared__ volatile float s_phi[kFMaxG];
    __shared__ unsigned s_msk[kFEpiWarps][kFQW];  // per epilogue warp: survivor ballots of its queries

    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(f_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* s_a = smem;                                        // [kFStages][128 x 32]
    unsigned char* s_b = smem + kFStages * kFStageBytes;              // [2][nb][b_stride]
    float* s_topd = reinterpret_cast<float*>(s_b + 2 * (size_t)a.nb * a.b_stride);  // [G][KM]
    int32_t* s_topi = reinterpret_cast<int32_t*>(s_topd + (size_t)a.G * KM);         // [G][KM]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const int nb = a.nb, T = a.T, K = a.K, D = a.D, D_pad = a.D_pad;
    const int sub_per_tile = T / kFM;
    const int n_items = *a.n_items;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::saddr(&s_tmem)),
                     "r"(kFTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int s = 0; s < kFStages; ++s) {
            tc::bar_init(&full[s], 1);
            tc::bar_init(&empty[s], 1);
        }
        for (int b = 0; b < kFAcc; ++b) {
            tc::bar_init(&tfull[b], 1);
            tc::bar_init(&tempty[b], kFEpiWarps);
        }
        for (int b = 0; b < 2; ++b) {
            tc::bar_init(&bfull[b], 1);
            tc::bar_init(&bempty[b], 1);
        }
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    auto give_up = [&](int status) {
        *abort_flag = 1;
        atomicOr(a.err, status);
    };

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, armed = 0, armed_par = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const int4 item = a.items[it];
                const int64_t t0 = a.tile_off[item.x];
                const int L = (int)(a.row_off[item.x + 1] - a.row_off[item.x]);
                const int ns = (L + kFM - 1) / kFM;
                for (int s = 0; ok && s < ns; ++s) {
                    const int64_t tile = t0 + s / sub_per_tile;
                    const int h = s % sub_per_tile;
                    for (int b = 0; b < nb; ++b) {
                        if (!tc::bar_wait(&empty[stage], phase ^ 1u, a.polls, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc::bar_expect_tx(&full[stage], (uint32_t)kFStageBytes);
                        const int y = (int)((tile * nb + b) * T + h * kFM);
                        tc::tma_load_2d(s_a + (size_t)stage * kFStageBytes, &mcodes, 0, y, &full[stage]);
                        armed |= 1u << stage;
                        armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
                        if (++stage == kFStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok) give_up(TRIDENT_STATUS_MMA_TIMEOUT);
            for (int s = 0; s < kFStages; ++s)
                if (armed & (1u << s)) tc::bar_drain(&full[s], (armed_par >> s) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, g = 0;
            uint64_t* last_bar = nullptr;
            uint32_t last_par = 0;
            bool ok = true;
            int k = 0;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++k) {
                const int ib = k & 1;
                if (!tc::bar_wait(&bfull[ib], (uint32_t)(k >> 1) & 1u, a.polls, abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const int4 item = a.items[it];
                const int L = (int)(a.row_off[item.x + 1] - a.row_off[item.x]);
                const int ns = (L + kFM - 1) / kFM;
                const int N = round16(2 * item.z);
                const uint32_t idesc = idesc_i8(N);
                const uint32_t b0 = tc::saddr(s_b + (size_t)ib * nb * a.b_stride);
                for (int s = 0; ok && s < ns; ++s, ++g) {
                    const int acc = g & (kFAcc - 1);
                    if (!tc::bar_wait(&tempty[acc], ((g / kFAcc) & 1u) ^ 1u, a.polls, abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t d_tmem = tmem + (uint32_t)(acc * kFMaxN);
                    for (int b = 0; b < nb; ++b) {
                        if (!tc::bar_wait(&full[stage], phase, a.polls, abort_flag)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint64_t ad = desc_sw32(tc::saddr(s_a + (size_t)stage * kFStageBytes));
                        const uint64_t bd = desc_sw32(b0 + (uint32_t)(b * a.b_stride));
                        mma_i8(d_tmem, ad, bd, idesc, b > 0 ? 1u : 0u);
                        tc::mma_commit(&empty[stage]);
                        last_bar = &empty[stage];
                        last_par = phase;
                        if (++stage == kFStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    tc::mma_commit(&tfull[acc]);
                    last_bar = &tfull[acc];
                    last_par = (g / kFAcc) & 1u;
                }
                if (!ok) break;
                tc::mma_commit(&bempty[ib]);  // the B buffer is free once this item's MMAs complete
                last_bar = &bempty[ib];
                last_par = (uint32_t)(k >> 1) & 1u;
            }
            if (!ok) give_up(TRIDENT_STATUS_MMA_TIMEOUT);
            if (last_bar) tc::bar_drain(last_bar, last_par);
        }
    } else {
        // ---------------- epilogue warps
        const int ew = warp - 2;                 // 0 .. kFEpiWarps-1
        const int etid = tid - 64;               // 0 .. 32 kFEpiWarps - 1
        const int quarter = warp & 3;            // tensor-memory lanes this warp may read
        const int part = ew >> 2;                // which share of the item's queries
        unsigned long long st_cand = 0, st_surv = 0, st_ins = 0, st_items = 0;
        bool live = true;                        // false once a wait gave up: no more work, same barriers
        auto stop = [&]() {
            if (live && lane == 0) give_up(TRIDENT_STATUS_MMA_TIMEOUT);
            live = false;
        };

        // B operand of item `it` into buffer `buf`: per query j rows 2j (hi) and 2j+1 (lo) of every
        // code block, zero rows up to the padded N, and the item's constants.
        auto build_b = [&](int it, int buf) {
            const int4 item = a.items[it];
            const int c = item.x, pstart = item.y, n = item.z;
            const int N = round16(2 * n);
            unsigned char* bb = s_b + (size_t)buf * nb * a.b_stride;
            const int pad_words = (N - 2 * n) * 8;  // 32-bit words per block
            for (int i = etid; i < nb * pad_words; i += kFEpiWarps * 32) {
                const int b = i / pad_words, w = i - b * pad_words;
                reinterpret_cast<uint32_t*>(bb + (size_t)b * a.b_stride + 2 * n * 32)[w] = 0u;
            }
            const float* vm = a.vmin + (int64_t)c * D_pad;
            const float* dl = a.delta + (int64_t)c * D_pad;
            if (ew == 0) {  // E_c = ||eps_c||_2, per item
                double e2 = 0.0;
                for (int d = lane; d < D_pad; d += 32) {
                    const double e = (double)a.eps[(int64_t)c * D_pad + d];
                    e2 += e * e;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) e2 += __shfl_xor_sync(TB_FULL, e2, o);
                if (lane == 0) s_ec[buf] = sqrt(e2) * (1.0 + 1e-12) + 1e-300;
            }
            double pcap = 0.0;  // sum_d (255 delta_d)^2 >= P_r of every row of the list
            for (int d = lane; d < D_pad; d += 32) {
                const double t = 255.0 * (double)dl[d];
                pcap += t * t;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) pcap += __shfl_xor_sync(TB_FULL, pcap, o);
            for (int j = ew; j < n; j += kFEpiWarps) {
                const float* qr = a.qrot + (int64_t)a.pair_q[pstart + j] * D_pad;
                // lane l covers d = 4 l + 128 i + k; up to D_pad = 256 its weights stay in registers
                // between the two steps, above they are recomputed from a second read
                constexpr int kHeld = WIDE ? 1 : kFNarrowDPad / 128;
                double wv[kHeld][4];
                auto weights = [&](int i, double* w4, double* b4) {
                    const int d0 = 4 * lane + 128 * i;
                    const float4 v4 = *reinterpret_cast<const float4*>(vm + d0);
                    const float4 q4 = __ldg(reinterpret_cast<const float4*>(qr + d0));
                    const float4 d4 = *reinterpret_cast<const float4*>(dl + d0);
                    b4[0] = (double)v4.x - q4.x;
                    b4[1] = (double)v4.y - q4.y;
                    b4[2] = (double)v4.z - q4.z;
                    b4[3] = (double)v4.w - q4.w;
                    w4[0] = (double)d4.x * b4[0];
                    w4[1] = (double)d4.y * b4[1];
                    w4[2] = (double)d4.z * b4[2];
                    w4[3] = (double)d4.w * b4[3];
                };
                const int nch = (D_pad + 127) / 128;
                double wmax = 0.0, bsq = 0.0;
#pragma unroll
                for (int i = 0; i < (WIDE ? kFMaxDPad / 128 : kFNarrowDPad / 128); ++i) {
                    if (i < nch && 4 * lane + 128 * i < D_pad) {
                        double w4[4], b4[4];
                        weights(i, w4, b4);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            if (!WIDE) wv[WIDE ? 0 : i][k] = w4[k];
                            wmax = fmax(wmax, fabs(w4[k]));
                            bsq += b4[k] * b4[k];
                        }
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    wmax = fmax(wmax, __shfl_xor_sync(TB_FULL, wmax, o));
                    bsq += __shfl_xor_sync(TB_FULL, bsq, o);
                }
                const double sig = wmax > 0.0 ? wmax / 127.0 : 1.0;
                const double inv = 1.0 / sig;
                double rmax = 0.0;
#pragma unroll
                for (int i = 0; i < (WIDE ? kFMaxDPad / 128 : kFNarrowDPad / 128); ++i) {
                    const int d0 = 4 * lane + 128 * i;
                    if (i < nch && d0 < D_pad) {
                        double w4[4], b4[4];
                        if (WIDE) {
                            weights(i, w4, b4);
                        } else {
#pragma unroll
                            for (int k = 0; k < 4; ++k) w4[k] = wv[WIDE ? 0 : i][k];
                        }
                        uint32_t hw = 0, lw = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            // any split is valid: the residual is measured below against the exact w
                            const double w = w4[k];
                            const double h = fmin(fmax(rint(w * inv), -127.0), 127.0);
                            const double r = w - sig * h;
                            const double l = fmin(fmax(rint(r * inv * 254.0), -127.0), 127.0);
                            rmax = fmax(rmax, fabs(r - sig * l / 254.0));
                            hw |= ((uint32_t)(int32_t)h & 0xFFu) << (8 * k);
                            lw |= ((uint32_t)(int32_t)l & 0xFFu) << (8 * k);
                        }
                        const int b = d0 >> 5, kk = d0 & 31;
                        unsigned char* blk = bb + (size_t)b * a.b_stride;
                        *reinterpret_cast<uint32_t*>(blk + sw32_off(2 * j, kk)) = hw;
                        *reinterpret_cast<uint32_t*>(blk + sw32_off(2 * j + 1, kk)) = lw;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) rmax = fmax(rmax, __shfl_xor_sync(TB_FULL, rmax, o));
                if (lane == 0) {
                    // the float64 evaluation of the residual itself, then the term sizes for the roundings
                    rmax = rmax * (1.0 + 1e-9) + sig * 1e-12;
                    const double cmax = 255.0 * D_pad;                       // >= sum_d code_d
                    const double xmag = 2.0 * sig * 127.0 * cmax * (1.0 + 1.0 / 254.0);
                    const double mag = pcap + bsq + xmag;
                    s_slack[buf][j] = 8.0 * kU * mag + 2.0 * rmax * cmax;
                    const float base = f32_down(bsq * (1.0 - 1e-12));
                    if (WIDE) {
                        s_qc[buf][j] = make_float2((float)(2.0 * sig), base);
                        s_qlo[buf][j] = (float)(2.0 * sig / 254.0);
                    } else {
                        s_qc[buf][j] = make_float2((float)(2.0 * sig / 254.0), base);
                    }
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the tensor core reads B
        };

        int k = 0;
        uint32_t g = 0;
        if ((int)blockIdx.x < n_items) build_b(blockIdx.x, 0);
        epi_sync();
        if (etid == 0 && (int)blockIdx.x < n_items) tc::bar_arrive(&bfull[0]);
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++k) {
            const int ib = k & 1;
            const int nxt = it + gridDim.x;
            // the next item's B operand, while this item's MMAs run
            if (nxt < n_items) {
                const int m = k + 1;
                if (m >= 2) {
                    const bool w =
                        live && tc::bar_wait(&bempty[m & 1], (uint32_t)((m >> 1) - 1) & 1u, a.polls, abort_flag);
                    if (!__all_sync(TB_FULL, w)) stop();
                }
                if (live) build_b(nxt, m & 1);
                epi_sync();
                if (etid == 0) tc::bar_arrive(&bfull[m & 1]);
            }
            const int4 item = a.items[it];
            const int c = item.x, pstart = item.y, n = item.z;
            const int64_t r0 = a.row_off[c];
            const int64_t t0 = a.tile_off[c];
            const int L = (int)(a.row_off[c + 1] - r0);
            const int ns = (L + kFM - 1) / kFM;
            const double E = s_ec[ib];
            if (etid < n) {
                const int q = a.pair_q[pstart + etid];
                s_qid[etid] = q;
                s_pp[etid] = a.pair_p[pstart + etid];
                const float sig = a.qinfo[(int64_t)q * QI_LEN + QI_SIGMA];
                const float tq = ld_volatile_f32(a.tau + q);
                s_sig[etid] = sig;
                s_tau[etid] = tq;
                s_lock[etid] = 0;
                s_phi[etid] = phi_of(prune_threshold(tq, sig, a.rho), E, s_slack[ib][etid]);
            }
            for (int j = ew; j < n; j += kFEpiWarps) list_init<KM>(s_topd + j * KM, s_topi + j * KM, lane);
            if (etid == 0) ++st_items;
            epi_sync();

            // this warp's queries: a contiguous share of the item's, two accumulator columns each
            const int qper = (n + kFParts - 1) / kFParts;
            const int jb = part * qper;
            const int jn = max(0, min(n, jb + qper) - jb);
            for (int s = 0; s < ns; ++s, ++g) {
                const int acc = g & (kFAcc - 1);
                const int rl = s * kFM + quarter * 32 + lane;  // list-local row of this lane
                const bool valid = rl < L;
                const int64_t tile = t0 + s / sub_per_tile;
                const int slot = (s % sub_per_tile) * kFM + quarter * 32 + lane;
                // the row term is loaded before the wait, so its latency overlaps it
                const float P = (valid && live) ? __ldg(a.rowp + tile * T + slot) : 0.0f;
                const bool w = live && tc::bar_wait(&tfull[acc], (g / kFAcc) & 1u, a.polls, abort_flag);
                if (!__all_sync(TB_FULL, w)) stop();
                if (!live) continue;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t taddr =
                    tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * kFMaxN) + (uint32_t)(2 * jb);
                // per group of eight queries: the loads (jn is warp-uniform), one wait, the bound; the
                // ballots with survivors go to shared memory, their query slots to the bits of `nz`
                uint32_t nz = 0;
#pragma unroll
                for (int g8 = 0; g8 < kFQW; g8 += 8) {
                    if (g8 < jn) {
                        uint32_t r[16];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            if (g8 + i < jn)
                                asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                                             : "=r"(r[2 * i]), "=r"(r[2 * i + 1])
                                             : "r"(taddr + (uint32_t)(2 * (g8 + i))));
                        }
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            if (g8 + i < jn) {
                                const float2 qc = s_qc[ib][jb + g8 + i];
                                const int32_t hi = (int32_t)r[2 * i], lo = (int32_t)r[2 * i + 1];
                                const float v = WIDE ? fmaf(s_qlo[ib][jb + g8 + i], (float)lo, fmaf(qc.x, (float)hi, P + qc.y))
                                                     : fmaf(qc.x, (float)(hi * 254 + lo), P + qc.y);
                                const unsigned mk = __ballot_sync(TB_FULL, valid && v <= s_phi[jb + g8 + i]);
                                if (mk) {
                                    nz |= 1u << (g8 + i);
                                    if (lane == 0) s_msk[ew][g8 + i] = mk;
                                }
                            }
                        }
                    }
                }
                // the accumulator is in registers: release it before the survivors are refined
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) tc::bar_arrive(&tempty[acc]);
                st_cand += valid ? (unsigned long long)jn : 0ull;
                while (nz) {
                    const int i = __ffs(nz) - 1;
                    nz &= nz - 1;
                    const int j = jb + i;
                    const unsigned m = s_msk[ew][i];
                    const int q = s_qid[j];
                    // every survivor's exact distance (whole warp each), kept by the survivor's own lane
                    float my_d = kInf;
                    for (unsigned mm = m; mm;) {
                        const int sl = __ffs(mm) - 1;
                        mm &= mm - 1;
                        const int64_t grow = r0 + (int64_t)(s * kFM + quarter * 32 + sl);
                        const float dist = exact_dist_warp<VEC4, 2>(a.xb + grow * D, a.xq + (int64_t)q * D, D, lane);
                        const float d0 = __shfl_sync(TB_FULL, dist, 0);
                        if (lane == sl) my_d = d0;
                    }
                    const bool mine = (m >> lane) & 1u;
                    const int32_t my_id = mine ? __ldg(a.oid + r0 + (int64_t)(s * kFM + quarter * 32 + lane)) : -1;
                    if (lane == 0) st_surv += (unsigned)__popc(m);
                    // one insertion of all of them under the query's lock
                    int got = 0;
                    if (lane == 0) {
                        for (uint32_t spin = 0; spin < a.lock_spins; ++spin) {
                            if (atomicCAS(&s_lock[j], 0, 1) == 0) {
                                got = 1;
                                break;
                            }
                            __nanosleep(64);
                        }
                    }
                    got = __shfl_sync(TB_FULL, got, 0);
                    if (!got) {
                        if (lane == 0) atomicOr(a.err, TRIDENT_STATUS_LOCK_TIMEOUT);
                        continue;
                    }
                    __threadfence_block();
                    float* ld = s_topd + j * KM;
                    int32_t* li = s_topi + j * KM;
                    const int ins = list_offer<KM>(ld, li, K, mine, my_d, my_id, lane);
                    if (lane == 0) {
                        st_ins += (unsigned)ins;
                        const float kth = ld[K - 1];
                        const float gq = ld_volatile_f32(a.tau + q);
                        const float t_old = s_tau[j];
                        const float tq = fminf(fminf(t_old, kth), gq);
                        if (tq < t_old) {
                            s_tau[j] = tq;
                            s_phi[j] = phi_of(prune_threshold(tq, s_sig[j], a.rho), E, s_slack[ib][j]);
                        }
                        __threadfence_block();
                        atomicExch(&s_lock[j], 0);
                        if (kth < t_old && kth < gq) atomicMin(a.tau + q, __float_as_uint(kth));
                    }
                    __syncwarp();
                }
            }
            epi_sync();
            // this item's per-query lists into the (query, probe) candidate slots
            for (int i = etid; i < n * K; i += kFEpiWarps * 32) {
                const int j = i / K, kk = i - j * K;
                float d = s_topd[j * KM + kk];
                int32_t id = s_topi[j * KM + kk];
                if (!(id >= 0 && d <= s_tau[j])) {
                    d = kInf;
                    id = -1;
                }
                const int64_t slot = ((int64_t)s_qid[j] * a.nprobe + s_pp[j]) * K + kk;
                a.cand_d[slot] = d;
                a.cand_i[slot] = id;
            }
            epi_sync();
        }
        if (a.stats) {
            unsigned long long v[5] = {st_cand, st_cand * (unsigned long long)D_pad, st_surv, st_ins, st_items};
#pragma unroll
            for (int i = 0; i < 5; ++i) {
                unsigned long long x = v[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(TB_FULL, x, o);
                if (lane == 0 && x) atomicAdd(a.stats + i + (i == 4 ? 1 : 0), x);
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFTmemCols));
    }
}

int km_of(int K) { return K <= 32 ? 32 : 128; }

size_t filter_smem(const trident_index& idx, int K, int G) {
    const size_t b_stride = (size_t)round16(2 * G) * 32;
    return 1024 + (size_t)kFStages * kFStageBytes + 2 * (size_t)idx.num_blocks * b_stride +
           (size_t)G * km_of(K) * (sizeof(float) + sizeof(int32_t));
}

template <int KM, bool VEC4, bool WIDE>
cudaError_t launch_t(const CUtensorMap& map, const FilterArgs& a, size_t smem, int grid, cudaStream_t st) {
    auto kern = filter_kernel<KM, VEC4, WIDE>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kFThreads, smem, st>>>(map, a);
    return cudaGetLastError();
}

}  // namespace

int filter_group_size(const trident_index& idx, int K) {
    int G = kFMaxG;
    while (G > 1 && filter_smem(idx, K, G) > (size_t)(kFSmemLimit - kFStatic)) --G;
    return G;
}

bool filter_eligible(const trident_index& idx, int K, bool lb, bool ub_items, int64_t pairs) {
    if (!lb || ub_items || idx.row_p == nullptr || K > 128) return false;
    if (idx.tile_size % kFM != 0 || idx.D_pad % 32 != 0 || idx.D_pad > kFMaxDPad) return false;
    // measured on B200: faster than scan_kernel at c3 / c4 shapes (K = 10 and 100), slower with few
    // pairs (the items' operand set-up is not amortised) and at D = 960 (c2)
    if (!(idx.flags & TRIDENT_INDEX_TENSOR_STAGE_Y_ALWAYS) && (pairs < kFMinPairs || idx.D_pad > kFNarrowDPad))
        return false;
    // every code row of the 2-D view must have a 32-bit coordinate
    const int64_t max_tiles = idx.N / idx.tile_size + idx.nlist + 1;
    if (max_tiles * idx.num_blocks * idx.tile_size >= ((int64_t)1 << 31)) return false;
    return filter_smem(idx, K, 1) <= (size_t)(kFSmemLimit - kFStatic);
}

cudaError_t launch_filter(const trident_index& idx, const float* xq, const Workspace& ws, const ScanLaunch& sl,
                          unsigned long long* stats, cudaStream_t st) {
    if (sl.max_items <= 0) return cudaSuccess;
    CUtensorMap map;
    const int64_t max_tiles = idx.N / idx.tile_size + idx.nlist + 1;
    if (!make_codes_map(&map, idx.codes, max_tiles * idx.num_blocks * idx.tile_size)) return cudaErrorNotSupported;
    FilterArgs a;
    a.xb = idx.xb_sorted;
    a.oid = idx.orig_ids_sorted;
    a.row_off = idx.list_row_off;
    a.tile_off = idx.list_tile_off;
    a.rowp = idx.row_p;
    a.vmin = idx.vmin;
    a.delta = idx.delta;
    a.eps = idx.eps;
    a.xq = xq;
    a.qrot = ws.qrot;
    a.qinfo = ws.qinfo;
    a.items = (sl.pass == 1 ? ws.items_lpt : ws.items) + (sl.pass == 1 ? 0 : sl.item_base);
    a.n_items = ws.ctr + sl.pass;
    a.pair_q = ws.pair_q;
    a.pair_p = ws.pair_p;
    a.tau = ws.tau;
    a.cand_d = ws.cand_d;
    a.cand_i = ws.cand_i;
    a.stats = stats;
    a.err = ws.ctr + kStatusWord;
    a.lock_spins = lock_spin_limit();
    a.polls = mma_wait_limit();
    a.D = idx.D;
    a.D_pad = idx.D_pad;
    a.nb = idx.num_blocks;
    a.T = idx.tile_size;
    a.K = sl.K;
    a.nprobe = sl.nprobe;
    a.G = sl.G;
    a.b_stride = round16(2 * sl.G) * 32;
    a.rho = idx.lb_rel_slack;
    if (sl.G > kFMaxG || sl.G < 1) return cudaErrorInvalidValue;
    const size_t smem = filter_smem(idx, sl.K, sl.G);
    int grid = num_sms();
    if (grid > sl.max_items) grid = sl.max_items;
    const bool vec4 = (idx.D % 4) == 0 && (((uintptr_t)idx.xb_sorted | (uintptr_t)xq) & 15) == 0;
    const int KM = km_of(sl.K);
    const bool wide = idx.D_pad > kFNarrowDPad;
#define TB_FILTER_CASE(km, v, w) \
    if (KM == km && vec4 == v && wide == w) return launch_t<km, v, w>(map, a, smem, grid, st);
    TB_FILTER_CASE(32, true, false)
    TB_FILTER_CASE(32, false, false)
    TB_FILTER_CASE(128, true, false)
    TB_FILTER_CASE(128, false, false)
    TB_FILTER_CASE(32, true, true)
    TB_FILTER_CASE(32, false, true)
    TB_FILTER_CASE(128, true, true)
    TB_FILTER_CASE(128, false, true)
#undef TB_FILTER_CASE
    return cudaErrorInvalidValue;
}

}  // namespace tb
