// Persistent tcgen05 GEMM of queries (or rows) against centroids, with TMA-fed operands:
//   coarse stage:  a[j][c] = ||c||^2 - 2 q_j.c for every list c (3xTF32), plus each row's minimum
//                  over every 128-list tile (the probe selection's upper bound);
//   index build:   argmin_c (||c||^2 - 2 x.c) for every row x (1xTF32), the list assignment.
//
// The reference computes the coarse product with a cuBLAS SGEMM (at::addmm_out,
// src/trident_v4_kernels.cu:1233-1246) and assigns rows with faiss (benchmarks/phase4a_suite.py:
// 389-421). Here one CTA per SM runs a loop over output tiles of 128 x 128 with three warp roles:
//   warp 0      TMA producer: for each K = 32 slice of a tile, one elected lane waits until a
//               shared-memory stage is free, arms its mbarrier with the stage's byte count and
//               issues the tensor copies (A = 128 query rows, B = 128 centroid rows; hi and lo
//               splits for 3xTF32): one 2-D copy of 32 floats x 128 rows per operand, 128-byte
//               swizzled, which is the canonical K-major SWIZZLE_128B UMMA layout (each row's slice
//               is one 128-byte request).
//   warp 1      MMA issuer: one elected lane waits for a stage, issues tcgen05.mma kind::tf32
//               (12 per slice for 3xTF32: hi*hi + hi*lo + lo*hi; 4 for 1xTF32) into one of two
//               tensor-memory accumulators and commits the stage back to the producer; after the
//               tile's last slice it commits the accumulator to the epilogue.
//   epilogue    each thread owns one accumulator row (tensor-memory lane): eight warps of 64
//               columns write distances and each row's minimum over its 64 lists (two warps per lane
//               quarter), or four warps of 128 columns keep a running argmin. They read the
//               accumulator with tcgen05.ld and free it, so the next tile's MMAs overlap them.
// Shared memory holds three stages (64 KB each for 3xTF32). Every wait is bounded: a wait that
// gives up (or sees another warp give up) sets the status word, the producer then waits (bounded)
// for the copies it issued, the MMA warp for its last commit, and the tensor memory is freed.
//
// Error bound of the 3xTF32 coarse values (unchanged from a register-staged version; any internal
// accumulation order of the tensor core is allowed):
//   |a - exact| <= ((3D + 16) 2^-22 + 3.02 * 2^-20) * 1.01 * (2 ||q|| Cmax + Cmax^2).
// The operand splits hi = x with the low 13 bits cleared, lo = (x - hi) with the same mask are made
// by split_tf32_kernel; the 1xTF32 assignment feeds the rows and centroids unsplit (the list
// assignment is an input of the index and needs no particular rounding).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "tb_common.cuh"
#include "tb_internal.h"
#include "tb_tc.cuh"

namespace tb {

namespace {

constexpr int kGM = 128;                 // rows of A per tile (UMMA M)
constexpr int kGN = kCoarseTileN;        // rows of B per tile (UMMA N)
constexpr int kGK = 32;                  // K per stage
constexpr int kGStages = 3;
// producer, MMA issuer, then the epilogue: four warps of 128 columns (argmin: each row's minimum stays
// in one thread) or eight of 64 (distances: two warps per tensor-memory lane quarter)
template <bool ARGMIN>
struct EpiShape {
    static constexpr int kWarps = ARGMIN ? 4 : 8;
    static constexpr int kCols = kCoarseTileN * 4 / kWarps;
    static constexpr int kThreads = 64 + 32 * kWarps;
};
constexpr int kGOpBytes = kGM * kGK * 4; // one operand split of one stage: 16 KB
constexpr uint32_t kGTmemCols = 2 * kGN; // two accumulators of 128 columns

static_assert(kGM == kGN, "square tiles: A and B stage buffers have the same size");
static_assert(EpiShape<false>::kCols == kCoarseMinSpan, "one row minimum per epilogue warp and tile");

template <int SPLITS>
struct GemmShape {
    static constexpr int kOps = SPLITS == 3 ? 4 : 2;          // A_hi [A_lo] B_hi [B_lo]
    static constexpr int kStageBytes = kOps * kGOpBytes;
    static constexpr int kSmem = kGStages * kStageBytes + 1024;  // + alignment slack
};

// Instruction descriptor: D = F32, A = B = TF32, both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
constexpr uint32_t kGIdesc =
    (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kGN >> 3) << 17) | ((uint32_t)(kGM >> 4) << 24);

using tc::saddr;

// K-major descriptor of a 128-byte-swizzled tile (the layout a SWIZZLE_128B tensor copy of 32
// floats x 128 rows writes: row r at r * 128 bytes, its 16-byte chunk j at chunk j ^ (r % 8)):
// leading byte offset 16 (unused within a swizzle atom), stride byte offset 1024 between 8-row
// groups, descriptor version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63). The k-th
// 8-deep step of the 32-float slice starts 32 * k bytes further (the swizzle is applied to the
// absolute address, so each tile must start 1024-byte aligned).
__device__ __forceinline__ uint64_t gdesc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void gmma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kGIdesc), "r"(accumulate));
}

__device__ __forceinline__ void gcommit(uint64_t* bar) { tc::mma_commit(bar); }
__device__ __forceinline__ void gbar_init(uint64_t* bar, uint32_t count) { tc::bar_init(bar, count); }
__device__ __forceinline__ void gbar_arrive(uint64_t* bar) { tc::bar_arrive(bar); }
__device__ __forceinline__ void gbar_expect_tx(uint64_t* bar, uint32_t bytes) { tc::bar_expect_tx(bar, bytes); }
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, uint32_t polls, volatile int* abort) {
    return tc::bar_wait(bar, parity, polls, abort);
}
__device__ __forceinline__ void gdrain(uint64_t* bar, uint32_t parity) { tc::bar_drain(bar, parity); }

// One K = 32 slice (128 bytes per row) of 128 rows starting at `row0` into `dst` (16 KB, 1024-byte
// aligned), 128-byte swizzled.
__device__ __forceinline__ void tma_slice(void* dst, const CUtensorMap* map, int row0, int kc, uint64_t* bar) {
    tc::tma_load_2d(dst, map, kc * kGK, row0, bar);
}

struct GemmParams {
    int M, N, KT;           // rows of A, rows of B, K slices of 32
    int n_tiles, n_split;   // B tiles, B-tile ranges per A block (units = m_blocks * n_split)
    int n_min;              // entries per row of the row-minimum array: ceil(N / kCoarseMinSpan)
    int units;
    uint32_t polls;
    const float* cn;        // [N] ||c||^2
    float* out;             // coarse: [M, N] distances
    float* tilemin;         // coarse: [M, n_min] minima over 64-column spans (optional)
    int32_t* arg_out;       // assignment: [M] nearest row of B
    int32_t* err;
};

// The CTA's tile sequence: units u = blockIdx.x, blockIdx.x + gridDim.x, ...; unit u covers A block
// m = u / n_split and B tiles [lo, hi) of its range.
__device__ __forceinline__ void unit_range(const GemmParams& p, int u, int& m, int& lo, int& hi) {
    m = u / p.n_split;
    const int s = u - m * p.n_split;
    lo = (int)((int64_t)s * p.n_tiles / p.n_split);
    hi = (int)((int64_t)(s + 1) * p.n_tiles / p.n_split);
}

template <int SPLITS, bool ARGMIN>
__global__ void __launch_bounds__(EpiShape<ARGMIN>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mA_hi, const __grid_constant__ CUtensorMap mA_lo,
                   const __grid_constant__ CUtensorMap mB_hi, const __grid_constant__ CUtensorMap mB_lo,
                   const GemmParams p) {
    using S = GemmShape<SPLITS>;
    extern __shared__ unsigned char g_smem_raw[];
    __shared__ __align__(8) uint64_t full[kGStages], empty[kGStages], tfull[2], tempty[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    using E = EpiShape<ARGMIN>;
    __shared__ float s_cn[E::kWarps][E::kCols];  // per epilogue warp: its columns' ||c||^2
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&s_tmem)),
                     "r"(kGTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int s = 0; s < kGStages; ++s) {
            gbar_init(&full[s], 1);
            gbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            gbar_init(&tfull[b], 1);
            gbar_init(&tempty[b], E::kWarps);
        }
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    auto give_up = [&]() {
        *abort_flag = 1;
        atomicOr(p.err, TRIDENT_STATUS_MMA_TIMEOUT);
    };

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_par = 0;  // stages with copies issued, parity of their last phase
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                int m, lo, hi;
                unit_range(p, u, m, lo, hi);
                for (int n = lo; ok && n < hi; ++n) {
                    for (int kc = 0; kc < p.KT; ++kc) {
                        if (!gwait(&empty[stage], phase ^ 1u, p.polls, abort_flag)) {
                            ok = false;
                            break;
                        }
                        unsigned char* st = smem + (size_t)stage * S::kStageBytes;
                        gbar_expect_tx(&full[stage], (uint32_t)S::kStageBytes);
                        tma_slice(st, &mA_hi, m * kGM, kc, &full[stage]);
                        if (SPLITS == 3) {
                            tma_slice(st + kGOpBytes, &mA_lo, m * kGM, kc, &full[stage]);
                            tma_slice(st + 2 * kGOpBytes, &mB_hi, n * kGN, kc, &full[stage]);
                            tma_slice(st + 3 * kGOpBytes, &mB_lo, n * kGN, kc, &full[stage]);
                        } else {
                            tma_slice(st + kGOpBytes, &mB_hi, n * kGN, kc, &full[stage]);
                        }
                        armed |= 1u << stage;
                        armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
                        if (++stage == kGStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok) give_up();
            // every copy this warp issued lands before the CTA can exit
            for (int s = 0; s < kGStages; ++s)
                if (armed & (1u << s)) gdrain(&full[s], (armed_par >> s) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t tile_iter = 0;
            uint64_t* last_bar = nullptr;
            uint32_t last_par = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                int m, lo, hi;
                unit_range(p, u, m, lo, hi);
                for (int n = lo; ok && n < hi; ++n, ++tile_iter) {
                    const int buf = tile_iter & 1;
                    const uint32_t tpar = (tile_iter >> 1) & 1u;
                    if (!gwait(&tempty[buf], tpar ^ 1u, p.polls, abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t d_tmem = tmem + (uint32_t)(buf * kGN);
                    for (int kc = 0; kc < p.KT; ++kc) {
                        if (!gwait(&full[stage], phase, p.polls, abort_flag)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t st = saddr(smem + (size_t)stage * S::kStageBytes);
#pragma unroll
                        for (int ks = 0; ks < kGK / 8; ++ks) {
                            const uint32_t off = (uint32_t)ks * 32;  // 8 floats into each 128-byte row
                            const uint32_t acc0 = (kc > 0 || ks > 0) ? 1u : 0u;
                            if (SPLITS == 3) {
                                const uint64_t aH = gdesc_sw128(st + off);
                                const uint64_t aL = gdesc_sw128(st + kGOpBytes + off);
                                const uint64_t bH = gdesc_sw128(st + 2 * kGOpBytes + off);
                                const uint64_t bL = gdesc_sw128(st + 3 * kGOpBytes + off);
                                gmma(d_tmem, aH, bH, acc0);
                                gmma(d_tmem, aH, bL, 1u);
                                gmma(d_tmem, aL, bH, 1u);
                            } else {
                                const uint64_t a = gdesc_sw128(st + off);
                                const uint64_t b = gdesc_sw128(st + kGOpBytes + off);
                                gmma(d_tmem, a, b, acc0);
                            }
                        }
                        gcommit(&empty[stage]);  // the stage is free once these MMAs complete
                        last_bar = &empty[stage];
                        last_par = phase;
                        if (++stage == kGStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    gcommit(&tfull[buf]);
                    last_bar = &tfull[buf];
                    last_par = tpar;
                }
            }
            if (!ok) give_up();
            if (last_bar) gdrain(last_bar, last_par);  // no MMA in flight when tensor memory is freed
        }
    } else {
        // ---------------- epilogue: thread = accumulator row
        const int quarter = warp & 3;      // tensor-memory lanes 32 * quarter ... (each run of 4 warps covers 0-3)
        const int half = (warp - 2) >> 2;  // which 64-column half (eight epilogue warps; 0 with four)
        const int cbeg = half * E::kCols;  // this warp's first column of the tile
        float* cnw = s_cn[warp - 2];       // this warp's copy of its columns' norms (no cross-warp barrier)
        const bool vec = !ARGMIN && ((p.N & 3) == 0) && ((((uintptr_t)p.out) | ((uintptr_t)p.cn)) & 15) == 0;
        uint32_t tile_iter = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
            int m, lo, hi;
            unit_range(p, u, m, lo, hi);
            const int row = m * kGM + quarter * 32 + lane;
            float best_d = kInf;
            int32_t best_i = -1;
            for (int n = lo; n < hi; ++n, ++tile_iter) {
                const int buf = tile_iter & 1;
                const uint32_t tpar = (tile_iter >> 1) & 1u;
                const int col_base = n * kGN + cbeg;
                // this warp's norms: issued before the wait, so their latency overlaps it
                float cnv[E::kCols / 32];
#pragma unroll
                for (int i = 0; i < E::kCols / 32; ++i) {
                    const int col = col_base + i * 32 + lane;
                    cnv[i] = col < p.N ? __ldg(p.cn + col) : 0.0f;
                }
                // warp-uniform: the tensor-memory loads below are .sync.aligned
                const bool w = gwait(&tfull[buf], tpar, p.polls, abort_flag);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int i = 0; i < E::kCols / 32; ++i) cnw[i * 32 + lane] = cnv[i];
                __syncwarp();
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t taddr =
                    tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * kGN) + (uint32_t)cbeg;
                float rmin = kInf;
                float* dst = (!ARGMIN && row < p.M) ? p.out + (int64_t)row * p.N + col_base : nullptr;
#pragma unroll 1
                for (int c0 = 0; c0 < E::kCols; c0 += 32) {
                    uint32_t r[32];
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
                        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
                        "%28, %29, %30, %31}, [%32];"
                        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
                          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
                          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                        : "r"(taddr + (uint32_t)c0));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (row >= p.M) continue;
                    const int col0 = col_base + c0;
                    if (ARGMIN) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float dv = cnw[c0 + j] - 2.0f * __uint_as_float(r[j]);
                            if (dv < best_d && col0 + j < p.N) {  // ascending columns: ties keep the smaller id
                                best_d = dv;
                                best_i = col0 + j;
                            }
                        }
                    } else if (vec && col0 + 32 <= p.N) {
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            float4 o;
                            o.x = cnw[c0 + 4 * v + 0] - 2.0f * __uint_as_float(r[4 * v + 0]);
                            o.y = cnw[c0 + 4 * v + 1] - 2.0f * __uint_as_float(r[4 * v + 1]);
                            o.z = cnw[c0 + 4 * v + 2] - 2.0f * __uint_as_float(r[4 * v + 2]);
                            o.w = cnw[c0 + 4 * v + 3] - 2.0f * __uint_as_float(r[4 * v + 3]);
                            rmin = fminf(rmin, fminf(fminf(o.x, o.y), fminf(o.z, o.w)));
                            // streaming store: the distances must not evict the operands from L2
                            __stcs(reinterpret_cast<float4*>(dst + c0) + v, o);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j < p.N) {
                                const float o = cnw[c0 + j] - 2.0f * __uint_as_float(r[j]);
                                rmin = fminf(rmin, o);
                                __stcs(dst + c0 + j, o);
                            }
                        }
                    }
                }
                // the accumulator may be overwritten once every epilogue warp has read it
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) gbar_arrive(&tempty[buf]);
                if (!ARGMIN && p.tilemin && row < p.M) {
                    const int span = n * (kGN / kCoarseMinSpan) + half;  // E::kCols == kCoarseMinSpan here
                    if (span < p.n_min) __stcs(p.tilemin + (int64_t)row * p.n_min + span, rmin);
                }
            }
            if (ARGMIN && ok && row < p.M) p.arg_out[row] = best_i;
        }
        if (!ok && lane == 0) give_up();
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGTmemCols));
    }
}

// hi = x with the low 13 mantissa bits cleared, lo = (x - hi) likewise; [rows, D] -> [rows, D_pad]
// (zeros beyond D).
__global__ void split_tf32_kernel(const float* __restrict__ src, int64_t rows, int D, int D_pad,
                                  float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t total = rows * D_pad;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / D_pad;
        const int d = (int)(i - r * D_pad);
        const float x = d < D ? src[r * D + d] : 0.0f;
        const float h = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
        hi[i] = h;
        lo[i] = __uint_as_float(__float_as_uint(x - h) & 0xFFFFE000u);
    }
}

// ------------------------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no link-time dependency on libcuda).
// ------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, []() {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// 2-D view {kdim, rows} of a row-major [rows, ld] float matrix, box {32, 128}, 128-byte swizzle:
// one copy writes a K = 32 slice of 128 rows in the layout gdesc_sw128 describes. Rows past `rows`
// and columns past `kdim` read as zeros.
bool make_map(CUtensorMap* m, const float* base, int64_t rows, int ld, int kdim) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kdim, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {(cuuint32_t)kGK, (cuuint32_t)kGM};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_maps(CUtensorMap* maps, const float* const* bases, const int64_t* rows, int n, int ld, int kdim) {
    for (int i = 0; i < n; ++i)
        if (!make_map(&maps[i], bases[i], rows[i], ld, kdim)) return false;
    return true;
}

template <int SPLITS, bool ARGMIN>
cudaError_t launch_gemm(const CUtensorMap* maps, GemmParams p, cudaStream_t st) {
    using S = GemmShape<SPLITS>;
    auto kern = tc_gemm_kernel<SPLITS, ARGMIN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem);
    if (e != cudaSuccess) return e;
    const int grid = p.units < num_sms() ? p.units : num_sms();
    kern<<<grid, EpiShape<ARGMIN>::kThreads, S::kSmem, st>>>(maps[0], maps[SPLITS == 3 ? 1 : 0], maps[SPLITS == 3 ? 2 : 1],
                                            maps[SPLITS == 3 ? 3 : 1], p);
    return cudaGetLastError();
}

}  // namespace

// 2-D view {32 bytes, rows} of the blocked SQ8 codes, one 32-dim block of one row per view row,
// box {32, 128}, 32-byte swizzle: one copy writes one code block of 128 rows in the canonical K-major
// SWIZZLE_32B layout of an 8-bit UMMA operand (row r at r * 32 bytes, its 16-byte half h at
// h ^ ((r / 4) % 2)).
bool make_codes_map(CUtensorMap* m, const uint8_t* codes, int64_t rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {32, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {32};
    const cuuint32_t box[2] = {32, 128};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(codes), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t coarse_split_bytes(const trident_index& idx, int B) {
    return ((size_t)B + (size_t)idx.nlist) * (size_t)idx.D_pad * 2 * sizeof(float);
}

cudaError_t launch_coarse_gemm(const trident_index& idx, const float* xq, int B, float* coarse, float* tilemin,
                               float* splits, int32_t* err, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    const int Dp = idx.D_pad;
    float* qhi = splits;
    float* qlo = qhi + (size_t)B * Dp;
    float* chi = qlo + (size_t)B * Dp;
    float* clo = chi + (size_t)idx.nlist * Dp;
    split_tf32_kernel<<<1184, 256, 0, st>>>(xq, B, idx.D, Dp, qhi, qlo);
    split_tf32_kernel<<<1184, 256, 0, st>>>(idx.centroids, idx.nlist, idx.D, Dp, chi, clo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap maps[4];
    const float* bases[4] = {qhi, qlo, chi, clo};
    const int64_t rows[4] = {B, B, idx.nlist, idx.nlist};
    GemmParams p{};
    if (!make_maps(maps, bases, rows, 4, Dp, Dp)) return cudaErrorNotSupported;
    p.M = B;
    p.N = idx.nlist;
    p.KT = Dp / kGK;
    p.n_tiles = (idx.nlist + kGN - 1) / kGN;
    p.n_min = (idx.nlist + kCoarseMinSpan - 1) / kCoarseMinSpan;
    const int m_blocks = (B + kGM - 1) / kGM;
    // enough units for two per SM, each a contiguous range of B tiles of one A block
    int ns = (2 * num_sms() + m_blocks - 1) / m_blocks;
    if (ns > p.n_tiles) ns = p.n_tiles;
    if (ns < 1) ns = 1;
    p.n_split = ns;
    p.units = m_blocks * ns;
    p.polls = mma_wait_limit();
    p.cn = idx.centroid_norm_sq;
    p.out = coarse;
    p.tilemin = tilemin;
    p.arg_out = nullptr;
    p.err = err;
    return launch_gemm<3, false>(maps, p, st);
}

cudaError_t launch_assign(const float* x, int64_t n, int D, const float* cent, const float* cnorm, int nlist,
                          int32_t* out, int32_t* err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    CUtensorMap maps[2];
    const float* bases[2] = {x, cent};
    const int64_t rows[2] = {n, nlist};
    GemmParams p{};
    if (!make_maps(maps, bases, rows, 2, D, D)) return cudaErrorNotSupported;
    p.M = (int)n;
    p.N = nlist;
    p.KT = (D + kGK - 1) / kGK;
    p.n_tiles = (nlist + kGN - 1) / kGN;
    p.n_split = 1;  // each unit covers every centroid tile of its rows: the argmin stays in registers
    p.units = (int)((n + kGM - 1) / kGM);
    p.polls = mma_wait_limit();
    p.cn = cnorm;
    p.out = nullptr;
    p.tilemin = nullptr;
    p.arg_out = out;
    p.err = err;
    return launch_gemm<1, true>(maps, p, st);
}

}  // namespace tb
