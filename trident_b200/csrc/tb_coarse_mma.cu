// Coarse distances a[j][c] = ||c||^2 - 2 q_j.c on the 5th-generation tensor cores (tcgen05).
//
// The reference computes q.C^T with a cuBLAS SGEMM (at::addmm_out, src/trident_v4_kernels.cu:
// 1233-1246) and trusts its rounding. Here one CTA computes a 128 x 128 tile (queries x lists)
// with tcgen05.mma kind::tf32. The accumulator lives in tensor memory (128 lanes x 128 columns).
// To keep FP32-level accuracy, each operand x is split into two TF32 values:
//   hi = x with the low 13 mantissa bits cleared,
//   lo = (x - hi) with the same mask.
// The three products hi*hi + hi*lo + lo*hi accumulate into the same tile ("3xTF32"). The selection
// that follows re-checks every list within a certified bound of the nprobe-th value in float64
// (probe_select_kernel), so the tensor-core rounding never changes the probe set. The bound is:
//   |a - exact| <= ((3D + 16) 2^-22 + 3.02 * 2^-20) * 1.01 * (2 ||q|| Cmax + Cmax^2).
// Why it holds:
//   - dropping lo*lo and the masking of lo costs <= 3.01 * 2^-20 |x_d||y_d| per term;
//   - 3D accumulations at a relative error of <= 2^-22 each allow any internal order and rounding
//     mode of the tensor core;
//   - the epilogue adds two float32 roundings.
//
// Pipeline: two shared-memory stages of K = 32. All 128 threads load the next stage's fp32
// rows (16-byte loads), split them and store them in the canonical K-major no-swizzle UMMA
// layout. One thread issues 12 MMAs and commits them to the stage's mbarrier. A stage is
// rewritten only after its mbarrier reports those MMAs complete. Every wait is bounded: on a
// timeout the kernel sets the error word that marks the search's results (NaN, -2), waits (also
// bounded) for its MMAs, frees its tensor memory and returns.
#include <cuda_runtime.h>
#include <stdint.h>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

constexpr int kCM = 128;  // queries per tile (UMMA M)
constexpr int kCN = kCoarseTileN;  // lists per tile (UMMA N)
constexpr int kCK = 32;   // K per stage: 4 UMMA k-steps of 8 TF32 values
constexpr int kCThreads = 128;
constexpr int kCChunks = kCK / 4;                // 16-byte K chunks per stage
constexpr int kCAbytes = kCChunks * kCM * 16;    // one split of the A tile
constexpr int kCBbytes = kCChunks * kCN * 16;    // one split of the B tile
constexpr int kCStageBytes = 2 * kCAbytes + 2 * kCBbytes;
// two stages + alignment slack + a 32 KB guard: a descriptor whose two strides were read the other
// way round would still address only this CTA's shared memory
constexpr int kCSmem = 2 * kCStageBytes + 32768 + 1024;
constexpr uint32_t kCWaitTries = 1u << 22;       // bounded mbarrier polling while draining after a timeout
constexpr uint32_t kCTmemCols = kCN;  // one float32 column per list of the tile (a power of 2 >= 32)

// Instruction descriptor: D = F32 (bits 4-5 = 1), A = B = TF32 (bits 7-9, 10-12 = 2), both
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdescTF32 =
    (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kCN >> 3) << 17) | ((uint32_t)(kCM >> 4) << 24);

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor, K-major without swizzle: core matrices of 8 rows x 16 bytes;
// lbo = byte distance between the two 16-byte K halves of an 8-element k-step, sbo = byte
// distance between consecutive 8-row groups; bits 46-47 = 1 (the Blackwell descriptor version).
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdescTF32), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity (at most `polls` polls); false if it did not
// complete in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t polls) {
    for (uint32_t i = 0; i < polls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// Load one stage's 32-wide K slice of row `row` (zero outside [0, rows) x [0, D)) and store its
// hi/lo splits at chunk-major positions: chunk c of row r at byte (c * 128 + r) * 16.
template <bool VEC>
__device__ __forceinline__ void load_split_row(const float* __restrict__ src, int rows, int D, int row, int k0,
                                               float4 (&v)[kCChunks]) {
    if (row < rows) {
        const float* p = src + (int64_t)row * D + k0;
        if (VEC && k0 + kCK <= D) {
#pragma unroll
            for (int c = 0; c < kCChunks; ++c) v[c] = __ldg(reinterpret_cast<const float4*>(p) + c);
        } else {
#pragma unroll
            for (int c = 0; c < kCChunks; ++c) {
                const int k = k0 + 4 * c;
                v[c].x = k + 0 < D ? __ldg(p + 4 * c + 0) : 0.0f;
                v[c].y = k + 1 < D ? __ldg(p + 4 * c + 1) : 0.0f;
                v[c].z = k + 2 < D ? __ldg(p + 4 * c + 2) : 0.0f;
                v[c].w = k + 3 < D ? __ldg(p + 4 * c + 3) : 0.0f;
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < kCChunks; ++c) v[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
}

// rows = the tile's row count (the chunk stride of the chunk-major layout)
template <int ROWS>
__device__ __forceinline__ void store_split(unsigned char* hi, unsigned char* lo, int r, const float4 (&v)[kCChunks]) {
#pragma unroll
    for (int c = 0; c < kCChunks; ++c) {
        const float4 x = v[c];
        const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
        const float4 l = make_float4(tf32_hi(x.x - h.x), tf32_hi(x.y - h.y), tf32_hi(x.z - h.z), tf32_hi(x.w - h.w));
        *reinterpret_cast<float4*>(hi + ((size_t)c * ROWS + r) * 16) = h;
        *reinterpret_cast<float4*>(lo + ((size_t)c * ROWS + r) * 16) = l;
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kCThreads, 1) coarse_mma_kernel(const float* __restrict__ xq,
                                                                  const float* __restrict__ cent,
                                                                  const float* __restrict__ cn, int B, int nlist,
                                                                  int D, float* __restrict__ out,
                                                                  float* __restrict__ tilemin,
                                                                  int32_t* __restrict__ err, uint32_t polls,
                                                                  int vec_out) {
    extern __shared__ unsigned char c_smem_raw[];
    __shared__ __align__(8) uint64_t s_bar[2];
    __shared__ uint32_t s_tmem;
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(c_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * kCM, n0 = blockIdx.x * kCN;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(kCTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init(&s_bar[0], 1);
        mbar_init(&s_bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    const int KT = (D + kCK - 1) / kCK;
    bool ok = true;
    int committed = 0;  // tiles whose MMAs were committed (the same count in every thread)
    for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt & 1;
        unsigned char* aH = smem + (size_t)s * kCStageBytes;
        unsigned char* aL = aH + kCAbytes;
        unsigned char* bH = aL + kCAbytes;
        unsigned char* bL = bH + kCBbytes;
        float4 va[kCChunks], vb[kCChunks];
        load_split_row<VEC>(xq, B, D, m0 + tid, kt * kCK, va);
        if (tid < kCN) load_split_row<VEC>(cent, nlist, D, n0 + tid, kt * kCK, vb);
        if (kt >= 2 && !mbar_wait(&s_bar[s], (uint32_t)((kt - 2) >> 1) & 1u, polls)) ok = false;  // stage free?
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        store_split<kCM>(aH, aL, tid, va);
        if (tid < kCN) store_split<kCN>(bH, bL, tid, vb);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor core
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int ks = 0; ks < kCK / 8; ++ks) {
                const uint32_t off = (uint32_t)(2 * ks) * kCM * 16;  // chunks 2ks, 2ks+1
                const uint32_t offb = (uint32_t)(2 * ks) * kCN * 16;
                const uint64_t dAH = umma_desc(smem_addr(aH) + off, kCM * 16, 128);
                const uint64_t dAL = umma_desc(smem_addr(aL) + off, kCM * 16, 128);
                const uint64_t dBH = umma_desc(smem_addr(bH) + offb, kCN * 16, 128);
                const uint64_t dBL = umma_desc(smem_addr(bL) + offb, kCN * 16, 128);
                umma_tf32(tmem, dAH, dBH, (kt > 0 || ks > 0) ? 1u : 0u);
                umma_tf32(tmem, dAH, dBL, 1u);
                umma_tf32(tmem, dAL, dBH, 1u);
            }
            umma_commit(&s_bar[s]);
        }
        committed = kt + 1;
    }
    // the last commit covers every MMA issued before it
    const int last = committed - 1;
    if (ok && last >= 0 && !mbar_wait(&s_bar[last & 1], (uint32_t)(last >> 1) & 1u, polls)) ok = false;
    ok = __syncthreads_and(ok) != 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    if (ok) {
        // epilogue: warp w reads tensor-memory lanes 32w..32w+31 (rows), 16 columns per load; each
        // thread also keeps its row's minimum over the tile's lists (the selection's upper bound)
        const int row = m0 + warp * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        float rmin = kInf;
        for (int c0 = 0; c0 < kCN; c0 += 16) {
            uint32_t r[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                "%13, %14, %15}, [%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15])
                : "r"(taddr + (uint32_t)c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < B) {
                const int col0 = n0 + c0;
                float* dst = out + (int64_t)row * nlist + col0;
                if (vec_out && col0 + 16 <= nlist) {
                    const float4* cn4 = reinterpret_cast<const float4*>(cn + col0);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const float4 c = __ldg(cn4 + v);
                        float4 o;
                        o.x = c.x - 2.0f * __uint_as_float(r[4 * v + 0]);
                        o.y = c.y - 2.0f * __uint_as_float(r[4 * v + 1]);
                        o.z = c.z - 2.0f * __uint_as_float(r[4 * v + 2]);
                        o.w = c.w - 2.0f * __uint_as_float(r[4 * v + 3]);
                        rmin = fminf(rmin, fminf(fminf(o.x, o.y), fminf(o.z, o.w)));
                        reinterpret_cast<float4*>(dst)[v] = o;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (col0 + j < nlist) {
                            const float o = __ldg(cn + col0 + j) - 2.0f * __uint_as_float(r[j]);
                            rmin = fminf(rmin, o);
                            dst[j] = o;
                        }
                    }
                }
            }
        }
        if (tilemin && row < B) tilemin[(int64_t)row * gridDim.x + blockIdx.x] = rmin;
    } else {
        if (tid == 0) atomicOr(err, TRIDENT_STATUS_MMA_TIMEOUT);
        // let any MMA still in flight finish (bounded, at the full default limit whatever `polls`
        // is) before the tensor memory is released
        if (last >= 0) mbar_wait(&s_bar[last & 1], (uint32_t)(last >> 1) & 1u, kCWaitTries);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCTmemCols));
    }
}

cudaError_t launch_coarse_gemm(const trident_index& idx, const float* xq, int B, float* coarse, float* tilemin,
                               int32_t* err, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    const bool vec = (idx.D % 4) == 0 && (((uintptr_t)xq | (uintptr_t)idx.centroids) & 15) == 0;
    dim3 grid((idx.nlist + kCN - 1) / kCN, (B + kCM - 1) / kCM);
    // 16-byte epilogue stores and norm loads: rows start 16-byte aligned (the workspace region is
    // 256-byte aligned) when nlist % 4 == 0, and the norms must be 16-byte aligned too
    const int vec_out = (idx.nlist % 4) == 0 && (((uintptr_t)coarse | (uintptr_t)idx.centroid_norm_sq) & 15) == 0;
    cudaError_t e;
    if (vec) {
        e = cudaFuncSetAttribute(coarse_mma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kCSmem);
        if (e != cudaSuccess) return e;
        coarse_mma_kernel<true><<<grid, kCThreads, kCSmem, st>>>(xq, idx.centroids, idx.centroid_norm_sq, B,
                                                                 idx.nlist, idx.D, coarse, tilemin, err, mma_wait_limit(), vec_out);
    } else {
        e = cudaFuncSetAttribute(coarse_mma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kCSmem);
        if (e != cudaSuccess) return e;
        coarse_mma_kernel<false><<<grid, kCThreads, kCSmem, st>>>(xq, idx.centroids, idx.centroid_norm_sq, B,
                                                                  idx.nlist, idx.D, coarse, tilemin, err, mma_wait_limit(), vec_out);
    }
    return cudaGetLastError();
}

}  // namespace tb
