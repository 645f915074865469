// Device helpers shared by the trident_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trident_b200.h"

#define TB_FULL 0xffffffffu

namespace tb {

constexpr float kInf = __builtin_huge_valf();

// Squared-distance partial reduction over a warp, the reference's shfl_down butterfly
// (src/trident_v4_kernels.cu:11-17). Lane 0 ends with the distance; the tree (offsets 16..1)
// fixes the FP32 summation order that the CPU oracle restates.
__device__ __forceinline__ float warp_sum_ref(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(TB_FULL, v, off);
    return v;
}

// Exact uint8 -> float conversion of byte k of w in two full-rate ops: PRMT builds the float
// 2^23 + b (exponent byte 0x4B, the code in the low mantissa byte) and one FADD removes 2^23.
__device__ __forceinline__ float u8f(uint32_t w, int k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)k)) - 8388608.0f;
}

// Bytes k and k+1 of w as exact floats: two PRMTs and one packed FADD.
__device__ __forceinline__ float2 u8f2(uint32_t w, int k) {
    const float2 t = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)k)),
                                 __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)(k + 1))));
    return __fadd2_rn(t, make_float2(-8388608.0f, -8388608.0f));
}

// (d, id) strict order used by every top-K in the path (reference :26-31).
__device__ __forceinline__ bool better(float d, int32_t id, float kd, int32_t kid) {
    return d < kd || (d == kd && id < kid);
}

// Exact FP32 squared L2 distance of one row against one query by a whole warp, in the
// reference's order: lane l accumulates d = 4l + 128k + j, then the butterfly. Bit-identical to
// the reference's CM-FP32 scan (:321-336) and Stage-Z refine (:870-883).
// With VEC4 (D % 4 == 0), NL chunks of 128 dims are loaded together before their FMAs (the
// missing chunks of a lane's last batch are predicated off), so a 960-dim row costs ceil(8 / NL)
// memory round trips instead of 8; each lane's FMA order is unchanged.
template <bool VEC4, int NL = 1>
__device__ __forceinline__ float exact_dist_warp(const float* __restrict__ x, const float* __restrict__ q,
                                                 int D, int lane) {
    float part = 0.0f;
    int d = lane * 4;
    if constexpr (VEC4 && NL > 1) {
        for (; d < D; d += 128 * NL) {
            float4 xv[NL], qv[NL];
#pragma unroll
            for (int k = 0; k < NL; ++k) {
                if (d + 128 * k < D) {
                    xv[k] = __ldg(reinterpret_cast<const float4*>(x + d + 128 * k));
                    qv[k] = __ldg(reinterpret_cast<const float4*>(q + d + 128 * k));
                }
            }
#pragma unroll
            for (int k = 0; k < NL; ++k) {
                if (d + 128 * k < D) {
                    float df0 = xv[k].x - qv[k].x; part = fmaf(df0, df0, part);
                    float df1 = xv[k].y - qv[k].y; part = fmaf(df1, df1, part);
                    float df2 = xv[k].z - qv[k].z; part = fmaf(df2, df2, part);
                    float df3 = xv[k].w - qv[k].w; part = fmaf(df3, df3, part);
                }
            }
        }
        return warp_sum_ref(part);
    } else {
        if constexpr (VEC4) {
            for (; d + 3 < D; d += 128) {
                const float4 xv = __ldg(reinterpret_cast<const float4*>(x + d));
                const float4 qv = __ldg(reinterpret_cast<const float4*>(q + d));
                float df0 = xv.x - qv.x; part = fmaf(df0, df0, part);
                float df1 = xv.y - qv.y; part = fmaf(df1, df1, part);
                float df2 = xv.z - qv.z; part = fmaf(df2, df2, part);
                float df3 = xv.w - qv.w; part = fmaf(df3, df3, part);
            }
        } else {
            for (; d + 3 < D; d += 128) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float df = __ldg(x + d + j) - __ldg(q + d + j);
                    part = fmaf(df, df, part);
                }
            }
        }
        for (int dr = d; dr < d + 4 && dr < D; ++dr) {
            float df = __ldg(x + dr) - __ldg(q + dr);
            part = fmaf(df, df, part);
        }
        return warp_sum_ref(part);
    }
}

// Warp-cooperative sorted top-K list in shared memory: ld/li hold K entries ascending by
// (d, id); empty entries are (+inf, -1). KM (a multiple of 32) is the storage capacity.
template <int KM>
__device__ __forceinline__ void list_init(float* ld, int32_t* li, int lane) {
#pragma unroll
    for (int m = 0; m < KM / 32; ++m) {
        ld[lane + 32 * m] = kInf;
        li[lane + 32 * m] = -1;
    }
}

// Insert (d, id), known to beat entry K-1, keeping the list sorted. Called by all 32 lanes with
// the same (d, id).
template <int KM>
__device__ __forceinline__ void list_insert(float* ld, int32_t* li, int K, float d, int32_t id, int lane) {
    float od[KM / 32], pd[KM / 32];
    int32_t oi[KM / 32], pi[KM / 32];
    int less = 0;
#pragma unroll
    for (int m = 0; m < KM / 32; ++m) {
        const int i = lane + 32 * m;
        od[m] = ld[i];
        oi[m] = li[i];
        pd[m] = (i > 0) ? ld[i - 1] : kInf;
        pi[m] = (i > 0) ? li[i - 1] : -1;
        if (i < K && better(od[m], oi[m], d, id)) ++less;
    }
    const int pos = __reduce_add_sync(TB_FULL, (unsigned)less);
    __syncwarp();
#pragma unroll
    for (int m = 0; m < KM / 32; ++m) {
        const int i = lane + 32 * m;
        if (i < K) {
            if (i > pos) { ld[i] = pd[m]; li[i] = pi[m]; }
            else if (i == pos) { ld[i] = d; li[i] = id; }
        }
    }
    __syncwarp();
}

// True when (d, id) is already among the first K entries (a row refined twice for one query
// produces the bit-identical distance, so it must not take a second slot).
template <int KM>
__device__ __forceinline__ bool list_contains(const float* ld, const int32_t* li, int K, float d, int32_t id, int lane) {
    bool hit = false;
#pragma unroll
    for (int m = 0; m < KM / 32; ++m) {
        const int i = lane + 32 * m;
        hit |= (i < K) && li[i] == id && ld[i] == d;
    }
    return __any_sync(TB_FULL, hit);
}

// Offer one candidate per lane (valid lanes only) to the list; returns the number inserted.
template <int KM>
__device__ __forceinline__ int list_offer(float* ld, int32_t* li, int K, bool valid, float d, int32_t id, int lane) {
    float kd = ld[K - 1];
    int32_t ki = li[K - 1];
    unsigned mask = __ballot_sync(TB_FULL, valid && better(d, id, kd, ki));
    int inserted = 0;
    while (mask) {
        const int s = __ffs(mask) - 1;
        mask &= mask - 1;
        const float sd = __shfl_sync(TB_FULL, d, s);
        const int32_t si = __shfl_sync(TB_FULL, id, s);
        kd = ld[K - 1];
        ki = li[K - 1];
        if (better(sd, si, kd, ki) && !list_contains<KM>(ld, li, K, sd, si, lane)) {
            list_insert<KM>(ld, li, K, sd, si, lane);
            ++inserted;
        }
    }
    return inserted;
}

// Ordered-uint32 image of a float (monotone for all non-NaN values).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ float ld_volatile_f32(const uint32_t* p) {
    return __uint_as_float(*reinterpret_cast<const volatile uint32_t*>(p));
}
__device__ __forceinline__ int32_t ld_volatile_i32(const int32_t* p) { return *reinterpret_cast<const volatile int32_t*>(p); }

// Prune threshold for a query whose current K-th exact distance is tau: a row is dropped when its
// partial bound exceeds (sqrt(tau (1 + rho)) + sigma)^2. rho covers the float32 accumulation of
// the bound and of the exact distance, sigma the query-side roundings (Minkowski); the final
// factor covers the roundings of this expression.
__device__ __forceinline__ float prune_threshold(float tau, float sigma, float rho) {
    if (!(tau < kInf)) return kInf;
    const float s = sqrtf(tau * (1.0f + rho)) + sigma;
    return s * s * (1.0f + 1e-6f);
}

// Threshold implied by an SQ8 upper bound ub of one row: its exact FP32 distance is at most this.
__device__ __forceinline__ float ub_threshold(float ub, float sigma, float rho) {
    if (!(ub < kInf)) return kInf;
    const float s = sqrtf(ub * (1.0f + 2.0f * rho)) + sigma;
    return s * s * (1.0f + 2.0f * rho) * (1.0f + 1e-6f);
}

}  // namespace tb
