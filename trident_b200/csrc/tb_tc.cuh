// Shared-memory barrier, tensor-copy and tensor-core helpers of the tcgen05 kernels (tb_gemm.cu,
// tb_filter.cu). Every wait is bounded: a poll may suspend the thread for about 256 ns (the
// suspend-time hint), so a limit of 2^22 polls ends within about a second.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace tb {
namespace tc {

constexpr uint32_t kDrainPolls = 1u << 22;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}

// One poll of the phase of `parity`.
__device__ __forceinline__ bool bar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, 256;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `parity`; gives up after `polls` polls or once another warp has set
// *abort. Returns whether the phase completed.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint32_t polls, volatile int* abort) {
    for (uint32_t i = 0; i < polls; ++i) {
        if (bar_try(bar, parity)) return true;
        if (*abort) return false;
    }
    return false;
}

// Bounded wait without an abort check (draining after an abort).
__device__ __forceinline__ void bar_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kDrainPolls; ++i)
        if (bar_try(bar, parity)) return;
}

// The barrier's next phase completes once every tcgen05 operation this thread issued before has.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                 : "memory");
}

// 2-D tensor copy of one box at (x, y) into `dst`, completing on `bar` (bytes counted).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(bar))
        : "memory");
}

}  // namespace tc
}  // namespace tb
