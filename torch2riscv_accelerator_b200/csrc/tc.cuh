// tcgen05 helpers of the tensor-core kernels (gemm.cu):
// fences around thread syncs, the shared-memory operand descriptor of a
// K-major 128-byte-swizzled tile, the kind::i8 instruction descriptor, MMA
// issue and commit, and TMEM loads.
#pragma once
#include "pdl.cuh"

namespace w8a8 {

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile in shared memory, 128-byte rows, 128-byte swizzle:
// start address >> 4, LBO 1 (unused by this layout), SBO 1024 B (8 rows),
// version 1, layout type 2 (SWIZZLE_128B). The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc(const void* tile) {
    const uint64_t a = (uint64_t)((smem_u32(tile) >> 4) & 0x3FFFu);
    return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::i8 instruction descriptor: D s32, A and B signed int8, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive int32 columns of this warp's 32 lanes (one row per thread)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


}  // namespace w8a8
