// Programmatic dependent launch (PDL) and bulk-copy helpers for sm_100a.
//
// Every kernel of the decode chain is launched with programmatic stream
// serialization, so it may start while its predecessor still runs. The rule
// each kernel follows:
//   - before pdl_wait(): read only data that no kernel of the current chain
//     position i-1 writes (weights, cache rows of earlier steps); a kernel calls
//     pdl_trigger() only after its own pdl_wait(), so when kernel i+1 runs its
//     pre-wait code, every kernel up to i-1 has completed;
//   - after pdl_wait(): everything the predecessors wrote is visible.
// Without the launch attribute both instructions are no-ops.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace w8a8 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk copy global -> shared, completion counted on the mbarrier.
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Barrier `id` (1..15) among the first n threads of the block (warps that
// take part call it; barrier 0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// 2-D tile load (TMA) of a tensor map into shared memory, completion counted on
// the mbarrier. x: the innermost coordinate (a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Bounded wait for the mbarrier phase with the given parity: try_wait suspends
// the thread in hardware until the phase completes or a ~1 us time hint runs
// out; at most 2^20 tries (about a second). Returns false when it gave up (the
// caller records an error and stops using the stage).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (int i = 0; i < (1 << 20); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(1000u)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Bounded spin on the mbarrier phase (test_wait never suspends the thread):
// for one thread of a tight producer / consumer pipeline, where a suspended
// wait would wake late. At most 2^26 polls (a fraction of a second).
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (int i = 0; i < (1 << 26); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Sense-reversing barrier among `n` CTAs over global memory: count[0] counts
// arrivals, gen[0] is bumped by the last one. Bounded: gives up after ~2^22
// polls (about 0.2 s) and returns false. Call with the whole CTA; the CTA's
// prior global writes are released before it arrives, and what the others
// wrote is visible after it returns.
__device__ __forceinline__ bool cta_barrier(unsigned int* count, volatile unsigned int* gen, unsigned int n) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int g0 = *gen;
        __threadfence();
        int ok = 1;
        if (atomicAdd(count, 1u) == n - 1) {
            *count = 0u;
            __threadfence();
            atomicAdd((unsigned int*)gen, 1u);
        } else {
            int it = 0;
            while (*gen == g0) {
                if (++it > (1 << 22)) {
                    ok = 0;
                    break;
                }
                if (it > 32) __nanosleep(32);
            }
        }
        __threadfence();
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

}  // namespace w8a8

namespace w8a8 {

extern int g_use_pdl;   // launch with programmatic stream serialization (w8a8_set_pdl)

// cudaLaunchKernelEx with the PDL attribute (when enabled).
template <typename... Exp, typename... Act>
inline cudaError_t launch_k(void (*kern)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Act&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Exp>(args)...);
}

}  // namespace w8a8
