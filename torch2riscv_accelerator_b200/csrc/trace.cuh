// Device timeline of the decode kernels (trace builds only: -DW8A8_TRACE).
//
// The B200 counterpart of the overlay's event counters and profile dump
// (rtl/sysarray/sa_perf.v, compiler/runtime/sa/sa_context.c:507-535): each
// CTA of an instrumented kernel records the global timer, its SM clock and SM
// id at fixed points of the kernel (entry, after the programmatic-launch wait,
// after its prologue, ...). A CTA reserves kTraceMarks records with one atomic
// at entry; its marks are plain stores by thread 0 (no contention on the
// critical path); marks are taken by thread 0 wherever it passes them. Without
// W8A8_TRACE the macros expand to nothing.
//
// Record (3 x u64): global timer ns, clock64,
// kind << 56 | tag << 48 | smid << 32 | CTAs of the launch << 16 | cta (low 16 bits).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace w8a8 {

constexpr int kTraceMarks = 16;
enum TraceKind { TR_GEMV = 1, TR_ATTN = 2, TR_EMBED = 3, TR_ADVANCE = 4 };

#ifdef W8A8_TRACE
namespace {
__device__ unsigned long long* g_tr_buf;   // per translation unit: bound by trace_bind_<unit>
__device__ unsigned int* g_tr_n;
__device__ unsigned int g_tr_cap;

__device__ __forceinline__ void tr_write(unsigned int slot, int kind, int tag) {
    uint64_t gt;
    uint32_t sm;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    const uint64_t ck = clock64();
    const uint32_t cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    const uint32_t ctas = gridDim.x * gridDim.y * gridDim.z;
    unsigned long long* r = g_tr_buf + 3ull * slot;
    r[0] = gt;
    r[1] = ck;
    r[2] = ((uint64_t)kind << 56) | ((uint64_t)tag << 48) | ((uint64_t)(sm & 0xFFu) << 32) |
           ((uint64_t)(ctas & 0xFFFFu) << 16) | (cta & 0xFFFFu);
}

// The CTA's base slot (shared by every function of the kernel).
__device__ __forceinline__ unsigned int& tr_base() {
    __shared__ unsigned int b;
    return b;
}

// Thread 0: reserve this CTA's records and write mark 0.
__device__ __forceinline__ void tr_begin(int kind) {
    if (threadIdx.x != 0) return;
    unsigned int b = ~0u;
    if (g_tr_buf != nullptr) {
        b = atomicAdd(g_tr_n, (unsigned int)kTraceMarks);
        if (b + kTraceMarks > g_tr_cap) b = ~0u;
    }
    tr_base() = b;
    if (b != ~0u) tr_write(b, kind, 0);
}

// Mark `tag` (thread 0; any function of an instrumented kernel).
__device__ __forceinline__ void tr_mark(int kind, int tag) {
    if (threadIdx.x != 0) return;
    const unsigned int b = tr_base();
    if (b != ~0u) tr_write(b + (unsigned int)tag, kind, tag);
}

// Host: point this unit's instrumentation at a record buffer.
static inline int tr_bind_unit(void* buf, void* n, unsigned int cap) {
    unsigned long long* b = static_cast<unsigned long long*>(buf);
    unsigned int* c = static_cast<unsigned int*>(n);
    if (cudaMemcpyToSymbol(g_tr_buf, &b, sizeof(b)) != cudaSuccess) return 1;
    if (cudaMemcpyToSymbol(g_tr_n, &c, sizeof(c)) != cudaSuccess) return 1;
    return cudaMemcpyToSymbol(g_tr_cap, &cap, sizeof(cap)) != cudaSuccess;
}
}  // namespace
#define W8A8_TRACE_BEGIN(kind) ::w8a8::tr_begin(kind)
#define W8A8_MARK(kind, tag) ::w8a8::tr_mark(kind, tag)
#define W8A8_TRACE_BINDER(name) \
    int name(void* buf, void* n, unsigned int cap) { return tr_bind_unit(buf, n, cap); }
#else
#define W8A8_TRACE_BEGIN(kind) ((void)0)
#define W8A8_MARK(kind, tag) ((void)0)
#define W8A8_TRACE_BINDER(name) \
    int name(void*, void*, unsigned int) { return 1; }
#endif

// One binder per translation unit that holds instrumented kernels.
int trace_bind_gemv(void* buf, void* n, unsigned int cap);
int trace_bind_attn(void* buf, void* n, unsigned int cap);
int trace_bind_misc(void* buf, void* n, unsigned int cap);

}  // namespace w8a8
