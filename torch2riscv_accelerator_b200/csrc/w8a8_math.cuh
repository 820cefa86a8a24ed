// Device numerics of the W8A8 path: the overlay's fp32 vector engine and SFU,
// restated for sm_100a.
//
// - fp32 add / mul: one IEEE round-to-nearest-even rounding each, never fused
//   (__fadd_rn / __fmul_rn are never contracted into FMA; the library is also
//   built with -fmad=false). Reference: llm/fp32.py:1-20, llm/ref_model.py:151-163.
// - EXP / RECIP / RSQRT: the SFU's table + one Newton step sequences
//   (llm/sfu.py:1-26, :69-114), with its input flush-to-zero and the flushing
//   exponent scaling (llm/fp32.py:145-151). Tables: sfu_tables.h.
// - int8 conversion: round to nearest even, saturate +-127, NaN -> 0
//   (llm/ref_model.py:136-139).
// - fixed-order sum over D = 16 lanes (llm/ref_model.py:179-186).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "sfu_tables.h"

namespace w8a8 {

constexpr uint32_t kQNaN = 0x7FC00000u;
constexpr uint32_t kPInf = 0x7F800000u;
constexpr int kLanes = 16;                  // D: the reduction lane count of the overlay

// F(1/127) and F(1.4426950408889634) as bit patterns (host-rounded constants).
#define W8A8_C127 __uint_as_float(0x3C010204u)
#define W8A8_LOG2E __uint_as_float(0x3FB8AA3Bu)

// The SFU tables live in constant memory: the scalar uses (the scales of
// quant_act, RMSNorm) index them uniformly across a warp. Kernels that evaluate
// EXP per element stage the EXP table in shared memory (sfu_exp_tab).
__constant__ __align__(16) static uint32_t g_exp_t[64] = W8A8_SFU_EXP_T_INIT;
__constant__ __align__(16) static uint32_t g_exp_s[64] = W8A8_SFU_EXP_S_INIT;
__constant__ __align__(16) static uint32_t g_rec_t[64] = W8A8_SFU_RECIP_T_INIT;
__constant__ __align__(16) static uint32_t g_rec_s[64] = W8A8_SFU_RECIP_S_INIT;
__constant__ __align__(16) static uint32_t g_rsq_t[128] = W8A8_SFU_RSQRT_T_INIT;
__constant__ __align__(16) static uint32_t g_rsq_s[128] = W8A8_SFU_RSQRT_S_INIT;

// The same tables in global memory, in the layouts the kernels stage into
// shared memory: a warp reading constant memory at 32 different indices is
// served one index at a time, a 16-byte global load per thread at once. So
// staging (before a kernel's programmatic-launch wait, on the path of the
// launch when the previous kernel ends early) copies these blocks.
// g_sfu_block: RECIP T | S, RSQRT T | S (SfuSmem); g_gate_block: EXP T | S,
// RECIP T | S (the gate tables; its first half is the EXP table alone).
__device__ __align__(16) static const uint32_t g_sfu_block[384] = {
    W8A8_SFU_RECIP_T_LIST, W8A8_SFU_RECIP_S_LIST, W8A8_SFU_RSQRT_T_LIST, W8A8_SFU_RSQRT_S_LIST};
__device__ __align__(16) static const uint32_t g_gate_block[256] = {
    W8A8_SFU_EXP_T_LIST, W8A8_SFU_EXP_S_LIST, W8A8_SFU_RECIP_T_LIST, W8A8_SFU_RECIP_S_LIST};

// Copy `words` (a multiple of 4) of a 16-byte aligned global block into
// 16-byte aligned shared memory, one 16-byte load per thread.
__device__ __forceinline__ void stage_block16(uint32_t* dst, const uint32_t* src, int words) {
    for (int i = threadIdx.x; i < words / 4; i += blockDim.x)
        reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}

// The EXP table (T | S, 128 words) into 16-byte aligned shared memory.
__device__ __forceinline__ void stage_exp_table(uint32_t* etab) { stage_block16(etab, g_gate_block, 128); }

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }
__device__ __forceinline__ float tab(const uint32_t* t, int i) { return __uint_as_float(t[i]); }

__device__ __forceinline__ int to_i8(float v) {
    if (v != v) return 0;
    float r = rintf(v);
    r = fminf(fmaxf(r, -127.f), 127.f);
    return (int)r;
}

// max that propagates NaN (np.max semantics)
__device__ __forceinline__ float nanmax(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return fmaxf(a, b);
}

__device__ __forceinline__ float ftz(float x) {
    uint32_t b = __float_as_uint(x);
    return ((b >> 23) & 0xFFu) == 0 ? __uint_as_float(b & 0x80000000u) : x;
}

// y * 2^n by exponent addition: below-normal -> signed zero, overflow -> signed inf.
__device__ __forceinline__ float ldexp_ftz(float y, int n) {
    uint32_t b = __float_as_uint(y);
    uint32_t s = b & 0x80000000u;
    int e = (int)((b >> 23) & 0xFFu);
    if (e == 0) return __uint_as_float(s);
    if (e == 255) return (b & 0x7FFFFFu) ? __uint_as_float(kQNaN) : y;
    int ne = e + n;
    if (ne < 1) return __uint_as_float(s);
    if (ne > 254) return __uint_as_float(s | kPInf);
    return __uint_as_float(s | ((uint32_t)ne << 23) | (b & 0x7FFFFFu));
}

// EXP (llm/sfu.py:69-82): t = x*log2e, n = floor(t), f = t - n, u = 64f,
// i = floor(u) (at most 63), r = u - i, y = T[i] + r*S[i], y * 2^n.
// tt / ts: the table (T, S bit patterns) wherever the caller keeps it.
__device__ __forceinline__ float sfu_exp_tab(float x, const uint32_t* tt, const uint32_t* ts) {
    x = ftz(x);
    if (x != x) return __uint_as_float(kQNaN);
    if (x >= 89.f) return __uint_as_float(kPInf);
    if (x <= -104.f) return 0.f;
    float t = fmul(x, W8A8_LOG2E);
    float fl = floorf(t);
    int n = (int)fl;
    float f = fsub(t, i2f(n));
    float u = fmul(f, 64.f);
    int i = (int)floorf(u);
    i = i < 0 ? 0 : (i > 63 ? 63 : i);
    float r = fsub(u, i2f(i));
    float y = fadd(__uint_as_float(tt[i]), fmul(r, __uint_as_float(ts[i])));
    return ldexp_ftz(y, n);
}

__device__ __forceinline__ float sfu_exp(float x) {
    x = ftz(x);
    if (x != x) return __uint_as_float(kQNaN);
    if (x >= 89.f) return __uint_as_float(kPInf);
    if (x <= -104.f) return 0.f;
    float t = fmul(x, W8A8_LOG2E);
    float fl = floorf(t);
    int n = (int)fl;
    float f = fsub(t, i2f(n));
    float u = fmul(f, 64.f);
    int i = (int)floorf(u);
    i = i < 0 ? 0 : (i > 63 ? 63 : i);
    float r = fsub(u, i2f(i));
    float y = fadd(tab(g_exp_t, i), fmul(r, tab(g_exp_s, i)));
    return ldexp_ftz(y, n);
}

// RECIP (llm/sfu.py:85-96): x = +-m*2^E, i = top 6 fraction bits,
// y0 = T[i] + r*S[i], y1 = y0*(2 - m*y0), +-y1*2^-E.
__device__ __forceinline__ float sfu_recip_tab(float x, const uint32_t* rt, const uint32_t* rs) {
    uint32_t b = __float_as_uint(ftz(x));
    uint32_t s = b & 0x80000000u;
    int e = (int)((b >> 23) & 0xFFu);
    uint32_t frac = b & 0x7FFFFFu;
    if (e == 0) return __uint_as_float(s | kPInf);
    if (e == 255) return frac ? __uint_as_float(kQNaN) : __uint_as_float(s);
    int i = (int)(frac >> 17);
    float m = __uint_as_float(frac | 0x3F800000u);
    float r = fmul(i2f((int)(frac & 0x1FFFFu)), 0x1p-17f);
    float y0 = fadd(__uint_as_float(rt[i]), fmul(r, __uint_as_float(rs[i])));
    float y1 = fmul(y0, fsub(2.f, fmul(m, y0)));
    return __uint_as_float(__float_as_uint(ldexp_ftz(y1, 127 - e)) | s);
}

__device__ __forceinline__ float sfu_recip(float x) { return sfu_recip_tab(x, g_rec_t, g_rec_s); }

// RSQRT (llm/sfu.py:99-114): x = m*2^E, odd E uses m' = 2m; j = 64*(E odd) +
// top 6 fraction bits; y1 = y0*(1.5 - (m'*(y0*y0))*0.5); y1 * 2^(-(E - odd)/2).
// rt, rs: the T and S tables wherever the caller keeps them.
__device__ __forceinline__ float sfu_rsqrt_tab(float x, const uint32_t* rt, const uint32_t* rs) {
    uint32_t b = __float_as_uint(ftz(x));
    uint32_t s = b >> 31;
    int e = (int)((b >> 23) & 0xFFu);
    uint32_t frac = b & 0x7FFFFFu;
    if (e == 255 && frac) return __uint_as_float(kQNaN);
    if (e == 0) return __uint_as_float(kPInf);
    if (s) return __uint_as_float(kQNaN);
    if (e == 255) return 0.f;
    int E = e - 127;
    int odd = E & 1;
    int j = odd * 64 + (int)(frac >> 17);
    float m2 = __uint_as_float(frac | ((uint32_t)(127 + odd) << 23));
    float r = fmul(i2f((int)(frac & 0x1FFFFu)), 0x1p-17f);
    float y0 = fadd(__uint_as_float(rt[j]), fmul(r, __uint_as_float(rs[j])));
    float d = fsub(1.5f, fmul(fmul(m2, fmul(y0, y0)), 0.5f));
    float y1 = fmul(y0, d);
    return ldexp_ftz(y1, -((E - odd) / 2));
}

__device__ __forceinline__ float sfu_rsqrt(float x) { return sfu_rsqrt_tab(x, g_rsq_t, g_rsq_s); }

// RECIP and RSQRT tables in shared memory, for the scalar lookups on a
// kernel's critical path (quant_act's scale, RMSNorm's factor): a lookup in
// constant memory that misses the SM's constant cache costs an L2 round trip.
struct __align__(16) SfuSmem {
    uint32_t rec_t[64], rec_s[64], rsq_t[128], rsq_s[128];
};

// Every thread of the block takes part; a block barrier must separate it from
// the first lookup.
__device__ __forceinline__ void stage_sfu(SfuSmem* sf) { stage_block16(sf->rec_t, g_sfu_block, 384); }

__device__ __forceinline__ float sfu_recip_s(float x, const SfuSmem* sf) { return sfu_recip_tab(x, sf->rec_t, sf->rec_s); }
__device__ __forceinline__ float sfu_rsqrt_s(float x, const SfuSmem* sf) { return sfu_rsqrt_tab(x, sf->rsq_t, sf->rsq_s); }

// SiLU gating (llm/ref_model.py:249-250): (g * RECIP(1 + EXP(g * -1))) * u
__device__ __forceinline__ float silu_gate(float g, float u) {
    float sig = sfu_recip(fadd(1.f, sfu_exp(fmul(g, -1.f))));
    return fmul(fmul(g, sig), u);
}

// The same with the EXP and RECIP tables wherever the caller keeps them (tab:
// EXP T | EXP S | RECIP T | RECIP S, 64 words each; shared memory when every
// lane looks up its own index: constant memory serializes divergent reads).
__device__ __forceinline__ float silu_gate_tab(float g, float u, const uint32_t* tab) {
    float sig = sfu_recip_tab(fadd(1.f, sfu_exp_tab(fmul(g, -1.f), tab, tab + 64)), tab + 128, tab + 192);
    return fmul(fmul(g, sig), u);
}

// GELU's tanh approximation as the overlay computes it
// (compiler/frontend/hf_generic.py:840-856, SaGELUTanh): z = g * (A + (g * g) * B),
// g * RECIP(EXP(z) + 1) -- multiplies, adds, EXP and RECIP only -- then * u.
// A = F(-2 sqrt(2 / pi)), B = F(-2 sqrt(2 / pi) * 0.044715), from the host.
__device__ __forceinline__ float gelu_gate(float g, float u, float a, float b) {
    const float z = fmul(g, fadd(a, fmul(fmul(g, g), b)));
    return fmul(fmul(g, sfu_recip(fadd(sfu_exp(z), 1.f))), u);
}

__device__ __forceinline__ float gelu_gate_tab(float g, float u, const uint32_t* tab, float a, float b) {
    const float z = fmul(g, fadd(a, fmul(fmul(g, g), b)));
    return fmul(fmul(g, sfu_recip_tab(fadd(sfu_exp_tab(z, tab, tab + 64), 1.f), tab + 128, tab + 192)), u);
}

// The gated activation of a kind (0 SiLU, 1 GELU-tanh): act(g) * u.
struct GateAct {
    int kind;
    float a, b;                // GELU-tanh constants
};

__device__ __forceinline__ float gate_tab(float g, float u, const uint32_t* tab, const GateAct& act) {
    return act.kind == 1 ? gelu_gate_tab(g, u, tab, act.a, act.b) : silu_gate_tab(g, u, tab);
}

__device__ __forceinline__ float gate(float g, float u, const GateAct& act) {
    return act.kind == 1 ? gelu_gate(g, u, act.a, act.b) : silu_gate(g, u);
}

// Copy the four 64-word tables of silu_gate_tab into 16-byte aligned shared
// memory (whole block).
__device__ __forceinline__ void stage_silu_tables(uint32_t* tab) { stage_block16(tab, g_gate_block, 256); }

// Fixed-order sum of n values v(i) (llm/ref_model.py:179-186), computed by one
// full warp: lane l < 16 adds v(l), v(16 + l), v(32 + l), ... in order (zero
// padding included), then the pairwise tree lane 2j + lane 2j+1 per level.
// Returns the sum on every lane.
template <typename Fn>
__device__ __forceinline__ float red_sum16(Fn v, int n, int lane) {
    float acc = 0.f;
    if (lane < kLanes) {
        acc = lane < n ? v(lane) : 0.f;
        const int groups = (n + kLanes - 1) / kLanes;
        const int full = n / kLanes;                         // groups without padding
        int g = 1;
        for (; g + 8 <= full; g += 8) {                      // 8 independent reads, then the ordered adds
            float t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) t[j] = v((g + j) * kLanes + lane);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fadd(acc, t[j]);
        }
        for (; g < groups; ++g) {
            const int i = g * kLanes + lane;
            acc = fadd(acc, i < n ? v(i) : 0.f);
        }
    }
#pragma unroll
    for (int s = 1; s < kLanes; s <<= 1) {
        float o = __shfl_down_sync(0xffffffffu, acc, s);
        if ((lane & (2 * s - 1)) == 0) acc = fadd(acc, o);
    }
    return __shfl_sync(0xffffffffu, acc, 0);
}

__device__ __forceinline__ float warp_nanmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nanmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide NaN-propagating max; red: shared scratch of >= 32 floats.
__device__ __forceinline__ float block_nanmax(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_nanmax(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = lane < nw ? red[lane] : 0.f;
    r = warp_nanmax(r);
    return r;
}

__device__ __forceinline__ int block_sum_i(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_i(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int r = lane < nw ? red[lane] : 0;
    return warp_sum_i(r);
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// 16-byte weight load through the read-only path, not kept in L1.
__device__ __forceinline__ int4 ld_stream16(const void* p) {
    int4 v;
    asm("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace w8a8
