// Pieces shared by the two W8A8 linear kernels (linear.cu: many rows, direct
// loads; gemv.cu: decode rows, bulk-copied weight tiles): the activation
// prologue and the greedy argmax key.
#pragma once
#include "w8a8_internal.h"
#include "w8a8_math.cuh"

namespace w8a8 {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <int MR, int PRO>
// gain: the RMSNorm gain staged in shared memory, or null to read p.norm_g.
__device__ __forceinline__ void prologue(const LinearParams& p, int8_t* xs, float* xf, float* sx, float* red,
                                         const float* gain = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = p.k;
    if (PRO == PRO_I8) {
        for (int m = 0; m < MR; ++m) {
            int4* dst = reinterpret_cast<int4*>(xs + (size_t)m * k);
            const int4* src = reinterpret_cast<const int4*>(p.xq + (size_t)m * k);
            for (int c = tid; c < k / 16; c += (int)blockDim.x) dst[c] = m < p.m ? __ldg(src + c) : make_int4(0, 0, 0, 0);
        }
        if (tid < MR) sx[tid] = tid < p.m ? p.s_x[tid] : 0.f;
        __syncthreads();
        return;
    }
    __shared__ float rr;
    // one row at a time through the fp32 staging buffer xf [k]: coalesced
    // float4 loads, the ordered sum of squares from shared memory (warp 0),
    // then amax and the int8 row.
    for (int m = 0; m < MR; ++m) {
        char4* dst = reinterpret_cast<char4*>(xs + (size_t)m * k);
        if (m >= p.m) {
            for (int c = tid; c < k / 4; c += (int)blockDim.x) dst[c] = make_char4(0, 0, 0, 0);
            if (tid == 0) sx[m] = 0.f;
            continue;
        }
        const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)m * k);
        float4* xf4 = reinterpret_cast<float4*>(xf);
        __syncthreads();                                         // xf free (previous row done)
        for (int c = tid; c < k / 4; c += (int)blockDim.x) xf4[c] = xr[c];
        __syncthreads();
        float r = 1.f;
        if (PRO == PRO_RMSQ) {
            if (warp == 0) {
                float ss = red_sum16([&](int i) { float v = xf[i]; return fmul(v, v); }, k, lane);
                if (lane == 0) rr = sfu_rsqrt(fadd(fmul(ss, p.inv_k), p.eps));
            }
            __syncthreads();
            r = rr;
        }
        const float4* gr = reinterpret_cast<const float4*>(gain != nullptr ? gain : p.norm_g);
        auto val = [&](int c) {
            float4 v = xf4[c];
            if (PRO == PRO_RMSQ) {
                float4 g = gr[c];
                v.x = fmul(fmul(v.x, r), g.x);
                v.y = fmul(fmul(v.y, r), g.y);
                v.z = fmul(fmul(v.z, r), g.z);
                v.w = fmul(fmul(v.w, r), g.w);
            }
            return v;
        };
        float a = 0.f;
        for (int c = tid; c < k / 4; c += (int)blockDim.x) {
            float4 v = val(c);
            a = nanmax(a, nanmax(nanmax(fabsf(v.x), fabsf(v.y)), nanmax(fabsf(v.z), fabsf(v.w))));
        }
        a = block_nanmax(a, red);
        const float s = fmul(a, W8A8_C127);
        const float inv = sfu_recip(s);
        for (int c = tid; c < k / 4; c += (int)blockDim.x) {
            float4 v = val(c);
            dst[c] = make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)),
                                to_i8(fmul(v.w, inv)));
        }
        if (tid == 0) {
            sx[m] = s;
            if (p.s_x_out != nullptr && blockIdx.x == 0) p.s_x_out[m] = s;
        }
    }
    __syncthreads();
}

// Greedy argmax key: larger value first, then the lower index (np.argmax's
// first maximum; NaN above everything, -0 as +0).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
    uint32_t ord = (v != v) ? 0xFFFFFFFFu : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

}  // namespace w8a8
