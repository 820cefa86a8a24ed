// W8A8 linear layers for decode (GEMV) and small row counts (M <= 16):
// y = (f32(xq . W[n]) * s_w[n]) * s_x   (llm/ref_model.py:198-202)
//
// HBM-bound weight streaming on the CUDA cores (no tensor cores at these row
// counts): every warp owns R output rows; each lane streams 16-byte chunks of
// those rows (ld.global.nc, L1 no-allocate), 4 dp4a per chunk and row against
// the int8 activations staged once per CTA in shared memory; a butterfly of
// warp shuffles sums the int32 partials (exact in any order).
//
// Prologues (fused, recomputed by every CTA from an L2-resident vector):
//   PRO_I8    int8 activations + scales given;
//   PRO_QUANT quant_act(x)              (llm/ref_model.py:191-196);
//   PRO_RMSQ  quant_act(rmsnorm(x, g))  (llm/ref_model.py:204-207, :224).
// Epilogues:
//   EPI_STORE  y = dequant;
//   EPI_RESID  y = resid + dequant      (llm/ref_model.py:245, :251);
//   EPI_SWIGLU the decode FFN dispatch (llm/ref_model.py:246-250;
//              compile_model.ffn_up :307-328): gate and up rows of the same
//              channel in one pass, h = (g*RECIP(1 + EXP(-g)))*u, the row amax
//              of |h| through a global atomic max, and the last CTA to finish
//              requantizes h to int8 (quant_act) for the down projection.
#include <cstdio>

#include "linear_common.cuh"
#include "pdl.cuh"

namespace w8a8 {

template <int MR, int PRO, int EPI, int R>
__global__ void __launch_bounds__(kThreads) linear_kernel(LinearParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int8_t* xs = reinterpret_cast<int8_t*>(smem_raw);
    __shared__ float sx[MR];
    __shared__ float red[32];
    __shared__ uint32_t bamax[MR];
    __shared__ int last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = p.k, kpad = k;                 // k % 16 == 0 (checked on the host)
    float* xf = reinterpret_cast<float*>(smem_raw + (size_t)MR * k);   // fp32 staging row [k]
    __shared__ unsigned long long bkey[MR];
    if (tid < MR) {
        bamax[tid] = 0u;
        bkey[tid] = 0ull;
    }
    pdl_wait();
    pdl_trigger();
    prologue<MR, PRO>(p, xs, xf, sx, red);

    constexpr bool kTwo = EPI == EPI_SWIGLU;
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    const int nch = k / 16;
    int acc[R][MR], acc2[kTwo ? R : 1][MR];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            acc[r][m] = 0;
            if (kTwo) acc2[r][m] = 0;
        }
    const int8_t* wrow[R];
    const int8_t* wrow2[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int n = min(row0 + r, p.n - 1);
        wrow[r] = p.w + (size_t)n * k;
        if (kTwo) wrow2[r] = p.w2 + (size_t)n * k;
    }
    if (row0 < p.n) {
#pragma unroll 2
        for (int c = lane; c < nch; c += 32) {
            int4 wv[R], wv2[kTwo ? R : 1];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                wv[r] = ld_stream16(wrow[r] + (size_t)c * 16);
                if (kTwo) wv2[r] = ld_stream16(wrow2[r] + (size_t)c * 16);
            }
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                const int4 xv = *reinterpret_cast<const int4*>(xs + (size_t)m * kpad + (size_t)c * 16);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    acc[r][m] = dp4a(wv[r].x, xv.x, acc[r][m]);
                    acc[r][m] = dp4a(wv[r].y, xv.y, acc[r][m]);
                    acc[r][m] = dp4a(wv[r].z, xv.z, acc[r][m]);
                    acc[r][m] = dp4a(wv[r].w, xv.w, acc[r][m]);
                    if (kTwo) {
                        acc2[r][m] = dp4a(wv2[r].x, xv.x, acc2[r][m]);
                        acc2[r][m] = dp4a(wv2[r].y, xv.y, acc2[r][m]);
                        acc2[r][m] = dp4a(wv2[r].z, xv.z, acc2[r][m]);
                        acc2[r][m] = dp4a(wv2[r].w, xv.w, acc2[r][m]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            acc[r][m] = warp_sum_i(acc[r][m]);
            if (kTwo) acc2[r][m] = warp_sum_i(acc2[r][m]);
        }
    // epilogue: lane j handles (r, m) pairs j, j + 32, ...
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int n = row0 + r;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if ((r * MR + m) % 32 != lane || n >= p.n || m >= p.m) continue;
            const size_t o = (size_t)m * p.n + n;
            const float v = fmul(fmul(i2f(acc[r][m]), __ldg(p.s_w + n)), sx[m]);
            if (EPI == EPI_STORE) {
                p.y[o] = v;
                if (p.acc != nullptr) p.acc[o] = acc[r][m];
                if (p.argmax_key != nullptr) atomicMax(&bkey[m], argmax_key(v, n));
            } else if (EPI == EPI_RESID) {
                p.y[o] = fadd(p.resid[o], v);
            } else {
                const float u = fmul(fmul(i2f(acc2[kTwo ? r : 0][m]), __ldg(p.s_w2 + n)), sx[m]);
                const float h = gate(v, u, GateAct{p.act, p.act_a, p.act_b});
                p.y[o] = h;
                atomicMax(&bamax[m], __float_as_uint(fabsf(h)));
            }
        }
    }
    if (EPI == EPI_STORE && p.argmax_key != nullptr) {
        __syncthreads();
        if (tid < p.m && tid < MR) atomicMax(p.argmax_key + tid, bkey[tid]);
    }
    if (EPI != EPI_SWIGLU || p.hq == nullptr) return;
    // row amax across the grid, then the last CTA requantizes (quant_act of h)
    __syncthreads();
    if (tid < p.m && tid < MR) atomicMax(p.amax_bits + tid, bamax[tid]);
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int m = 0; m < p.m; ++m) {
        const float amax = __uint_as_float(__ldcg(p.amax_bits + m));
        const float s = fmul(amax, W8A8_C127);
        const float inv = sfu_recip(s);
        const float* hr = p.y + (size_t)m * p.n;
        int8_t* qr = p.hq + (size_t)m * p.n;
        for (int i = tid; i < p.n; i += kThreads) qr[i] = (int8_t)to_i8(fmul(__ldcg(hr + i), inv));
        if (tid == 0) p.s_h[m] = s;
    }
    __syncthreads();
    if (tid < p.m) p.amax_bits[tid] = 0u;
    if (tid == 0) *p.counter = 0u;
}

template <int MR, int PRO, int EPI, int R>
static cudaError_t launch_t(const LinearParams& p, cudaStream_t st) {
    const int rows_per_cta = kWarps * R;
    const int grid = (p.n + rows_per_cta - 1) / rows_per_cta;
    const size_t smem = (size_t)MR * p.k + (PRO == PRO_I8 ? 0 : (size_t)p.k * 4);
    auto kern = linear_kernel<MR, PRO, EPI, R>;
    if (smem > 32 * 1024) {            // with the static shared arrays: opt in above the 48 KB default
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(kern, dim3(grid), dim3(kThreads), smem, st, p);
}

template <int MR, int PRO, int EPI>
static cudaError_t launch_r(const LinearParams& p, cudaStream_t st) {
    // enough CTAs for every SM to hold two; more rows per warp for tall matrices
    if (p.n >= 148 * 2 * kWarps * 4) return launch_t<MR, PRO, EPI, 4>(p, st);
    if (p.n >= 148 * 2 * kWarps * 2) return launch_t<MR, PRO, EPI, 2>(p, st);
    return launch_t<MR, PRO, EPI, 1>(p, st);
}

template <int PRO, int EPI>
static cudaError_t launch_m(const LinearParams& p, cudaStream_t st) {
    if (p.m <= 1) return launch_r<1, PRO, EPI>(p, st);
    if (p.m <= 2) return launch_r<2, PRO, EPI>(p, st);
    if (p.m <= 4) return launch_r<4, PRO, EPI>(p, st);
    if (p.m <= 8) return launch_r<8, PRO, EPI>(p, st);
    return launch_r<16, PRO, EPI>(p, st);
}

cudaError_t launch_linear(const LinearParams& p, int pro, int epi, cudaStream_t st) {
    if (gemv_fits(p, pro, epi)) return launch_gemv(p, pro, epi, st);
    if (pro == PRO_I8 && epi == EPI_STORE) return launch_m<PRO_I8, EPI_STORE>(p, st);
    if (pro == PRO_I8 && epi == EPI_RESID) return launch_m<PRO_I8, EPI_RESID>(p, st);
    if (pro == PRO_QUANT && epi == EPI_STORE) return launch_m<PRO_QUANT, EPI_STORE>(p, st);
    if (pro == PRO_QUANT && epi == EPI_RESID) return launch_m<PRO_QUANT, EPI_RESID>(p, st);
    if (pro == PRO_RMSQ && epi == EPI_STORE) return launch_m<PRO_RMSQ, EPI_STORE>(p, st);
    if (pro == PRO_RMSQ && epi == EPI_SWIGLU) return launch_m<PRO_RMSQ, EPI_SWIGLU>(p, st);
    if (pro == PRO_I8 && epi == EPI_SWIGLU) return launch_m<PRO_I8, EPI_SWIGLU>(p, st);
    return cudaErrorInvalidValue;
}

}  // namespace w8a8
