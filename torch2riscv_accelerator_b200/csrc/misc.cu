// Small kernels of the decode path: embedding dequant, RMSNorm, quant_act,
// greedy argmax, and elementwise SFU evaluation (the device functions exposed
// for testing).
#include "linear_common.cuh"
#include "pdl.cuh"

namespace w8a8 {

// Rows of x -> int8 rows and scales for the tensor-core GEMM: quant_act(x), or
// quant_act(rmsnorm(x, g)) with the overlay's ordered sum (the GEMV prologue's
// arithmetic; llm/ref_model.py:191-196, :204-207). One CTA per row.
__global__ void __launch_bounds__(kThreads) norm_quant_kernel(const float* x, const float* g, int k, float eps,
                                                             float inv_k, int8_t* xq, float* s_x) {
    extern __shared__ __align__(16) unsigned char nq_smem[];
    int8_t* xs = reinterpret_cast<int8_t*>(nq_smem);                   // [k]
    float* xf = reinterpret_cast<float*>(nq_smem + ((k + 15) & ~15));  // [k]
    __shared__ float sx[1], red[32];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    LinearParams lp{};
    lp.m = 1, lp.k = k, lp.x = x + (size_t)row * k, lp.norm_g = g, lp.eps = eps, lp.inv_k = inv_k;
    if (g != nullptr) prologue<1, PRO_RMSQ>(lp, xs, xf, sx, red);
    else prologue<1, PRO_QUANT>(lp, xs, xf, sx, red);
    for (int c = threadIdx.x; c < k / 16; c += blockDim.x)
        reinterpret_cast<int4*>(xq + (size_t)row * k)[c] = reinterpret_cast<const int4*>(xs)[c];
    if (threadIdx.x == 0) s_x[row] = sx[0];
}

cudaError_t launch_norm_quant(const float* x, const float* g, int m, int k, float eps, float inv_k, int8_t* xq,
                              float* s_x, cudaStream_t st) {
    const size_t sm = (size_t)((k + 15) & ~15) + (size_t)k * 4;
    cudaError_t e = cudaFuncSetAttribute(norm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    cudaFuncSetAttribute(norm_quant_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(norm_quant_kernel, dim3(m), dim3(kThreads), sm, st, x, g, k, eps, inv_k, xq, s_x);
}

// Device error word of this library (bit 0: a token outside [0, vocab) reached
// the embedding kernel). Read and cleared by w8a8_error_flags().
__device__ unsigned int g_w8a8_errors;

// x = f32(q[tok]) * s[tok]  (llm/ref_model.py:221, hf_generic.QEmbedding :698-706);
// a token outside the table reads nothing: its row is zero and the error bit is set.
__global__ void embed_kernel(const int32_t* tokens, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
                             float* x) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    const int tok = tokens[m];
    if (tok < 0 || tok >= vocab) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)m * dim + i] = 0.f;
        if (threadIdx.x == 0) atomicOr(&g_w8a8_errors, 1u);
        return;
    }
    const float s = emb_s[tok];
    const int8_t* q = emb_q + (size_t)tok * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)m * dim + i] = fmul(i2f(q[i]), s);
}

cudaError_t launch_embed(const int32_t* tokens, int m, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
                         float* x, cudaStream_t st) {
    cudaFuncSetAttribute(embed_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(embed_kernel, dim3(m), dim3(256), 0, st, tokens, emb_q, emb_s, vocab, dim, x);
}

cudaError_t read_clear_errors(unsigned int* out) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_w8a8_errors, sizeof(unsigned int));
    if (e != cudaSuccess) return e;
    const unsigned int zero = 0;
    return cudaMemcpyToSymbol(g_w8a8_errors, &zero, sizeof(unsigned int));
}

// RMSNorm rows (llm/ref_model.py:204-207): ss = red_sum16(x*x),
// r = RSQRT(ss*F(1/n) + eps), y = (x*r)*g
__global__ void rmsnorm_kernel(const float* x, const float* g, int n, float eps, float inv_n, float* y) {
    pdl_wait();
    pdl_trigger();
    __shared__ float r;
    const int m = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (size_t)m * n;
    if (tid < 32) {
        float ss = red_sum16([&](int i) { float v = xr[i]; return fmul(v, v); }, n, tid);
        if (tid == 0) r = sfu_rsqrt(fadd(fmul(ss, inv_n), eps));
    }
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) y[(size_t)m * n + i] = fmul(fmul(xr[i], r), g[i]);
}

cudaError_t launch_rmsnorm(const float* x, const float* g, int m, int n, float eps, float inv_n, float* y,
                           cudaStream_t st) {
    return launch_k(rmsnorm_kernel, dim3(m), dim3(256), 0, st, x, g, n, eps, inv_n, y);
}

// quant_act rows (llm/ref_model.py:191-196)
__global__ void quant_act_kernel(const float* x, int k, int8_t* xq, float* s_x) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (size_t)m * k;
    float a = 0.f;
    for (int i = tid; i < k; i += blockDim.x) a = nanmax(a, fabsf(xr[i]));
    a = block_nanmax(a, red);
    const float s = fmul(a, W8A8_C127);
    const float inv = sfu_recip(s);
    for (int i = tid; i < k; i += blockDim.x) xq[(size_t)m * k + i] = (int8_t)to_i8(fmul(xr[i], inv));
    if (tid == 0) s_x[m] = s;
}

cudaError_t launch_quant_act(const float* x, int m, int k, int8_t* xq, float* s_x, cudaStream_t st) {
    return launch_k(quant_act_kernel, dim3(m), dim3(256), 0, st, x, k, xq, s_x);
}

// Greedy sampling (llm/runtime.py:55-57, np.argmax: the first maximum; a NaN
// wins as np.argmax's first NaN does).
struct ArgMax {
    float v;
    int i;
};

__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
    const bool an = a.v != a.v, bn = b.v != b.v;
    if (an || bn) {
        if (an && bn) return a.i < b.i ? a : b;
        return an ? a : b;
    }
    if (a.v > b.v) return a;
    if (b.v > a.v) return b;
    return a.i < b.i ? a : b;
}

__global__ void argmax_kernel(const float* logits, int n, int32_t* out) {
    pdl_wait();
    pdl_trigger();
    __shared__ ArgMax red[32];
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* row = logits + (size_t)m * n;
    ArgMax best{-INFINITY, n};
    for (int i = tid; i < n; i += blockDim.x) best = better(best, ArgMax{row[i], i});
    for (int o = 16; o > 0; o >>= 1) {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = better(best, other);
    }
    if (lane == 0) red[warp] = best;
    __syncthreads();
    if (warp == 0) {
        best = lane < (int)(blockDim.x >> 5) ? red[lane] : ArgMax{-INFINITY, n};
        for (int o = 16; o > 0; o >>= 1) {
            ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
            best = better(best, other);
        }
        if (lane == 0) out[m] = best.i < n ? best.i : 0;
    }
}

cudaError_t launch_argmax(const float* logits, int m, int n, int32_t* out, cudaStream_t st) {
    return launch_k(argmax_kernel, dim3(m), dim3(1024), 0, st, logits, n, out);
}

// func: 0 EXP, 1 RECIP, 2 RSQRT, 3 SiLU gate g*sigma(g) (u = 1)
__global__ void sfu_kernel(int func, const float* x, float* y, long long n) {
    pdl_wait();
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        y[i] = func == 0 ? sfu_exp(v) : func == 1 ? sfu_recip(v) : func == 2 ? sfu_rsqrt(v) : silu_gate(v, 1.f);
    }
}

cudaError_t launch_sfu(int func, const float* x, float* y, long long n, cudaStream_t st) {
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    return launch_k(sfu_kernel, dim3((int)blocks), dim3(256), 0, st, func, x, y, n);
}

// The on-device decode loop's step: the previous step's greedy token (the
// packed key of the fused classifier argmax) becomes this step's input, one
// position later; the key is cleared for the next classifier launch
// (llm/runtime.py:127-148 on the host).
__global__ void decode_advance_kernel(int32_t* tokens, int32_t* pos, unsigned long long* key, int32_t* next,
                                      int rows) {
    pdl_wait();
    pdl_trigger();
    const int m = threadIdx.x;
    if (m < rows) {
        const int t = (int)(0xFFFFFFFFu - (uint32_t)(key[m] & 0xFFFFFFFFull));
        tokens[m] = t;
        if (next != nullptr) next[m] = t;
        key[m] = 0ull;
        pos[m] += 1;
    }
}

cudaError_t launch_decode_advance(int32_t* tokens, int32_t* pos, unsigned long long* key, int32_t* next, int rows,
                                  cudaStream_t st) {
    cudaFuncSetAttribute(decode_advance_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(decode_advance_kernel, dim3(1), dim3(32), 0, st, tokens, pos, key, next, rows);
}

}  // namespace w8a8
