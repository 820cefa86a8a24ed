// Small kernels of the decode path: embedding dequant, RMSNorm, quant_act,
// greedy argmax, and elementwise SFU evaluation (the device functions exposed
// for testing).
#include "linear_common.cuh"
#include "pdl.cuh"
#include "tp.cuh"
#include "trace.cuh"

namespace w8a8 {

W8A8_TRACE_BINDER(trace_bind_misc)

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
                             float* x, uint32_t* epoch) {
    W8A8_TRACE_BEGIN(TR_EMBED);
    pdl_wait();
    W8A8_MARK(TR_EMBED, 1);
    pdl_trigger();
    const int m = blockIdx.x;
    if (epoch != nullptr && m == 0 && threadIdx.x == 0) *epoch += 1u;   // tensor parallel: a new step
    const int tok = tokens[m];
    if (tok < 0 || tok >= vocab) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)m * dim + i] = 0.f;
        if (threadIdx.x == 0) atomicOr(&g_w8a8_errors, 1u);
        return;
    }
    const float s = emb_s[tok];
    const int8_t* q = emb_q + (size_t)tok * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)m * dim + i] = fmul(i2f(q[i]), s);
    W8A8_MARK(TR_EMBED, 2);
}

cudaError_t launch_embed(const int32_t* tokens, int m, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
                         float* x, cudaStream_t st, uint32_t* epoch) {
    cudaFuncSetAttribute(embed_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(embed_kernel, dim3(m), dim3(256), 0, st, tokens, emb_q, emb_s, vocab, dim, x, epoch);
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
__global__ void sfu_kernel(int func, const float* x, float* y, long long n, float gelu_a, float gelu_b) {
    pdl_wait();
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        y[i] = func == 0   ? sfu_exp(v)
               : func == 1 ? sfu_recip(v)
               : func == 2 ? sfu_rsqrt(v)
               : func == 3 ? silu_gate(v, 1.f)
                           : gelu_gate(v, 1.f, gelu_a, gelu_b);
    }
}

cudaError_t launch_sfu(int func, const float* x, float* y, long long n, cudaStream_t st) {
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    return launch_k(sfu_kernel, dim3((int)blocks), dim3(256), 0, st, func, x, y, n, gelu_a_const(), gelu_b_const());
}

// The on-device decode loop's step: the previous step's greedy token (the
// packed key of the fused classifier argmax) becomes this step's input, one
// position later; the key is cleared for the next classifier launch
// (llm/runtime.py:127-148 on the host).
__global__ void decode_advance_kernel(int32_t* tokens, int32_t* pos, unsigned long long* key, int32_t* next,
                                      int rows) {
    W8A8_TRACE_BEGIN(TR_ADVANCE);
    pdl_wait();
    W8A8_MARK(TR_ADVANCE, 1);
    pdl_trigger();
    const int m = threadIdx.x;
    if (m < rows) {
        const int t = (int)(0xFFFFFFFFu - (uint32_t)(key[m] & 0xFFFFFFFFull));
        tokens[m] = t;
        if (next != nullptr) next[m] = t;
        key[m] = 0ull;
        pos[m] += 1;
    }
    W8A8_MARK(TR_ADVANCE, 2);
}

cudaError_t launch_decode_advance(int32_t* tokens, int32_t* pos, unsigned long long* key, int32_t* next, int rows,
                                  cudaStream_t st) {
    cudaFuncSetAttribute(decode_advance_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(decode_advance_kernel, dim3(1), dim3(32), 0, st, tokens, pos, key, next, rows);
}

// ---------------------------------------------------------------------------
// Tensor-parallel decode loop: the greedy token of the last step from every
// rank's classifier CTAs (keys of the global vocabulary index, so the maximum
// over all of them is the full row's np.argmax), then the next position. Every
// rank computes the same token. Bit 5 of the error word: a wait gave up.
__global__ void __launch_bounds__(256) tp_advance_kernel(TpCtx tp, const uint64_t* keys, int32_t* tokens,
                                                         int32_t* pos, int32_t* next, int rows) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t cnt[kTpMaxRanks + 1];
    __shared__ unsigned long long best[kTpRows];
    const int tid = threadIdx.x, nt = blockDim.x;
    const uint32_t ep = tp_epoch(tp);
    bool ok = true;
    if (tid < tp.ranks) {
        const uint32_t c = ll_wait(keys + 2 * ll_cta_idx(tid, -1, 0), ep, ok);
        cnt[tid] = c > (uint32_t)kTpCtas ? (uint32_t)kTpCtas : c;
    }
    if (tid < kTpRows) best[tid] = 0ull;
    __syncthreads();
    if (tid == 0) {
        uint32_t o = 0;
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q) {
            const uint32_t c = q < tp.ranks ? cnt[q] : 0u;
            cnt[q] = o;
            o += c;
        }
        cnt[kTpMaxRanks] = o;
    }
    __syncthreads();
    const int E = (int)cnt[kTpMaxRanks];
    for (int m = 0; m < rows && m < kTpRows; ++m) {
        auto addr = [&](int e) {
            int q = 0;
#pragma unroll
            for (int r = 1; r < kTpMaxRanks; ++r) q += (r < tp.ranks && e >= (int)cnt[r]) ? 1 : 0;
            return keys + 2 * ll_cta_idx(q, e - (int)cnt[q], m);
        };
        unsigned long long mx = 0ull;
        for (int e0 = tid; e0 < E; e0 += 8 * nt) {             // up to 8 entries' loads in flight
            uint32_t pending = 0u;
#pragma unroll
            for (int u = 0; u < 8; ++u) pending |= (e0 + u * nt < E) ? (1u << u) : 0u;
            for (int spins = 0; pending != 0u; ++spins) {
                uint64_t w0[8], w1[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (pending & (1u << u)) ll_load2(addr(e0 + u * nt), w0[u], w1[u]);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if ((pending & (1u << u)) && (uint32_t)(w0[u] >> 32) == ep && (uint32_t)(w1[u] >> 32) == ep) {
                        const unsigned long long k = ((unsigned long long)(uint32_t)w0[u] << 32) | (uint32_t)w1[u];
                        mx = k > mx ? k : mx;
                        pending &= ~(1u << u);
                    }
                }
                if (pending == 0u) break;
                if (!ok || spins >= kLlLimit) {
                    ok = false;
                    break;
                }
                if (spins >= kLlSpin) __nanosleep(128);
            }
        }
        if (mx != 0ull) atomicMax(&best[m], mx);
    }
    if (!ok) atomicOr(&g_w8a8_errors, 32u);
    __syncthreads();
    if (tid < rows && tid < kTpRows) {
        const int t = (int)(0xFFFFFFFFu - (uint32_t)(best[tid] & 0xFFFFFFFFull));
        tokens[tid] = t;
        if (next != nullptr) next[tid] = t;
        pos[tid] += 1;
    }
}

cudaError_t launch_tp_advance(const TpCtx& tp, const uint64_t* keys, int32_t* tokens, int32_t* pos, int32_t* next,
                              int rows, cudaStream_t st) {
    cudaFuncSetAttribute(tp_advance_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return launch_k(tp_advance_kernel, dim3(1), dim3(256), 0, st, tp, keys, tokens, pos, next, rows);
}

// Seed the tensor-parallel decode loop on this rank: the key block holds, for
// the current epoch, one entry (rank 0, CTA 0, row 0) whose key names `token`
// and no entries of the other ranks (as a single-GPU seed key, 0xFFFFFFFF -
// token).
__global__ void tp_seed_kernel(TpCtx tp, uint64_t* keys, int32_t token) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    const uint32_t ep = tp_epoch(tp);
    for (int q = 0; q < tp.ranks; ++q) ll_store(keys + 2 * ll_cta_idx(q, -1, 0), q == 0 ? 1u : 0u, ep);
    ll_store(keys + 2 * ll_cta_idx(0, 0, 0), 0u, ep);
    ll_store(keys + 2 * ll_cta_idx(0, 0, 0) + 1, 0xFFFFFFFFu - (uint32_t)token, ep);
}

cudaError_t launch_tp_seed(const TpCtx& tp, uint64_t* keys, int32_t token, cudaStream_t st) {
    return launch_k(tp_seed_kernel, dim3(1), dim3(32), 0, st, tp, keys, token);
}

// ---------------------------------------------------------------------------
// Tensor-parallel prefill pieces (rows beyond the decode GEMV; the exchange is
// a collective of the caller's): quant_act split in two, so that the row
// maxima of a column-split activation can be combined across ranks first.
// max|x| per row as float bits (NaN above every number, as nanmax keeps it).
__global__ void __launch_bounds__(kThreads) row_amax_kernel(const float* x, int k, uint32_t* amax) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float* xr = x + (size_t)m * k;
    float a = 0.f;
    for (int i = threadIdx.x; i < k; i += blockDim.x) a = nanmax(a, fabsf(xr[i]));
    a = block_nanmax(a, red);
    if (threadIdx.x == 0) amax[m] = __float_as_uint(a);
}

cudaError_t launch_row_amax(const float* x, int m, int k, uint32_t* amax, cudaStream_t st) {
    return launch_k(row_amax_kernel, dim3(m), dim3(kThreads), 0, st, x, k, amax);
}

// quant_act of x rows with a given max|x| (llm/ref_model.py:191-196 after the
// reduction): s = amax * F(1/127), xq = i8(x * RECIP(s)).
__global__ void __launch_bounds__(kThreads) quant_posted_kernel(const float* x, const uint32_t* amax, int k,
                                                                int8_t* xq, float* s_x) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    const float s = fmul(__uint_as_float(amax[m]), W8A8_C127);
    const float inv = sfu_recip(s);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m * k);
    char4* dst = reinterpret_cast<char4*>(xq + (size_t)m * k);
    for (int c = threadIdx.x; c < k / 4; c += blockDim.x) {
        const float4 v = xr[c];
        dst[c] = make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)), to_i8(fmul(v.w, inv)));
    }
    if (threadIdx.x == 0) s_x[m] = s;
}

cudaError_t launch_quant_posted(const float* x, const uint32_t* amax, int m, int k, int8_t* xq, float* s_x,
                                cudaStream_t st) {
    return launch_k(quant_posted_kernel, dim3(m), dim3(kThreads), 0, st, x, amax, k, xq, s_x);
}

// The W8A8 linear's epilogue on exact int32 sums (after an all-reduce of the
// row-split partials): y = resid + (f32(acc) * s_w) * s_x, or without resid.
__global__ void __launch_bounds__(kThreads) dequant_resid_kernel(const int32_t* acc, const float* s_x,
                                                                 const float* s_w, int n, const float* resid,
                                                                 float* y) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.y;
    const float sx = s_x[m];
    const size_t o = (size_t)m * n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = fmul(fmul(i2f(acc[o + i]), s_w[i]), sx);
        y[o + i] = resid != nullptr ? fadd(resid[o + i], v) : v;
    }
}

cudaError_t launch_dequant_resid(const int32_t* acc, const float* s_x, const float* s_w, int m, int n,
                                 const float* resid, float* y, cudaStream_t st) {
    const int bx = (n + kThreads - 1) / kThreads;
    return launch_k(dequant_resid_kernel, dim3(bx < 8 ? bx : 8, m), dim3(kThreads), 0, st, acc, s_x, s_w, n, resid,
                    y);
}

}  // namespace w8a8
