// W8A8 GEMV for decode rows (M <= 4): a persistent grid (one CTA per SM) that
// streams the weight matrix through shared memory with 1-D bulk copies
// (cp.async.bulk, completion on mbarriers), several tiles in flight per CTA.
//
// Weight tiles are independent of every earlier kernel, so each CTA issues its
// first tiles before griddepcontrol.wait: under programmatic dependent launch
// the weight stream of this layer overlaps the tail of the previous kernel.
// After the wait come the activation prologue (the same fused rmsnorm /
// quant_act as linear.cu) and the dot products from shared memory: a warp owns
// one tile row (or a K-slice of it for long rows), lanes read consecutive
// 16-byte chunks (no bank conflicts), dp4a per 4 bytes, shuffles sum the int32
// partials (exact in any order). Epilogues as linear.cu: dequant
// (f32(acc)*s_w)*s_x, + residual, SwiGLU with the row amax and the last CTA's
// int8 requant, or the classifier's fused greedy argmax.
// Reference semantics: llm/ref_model.py:191-202 (quant_act, linear),
// llm/sa_funcsim.py:138-162 (the GEMV command), llm/compile_model.py:295-328
// (ffn_up with fused SiLU).
#include "linear_common.cuh"
#include "pdl.cuh"

namespace w8a8 {

__device__ unsigned int g_gemv_errors;                        // bit 1: a tile wait gave up

constexpr int kMaxStages = 8;
constexpr size_t kRingBytes = 96 * 1024;                      // weight ring per CTA

// Row n is the j-th row of this CTA: its scales (and residuals) were staged in
// shared memory (sw, sw2: [rows of the CTA]; rs: [MR][rows of the CTA]).
template <int MR, int EPI>
__device__ __forceinline__ void epilogue_row(const LinearParams& p, int n, int j, int nj, const int* acc,
                                             const int* acc2, const float* sx, const float* sw, const float* sw2,
                                             const float* rs, uint32_t* bamax, unsigned long long* bkey) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        if (m >= p.m) continue;
        const size_t o = (size_t)m * p.n + n;
        const float v = fmul(fmul(i2f(acc[m]), sw[j]), sx[m]);
        if (EPI == EPI_STORE) {
            p.y[o] = v;
            if (p.acc != nullptr) p.acc[o] = acc[m];
            if (p.argmax_key != nullptr) atomicMax(&bkey[m], argmax_key(v, n));
        } else if (EPI == EPI_RESID) {
            p.y[o] = fadd(rs[m * nj + j], v);
        } else {
            const float u = fmul(fmul(i2f(acc2[m]), sw2[j]), sx[m]);
            const float h = silu_gate(v, u);
            p.y[o] = h;
            atomicMax(&bamax[m], __float_as_uint(fabsf(h)));
        }
    }
}

constexpr int kConsumers = kThreads;                          // 8 consumer warps
constexpr int kGemvThreads = kThreads + 32;                   // + 1 producer warp

template <int MR, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1)
    gemv_kernel(LinearParams p, int tr, int S, int stages, int ntiles) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr bool kTwo = EPI == EPI_SWIGLU;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool producer = warp == kWarps;
    const int k = p.k, nch = k / 16;
    const size_t tile_bytes = (size_t)tr * k;
    const size_t stage_bytes = tile_bytes * (kTwo ? 2 : 1);
    unsigned char* ring = smem;
    int8_t* xs = reinterpret_cast<int8_t*>(smem + stages * stage_bytes);   // [MR][k]
    float* xf = reinterpret_cast<float*>(xs + (size_t)MR * k);            // [k]
    const int nj = ((ntiles + (int)gridDim.x - 1) / (int)gridDim.x) * tr;   // rows of a CTA, at most
    float* sw = xf + (PRO == PRO_I8 ? 0 : k);                               // [nj] row scales
    float* sw2 = sw + nj;                                                   // [nj] (SwiGLU up rows)
    float* rs = sw2 + (kTwo ? nj : 0);                                      // [MR][nj] residual rows
    float* gs = rs + (EPI == EPI_RESID ? MR * nj : 0);                      // [k] RMSNorm gain
    __shared__ __align__(8) uint64_t full[kMaxStages];         // tile landed (bulk-copy bytes)
    __shared__ __align__(8) uint64_t empty[kMaxStages];        // the 8 consumer warps are done with it
    __shared__ float sx[MR];
    __shared__ float red[32];
    __shared__ uint32_t bamax[MR];
    __shared__ unsigned long long bkey[MR];
    __shared__ int last, failed;
    const int my = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // tiles of this CTA
    if (tid < MR) {
        bamax[tid] = 0u;
        bkey[tid] = 0ull;
    }
    if (tid == 0) {
        failed = 0;
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int i) {                                  // tile i of this CTA -> stage i % stages
        const int s = i % stages;
        const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * tr;
        const uint32_t bytes = (uint32_t)(min(tr, p.n - row0) * k);
        mbar_expect_tx(&full[s], bytes * (kTwo ? 2u : 1u));
        bulk_g2s(ring + s * stage_bytes, p.w + (size_t)row0 * k, bytes, &full[s]);
        if (kTwo) bulk_g2s(ring + s * stage_bytes + tile_bytes, p.w2 + (size_t)row0 * k, bytes, &full[s]);
    };
    const int first = min(stages, my);
    if (producer && lane == 0)
        for (int i = 0; i < first; ++i) issue(i);              // weights: before the wait
    // row j of this CTA = tile j / tr, row j % tr; its scales are constants too
    for (int j = tid; j < my * tr; j += kGemvThreads) {
        const int n = ((int)blockIdx.x + (j / tr) * (int)gridDim.x) * tr + j % tr;
        if (n < p.n) {
            sw[j] = __ldg(p.s_w + n);
            if (kTwo) sw2[j] = __ldg(p.s_w2 + n);
        }
    }
    if (PRO == PRO_RMSQ)                                       // the norm gain: a constant, staged now
        for (int c = tid; c < k; c += kGemvThreads) gs[c] = __ldg(p.norm_g + c);
    if (PRO != PRO_I8 && warp == 0) {                          // bring the RECIP / RSQRT table lines in
        uint32_t t = g_rec_t[lane * 2] ^ g_rec_s[lane * 2] ^ g_rsq_t[lane * 4] ^ g_rsq_s[lane * 4];
        t = __reduce_xor_sync(0xffffffffu, t);
        if (lane == 0) red[31] = __uint_as_float(t);          // (kept: red is rewritten by the prologue)
    }
    pdl_wait();
    pdl_trigger();
    if (EPI == EPI_RESID) {                                    // residual rows: written by earlier kernels
        for (int j = tid; j < my * tr * MR; j += kGemvThreads) {
            const int m = j / (my * tr), jj = j % (my * tr);
            const int n = ((int)blockIdx.x + (jj / tr) * (int)gridDim.x) * tr + jj % tr;
            if (n < p.n && m < p.m) rs[m * nj + jj] = p.resid[(size_t)m * p.n + n];
        }
    }
    prologue<MR, PRO>(p, xs, xf, sx, red, gs);

    if (producer) {
        if (lane == 0) {                                       // refill each stage once its consumers are done
            for (int i = first; i < my; ++i) {
                const int s = i % stages;
                if (!mbar_wait(&empty[s], (uint32_t)(((i / stages) - 1) & 1))) {
                    atomicOr(&g_gemv_errors, 2u);
                    failed = 1;
                    break;
                }
                issue(i);
            }
        }
    } else {
        // Consumer thread t owns row r = t / S of a tile and K-slice s = t % S
        // (S <= 32 threads per row, within one warp): chunks s, s + S, ... of 16
        // bytes; lanes read consecutive chunks (conflict-free); the row is summed
        // with shuffles. A warp releases the stage before its epilogue.
        const int r = tid / S, sl = tid % S;
        for (int i = 0; i < my; ++i) {
            const int s = i % stages;
            if (!mbar_wait(&full[s], (uint32_t)((i / stages) & 1))) {
                atomicOr(&g_gemv_errors, 2u);
                failed = 1;
                break;
            }
            const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * tr;
            const int rows = min(tr, p.n - row0);
            const int8_t* wr = reinterpret_cast<const int8_t*>(ring + s * stage_bytes) + (size_t)r * k;
            const int8_t* wr2 = wr + tile_bytes;
            int acc[MR], acc2[MR];
#pragma unroll
            for (int m = 0; m < MR; ++m) acc[m] = acc2[m] = 0;
            if (r < rows) {
#pragma unroll 4
                for (int c = sl; c < nch; c += S) {
                    const int4 w4 = *reinterpret_cast<const int4*>(wr + c * 16);
                    int4 u4;
                    if (kTwo) u4 = *reinterpret_cast<const int4*>(wr2 + c * 16);
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        const int4 x4 = *reinterpret_cast<const int4*>(xs + (size_t)m * k + c * 16);
                        acc[m] = dp4a(w4.w, x4.w, dp4a(w4.z, x4.z, dp4a(w4.y, x4.y, dp4a(w4.x, x4.x, acc[m]))));
                        if (kTwo)
                            acc2[m] = dp4a(u4.w, x4.w, dp4a(u4.z, x4.z, dp4a(u4.y, x4.y, dp4a(u4.x, x4.x, acc2[m]))));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                for (int o = S / 2; o > 0; o >>= 1) {
                    acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                    if (kTwo) acc2[m] += __shfl_xor_sync(0xffffffffu, acc2[m], o);
                }
            }
            if (sl == 0 && r < rows)
                epilogue_row<MR, EPI>(p, row0 + r, i * tr + r, nj, acc, acc2, sx, sw, sw2, rs, bamax, bkey);
        }
    }
    __syncthreads();
    if (failed) {                                              // a wait gave up: drain what is in flight, stop
        if (producer && lane == 0)
            for (int s = 0; s < stages; ++s) mbar_wait(&full[s], 0u), mbar_wait(&full[s], 1u);
        __syncthreads();
        return;
    }
    if (EPI == EPI_STORE && p.argmax_key != nullptr) {
        if (tid < p.m && tid < MR) atomicMax(p.argmax_key + tid, bkey[tid]);
    }
    if (EPI != EPI_SWIGLU || p.hq == nullptr) return;
    // the row amax across the grid; the last CTA requantizes h (quant_act)
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
        const float4* hr = reinterpret_cast<const float4*>(p.y + (size_t)m * p.n);
        char4* qr = reinterpret_cast<char4*>(p.hq + (size_t)m * p.n);
        const int n4 = p.n / 4;
        for (int j0 = tid; j0 < n4; j0 += 4 * kGemvThreads) {   // four independent loads in flight
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + u * kGemvThreads;
                if (j < n4) v[u] = __ldcg(hr + j);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + u * kGemvThreads;
                if (j < n4)
                    qr[j] = make_char4(to_i8(fmul(v[u].x, inv)), to_i8(fmul(v[u].y, inv)), to_i8(fmul(v[u].z, inv)),
                                       to_i8(fmul(v[u].w, inv)));
            }
        }
        if (tid == 0) p.s_h[m] = s;
    }
    __syncthreads();
    if (tid < p.m) p.amax_bits[tid] = 0u;
    if (tid == 0) *p.counter = 0u;
}

static int sm_count() {
    static int cached[64] = {0};
    int d = 0;
    cudaGetDevice(&d);
    if (d < 0 || d >= 64) d = 0;
    if (cached[d] == 0) cudaDeviceGetAttribute(&cached[d], cudaDevAttrMultiProcessorCount, d);
    return cached[d] > 0 ? cached[d] : 148;
}

struct Tiling {
    int tr, slices, stages, ntiles, grid;
    size_t smem;
};

// tile rows: about 16 KB per matrix (power of two, at most 64 rows); warps
// split a row's K when a tile has fewer than 8 rows; a 64 KB ring of stages.
static Tiling tiling(const LinearParams& p, int mr, int pro, int epi) {
    Tiling t{};
    int tr = 16384 / p.k;                                      // ~16 KB per matrix, at least 8 rows
    tr = tr < kWarps ? kWarps : (tr > kConsumers ? kConsumers : tr);
    int pw = 1;
    while (pw * 2 <= tr) pw *= 2;
    t.tr = pw;
    t.slices = kConsumers / t.tr;                              // consumer threads per row, at most 32
    const size_t stage = (size_t)t.tr * p.k * (epi == EPI_SWIGLU ? 2 : 1);
    size_t st = kRingBytes / stage;
    t.stages = (int)(st < 2 ? 2 : (st > (size_t)kMaxStages ? kMaxStages : st));
    t.ntiles = (p.n + t.tr - 1) / t.tr;
    t.grid = t.ntiles < sm_count() ? t.ntiles : sm_count();
    const size_t nj = (size_t)((t.ntiles + t.grid - 1) / t.grid) * t.tr;   // rows of a CTA, at most
    t.smem = (size_t)t.stages * stage + (size_t)mr * p.k + (pro == PRO_I8 ? 0 : (size_t)p.k * 4) +
             nj * 4 * ((epi == EPI_SWIGLU ? 2 : 1) + (epi == EPI_RESID ? mr : 0)) +
             (pro == PRO_RMSQ ? (size_t)p.k * 4 : 0);
    return t;
}

template <int MR, int PRO, int EPI>
static cudaError_t launch_g(const LinearParams& p, cudaStream_t st) {
    const Tiling t = tiling(p, MR, PRO, EPI);
    auto kern = gemv_kernel<MR, PRO, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)t.smem);
    if (e != cudaSuccess) return e;
    // one shared-memory carveout for every kernel of the chain: no L1 / shared
    // reconfiguration of an SM between consecutive kernels
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return launch_k(kern, dim3(t.grid), dim3(kGemvThreads), t.smem, st, p, t.tr, t.slices, t.stages, t.ntiles);
}

template <int PRO, int EPI>
static cudaError_t launch_gm(const LinearParams& p, cudaStream_t st) {
    if (p.m <= 1) return launch_g<1, PRO, EPI>(p, st);
    if (p.m <= 2) return launch_g<2, PRO, EPI>(p, st);
    return launch_g<4, PRO, EPI>(p, st);
}

bool gemv_fits(const LinearParams& p, int pro, int epi) {
    if (p.m > 4) return false;
    const int mr = p.m <= 1 ? 1 : (p.m <= 2 ? 2 : 4);
    return tiling(p, mr, pro, epi).smem <= 200 * 1024;
}

cudaError_t launch_gemv(const LinearParams& p, int pro, int epi, cudaStream_t st) {
    if (pro == PRO_I8 && epi == EPI_STORE) return launch_gm<PRO_I8, EPI_STORE>(p, st);
    if (pro == PRO_I8 && epi == EPI_RESID) return launch_gm<PRO_I8, EPI_RESID>(p, st);
    if (pro == PRO_QUANT && epi == EPI_STORE) return launch_gm<PRO_QUANT, EPI_STORE>(p, st);
    if (pro == PRO_QUANT && epi == EPI_RESID) return launch_gm<PRO_QUANT, EPI_RESID>(p, st);
    if (pro == PRO_RMSQ && epi == EPI_STORE) return launch_gm<PRO_RMSQ, EPI_STORE>(p, st);
    if (pro == PRO_RMSQ && epi == EPI_SWIGLU) return launch_gm<PRO_RMSQ, EPI_SWIGLU>(p, st);
    return cudaErrorInvalidValue;
}

unsigned int gemv_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_gemv_errors, sizeof(v));
    cudaMemcpyToSymbol(g_gemv_errors, &zero, sizeof(zero));
    return v;
}

}  // namespace w8a8
