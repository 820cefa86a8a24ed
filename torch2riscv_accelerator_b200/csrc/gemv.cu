// W8A8 GEMV for decode rows (M <= 4): a persistent grid (one CTA per SM) that
// streams the weight matrix through shared memory with 1-D bulk copies
// (cp.async.bulk, completion on mbarriers), several tiles in flight per CTA.
//
// Weight tiles are independent of every earlier kernel, so each CTA issues its
// first tiles before griddepcontrol.wait: under programmatic dependent launch
// the weight stream of this layer overlaps the tail of the previous kernel.
// After the wait come the activation prologue (fused rmsnorm / quant_act) and
// the dot products from shared memory: consumer thread t owns row t / S of a
// tile and a K-slice of it, dp4a per 4 bytes, shuffles sum the int32 partials
// (exact in any order). Epilogues: dequant (f32(acc)*s_w)*s_x, + residual,
// SwiGLU with the row amax and the last CTA's int8 requant, or the
// classifier's fused greedy argmax.
//
// Code size is part of the design. A decode step runs a chain of short
// kernels; the code a kernel runs once per launch (everything after the wait
// but the dot-product loop) is fetched cold at every launch (an SM's
// instruction caches do not keep it from one launch to the next), at about 10
// cycles per instruction from L2 against 1.5-4.5 from the SM's own caches. So
// only the dot-product loop is unrolled, and the decode chain's three
// prologue / epilogue pairs are compiled in (no run-time kind switches on its
// path); other uses take the kinds at run time.
//
// Reference semantics: llm/ref_model.py:191-202 (quant_act, linear),
// :204-207 (rmsnorm), llm/sa_funcsim.py:138-162 (the GEMV command),
// llm/compile_model.py:295-328 (ffn_up with fused SiLU).
#include "linear_common.cuh"
#include "pdl.cuh"
#include "tp.cuh"
#include "trace.cuh"

namespace w8a8 {

W8A8_TRACE_BINDER(trace_bind_gemv)

__device__ unsigned int g_gemv_errors;    // bit 1: a tile wait gave up; bit 5: a tensor-parallel exchange wait

constexpr int kMaxStages = 8;
constexpr size_t kRingBytes = 96 * 1024;                      // weight ring per CTA
constexpr size_t kStreamRingBytes = 96 * 1024;                // ... for a GEMV of many tiles per CTA
constexpr int kStreamCtasPerSm = 2;                           // streaming: two CTAs per SM hide more latency
constexpr size_t kWideRingBytes = 160 * 1024;                 // ... but rows of >= 2 KB: one CTA, a deeper ring
constexpr size_t kStreamBytes = (size_t)64 << 20;             // weights from which a GEMV counts as streaming
constexpr size_t kGemvSmemMax = 200 * 1024;                   // dynamic shared memory of a launch, at most
constexpr int kConsumers = kThreads;                          // 8 consumer warps
constexpr int kGemvThreads = kThreads + 32;                   // + 1 producer warp

struct GemvCfg {
    int pro, epi;             // Prologue / Epilogue kinds
    int tr, S, ls, lt;        // tile rows (tr = 1 << lt); consumer threads per row (S = 1 << ls)
    int stages, ntiles;
};

// Ordered sum of squares over D = 16 lanes (llm/ref_model.py:179-186): lane
// l < 16 adds x[l]^2, x[l + 16]^2, ... in order, 8 loads ahead of the adds;
// then the pairwise tree. Whole warp; the sum on every lane.
__device__ __forceinline__ float sumsq16(const float* xf, int k, int lane) {
    float acc = 0.f;
    if (lane < kLanes) {
        const int groups = k / kLanes;                        // k is a multiple of 16
        int g = 0;
#pragma unroll 1
        for (; g + 8 <= groups; g += 8) {
            float t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) t[j] = xf[(g + j) * kLanes + lane];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fadd(acc, fmul(t[j], t[j]));
        }
#pragma unroll 1
        for (; g < groups; ++g) {
            const float t = xf[g * kLanes + lane];
            acc = fadd(acc, fmul(t, t));
        }
    }
#pragma unroll
    for (int s = 1; s < kLanes; s <<= 1) {
        const float o = __shfl_down_sync(0xffffffffu, acc, s);
        if ((lane & (2 * s - 1)) == 0) acc = fadd(acc, o);
    }
    return __shfl_sync(0xffffffffu, acc, 0);
}

// Activation prologue: rows m < MR of x -> int8 rows xs [MR][k] and scales
// sx [MR] (zero rows beyond p.m). xf: fp32 staging [k]; gs: the RMSNorm gain
// in shared memory. Every thread of the block takes part.
template <int MR, bool TP>
__device__ __forceinline__ void gemv_prologue(const LinearParams& p, int pro, int8_t* xs, float* xf, float* sx,
                                              const float* gs, float* red, float* bc, uint32_t ep, bool& ok,
                                              uint32_t* cnt, const SfuSmem* sf) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, k = p.k, nt = (int)blockDim.x;
    if (pro == PRO_I8) {
#pragma unroll 1
        for (int m = 0; m < MR; ++m) {
            int4* dst = reinterpret_cast<int4*>(xs + (size_t)m * k);
            const int4* src = reinterpret_cast<const int4*>(p.xq + (size_t)m * k);
#pragma unroll 1
            for (int c = tid; c < k / 16; c += nt) dst[c] = m < p.m ? __ldcg(src + c) : make_int4(0, 0, 0, 0);
        }
        if (tid < MR) sx[tid] = tid < p.m ? __ldcg(p.s_x + tid) : 0.f;
        __syncthreads();
        return;
    }
    float4* xf4 = reinterpret_cast<float4*>(xf);
    const float4* g4 = reinterpret_cast<const float4*>(gs);
#pragma unroll 1
    for (int m = 0; m < MR; ++m) {
        char4* dst = reinterpret_cast<char4*>(xs + (size_t)m * k);
        if (m >= p.m) {
#pragma unroll 1
            for (int c = tid; c < k / 4; c += nt) dst[c] = make_char4(0, 0, 0, 0);
            if (tid == 0) sx[m] = 0.f;
            continue;
        }
        const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)m * k);
        const bool posted = pro == PRO_QUANT && (p.amax_in != nullptr || (TP && p.amax_ll != nullptr));
        uint32_t pa = pro == PRO_QUANT && p.amax_in != nullptr ? __ldcg(p.amax_in + m) : 0u;   // with the x loads
        if (TP && p.part_in != nullptr) {
            // tensor parallel: the row-split linear before this one left its int32
            // partials at every rank; x = resid + (f32(sum) * s_w) * s_x (its
            // epilogue, with the exact sum), kept by CTA 0 as the residual stream
            const float sxp = __ldcg(p.part_sx + m);
            float2* xf2 = reinterpret_cast<float2*>(xf);
            const float2* rr = reinterpret_cast<const float2*>(p.part_resid + (size_t)m * k);
            const float2* pw = reinterpret_cast<const float2*>(p.part_sw);
            float2* xo = reinterpret_cast<float2*>(p.x_out + (size_t)m * k);
#pragma unroll 1
            for (int c = tid; c < k / 2; c += nt) {
                const float2 r = __ldcg(rr + c), w = __ldg(pw + c);
                int s0, s1;
                ll_sum_pair(p.tp, p.part_in, m, k, 2 * c, ep, ok, s0, s1);
                const float2 v = make_float2(fadd(r.x, fmul(fmul(i2f(s0), w.x), sxp)),
                                             fadd(r.y, fmul(fmul(i2f(s1), w.y), sxp)));
                xf2[c] = v;
                if (blockIdx.x == 0) xo[c] = v;
            }
        } else {
#pragma unroll 4
            for (int c = tid; c < k / 4; c += nt) xf4[c] = __ldcg(xr + c);  // loads batched: 1-3 per thread
        }
        if (TP && pro == PRO_QUANT && p.amax_ll != nullptr)        // every rank's max|x| (its producer CTAs)
            pa = ll_block_max(p.tp, p.amax_ll, m, ep, ok, cnt, reinterpret_cast<uint32_t*>(red));
        __syncthreads();
        W8A8_MARK(TR_GEMV, 6);
        float r = 1.f;
        if (pro == PRO_RMSQ) {
            if (warp == 0) {
                const float ss = sumsq16(xf, k, lane);
                if (lane == 0) bc[0] = sfu_rsqrt_s(fadd(fmul(ss, p.inv_k), p.eps), sf);
            }
            __syncthreads();
            r = bc[0];
            W8A8_MARK(TR_GEMV, 7);
        }
        // y = (x * r) * g in place, and the row amax (unless the producer posted it).
        // This loop and the int8 one below run once or a few times per thread
        // from shared memory: not unrolled (their code is fetched cold each launch)
        float a = 0.f;
#pragma unroll 1
        for (int c = posted ? k / 4 : tid; c < k / 4; c += nt) {
            float4 v = xf4[c];
            if (pro == PRO_RMSQ) {
                const float4 g = g4[c];
                v = make_float4(fmul(fmul(v.x, r), g.x), fmul(fmul(v.y, r), g.y), fmul(fmul(v.z, r), g.z),
                                fmul(fmul(v.w, r), g.w));
                xf4[c] = v;
            }
            a = nanmax(a, nanmax(nanmax(fabsf(v.x), fabsf(v.y)), nanmax(fabsf(v.z), fabsf(v.w))));
        }
        if (posted) a = __uint_as_float(pa);
        else a = block_nanmax(a, red);
        W8A8_MARK(TR_GEMV, 8);
        const float s = fmul(a, W8A8_C127);
        const float inv = sfu_recip_s(s, sf);
        W8A8_MARK(TR_GEMV, 9);
#pragma unroll 1
        for (int c = tid; c < k / 4; c += nt) {
            const float4 v = xf4[c];
            dst[c] = make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)),
                                to_i8(fmul(v.w, inv)));
        }
        if (tid == 0) {
            sx[m] = s;
            if (p.s_x_out != nullptr && blockIdx.x == 0) p.s_x_out[m] = s;
        }
        __syncthreads();                                       // xf free for the next row
    }
}

// Dot products of one row slice of a tile: 16-byte chunks c = sl, sl + S, ...
// of the row (TWO: the gate and up rows), two independent dp4a chains.
template <int MR, bool TWO>
__device__ __forceinline__ void tile_dots(const int8_t* wr, const int8_t* wr2, const int8_t* xs, int k, int nch,
                                          int sl, int S, int* acc, int* acc2) {
    int a0[MR], a1[MR], b0[MR], b1[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) a0[m] = a1[m] = b0[m] = b1[m] = 0;
    const int4 z = make_int4(0, 0, 0, 0);
#pragma unroll 2
    for (int c = sl; c < nch; c += 2 * S) {
        const bool hi = c + S < nch;
        const int4 w0 = *reinterpret_cast<const int4*>(wr + c * 16);
        const int4 w1 = hi ? *reinterpret_cast<const int4*>(wr + (c + S) * 16) : z;
        int4 u0 = z, u1 = z;
        if (TWO) {
            u0 = *reinterpret_cast<const int4*>(wr2 + c * 16);
            u1 = hi ? *reinterpret_cast<const int4*>(wr2 + (c + S) * 16) : z;
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            const int4 x0 = *reinterpret_cast<const int4*>(xs + (size_t)m * k + c * 16);
            const int4 x1 = hi ? *reinterpret_cast<const int4*>(xs + (size_t)m * k + (c + S) * 16) : z;
            a0[m] = dp4a(w0.w, x0.w, dp4a(w0.z, x0.z, dp4a(w0.y, x0.y, dp4a(w0.x, x0.x, a0[m]))));
            a1[m] = dp4a(w1.w, x1.w, dp4a(w1.z, x1.z, dp4a(w1.y, x1.y, dp4a(w1.x, x1.x, a1[m]))));
            if (TWO) {
                b0[m] = dp4a(u0.w, x0.w, dp4a(u0.z, x0.z, dp4a(u0.y, x0.y, dp4a(u0.x, x0.x, b0[m]))));
                b1[m] = dp4a(u1.w, x1.w, dp4a(u1.z, x1.z, dp4a(u1.y, x1.y, dp4a(u1.x, x1.x, b1[m]))));
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {                             // int32 sums: exact in any order
        acc[m] = a0[m] + a1[m];
        acc2[m] = b0[m] + b1[m];
    }
}

// The last CTA of a SwiGLU launch: h -> int8 rows with the grid-wide amax.
__device__ __forceinline__ void swiglu_requant(const LinearParams& p, const SfuSmem* sf) {
    const int tid = threadIdx.x;
    __threadfence();
#pragma unroll 1
    for (int m = 0; m < p.m; ++m) {
        const float amax = __uint_as_float(__ldcg(p.amax_bits + m));
        const float s = fmul(amax, W8A8_C127);
        const float inv = sfu_recip_s(s, sf);
        const float4* hr = reinterpret_cast<const float4*>(p.y + (size_t)m * p.n);
        char4* qr = reinterpret_cast<char4*>(p.hq + (size_t)m * p.n);
        const int n4 = p.n / 4;
#pragma unroll 1
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

// TP: the tensor-parallel exchanges (a separate instantiation: the one-GPU
// kernel keeps its code size and registers). PRO / EPI >= 0: the prologue /
// epilogue kind fixed at compile time (the decode chain's three pairs), -1:
// taken from cf at run time.
template <int MR, bool TP, int PRO = -1, int EPI = -1>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(LinearParams p, GemvCfg cf) {
    extern __shared__ __align__(128) unsigned char smem[];
    W8A8_TRACE_BEGIN(TR_GEMV);
    const int pro = PRO >= 0 ? PRO : cf.pro, epi = EPI >= 0 ? EPI : cf.epi;
    const int tr = cf.tr, S = cf.S, stages = cf.stages, ntiles = cf.ntiles;
    const bool two = epi == EPI_SWIGLU;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool producer = warp == kWarps;
    const int k = p.k, nch = k / 16;
    const size_t tile_bytes = (size_t)tr * k;
    const size_t stage_bytes = tile_bytes * (two ? 2 : 1);
    const int my = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // tiles of this CTA
    const int nj = ((ntiles + (int)gridDim.x - 1) / (int)gridDim.x) * tr;              // rows of a CTA, at most
    unsigned char* ring = smem;
    int8_t* xs = reinterpret_cast<int8_t*>(smem + stages * stage_bytes);   // [MR][k]
    float* xf = reinterpret_cast<float*>(xs + (size_t)MR * k);            // [k] (fp32 prologues)
    float* sw = xf + (pro == PRO_I8 ? 0 : k);                               // [nj] row scales
    float* sw2 = sw + nj;                                                   // [nj] (SwiGLU up rows)
    float* rs = sw2 + (two ? nj : 0);                                       // [MR][nj] residual rows
    float* gs = rs + (epi == EPI_RESID ? MR * nj : 0);                      // [k] RMSNorm gain
    __shared__ __align__(8) uint64_t full[kMaxStages];         // tile landed (bulk-copy bytes)
    __shared__ __align__(8) uint64_t empty[kMaxStages];        // the 8 consumer warps are done with it
    __shared__ float sx[MR];
    __shared__ float red[32];
    __shared__ float bc[2];
    __shared__ uint32_t bamax[MR];
    __shared__ unsigned long long bkey[MR];
    __shared__ int last, failed;
    __shared__ uint32_t llcnt[kTpMaxRanks + 1];
    __shared__ __align__(16) uint32_t silu_tab[256];           // EXP / RECIP tables (SwiGLU epilogue)
    __shared__ SfuSmem sfs;                                    // RECIP / RSQRT (prologue, requant)
    if (tid < MR) {
        bamax[tid] = 0u;
        bkey[tid] = 0ull;
    }
    if (tid == 0) {
        failed = 0;
#pragma unroll 1
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int i, int s) {                           // tile i of this CTA -> stage s = i % stages
        const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * tr;
        const uint32_t bytes = (uint32_t)(min(tr, p.n - row0) * k);
        mbar_expect_tx(&full[s], bytes * (two ? 2u : 1u));
        bulk_g2s(ring + s * stage_bytes, p.w + (size_t)row0 * k, bytes, &full[s]);
        if (two) bulk_g2s(ring + s * stage_bytes + tile_bytes, p.w2 + (size_t)row0 * k, bytes, &full[s]);
    };
    const int first = min(stages, my);
    if (producer && lane == 0) {
#pragma unroll 1
        for (int i = 0; i < first; ++i) issue(i, i);          // weights: before the wait
    }
    // Constants, staged now. Each thread issues all its loads before its first
    // store (a store waits for its load: one memory latency per batch, not per
    // element). Row j of this CTA = tile j / tr, row j % tr.
#pragma unroll 1
    for (int j0 = tid; j0 < my * tr; j0 += 2 * kGemvThreads) {
        float a[2], b[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = j0 + u * kGemvThreads;
            const int n = ((int)blockIdx.x + (j >> cf.lt) * (int)gridDim.x) * tr + (j & (tr - 1));
            const bool v = j < my * tr && n < p.n;
            a[u] = v ? __ldg(p.s_w + n) : 0.f;
            b[u] = v && two ? __ldg(p.s_w2 + n) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = j0 + u * kGemvThreads;
            if (j < my * tr) {
                sw[j] = a[u];
                if (two) sw2[j] = b[u];
            }
        }
    }
    if (two) stage_silu_tables(silu_tab);
    if (pro == PRO_RMSQ) {                                     // the norm gain
#pragma unroll 1
        for (int c0 = tid; c0 < k; c0 += 4 * kGemvThreads) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + u * kGemvThreads;
                v[u] = c < k ? __ldg(p.norm_g + c) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + u * kGemvThreads < k) gs[c0 + u * kGemvThreads] = v[u];
        }
    }
    if (pro != PRO_I8 || two) stage_sfu(&sfs);               // (read after later barriers)
    W8A8_MARK(TR_GEMV, 12);
    pdl_wait();
    W8A8_MARK(TR_GEMV, 1);
    pdl_trigger();
    if (p.clear != nullptr && blockIdx.x == 0 && tid < p.clear_n) p.clear[tid] = 0u;   // its readers are done
    if (epi == EPI_RESID) {                                    // residual rows: written by earlier kernels
#pragma unroll 4
        for (int j = tid; j < my * tr * MR; j += kGemvThreads) {
            const int m = MR == 1 ? 0 : j / (my * tr), jj = MR == 1 ? j : j % (my * tr);
            const int n = ((int)blockIdx.x + (jj >> cf.lt) * (int)gridDim.x) * tr + (jj & (tr - 1));
            if (n < p.n && m < p.m) rs[m * nj + jj] = __ldcg(p.resid + (size_t)m * p.n + n);
        }
    }
    const uint32_t ep = TP ? tp_epoch(p.tp) : 0u;             // this step's exchange words
    bool ok = true;
    gemv_prologue<MR, TP>(p, pro, xs, xf, sx, gs, red, bc, ep, ok, llcnt, &sfs);   // ends with a block barrier
    if (TP && !ok) atomicOr(&g_gemv_errors, 32u);
    W8A8_MARK(TR_GEMV, 2);

    if (producer) {
        if (lane == 0) {                                       // refill each stage once its consumers are done
            int s = 0, ph = 0;                                 // tile i -> stage s, reuse phase ph
#pragma unroll 1
            for (int i = first; i < my; ++i) {
                if (!mbar_wait(&empty[s], (uint32_t)ph)) {
                    atomicOr(&g_gemv_errors, 2u);
                    failed = 1;
                    break;
                }
                issue(i, s);
                if (++s == stages) s = 0, ph ^= 1;
            }
        }
    } else {
        // Consumer thread t owns row r = t / S of a tile and K-slice s = t % S
        // (S <= 32 threads per row, within one warp); the row is summed with
        // shuffles. A warp releases the stage before its epilogue. The argmax
        // key and the SwiGLU row amax are kept per thread and merged at the end.
        const int r = tid >> cf.ls, sl = tid & (S - 1);
        uint32_t tamax[MR];
        unsigned long long tkey[MR];
#pragma unroll
        for (int m = 0; m < MR; ++m) tamax[m] = 0u, tkey[m] = 0ull;
        int s = 0, ph = 0;                                     // tile i -> stage s, fill phase ph
#pragma unroll 1
        for (int i = 0; i < my; ++i, (++s == stages ? (s = 0, ph ^= 1) : 0)) {
            if (!mbar_wait_spin(&full[s], (uint32_t)ph)) {      // a spin: a suspended wait wakes late
                atomicOr(&g_gemv_errors, 2u);
                failed = 1;
                break;
            }
            if (i == 0) W8A8_MARK(TR_GEMV, 10);
            const int row0 = ((int)blockIdx.x + i * (int)gridDim.x) * tr;
            const int rows = min(tr, p.n - row0);
            const int8_t* wr = reinterpret_cast<const int8_t*>(ring + s * stage_bytes) + (size_t)r * k;
            int acc[MR], acc2[MR];
#pragma unroll
            for (int m = 0; m < MR; ++m) acc[m] = acc2[m] = 0;
            if (r < rows) {
                if (two) tile_dots<MR, true>(wr, wr + tile_bytes, xs, k, nch, sl, S, acc, acc2);
                else tile_dots<MR, false>(wr, nullptr, xs, k, nch, sl, S, acc, acc2);
            }
            __syncwarp();
            if (i == 0) W8A8_MARK(TR_GEMV, 11);
            if (lane == 0 && i + stages < my) mbar_arrive(&empty[s]);   // only a stage that is refilled
#pragma unroll
            for (int m = 0; m < MR; ++m) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {             // S <= 32: the levels below S
                    if (o < S) {
                        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                        if (two) acc2[m] += __shfl_xor_sync(0xffffffffu, acc2[m], o);
                    }
                }
            }
            if (sl == 0 && r < rows) {
                const int n = row0 + r, j = i * tr + r;
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    if (m >= p.m) continue;
                    const size_t o = (size_t)m * p.n + n;
                    const float v = fmul(fmul(i2f(acc[m]), sw[j]), sx[m]);
                    if (epi == EPI_STORE) {
                        p.y[o] = v;
                        if (p.acc != nullptr) p.acc[o] = acc[m];
                        if (p.argmax_key != nullptr || (TP && p.key_out != nullptr)) {
                            const unsigned long long key = argmax_key(v, TP ? n + p.n_offset : n);
                            tkey[m] = key > tkey[m] ? key : tkey[m];
                        }
                    } else if (epi == EPI_RESID) {
                        p.y[o] = fadd(rs[m * nj + j], v);
                    } else if (TP && epi == EPI_PARTIAL) {     // the int32 sum to every rank
                        const size_t w = (size_t)(p.tp.rank * kTpRows + m) * p.n + n;
#pragma unroll
                        for (int q = 0; q < kTpMaxRanks; ++q)
                            if (q < p.tp.ranks) ll_store(tp_at(p.tp, p.part_out, q) + w, (uint32_t)acc[m], ep);
                    } else {
                        const float u = fmul(fmul(i2f(acc2[m]), sw2[j]), sx[m]);
                        const float h = gate_tab(v, u, silu_tab, GateAct{p.act, p.act_a, p.act_b});
                        p.y[o] = h;
                        tamax[m] = max(tamax[m], __float_as_uint(fabsf(h)));   // as bits: NaN above numbers
                    }
                }
            }
        }
        if (sl == 0) {                                         // merge the per-thread maxima
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                if (tkey[m] != 0ull) atomicMax(&bkey[m], tkey[m]);
                if (tamax[m] != 0u) atomicMax(&bamax[m], tamax[m]);
            }
        }
    }
    W8A8_MARK(TR_GEMV, 3);
    __syncthreads();
    if (failed) {                                              // a wait gave up: drain what is in flight, stop
        if (producer && lane == 0) {
#pragma unroll 1
            for (int s = 0; s < stages; ++s) mbar_wait(&full[s], 0u), mbar_wait(&full[s], 1u);
        }
        __syncthreads();
        return;
    }
    if (epi == EPI_STORE && p.argmax_key != nullptr) {
        if (tid < p.m && tid < MR) atomicMax(p.argmax_key + tid, bkey[tid]);
    }
    if (epi == EPI_SWIGLU && p.amax_out != nullptr) {         // max|h| for the next kernel's prologue
        if (tid < p.m && tid < MR && bamax[tid] != 0u) atomicMax(p.amax_out + tid, bamax[tid]);
    }
    if (TP && tid < kTpRows) {                                 // this CTA's row maxima / keys to every rank
        const int m = tid;
        if (epi == EPI_SWIGLU && p.amax_ll_out != nullptr)
            ll_post_cta(p.tp, p.amax_ll_out, blockIdx.x, gridDim.x, m, m < p.m && m < MR ? bamax[m] : 0u, ep);
        if (epi == EPI_STORE && p.key_out != nullptr)
            ll_post_key(p.tp, p.key_out, blockIdx.x, gridDim.x, m, m < p.m && m < MR ? bkey[m] : 0ull, ep);
    }
    W8A8_MARK(TR_GEMV, 4);
    if (epi != EPI_SWIGLU || p.hq == nullptr) return;
    // the row amax across the grid; the last CTA requantizes h (quant_act)
    if (tid < p.m && tid < MR) atomicMax(p.amax_bits + tid, bamax[tid]);
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) swiglu_requant(p, &sfs);
    W8A8_MARK(TR_GEMV, 5);
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
    GemvCfg cf;
    int grid;
    size_t smem;
};

// Tile rows: a power of two between 8 and 256. A GEMV whose rows fit one tile
// per CTA (up to 32 KB per matrix) takes that: the per-tile code then runs
// once, and the ring is one tile (small, so the next kernel's CTAs fit beside
// it). Otherwise about 16 KB per matrix, or, when the weights stream through
// each CTA many times, 32 KB tiles (less fixed work per byte) in a 96 KB ring
// with two CTAs per SM (more warps to hide the dot products' latency); for
// rows of 2 KB or more one CTA per SM with a 160 KB ring (measured on the
// 128256 x 2048 classifier: 58.5 against 64.4 us; the 151936 x 1024 one is
// faster with two CTAs, 33.4 against 36.4 us).
// Consumer threads split a row's K (256 / rows threads per row).
static Tiling tiling(const LinearParams& p, int mr, int pro, int epi) {
    Tiling t{};
    const bool stream = (size_t)p.n * p.k >= kStreamBytes;
    int tr = (stream ? 32768 : 16384) / p.k;
    const int sms = sm_count();
    int one = 1;                                               // rows for one tile per CTA
    while (one * sms < p.n) one *= 2;
    if (!stream && one > tr && (size_t)one * p.k <= 32768) tr = one;
    tr = tr < kWarps ? kWarps : (tr > kConsumers ? kConsumers : tr);
    int pw = 1;
    while (pw * 2 <= tr) pw *= 2;
    t.cf.pro = pro;
    t.cf.epi = epi;
    t.cf.tr = pw;
    t.cf.S = kConsumers / pw;                                 // consumer threads per row, at most 32
    t.cf.ls = 0;
    while ((1 << t.cf.ls) < t.cf.S) ++t.cf.ls;
    t.cf.lt = 0;
    while ((1 << t.cf.lt) < pw) ++t.cf.lt;
    const size_t stage = (size_t)pw * p.k * (epi == EPI_SWIGLU ? 2 : 1);
    const bool wide = stream && p.k >= 2048;
    size_t st = (wide ? kWideRingBytes : stream ? kStreamRingBytes : kRingBytes) / stage;
    t.cf.stages = (int)(st < 2 ? 2 : (st > (size_t)kMaxStages ? kMaxStages : st));
    t.cf.ntiles = (p.n + pw - 1) / pw;
    const int slots = stream && !wide ? kStreamCtasPerSm * sms : sms;
    t.grid = t.cf.ntiles < slots ? t.cf.ntiles : slots;
    const int per = (t.cf.ntiles + t.grid - 1) / t.grid;     // tiles of a CTA, at most
    if (t.cf.stages > per) t.cf.stages = per;
    const size_t nj = (size_t)((t.cf.ntiles + t.grid - 1) / t.grid) * pw;   // rows of a CTA, at most
    const size_t rest = (size_t)mr * p.k + (pro == PRO_I8 ? 0 : (size_t)p.k * 4) +
                        nj * 4 * ((epi == EPI_SWIGLU ? 2 : 1) + (epi == EPI_RESID ? mr : 0)) +
                        (pro == PRO_RMSQ ? (size_t)p.k * 4 : 0);
    while (wide && t.cf.stages > 2 && t.cf.stages * stage + rest > kGemvSmemMax) --t.cf.stages;
    t.smem = (size_t)t.cf.stages * stage + rest;
    return t;
}

template <int MR>
static cudaError_t launch_g(const LinearParams& p, int pro, int epi, cudaStream_t st) {
    const Tiling t = tiling(p, MR, pro, epi);
    auto kern = p.tp.ranks > 1 ? gemv_kernel<MR, true> : gemv_kernel<MR, false>;
    // the one-row decode chain: its kinds compiled in (code a launch runs
    // once is fetched cold; run-time kind switches add to it)
    if (MR == 1 && p.tp.ranks <= 1) {
        if (pro == PRO_RMSQ && epi == EPI_STORE) kern = gemv_kernel<MR, false, PRO_RMSQ, EPI_STORE>;
        else if (pro == PRO_QUANT && epi == EPI_RESID) kern = gemv_kernel<MR, false, PRO_QUANT, EPI_RESID>;
        else if (pro == PRO_RMSQ && epi == EPI_SWIGLU) kern = gemv_kernel<MR, false, PRO_RMSQ, EPI_SWIGLU>;
    }
    // the launch's own size, not a common maximum: the block scheduler reserves
    // this much per CTA, and the next kernel's CTAs must fit beside this one's
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)t.smem);
    if (e != cudaSuccess) return e;
    // one shared-memory carveout for every kernel of the chain: no L1 / shared
    // reconfiguration of an SM between consecutive kernels
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return launch_k(kern, dim3(t.grid), dim3(kGemvThreads), t.smem, st, p, t.cf);
}

int gemv_grid(const LinearParams& p, int pro, int epi) {
    const int mr = p.m <= 1 ? 1 : (p.m <= 2 ? 2 : 4);
    return tiling(p, mr, pro, epi).grid;
}

bool gemv_fits(const LinearParams& p, int pro, int epi) {
    if (p.m > 4) return false;
    const int mr = p.m <= 1 ? 1 : (p.m <= 2 ? 2 : 4);
    return tiling(p, mr, pro, epi).smem <= kGemvSmemMax;
}

cudaError_t launch_gemv(const LinearParams& p, int pro, int epi, cudaStream_t st) {
    if (pro < PRO_I8 || pro > PRO_RMSQ || epi < EPI_STORE || epi > EPI_PARTIAL) return cudaErrorInvalidValue;
    if (pro == PRO_I8 && epi == EPI_SWIGLU) return cudaErrorInvalidValue;
    if (p.m <= 1) return launch_g<1>(p, pro, epi, st);
    if (p.m <= 2) return launch_g<2>(p, pro, epi, st);
    return launch_g<4>(p, pro, epi, st);
}

unsigned int gemv_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_gemv_errors, sizeof(v));
    cudaMemcpyToSymbol(g_gemv_errors, &zero, sizeof(zero));
    return v;
}

}  // namespace w8a8
