// Mixture-of-experts FFN of the W8A8 decoder (hf_generic.QMixtralMoe.route /
// _row, compiler/frontend/hf_generic.py:641-657; the Granite-MoE router is the
// same softmax over the Top-k logits): y = resid + sum_k w_k * expert_k(x_n),
// x_n = rmsnorm(x), every expert a SwiGLU of W8A8 linears, for up to 16 rows,
// each row with its own Top-k.
//
// Three launches (programmatic dependent launch between them):
//  1. router, one CTA per row: fused rmsnorm + quant_act prologue (the int8
//     row is kept for the experts), the router GEMV (its rows bulk-copied before
//     the wait), the Top-k by value then lower id (llm docs:
//     moe_native_lowering_design.md:342-345), e = EXP(v - v0), w = e*RECIP(sum e)
//     with the D = 16 ordered sum; clears the experts' amax slots;
//  2. gate / up, one CTA per (row, slot, 16 rows of the expert's hidden):
//     h = (g*RECIP(1 + EXP(-g)))*u, the slot's amax |h| by atomic max;
//  3. down + combine, one CTA per (row, 16 outputs): every slot's h requantized
//     (quant_act with that amax), the k down GEMVs, and the combine folded in
//     k order from 0: y = ((0 + w_0 y_0) + w_1 y_1) + ..., then resid + y.
// The expert ids are known only after launch 1, so the expert weights are
// fetched after the wait (bulk copies of whole row tiles).
#include "linear_common.cuh"
#include "pdl.cuh"
#include "tp.cuh"

namespace w8a8 {

__device__ unsigned int g_moe_errors;     // bit 3: a weight-tile copy wait gave up; bit 5: an exchange wait;
                                          // bit 6: more pairs of one expert than rows

constexpr int kMoeThreads = 256;
constexpr int kMoeTile = 16;                                   // expert rows per CTA (launches 2 and 3)

// ---------------------------------------------------------------- launch 1
__global__ void __launch_bounds__(kMoeThreads) moe_router_kernel(MoeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = p.experts, K = p.top_k, dim = p.dim;
    int8_t* wt = reinterpret_cast<int8_t*>(smem);                         // router rows [E][dim]
    int8_t* xs = wt + (size_t)E * dim;                                    // [dim]
    float* xf = reinterpret_cast<float*>(xs + dim);                       // [dim] staging
    __shared__ __align__(8) uint64_t bar;
    __shared__ float sx[1], red[32], sc[kMoeMaxExperts], ev[kMoeMaxExperts];
    __shared__ int ids_s[kMoeMaxExperts];
    if (tid == 0) {                                                       // router weights: constants
        mbar_init(&bar, 1);
        mbar_fence_init();
        mbar_expect_tx(&bar, (uint32_t)(E * dim));
        bulk_g2s(wt, p.rq, (uint32_t)(E * dim), &bar);
    }
    pdl_wait();
    pdl_trigger();
    LinearParams lp{};
    lp.m = 1, lp.k = dim, lp.x = p.x + (size_t)row * dim, lp.norm_g = p.norm_g, lp.eps = p.eps;
    lp.inv_k = p.inv_dim;
    if (p.norm_g != nullptr) prologue<1, PRO_RMSQ>(lp, xs, xf, sx, red);   // both end with a block barrier
    else prologue<1, PRO_QUANT>(lp, xs, xf, sx, red);
    for (int c = tid; c < dim / 16; c += kMoeThreads)                     // the int8 row, for the experts
        reinterpret_cast<int4*>(p.xq + (size_t)row * dim)[c] = reinterpret_cast<const int4*>(xs)[c];
    if (tid == 0) p.s_x[row] = sx[0];
    if (tid < K) p.amax[row * K + tid] = 0u;                              // the experts' atomic maxima
    const bool ok = mbar_wait(&bar, 0u);
    if (!ok && tid == 0) atomicOr(&g_moe_errors, 8u);
    // scores: warp w takes rows w, w + 8, ...; (f32(acc) * s_r) * s_x
    for (int e = warp; e < E; e += kMoeThreads / 32) {
        int acc = 0;
        const int4* wr = reinterpret_cast<const int4*>(wt + (size_t)e * dim);
        const int4* xr = reinterpret_cast<const int4*>(xs);
        for (int c = lane; c < dim / 16; c += 32) {
            const int4 a = wr[c], b = xr[c];
            acc = dp4a(a.w, b.w, dp4a(a.z, b.z, dp4a(a.y, b.y, dp4a(a.x, b.x, acc))));
        }
        acc = warp_sum_i(acc);
        if (lane == 0) sc[e] = fmul(fmul(i2f(acc), __ldg(p.rs + e)), sx[0]);
    }
    __syncthreads();
    if (warp == 0) {
        // Top-k: keys (value, then the lower id) held two per lane; k rounds of a warp max
        unsigned long long k0 = lane < E ? argmax_key(sc[lane], lane) : 0ull;
        unsigned long long k1 = lane + 32 < E ? argmax_key(sc[lane + 32], lane + 32) : 0ull;
        for (int j = 0; j < K; ++j) {
            unsigned long long best = k0 > k1 ? k0 : k1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
                best = t > best ? t : best;
            }
            const int id = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
            if (best == k0) k0 = 0ull;                                    // keys are unique: one lane owns it
            if (best == k1) k1 = 0ull;
            if (lane == 0) ids_s[j] = id;
        }
        __syncwarp();
        // e_j = EXP(v_j - v_0), w_j = e_j * RECIP(sum e) (the sum in the D = 16 order)
        const float v0 = sc[ids_s[0]];
        for (int j = lane; j < K; j += 32) ev[j] = sfu_exp(fsub(sc[ids_s[j]], v0));
        __syncwarp();
        const float s = red_sum16([&](int i) { return ev[i]; }, K, lane);
        const float rs = sfu_recip(s);
        for (int j = lane; j < K; j += 32) {
            p.ids[row * K + j] = ids_s[j];
            p.w[row * K + j] = fmul(ev[j], rs);
        }
    }
    if (p.slab_x != nullptr) {                                            // tensor-core path: into the slabs
        __shared__ int pos_s[kMoeMaxTopK];
        __syncthreads();                                                  // ids_s complete
        if (tid < K) {
            const int e = ids_s[tid] - p.e_lo;
            int pos = -1;
            if (e >= 0 && e < p.e_n) {                                    // this rank's expert: the next slab row
                const int r = atomicAdd(p.cnt + e, 1);                    // (< m <= mcap: one pair per row)
                if (r < p.mcap) {
                    pos = e * p.mcap + r;
                    p.slab_pair[pos] = row * K + tid;
                } else {
                    atomicOr(&g_moe_errors, 64u);
                }
            }
            pos_s[tid] = pos;
            p.pair_pos[row * K + tid] = pos;
        }
        __syncthreads();
        for (int c = tid; c < K * (dim / 16); c += kMoeThreads) {
            const int j = c / (dim / 16), cc = c % (dim / 16);
            if (pos_s[j] >= 0)
                reinterpret_cast<int4*>(p.slab_x + (size_t)pos_s[j] * dim)[cc] = reinterpret_cast<const int4*>(xs)[cc];
        }
    }
}

// ---------------------------------------------------------------- launch 2
__global__ void __launch_bounds__(kMoeThreads) moe_up_kernel(MoeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tile = blockIdx.x, slot = blockIdx.y, row = blockIdx.z, tid = threadIdx.x, lane = tid & 31;
    const int K = p.top_k, dim = p.dim, ih = p.ih, i0 = tile * kMoeTile;
    int8_t* wg = reinterpret_cast<int8_t*>(smem);                        // gate rows [16][dim]
    int8_t* wu = wg + (size_t)kMoeTile * dim;                            // up rows [16][dim]
    int8_t* xs = wu + (size_t)kMoeTile * dim;                            // [dim]
    __shared__ __align__(8) uint64_t bar;
    __shared__ int e_s;
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    pdl_wait();
    pdl_trigger();
    if (tid == 0) {                                                       // the slot's expert: known now
        const int e = p.ids[row * K + slot] - p.e_lo;                     // this rank's index of it
        e_s = e;
        if (e >= 0 && e < p.e_n) {                                        // (another rank's expert: nothing)
            const uint32_t bytes = (uint32_t)(kMoeTile * dim);
            mbar_expect_tx(&bar, 2u * bytes);
            bulk_g2s(wg, p.gq + ((size_t)e * ih + i0) * dim, bytes, &bar);
            bulk_g2s(wu, p.uq + ((size_t)e * ih + i0) * dim, bytes, &bar);
        }
    }
    for (int c = tid; c < dim / 16; c += kMoeThreads)
        reinterpret_cast<int4*>(xs)[c] = __ldcg(reinterpret_cast<const int4*>(p.xq + (size_t)row * dim) + c);
    const float sx = __ldcg(p.s_x + row);
    __syncthreads();
    const int e = e_s;
    if (e < 0 || e >= p.e_n) return;                                      // no copy was issued
    const bool ok = mbar_wait(&bar, 0u);
    if (!ok && tid == 0) atomicOr(&g_moe_errors, 8u);
    // thread t: row r = t / 16 of the tile, 16-byte chunks s, s + 16, ... of it
    const int r = tid / 16, sl = tid % 16;
    int ag = 0, au = 0;
    for (int c = sl; c < dim / 16; c += 16) {
        const int4 x = reinterpret_cast<const int4*>(xs)[c];
        const int4 a = reinterpret_cast<const int4*>(wg + (size_t)r * dim)[c];
        const int4 b = reinterpret_cast<const int4*>(wu + (size_t)r * dim)[c];
        ag = dp4a(a.w, x.w, dp4a(a.z, x.z, dp4a(a.y, x.y, dp4a(a.x, x.x, ag))));
        au = dp4a(b.w, x.w, dp4a(b.z, x.z, dp4a(b.y, x.y, dp4a(b.x, x.x, au))));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        ag += __shfl_xor_sync(0xffffffffu, ag, o);
        au += __shfl_xor_sync(0xffffffffu, au, o);
    }
    uint32_t am = 0u;
    if (sl == 0) {
        const int i = i0 + r;
        const float g = fmul(fmul(i2f(ag), __ldg(p.gs + (size_t)e * ih + i)), sx);
        const float u = fmul(fmul(i2f(au), __ldg(p.us + (size_t)e * ih + i)), sx);
        const float h = silu_gate(g, u);
        p.h[((size_t)row * K + slot) * ih + i] = h;
        am = __float_as_uint(fabsf(h));                                   // as bits: NaN above numbers
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = max(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0 && am != 0u) atomicMax(p.amax + row * K + slot, am);
    if (!ok) mbar_wait(&bar, 0u);                                         // no copy may land after exit
}

// ---------------------------------------------------------------- launch 3
__global__ void __launch_bounds__(kMoeThreads) moe_down_kernel(MoeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tile = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
    const int K = p.top_k, dim = p.dim, ih = p.ih, n0 = tile * kMoeTile;
    int8_t* wd = reinterpret_cast<int8_t*>(smem);                        // [K][16][ih] down rows
    int8_t* hq = wd + (size_t)K * kMoeTile * ih;                         // [K][ih]
    __shared__ __align__(8) uint64_t bar;
    __shared__ int e_s[kMoeMaxTopK];                                     // this rank's index, or -1
    __shared__ float w_s[kMoeMaxTopK], sh_s[kMoeMaxTopK], inv_s[kMoeMaxTopK];
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    pdl_wait();
    pdl_trigger();
    const uint32_t ep = p.wy_ll != nullptr ? tp_epoch(p.tp) : 0u;
    if (p.wy_ll != nullptr && tile == 0 && tid == 0) {               // this rank reached layer's down: presence
        const size_t pw = (size_t)kTpRows * K * dim + (size_t)p.tp.rank * kTpRows + row;
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
            if (q < p.tp.ranks) ll_store(tp_at(p.tp, p.wy_ll, q) + pw, 1u, ep);
    }
    if (tid < K) {
        const int e = p.ids[row * K + tid] - p.e_lo;
        e_s[tid] = e >= 0 && e < p.e_n ? e : -1;
        w_s[tid] = p.w[row * K + tid];
        const float s = fmul(__uint_as_float(__ldcg(p.amax + row * K + tid)), W8A8_C127);
        sh_s[tid] = s;
        inv_s[tid] = sfu_recip(s);
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t bytes = (uint32_t)(kMoeTile * ih);
        uint32_t own = 0;
        for (int j = 0; j < K; ++j) own += e_s[j] >= 0 ? 1u : 0u;
        mbar_expect_tx(&bar, own * bytes);
        for (int j = 0; j < K; ++j)
            if (e_s[j] >= 0)
                bulk_g2s(wd + (size_t)j * kMoeTile * ih, p.dq + ((size_t)e_s[j] * dim + n0) * ih, bytes, &bar);
    }
    // every slot's h row -> int8 with its own scale (quant_act of that expert's h)
    for (int i = tid; i < K * ih / 4; i += kMoeThreads) {
        const int j = (i * 4) / ih;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.h + (size_t)row * K * ih) + i);
        const float inv = inv_s[j];
        reinterpret_cast<char4*>(hq)[i] =
            make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)), to_i8(fmul(v.w, inv)));
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0u);
    if (!ok && tid == 0) atomicOr(&g_moe_errors, 8u);
    const int r = tid / 16, sl = tid % 16, n = n0 + r;
    float y = 0.f;
    for (int j = 0; j < K; ++j) {                                         // k order: the combine's order
        if (e_s[j] < 0) {                                                 // another rank's expert
            if (p.wy != nullptr && sl == 0) p.wy[((size_t)row * K + j) * dim + n] = 0.f;
            continue;                                                     // (exchange: its owner writes it)
        }
        int acc = 0;
        const int4* a4 = reinterpret_cast<const int4*>(wd + ((size_t)j * kMoeTile + r) * ih);
        const int4* h4 = reinterpret_cast<const int4*>(hq + (size_t)j * ih);
        for (int c = sl; c < ih / 16; c += 16) {
            const int4 a = a4[c], b = h4[c];
            acc = dp4a(a.w, b.w, dp4a(a.z, b.z, dp4a(a.y, b.y, dp4a(a.x, b.x, acc))));
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const float yk = fmul(fmul(i2f(acc), __ldg(p.ds + (size_t)e_s[j] * dim + n)), sh_s[j]);
        const float t = fmul(w_s[j], yk);
        if (p.wy_ll != nullptr) {                                         // the term to every rank
            if (sl == 0) {
                const size_t w = ((size_t)row * K + j) * dim + n;
#pragma unroll
                for (int q = 0; q < kTpMaxRanks; ++q)
                    if (q < p.tp.ranks) ll_store(tp_at(p.tp, p.wy_ll, q) + w, __float_as_uint(t), ep);
            }
        } else if (p.wy != nullptr) {
            if (sl == 0) p.wy[((size_t)row * K + j) * dim + n] = t;
        } else {
            y = fadd(y, t);
        }
    }
    if (sl == 0 && p.wy == nullptr && p.wy_ll == nullptr)
        p.y[(size_t)row * dim + n] = fadd(__ldcg(p.resid + (size_t)row * dim + n), y);
    if (!ok) mbar_wait(&bar, 0u);
}

// ---------------------------------------------------------------- combine
// Expert parallelism, after the ranks' w_j * y_j terms were summed (each has one
// nonzero contributor, so the sum is that term; a -0 becoming +0 does not change
// the fold, which starts from +0): y = resid + (((0 + t_0) + t_1) + ...), k order.
__global__ void __launch_bounds__(kMoeThreads) moe_combine_kernel(const float* wy, int K, int dim, const float* resid,
                                                                  float* y) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.y;
    for (int n = blockIdx.x * kMoeThreads + threadIdx.x; n < dim; n += gridDim.x * kMoeThreads) {
        float acc = 0.f;
        for (int j = 0; j < K; ++j) acc = fadd(acc, __ldcg(wy + ((size_t)row * K + j) * dim + n));
        y[(size_t)row * dim + n] = fadd(__ldcg(resid + (size_t)row * dim + n), acc);
    }
}

cudaError_t launch_moe_combine(const float* wy, int m, int top_k, int dim, const float* resid, float* y,
                               cudaStream_t st) {
    const int bx = (dim + kMoeThreads - 1) / kMoeThreads;
    return launch_k(moe_combine_kernel, dim3(bx, m), dim3(kMoeThreads), 0, st, wy, top_k, dim, resid, y);
}

// The same combine over exchange words: every rank's presence word of the row
// first (the ordering between steps), then the k terms of each output (each
// written by its expert's rank; all k loads in flight), folded in k order.
__global__ void __launch_bounds__(kMoeThreads) moe_combine_ll_kernel(TpCtx tp, const uint64_t* wy, int K, int dim,
                                                                     const float* resid, float* y) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.y, tid = threadIdx.x;
    const uint32_t ep = tp_epoch(tp);
    bool ok = true;
    if (tid < tp.ranks) ll_wait(wy + (size_t)kTpRows * K * dim + (size_t)tid * kTpRows + row, ep, ok);
    __syncthreads();
    for (int n = blockIdx.x * kMoeThreads + tid; n < dim; n += gridDim.x * kMoeThreads) {
        uint64_t w[kMoeMaxTopK];
        uint32_t pending = (1u << K) - 1u;
        for (int spins = 0; pending != 0u; ++spins) {
#pragma unroll
            for (int j = 0; j < kMoeMaxTopK; ++j)
                if (pending & (1u << j)) w[j] = ll_load(wy + ((size_t)row * K + j) * dim + n);
#pragma unroll
            for (int j = 0; j < kMoeMaxTopK; ++j)
                if ((pending & (1u << j)) && (uint32_t)(w[j] >> 32) == ep) pending &= ~(1u << j);
            if (pending == 0u) break;
            if (!ok || spins >= kLlLimit) {
                ok = false;
                break;
            }
            if (spins >= kLlSpin) __nanosleep(128);
        }
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < kMoeMaxTopK; ++j)                             // k order
            if (j < K) acc = fadd(acc, (pending & (1u << j)) ? 0.f : __uint_as_float((uint32_t)w[j]));
        y[(size_t)row * dim + n] = fadd(__ldcg(resid + (size_t)row * dim + n), acc);
    }
    if (!ok) atomicOr(&g_moe_errors, 32u);
}

cudaError_t launch_moe_combine_ll(const TpCtx& tp, const uint64_t* wy_ll, int m, int top_k, int dim,
                                  const float* resid, float* y, cudaStream_t st) {
    const int bx = (dim + kMoeThreads - 1) / kMoeThreads;
    return launch_k(moe_combine_ll_kernel, dim3(bx, m), dim3(kMoeThreads), 0, st, tp, wy_ll, top_k, dim, resid, y);
}

// ---------------------------------------------------------------- many rows
// Batched decode and prefill chunks: the rows' (row, slot) pairs grouped by
// expert, so that each expert's weight tiles are read once for all the rows that
// chose it (the per-row kernels above read them once per pair). Launches: the
// router (as above); gate/up and down with one CTA per (tile, expert), each
// listing its expert's pairs from the routing ids itself (expert parallelism
// adds a down column for the other ranks' pairs, stored as +0); then the
// k-order combine (moe_combine_kernel) unless the terms go out for an
// expert-parallel sum. Each pair's arithmetic is the per-row kernels' own, so
// the results are the same bit for bit.
constexpr int kMoePairs = 16;                                  // pairs per pass of a grouped CTA
constexpr int kMoeDownTile = 32;                               // down rows per grouped CTA
constexpr int kMoePad = 16;                                    // bytes after each staged row (banks)

// The pairs q = row * k + slot of this rank's expert e into list[], in q
// order; their count. A row chooses an expert at most once, so at most m; list
// holds cap = m entries, and a larger count (routing that is not Top-k) stores
// none past it and sets error bit 6. Every thread of the CTA calls it (block
// barriers inside). Each CTA scans the routing itself: one read of the ids, no
// separate list launch.
__device__ int moe_list_pairs(const MoeParams& p, int e, int* list, int cap) {
    __shared__ int wcnt[kMoeThreads / 32];
    constexpr int kPer = 8;                                       // ids per thread per round
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, n = p.m * p.top_k;
    int total = 0;
    for (int base = 0; base < n; base += kPer * kMoeThreads) {
        int id[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {                          // all loads of the round in flight
            const int q = base + u * kMoeThreads + tid;
            id[u] = q < n ? __ldcg(p.ids + q) : -1;
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            if (base + u * kMoeThreads >= n) break;               // (uniform)
            const int q = base + u * kMoeThreads + tid;
            const bool mine = q < n && id[u] - p.e_lo == e;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (lane == 0) wcnt[warp] = __popc(bal);
            __syncthreads();
            int off = total, all = 0;
#pragma unroll
            for (int w = 0; w < kMoeThreads / 32; ++w) {
                off += w < warp ? wcnt[w] : 0;
                all += wcnt[w];
            }
            const int at = off + __popc(bal & ((1u << lane) - 1u));
            if (mine && at < cap) list[at] = q;
            total += all;
            __syncthreads();                                      // wcnt free for the next round
        }
    }
    if (total > cap) {
        if (tid == 0) atomicOr(&g_moe_errors, 64u);
        total = cap;
    }
    return total;
}

// gate / up: CTA (tile, expert) holds the expert's 16 gate and up rows; per
// pass, the int8 rows of up to 16 of its pairs. Thread (r, j) computes row
// i0 + r of pair j over the whole dim: h and, through shared memory, the
// pair's max|h| over the tile.
__global__ void __launch_bounds__(kMoeThreads) moe_up_rows_kernel(MoeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tile = blockIdx.x, e = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int K = p.top_k, dim = p.dim, ih = p.ih, i0 = tile * kMoeTile, nc = dim / 16, xstr = dim + kMoePad;
    int8_t* wg = reinterpret_cast<int8_t*>(smem);                        // gate rows [16][dim]
    int8_t* wu = wg + (size_t)kMoeTile * dim;                            // up rows [16][dim]
    int8_t* xs = wu + (size_t)kMoeTile * dim;                            // [kMoePairs][dim + pad]
    int* list = reinterpret_cast<int*>(xs + (size_t)kMoePairs * xstr);  // [m]: this expert's pairs
    __shared__ __align__(8) uint64_t bar;
    __shared__ int pr_s[kMoePairs];
    __shared__ float sx_s[kMoePairs];
    __shared__ uint32_t am_s[kMoePairs];
    if (tid == 0) {                                                       // the weights: constants
        mbar_init(&bar, 1);
        mbar_fence_init();
        const uint32_t bytes = (uint32_t)(kMoeTile * dim);
        mbar_expect_tx(&bar, 2u * bytes);
        bulk_g2s(wg, p.gq + ((size_t)e * ih + i0) * dim, bytes, &bar);
        bulk_g2s(wu, p.uq + ((size_t)e * ih + i0) * dim, bytes, &bar);
    }
    pdl_wait();
    pdl_trigger();
    const int q0 = 0, q1 = moe_list_pairs(p, e, list, p.m);             // (ends with a block barrier)
    const int r = tid / kMoePairs, j = tid % kMoePairs, i = i0 + r;
    const float gs = __ldg(p.gs + (size_t)e * ih + i), us = __ldg(p.us + (size_t)e * ih + i);
    const bool ok = mbar_wait(&bar, 0u);
    if (!ok && tid == 0) atomicOr(&g_moe_errors, 8u);
    const int4* ga = reinterpret_cast<const int4*>(wg + (size_t)r * dim);
    const int4* ua = reinterpret_cast<const int4*>(wu + (size_t)r * dim);
    const int4* xa = reinterpret_cast<const int4*>(xs + (size_t)j * xstr);
    for (int q = q0; q < q1 && ok; q += kMoePairs) {
        const int np = min(kMoePairs, q1 - q);
        if (tid < np) {
            const int pr = list[q + tid];
            pr_s[tid] = pr;
            sx_s[tid] = __ldcg(p.s_x + pr / K);
            am_s[tid] = 0u;
        }
        __syncthreads();
        for (int c = tid; c < np * nc; c += kMoeThreads) {                // every row of the pass at once
            const int jj = c / nc, cc = c % nc;
            reinterpret_cast<int4*>(xs + (size_t)jj * xstr)[cc] =
                __ldcg(reinterpret_cast<const int4*>(p.xq + (size_t)(pr_s[jj] / K) * dim) + cc);
        }
        __syncthreads();
        uint32_t am = 0u;
        if (j < np) {
            int ag = 0, au = 0, ag1 = 0, au1 = 0;                        // two chains each (exact int32)
#pragma unroll 4
            for (int c = 0; c < nc; c += 2) {                             // (nc even: dim % 32 == 0)
                const int4 a = ga[c], b = ua[c], x = xa[c];
                const int4 a1 = ga[c + 1], b1 = ua[c + 1], x1 = xa[c + 1];
                ag = dp4a(a.w, x.w, dp4a(a.z, x.z, dp4a(a.y, x.y, dp4a(a.x, x.x, ag))));
                au = dp4a(b.w, x.w, dp4a(b.z, x.z, dp4a(b.y, x.y, dp4a(b.x, x.x, au))));
                ag1 = dp4a(a1.w, x1.w, dp4a(a1.z, x1.z, dp4a(a1.y, x1.y, dp4a(a1.x, x1.x, ag1))));
                au1 = dp4a(b1.w, x1.w, dp4a(b1.z, x1.z, dp4a(b1.y, x1.y, dp4a(b1.x, x1.x, au1))));
            }
            ag += ag1, au += au1;
            const float sx = sx_s[j];
            const float g = fmul(fmul(i2f(ag), gs), sx);
            const float u = fmul(fmul(i2f(au), us), sx);
            const float h = silu_gate(g, u);
            p.h[(size_t)pr_s[j] * ih + i] = h;
            am = __float_as_uint(fabsf(h));                               // as bits: NaN above numbers
        }
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 16));               // rows r, r + 1: the same pair
        if (lane < 16 && am != 0u) atomicMax(&am_s[j], am);
        __syncthreads();
        if (tid < np && am_s[tid] != 0u) atomicMax(p.amax + pr_s[tid], am_s[tid]);
        __syncthreads();                                                  // xs, pr_s free for the next pass
    }
    if (!ok) mbar_wait(&bar, 0u);                                         // no copy may land after exit
}

// down: CTA (tile, expert) holds 32 of the expert's down rows; per pass, up to
// 16 of its pairs' h rows requantized (quant_act with each pair's max). Thread
// (r, j) computes rows n0 + r and n0 + r + 16 of pair j and stores w_j * y_j.
// CTAs (tile, e_n) store +0 for the pairs of other ranks' experts.
__global__ void __launch_bounds__(kMoeThreads) moe_down_rows_kernel(MoeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tile = blockIdx.x, e = blockIdx.y, tid = threadIdx.x;
    const int dim = p.dim, ih = p.ih, n0 = tile * kMoeDownTile, nc = ih / 16, hstr = ih + kMoePad;
    int8_t* wd = reinterpret_cast<int8_t*>(smem);                        // [32][ih] down rows
    int8_t* hq = wd + (size_t)kMoeDownTile * ih;                         // [kMoePairs][ih + pad]
    int* list = reinterpret_cast<int*>(hq + (size_t)kMoePairs * hstr);  // [m]: this bucket's pairs
    __shared__ __align__(8) uint64_t bar;
    __shared__ int pr_s[kMoePairs];
    __shared__ float s_s[kMoePairs], inv_s[kMoePairs], w_s[kMoePairs];
    const bool own = e < p.e_n;
    if (tid == 0 && own) {                                                // the weights: constants
        mbar_init(&bar, 1);
        mbar_fence_init();
        const uint32_t bytes = (uint32_t)(kMoeDownTile * ih);
        mbar_expect_tx(&bar, bytes);
        bulk_g2s(wd, p.dq + ((size_t)e * dim + n0) * ih, bytes, &bar);
    }
    pdl_wait();
    pdl_trigger();
    if (!own) {                                                           // other ranks' experts: +0
        const int n = p.m * p.top_k;                                     // (up to k per row: no list)
        for (int t = tid; t < n * kMoeDownTile; t += kMoeThreads) {
            const int q = t / kMoeDownTile, x = __ldcg(p.ids + q) - p.e_lo;
            if (x < 0 || x >= p.e_n) p.wy[(size_t)q * dim + n0 + t % kMoeDownTile] = 0.f;
        }
        return;
    }
    const int q0 = 0, q1 = moe_list_pairs(p, e, list, p.m);             // (ends with a block barrier)
    const int r = tid / kMoePairs, j = tid % kMoePairs, n = n0 + r;
    const float ds0 = __ldg(p.ds + (size_t)e * dim + n), ds1 = __ldg(p.ds + (size_t)e * dim + n + 16);
    const bool ok = mbar_wait(&bar, 0u);
    if (!ok && tid == 0) atomicOr(&g_moe_errors, 8u);
    const int4* a0 = reinterpret_cast<const int4*>(wd + (size_t)r * ih);
    const int4* a1 = reinterpret_cast<const int4*>(wd + (size_t)(r + 16) * ih);
    const int4* ha = reinterpret_cast<const int4*>(hq + (size_t)j * hstr);
    for (int q = q0; q < q1 && ok; q += kMoePairs) {
        const int np = min(kMoePairs, q1 - q);
        if (tid < np) {
            const int pr = list[q + tid];
            pr_s[tid] = pr;
            const float s = fmul(__uint_as_float(__ldcg(p.amax + pr)), W8A8_C127);
            s_s[tid] = s;
            inv_s[tid] = sfu_recip(s);
            w_s[tid] = __ldcg(p.w + pr);
        }
        __syncthreads();
        for (int c = tid; c < np * (ih / 4); c += kMoeThreads) {          // every h row of the pass at once
            const int jj = c / (ih / 4), cc = c % (ih / 4);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(p.h + (size_t)pr_s[jj] * ih) + cc);
            const float inv = inv_s[jj];
            reinterpret_cast<char4*>(hq + (size_t)jj * hstr)[cc] =
                make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)),
                           to_i8(fmul(v.w, inv)));
        }
        __syncthreads();
        if (j < np) {
            int c0 = 0, c1 = 0;
#pragma unroll 4
            for (int c = 0; c < nc; ++c) {
                const int4 x = ha[c], u = a0[c], v = a1[c];
                c0 = dp4a(u.w, x.w, dp4a(u.z, x.z, dp4a(u.y, x.y, dp4a(u.x, x.x, c0))));
                c1 = dp4a(v.w, x.w, dp4a(v.z, x.z, dp4a(v.y, x.y, dp4a(v.x, x.x, c1))));
            }
            const int pr = pr_s[j];
            const float s = s_s[j], w = w_s[j];
            p.wy[(size_t)pr * dim + n] = fmul(w, fmul(fmul(i2f(c0), ds0), s));
            p.wy[(size_t)pr * dim + n + 16] = fmul(w, fmul(fmul(i2f(c1), ds1), s));
        }
        __syncthreads();                                                  // hq, pr_s free for the next pass
    }
    if (!ok) mbar_wait(&bar, 0u);
}

// Tensor-core path, between the grouped gate/up and down GEMMs: each pair's h
// requantized (quant_act with its max|h|, the per-row kernels' arithmetic) into
// its slab row, its scale into s_h; a pair of another rank's expert stores +0
// terms instead. One CTA per pair.
constexpr int kQuantHThreads = 128;
__global__ void __launch_bounds__(kQuantHThreads) moe_quant_h_kernel(MoeParams p) {
    const int pr = blockIdx.x, tid = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    const int pos = __ldcg(p.pair_pos + pr);
    if (pos < 0) {
        for (int n = tid; n < p.dim; n += kQuantHThreads) p.wy[(size_t)pr * p.dim + n] = 0.f;
        return;
    }
    const float s = fmul(__uint_as_float(__ldcg(p.amax + pr)), W8A8_C127);
    const float inv = sfu_recip(s);
    if (tid == 0) p.s_h[pr] = s;
    const float4* h4 = reinterpret_cast<const float4*>(p.h + (size_t)pr * p.ih);
    char4* d4 = reinterpret_cast<char4*>(p.slab_h + (size_t)pos * p.ih);
    for (int i = tid; i < p.ih / 4; i += kQuantHThreads) {
        const float4 v = __ldcg(h4 + i);
        d4[i] = make_char4(to_i8(fmul(v.x, inv)), to_i8(fmul(v.y, inv)), to_i8(fmul(v.z, inv)),
                           to_i8(fmul(v.w, inv)));
    }
}

// Many rows on the tensor cores: the router fills each expert's slab; a
// grouped tcgen05 GEMM per matrix pair (gate / up with the SwiGLU and each
// pair's max|h| in its epilogue; down with w_j folded in), the requantizer in
// between; then the k-order combine unless the terms go out for an
// expert-parallel sum.
static cudaError_t launch_moe_rows_tc(const MoeParams& p, bool combine, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(p.cnt, 0, (size_t)p.e_n * sizeof(int), st);
    if (e != cudaSuccess) return e;
    const size_t sm0 = moe_smem(p, 0);
    e = cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm0);
    if (e != cudaSuccess) return e;
    e = launch_k(moe_router_kernel, dim3(p.m), dim3(kMoeThreads), sm0, st, p);
    if (e != cudaSuccess) return e;
    GemmParams g{};
    g.g_cnt = p.cnt, g.g_pair = p.slab_pair, g.g_mcap = p.mcap, g.g_mtiles = p.mcap / 128, g.g_top_k = p.top_k;
    GemmOperands up{};
    up.xq = p.slab_x, up.w = p.gq, up.w2 = p.uq;
    GemmParams gu = g;
    gu.m = p.e_n * p.mcap, gu.n = p.ih, gu.k = p.dim, gu.s_x = p.s_x, gu.s_w = p.gs, gu.s_w2 = p.us, gu.y = p.h;
    gu.act = 0, gu.g_amax = p.amax;                                       // SiLU
    e = launch_gemm_grouped(up, gu, p.e_n, st);
    if (e != cudaSuccess) return e;
    e = launch_k(moe_quant_h_kernel, dim3(p.m * p.top_k), dim3(kQuantHThreads), 0, st, p);
    if (e != cudaSuccess) return e;
    GemmOperands dn{};
    dn.xq = p.slab_h, dn.w = p.dq;
    GemmParams gd = g;
    gd.m = p.e_n * p.mcap, gd.n = p.dim, gd.k = p.ih, gd.s_x = p.s_h, gd.s_w = p.ds, gd.y = p.wy, gd.g_w = p.w;
    e = launch_gemm_grouped(dn, gd, p.e_n, st);
    if (e != cudaSuccess) return e;
    return combine ? launch_moe_combine(p.wy, p.m, p.top_k, p.dim, p.resid, p.y, st) : cudaSuccess;
}

size_t moe_rows_smem(const MoeParams& p, int which) {
    const size_t list = (size_t)p.m * 4;                                 // a bucket holds at most one pair per row
    if (which == 1) return (size_t)2 * kMoeTile * p.dim + (size_t)kMoePairs * (p.dim + kMoePad) + list;
    return (size_t)kMoeDownTile * p.ih + (size_t)kMoePairs * (p.ih + kMoePad) + list;
}

// ---------------------------------------------------------------- host side
size_t moe_smem(const MoeParams& p, int which) {
    if (which == 0) return (size_t)p.experts * p.dim + (size_t)p.dim * 5;
    if (which == 1) return (size_t)2 * kMoeTile * p.dim + p.dim;
    return (size_t)p.top_k * kMoeTile * p.ih + (size_t)p.top_k * p.ih;
}

cudaError_t launch_moe(const MoeParams& p, cudaStream_t st) {
    void (*kern[3])(MoeParams) = {moe_router_kernel, moe_up_kernel, moe_down_kernel};
    const dim3 grids[3] = {dim3(p.m), dim3(p.ih / kMoeTile, p.top_k, p.m), dim3(p.dim / kMoeTile, p.m)};
    for (int i = 0; i < 3; ++i) {
        const size_t sm = moe_smem(p, i);
        cudaError_t e = cudaFuncSetAttribute(kern[i], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kern[i], cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        e = launch_k(kern[i], grids[i], dim3(kMoeThreads), sm, st, p);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_moe_rows(const MoeParams& p, bool combine, cudaStream_t st) {
    if (p.slab_x != nullptr) return launch_moe_rows_tc(p, combine, st);
    struct L {
        void (*k)(MoeParams);
        dim3 grid;
        size_t sm;
    } ls[3] = {{moe_router_kernel, dim3(p.m), moe_smem(p, 0)},
               {moe_up_rows_kernel, dim3(p.ih / kMoeTile, p.e_n), moe_rows_smem(p, 1)},
               {moe_down_rows_kernel, dim3(p.dim / kMoeDownTile, p.e_n + (p.e_n < p.experts ? 1 : 0)),
                moe_rows_smem(p, 2)}};
    for (const L& l : ls) {
        cudaError_t e = cudaFuncSetAttribute(l.k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)l.sm);
        if (e != cudaSuccess) return e;
        e = launch_k(l.k, l.grid, dim3(kMoeThreads), l.sm, st, p);
        if (e != cudaSuccess) return e;
    }
    return combine ? launch_moe_combine(p.wy, p.m, p.top_k, p.dim, p.resid, p.y, st) : cudaSuccess;
}

unsigned int moe_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_moe_errors, sizeof(v));
    cudaMemcpyToSymbol(g_moe_errors, &zero, sizeof(zero));
    return v;
}

}  // namespace w8a8
