// Fused per-layer attention over the int8 KV cache, one launch per layer, for
// one sequence's M rows (a decode step: M = 1; a prefill chunk: up to 16 rows,
// each computed exactly as a decode row, compiler/frontend/hf_generic.py:306-363;
// each head's cache is read once per call for all rows, docs/fusion_design.md 6.7).
//
// One thread-block cluster per KV head: CS <= 8 CTAs, CTA j owning the cache
// positions [j*chunk, (j+1)*chunk). The CTAs of a cluster exchange their chunk
// maxima and int32 p.V partials through distributed shared memory and meet at
// the hardware cluster barrier; nothing goes through global scratch memory.
//  1. q path of the G query heads of the KV head, every row: QK-norm (RMSNorm
//     over head_dim, D = 16 ordered sum), RoPE (v*cos + swapneg(v)*sin),
//     per-head quant_act -> int8 q. The CTA whose chunk holds a row's position
//     makes that row's K and V: QK-norm + RoPE + i8(k*inv_sk), i8(v*inv_sv),
//     into the cache (llm/ref_model.py:225-229, hf_generic.SaCache.update
//     :190-226) and into its tiles. Scores (f32(qq.k)*s_q)*a_k and the chunk's
//     maxima stay in shared memory.
//     -- cluster barrier: every row maximum is the max over the cluster's chunk
//     maxima (the global max comes before any int8 rounding: no online softmax)
//  2. e = EXP(s - m); QSUM: eq = i8(127e) and the chunk's sum of eq; NORM: each
//     CTA forms the whole row's e (reading the other chunks' scores) for the
//     ordered sum, pq = i8(127 e RECIP(sum)) (llm/ref_model.py:233-242;
//     hf_generic.py:275-290); int32 pq.V of the chunk.
//     -- cluster barrier --
//  3. reduce-scatter: CTA j adds the partials of its slice of the outputs
//     (exact in any order) and dequantizes them: NORM f32(acc)*a_v; QSUM
//     (f32(acc)*(RECIP(sum)*127))*a_v.
// Every value a CTA needs from another is pushed into its shared memory with
// remote stores before the barrier that publishes it; reads are then local.
// Cache layout per layer: K [kv_heads, seq_len, head_dim] int8 (a position's
// row contiguous), V transposed [kv_heads, head_dim, seq_len] int8 (a channel's
// positions contiguous, so p.V is a dot product over positions).
#include <cooperative_groups.h>

#include "tp.cuh"
#include "pdl.cuh"
#include "trace.cuh"
#include "w8a8_internal.h"
#include "w8a8_math.cuh"

namespace cg = cooperative_groups;

namespace w8a8 {

W8A8_TRACE_BINDER(trace_bind_attn)

__device__ unsigned int g_attn_errors;                        // bit 2: a cache-tile copy wait gave up

constexpr int kMaxG = 8;                                       // query heads per KV head
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxChunk = 512;

struct AttnGeom {
    int cs, chunk;
};

__host__ __device__ inline AttnGeom attn_geom(int seq_len) {
    AttnGeom g;
    const int blocks = (seq_len + 127) / 128;                  // 128-position blocks
    g.cs = blocks < kMaxCluster ? blocks : kMaxCluster;
    g.chunk = ((blocks + g.cs - 1) / g.cs) * 128;
    return g;
}

struct AttnSmem {                                              // offsets into the dynamic shared memory
    size_t ks, vs, qs, fbuf, scs, ps, tab, gain, etab, pvp, ebuf, total;
};

__host__ __device__ inline AttnSmem attn_smem(int M, int G, int hd, int T, int chunk, int variant) {
    auto a16 = [](size_t b) { return (b + 15) & ~size_t(15); };
    AttnSmem s{};
    size_t o = 0;
    s.ks = o;   o += a16((size_t)chunk * hd);                 // K tile [chunk][hd]
    s.vs = o;   o += a16((size_t)hd * (chunk + 16));          // V^T tile [hd][chunk + 16] (padded rows)
    s.qs = o;   o += a16((size_t)M * G * hd);                 // int8 q rows
    s.fbuf = o; o += a16((size_t)2 * kAttnWarps * hd * 4);    // per-warp fp32 head vectors (q | k)
    s.scs = o;  o += a16((size_t)M * G * chunk * 4);          // scores of the chunk
    s.ps = o;   o += a16((size_t)M * G * chunk);              // int8 probabilities of the chunk
    s.tab = o;  o += a16((size_t)M * 2 * hd * 4);             // cos | sin rows of each row's position
    s.gain = o; o += a16((size_t)2 * hd * 4);                 // q_norm | k_norm gains
    s.etab = o; o += a16(128 * 4);                            // the EXP table (T | S)
    // reduce-scatter of the int32 p.V partials: with CS CTAs, CTA j finishes the
    // outputs [j*seg, (j+1)*seg), seg = ceil(M G hd / CS), and receives every
    // CTA's partials of that slice: CS * seg <= M G hd + CS words
    s.pvp = o;  o += a16(((size_t)M * G * hd + kMaxCluster) * 4);   // [source CTA][seg]
    s.ebuf = o; o += variant == 0 ? a16((size_t)T * 4) : 0;   // NORM: the whole row's e
    s.total = o;
    return s;
}

size_t attn_smem_needed(int rows, int heads, int kv_heads, int head_dim, int seq_len, int variant) {
    const AttnGeom g = attn_geom(seq_len);
    return attn_smem(rows, heads / kv_heads, head_dim, seq_len, g.chunk, variant).total;
}

bool attn_supported(int rows, int heads, int kv_heads, int head_dim, int seq_len, int variant) {
    const AttnGeom g = attn_geom(seq_len);
    return g.chunk <= kMaxChunk && attn_smem_needed(rows, heads, kv_heads, head_dim, seq_len, variant) <= 200 * 1024;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nanmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One head vector in shared memory (buf[hd], loaded by the warp): optional
// RMSNorm with gain g, then RoPE with the position's table rows; in place.
__device__ __forceinline__ void warp_norm_rope(float* buf, int hd, const float* g, float eps, float inv_hd,
                                               const float* cosr, const float* sinr, int lane,
                                               const SfuSmem* sf = nullptr) {
    if (g != nullptr) {
        const float ss = red_sum16([&](int i) { return fmul(buf[i], buf[i]); }, hd, lane);
        const float x = fadd(fmul(ss, inv_hd), eps);
        const float r = sf != nullptr ? sfu_rsqrt_s(x, sf) : sfu_rsqrt(x);
        for (int c = lane; c < hd; c += 32) buf[c] = fmul(fmul(buf[c], r), g[c]);
        __syncwarp();
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        if (c < hd) {
            const float sw = (c & 1) ? buf[c - 1] : -buf[c + 1];
            o[i] = fadd(fmul(buf[c], cosr[c]), fmul(sw, sinr[c]));
        }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        if (c < hd) buf[c] = o[i];
    }
    __syncwarp();
}

// The same head vector in registers: lane l holds elements c = l + 32 i (i < 8,
// c < hd). RMSNorm's ordered sum is red_sum16's: lane l < 16 adds the squares
// of elements l, l + 16, l + 32, ... in order (the odd groups come from lane
// l + 16), then the pairwise tree over the 16 lanes. RoPE's neighbour c ^ 1 is
// lane l ^ 1. Every value is the shared-memory form's bit for bit.
__device__ __forceinline__ void reg_norm_rope(float (&v)[8], int hd, const float* g, float eps, float inv_hd,
                                              const float* cosr, const float* sinr, int lane, const SfuSmem* sf) {
    if (g != nullptr) {
        float sq[8], pt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sq[i] = lane + 32 * i < hd ? fmul(v[i], v[i]) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) pt[i] = __shfl_down_sync(0xffffffffu, sq[i], 16);
        float acc = 0.f;
        if (lane < kLanes) {
            acc = sq[0];
            const int groups = hd / kLanes;
#pragma unroll
            for (int j = 1; j < 16; ++j)
                if (j < groups) acc = fadd(acc, (j & 1) ? pt[j >> 1] : sq[j >> 1]);
        }
#pragma unroll
        for (int s = 1; s < kLanes; s <<= 1) {
            const float o = __shfl_down_sync(0xffffffffu, acc, s);
            if ((lane & (2 * s - 1)) == 0) acc = fadd(acc, o);
        }
        const float r = sfu_rsqrt_s(fadd(fmul(__shfl_sync(0xffffffffu, acc, 0), inv_hd), eps), sf);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = lane + 32 * i;
            if (c < hd) v[i] = fmul(fmul(v[i], r), g[c]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float nb = __shfl_xor_sync(0xffffffffu, v[i], 1);
        const int c = lane + 32 * i;
        if (c < hd) v[i] = fadd(fmul(v[i], cosr[c]), fmul((c & 1) ? nb : -nb, sinr[c]));
    }
}

// HD: the head dimension as a compile-time constant (0: p.head_dim). The
// per-lane loops over a head vector (8 groups of 32 lanes, for head dims up to
// 256) then keep only the groups the head has: their code runs once per launch
// and is fetched cold, so the dead groups of a runtime bound cost time.
// VAR (0 NORM, 1 QSUM) and GRP (1: prefill groups, 0: decode rows) >= 0 fix
// the softmax variant and the row mode the same way (-1: from p).
template <int HD, int VAR = -1, int GRP = -1>
__global__ void __maxnreg__(104) attn_kernel(AttnParams p) {
    extern __shared__ __align__(128) unsigned char sm[];
    W8A8_TRACE_BEGIN(TR_ATTN);
    cg::cluster_group cl = cg::this_cluster();
    const int hd = HD > 0 ? HD : p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, T = p.seq_len;
    const int variant = VAR >= 0 ? VAR : p.variant;
    // batched decode: grid z is the slot (one row, its own position, qkv / att
    // rows and caches); prefill groups: z is a group of <= 16 rows of one
    // sequence (their K / V already in the cache); otherwise z = 0 and one
    // sequence's M rows
    const bool grp = GRP >= 0 ? GRP == 1 : p.groups > 0;
    const size_t b = blockIdx.z, r0 = grp ? b * kMaxRows : b;
    const int M = grp ? min(kMaxRows, p.rows - (int)r0) : p.rows;
    const int32_t* const pos_p = p.pos + r0;
    const float* const qkv_p = p.qkv + r0 * (size_t)(H + 2 * Hk) * hd;
    float* const att_p = p.att + r0 * (size_t)H * hd;
    int8_t* const kc_p = p.kc + (grp ? 0 : b * p.slot_stride);
    int8_t* const vc_p = p.vc + (grp ? 0 : b * p.slot_stride);
    const int CH = p.chunk, CS = p.nsplit, MG = M * G;
    const int kvh = blockIdx.x, rank = (int)cl.block_rank(), t0 = rank * CH, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int vpr = hd / 16, vstride = CH + 16;
    const int seg = (MG * hd + CS - 1) / CS;                  // outputs finished by each CTA
    const int qkv_dim = (H + 2 * Hk) * hd, q_dim = H * hd, kv_dim = Hk * hd;
    const AttnSmem L = attn_smem(M, G, hd, T, CH, variant);
    int8_t* ks = reinterpret_cast<int8_t*>(sm + L.ks);          // [CH][hd]
    int8_t* vs = reinterpret_cast<int8_t*>(sm + L.vs);          // [hd][CH + 16]: V transposed
    int8_t* qs = reinterpret_cast<int8_t*>(sm + L.qs);
    float* fbuf = reinterpret_cast<float*>(sm + L.fbuf);
    float* scs = reinterpret_cast<float*>(sm + L.scs);
    int8_t* ps = reinterpret_cast<int8_t*>(sm + L.ps);
    float* tabs = reinterpret_cast<float*>(sm + L.tab);         // row m: cos at [2m hd], sin at [(2m+1) hd]
    float* gains = reinterpret_cast<float*>(sm + L.gain);       // q_norm | k_norm
    uint32_t* etab = reinterpret_cast<uint32_t*>(sm + L.etab);  // EXP T | S
    int32_t* pvp = reinterpret_cast<int32_t*>(sm + L.pvp);
    float* ebuf = reinterpret_cast<float*>(sm + L.ebuf);
    __shared__ float lmax[kMaxCluster][kMaxRows * kMaxG];     // every CTA's chunk maxima (pushed by each)
    __shared__ float gmx[kMaxRows * kMaxG];
    __shared__ int lsum[kMaxCluster][kMaxRows * kMaxG];      // every CTA's sums of eq (pushed to all)
    __shared__ int wsum[kAttnWarps][kMaxRows * kMaxG];
    __shared__ float sq[kMaxRows * kMaxG];
    __shared__ float wred[kAttnWarps][kMaxRows * kMaxG];
    __shared__ float rsum;
    __shared__ int lim_s[kMaxRows];
    __shared__ uint32_t amx[kMaxRows];                         // max|att| bits per row (decode chain)
    __shared__ __align__(8) uint64_t tbar;                     // the cache tiles' bulk copies landed
    __shared__ SfuSmem sfs;                                    // RECIP / RSQRT on the critical path

    // every CTA of the cluster must have started before any remote store into its
    // shared memory: arrive now, wait just before the first push
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // ---- before the wait: positions, cache tiles of earlier positions, constant tables
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, pos_p[m]);
    const int nvalid = min(CH, maxpos + 1 - t0);
    const int nv16 = (nvalid + 15) & ~15;                      // V^T rows are read in 16-position words
    if (tid < M) lim_s[tid] = min(nvalid, pos_p[tid] + 1 - t0);  // positions of the chunk row m attends
    stage_exp_table(etab);
    stage_sfu(&sfs);                                           // (read after the barrier below the wait)
    // the chunk's cache tiles: K rows as one contiguous block by one 1-D bulk copy
    // (16-byte aligned: head_dim and the chunk start are multiples of 16), the
    // V^T rows (a short run of positions per channel: one bulk copy each would
    // queue hundreds of small copies) by 16-byte loads. Before the wait when they
    // hold earlier steps' rows; after it for prefill groups (the rows of this
    // call were appended by the kernel before)
    auto load_tiles = [&]() {
        if (tid == 0) {
            mbar_init(&tbar, 1);
            mbar_fence_init();
            mbar_expect_tx(&tbar, (uint32_t)(nvalid * hd));
            bulk_g2s(ks, kc_p + ((size_t)kvh * T + t0) * hd, (uint32_t)(nvalid * hd), &tbar);
        }
        // 4 words in flight per thread: a store waits for its load, so one
        // memory latency per 4 words, not per word
        const int vw = nv16 / 16, nw = hd * vw;               // 16-byte words per V^T row, in all
        for (int i0 = tid; i0 < nw; i0 += 4 * kAttnThreads) {
            int4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kAttnThreads, c = i / vw, w = i % vw;
                if (i < nw) v[u] = __ldcg(reinterpret_cast<const int4*>(vc_p + ((size_t)kvh * hd + c) * T + t0) + w);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kAttnThreads, c = i / vw, w = i % vw;
                if (i < nw) *reinterpret_cast<int4*>(vs + c * vstride + w * 16) = v[u];
            }
        }
    };
    if (nvalid > 0) {
        if (!grp) load_tiles();
        for (int i = tid; i < M * hd; i += kAttnThreads) {
            const int m = i / hd, c = i % hd, pos = pos_p[m];
            tabs[2 * m * hd + c] = __ldg(p.cos + (size_t)pos * hd + c);
            tabs[(2 * m + 1) * hd + c] = __ldg(p.sin + (size_t)pos * hd + c);
        }
        if (p.qk_norm)
            for (int c = tid; c < hd; c += kAttnThreads) {
                gains[c] = __ldg(p.q_norm + c);
                gains[hd + c] = __ldg(p.k_norm + c);
            }
    }
    W8A8_MARK(TR_ATTN, 14);
    pdl_wait();
    W8A8_MARK(TR_ATTN, 1);
    pdl_trigger();
    // the q rows of this warp's first (row, query head), and the K / V row of a
    // position in this chunk, loaded into registers now: their latency overlaps
    // the barrier below (the cache tiles' own stores must finish before a K / V
    // row is patched into them)
    const int r_first = warp;
    float qv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] = 0.f;
    if (nvalid > 0 && r_first < MG) {
        const int m = r_first / G, h = kvh * G + r_first % G;
        const float* src = qkv_p + (size_t)m * qkv_dim + (size_t)h * hd;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (lane + 32 * i < hd) qv[i] = src[lane + 32 * i];
    }
    if (grp && nvalid > 0) load_tiles();
    __syncthreads();
    W8A8_MARK(TR_ATTN, 8);
    bool tiles_ok = true;
    if (nvalid > 0) {
        // q path of every row and query head of this KV head (warps from 0), in
        // registers, and the K / V rows of the positions in this chunk (warps
        // from the last one) at the same time
        for (int r = warp; r < MG; r += kAttnWarps) {
            const int m = r / G, h = kvh * G + r % G;
            float v[8];
            if (r == r_first) {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = qv[i];
            } else {
                const float* src = qkv_p + (size_t)m * qkv_dim + (size_t)h * hd;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = lane + 32 * i < hd ? src[lane + 32 * i] : 0.f;
            }
            float kch[8];                                      // K per channel: its scale folded into q
#pragma unroll
            for (int i = 0; i < 8; ++i) kch[i] = p.k_ch != nullptr && lane + 32 * i < hd ? __ldg(p.k_ch + kvh * hd + lane + 32 * i) : 1.f;
            if (r == 0) W8A8_MARK(TR_ATTN, 10);
            reg_norm_rope(v, hd, p.qk_norm ? gains : nullptr, p.eps, p.inv_hd, tabs + 2 * m * hd,
                          tabs + (2 * m + 1) * hd, lane, &sfs);
            if (r == 0) W8A8_MARK(TR_ATTN, 11);
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (p.k_ch != nullptr) v[i] = fmul(v[i], kch[i]);
                if (lane + 32 * i < hd) a = nanmax(a, fabsf(v[i]));
            }
            a = warp_max(a);
            const float s = fmul(a, W8A8_C127);
            const float inv = sfu_recip_s(s, &sfs);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (lane + 32 * i < hd) qs[r * hd + lane + 32 * i] = (int8_t)to_i8(fmul(v[i], inv));
            if (lane == 0) sq[r] = s;
            if (r == 0) W8A8_MARK(TR_ATTN, 12);
        }
        // K and V rows of the positions in this chunk: into the cache and the tiles
        // (prefill groups: already in both)
        for (int m = kAttnWarps - 1 - warp; !grp && m < M; m += kAttnWarps) {
            const int pos = pos_p[m];
            if (pos < t0 || pos >= t0 + CH) continue;
            const float* ksrc = qkv_p + (size_t)m * qkv_dim + q_dim + (size_t)kvh * hd;
            const float* vsrc = ksrc + kv_dim;
            float kv[8], vv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const bool in = lane + 32 * i < hd;
                kv[i] = in ? ksrc[lane + 32 * i] : 0.f;
                vv[i] = in ? vsrc[lane + 32 * i] : 0.f;
            }
            reg_norm_rope(kv, hd, p.qk_norm ? gains + hd : nullptr, p.eps, p.inv_hd, tabs + 2 * m * hd,
                          tabs + (2 * m + 1) * hd, lane, &sfs);
            const bool landed = mbar_wait(&tbar, 0u);          // the tiles' copy first, then the patch
            if (!landed && lane == 0) atomicOr(&g_attn_errors, 4u);
            int8_t* kdst = kc_p + ((size_t)kvh * T + pos) * hd;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = lane + 32 * i;
                if (c >= hd) continue;
                const int8_t kq = (int8_t)to_i8(fmul(kv[i], p.inv_sk_ch ? p.inv_sk_ch[kvh * hd + c] : p.inv_sk));
                const int8_t vq = (int8_t)to_i8(fmul(vv[i], p.inv_sv_ch ? p.inv_sv_ch[kvh * hd + c] : p.inv_sv));
                kdst[c] = kq;
                vc_p[((size_t)kvh * hd + c) * T + pos] = vq;
                ks[(pos - t0) * hd + c] = kq;
                vs[c * vstride + (pos - t0)] = vq;
            }
            __syncwarp();
        }
        tiles_ok = mbar_wait(&tbar, 0u);                       // (issued before the wait: landed by now)
        if (!tiles_ok && tid == 0) atomicOr(&g_attn_errors, 4u);
        __syncthreads();
        W8A8_MARK(TR_ATTN, 2);
        // scores: thread t <-> positions t0 + t (+ 256); the row's 16-byte words are
        // read in a rotated order (conflict-free without padding)
        for (int r = 0; r < MG; ++r) {
            const int lim = lim_s[r / G];
            float mx = -INFINITY;
            for (int t = tid; t < lim; t += kAttnThreads) {
                int a = 0;
                const int4* kr = reinterpret_cast<const int4*>(ks + t * hd);
                const int4* qr = reinterpret_cast<const int4*>(qs + r * hd);
                int c = t % vpr;
#pragma unroll 8
                for (int j = 0; j < vpr; ++j) {
                    const int4 x = kr[c], y = qr[c];
                    c = c + 1 == vpr ? 0 : c + 1;
                    a = dp4a(x.x, y.x, a);
                    a = dp4a(x.y, y.y, a);
                    a = dp4a(x.z, y.z, a);
                    a = dp4a(x.w, y.w, a);
                }
                const float sc = fmul(fmul(i2f(a), sq[r]), p.a_k);
                scs[r * CH + t] = sc;
                mx = nanmax(mx, sc);
            }
            mx = warp_max(mx);
            if (lane == 0) wred[warp][r] = mx;
        }
        __syncthreads();
    }
    W8A8_MARK(TR_ATTN, 3);
    // this chunk's maxima, pushed into every CTA of the cluster (remote stores)
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    for (int i = tid; i < MG * CS; i += kAttnThreads) {
        const int r = i % MG, j = i / MG;
        float s = -INFINITY;
        if (nvalid > 0) {
            s = wred[0][r];
            for (int w = 1; w < kAttnWarps; ++w) s = nanmax(s, wred[w][r]);
        }
        *cl.map_shared_rank(&lmax[rank][r], j) = s;
    }
    cl.sync();                                                 // every chunk's maxima are in place
    W8A8_MARK(TR_ATTN, 4);
    if (tid < MG) {
        float mx = -INFINITY;
        for (int j = 0; j < CS; ++j) mx = nanmax(mx, lmax[j][tid]);
        gmx[tid] = mx;
    }
    __syncthreads();
    if (nvalid > 0) {
        if (variant == 0) {                                    // NORM: each row's whole e for the ordered sum
            for (int r = 0; r < MG; ++r) {
                const int m = r / G;
                const int lim = lim_s[m];
                if (lim > 0) {
                    const int n = pos_p[m] + 1;
                    const float mx = gmx[r];
                    for (int t = tid; t < n; t += kAttnThreads) {
                        const int j = t / CH;
                        const float s = *cl.map_shared_rank(scs + r * CH + (t - j * CH), j);
                        ebuf[t] = sfu_exp_tab(fsub(s, mx), etab, etab + 64);
                    }
                    __syncthreads();
                    if (warp == 0) {
                        const float ssum = red_sum16([&](int i) { return ebuf[i]; }, n, lane);
                        if (lane == 0) rsum = sfu_recip_s(ssum, &sfs);
                    }
                    __syncthreads();
                }
                const float rc = rsum;
                for (int t = tid; t < CH; t += kAttnThreads)
                    ps[r * CH + t] = t < lim ? (int8_t)to_i8(fmul(fmul(ebuf[t0 + t], rc), 127.f)) : (int8_t)0;
                __syncthreads();
            }
        } else {                                               // QSUM: this chunk's e only, all rows in one pass
            for (int r = 0; r < MG; ++r) {
                const int lim = lim_s[r / G];
                const float mx = gmx[r];
                int sum = 0;
                for (int t = tid; t < CH; t += kAttnThreads) {
                    int q = 0;
                    if (t < lim) q = to_i8(fmul(sfu_exp_tab(fsub(scs[r * CH + t], mx), etab, etab + 64), 127.f));
                    ps[r * CH + t] = (int8_t)q;
                    sum += q;
                }
                sum = warp_sum_i(sum);
                if (lane == 0) wsum[warp][r] = sum;
            }
            __syncthreads();
            for (int i = tid; i < MG * CS; i += kAttnThreads) {   // to every CTA
                const int r = i % MG, j = i / MG;
                int sum = 0;
                for (int w = 0; w < kAttnWarps; ++w) sum += wsum[w][r];
                *cl.map_shared_rank(&lsum[rank][r], j) = sum;
            }
        }
        __syncthreads();
        W8A8_MARK(TR_ATTN, 13);
        // p.V: thread <-> (row r, channel c) pairs; dp4a over 16-position words of
        // the int8 probabilities and the V^T row (padded: conflict-free)
        for (int i = tid; i < MG * hd; i += kAttnThreads) {
            const int r = i / hd, c = i % hd;
            const int words = (lim_s[r / G] + 15) / 16;
            const int4* pr = reinterpret_cast<const int4*>(ps + r * CH);
            const int4* vr = reinterpret_cast<const int4*>(vs + c * vstride);
            int a0 = 0, a1 = 0;
#pragma unroll 4
            for (int w = 0; w < words; ++w) {
                const int4 x = pr[w], y = vr[w];
                a0 = dp4a(x.x, y.x, a0);
                a1 = dp4a(x.y, y.y, a1);
                a0 = dp4a(x.z, y.z, a0);
                a1 = dp4a(x.w, y.w, a1);
            }
            const int own = i / seg;                           // the CTA that finishes output i
            *cl.map_shared_rank(pvp + rank * seg + (i - own * seg), own) = a0 + a1;
        }
    } else {
        for (int i = tid; i < MG * hd; i += kAttnThreads) {
            const int own = i / seg;
            *cl.map_shared_rank(pvp + rank * seg + (i - own * seg), own) = 0;
        }
        for (int i = tid; i < MG * CS; i += kAttnThreads) *cl.map_shared_rank(&lsum[rank][i % MG], i / MG) = 0;
    }
    W8A8_MARK(TR_ATTN, 5);
    cl.sync();                                                 // every CTA holds the partials of its slice
    W8A8_MARK(TR_ATTN, 6);
    {
        const bool post = p.amax_out != nullptr || p.amax_ll_out != nullptr;
        if (tid < kMaxRows) amx[tid] = 0u;
        if (post) __syncthreads();
        const int lo = rank * seg, hi = min(MG * hd, lo + seg);
        for (int i = lo + tid; i < hi; i += kAttnThreads) {
            const int r = i / hd, c = i % hd;
            const int m = r / G, h = kvh * G + r % G;
            int acc = 0, ssum = 0;
            for (int j = 0; j < CS; ++j) {
                acc += pvp[j * seg + (i - lo)];
                if (variant == 1) ssum += lsum[j][r];
            }
            const float o = i2f(acc);
            const float av = p.a_v_ch ? p.a_v_ch[kvh * hd + c] : p.a_v;   // V per channel or per layer
            float out;
            if (variant == 0) {
                out = fmul(o, av);
            } else {
                const float rq = fmul(sfu_recip_s(i2f(ssum), &sfs), 127.f);   // sum <= 127 T: exact in fp32
                out = fmul(fmul(o, rq), av);
            }
            att_p[((size_t)m * H + h) * hd + c] = out;
            if (post) atomicMax(&amx[m], __float_as_uint(fabsf(out)));
        }
        if (post) __syncthreads();
        if (p.amax_out != nullptr) {                           // max|att| per row for the o-projection
            if (tid < M && amx[tid] != 0u) atomicMax(p.amax_out + tid, amx[tid]);
        }
        if (p.amax_ll_out != nullptr && tid < kTpRows) {       // tensor parallel: to every rank
            const uint32_t ep = tp_epoch(p.tp);
            ll_post_cta(p.tp, p.amax_ll_out, kvh * (int)gridDim.y + rank, (int)(gridDim.x * gridDim.y), tid,
                        tid < M ? amx[tid] : 0u, ep);
        }
    }
    if (!tiles_ok) mbar_wait(&tbar, 0u);                      // no copy may land after the CTA exits
    W8A8_MARK(TR_ATTN, 7);
}

unsigned int attn_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_attn_errors, sizeof(v));
    cudaMemcpyToSymbol(g_attn_errors, &zero, sizeof(zero));
    return v;
}

// ---------------------------------------------------------------------------
// Batched decode: one CTA per (KV head, slot), no cluster. The slot's cache
// streams through a 3-stage ring filled by a producer warp: its K rows as TMA
// tiles of tp positions x head_dim, then its V^T rows by channel group (cg
// channels x positions 0 .. pos, one contiguous bulk copy per channel: V^T
// tiles along positions would read 128-byte pieces of 2 KB rows, which the
// HBM served at a third of its bandwidth); the scores of every position stay in shared memory, so the softmax
// (global max, EXP, int8 p; NORM's ordered sum over the whole row) needs no
// exchange. The current position's K / V row is written to the cache and
// patched into its tile when that tile lands. Same arithmetic, step for step,
// as the cluster kernel above (and so as a one-row decode).
// Ring stages and CTAs per SM of the batched kernel: 3 x 3 measured best at
// 128 slots of the Qwen3 shape (138 us; 4 stages x 2 CTAs 162 us)
#ifndef W8A8_SB_STAGES
#define W8A8_SB_STAGES 3
#endif
#ifndef W8A8_SB_TP
#define W8A8_SB_TP 128
#endif
#ifndef W8A8_SB_MINB
#define W8A8_SB_MINB 3
#endif
constexpr int kSbStages = W8A8_SB_STAGES;                      // ring stages (at least)
constexpr int kSbMaxStages = 8;                                // ring stages (at most)
constexpr int kSbTile = W8A8_SB_TP;                            // cache positions per tile (at most)
constexpr int kSbThreads = 288;                                // 8 compute warps + 1 producer warp
constexpr int kSbWarps = 8;

struct StreamMaps {
    CUtensorMap k;                                             // K rows [.][hd]
};

struct SbSmem {
    size_t ring, scs, ps, qs, fbuf, tab, gain, etab, newk, newv, total;
};

// bytes of a ring stage: a K tile (tp x hd), at least one V^T row (T)
__host__ __device__ inline size_t sb_stage(int hd, int T, int tp) {
    const size_t k = (size_t)tp * hd, tp_round = (size_t)((T + tp - 1) / tp * tp);
    return k > tp_round ? k : tp_round;
}

__host__ __device__ inline SbSmem sb_smem(int G, int hd, int T, int tp, int ns) {
    auto a16 = [](size_t b) { return (b + 15) & ~size_t(15); };
    const int Tp = (T + tp - 1) / tp * tp;
    SbSmem s{};
    size_t o = 0;
    s.ring = o; o += a16((size_t)ns * sb_stage(hd, T, tp));   // [stage]: a K tile or a V^T channel group
    s.scs = o;  o += a16((size_t)G * Tp * 4);                 // scores / e of every position, per row
    s.ps = o;   o += a16((size_t)G * Tp);                     // int8 p
    s.qs = o;   o += a16((size_t)G * hd);
    s.fbuf = o; o += a16((size_t)((G < kSbWarps ? G : kSbWarps) + 1) * hd * 4);   // fp32 q rows (a warp each), the K row
    s.tab = o;  o += a16((size_t)2 * hd * 4);                 // cos | sin of the slot's position
    s.gain = o; o += a16((size_t)2 * hd * 4);                 // q_norm | k_norm
    s.etab = o; o += a16(128 * 4);
    s.newk = o; o += a16((size_t)hd);                         // the new K / V rows (int8)
    s.newv = o; o += a16((size_t)hd);
    s.total = o;
    return s;
}

// HD, TP: head_dim and positions per K tile when known at compile time (the
// common shapes: constant indexing, unrolled dot loops), or 0: from the launch.
// MINB: CTAs an SM must hold by registers (4: for shapes whose shared memory
// allows 4, e.g. 64-dim heads with two query heads per KV head)
template <int HD, int TP, int MINB = W8A8_SB_MINB>
__global__ void __launch_bounds__(kSbThreads, MINB)
    attn_stream_kernel(const __grid_constant__ StreamMaps maps, AttnParams p, int tp_arg, int ns) {
    extern __shared__ __align__(128) unsigned char sm[];
    const int hd = HD > 0 ? HD : p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, T = p.seq_len;
    const int tp = TP > 0 ? TP : tp_arg;
    const int kvh = blockIdx.x, slot = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool producer = warp == kSbWarps;
    const int Tp = (T + tp - 1) / tp * tp;
    const int qkv_dim = (H + 2 * Hk) * hd, q_dim = H * hd, kv_dim = Hk * hd;
    const SbSmem L = sb_smem(G, hd, T, tp, ns);
    int8_t* ring = reinterpret_cast<int8_t*>(sm + L.ring);
    float* scs = reinterpret_cast<float*>(sm + L.scs);
    int8_t* ps = reinterpret_cast<int8_t*>(sm + L.ps);
    int8_t* qs = reinterpret_cast<int8_t*>(sm + L.qs);
    float* fbuf = reinterpret_cast<float*>(sm + L.fbuf);
    float* tabs = reinterpret_cast<float*>(sm + L.tab);
    float* gains = reinterpret_cast<float*>(sm + L.gain);
    uint32_t* etab = reinterpret_cast<uint32_t*>(sm + L.etab);
    int8_t* newk = reinterpret_cast<int8_t*>(sm + L.newk);
    int8_t* newv = reinterpret_cast<int8_t*>(sm + L.newv);
    __shared__ __align__(8) uint64_t full[kSbMaxStages], empty[kSbMaxStages];
    __shared__ float sq[kMaxG], gmx[kMaxG], wred[kSbWarps][kMaxG], rcp[kMaxG];
    __shared__ int wsum[kSbWarps][kMaxG], lsum[kMaxG];
    __shared__ float rqs[kMaxG];                               // QSUM: RECIP(sum eq) * 127 per row
    __shared__ SfuSmem sfs;                                    // RECIP / RSQRT (q path, softmax scales)
    __shared__ int failed;
    const int pos = p.pos[slot];                               // written by an earlier step: read before the wait
    const int nt = pos / tp + 1;                               // K tiles with positions <= pos
    const size_t krow0 = (size_t)slot * (p.slot_stride / hd) + (size_t)kvh * T;
    const int8_t* vbase = p.vc + (size_t)slot * p.slot_stride + (size_t)kvh * hd * T;   // this head's V^T rows
    const uint32_t tile_bytes = (uint32_t)(tp * hd);             // a K tile
    const size_t stage_bytes = sb_stage(hd, T, tp);
    // V^T tiles by channel group: cg channels x positions [0, nv) each, every
    // channel's run one contiguous bulk copy (sequential HBM reads); cg the
    // largest divisor of hd, at most 16 (copies per tile), whose tile fits a stage
    const int nv = ((pos + 1) + 15) & ~15;
    int cg = hd < 16 ? hd : 16;
    while (cg > 1 && (hd % cg != 0 || (size_t)cg * nv > stage_bytes)) --cg;
    const int nvt = hd / cg, ntiles = nt + nvt;
    if (tid == 0) {
        failed = 0;
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSbWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int i) {                                  // ring tile i: K tile i, then V tile i - nt
        const int s = i % ns;
        int8_t* dst = ring + (size_t)s * stage_bytes;
        if (i < nt) {
            mbar_expect_tx(&full[s], tile_bytes);
            tma_load_2d(dst, &maps.k, 0, (int)(krow0 + (size_t)i * tp), &full[s]);
        } else {
            const int c0 = (i - nt) * cg;
            mbar_expect_tx(&full[s], (uint32_t)(cg * nv));
            for (int c = 0; c < cg; ++c) bulk_g2s(dst + (size_t)c * nv, vbase + (size_t)(c0 + c) * T, (uint32_t)nv, &full[s]);
        }
    };
    if (producer && lane == 0)                                 // cache rows of earlier steps: before the wait
        for (int i = 0; i < ns && i < ntiles; ++i) issue(i);
    stage_exp_table(etab);
    stage_sfu(&sfs);                                           // (read after the barrier below the wait)
    for (int c = tid; c < hd; c += kSbThreads) {
        tabs[c] = __ldg(p.cos + (size_t)pos * hd + c);
        tabs[hd + c] = __ldg(p.sin + (size_t)pos * hd + c);
        if (p.qk_norm) {
            gains[c] = __ldg(p.q_norm + c);
            gains[hd + c] = __ldg(p.k_norm + c);
        }
    }
    pdl_wait();
    pdl_trigger();
    __syncthreads();

    if (producer) {
        if (lane == 0) {                                       // refill each stage once the 8 warps are done
            for (int i = ns; i < ntiles; ++i) {
                const int s = i % ns;
                if (!mbar_wait(&empty[s], (uint32_t)(((i / ns) - 1) & 1))) {   // suspends: no issue slots
                    atomicOr(&g_attn_errors, 4u);
                    failed = 1;
                    break;
                }
                issue(i);
            }
        }
    } else {
        const float* qrow = p.qkv + (size_t)slot * qkv_dim;
        // q path (warps from 0) and this position's K / V rows (the last warp)
        for (int r = warp; r < G; r += kSbWarps) {
            float* buf = fbuf + warp * hd;
            const float* src = qrow + (size_t)(kvh * G + r) * hd;
            for (int c = lane; c < hd; c += 32) buf[c] = src[c];
            __syncwarp();
            warp_norm_rope(buf, hd, p.qk_norm ? gains : nullptr, p.eps, p.inv_hd, tabs, tabs + hd, lane, &sfs);
            if (p.k_ch != nullptr) {                           // K per channel: its scale folded into q
                for (int c = lane; c < hd; c += 32) buf[c] = fmul(buf[c], p.k_ch[kvh * hd + c]);
                __syncwarp();
            }
            float a = 0.f;
            for (int c = lane; c < hd; c += 32) a = nanmax(a, fabsf(buf[c]));
            a = warp_max(a);
            const float sc = fmul(a, W8A8_C127);
            const float inv = sfu_recip_s(sc, &sfs);
            for (int c = lane; c < hd; c += 32) qs[r * hd + c] = (int8_t)to_i8(fmul(buf[c], inv));
            if (lane == 0) sq[r] = sc;
            __syncwarp();
        }
        if (warp == kSbWarps - 1) {
            float* kb = fbuf + (G < kSbWarps ? G : kSbWarps) * hd;   // after the q rows' buffers
            const float* ksrc = qrow + q_dim + (size_t)kvh * hd;
            const float* vsrc = qrow + q_dim + kv_dim + (size_t)kvh * hd;
            for (int c = lane; c < hd; c += 32) kb[c] = ksrc[c];
            __syncwarp();
            warp_norm_rope(kb, hd, p.qk_norm ? gains + hd : nullptr, p.eps, p.inv_hd, tabs, tabs + hd, lane, &sfs);
            int8_t* kdst = p.kc + (size_t)slot * p.slot_stride + ((size_t)kvh * T + pos) * hd;
            int8_t* vdst = p.vc + (size_t)slot * p.slot_stride + (size_t)kvh * hd * T + pos;
            for (int c = lane; c < hd; c += 32) {
                const int8_t kq = (int8_t)to_i8(fmul(kb[c], p.inv_sk_ch ? p.inv_sk_ch[kvh * hd + c] : p.inv_sk));
                const int8_t vq = (int8_t)to_i8(fmul(vsrc[c], p.inv_sv_ch ? p.inv_sv_ch[kvh * hd + c] : p.inv_sv));
                kdst[c] = kq;
                vdst[(size_t)c * T] = vq;
                newk[c] = kq;
                newv[c] = vq;
            }
        }
        named_barrier_sync(1, kSbWarps * 32);                  // q rows and the new K / V rows are ready
        // ---- pass 1: scores of positions <= pos; thread <-> (row, position of the tile)
        const int vpr = hd / 16;
        // running maxima: with a compile-time tile that divides the 256 consumer
        // threads, pass k of a thread is always row tid / TP + k * (256 / TP) (one
        // per warp); otherwise one per row, selected per position
        constexpr bool kRowOf = TP > 0 && (kSbWarps * 32) % (TP > 0 ? TP : 1) == 0;
        constexpr int kPasses = kRowOf ? (kMaxG * TP + kSbWarps * 32 - 1) / (kSbWarps * 32) : 1;
        float mk[kPasses];
#pragma unroll
        for (int k = 0; k < kPasses; ++k) mk[k] = -INFINITY;
        float mx[kRowOf ? 1 : kMaxG];
#pragma unroll
        for (int r = 0; r < (kRowOf ? 1 : kMaxG); ++r) mx[r] = -INFINITY;
        for (int i = 0; i < nt; ++i) {
            const int s = i % ns;
            if (!mbar_wait(&full[s], (uint32_t)((i / ns) & 1))) {   // (suspends: no polling issue slots)
                if (tid == 0) atomicOr(&g_attn_errors, 4u);
                failed = 1;
            }
            int8_t* kt = ring + (size_t)s * stage_bytes;        // [tp][hd]
            if (i == nt - 1) {                                 // the tile holding pos: the new K row
                if (tid < hd / 16) {
                    reinterpret_cast<int4*>(kt + (size_t)(pos - i * tp) * hd)[tid] = reinterpret_cast<const int4*>(newk)[tid];
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // before the stage's next copy
                }
                named_barrier_sync(1, kSbWarps * 32);
            }
#pragma unroll
            for (int k = 0; k < (kRowOf ? kPasses : 1); ++k)
            for (int pr = tid + k * kSbWarps * 32; pr < G * tp; pr += (kRowOf ? kPasses : 1) * kSbWarps * 32) {
                const int r = pr / tp, t = pr % tp, tpos = i * tp + t;
                if (tpos > pos) continue;
                const int4* kr = reinterpret_cast<const int4*>(kt + (size_t)t * hd);
                const int4* qr = reinterpret_cast<const int4*>(qs + r * hd);
                int a = 0;
                if (HD > 0) {                                  // rows' words in a rotated order: conflict-free
                    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;        // four independent chains
#pragma unroll
                    for (int j = 0; j < HD / 16; ++j) {
                        const int c = (t + j) & (HD / 16 - 1);
                        const int4 x = kr[c], y = qr[c];
                        a0 = dp4a(x.x, y.x, a0);
                        a1 = dp4a(x.y, y.y, a1);
                        a2 = dp4a(x.z, y.z, a2);
                        a3 = dp4a(x.w, y.w, a3);
                    }
                    a = (a0 + a1) + (a2 + a3);
                } else {
                    int c = t % vpr;
                    for (int j = 0; j < vpr; ++j) {
                        const int4 x = kr[c], y = qr[c];
                        c = c + 1 == vpr ? 0 : c + 1;
                        a = dp4a(x.x, y.x, a);
                        a = dp4a(x.y, y.y, a);
                        a = dp4a(x.z, y.z, a);
                        a = dp4a(x.w, y.w, a);
                    }
                }
                const float sc = fmul(fmul(i2f(a), sq[r]), p.a_k);
                scs[r * Tp + tpos] = sc;
                if constexpr (kRowOf) {
                    mk[k] = nanmax(mk[k], sc);
                } else {
#pragma unroll
                    for (int rr = 0; rr < (kRowOf ? 1 : kMaxG); ++rr)
                        if (rr == r) mx[rr] = nanmax(mx[rr], sc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if constexpr (kRowOf) {
            if (lane < G) wred[warp][lane] = -INFINITY;              // rows this warp never visits
            __syncwarp();
#pragma unroll
            for (int k = 0; k < kPasses; ++k) {
                const int pr0 = warp * 32 + k * kSbWarps * 32;      // the warp's first (row, position)
                const float m = warp_max(mk[k]);
                if (lane == 0 && pr0 < G * tp) wred[warp][pr0 / TP] = m;
            }
        } else {
#pragma unroll
            for (int r = 0; r < (kRowOf ? 1 : kMaxG); ++r) {
                const float m = warp_max(mx[r]);
                if (lane == 0 && r < G) wred[warp][r] = m;
            }
        }
        named_barrier_sync(1, kSbWarps * 32);
        if (tid < G) {
            float m = wred[0][tid];
            for (int w = 1; w < kSbWarps; ++w) m = nanmax(m, wred[w][tid]);
            gmx[tid] = m;
        }
        named_barrier_sync(1, kSbWarps * 32);
        // ---- the softmax over positions 0 .. pos of every row (row by row, four
        // positions per thread)
        const int n = pos + 1;
        constexpr int kC = kSbWarps * 32;                      // consumer threads
        if (p.variant == 0) {                                  // NORM: e, the ordered sum, p = i8(127 e / sum)
            for (int r = 0; r < G; ++r) {
                float* er = scs + r * Tp;
                const float m = gmx[r];
                for (int t = tid; t < n; t += kC) er[t] = sfu_exp_tab(fsub(er[t], m), etab, etab + 64);
            }
            named_barrier_sync(1, kSbWarps * 32);
            for (int r = warp; r < G; r += kSbWarps) {
                const float* er = scs + r * Tp;
                const float ssum = red_sum16([&](int i) { return er[i]; }, n, lane);
                if (lane == 0) rcp[r] = sfu_recip_s(ssum, &sfs);
            }
            named_barrier_sync(1, kSbWarps * 32);
            for (int r = 0; r < G; ++r) {
                const float* er = scs + r * Tp;
                const float rr = rcp[r];
                for (int t4 = 4 * tid; t4 < Tp; t4 += 4 * kC) {
                    int q[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        q[u] = t4 + u < n ? to_i8(fmul(fmul(er[t4 + u], rr), 127.f)) : 0;
                    *reinterpret_cast<char4*>(ps + r * Tp + t4) = make_char4(q[0], q[1], q[2], q[3]);
                }
            }
        } else {                                               // QSUM: eq = i8(127 e) and its exact sum
            for (int r = 0; r < G; ++r) {
                const float* sr = scs + r * Tp;
                const float m = gmx[r];
                int sum = 0;
                for (int t4 = 4 * tid; t4 < Tp; t4 += 4 * kC) {
                    int q[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        q[u] = t4 + u < n ? to_i8(fmul(sfu_exp_tab(fsub(sr[t4 + u], m), etab, etab + 64), 127.f)) : 0;
                    *reinterpret_cast<char4*>(ps + r * Tp + t4) = make_char4(q[0], q[1], q[2], q[3]);
                    sum += (q[0] + q[1]) + (q[2] + q[3]);
                }
                sum = warp_sum_i(sum);
                if (lane == 0) wsum[warp][r] = sum;
            }
            named_barrier_sync(1, kSbWarps * 32);
            if (tid < G) {
                int v = 0;
                for (int w = 0; w < kSbWarps; ++w) v += wsum[w][tid];
                lsum[tid] = v;
                rqs[tid] = fmul(sfu_recip_s(i2f(v), &sfs), 127.f);   // sum <= 127 T: exact in fp32
            }
        }
        named_barrier_sync(1, kSbWarps * 32);
        // ---- pass 2: p.V over the channel-group tiles: each output (row r,
        // channel c) is one dot product of p[r][0, nv) with V^T[c][0, nv) inside
        // one tile (positions past pos have p = 0); 16 threads per output, a
        // shuffle sum (int32: exact in any order)
        float* att = p.att + (size_t)slot * q_dim;
        uint32_t am = 0u;
        const int nw = nv / 16, sl = tid & 15;                  // 16-byte words per row; this thread's slice
        for (int j = 0; j < nvt; ++j) {
            const int ri = nt + j, s = ri % ns, c0 = j * cg;
            if (!mbar_wait(&full[s], (uint32_t)((ri / ns) & 1))) {
                if (tid == 0) atomicOr(&g_attn_errors, 4u);
                failed = 1;
            }
            const int8_t* vt = ring + (size_t)s * stage_bytes;  // [cg][nv]
            for (int o0 = 0; o0 < G * cg; o0 += kSbWarps * 32 / 16) {
                const int o = o0 + (tid >> 4);
                const int r = o / cg, cl = o - r * cg;
                int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
                if (o < G * cg) {
                    const int4* vr = reinterpret_cast<const int4*>(vt + (size_t)cl * nv);
                    const int4* pp = reinterpret_cast<const int4*>(ps + (size_t)r * Tp);
                    for (int w = sl; w < nw; w += 16) {
                        const int4 x = pp[w], y = vr[w];
                        a0 = dp4a(x.x, y.x, a0);
                        a1 = dp4a(x.y, y.y, a1);
                        a2 = dp4a(x.z, y.z, a2);
                        a3 = dp4a(x.w, y.w, a3);
                    }
                }
                int a = (a0 + a1) + (a2 + a3);
#pragma unroll
                for (int m = 8; m > 0; m >>= 1) a += __shfl_xor_sync(0xffffffffu, a, m);
                if (sl == 0 && o < G * cg) {
                    const int c = c0 + cl;
                    // the copy brought the cache's column pos before or after this
                    // step's write: exchange it for the new V value (exact int32)
                    const int pq = ps[(size_t)r * Tp + pos];
                    a += pq * ((int)newv[c] - (int)vt[(size_t)cl * nv + pos]);
                    const float ov = i2f(a);
                    const float av = p.a_v_ch ? p.a_v_ch[kvh * hd + c] : p.a_v;   // V per channel or per layer
                    float out;
                    if (p.variant == 0) out = fmul(ov, av);
                    else out = fmul(fmul(ov, rqs[r]), av);
                    att[(size_t)(kvh * G + r) * hd + c] = out;
                    am = max(am, __float_as_uint(fabsf(out)));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (p.amax_out != nullptr) {                           // max|att| of the slot's row (decode chain)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) am = max(am, __shfl_xor_sync(0xffffffffu, am, o));
            if (lane == 0 && am != 0u) atomicMax(p.amax_out + slot, am);
        }
    }
    __syncthreads();
    if (failed && producer && lane == 0)                       // no copy may land after the CTA exits
        for (int s = 0; s < ns; ++s) mbar_wait(&full[s], 0u), mbar_wait(&full[s], 1u);
}

size_t attn_stream_smem(int heads, int kv_heads, int head_dim, int seq_len) {
    const int tp = seq_len < kSbTile ? seq_len : kSbTile, G = heads / kv_heads;
    return sb_smem(G, head_dim, seq_len, tp, kSbStages).total;             // (the launch may add stages)
}

using SbKernel = void (*)(StreamMaps, AttnParams, int, int);

// Ring stages: the most CTAs on an SM first, then as many stages as keep that
// count (small stages, as at head_dim 64, then hold more bytes in flight); at
// least kSbStages. Each host thread keeps its last answer (one shape per model).
static int sb_stages(SbKernel kern, int G, int hd, int T, int tp) {
    static thread_local SbKernel c_kern = nullptr;
    static thread_local int c_key[4] = {0, 0, 0, 0}, c_ns = 0;
    if (kern == c_kern && c_key[0] == G && c_key[1] == hd && c_key[2] == T && c_key[3] == tp) return c_ns;
    int best = kSbStages, occ_best = -1;
    for (int ns = kSbStages; ns <= kSbMaxStages; ++ns) {
        const size_t smem = sb_smem(G, hd, T, tp, ns).total;
        if (smem > 200 * 1024) break;
        int occ = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSbThreads, smem) != cudaSuccess)
            break;
        if (occ >= occ_best && occ > 0) best = ns, occ_best = occ;
    }
    c_kern = kern, c_key[0] = G, c_key[1] = hd, c_key[2] = T, c_key[3] = tp, c_ns = best;
    return best;
}

cudaError_t launch_attn_stream(const AttnParams& p, cudaStream_t st) {
    const int hd = p.head_dim, T = p.seq_len, G = p.heads / p.kv_heads;
    const int tp = T < kSbTile ? T : kSbTile;
    const size_t slot_k_rows = p.slot_stride / hd;
    StreamMaps maps{};
    const uint64_t krows = (uint64_t)(p.slots - 1) * slot_k_rows + (uint64_t)p.kv_heads * T;
    if (!make_map_u8(&maps.k, p.kc, (uint64_t)hd, krows, (uint64_t)hd, (uint32_t)hd, (uint32_t)tp, false))
        return cudaErrorInvalidValue;
    SbKernel kern = hd == 128 && tp == 128 ? attn_stream_kernel<128, 128>
                    : hd == 64 && tp == 128 ? attn_stream_kernel<64, 128> : attn_stream_kernel<0, 0>;
    if (hd == 64 && tp == 128) {                               // 4 CTAs on an SM where the memory allows it
        SbKernel k4 = attn_stream_kernel<64, 128, 4>;
        const size_t sm3 = sb_smem(G, hd, T, tp, kSbStages).total;
        int occ = 0;
        if (sm3 <= 200 * 1024 &&
            cudaFuncSetAttribute(k4, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm3) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k4, kSbThreads, sm3) == cudaSuccess && occ >= 4)
            kern = k4;
    }
    const int ns = sb_stages(kern, G, hd, T, tp);
    const size_t smem = sb_smem(G, hd, T, tp, ns).total;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return launch_k(kern, dim3(p.kv_heads, p.slots), dim3(kSbThreads), smem, st, maps, p, tp, ns);
}

// Prefill: every row's K and V (QK-norm + RoPE + int8, the attention kernel's
// own arithmetic) into the cache, before one attention launch over all the
// rows' groups. One CTA per row, one warp per KV head.
__global__ void __launch_bounds__(kAttnThreads) kv_append_kernel(AttnParams p) {
    extern __shared__ __align__(16) unsigned char kv_sm[];
    const int hd = p.head_dim, H = p.heads, Hk = p.kv_heads, T = p.seq_len;
    const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int qkv_dim = (H + 2 * Hk) * hd, q_dim = H * hd, kv_dim = Hk * hd;
    float* buf = reinterpret_cast<float*>(kv_sm) + warp * hd;
    pdl_wait();
    pdl_trigger();
    const int pos = p.pos[m];
    const float* row = p.qkv + (size_t)m * qkv_dim;
    for (int h = warp; h < Hk; h += kAttnWarps) {
        for (int c = lane; c < hd; c += 32) buf[c] = row[q_dim + h * hd + c];
        __syncwarp();
        warp_norm_rope(buf, hd, p.qk_norm ? p.k_norm : nullptr, p.eps, p.inv_hd, p.cos + (size_t)pos * hd,
                       p.sin + (size_t)pos * hd, lane);
        const float* vsrc = row + q_dim + kv_dim + (size_t)h * hd;
        for (int c = lane; c < hd; c += 32) {
            p.kc[((size_t)h * T + pos) * hd + c] =
                (int8_t)to_i8(fmul(buf[c], p.inv_sk_ch ? p.inv_sk_ch[h * hd + c] : p.inv_sk));
            p.vc[((size_t)h * hd + c) * T + pos] =
                (int8_t)to_i8(fmul(vsrc[c], p.inv_sv_ch ? p.inv_sv_ch[h * hd + c] : p.inv_sv));
        }
        __syncwarp();
    }
}

cudaError_t launch_kv_append(const AttnParams& p, cudaStream_t st) {
    const size_t smem = (size_t)kAttnWarps * p.head_dim * 4;
    return launch_k(kv_append_kernel, dim3(p.rows), dim3(kAttnThreads), smem, st, p);
}

using AttnKern = void (*)(AttnParams);

// The instance for a head dim: decode rows with the variant compiled in, or
// prefill groups (either variant).
template <int HD>
static AttnKern attn_pick(int variant, bool grp) {
    if (grp) return attn_kernel<HD, -1, 1>;
    return variant == 0 ? attn_kernel<HD, 0, 0> : attn_kernel<HD, 1, 0>;
}

cudaError_t launch_attn(const AttnParams& q, cudaStream_t st) {
    AttnParams p = q;
    const AttnGeom g = attn_geom(p.seq_len);
    p.nsplit = g.cs;
    p.chunk = g.chunk;
    const int mr = p.groups > 0 ? (p.rows < kMaxRows ? p.rows : kMaxRows) : p.rows;   // rows of a CTA, at most
    const AttnSmem L = attn_smem(mr, p.heads / p.kv_heads, p.head_dim, p.seq_len, p.chunk, p.variant);
    const bool grp = p.groups > 0;
    const int var = p.variant;
    auto kern = p.head_dim == 128 ? attn_pick<128>(var, grp)
              : p.head_dim == 64  ? attn_pick<64>(var, grp)
              : p.head_dim == 48  ? attn_pick<48>(var, grp)
                                  : attn_kernel<0>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    // one shared-memory carveout for every kernel of the chain: no L1 / shared
    // reconfiguration of an SM between consecutive kernels
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.kv_heads, g.cs, p.slots > 0 ? p.slots : p.groups > 0 ? p.groups : 1);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = g.cs;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_use_pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace w8a8
