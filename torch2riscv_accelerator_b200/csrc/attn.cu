// Fused per-layer attention over the int8 KV cache, for one sequence's M rows
// (a decode step: M = 1; a prefill chunk: M = 16 rows, each exactly a decode
// row, `compiler/frontend/hf_generic.py:306-363`, `docs/fusion_design.md`
// 6.7: the chunk's K/V rows are written first, each head's cache is read once
// per chunk).
//
// Three launches per layer (stream-ordered, no spin waits):
//  1. attn_prep   per (row, head slot): QK-norm (RMSNorm over head_dim, ordered
//                 sum), RoPE (v*cos + swapneg(v)*sin), then
//                 q: quant_act per head -> int8 q, s_q;
//                 k: i8(k*inv_sk) -> cache; v: i8(v*inv_sv) -> cache
//                 (llm/ref_model.py:225-229, hf_generic.SaCache.update :190-226).
//  2. attn_scores per (KV head, 128-position chunk): the chunk of K is read
//                 once into shared memory for all rows and the G query heads of
//                 the group; scores (f32(qq.k)*s_q)*a_k; per-chunk maxima. The
//                 last CTA of the KV head (atomic ticket) does the softmax of
//                 its rows over the whole valid range: m = max,
//                 e = EXP(s - m); NORM: p = e*RECIP(red_sum16(e)), pq = i8(127p);
//                 QSUM: eq = i8(127e), rq = RECIP(sum eq)*127
//                 (llm/ref_model.py:233-242; hf_generic.py:275-290).
//                 The global max comes before any int8 rounding: no online
//                 softmax (docs/fusion_design.md: p's int8 rounding equals
//                 decode's).
//  3. attn_pv     per (KV head, chunk): int32 pq.V partials (exact in any
//                 order); the last CTA of the KV head sums the partials and
//                 dequantizes: NORM f32(acc)*a_v; QSUM (f32(acc)*rq)*a_v.
// Cache layout: [kv_heads, seq_len, head_dim] int8 per layer (a head's chunk is
// one contiguous block).
#include "w8a8_internal.h"
#include "w8a8_math.cuh"

namespace w8a8 {

size_t attn_scratch_bytes(int rows, int heads, int kv_heads, int head_dim, int seq_len) {
    const size_t M = rows, H = heads, hd = head_dim, T = seq_len;
    const size_t ns = (T + kChunk - 1) / kChunk;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    return al(M * H * hd) + al(M * H * 4) + al(M * H * T * 4) + al(M * H * ns * 4) + al(M * H * T) +
           al(M * H * 4) + al(M * H * ns * hd * 4) + al(2 * (size_t)kv_heads * 4);
}

void attn_carve(AttnParams& p, void* scratch) {
    const size_t M = p.rows, H = p.heads, hd = p.head_dim, T = p.seq_len;
    const size_t ns = (T + kChunk - 1) / kChunk;
    p.nsplit = (int)ns;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    char* c = static_cast<char*>(scratch);
    p.qq = reinterpret_cast<int8_t*>(c);
    c += al(M * H * hd);
    p.s_q = reinterpret_cast<float*>(c);
    c += al(M * H * 4);
    p.sc = reinterpret_cast<float*>(c);
    c += al(M * H * T * 4);
    p.pmax = reinterpret_cast<float*>(c);
    c += al(M * H * ns * 4);
    p.pq = reinterpret_cast<int8_t*>(c);
    c += al(M * H * T);
    p.rq = reinterpret_cast<float*>(c);
    c += al(M * H * 4);
    p.part = reinterpret_cast<int32_t*>(c);
    c += al(M * H * ns * hd * 4);
    p.cnt = reinterpret_cast<uint32_t*>(c);
}

// ---------------------------------------------------------------- 1. prep
__global__ void __launch_bounds__(256) attn_prep(AttnParams p) {
    __shared__ float v[256];
    __shared__ float red[32];
    __shared__ float rr;
    const int m = blockIdx.x, slot = blockIdx.y, c = threadIdx.x, lane = c & 31;
    const int H = p.heads, Hk = p.kv_heads, hd = p.head_dim;
    const int pos = p.pos[m];
    const int qkv_dim = (H + 2 * Hk) * hd;
    const float* src = p.qkv + (size_t)m * qkv_dim + (size_t)slot * hd;   // q heads | k heads | v heads
    const bool is_q = slot < H, is_k = !is_q && slot < H + Hk;
    if (c < hd) v[c] = src[c];
    __syncthreads();
    if (!is_q && !is_k) {                                      // V row
        const int kvh = slot - H - Hk;
        if (c < hd) p.vc[((size_t)kvh * p.seq_len + pos) * hd + c] = (int8_t)to_i8(fmul(v[c], p.inv_sv));
        return;
    }
    if (p.qk_norm) {                                           // RMSNorm over the head (qhf.py:335-337)
        const float* g = is_q ? p.q_norm : p.k_norm;
        if (c < 32) {
            float ss = red_sum16([&](int i) { return fmul(v[i], v[i]); }, hd, lane);
            if (lane == 0) rr = sfu_rsqrt(fadd(fmul(ss, p.inv_hd), p.eps));
        }
        __syncthreads();
        float y = c < hd ? fmul(fmul(v[c], rr), g[c]) : 0.f;
        __syncthreads();
        if (c < hd) v[c] = y;
        __syncthreads();
    }
    float o = 0.f;
    if (c < hd) {                                              // RoPE: (v*cos) + (swapneg(v)*sin)
        const float sw = (c & 1) ? v[c - 1] : -v[c + 1];
        o = fadd(fmul(v[c], p.cos[(size_t)pos * hd + c]), fmul(sw, p.sin[(size_t)pos * hd + c]));
    }
    if (is_k) {
        const int kvh = slot - H;
        if (c < hd) p.kc[((size_t)kvh * p.seq_len + pos) * hd + c] = (int8_t)to_i8(fmul(o, p.inv_sk));
        return;
    }
    // q: quant_act per head
    float a = block_nanmax(c < hd ? fabsf(o) : 0.f, red);
    const float s = fmul(a, W8A8_C127);
    const float inv = sfu_recip(s);
    if (c < hd) p.qq[((size_t)m * H + slot) * hd + c] = (int8_t)to_i8(fmul(o, inv));
    if (c == 0) p.s_q[(size_t)m * H + slot] = s;
}

// ---------------------------------------------------------------- 2. scores
constexpr int kMaxG = 8;                                       // query heads per KV head
constexpr int kMaxHd = 256;

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nanmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void __launch_bounds__(kChunk) attn_scores(AttnParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int hd = p.head_dim, H = p.heads, G = H / p.kv_heads, M = p.rows, T = p.seq_len;
    const int kvh = blockIdx.x, split = blockIdx.y, t0 = split * kChunk, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int kstride = hd + 16;                               // padded rows: conflict-free 16-byte reads
    int8_t* ks = reinterpret_cast<int8_t*>(sm);                // [kChunk][hd + 16]
    int8_t* qs = ks + kChunk * kstride;                        // [M*G][hd]
    __shared__ float wmax[kChunk / 32][kMaxRows * kMaxG];
    __shared__ float sq[kMaxRows * kMaxG];
    __shared__ int last;
    __shared__ float red[32];
    __shared__ int redi[32];
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, p.pos[m]);
    const int nvalid = max(0, min(kChunk, maxpos + 1 - t0));
    if (nvalid > 0) {
        const int vpr = hd / 16;                               // 16-byte vectors per row
        const int8_t* kbase = p.kc + ((size_t)kvh * T + t0) * hd;
        for (int i = tid; i < nvalid * vpr; i += kChunk) {
            const int t = i / vpr, c = i % vpr;
            *reinterpret_cast<int4*>(ks + t * kstride + c * 16) =
                __ldg(reinterpret_cast<const int4*>(kbase + (size_t)t * hd) + c);
        }
        for (int i = tid; i < M * G * vpr; i += kChunk) {
            const int r = i / vpr, c = i % vpr, m = r / G, g = r % G;
            *reinterpret_cast<int4*>(qs + r * hd + c * 16) =
                *reinterpret_cast<const int4*>(p.qq + ((size_t)m * H + kvh * G + g) * hd + c * 16);
        }
        if (tid < M * G) sq[tid] = p.s_q[(size_t)(tid / G) * H + kvh * G + tid % G];
        __syncthreads();
        const int t = t0 + tid;
        for (int r = 0; r < M * G; ++r) {
            const int m = r / G, h = kvh * G + r % G;
            float s = -INFINITY;
            if (tid < nvalid && t <= p.pos[m]) {
                int acc = 0;
                const int4* kr = reinterpret_cast<const int4*>(ks + tid * kstride);
                const int4* qr = reinterpret_cast<const int4*>(qs + r * hd);
                for (int c = 0; c < hd / 16; ++c) {
                    const int4 a = kr[c], b = qr[c];
                    acc = dp4a(a.x, b.x, acc);
                    acc = dp4a(a.y, b.y, acc);
                    acc = dp4a(a.z, b.z, acc);
                    acc = dp4a(a.w, b.w, acc);
                }
                s = fmul(fmul(i2f(acc), sq[r]), p.a_k);
                p.sc[((size_t)m * H + h) * T + t] = s;
            }
            s = warp_max_f(s);
            if (lane == 0) wmax[warp][r] = s;
        }
        __syncthreads();
        if (tid < M * G) {
            float s = wmax[0][tid];
            for (int w = 1; w < kChunk / 32; ++w) s = nanmax(s, wmax[w][tid]);
            const int m = tid / G, h = kvh * G + tid % G;
            p.pmax[((size_t)m * H + h) * p.nsplit + split] = s;
        }
    }
    // the last CTA of this KV head does the softmax of its rows
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(p.cnt + kvh, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int r = 0; r < M * G; ++r) {
        const int m = r / G, h = kvh * G + r % G;
        const int n = p.pos[m] + 1;
        const int nsp = (n + kChunk - 1) / kChunk;
        const float* pm = p.pmax + ((size_t)m * H + h) * p.nsplit;
        float mx = -INFINITY;
        for (int j = 0; j < nsp; ++j) mx = nanmax(mx, __ldcg(pm + j));
        const float* sr = p.sc + ((size_t)m * H + h) * T;
        int8_t* pr = p.pq + ((size_t)m * H + h) * T;
        auto e_of = [&](int t) { return sfu_exp(fsub(__ldcg(sr + t), mx)); };
        if (p.variant == 0) {                                  // NORM
            float* ebuf = reinterpret_cast<float*>(sm);        // [n] (the K chunk is no longer needed)
            __shared__ float rsum;
            for (int t = tid; t < n; t += kChunk) ebuf[t] = e_of(t);
            __syncthreads();
            if (warp == 0) {
                float ssum = red_sum16([&](int i) { return ebuf[i]; }, n, lane);
                if (lane == 0) rsum = sfu_recip(ssum);
            }
            __syncthreads();
            const float rc = rsum;
            for (int t = tid; t < n; t += kChunk) pr[t] = (int8_t)to_i8(fmul(fmul(ebuf[t], rc), 127.f));
            __syncthreads();
        } else {                                               // QSUM
            int part = 0;
            for (int t = tid; t < n; t += kChunk) {
                const int q = to_i8(fmul(e_of(t), 127.f));
                pr[t] = (int8_t)q;
                part += q;
            }
            part = block_sum_i(part, redi);
            if (tid == 0) p.rq[(size_t)m * H + h] = fmul(sfu_recip(i2f(part)), 127.f);
            __syncthreads();
        }
    }
    (void)red;
    if (tid == 0) p.cnt[kvh] = 0u;
}

// ---------------------------------------------------------------- 3. p.V
__global__ void __launch_bounds__(kMaxHd) attn_pv(AttnParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int hd = p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, M = p.rows, T = p.seq_len;
    const int kvh = blockIdx.x, split = blockIdx.y, t0 = split * kChunk, c = threadIdx.x;
    int8_t* vs = reinterpret_cast<int8_t*>(sm);                // [kChunk][hd]
    int8_t* ps = vs + kChunk * hd;                             // [M*G][kChunk]
    __shared__ int last;
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, p.pos[m]);
    const int nvalid = max(0, min(kChunk, maxpos + 1 - t0));
    if (nvalid > 0) {
        const int vpr = hd / 16;
        const int8_t* vbase = p.vc + ((size_t)kvh * T + t0) * hd;
        for (int i = c; i < nvalid * vpr; i += blockDim.x)
            reinterpret_cast<int4*>(vs)[i] = __ldg(reinterpret_cast<const int4*>(vbase) + i);
        for (int i = c; i < M * G * kChunk; i += blockDim.x) {
            const int r = i / kChunk, t = i % kChunk, m = r / G, h = kvh * G + r % G;
            const int tt = t0 + t;
            ps[i] = (tt <= p.pos[m]) ? p.pq[((size_t)m * H + h) * T + tt] : (int8_t)0;
        }
        __syncthreads();
        if (c < hd) {
            for (int r = 0; r < M * G; ++r) {
                const int m = r / G, h = kvh * G + r % G;
                const int lim = min(nvalid, p.pos[m] + 1 - t0);
                int acc = 0;
                for (int t = 0; t < lim; ++t) acc += (int)ps[r * kChunk + t] * (int)vs[t * hd + c];
                if (lim > 0) p.part[(((size_t)m * H + h) * p.nsplit + split) * hd + c] = acc;
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (c == 0) last = atomicAdd(p.cnt + Hk + kvh, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (c < hd) {
        for (int r = 0; r < M * G; ++r) {
            const int m = r / G, h = kvh * G + r % G;
            const int nsp = (p.pos[m] + kChunk) / kChunk;
            int acc = 0;
            for (int j = 0; j < nsp; ++j) acc += __ldcg(p.part + (((size_t)m * H + h) * p.nsplit + j) * hd + c);
            float o = i2f(acc);
            o = p.variant == 0 ? fmul(o, p.a_v) : fmul(fmul(o, __ldcg(p.rq + (size_t)m * H + h)), p.a_v);
            p.att[((size_t)m * H + h) * hd + c] = o;
        }
    }
    __syncthreads();
    if (c == 0) p.cnt[Hk + kvh] = 0u;
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t st) {
    const int slots = p.heads + 2 * p.kv_heads;
    const int pthreads = ((p.head_dim + 31) / 32) * 32;
    attn_prep<<<dim3(p.rows, slots), pthreads, 0, st>>>(p);
    const int G = p.heads / p.kv_heads;
    size_t smem_s = (size_t)kChunk * (p.head_dim + 16) + (size_t)p.rows * G * p.head_dim;
    if (smem_s < (size_t)p.seq_len * 4) smem_s = (size_t)p.seq_len * 4;   // the softmax's e row
    if (smem_s > 32 * 1024)
        cudaFuncSetAttribute(attn_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_s);
    attn_scores<<<dim3(p.kv_heads, p.nsplit), kChunk, smem_s, st>>>(p);
    const size_t smem_v = (size_t)kChunk * p.head_dim + (size_t)p.rows * G * kChunk;
    if (smem_v > 32 * 1024)
        cudaFuncSetAttribute(attn_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_v);
    attn_pv<<<dim3(p.kv_heads, p.nsplit), pthreads, smem_v, st>>>(p);
    return cudaGetLastError();
}

}  // namespace w8a8
