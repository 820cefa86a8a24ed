// Fused per-layer attention over the int8 KV cache, one launch per layer, for
// one sequence's M rows (a decode step: M = 1; a prefill chunk: up to 16 rows,
// each computed exactly as a decode row, compiler/frontend/hf_generic.py:306-363;
// each head's cache is read once per call for all rows, docs/fusion_design.md 6.7).
//
// Grid (KV head, 128-position chunk); the chunks of one KV head meet twice at a
// bounded barrier over global memory (all CTAs of the grid are resident at
// once: the host checks the occupancy before launching):
//  1. q path of the G query heads of the KV head, every row: QK-norm (RMSNorm
//     over head_dim, D = 16 ordered sum), RoPE (v*cos + swapneg(v)*sin),
//     per-head quant_act -> int8 q. The CTA whose chunk holds a row's position
//     makes that row's K and V: QK-norm + RoPE + i8(k*inv_sk), i8(v*inv_sv),
//     into the cache (llm/ref_model.py:225-229, hf_generic.SaCache.update
//     :190-226) and into its tiles. Scores (f32(qq.k)*s_q)*a_k stay in shared
//     memory; the chunk maxima go to a global atomic max per row and head.
//     -- barrier A: the row maxima are final (the global max comes before any
//     int8 rounding: no online softmax) --
//  2. e = EXP(s - m); QSUM: eq = i8(127e), sum eq; NORM: the whole row's e (from
//     the scores in global memory) for the ordered sum, pq = i8(127 e RECIP(sum))
//     (llm/ref_model.py:233-242; hf_generic.py:275-290); int32 pq.V of the chunk,
//     added into global int32 sums with atomics (exact in any order).
//     -- barrier B --
//  3. the chunk-0 CTA dequantizes: NORM f32(acc)*a_v; QSUM
//     (f32(acc)*(RECIP(sum)*127))*a_v, and clears the sums and maxima.
// Cache layout: [kv_heads, seq_len, head_dim] int8 per layer.
#include "pdl.cuh"
#include "w8a8_internal.h"
#include "w8a8_math.cuh"

namespace w8a8 {

__device__ unsigned int g_attn_errors;                         // bit 2: a chunk barrier gave up

constexpr int kMaxG = 8;                                       // query heads per KV head
constexpr int kAttnThreads = kChunk;                           // one thread per position
constexpr int kAttnWarps = kAttnThreads / 32;

static size_t al256(size_t b) { return (b + 255) & ~size_t(255); }

size_t attn_scratch_bytes(int rows, int heads, int kv_heads, int head_dim, int seq_len) {
    const size_t M = rows, H = heads, hd = head_dim, T = seq_len;
    return al256(M * H * T * 4) + al256(M * H * 4) + al256(M * H * 4) + al256(M * H * hd * 4) +
           al256((size_t)kv_heads * 128);
}

void attn_carve(AttnParams& p, void* scratch) {
    const size_t M = p.rows, H = p.heads, hd = p.head_dim, T = p.seq_len;
    p.nsplit = (int)((T + kChunk - 1) / kChunk);
    char* c = static_cast<char*>(scratch);
    p.sc = reinterpret_cast<float*>(c);
    c += al256(M * H * T * 4);
    p.gmax = reinterpret_cast<uint32_t*>(c);
    c += al256(M * H * 4);
    p.psum = reinterpret_cast<int32_t*>(c);
    c += al256(M * H * 4);
    p.acc = reinterpret_cast<int32_t*>(c);
    c += al256(M * H * hd * 4);
    p.sync = reinterpret_cast<uint32_t*>(c);
}

// order-preserving uint encoding of a float for atomicMax (NaN above all, as
// np.max propagates it; 0 is below every encoded value)
__device__ __forceinline__ uint32_t ord_enc(float v) {
    if (v != v) return 0xFFFFFFFFu;
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_dec(uint32_t e) {
    if (e == 0xFFFFFFFFu) return __uint_as_float(kQNaN);
    return __uint_as_float((e & 0x80000000u) ? (e & 0x7FFFFFFFu) : ~e);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nanmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One head vector in shared memory (buf[hd], loaded by the warp): optional
// RMSNorm with gain g, then RoPE with the position's table rows; in place.
__device__ __forceinline__ void warp_norm_rope(float* buf, int hd, const float* g, float eps, float inv_hd,
                                               const float* cosr, const float* sinr, int lane) {
    if (g != nullptr) {
        const float ss = red_sum16([&](int i) { return fmul(buf[i], buf[i]); }, hd, lane);
        const float r = sfu_rsqrt(fadd(fmul(ss, inv_hd), eps));
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

struct AttnSmem {                                              // offsets into the dynamic shared memory
    size_t ks, vs, qs, fbuf, scs, ps, tab, gain, ebuf, total;
};

__host__ __device__ inline AttnSmem attn_smem(int M, int G, int hd, int T, int variant) {
    auto a16 = [](size_t b) { return (b + 15) & ~size_t(15); };
    AttnSmem s{};
    size_t o = 0;
    s.ks = o;   o += a16((size_t)kChunk * (hd + 16));         // K tile, padded rows
    s.vs = o;   o += a16((size_t)kChunk * hd);                // V tile
    s.qs = o;   o += a16((size_t)M * G * hd);                 // int8 q rows
    s.fbuf = o; o += a16((size_t)kAttnWarps * hd * 4);        // per-warp fp32 head vector
    s.scs = o;  o += a16((size_t)M * G * kChunk * 4);         // scores of the chunk
    s.ps = o;   o += a16((size_t)M * G * kChunk);             // int8 probabilities of the chunk
    s.tab = o;  o += a16((size_t)M * 2 * hd * 4);             // cos | sin rows of each row's position
    s.gain = o; o += a16((size_t)2 * hd * 4);                 // q_norm | k_norm gains
    s.ebuf = o; o += variant == 0 ? a16((size_t)T * 4) : 0;   // NORM: the whole row's e
    s.total = o;
    return s;
}

__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int hd = p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, M = p.rows, T = p.seq_len;
    const int kvh = blockIdx.x, split = blockIdx.y, t0 = split * kChunk, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int kstride = hd + 16, vpr = hd / 16;
    const int qkv_dim = (H + 2 * Hk) * hd, q_dim = H * hd, kv_dim = Hk * hd;
    const AttnSmem L = attn_smem(M, G, hd, T, p.variant);
    int8_t* ks = reinterpret_cast<int8_t*>(sm + L.ks);
    int8_t* vs = reinterpret_cast<int8_t*>(sm + L.vs);
    int8_t* qs = reinterpret_cast<int8_t*>(sm + L.qs);
    float* fbuf = reinterpret_cast<float*>(sm + L.fbuf);
    float* scs = reinterpret_cast<float*>(sm + L.scs);
    int8_t* ps = reinterpret_cast<int8_t*>(sm + L.ps);
    float* tabs = reinterpret_cast<float*>(sm + L.tab);         // row m: cos at [2m hd], sin at [(2m+1) hd]
    float* gains = reinterpret_cast<float*>(sm + L.gain);       // q_norm | k_norm
    float* ebuf = reinterpret_cast<float*>(sm + L.ebuf);
    __shared__ float sq[kMaxRows * kMaxG];
    __shared__ float wmax[kAttnWarps][kMaxRows * kMaxG];
    __shared__ int redi[32];
    __shared__ float rsum;
    __shared__ int lim_s[kMaxRows];
    unsigned int* bar_count = p.sync + kvh * 32;
    volatile unsigned int* bar_gen = p.sync + kvh * 32 + 1;

    // ---- before the wait: positions, cache tiles of earlier positions, tables
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, p.pos[m]);
    const int nvalid = min(kChunk, maxpos + 1 - t0);
    if (tid < M) lim_s[tid] = min(nvalid, p.pos[tid] + 1 - t0);   // positions of the chunk row m attends
    if (nvalid > 0) {
        const int8_t* kbase = p.kc + ((size_t)kvh * T + t0) * hd;
        const int8_t* vbase = p.vc + ((size_t)kvh * T + t0) * hd;
        for (int i = tid; i < nvalid * vpr; i += kAttnThreads) {
            const int t = i / vpr, c = i % vpr;
            *reinterpret_cast<int4*>(ks + t * kstride + c * 16) = __ldg(reinterpret_cast<const int4*>(kbase) + i);
            reinterpret_cast<int4*>(vs)[i] = __ldg(reinterpret_cast<const int4*>(vbase) + i);
        }
        for (int i = tid; i < M * hd; i += kAttnThreads) {
            const int m = i / hd, c = i % hd, pos = p.pos[m];
            tabs[2 * m * hd + c] = __ldg(p.cos + (size_t)pos * hd + c);
            tabs[(2 * m + 1) * hd + c] = __ldg(p.sin + (size_t)pos * hd + c);
        }
        if (p.qk_norm)
            for (int c = tid; c < hd; c += kAttnThreads) {
                gains[c] = __ldg(p.q_norm + c);
                gains[hd + c] = __ldg(p.k_norm + c);
            }
    }
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    bool ok = true;
    if (nvalid > 0) {
        float* buf = fbuf + warp * hd;
        // q path of every row and query head of this KV head
        for (int r = warp; r < M * G; r += kAttnWarps) {
            const int m = r / G, h = kvh * G + r % G;
            const float* src = p.qkv + (size_t)m * qkv_dim + (size_t)h * hd;
            for (int c = lane; c < hd; c += 32) buf[c] = src[c];
            __syncwarp();
            warp_norm_rope(buf, hd, p.qk_norm ? gains : nullptr, p.eps, p.inv_hd, tabs + 2 * m * hd,
                           tabs + (2 * m + 1) * hd, lane);
            float a = 0.f;
            for (int c = lane; c < hd; c += 32) a = nanmax(a, fabsf(buf[c]));
            a = warp_max(a);
            const float s = fmul(a, W8A8_C127);
            const float inv = sfu_recip(s);
            for (int c = lane; c < hd; c += 32) qs[r * hd + c] = (int8_t)to_i8(fmul(buf[c], inv));
            if (lane == 0) sq[r] = s;
            __syncwarp();
        }
        // K and V rows of the positions in this chunk: into the cache and the tiles
        for (int m = warp; m < M; m += kAttnWarps) {
            const int pos = p.pos[m];
            if (pos < t0 || pos >= t0 + kChunk) continue;
            const float* ksrc = p.qkv + (size_t)m * qkv_dim + q_dim + (size_t)kvh * hd;
            for (int c = lane; c < hd; c += 32) buf[c] = ksrc[c];
            __syncwarp();
            warp_norm_rope(buf, hd, p.qk_norm ? gains + hd : nullptr, p.eps, p.inv_hd, tabs + 2 * m * hd,
                           tabs + (2 * m + 1) * hd, lane);
            int8_t* kdst = p.kc + ((size_t)kvh * T + pos) * hd;
            int8_t* vdst = p.vc + ((size_t)kvh * T + pos) * hd;
            const float* vsrc = p.qkv + (size_t)m * qkv_dim + q_dim + kv_dim + (size_t)kvh * hd;
            for (int c = lane; c < hd; c += 32) {
                const int8_t kq = (int8_t)to_i8(fmul(buf[c], p.inv_sk));
                const int8_t vq = (int8_t)to_i8(fmul(vsrc[c], p.inv_sv));
                kdst[c] = kq;
                vdst[c] = vq;
                ks[(pos - t0) * kstride + c] = kq;
                vs[(pos - t0) * hd + c] = vq;
            }
            __syncwarp();
        }
        __syncthreads();
        // scores of the chunk: thread t <-> position t0 + t
        for (int r = 0; r < M * G; ++r) {
            const int m = r / G, h = kvh * G + r % G;
            float s = -INFINITY;
            if (tid < lim_s[m]) {
                int a = 0;
                const int4* kr = reinterpret_cast<const int4*>(ks + tid * kstride);
                const int4* qr = reinterpret_cast<const int4*>(qs + r * hd);
                for (int c = 0; c < vpr; ++c) {
                    const int4 x = kr[c], y = qr[c];
                    a = dp4a(x.x, y.x, a);
                    a = dp4a(x.y, y.y, a);
                    a = dp4a(x.z, y.z, a);
                    a = dp4a(x.w, y.w, a);
                }
                s = fmul(fmul(i2f(a), sq[r]), p.a_k);
                scs[r * kChunk + tid] = s;
                if (p.variant == 0) p.sc[((size_t)m * H + h) * T + t0 + tid] = s;
            }
            s = warp_max(s);
            if (lane == 0) wmax[warp][r] = s;
        }
        __syncthreads();
        if (tid < M * G && lim_s[tid / G] > 0) {
            float s = wmax[0][tid];
            for (int w = 1; w < kAttnWarps; ++w) s = nanmax(s, wmax[w][tid]);
            atomicMax(p.gmax + (size_t)(tid / G) * H + kvh * G + tid % G, ord_enc(s));
        }
    }
    ok = cta_barrier(bar_count, bar_gen, gridDim.y) && ok;     // A: the row maxima are final
    if (nvalid > 0) {
        for (int r = 0; r < M * G; ++r) {
            const int m = r / G, h = kvh * G + r % G;
            const int lim = lim_s[m];
            if (lim <= 0) {
                for (int t = tid; t < kChunk; t += kAttnThreads) ps[r * kChunk + t] = 0;
                continue;
            }
            const float mx = ord_dec(__ldcg(p.gmax + (size_t)m * H + h));
            if (p.variant == 0) {                              // NORM: the whole row for the ordered sum
                const int n = p.pos[m] + 1;
                const float* sr = p.sc + ((size_t)m * H + h) * T;
                for (int t = tid; t < n; t += kAttnThreads) ebuf[t] = sfu_exp(fsub(__ldcg(sr + t), mx));
                __syncthreads();
                if (warp == 0) {
                    const float ssum = red_sum16([&](int i) { return ebuf[i]; }, n, lane);
                    if (lane == 0) rsum = sfu_recip(ssum);
                }
                __syncthreads();
                const float rc = rsum;
                ps[r * kChunk + tid] = tid < lim ? (int8_t)to_i8(fmul(fmul(ebuf[t0 + tid], rc), 127.f)) : (int8_t)0;
                __syncthreads();
            } else {                                           // QSUM: this chunk's e only
                int q = 0;
                if (tid < lim) q = to_i8(fmul(sfu_exp(fsub(scs[r * kChunk + tid], mx)), 127.f));
                ps[r * kChunk + tid] = (int8_t)q;
                q = block_sum_i(q, redi);
                if (tid == 0) atomicAdd(p.psum + (size_t)m * H + h, q);
            }
        }
        __syncthreads();
        for (int c = tid; c < hd; c += kAttnThreads) {
            for (int r = 0; r < M * G; ++r) {
                const int m = r / G, h = kvh * G + r % G;
                const int lim = lim_s[m];
                if (lim <= 0) continue;
                int a = 0;
#pragma unroll 8
                for (int t = 0; t < lim; ++t) a += (int)ps[r * kChunk + t] * (int)vs[t * hd + c];
                atomicAdd(p.acc + ((size_t)m * H + h) * hd + c, a);
            }
        }
    }
    ok = cta_barrier(bar_count, bar_gen, gridDim.y) && ok;     // B: the sums are final
    if (!ok && tid == 0) atomicOr(&g_attn_errors, 4u);
    if (split != 0) return;
    for (int r = 0; r < M * G; ++r) {
        const int m = r / G, h = kvh * G + r % G;
        const size_t mh = (size_t)m * H + h;
        float rq = 0.f;
        if (p.variant == 1) rq = fmul(sfu_recip(i2f(__ldcg(p.psum + mh))), 127.f);   // sum <= 127 T: exact
        for (int c = tid; c < hd; c += kAttnThreads) {
            const float o = i2f(__ldcg(p.acc + mh * hd + c));
            p.att[mh * hd + c] = p.variant == 0 ? fmul(o, p.a_v) : fmul(fmul(o, rq), p.a_v);
            p.acc[mh * hd + c] = 0;
        }
        if (tid == 0) {
            p.psum[mh] = 0;
            p.gmax[mh] = 0u;
        }
    }
}

static int attn_occupancy(size_t smem) {
    int per_sm = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_kernel, kAttnThreads, smem);
    return per_sm * sms;
}

int attn_max_ctas(int rows, int heads, int kv_heads, int head_dim, int seq_len, int variant) {
    const AttnSmem L = attn_smem(rows, heads / kv_heads, head_dim, seq_len, variant);
    if (L.total > 200 * 1024) return 0;
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    return attn_occupancy(L.total);
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t st) {
    const int G = p.heads / p.kv_heads;
    const AttnSmem L = attn_smem(p.rows, G, p.head_dim, p.seq_len, p.variant);
    cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    return launch_k(attn_kernel, dim3(p.kv_heads, p.nsplit), dim3(kAttnThreads), L.total, st, p);
}

unsigned int attn_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_attn_errors, sizeof(v));
    cudaMemcpyToSymbol(g_attn_errors, &zero, sizeof(zero));
    return v;
}

}  // namespace w8a8
