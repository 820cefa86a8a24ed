// Fused per-layer attention over the int8 KV cache, for one sequence's M rows
// (a decode step: M = 1; a prefill chunk: up to 16 rows, each computed exactly
// as a decode row, compiler/frontend/hf_generic.py:306-363; each head's cache
// chunk is read once per call for all rows, docs/fusion_design.md 6.7).
//
// Two launches per layer, grid (KV head, 128-position chunk), no spin waits:
//  1. attn_scores  q path of the G query heads of the KV head for every row:
//                  QK-norm (RMSNorm over head_dim, D = 16 ordered sum), RoPE
//                  (v*cos + swapneg(v)*sin), per-head quant_act -> int8 q.
//                  The CTA whose chunk holds a row's position also makes that
//                  row's K and V: QK-norm + RoPE + i8(k*inv_sk), i8(v*inv_sv),
//                  written to the cache (llm/ref_model.py:225-229,
//                  hf_generic.SaCache.update :190-226). Then the chunk of K,
//                  read once into shared memory, gives the scores
//                  (f32(qq.k)*s_q)*a_k of every row and head, and the chunk's
//                  maxima.
//  2. attn_pv      the row maximum over the chunk maxima (the global max comes
//                  before any int8 rounding: no online softmax), e = EXP(s - m);
//                  QSUM: eq = i8(127e) and the chunk's sum of eq; NORM: every CTA
//                  forms the whole row's e for the ordered sum, p = e*RECIP(sum),
//                  pq = i8(127p) (llm/ref_model.py:233-242; hf_generic.py:275-290);
//                  int32 pq.V partials of the chunk (exact in any order). The
//                  last CTA of the KV head (atomic ticket) adds the partials and
//                  dequantizes: NORM f32(acc)*a_v; QSUM (f32(acc)*(RECIP(sum)*127))*a_v.
// Cache layout: [kv_heads, seq_len, head_dim] int8 per layer.
#include "w8a8_internal.h"
#include "w8a8_math.cuh"
#include "pdl.cuh"

namespace w8a8 {

constexpr int kMaxG = 8;                                       // query heads per KV head
constexpr int kScoreThreads = kChunk;                          // one thread per position
constexpr int kScoreWarps = kScoreThreads / 32;
constexpr int kPvThreads = 128;

size_t attn_scratch_bytes(int rows, int heads, int kv_heads, int head_dim, int seq_len) {
    const size_t M = rows, H = heads, hd = head_dim, T = seq_len;
    const size_t ns = (T + kChunk - 1) / kChunk;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    return al(M * H * T * 4) + al(M * H * ns * 4) + al(M * H * ns * hd * 4) + al(M * H * ns * 4) +
           al((size_t)kv_heads * 4);
}

void attn_carve(AttnParams& p, void* scratch) {
    const size_t M = p.rows, H = p.heads, hd = p.head_dim, T = p.seq_len;
    const size_t ns = (T + kChunk - 1) / kChunk;
    p.nsplit = (int)ns;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    char* c = static_cast<char*>(scratch);
    p.sc = reinterpret_cast<float*>(c);
    c += al(M * H * T * 4);
    p.pmax = reinterpret_cast<float*>(c);
    c += al(M * H * ns * 4);
    p.part = reinterpret_cast<int32_t*>(c);
    c += al(M * H * ns * hd * 4);
    p.psum = reinterpret_cast<int32_t*>(c);
    c += al(M * H * ns * 4);
    p.cnt = reinterpret_cast<uint32_t*>(c);
}

__device__ __forceinline__ float warp_absmax(float v) {
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
        for (int c = lane; c < hd; c += 32) buf[c] = fmul(fmul(buf[c], r), __ldg(g + c));
        __syncwarp();
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        if (c < hd) {
            const float sw = (c & 1) ? buf[c - 1] : -buf[c + 1];
            o[i] = fadd(fmul(buf[c], __ldg(cosr + c)), fmul(sw, __ldg(sinr + c)));
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

// ---------------------------------------------------------------- 1. scores
__global__ void __launch_bounds__(kScoreThreads) attn_scores(AttnParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int hd = p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, M = p.rows, T = p.seq_len;
    const int kvh = blockIdx.x, split = blockIdx.y, t0 = split * kChunk, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int kstride = hd + 16;                               // padded rows: conflict-free 16-byte reads
    const int qkv_dim = (H + 2 * Hk) * hd, q_dim = H * hd, kv_dim = Hk * hd;
    int8_t* ks = reinterpret_cast<int8_t*>(sm);                // [kChunk][hd + 16]
    int8_t* qs = ks + kChunk * kstride;                        // [M*G][hd]
    float* fbuf = reinterpret_cast<float*>(qs + ((M * G * hd + 15) & ~15));   // [warps][hd]
    __shared__ float wmax[kScoreWarps][kMaxRows * kMaxG];
    __shared__ float sq[kMaxRows * kMaxG];
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, p.pos[m]);
    const int nvalid = min(kChunk, maxpos + 1 - t0);
    if (nvalid <= 0) {                                         // beyond every row: nothing to do
        pdl_wait();
        pdl_trigger();
        return;
    }
    // the chunk of K already in the cache
    const int vpr = hd / 16;
    const int8_t* kbase = p.kc + ((size_t)kvh * T + t0) * hd;
    for (int i = tid; i < nvalid * vpr; i += kScoreThreads) {
        const int t = i / vpr, c = i % vpr;
        *reinterpret_cast<int4*>(ks + t * kstride + c * 16) = __ldg(reinterpret_cast<const int4*>(kbase) + i);
    }
    // the rows above come from earlier steps (positions below this call's
    // rows, whose own K rows are made below): loaded before the wait
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    float* buf = fbuf + warp * hd;
    // q path of every row and query head of this KV head
    for (int r = warp; r < M * G; r += kScoreWarps) {
        const int m = r / G, h = kvh * G + r % G, pos = p.pos[m];
        const float* src = p.qkv + (size_t)m * qkv_dim + (size_t)h * hd;
        for (int c = lane; c < hd; c += 32) buf[c] = src[c];
        __syncwarp();
        warp_norm_rope(buf, hd, p.qk_norm ? p.q_norm : nullptr, p.eps, p.inv_hd, p.cos + (size_t)pos * hd,
                       p.sin + (size_t)pos * hd, lane);
        float a = 0.f;
        for (int c = lane; c < hd; c += 32) a = nanmax(a, fabsf(buf[c]));
        a = warp_absmax(a);
        const float s = fmul(a, W8A8_C127);
        const float inv = sfu_recip(s);
        for (int c = lane; c < hd; c += 32) qs[r * hd + c] = (int8_t)to_i8(fmul(buf[c], inv));
        if (lane == 0) sq[r] = s;
        __syncwarp();
    }
    // K and V rows of the positions in this chunk (into the cache; K also into the tile)
    for (int m = warp; m < M; m += kScoreWarps) {
        const int pos = p.pos[m];
        if (pos < t0 || pos >= t0 + kChunk) continue;
        const float* ksrc = p.qkv + (size_t)m * qkv_dim + q_dim + (size_t)kvh * hd;
        for (int c = lane; c < hd; c += 32) buf[c] = ksrc[c];
        __syncwarp();
        warp_norm_rope(buf, hd, p.qk_norm ? p.k_norm : nullptr, p.eps, p.inv_hd, p.cos + (size_t)pos * hd,
                       p.sin + (size_t)pos * hd, lane);
        int8_t* kdst = p.kc + ((size_t)kvh * T + pos) * hd;
        for (int c = lane; c < hd; c += 32) {
            const int8_t q = (int8_t)to_i8(fmul(buf[c], p.inv_sk));
            kdst[c] = q;
            ks[(pos - t0) * kstride + c] = q;
        }
        const float* vsrc = p.qkv + (size_t)m * qkv_dim + q_dim + kv_dim + (size_t)kvh * hd;
        int8_t* vdst = p.vc + ((size_t)kvh * T + pos) * hd;
        for (int c = lane; c < hd; c += 32) vdst[c] = (int8_t)to_i8(fmul(vsrc[c], p.inv_sv));
        __syncwarp();
    }
    __syncthreads();
    // scores of the chunk: thread t <-> position t0 + t
    const int t = t0 + tid;
    for (int r = 0; r < M * G; ++r) {
        const int m = r / G, h = kvh * G + r % G;
        float s = -INFINITY;
        if (tid < nvalid && t <= p.pos[m]) {
            int acc = 0;
            const int4* kr = reinterpret_cast<const int4*>(ks + tid * kstride);
            const int4* qr = reinterpret_cast<const int4*>(qs + r * hd);
            for (int c = 0; c < vpr; ++c) {
                const int4 a = kr[c], b = qr[c];
                acc = dp4a(a.x, b.x, acc);
                acc = dp4a(a.y, b.y, acc);
                acc = dp4a(a.z, b.z, acc);
                acc = dp4a(a.w, b.w, acc);
            }
            s = fmul(fmul(i2f(acc), sq[r]), p.a_k);
            p.sc[((size_t)m * H + h) * T + t] = s;
        }
        s = warp_absmax(s);
        if (lane == 0) wmax[warp][r] = s;
    }
    __syncthreads();
    if (tid < M * G) {
        float s = wmax[0][tid];
        for (int w = 1; w < kScoreWarps; ++w) s = nanmax(s, wmax[w][tid]);
        const int m = tid / G, h = kvh * G + tid % G;
        p.pmax[((size_t)m * H + h) * p.nsplit + split] = s;
    }
}

// ---------------------------------------------------------------- 2. p.V
__global__ void __launch_bounds__(kPvThreads) attn_pv(AttnParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int hd = p.head_dim, H = p.heads, Hk = p.kv_heads, G = H / Hk, M = p.rows, T = p.seq_len;
    const int kvh = blockIdx.x, split = blockIdx.y, t0 = split * kChunk, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    int8_t* vs = reinterpret_cast<int8_t*>(sm);                // [kChunk][hd]
    int8_t* ps = vs + kChunk * hd;                             // [M*G][kChunk]
    float* ebuf = reinterpret_cast<float*>(sm + (((size_t)kChunk * hd + (size_t)M * G * kChunk + 15) & ~size_t(15)));
    __shared__ int redi[32];
    __shared__ float rsum;
    __shared__ int last;
    pdl_wait();
    pdl_trigger();
    int maxpos = 0;
    for (int m = 0; m < M; ++m) maxpos = max(maxpos, p.pos[m]);
    const int nvalid = min(kChunk, maxpos + 1 - t0);
    if (nvalid > 0) {
        const int vpr = hd / 16;
        const int8_t* vbase = p.vc + ((size_t)kvh * T + t0) * hd;
        for (int i = tid; i < nvalid * vpr; i += kPvThreads)
            reinterpret_cast<int4*>(vs)[i] = __ldg(reinterpret_cast<const int4*>(vbase) + i);
        for (int r = 0; r < M * G; ++r) {
            const int m = r / G, h = kvh * G + r % G;
            const int n = p.pos[m] + 1;
            const int lim = min(nvalid, n - t0);                // positions of this chunk the row attends
            if (lim <= 0) {
                for (int t = tid; t < kChunk; t += kPvThreads) ps[r * kChunk + t] = 0;
                continue;
            }
            const int nsp = (n + kChunk - 1) / kChunk;
            const float* pm = p.pmax + ((size_t)m * H + h) * p.nsplit;
            float mx = -INFINITY;                              // chunk maxima read in parallel
            for (int j = lane; j < nsp; j += 32) mx = nanmax(mx, __ldcg(pm + j));
            mx = warp_absmax(mx);
            const float* sr = p.sc + ((size_t)m * H + h) * T;
            if (p.variant == 0) {                              // NORM: the whole row for the ordered sum
                for (int t = tid; t < n; t += kPvThreads) ebuf[t] = sfu_exp(fsub(__ldcg(sr + t), mx));
                __syncthreads();
                if (warp == 0) {
                    const float ssum = red_sum16([&](int i) { return ebuf[i]; }, n, lane);
                    if (lane == 0) rsum = sfu_recip(ssum);
                }
                __syncthreads();
                const float rc = rsum;
                for (int t = tid; t < kChunk; t += kPvThreads)
                    ps[r * kChunk + t] = t < lim ? (int8_t)to_i8(fmul(fmul(ebuf[t0 + t], rc), 127.f)) : (int8_t)0;
                __syncthreads();
            } else {                                           // QSUM: this chunk's e only
                int part = 0;
                for (int t = tid; t < kChunk; t += kPvThreads) {
                    int q = 0;
                    if (t < lim) q = to_i8(fmul(sfu_exp(fsub(__ldcg(sr + t0 + t), mx)), 127.f));
                    ps[r * kChunk + t] = (int8_t)q;
                    part += q;
                }
                part = block_sum_i(part, redi);
                if (tid == 0) p.psum[((size_t)m * H + h) * p.nsplit + split] = part;
            }
        }
        __syncthreads();
        for (int c = tid; c < hd; c += kPvThreads) {
            for (int r = 0; r < M * G; ++r) {
                const int m = r / G, h = kvh * G + r % G;
                const int lim = min(nvalid, p.pos[m] + 1 - t0);
                if (lim <= 0) continue;
                int acc = 0;
                for (int t = 0; t < lim; ++t) acc += (int)ps[r * kChunk + t] * (int)vs[t * hd + c];
                p.part[(((size_t)m * H + h) * p.nsplit + split) * hd + c] = acc;
            }
        }
    }
    // the last CTA of this KV head combines the chunks
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(p.cnt + kvh, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int r = 0; r < M * G; ++r) {
        const int m = r / G, h = kvh * G + r % G;
        const int nsp = (p.pos[m] + kChunk) / kChunk;
        float rq = 0.f;
        if (p.variant == 1) {
            int ssum = 0;
            for (int j = lane; j < nsp; j += 32) ssum += __ldcg(p.psum + ((size_t)m * H + h) * p.nsplit + j);
            ssum = warp_sum_i(ssum);
            rq = fmul(sfu_recip(i2f(ssum)), 127.f);            // sum <= 127 T: exact in fp32
        }
        for (int c = tid; c < hd; c += kPvThreads) {
            int acc = 0;
            const int32_t* pp = p.part + ((size_t)m * H + h) * p.nsplit * hd + c;
#pragma unroll 8
            for (int j = 0; j < nsp; ++j) acc += __ldcg(pp + (size_t)j * hd);
            const float o = i2f(acc);
            p.att[((size_t)m * H + h) * hd + c] = p.variant == 0 ? fmul(o, p.a_v) : fmul(fmul(o, rq), p.a_v);
        }
    }
    __syncthreads();
    if (tid == 0) p.cnt[kvh] = 0u;
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t st) {
    const int G = p.heads / p.kv_heads;
    const size_t qbytes = ((size_t)p.rows * G * p.head_dim + 15) & ~size_t(15);
    const size_t smem_s = (size_t)kChunk * (p.head_dim + 16) + qbytes + (size_t)kScoreWarps * p.head_dim * 4;
    if (smem_s > 32 * 1024) {
        cudaError_t e0 = cudaFuncSetAttribute(attn_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_s);
        if (e0 != cudaSuccess) return e0;
    }
    cudaError_t e = launch_k(attn_scores, dim3(p.kv_heads, p.nsplit), dim3(kScoreThreads), smem_s, st, p);
    if (e != cudaSuccess) return e;
    size_t smem_v = (size_t)kChunk * p.head_dim + (size_t)p.rows * G * kChunk;
    if (p.variant == 0) smem_v = ((smem_v + 15) & ~size_t(15)) + (size_t)p.seq_len * 4;
    if (smem_v > 32 * 1024) {
        e = cudaFuncSetAttribute(attn_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_v);
        if (e != cudaSuccess) return e;
    }
    return launch_k(attn_pv, dim3(p.kv_heads, p.nsplit), dim3(kPvThreads), smem_v, st, p);
}

}  // namespace w8a8
