// Device side of the tensor-parallel exchange (LL words over NVLink).
//
// A word is 8 bytes: the step epoch (high half) and a 32-bit value (low half),
// written with one 8-byte store into the receiving rank's region and read with
// relaxed system-scope loads until the high half equals this step's epoch. An
// aligned 8-byte access is single-copy atomic, so a reader never sees the
// value of one step with the epoch of another; it needs no fence and no flag.
//
// Block layouts (words), identical on every rank:
//   partials  [ranks][kTpRows][n]          value = the int32 accumulator
//   per-CTA   [ranks][1 + kTpCtas][kTpRows] entry (src, 0, 0) = the source's
//             CTA count, entry (src, 1 + c, m) = CTA c's value for row m
//   keys      the per-CTA layout with two words per entry (high, low half of
//             the 64-bit greedy key)
// A block is reused every step: the producer of step s + 1 on any rank first
// depends on a value its receiver sends only after consuming step s's words.
#pragma once
#include "w8a8_internal.h"

namespace w8a8 {

constexpr int kLlSpin = 1 << 12;            // polls before the waits back off
constexpr int kLlLimit = 1 << 21;           // polls before a wait gives up (~0.2 s)

template <typename T>
__device__ __forceinline__ T* tp_at(const TpCtx& t, T* local, int r) {
    const char* l = reinterpret_cast<const char*>(local);
    return reinterpret_cast<T*>(t.base[r] + (l - t.self));
}

// The step epoch: the first word of this rank's region (advanced by the
// tensor-parallel embedding at the start of every step).
__device__ __forceinline__ uint32_t tp_epoch(const TpCtx& t) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(t.self) : "memory");
    return v;
}

__device__ __forceinline__ void ll_store(uint64_t* a, uint32_t v, uint32_t ep) {
    const uint64_t w = ((uint64_t)ep << 32) | v;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ll_load(const uint64_t* a) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
    return w;
}

__device__ __forceinline__ void ll_load2(const uint64_t* a, uint64_t& w0, uint64_t& w1) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(a) : "memory");
}

// Bounded wait for the word of epoch ep; its value. After a wait of this
// thread gave up (ok false), later waits take one poll only.
__device__ __forceinline__ uint32_t ll_wait(const uint64_t* a, uint32_t ep, bool& ok) {
    for (int i = 0;; ++i) {
        const uint64_t w = ll_load(a);
        if ((uint32_t)(w >> 32) == ep) return (uint32_t)w;
        if (!ok || i >= kLlLimit) {
            ok = false;
            return 0u;
        }
        if (i >= kLlSpin) __nanosleep(128);
    }
}

// The sums over the ranks of the int32 partials j, j + 1 (j even) of row m of
// a partials block [ranks][kTpRows][k] (wrapping int32 adds, exact in any
// order). One 16-byte load per rank in flight; only ranks whose words are not
// yet of this epoch are polled again.
__device__ __forceinline__ void ll_sum_pair(const TpCtx& t, const uint64_t* blk, int m, int k, int j, uint32_t ep,
                                            bool& ok, int& s0, int& s1) {
    uint32_t pending = (1u << t.ranks) - 1u, a0 = 0u, a1 = 0u;
    for (int spins = 0; pending != 0u; ++spins) {
        uint64_t w0[kTpMaxRanks], w1[kTpMaxRanks];
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
            if (pending & (1u << q)) ll_load2(blk + ((size_t)q * kTpRows + m) * k + j, w0[q], w1[q]);
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q) {
            if ((pending & (1u << q)) && (uint32_t)(w0[q] >> 32) == ep && (uint32_t)(w1[q] >> 32) == ep) {
                a0 += (uint32_t)w0[q];
                a1 += (uint32_t)w1[q];
                pending &= ~(1u << q);
            }
        }
        if (pending == 0u) break;
        if (!ok || spins >= kLlLimit) {
            ok = false;
            break;
        }
        if (spins >= kLlSpin) __nanosleep(128);
    }
    s0 = (int)a0, s1 = (int)a1;
}

// Per-CTA blocks: word index of entry (src, c, m) (c = -1: the count entry).
__device__ __forceinline__ size_t ll_cta_idx(int src, int c, int m) {
    return ((size_t)src * (1 + kTpCtas) + 1 + c) * kTpRows + m;
}

// This CTA's value of row m into the per-CTA block of every rank (CTA 0's row
// 0 also posts the CTA count).
__device__ __forceinline__ void ll_post_cta(const TpCtx& t, uint64_t* blk, int cta, int ctas, int m, uint32_t val,
                                            uint32_t ep) {
#pragma unroll
    for (int q = 0; q < kTpMaxRanks; ++q) {
        if (q < t.ranks) {
            uint64_t* dst = tp_at(t, blk, q);
            ll_store(dst + ll_cta_idx(t.rank, cta, m), val, ep);
            if (cta == 0 && m == 0) ll_store(dst + ll_cta_idx(t.rank, -1, 0), (uint32_t)ctas, ep);
        }
    }
}

// The same for a 64-bit greedy key (two words per entry).
__device__ __forceinline__ void ll_post_key(const TpCtx& t, uint64_t* blk, int cta, int ctas, int m,
                                            unsigned long long key, uint32_t ep) {
#pragma unroll
    for (int q = 0; q < kTpMaxRanks; ++q) {
        if (q < t.ranks) {
            uint64_t* dst = tp_at(t, blk, q);
            ll_store(dst + 2 * ll_cta_idx(t.rank, cta, m), (uint32_t)(key >> 32), ep);
            ll_store(dst + 2 * ll_cta_idx(t.rank, cta, m) + 1, (uint32_t)key, ep);
            if (cta == 0 && m == 0) ll_store(dst + 2 * ll_cta_idx(t.rank, -1, 0), (uint32_t)ctas, ep);
        }
    }
}

// The maximum (as unsigned bits) over every rank's CTAs of row m of a per-CTA
// block, on every thread of the block. cnt: shared [kTpMaxRanks + 1]; red:
// shared [32]. Contains block barriers. Each thread keeps up to 8 entries'
// loads in flight and re-polls only the entries not yet of this epoch.
__device__ __forceinline__ uint32_t ll_block_max(const TpCtx& t, const uint64_t* blk, int m, uint32_t ep, bool& ok,
                                                 uint32_t* cnt, uint32_t* red) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    if (tid < t.ranks) {
        const uint32_t c = ll_wait(blk + ll_cta_idx(tid, -1, 0), ep, ok);
        cnt[tid] = c > (uint32_t)kTpCtas ? (uint32_t)kTpCtas : c;
    }
    __syncthreads();
    if (tid == 0) {                                            // prefix sums: entry e of rank q from cnt[q]
        uint32_t o = 0;
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q) {
            const uint32_t c = q < t.ranks ? cnt[q] : 0u;
            cnt[q] = o;
            o += c;
        }
        cnt[kTpMaxRanks] = o;
    }
    __syncthreads();
    const int E = (int)cnt[kTpMaxRanks];
    uint32_t mx = 0u;
    auto addr = [&](int e) {
        int q = 0;
#pragma unroll
        for (int r = 1; r < kTpMaxRanks; ++r) q += (r < t.ranks && e >= (int)cnt[r]) ? 1 : 0;
        return blk + ll_cta_idx(q, e - (int)cnt[q], m);
    };
    for (int e0 = tid; e0 < E; e0 += 8 * nt) {
        uint32_t pending = 0u;
#pragma unroll
        for (int u = 0; u < 8; ++u) pending |= (e0 + u * nt < E) ? (1u << u) : 0u;
        for (int spins = 0; pending != 0u; ++spins) {
            uint64_t w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (pending & (1u << u)) w[u] = ll_load(addr(e0 + u * nt));
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if ((pending & (1u << u)) && (uint32_t)(w[u] >> 32) == ep) {
                    mx = max(mx, (uint32_t)w[u]);
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
    mx = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (nt >> 5) ? red[lane] : 0u;
        v = __reduce_max_sync(0xffffffffu, v);
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    const uint32_t r = red[0];
    __syncthreads();
    return r;
}

}  // namespace w8a8
