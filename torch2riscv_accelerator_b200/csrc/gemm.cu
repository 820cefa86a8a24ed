// W8A8 GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) for many
// rows at once (prefill chunks, batched decode):
//   acc[m][n] = sum_k xq[m][k] * W[n][k]   (int32, exact)
//   y[m][n]   = (f32(acc) * s_w[n]) * s_x[m]  [+ resid[m][n]]
// or, with a second weight matrix (the SwiGLU gate / up pair),
//   h[m][n]   = (g * RECIP(1 + EXP(-g))) * u
// (llm/ref_model.py:198-202, :246-250; hf_generic._qlinear :583-593). The int8
// activations come quantized per row (w8a8_quant_rows); the arithmetic after
// the exact int32 sum is the GEMV's, so the results equal it bit for bit.
//
// One CTA per 128 x BN output tile (BN = 128 or 256 columns), K in 128-byte
// steps through a ring of shared-memory stages:
//   warp 0, one thread: TMA 2-D tile loads of xq and W (128-byte swizzle), one
//     mbarrier per stage counting the bytes;
//   warp 1: allocates the TMEM accumulator (BN int32 columns x 128 lanes, twice
//     for the gate / up pair); one thread issues tcgen05.mma (M = 128, N = BN,
//     K = 32 bytes each, A and B K-major from shared memory) and commits each
//     stage back to the producer, then the finished accumulator to the epilogue;
//   warps 2-9: tcgen05.ld of their 32 lanes (rows), half the columns each,
//     dequant and 16-byte stores.
// Every wait is bounded (the producer and MMA threads spin on their stage
// barriers: a suspended wait wakes microseconds late, once per stage): on a
// timeout the kernel sets an error bit, still waits (bounded) for its MMAs,
// frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "pdl.cuh"
#include "tc.cuh"
#include "w8a8_internal.h"
#include "w8a8_math.cuh"

namespace w8a8 {

__device__ unsigned int g_gemm_errors;                        // bit 4: a GEMM pipeline wait gave up

constexpr int kGemmThreads = 320;                              // 10 warps: TMA, MMA, 8 epilogue
constexpr int kBM = 128;                                       // rows per tile (TMEM lanes)
constexpr int kBK = 128;                                       // K bytes per stage (one 128-byte swizzle row)
constexpr int kStages = 4;

struct GemmMaps {
    CUtensorMap a, b, b2;                                      // xq [M][K]; W [N][K]; W2 (SwiGLU up) or unused
};

template <int BN, bool TWO, bool GRP = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ GemmMaps maps, GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned stages: A [128][128] then B [BN][128] (then B2)
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int kA = kBM * kBK, kB = BN * kBK;
    constexpr int kStage = kA + kB * (TWO ? 2 : 1);
    __shared__ __align__(8) uint64_t full[kStages], empty[kStages], acc_full;
    __shared__ uint32_t tmem_base;
    __shared__ int failed;
    __shared__ __align__(16) uint32_t silu_tab[256];           // EXP / RECIP tables (SwiGLU epilogue)
    if (TWO) stage_silu_tables(silu_tab);
    const GateAct act{p.act, p.act_a, p.act_b};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // grouped: expert ge, tile gt of its slab; A and B rows offset to them
    const int ge = GRP ? (int)blockIdx.y / p.g_mtiles : 0, gt = GRP ? (int)blockIdx.y % p.g_mtiles : 0;
    const int n0 = blockIdx.x * BN, m0 = GRP ? ge * p.g_mcap + gt * kBM : blockIdx.y * kBM;
    const int nb0 = GRP ? ge * p.n + n0 : n0;                 // B row of column n0
    const int kt_n = (p.k + kBK - 1) / kBK;
    constexpr uint32_t kCols = TWO ? 2 * BN : BN;              // TMEM columns (a power of two >= 32)
    if (tid == 0) {
        failed = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) {                                           // TMEM accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    pdl_wait();                                                // xq comes from the previous kernel
    pdl_trigger();
    // grouped: a slab tile beyond the expert's row count has no valid row; its
    // CTA loads nothing and issues no MMA (most tiles of a long prefill chunk,
    // where each expert's slab is sized for every row)
    const bool idle = GRP && gt * kBM >= __ldcg(p.g_cnt + ge);

    if (idle) {
    } else if (warp == 0 && lane == 0) {
        // producer: stage s of step kt holds xq[m0.., kt*128..] and W[n0.., kt*128..]
        for (int kt = 0; kt < kt_n; ++kt) {
            const int s = kt % kStages;
            if (kt >= kStages && !mbar_wait_spin(&empty[s], (uint32_t)(((kt / kStages) - 1) & 1))) {
                atomicOr(&g_gemm_errors, 16u);
                failed = 1;
                break;
            }
            unsigned char* st = smem + (size_t)s * kStage;
            mbar_expect_tx(&full[s], (uint32_t)kStage);
            tma_load_2d(st, &maps.a, kt * kBK, m0, &full[s]);
            tma_load_2d(st + kA, &maps.b, kt * kBK, nb0, &full[s]);
            if (TWO) tma_load_2d(st + kA + kB, &maps.b2, kt * kBK, nb0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: 4 MMAs of K = 32 bytes per stage; the descriptor start
        // address advances 32 bytes (2 in 16-byte units) inside the swizzle row
        const uint32_t id = idesc_i8(kBM, BN);
        bool ok = true;
        for (int kt = 0; kt < kt_n; ++kt) {
            const int s = kt % kStages;
            if (!mbar_wait_spin(&full[s], (uint32_t)((kt / kStages) & 1))) {
                atomicOr(&g_gemm_errors, 16u);
                failed = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const unsigned char* st = smem + (size_t)s * kStage;
            const uint64_t da = smem_desc(st), db = smem_desc(st + kA);
            const uint64_t db2 = TWO ? smem_desc(st + kA + kB) : 0ull;
#pragma unroll
            for (int kk = 0; kk < kBK / 32; ++kk) {
                const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
                mma_i8(tmem, da + 2 * kk, db + 2 * kk, id, acc);
                if (TWO) mma_i8(tmem + BN, da + 2 * kk, db2 + 2 * kk, id, acc);
            }
            mma_commit(&empty[s]);                             // the stage is free once these MMAs read it
        }
        mma_commit(&acc_full);                                 // every MMA issued so far has completed
        (void)ok;
    } else if (warp >= 2) {
        // epilogue: warps 2-9, two per TMEM lane quarter: warp w reads lanes
        // 32*(w % 4) .. +31 (rows) and half of the columns, 16 at a time
        const bool ok = mbar_wait(&acc_full, 0u);
        tc_fence_after();
        if (!ok) {
            if (lane == 0) atomicOr(&g_gemm_errors, 16u);
        } else if (!failed) {
            const int q = warp & 3, half = (warp - 2) >> 2;
            const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
            // this thread's row: valid, its output row, s_x (grouped: the pair)
            int m = m0 + q * 32 + lane;
            bool valid = m < p.m;
            float sx = 0.f, wj = 0.f;
            if (GRP) {
                const int local = gt * kBM + q * 32 + lane;
                valid = local < __ldcg(p.g_cnt + ge);
                m = valid ? __ldcg(p.g_pair + (size_t)ge * p.g_mcap + local) : 0;
                if (valid) {
                    sx = __ldcg(p.s_x + (TWO ? m / p.g_top_k : m));
                    if (!TWO) wj = __ldcg(p.g_w + m);
                }
            } else if (valid) {
                sx = __ldg(p.s_x + m);
            }
            const float* s_w = p.s_w + (GRP ? (size_t)ge * p.n : 0);
            const float* s_w2 = TWO ? p.s_w2 + (GRP ? (size_t)ge * p.n : 0) : nullptr;
            uint32_t am = 0u;                                  // grouped, with w2: max|h| of the row
            const bool vec = (p.n & 3) == 0;                 // 16-byte rows: vector loads and stores
            for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
                int v[16], u[16];
                tmem_ld16(tmem + lane_addr + (uint32_t)c0, v);
                if (TWO) tmem_ld16(tmem + lane_addr + (uint32_t)(BN + c0), u);
                const int nb = n0 + c0;
                if (!valid || nb >= p.n) continue;                   // (after the warp-wide TMEM loads)
                float o[16];
                if (vec && nb + 16 <= p.n) {
                    float sw[16], sw2[16], rs[16];
                    const float4* s4 = reinterpret_cast<const float4*>(s_w + nb);
#pragma unroll
                    for (int j = 0; j < 4; ++j) reinterpret_cast<float4*>(sw)[j] = __ldg(s4 + j);
                    if (TWO) {
                        const float4* t4 = reinterpret_cast<const float4*>(s_w2 + nb);
#pragma unroll
                        for (int j = 0; j < 4; ++j) reinterpret_cast<float4*>(sw2)[j] = __ldg(t4 + j);
                    }
                    float4* y4 = reinterpret_cast<float4*>(p.y + (size_t)m * p.n + nb);
                    if (!GRP && !TWO && p.resid != nullptr) {
                        const float4* r4 = reinterpret_cast<const float4*>(p.resid + (size_t)m * p.n + nb);
#pragma unroll
                        for (int j = 0; j < 4; ++j) reinterpret_cast<float4*>(rs)[j] = r4[j];
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float g = fmul(fmul(i2f(v[j]), sw[j]), sx);
                        if (TWO) o[j] = gate_tab(g, fmul(fmul(i2f(u[j]), sw2[j]), sx), silu_tab, act);
                        else if (GRP) o[j] = fmul(wj, g);
                        else o[j] = p.resid != nullptr ? fadd(rs[j], g) : g;
                        if (GRP && TWO) am = max(am, __float_as_uint(fabsf(o[j])));   // NaN above numbers
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) y4[j] = reinterpret_cast<const float4*>(o)[j];
                    if (!GRP && !TWO && p.resid == nullptr && p.acc != nullptr) {
                        int4* a4 = reinterpret_cast<int4*>(p.acc + (size_t)m * p.n + nb);
#pragma unroll
                        for (int j = 0; j < 4; ++j) a4[j] = reinterpret_cast<const int4*>(v)[j];
                    }
                    continue;
                }
                if constexpr (!GRP) {                                // (grouped: n % 16 == 0, never ragged)
#pragma unroll
                for (int j = 0; j < 16; ++j) {                       // a ragged or unaligned edge
                    const int n = nb + j;
                    if (n >= p.n) continue;
                    const size_t off = (size_t)m * p.n + n;
                    const float g = fmul(fmul(i2f(v[j]), __ldg(s_w + n)), sx);
                    if (TWO) {
                        p.y[off] = gate_tab(g, fmul(fmul(i2f(u[j]), __ldg(s_w2 + n)), sx), silu_tab, act);
                    } else if (p.resid != nullptr) {
                        p.y[off] = fadd(p.resid[off], g);
                    } else {
                        p.y[off] = g;
                        if (p.acc != nullptr) p.acc[off] = v[j];
                    }
                }
                }
            }
            if (GRP && TWO && valid && am != 0u) atomicMax(p.g_amax + m, am);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        // the accumulator's last commit has arrived (or, after a failure, wait
        // for the MMAs issued so far before the memory goes back)
        if (failed) mbar_wait(&acc_full, 0u);
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride,
                 uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D int8 map of a row-major [rows][k] matrix, box 128 bytes x box_rows,
// 128-byte swizzle; rows or k beyond the matrix read as zero
static bool make_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows) {
    return make_map_u8(map, base, (uint64_t)k, (uint64_t)rows, (uint64_t)k, kBK, (uint32_t)box_rows, true);
}

size_t gemm_smem(int bn, bool two) { return (size_t)kStages * (kBM * kBK + (size_t)bn * kBK * (two ? 2 : 1)) + 1024; }

template <int BN, bool TWO, bool GRP = false>
static cudaError_t launch_gemm_t(const GemmOperands& a, const GemmParams& p, cudaStream_t st, int experts = 1) {
    GemmMaps maps{};
    // grouped: A = every expert's slab, B = every expert's n rows
    const int a_rows = GRP ? experts * p.g_mcap : p.m, b_rows = GRP ? experts * p.n : p.n;
    if (!make_map(&maps.a, a.xq, a_rows, p.k, kBM) || !make_map(&maps.b, a.w, b_rows, p.k, BN) ||
        (TWO && !make_map(&maps.b2, a.w2, b_rows, p.k, BN)))
        return cudaErrorInvalidValue;
    auto kern = gemm_kernel<BN, TWO, GRP>;
    const size_t sm = gemm_smem(BN, TWO);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    const dim3 grid((p.n + BN - 1) / BN, GRP ? experts * p.g_mtiles : (p.m + kBM - 1) / kBM);
    return launch_k(kern, grid, dim3(kGemmThreads), sm, st, maps, p);
}

// Tile width by an estimate of the GEMM's time: waves of CTAs (one per SM) x
// (a fixed cost per CTA + the bytes it streams, its 128-row A slab and its
// BN-row weight slab(s), at a per-CTA rate), with the constants fitted to
// B200 timings (2 us, 40 GB/s). A GEMM of few rows (batched decode: one
// 128-row tile) gets narrow tiles that spread the weight stream over the SMs;
// long prefill chunks and the classifier keep 256-column tiles.
static double gemm_cost(long tiles, int bn, int k, bool two, int sms) {
    const long waves = (tiles + sms - 1) / sms;
    return (double)waves * (2.0 + (double)(kBM + (two ? 2 : 1) * bn) * k / 40e3);
}

cudaError_t launch_gemm(const GemmOperands& a, const GemmParams& p, cudaStream_t st) {
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    const bool two = a.w2 != nullptr;
    const long mt = (p.m + kBM - 1) / kBM;
    int best = 32;
    double cbest = 1e300;
    for (int bn : {32, 64, 128, 256}) {
        if (two && bn > 128) continue;                         // 2 x BN TMEM columns
        const double c = gemm_cost((long)((p.n + bn - 1) / bn) * mt, bn, p.k, two, sms);
        if (c < cbest * (1.0 - 1e-9)) best = bn, cbest = c;   // ties: the narrower
    }
    if (two) {
        if (best == 128) return launch_gemm_t<128, true>(a, p, st);
        if (best == 64) return launch_gemm_t<64, true>(a, p, st);
        return launch_gemm_t<32, true>(a, p, st);
    }
    if (best == 256) return launch_gemm_t<256, false>(a, p, st);
    if (best == 128) return launch_gemm_t<128, false>(a, p, st);
    if (best == 64) return launch_gemm_t<64, false>(a, p, st);
    return launch_gemm_t<32, false>(a, p, st);
}

// Grouped (MoE experts): every expert's slab of g_mcap rows against its own
// weights; tile width by the same estimate over experts x slab tiles x column
// tiles. n a multiple of 16 (whole 16-column epilogue groups).
cudaError_t launch_gemm_grouped(const GemmOperands& a, const GemmParams& p, int experts, cudaStream_t st) {
    if (experts <= 0 || p.n % 16 != 0 || p.g_mcap % kBM != 0 || p.g_mtiles * kBM != p.g_mcap)
        return cudaErrorInvalidValue;
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    const bool two = a.w2 != nullptr;
    const long mt = (long)experts * p.g_mtiles;
    int best = 32;
    double cbest = 1e300;
    for (int bn : {32, 64, 128}) {
        const double c = gemm_cost((long)((p.n + bn - 1) / bn) * mt, bn, p.k, two, sms);
        if (c < cbest * (1.0 - 1e-9)) best = bn, cbest = c;
    }
    if (two) {
        if (best == 128) return launch_gemm_t<128, true, true>(a, p, st, experts);
        if (best == 64) return launch_gemm_t<64, true, true>(a, p, st, experts);
        return launch_gemm_t<32, true, true>(a, p, st, experts);
    }
    if (best == 128) return launch_gemm_t<128, false, true>(a, p, st, experts);
    if (best == 64) return launch_gemm_t<64, false, true>(a, p, st, experts);
    return launch_gemm_t<32, false, true>(a, p, st, experts);
}

unsigned int gemm_read_clear_errors() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_gemm_errors, sizeof(v));
    cudaMemcpyToSymbol(g_gemm_errors, &zero, sizeof(zero));
    return v;
}

}  // namespace w8a8
