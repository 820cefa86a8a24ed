// The extern "C" entry points of include/w8a8.h: argument checks, then the
// launches of the kernels in linear.cu, attn.cu and misc.cu.
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/w8a8.h"
#include "trace.cuh"
#include "w8a8_internal.h"

using namespace w8a8;

namespace w8a8 {
int g_use_pdl = 1;
}

namespace {

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? W8A8_OK : W8A8_ECUDA; }
inline float inv_of(int n) { return (float)(1.0 / (double)n); }   // F(1.0 / n), as the host computes it

// Scratch of w8a8_ffn_swiglu_noalloc: the CTA counter (bytes 0-255) and one
// amax slot per row, as w8a8_ffn_swiglu's caller-provided buffer. Static device
// storage exists once per device and is never allocated at run time.
static __device__ __align__(256) unsigned char g_ffn_noalloc_scratch[256 + 4 * W8A8_FFN_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// The device address of g_ffn_noalloc_scratch on the current device, looked up
// once per device (cudaGetSymbolAddress with that device current).
int noalloc_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return W8A8_ECUDA;
    if (dev < 0 || dev >= kMaxDevices) return W8A8_EINVAL;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_ffn_noalloc_scratch) != cudaSuccess || !p) return W8A8_ECUDA;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return W8A8_OK;
}

}  // namespace

extern "C" {

int w8a8_abi_version(void) { return W8A8_ABI_VERSION; }

const char* w8a8_status_string(int s) {
    switch (s) {
        case W8A8_OK: return "ok";
        case W8A8_EINVAL: return "invalid argument (null pointer, size or value)";
        case W8A8_EALIGN: return "pointer or row length not on the 16-byte grid";
        case W8A8_ECUDA: return "CUDA launch failed";
        case W8A8_ESCRATCH: return "scratch buffer too small";
        default: return "unknown status";
    }
}

int w8a8_sfu(int func, const float* x, float* y, int64_t n, void* stream) {
    if (func < 0 || func > 4 || n < 0 || (n > 0 && (!x || !y))) return W8A8_EINVAL;
    if (n == 0) return W8A8_OK;
    return cuda_status(launch_sfu(func, x, y, n, S(stream)));
}

int w8a8_quant_act(const float* x, int rows, int k, int8_t* xq, float* s_x, void* stream) {
    if (!x || !xq || !s_x || rows <= 0 || k <= 0) return W8A8_EINVAL;
    return cuda_status(launch_quant_act(x, rows, k, xq, s_x, S(stream)));
}

int w8a8_rmsnorm(const float* x, const float* g, int rows, int n, float eps, float* y, void* stream) {
    if (!x || !g || !y || rows <= 0 || n <= 0) return W8A8_EINVAL;
    return cuda_status(launch_rmsnorm(x, g, rows, n, eps, inv_of(n), y, S(stream)));
}

int w8a8_embed(const int32_t* tokens, int rows, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
               float* x, void* stream) {
    if (!tokens || !emb_q || !emb_s || !x || rows <= 0 || dim <= 0 || vocab <= 0) return W8A8_EINVAL;
    return cuda_status(launch_embed(tokens, rows, emb_q, emb_s, vocab, dim, x, S(stream)));
}

int w8a8_error_flags(uint32_t* flags) {
    if (!flags) return W8A8_EINVAL;
    unsigned int v = 0;
    int st = cuda_status(read_clear_errors(&v));
    *flags = v | gemv_read_clear_errors() | attn_read_clear_errors() | moe_read_clear_errors() |
             gemm_read_clear_errors();
    return st;
}

int w8a8_set_pdl(int enable) {
    const int old = g_use_pdl;
    g_use_pdl = enable ? 1 : 0;
    return old;
}

int w8a8_trace_bind(void* records, uint32_t* counter, uint32_t capacity) {
    if ((records == nullptr) != (counter == nullptr)) return W8A8_EINVAL;
    if (trace_bind_gemv(records, counter, capacity) || trace_bind_attn(records, counter, capacity) ||
        trace_bind_misc(records, counter, capacity))
        return W8A8_EINVAL;                                    // not a trace build
    return W8A8_OK;
}

static int check_linear(int rows, int k, const void* w, const float* s_w, int n, const void* y) {
    if (!w || !s_w || !y || rows <= 0 || rows > W8A8_MAX_ROWS || k <= 0 || n <= 0) return W8A8_EINVAL;
    if (k % 16 || !al16(w)) return W8A8_EALIGN;
    const int mr = rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : rows <= 8 ? 8 : 16;   // staged rows
    if ((size_t)(mr + 4) * k > 200 * 1024) return W8A8_EINVAL;                           // shared memory
    return W8A8_OK;
}

int w8a8_linear(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w, const float* s_w, int n,
                const float* resid, float* y, int32_t* acc, void* stream) {
    int st = check_linear(rows, k, w, s_w, n, y);
    if (st) return st;
    if (!xq || !s_x || (resid && acc)) return W8A8_EINVAL;
    if (!al16(xq)) return W8A8_EALIGN;
    LinearParams p{};
    p.m = rows, p.n = n, p.k = k, p.xq = xq, p.s_x = s_x, p.w = w, p.s_w = s_w, p.y = y, p.acc = acc;
    p.resid = resid;
    return cuda_status(launch_linear(p, PRO_I8, resid ? EPI_RESID : EPI_STORE, S(stream)));
}

int w8a8_linear_fused(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w,
                      const float* s_w, int n, const float* resid, float* y, float* s_x_out, void* stream) {
    int st = check_linear(rows, k, w, s_w, n, y);
    if (st) return st;
    if (!x) return W8A8_EINVAL;
    if (!al16(x) || (norm_g && !al16(norm_g))) return W8A8_EALIGN;
    LinearParams p{};
    p.m = rows, p.n = n, p.k = k, p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_k = inv_of(k);
    p.w = w, p.s_w = s_w, p.y = y, p.resid = resid, p.s_x_out = s_x_out;
    const int pro = norm_g ? PRO_RMSQ : PRO_QUANT;
    const int epi = resid ? EPI_RESID : EPI_STORE;
    if (pro == PRO_RMSQ && epi == EPI_RESID) return W8A8_EINVAL;
    return cuda_status(launch_linear(p, pro, epi, S(stream)));
}

int w8a8_linear_chain(const float* x, const float* norm_g, float eps, const uint32_t* x_amax, int rows, int k,
                      const int8_t* w, const float* s_w, int n, const float* resid, float* y, uint32_t* clear,
                      int clear_n, void* stream) {
    int st = check_linear(rows, k, w, s_w, n, y);
    if (st) return st;
    if (!x || (norm_g && (x_amax || resid)) || clear_n < 0 || clear_n > 256 || (clear_n > 0 && !clear))
        return W8A8_EINVAL;
    if (!al16(x) || (norm_g && !al16(norm_g))) return W8A8_EALIGN;
    LinearParams p{};
    p.m = rows, p.n = n, p.k = k, p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_k = inv_of(k);
    p.w = w, p.s_w = s_w, p.y = y, p.resid = resid;
    p.amax_in = x_amax, p.clear = clear, p.clear_n = clear ? clear_n : 0;
    const int pro = norm_g ? PRO_RMSQ : PRO_QUANT, epi = resid ? EPI_RESID : EPI_STORE;
    if (!gemv_fits(p, pro, epi)) return W8A8_EINVAL;                // the chain form is the decode GEMV's
    return cuda_status(launch_gemv(p, pro, epi, S(stream)));
}

int w8a8_ffn_swiglu_chain(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                          const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                          uint32_t* h_amax, uint32_t* clear, int clear_n, void* stream) {
    int st = check_linear(rows, k, w_gate, s_gate, hidden, h);
    if (st) return st;
    if (!x || !norm_g || !w_up || !s_up || !h_amax || clear_n < 0 || clear_n > 256 || (clear_n > 0 && !clear))
        return W8A8_EINVAL;
    if (!al16(x) || !al16(norm_g) || !al16(w_up)) return W8A8_EALIGN;
    LinearParams p{};
    p.m = rows, p.n = hidden, p.k = k, p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_k = inv_of(k);
    p.w = w_gate, p.s_w = s_gate, p.w2 = w_up, p.s_w2 = s_up, p.y = h;
    p.amax_out = h_amax, p.clear = clear, p.clear_n = clear ? clear_n : 0;
    if (!gemv_fits(p, PRO_RMSQ, EPI_SWIGLU)) return W8A8_EINVAL;
    return cuda_status(launch_gemv(p, PRO_RMSQ, EPI_SWIGLU, S(stream)));
}

size_t w8a8_ffn_scratch_bytes(int rows) { return 256 + 4 * (size_t)(rows > 0 ? rows : 0); }

static bool set_act(int act, int* kind, float* a, float* b) {
    if (act != W8A8_ACT_SILU && act != W8A8_ACT_GELU_TANH) return false;
    *kind = act, *a = gelu_a_const(), *b = gelu_b_const();
    return true;
}

int w8a8_ffn_swiglu(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                    const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                    int8_t* h_q, float* s_h, void* scratch, size_t scratch_bytes, void* stream) {
    return w8a8_ffn_gated(x, norm_g, eps, rows, k, w_gate, s_gate, w_up, s_up, hidden, W8A8_ACT_SILU, h, h_q, s_h,
                          scratch, scratch_bytes, stream);
}

int w8a8_ffn_gated(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                   const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, int act, float* h,
                   int8_t* h_q, float* s_h, void* scratch, size_t scratch_bytes, void* stream) {
    int st = check_linear(rows, k, w_gate, s_gate, hidden, h);
    if (st) return st;
    if (!x || !norm_g || !w_up || !s_up || (h_q == nullptr) != (s_h == nullptr)) return W8A8_EINVAL;
    if (h_q && !scratch) return W8A8_EINVAL;
    if (!al16(x) || !al16(norm_g) || !al16(w_up) || (scratch && !al16(scratch))) return W8A8_EALIGN;
    if (h_q && hidden % 4) return W8A8_EALIGN;
    if (h_q && scratch_bytes < w8a8_ffn_scratch_bytes(rows)) return W8A8_ESCRATCH;
    LinearParams p{};
    p.m = rows, p.n = hidden, p.k = k, p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_k = inv_of(k);
    p.w = w_gate, p.s_w = s_gate, p.w2 = w_up, p.s_w2 = s_up, p.y = h, p.hq = h_q, p.s_h = s_h;
    if (!set_act(act, &p.act, &p.act_a, &p.act_b)) return W8A8_EINVAL;
    if (scratch) {
        p.counter = static_cast<uint32_t*>(scratch);
        p.amax_bits = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + 256);
    }
    return cuda_status(launch_linear(p, PRO_RMSQ, EPI_SWIGLU, S(stream)));
}

int w8a8_ffn_swiglu_noalloc(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                            const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                            int8_t* h_q, float* s_h, void* stream) {
    if (rows > W8A8_FFN_NOALLOC_MAX_ROWS) return W8A8_ESCRATCH;
    const size_t need = w8a8_ffn_scratch_bytes(rows);
    if (need > sizeof(g_ffn_noalloc_scratch)) return W8A8_ESCRATCH;
    // the checks of w8a8_ffn_swiglu, made here too so that nothing is queued on an error
    int st = check_linear(rows, k, w_gate, s_gate, hidden, h);
    if (st) return st;
    if (!x || !norm_g || !w_up || !s_up || !h_q || !s_h) return W8A8_EINVAL;
    if (!al16(x) || !al16(norm_g) || !al16(w_up) || hidden % 4) return W8A8_EALIGN;
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st) return st;
    // the counter and the amax slots must start at zero; a completed call leaves
    // them zero, a call that gave up part-way may not, so clear them every time
    if (cudaMemsetAsync(scratch, 0, need, S(stream)) != cudaSuccess) return W8A8_ECUDA;
    return w8a8_ffn_swiglu(x, norm_g, eps, rows, k, w_gate, s_gate, w_up, s_up, hidden, h, h_q, s_h, scratch, need,
                           stream);
}

int w8a8_quant_rows(const float* x, const float* norm_g, float eps, int rows, int k, int8_t* xq, float* s_x,
                    void* stream) {
    if (!x || !xq || !s_x || rows <= 0 || k <= 0) return W8A8_EINVAL;
    if (k % 16 || !al16(x) || !al16(xq) || (norm_g && !al16(norm_g))) return W8A8_EALIGN;
    if ((size_t)k * 5 > 200 * 1024) return W8A8_EINVAL;
    return cuda_status(launch_norm_quant(x, norm_g, rows, k, eps, inv_of(k), xq, s_x, S(stream)));
}

static int check_gemm(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w, const float* s_w, int n,
                      const float* y) {
    if (!xq || !s_x || !w || !s_w || !y || rows <= 0 || k <= 0 || n <= 0) return W8A8_EINVAL;
    if (k % 16 || !al16(xq) || !al16(w)) return W8A8_EALIGN;
    return W8A8_OK;
}

int w8a8_gemm(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w, const float* s_w, int n,
              const float* resid, float* y, int32_t* acc, void* stream) {
    int st = check_gemm(xq, s_x, rows, k, w, s_w, n, y);
    if (st) return st;
    if (resid && acc) return W8A8_EINVAL;
    GemmOperands a{xq, w, nullptr};
    GemmParams p{};
    p.m = rows, p.n = n, p.k = k, p.s_x = s_x, p.s_w = s_w, p.resid = resid, p.y = y, p.acc = acc;
    return cuda_status(launch_gemm(a, p, S(stream)));
}

int w8a8_gemm_swiglu(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w_gate, const float* s_gate,
                     const int8_t* w_up, const float* s_up, int hidden, float* h, void* stream) {
    return w8a8_gemm_gated(xq, s_x, rows, k, w_gate, s_gate, w_up, s_up, hidden, W8A8_ACT_SILU, h, stream);
}

int w8a8_gemm_gated(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w_gate, const float* s_gate,
                    const int8_t* w_up, const float* s_up, int hidden, int act, float* h, void* stream) {
    int st = check_gemm(xq, s_x, rows, k, w_gate, s_gate, hidden, h);
    if (st) return st;
    if (!w_up || !s_up) return W8A8_EINVAL;
    if (!al16(w_up)) return W8A8_EALIGN;
    GemmOperands a{xq, w_gate, w_up};
    GemmParams p{};
    p.m = rows, p.n = hidden, p.k = k, p.s_x = s_x, p.s_w = s_gate, p.s_w2 = s_up, p.y = h;
    if (!set_act(act, &p.act, &p.act_a, &p.act_b)) return W8A8_EINVAL;
    return cuda_status(launch_gemm(a, p, S(stream)));
}

static size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t w8a8_moe_scratch_bytes(int rows, int dim, int top_k, int expert_hidden) {
    if (rows <= 0 || dim <= 0 || top_k <= 0 || expert_hidden <= 0) return 0;
    return a256((size_t)rows * dim) + a256((size_t)rows * 4) + a256((size_t)rows * top_k * expert_hidden * 4) +
           a256((size_t)rows * top_k * 4);
}

// the MoE launch of w8a8_moe_ffn (e_n = experts, wy NULL) and w8a8_moe_ffn_ep
static int moe_launch(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                      const float* router_s, int experts, int top_k, int e_lo, int e_n, const int8_t* gate_q,
                      const float* gate_s, const int8_t* up_q, const float* up_s, int expert_hidden,
                      const int8_t* down_q, const float* down_s, const float* resid, float* y, float* wy,
                      int32_t* ids, float* w, void* scratch, size_t scratch_bytes, void* stream,
                      const TpCtx* tp = nullptr, uint64_t* wy_ll = nullptr, bool grouped = false) {
    if (!x || !router_q || !router_s || !gate_q || !gate_s || !up_q || !up_s || !down_q || !down_s ||
        !ids || !w || !scratch || (wy == nullptr && wy_ll == nullptr && (!resid || !y)))
        return W8A8_EINVAL;
    if (e_lo < 0 || e_n <= 0 || e_lo + e_n > experts) return W8A8_EINVAL;
    if (rows <= 0 || rows > (grouped ? W8A8_MOE_MAX_ROWS : W8A8_MAX_ROWS) || dim <= 0 || experts <= 0 ||
        experts > kMoeMaxExperts || top_k <= 0 ||
        top_k > kMoeMaxTopK || top_k > experts || expert_hidden <= 0)
        return W8A8_EINVAL;
    if (dim % (grouped ? 32 : 16) || expert_hidden % 16) return W8A8_EALIGN;
    if (!al16(x) || (norm_g && !al16(norm_g)) || !al16(router_q) || !al16(gate_q) || !al16(up_q) || !al16(down_q) ||
        !al16(scratch))
        return W8A8_EALIGN;
    if (scratch_bytes < (grouped ? w8a8_moe_rows_scratch_bytes(rows, dim, experts, top_k, expert_hidden)
                                 : w8a8_moe_scratch_bytes(rows, dim, top_k, expert_hidden)))
        return W8A8_ESCRATCH;
    MoeParams p{};
    p.m = rows, p.dim = dim, p.experts = experts, p.top_k = top_k, p.ih = expert_hidden;
    p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_dim = inv_of(dim);
    p.rq = router_q, p.rs = router_s, p.gq = gate_q, p.gs = gate_s, p.uq = up_q, p.us = up_s;
    p.dq = down_q, p.ds = down_s, p.resid = resid, p.y = y, p.ids = ids, p.w = w;
    p.e_lo = e_lo, p.e_n = e_n, p.wy = wy, p.wy_ll = wy_ll;
    if (tp != nullptr) p.tp = *tp;
    char* sp = static_cast<char*>(scratch);
    p.xq = reinterpret_cast<int8_t*>(sp);
    sp += a256((size_t)rows * dim);
    p.s_x = reinterpret_cast<float*>(sp);
    sp += a256((size_t)rows * 4);
    p.h = reinterpret_cast<float*>(sp);
    sp += a256((size_t)rows * top_k * expert_hidden * 4);
    p.amax = reinterpret_cast<uint32_t*>(sp);
    if (grouped) {
        sp += a256((size_t)rows * top_k * 4);
        if (p.wy == nullptr) p.wy = reinterpret_cast<float*>(sp);          // the terms, then the combine
        sp += a256((size_t)rows * top_k * dim * 4);
        // the tensor-core path's slabs (sized for all `experts`: e_n <= experts).
        // Above 128 rows (prefill chunks) the tensor cores; at batched-decode
        // sizes the CUDA-core kernels, whose step measured faster on B200 (the
        // tensor-core path's count reset and two more launches cost more than
        // its GEMMs save there)
        const size_t mcap = ((size_t)rows + 127) / 128 * 128;
        if (rows > 128) {
            p.mcap = (int)mcap;
            p.slab_x = reinterpret_cast<int8_t*>(sp);
            sp += a256((size_t)experts * mcap * dim);
            p.slab_h = reinterpret_cast<int8_t*>(sp);
            sp += a256((size_t)experts * mcap * expert_hidden);
            p.cnt = reinterpret_cast<int*>(sp);
            sp += a256((size_t)experts * 4);
            p.slab_pair = reinterpret_cast<int*>(sp);
            sp += a256((size_t)experts * mcap * 4);
            p.pair_pos = reinterpret_cast<int*>(sp);
            sp += a256((size_t)rows * top_k * 4);
            p.s_h = reinterpret_cast<float*>(sp);
        }
        if (moe_smem(p, 0) > 200 * 1024 || moe_rows_smem(p, 1) > 200 * 1024 || moe_rows_smem(p, 2) > 200 * 1024)
            return W8A8_EINVAL;
        return cuda_status(launch_moe_rows(p, wy == nullptr, S(stream)));
    }
    for (int i = 0; i < 3; ++i)
        if (moe_smem(p, i) > 200 * 1024) return W8A8_EINVAL;
    return cuda_status(launch_moe(p, S(stream)));
}

size_t w8a8_moe_rows_scratch_bytes(int rows, int dim, int experts, int top_k, int expert_hidden) {
    if (rows <= 0 || dim <= 0 || experts <= 0 || top_k <= 0 || expert_hidden <= 0) return 0;
    const size_t mcap = ((size_t)rows + 127) / 128 * 128;                // slab rows per expert
    const size_t base = w8a8_moe_scratch_bytes(rows, dim, top_k, expert_hidden) + a256((size_t)rows * top_k * dim * 4);
    if (rows <= 128) return base;                                         // the CUDA-core kernels: no slabs
    return base + a256((size_t)experts * mcap * dim) + a256((size_t)experts * mcap * expert_hidden) +
           a256((size_t)experts * 4) + a256((size_t)experts * mcap * 4) + 2 * a256((size_t)rows * top_k * 4);
}

int w8a8_moe_ffn_rows(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                      const float* router_s, int experts, int top_k, int expert_lo, int experts_local,
                      const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
                      int expert_hidden, const int8_t* down_q, const float* down_s, const float* resid, float* y,
                      float* wy, int32_t* ids, float* w, void* scratch, size_t scratch_bytes, void* stream) {
    if (wy == nullptr && (expert_lo != 0 || experts_local != experts)) return W8A8_EINVAL;
    return moe_launch(x, norm_g, eps, rows, dim, router_q, router_s, experts, top_k, expert_lo, experts_local,
                      gate_q, gate_s, up_q, up_s, expert_hidden, down_q, down_s, wy ? nullptr : resid,
                      wy ? nullptr : y, wy, ids, w, scratch, scratch_bytes, stream, nullptr, nullptr, true);
}

int w8a8_moe_ffn(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                 const float* router_s, int experts, int top_k, const int8_t* gate_q, const float* gate_s,
                 const int8_t* up_q, const float* up_s, int expert_hidden, const int8_t* down_q, const float* down_s,
                 const float* resid, float* y, int32_t* ids, float* w, void* scratch, size_t scratch_bytes,
                 void* stream) {
    return moe_launch(x, norm_g, eps, rows, dim, router_q, router_s, experts, top_k, 0, experts, gate_q, gate_s,
                      up_q, up_s, expert_hidden, down_q, down_s, resid, y, nullptr, ids, w, scratch, scratch_bytes,
                      stream);
}

int w8a8_moe_ffn_ep(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                    const float* router_s, int experts, int top_k, int expert_lo, int experts_local,
                    const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
                    int expert_hidden, const int8_t* down_q, const float* down_s, float* wy, int32_t* ids, float* w,
                    void* scratch, size_t scratch_bytes, void* stream) {
    if (!wy) return W8A8_EINVAL;
    return moe_launch(x, norm_g, eps, rows, dim, router_q, router_s, experts, top_k, expert_lo, experts_local,
                      gate_q, gate_s, up_q, up_s, expert_hidden, down_q, down_s, nullptr, nullptr, wy, ids, w,
                      scratch, scratch_bytes, stream);
}

int w8a8_moe_combine(const float* wy, int rows, int top_k, int dim, const float* resid, float* y, void* stream) {
    if (!wy || !resid || !y || rows <= 0 || rows > 65535 || top_k <= 0 || top_k > kMoeMaxTopK || dim <= 0)
        return W8A8_EINVAL;
    return cuda_status(launch_moe_combine(wy, rows, top_k, dim, resid, y, S(stream)));
}

size_t w8a8_attn_scratch_bytes(int rows, int heads, int kv_heads, int head_dim, int seq_len) {
    (void)rows, (void)heads, (void)kv_heads, (void)head_dim, (void)seq_len;
    return 0;                                                 // the cluster kernel needs no global scratch
}

static int attn_params(const W8A8AttnArgs* a, AttnParams* out) {
    if (!a) return W8A8_EINVAL;
    if (a->rows <= 0 || a->rows > kMaxRows || a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads ||
        a->heads / a->kv_heads > 8 || a->head_dim <= 0 || a->head_dim > 256 || a->seq_len <= 0 ||
        (a->variant != 0 && a->variant != 1))
        return W8A8_EINVAL;
    if (!a->pos || !a->qkv || !a->rope_cos || !a->rope_sin || !a->k_cache || !a->v_cache || !a->att)
        return W8A8_EINVAL;
    if ((a->q_norm == nullptr) != (a->k_norm == nullptr)) return W8A8_EINVAL;
    if (a->head_dim % 16 || a->seq_len % 16 || !al16(a->k_cache) || !al16(a->v_cache)) return W8A8_EALIGN;
    if (!attn_supported(a->rows, a->heads, a->kv_heads, a->head_dim, a->seq_len, a->variant)) return W8A8_EINVAL;
    AttnParams p{};
    p.rows = a->rows, p.heads = a->heads, p.kv_heads = a->kv_heads, p.head_dim = a->head_dim;
    p.seq_len = a->seq_len, p.variant = a->variant, p.qk_norm = a->q_norm != nullptr;
    p.pos = a->pos, p.qkv = a->qkv, p.q_norm = a->q_norm, p.k_norm = a->k_norm, p.eps = a->eps;
    p.inv_hd = inv_of(a->head_dim), p.cos = a->rope_cos, p.sin = a->rope_sin;
    p.inv_sk = a->inv_sk, p.inv_sv = a->inv_sv, p.a_k = a->a_k, p.a_v = a->a_v;
    p.kc = a->k_cache, p.vc = a->v_cache, p.att = a->att, p.amax_out = a->att_amax;
    if ((a->k_scale == nullptr) != (a->inv_sk_ch == nullptr) || (a->inv_sv_ch == nullptr) != (a->a_v_ch == nullptr))
        return W8A8_EINVAL;                                   // a part is per channel or not, whole
    p.k_ch = a->k_scale, p.inv_sk_ch = a->inv_sk_ch, p.inv_sv_ch = a->inv_sv_ch, p.a_v_ch = a->a_v_ch;
    *out = p;
    return W8A8_OK;
}

int w8a8_attn(const W8A8AttnArgs* a, void* stream) {
    AttnParams p{};
    const int st = attn_params(a, &p);
    return st ? st : cuda_status(launch_attn(p, S(stream)));
}

// rows of one sequence beyond 16 (a prefill chunk): checked as a 16-row call
static int attn_rows_params(const W8A8AttnArgs* a, AttnParams* out) {
    if (!a || a->rows <= 0 || a->rows > 65535 * kMaxRows) return W8A8_EINVAL;
    W8A8AttnArgs c = *a;
    c.rows = a->rows < kMaxRows ? a->rows : kMaxRows;
    const int st = attn_params(&c, out);
    if (st) return st;
    out->rows = a->rows;
    return W8A8_OK;
}

int w8a8_kv_append(const W8A8AttnArgs* a, void* stream) {
    AttnParams p{};
    const int st = attn_rows_params(a, &p);
    return st ? st : cuda_status(launch_kv_append(p, S(stream)));
}

int w8a8_attn_prefill(const W8A8AttnArgs* a, void* stream) {
    AttnParams p{};
    const int st = attn_rows_params(a, &p);
    if (st) return st;
    p.groups = (a->rows + kMaxRows - 1) / kMaxRows;
    return cuda_status(launch_attn(p, S(stream)));
}

int w8a8_attn_batch(const W8A8AttnArgs* a, int slots, size_t slot_stride, void* stream) {
    AttnParams p{};
    const int st = attn_params(a, &p);
    if (st) return st;
    if (a->rows != 1 || slots <= 0 || slots > 65535) return W8A8_EINVAL;
    if (slot_stride % 16) return W8A8_EALIGN;
    if (slots > 1 && slot_stride < (size_t)a->kv_heads * a->seq_len * a->head_dim) return W8A8_EINVAL;
    if (slot_stride % (size_t)a->head_dim || slot_stride % (size_t)a->seq_len) return W8A8_EALIGN;
    if (attn_stream_smem(a->heads, a->kv_heads, a->head_dim, a->seq_len) > 200 * 1024) return W8A8_EINVAL;
    p.slots = slots, p.slot_stride = slot_stride;
    return cuda_status(launch_attn_stream(p, S(stream)));
}

int w8a8_argmax(const float* logits, int rows, int n, int32_t* out, void* stream) {
    if (!logits || !out || rows <= 0 || n <= 0) return W8A8_EINVAL;
    return cuda_status(launch_argmax(logits, rows, n, out, S(stream)));
}

int w8a8_classifier(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w,
                    const float* s_w, int n, float* logits, uint64_t* argmax_key, void* stream) {
    int st = check_linear(rows, k, w, s_w, n, logits);
    if (st) return st;
    if (!x || !norm_g) return W8A8_EINVAL;
    if (!al16(x) || !al16(norm_g)) return W8A8_EALIGN;
    LinearParams p{};
    p.m = rows, p.n = n, p.k = k, p.x = x, p.norm_g = norm_g, p.eps = eps, p.inv_k = inv_of(k);
    p.w = w, p.s_w = s_w, p.y = logits, p.argmax_key = reinterpret_cast<unsigned long long*>(argmax_key);
    return cuda_status(launch_linear(p, PRO_RMSQ, EPI_STORE, S(stream)));
}

int w8a8_decode_advance(int32_t* tokens, int32_t* pos, uint64_t* argmax_key, int32_t* next_token, int rows,
                        void* stream) {
    if (!tokens || !pos || !argmax_key || rows <= 0 || rows > 32) return W8A8_EINVAL;
    return cuda_status(launch_decode_advance(tokens, pos, reinterpret_cast<unsigned long long*>(argmax_key),
                                             next_token, rows, S(stream)));
}

// ---------------------------------------------------------------- tensor parallel
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
static_assert(W8A8_TP_MAX_RANKS == kTpMaxRanks && W8A8_TP_ROWS == kTpRows && W8A8_TP_CTAS == kTpCtas,
              "exchange layout");

static int tp_ctx(const W8A8TpComm* c, TpCtx* t) {
    if (!c || c->ranks < 2 || c->ranks > W8A8_TP_MAX_RANKS || c->rank < 0 || c->rank >= c->ranks ||
        c->bytes < W8A8_TP_HEADER)
        return W8A8_EINVAL;
    *t = TpCtx{};
    t->rank = c->rank, t->ranks = c->ranks;
    for (int r = 0; r < c->ranks; ++r) {
        if (!c->base[r]) return W8A8_EINVAL;
        if (!al16(c->base[r])) return W8A8_EALIGN;
        t->base[r] = static_cast<char*>(c->base[r]);
    }
    t->self = t->base[c->rank];
    return W8A8_OK;
}

// a block of `words` 8-byte words inside this rank's region, past the header
static bool tp_block(const W8A8TpComm* c, const void* p, size_t words) {
    if (!p || !al16(p)) return false;
    const char* b = static_cast<const char*>(c->base[c->rank]);
    const char* q = static_cast<const char*>(p);
    return q >= b + W8A8_TP_HEADER && (size_t)(q - b) + words * 8 <= c->bytes;
}

int w8a8_tp_alloc(size_t bytes, void** region) {
    if (!region || bytes < W8A8_TP_HEADER) return W8A8_EINVAL;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return W8A8_ECUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return W8A8_ECUDA;
    }
    *region = p;
    return W8A8_OK;
}

int w8a8_tp_free(void* region) { return region ? cuda_status(cudaFree(region)) : W8A8_EINVAL; }

int w8a8_ipc_handle(const void* region, uint8_t handle[64]) {
    if (!region || !handle) return W8A8_EINVAL;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void*>(region)) != cudaSuccess) return W8A8_ECUDA;
    memcpy(handle, &h, sizeof(h));
    return W8A8_OK;
}

int w8a8_ipc_open(const uint8_t handle[64], void** region) {
    if (!handle || !region) return W8A8_EINVAL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess));
}

int w8a8_ipc_close(void* region) { return region ? cuda_status(cudaIpcCloseMemHandle(region)) : W8A8_EINVAL; }

int w8a8_tp_embed(const W8A8TpComm* comm, const int32_t* tokens, int rows, const int8_t* emb_q, const float* emb_s,
                  int vocab, int dim, float* x, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    if (!tokens || !emb_q || !emb_s || !x || rows <= 0 || vocab <= 0 || dim <= 0) return W8A8_EINVAL;
    return cuda_status(launch_embed(tokens, rows, emb_q, emb_s, vocab, dim, x, S(stream),
                                    reinterpret_cast<uint32_t*>(t.self)));
}

int w8a8_tp_linear(const W8A8TpLinearArgs* a, void* stream) {
    if (!a) return W8A8_EINVAL;
    TpCtx t;
    int st = tp_ctx(a->comm, &t);
    if (st) return st;
    const W8A8TpComm* c = a->comm;
    const int epi = a->epilogue == W8A8_TP_STORE ? EPI_STORE
                    : a->epilogue == W8A8_TP_PARTIAL ? EPI_PARTIAL
                    : a->epilogue == W8A8_TP_SWIGLU ? EPI_SWIGLU : -1;
    if (epi < 0 || a->rows <= 0 || a->rows > W8A8_TP_ROWS) return W8A8_EINVAL;
    st = check_linear(a->rows, a->k, a->w, a->s_w, a->n, epi == EPI_PARTIAL ? (const void*)a->part_out : a->y);
    if (st) return st;
    LinearParams p{};
    p.m = a->rows, p.n = a->n, p.k = a->k, p.x = a->x, p.norm_g = a->norm_g, p.eps = a->eps;
    p.inv_k = inv_of(a->k), p.w = a->w, p.s_w = a->s_w, p.s_x_out = a->s_x_out, p.tp = t;
    if (a->part_in) {
        if (!tp_block(c, a->part_in, W8A8_TP_PART_WORDS(c->ranks, a->k)) || !a->part_s_w || !a->part_s_x ||
            !a->resid || !a->x_out || a->x_out == a->resid)
            return W8A8_EINVAL;
        if (!al16(a->resid) || !al16(a->x_out) || !al16(a->part_s_w)) return W8A8_EALIGN;
        p.part_in = a->part_in, p.part_sw = a->part_s_w, p.part_sx = a->part_s_x;
        p.part_resid = a->resid, p.x_out = a->x_out;
    } else {
        if (!a->x) return W8A8_EINVAL;
        if (!al16(a->x)) return W8A8_EALIGN;
    }
    if (a->norm_g && !al16(a->norm_g)) return W8A8_EALIGN;
    if (a->amax_in) {
        if (a->norm_g || !tp_block(c, a->amax_in, W8A8_TP_AMAX_WORDS(c->ranks))) return W8A8_EINVAL;
        p.amax_ll = a->amax_in;
    }
    const int pro = a->norm_g ? PRO_RMSQ : PRO_QUANT;
    if (epi == EPI_STORE) {
        if (a->key_out && !tp_block(c, a->key_out, W8A8_TP_KEY_WORDS(c->ranks))) return W8A8_EINVAL;
        if (a->n_offset < 0) return W8A8_EINVAL;
        p.y = a->y, p.key_out = a->key_out, p.n_offset = a->n_offset;
    } else if (epi == EPI_PARTIAL) {
        if (!tp_block(c, a->part_out, W8A8_TP_PART_WORDS(c->ranks, a->n))) return W8A8_EINVAL;
        p.part_out = a->part_out;
    } else {
        if (!a->w_up || !a->s_up || !tp_block(c, a->amax_out, W8A8_TP_AMAX_WORDS(c->ranks))) return W8A8_EINVAL;
        if (!al16(a->w_up)) return W8A8_EALIGN;
        p.w2 = a->w_up, p.s_w2 = a->s_up, p.y = a->y, p.amax_ll_out = a->amax_out;
        if (!set_act(a->act, &p.act, &p.act_a, &p.act_b)) return W8A8_EINVAL;
    }
    if (!gemv_fits(p, pro, epi) || gemv_grid(p, pro, epi) > kTpCtas) return W8A8_EINVAL;
    return cuda_status(launch_gemv(p, pro, epi, S(stream)));
}

int w8a8_tp_attn(const W8A8AttnArgs* a, const W8A8TpComm* comm, uint64_t* amax_out, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    AttnParams p{};
    st = attn_params(a, &p);
    if (st) return st;
    if (a->rows > W8A8_TP_ROWS || !tp_block(comm, amax_out, W8A8_TP_AMAX_WORDS(comm->ranks))) return W8A8_EINVAL;
    if ((size_t)a->kv_heads * kMaxCluster > (size_t)kTpCtas) return W8A8_EINVAL;
    p.tp = t, p.amax_ll_out = amax_out;
    return cuda_status(launch_attn(p, S(stream)));
}

int w8a8_tp_advance(const W8A8TpComm* comm, const uint64_t* keys, int32_t* tokens, int32_t* pos,
                    int32_t* next_token, int rows, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    if (!tokens || !pos || rows <= 0 || rows > W8A8_TP_ROWS || !tp_block(comm, keys, W8A8_TP_KEY_WORDS(comm->ranks)))
        return W8A8_EINVAL;
    return cuda_status(launch_tp_advance(t, keys, tokens, pos, next_token, rows, S(stream)));
}

int w8a8_tp_seed(const W8A8TpComm* comm, uint64_t* keys, int32_t token, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    if (token < 0 || !tp_block(comm, keys, W8A8_TP_KEY_WORDS(comm->ranks))) return W8A8_EINVAL;
    return cuda_status(launch_tp_seed(t, keys, token, S(stream)));
}

int w8a8_row_amax(const float* x, int rows, int k, uint32_t* amax_bits, void* stream) {
    if (!x || !amax_bits || rows <= 0 || rows > 65535 || k <= 0) return W8A8_EINVAL;
    return cuda_status(launch_row_amax(x, rows, k, amax_bits, S(stream)));
}

int w8a8_quant_rows_posted(const float* x, const uint32_t* amax_bits, int rows, int k, int8_t* xq, float* s_x,
                           void* stream) {
    if (!x || !amax_bits || !xq || !s_x || rows <= 0 || rows > 65535 || k <= 0) return W8A8_EINVAL;
    if (k % 4 || !al16(x) || (reinterpret_cast<uintptr_t>(xq) & 3u)) return W8A8_EALIGN;
    return cuda_status(launch_quant_posted(x, amax_bits, rows, k, xq, s_x, S(stream)));
}

int w8a8_dequant_resid(const int32_t* acc, const float* s_x, const float* s_w, int rows, int n, const float* resid,
                       float* y, void* stream) {
    if (!acc || !s_x || !s_w || !y || rows <= 0 || rows > 65535 || n <= 0) return W8A8_EINVAL;
    return cuda_status(launch_dequant_resid(acc, s_x, s_w, rows, n, resid, y, S(stream)));
}

int w8a8_tp_moe_ffn(const W8A8TpComm* comm, const float* x, const float* norm_g, float eps, int rows, int dim,
                    const int8_t* router_q, const float* router_s, int experts, int top_k, int expert_lo,
                    int experts_local, const int8_t* gate_q, const float* gate_s, const int8_t* up_q,
                    const float* up_s, int expert_hidden, const int8_t* down_q, const float* down_s, uint64_t* terms,
                    int32_t* ids, float* w, void* scratch, size_t scratch_bytes, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    if (rows <= 0 || rows > W8A8_TP_ROWS || top_k <= 0 || top_k > kMoeMaxTopK || dim <= 0 ||
        !tp_block(comm, terms, W8A8_TP_MOE_WORDS(comm->ranks, top_k, dim)))
        return W8A8_EINVAL;
    return moe_launch(x, norm_g, eps, rows, dim, router_q, router_s, experts, top_k, expert_lo, experts_local,
                      gate_q, gate_s, up_q, up_s, expert_hidden, down_q, down_s, nullptr, nullptr, nullptr, ids, w,
                      scratch, scratch_bytes, stream, &t, terms);
}

int w8a8_tp_moe_combine(const W8A8TpComm* comm, const uint64_t* terms, int rows, int top_k, int dim,
                        const float* resid, float* y, void* stream) {
    TpCtx t;
    int st = tp_ctx(comm, &t);
    if (st) return st;
    if (!resid || !y || rows <= 0 || rows > W8A8_TP_ROWS || top_k <= 0 || top_k > kMoeMaxTopK || dim <= 0 ||
        !tp_block(comm, terms, W8A8_TP_MOE_WORDS(comm->ranks, top_k, dim)))
        return W8A8_EINVAL;
    return cuda_status(launch_moe_combine_ll(t, terms, rows, top_k, dim, resid, y, S(stream)));
}

}  // extern "C"
