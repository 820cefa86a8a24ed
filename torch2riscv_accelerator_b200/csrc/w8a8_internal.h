// Kernel parameter blocks and launchers shared by the .cu files of the library.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>

namespace w8a8 {

// GELU-tanh constants as the reference computes them on the host
// (compiler/frontend/hf_generic.py:848-849: float64, rounded once to float32).
inline float gelu_a_const() { return (float)(-2.0 * std::sqrt(2.0 / 3.141592653589793)); }
inline float gelu_b_const() { return (float)(-2.0 * std::sqrt(2.0 / 3.141592653589793) * 0.044715); }

enum Prologue { PRO_I8 = 0, PRO_QUANT = 1, PRO_RMSQ = 2 };
enum Epilogue { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_PARTIAL = 3 };

// Tensor-parallel decode: every rank owns an exchange region of the same
// layout, mapped into every other rank's process (CUDA IPC over NVLink). A
// kernel addresses a block of another rank's region by the block's offset in
// its own. Exchanged values travel as 8-byte words, the step epoch in the high
// half and the value in the low half: one store carries both, so a reader
// polls the word until it holds this step's epoch (no fence, no flag).
constexpr int kTpMaxRanks = 8;
constexpr int kTpRows = 4;                // rows of a tensor-parallel decode call
constexpr int kTpCtas = 512;              // producer CTAs an exchange block holds
struct TpCtx {
    int rank, ranks;                      // ranks <= 1: no exchange
    char* self;                           // this rank's region (= base[rank])
    char* base[kTpMaxRanks];              // every rank's region (indexed by unrolled loops only)
};

struct LinearParams {
    int m, n, k;              // rows (tokens), outputs, inputs
    const float* x;           // [m, k] fp32 input (PRO_QUANT, PRO_RMSQ)
    const int8_t* xq;         // [m, k] int8 input (PRO_I8)
    const float* s_x;         // [m] its scales (PRO_I8)
    const float* norm_g;      // [k] RMSNorm gain (PRO_RMSQ)
    float eps, inv_k;         // RMSNorm eps and F(1/k)
    const int8_t* w;          // [n, k] int8 rows
    const float* s_w;         // [n]
    const int8_t* w2;         // [n, k] SwiGLU up rows (EPI_SWIGLU)
    const float* s_w2;        // [n]
    float* y;                 // [m, n] fp32 out (EPI_SWIGLU: h)
    const float* resid;       // [m, n] residual (EPI_RESID; may alias y)
    int32_t* acc;             // [m, n] raw int32 accumulators (optional)
    float* s_x_out;           // [m] activation scales of the prologue (optional)
    int8_t* hq;               // [m, n] SwiGLU int8 output
    float* s_h;               // [m] its scales
    uint32_t* amax_bits;      // [m] scratch, zero between launches (EPI_SWIGLU)
    uint32_t* counter;        // [1] scratch, zero between launches (EPI_SWIGLU)
    unsigned long long* argmax_key;   // [m] greedy keys (EPI_STORE, optional; zero before the launch)
    // decode chain (optional): the producer of x posted max|x| per row by atomic
    // max (PRO_QUANT reads it instead of reducing); a SwiGLU posts max|h| per
    // row; `clear` (clear_n words) is zeroed after the wait (a slot whose readers
    // have all finished)
    const uint32_t* amax_in;
    uint32_t* amax_out;
    uint32_t* clear;
    int clear_n;
    int act;                  // EPI_SWIGLU's gate: 0 SiLU, 1 GELU-tanh (constants act_a, act_b)
    float act_a, act_b;
    // tensor-parallel decode (tp.ranks > 1); blocks are addresses in this rank's region
    TpCtx tp;
    const uint64_t* part_in;  // [ranks][kTpRows][k]: the previous row-split linear's int32 partials;
    const float* part_sw;     //   the prologue forms x = part_resid + (f32(sum) * part_sw) * part_sx
    const float* part_sx;     //   ([k], [m]) and CTA 0 stores it to x_out
    const float* part_resid;  // [m, k]
    float* x_out;             // [m, k]
    const uint64_t* amax_ll;  // PRO_QUANT: max|x| words of every rank's producer CTAs
    uint64_t* part_out;       // EPI_PARTIAL: int32 accumulators to every rank
    uint64_t* amax_ll_out;    // EPI_SWIGLU: max|h| of this CTA to every rank
    uint64_t* key_out;        // EPI_STORE: the greedy key of this CTA to every rank
    int n_offset;             // global index of output 0 (a vocabulary slice)
};

cudaError_t launch_linear(const LinearParams& p, int pro, int epi, cudaStream_t st);
bool gemv_fits(const LinearParams& p, int pro, int epi);
int gemv_grid(const LinearParams& p, int pro, int epi);   // CTAs of the decode GEMV launch
cudaError_t launch_gemv(const LinearParams& p, int pro, int epi, cudaStream_t st);
unsigned int gemv_read_clear_errors();
unsigned int attn_read_clear_errors();

struct AttnParams {
    int rows;                 // M query rows of one sequence
    int heads, kv_heads, head_dim, seq_len;
    int variant;              // 0 NORM, 1 QSUM
    int qk_norm;
    const int32_t* pos;       // [M] positions (device)
    const float* qkv;         // [M, (H + 2 Hk) hd]
    const float* q_norm;      // [hd] or null
    const float* k_norm;      // [hd] or null
    float eps, inv_hd;
    const float* cos;         // [seq_len, hd]
    const float* sin;
    float inv_sk, inv_sv, a_k, a_v;
    int8_t* kc;               // [Hk, seq_len, hd] this layer's K cache
    int8_t* vc;               // [Hk, seq_len, hd]
    float* att;               // [M, H hd] out
    int nsplit;               // CTAs per KV head (one thread-block cluster)
    int chunk;                // cache positions per CTA
    int slots;                // batched decode: sequences (one row each; grid z), or 0
    size_t slot_stride;       // bytes between consecutive slots' caches (batched decode)
    int groups;               // prefill: grid z = groups of <= 16 of the rows, whose K / V rows
                              // are already in the cache (kv_append); or 0
    uint32_t* amax_out;       // [rows or slots] max|att| per row by atomic max, or null (decode chain)
    // per cache channel [kv_heads * head_dim], or null for the per-layer scalars:
    // K's scale (folded into q before its quantization) and 1 / s_k; 1 / s_v, a_v
    const float* k_ch;
    const float* inv_sk_ch;
    const float* inv_sv_ch;
    const float* a_v_ch;
    TpCtx tp;                 // tensor-parallel decode: max|att| words of this CTA to every rank
    uint64_t* amax_ll_out;
};

// Tensor-core GEMM (gemm.cu): int8 operands row-major [rows][k], K-major.
struct GemmOperands {
    const int8_t* xq;         // [m, k] activations, quantized per row
    const int8_t* w;          // [n, k]
    const int8_t* w2;         // [n, k] SwiGLU up rows, or null
};
struct GemmParams {
    int m, n, k;
    const float* s_x;         // [m]
    const float* s_w;         // [n]
    const float* s_w2;        // [n] (with w2)
    const float* resid;       // [m, n] or null (may alias y)
    float* y;                 // [m, n]: dequant (+ resid), or h with w2
    int32_t* acc;             // [m, n] raw accumulators, or null (without resid / w2)
    int act;                  // with w2: the gate, 0 SiLU, 1 GELU-tanh (constants act_a, act_b)
    float act_a, act_b;
    // grouped (MoE experts): CTA row blockIdx.y = expert e * g_mtiles + tile;
    // A rows come from e's slab of g_mcap rows, B rows and the column scales
    // from e's block of n rows; slab row r < g_cnt[e] holds pair
    // g_pair[e * g_mcap + r] (row * g_top_k + slot), the output row. s_x is
    // per input row (index pair / g_top_k) with w2, per pair without.
    const int* g_cnt;
    const int* g_pair;
    int g_mcap, g_mtiles, g_top_k;
    const float* g_w;         // without w2: the pair's weight folded in (w_j * y_j)
    uint32_t* g_amax;         // with w2: the pair's max|h| (float bits, atomic max)
};
size_t gemm_smem(int bn, bool two);
// A 2-D uint8 TMA map: [rows][inner] with row_stride bytes between rows
// (16-byte multiples), box box_inner x box_rows, optional 128-byte swizzle.
bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride,
                 uint32_t box_inner, uint32_t box_rows, bool swizzle128);
cudaError_t launch_gemm(const GemmOperands& a, const GemmParams& p, cudaStream_t st);
// grouped: a.xq = the slabs [experts * g_mcap][k], a.w (a.w2) = [experts * n][k]
cudaError_t launch_gemm_grouped(const GemmOperands& a, const GemmParams& p, int experts, cudaStream_t st);
unsigned int gemm_read_clear_errors();
cudaError_t launch_norm_quant(const float* x, const float* g, int m, int k, float eps, float inv_k, int8_t* xq,
                              float* s_x, cudaStream_t st);

// Mixture-of-experts FFN (moe.cu): rows m, model dim, experts E, Top-k, expert hidden ih.
constexpr int kMoeMaxExperts = 64;
constexpr int kMoeMaxTopK = 16;
struct MoeParams {
    int m, dim, experts, top_k, ih;
    const float* x;           // [m, dim] residual stream (the FFN input before its RMSNorm)
    const float* norm_g;      // [dim] the FFN RMSNorm gain
    float eps, inv_dim;
    const int8_t* rq;         // [E, dim] router rows
    const float* rs;          // [E]
    const int8_t* gq;         // [E, ih, dim] gate rows
    const float* gs;          // [E, ih]
    const int8_t* uq;         // [E, ih, dim] up rows
    const float* us;          // [E, ih]
    const int8_t* dq;         // [E, dim, ih] down rows
    const float* ds;          // [E, dim]
    const float* resid;       // [m, dim] (may equal y)
    float* y;                 // [m, dim] out: resid + moe
    int32_t* ids;             // [m, k] chosen experts (out)
    float* w;                 // [m, k] their weights (out)
    int8_t* xq;               // scratch [m, dim]
    float* s_x;               // scratch [m]
    float* h;                 // scratch [m, k, ih]
    uint32_t* amax;           // scratch [m, k]
    // expert parallelism: this rank holds experts [e_lo, e_lo + e_n) (gq .. ds
    // index them from 0); wy [m, k, dim], when set, receives w_j * y_j of the
    // slots of those experts and +0 for the others instead of the combine
    int e_lo, e_n;
    float* wy;
    // ... or, for decode rows (m <= kTpRows), the terms as exchange words into
    // every rank's block: [kTpRows][k][dim] terms, then [ranks][kTpRows]
    // presence words (each rank's down launch started: its earlier kernels,
    // the previous combine included, are complete)
    TpCtx tp;
    uint64_t* wy_ll;
    // many rows on the tensor cores: each of this rank's experts has a slab of
    // mcap rows (a multiple of 128) that the router fills in arrival order
    int8_t* slab_x;           // [e_n][mcap][dim] the int8 rows of the expert's pairs
    int8_t* slab_h;           // [e_n][mcap][ih] their requantized h
    int* cnt;                 // [e_n] rows in each slab (zeroed before the router)
    int* slab_pair;           // [e_n][mcap] the pair (row * k + slot) of each slab row
    int* pair_pos;            // [m * k] the slab row (e * mcap + r) of each pair, -1: another rank's expert
    float* s_h;               // [m * k] each pair's h scale
    int mcap;
};
size_t moe_smem(const MoeParams& p, int which);
cudaError_t launch_moe(const MoeParams& p, cudaStream_t st);
cudaError_t launch_moe_combine(const float* wy, int m, int top_k, int dim, const float* resid, float* y,
                               cudaStream_t st);
// many rows, grouped by expert (combine: fold p.wy onto p.resid into p.y)
cudaError_t launch_moe_rows(const MoeParams& p, bool combine, cudaStream_t st);
size_t moe_rows_smem(const MoeParams& p, int which);
cudaError_t launch_moe_combine_ll(const TpCtx& tp, const uint64_t* wy_ll, int m, int top_k, int dim,
                                  const float* resid, float* y, cudaStream_t st);
unsigned int moe_read_clear_errors();

constexpr int kMaxRows = 16;  // query rows per attention call
constexpr int kMaxCluster = 8;  // attention CTAs per KV head (portable cluster size)

// 0 when the call is supported (the cache chunk of a CTA fits in shared memory),
// else the shared memory it would need
size_t attn_smem_needed(int rows, int heads, int kv_heads, int head_dim, int seq_len, int variant);
bool attn_supported(int rows, int heads, int kv_heads, int head_dim, int seq_len, int variant);
cudaError_t launch_attn(const AttnParams& p, cudaStream_t st);
cudaError_t launch_kv_append(const AttnParams& p, cudaStream_t st);   // rows' K / V into the cache
// batched decode (p.slots > 0, one row per slot): the streaming kernel
size_t attn_stream_smem(int heads, int kv_heads, int head_dim, int seq_len);
cudaError_t launch_attn_stream(const AttnParams& p, cudaStream_t st);

cudaError_t launch_embed(const int32_t* tokens, int m, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
                         float* x, cudaStream_t st, uint32_t* epoch = nullptr);
cudaError_t launch_tp_advance(const TpCtx& tp, const uint64_t* keys, int32_t* tokens, int32_t* pos, int32_t* next,
                              int rows, cudaStream_t st);
cudaError_t launch_tp_seed(const TpCtx& tp, uint64_t* keys, int32_t token, cudaStream_t st);
cudaError_t launch_row_amax(const float* x, int m, int k, uint32_t* amax, cudaStream_t st);
cudaError_t launch_quant_posted(const float* x, const uint32_t* amax, int m, int k, int8_t* xq, float* s_x,
                                cudaStream_t st);
cudaError_t launch_dequant_resid(const int32_t* acc, const float* s_x, const float* s_w, int m, int n,
                                 const float* resid, float* y, cudaStream_t st);
cudaError_t read_clear_errors(unsigned int* out);
cudaError_t launch_argmax(const float* logits, int m, int n, int32_t* out, cudaStream_t st);
cudaError_t launch_sfu(int func, const float* x, float* y, long long n, cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, const float* g, int m, int n, float eps, float inv_n, float* y,
                           cudaStream_t st);
cudaError_t launch_decode_advance(int32_t* tokens, int32_t* pos, unsigned long long* key, int32_t* next, int rows,
                                  cudaStream_t st);
cudaError_t launch_quant_act(const float* x, int m, int k, int8_t* xq, float* s_x, cudaStream_t st);

}  // namespace w8a8
