/* C ABI of the B200 W8A8 decode path (libw8a8_b200.so).
 *
 * Drop-in backend for the operators that Torch2RISCV-accelerator's host runtime
 * submits to the overlay as descriptor lists (llm/compile_model.py builds them,
 * llm/sa_funcsim.py is their bit-exact model, driver/pynq_matmul.py
 * Device.submit/wait runs them). Each entry point replaces one fused dispatch
 * and states the reference code it replaces.
 *
 * Conventions
 * - All pointers are device pointers (cudaMalloc / torch tensors), row-major,
 *   16-byte aligned; int8 row lengths (k, hidden) are multiples of 16.
 * - `stream` is a cudaStream_t (NULL: the legacy default stream). Calls are
 *   asynchronous and stream-ordered; nothing allocates, nothing synchronizes.
 * - Return 0 (W8A8_OK) or an error code; nothing is launched on an error
 *   (arguments are checked before any launch). No exceptions cross the ABI.
 * - Numerics are the overlay's: fp32 steps rounded once each (RNE, never fused),
 *   EXP/RECIP/RSQRT from the SFU tables (llm/sfu.py), fixed D = 16 lane sums,
 *   int8 = RNE saturated to +-127 with NaN -> 0.
 */
#ifndef W8A8_B200_H
#define W8A8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W8A8_OK 0
#define W8A8_EINVAL 1   /* a null pointer, a bad size or an unsupported value */
#define W8A8_EALIGN 2   /* a pointer or a row length off the 16-byte grid */
#define W8A8_ECUDA 3    /* the CUDA launch failed (cudaGetLastError) */
#define W8A8_ESCRATCH 4 /* the scratch buffer is smaller than required */

#define W8A8_ABI_VERSION 6
#define W8A8_MAX_ROWS 16 /* query rows per call (decode: 1, prefill chunk: 16) */

/* ABI version (W8A8_ABI_VERSION) and a message for a status code. */
int w8a8_abi_version(void);
const char* w8a8_status_string(int status);

/* Elementwise SFU: func 0 EXP, 1 RECIP, 2 RSQRT (llm/sfu.py:69, :85, :99),
 * 3 SiLU g*RECIP(1 + EXP(-g)) (llm/ref_model.py:249), 4 GELU-tanh
 * g*RECIP(EXP(g*(A + (g*g)*B)) + 1) (compiler/frontend/hf_generic.py:840-856). */
int w8a8_sfu(int func, const float* x, float* y, int64_t n, void* stream);

/* Per-token dynamic int8 of `rows` rows of k values: s_x = max|x| * F(1/127),
 * xq = i8(x * RECIP(s_x)). Replaces DeviceModel.quant_act (llm/ref_model.py:191)
 * and compile_layer.quant_act (llm/compile_layer.py:66-77). */
int w8a8_quant_act(const float* x, int rows, int k, int8_t* xq, float* s_x, void* stream);

/* RMSNorm rows: y = (x * RSQRT(red_sum16(x*x) * F(1/n) + eps)) * g.
 * Replaces DeviceModel.rmsnorm (llm/ref_model.py:204) and
 * ModelCompiler.rmsnorm (llm/compile_model.py:147-156). */
int w8a8_rmsnorm(const float* x, const float* g, int rows, int n, float eps, float* y, void* stream);

/* Embedding rows: x[m] = f32(emb_q[tokens[m]]) * emb_s[tokens[m]], emb_q [vocab, dim].
 * A token outside [0, vocab) gives a zero row and sets bit 0 of the device
 * error flags. Replaces ModelCompiler.embed (llm/compile_model.py:192-201). */
int w8a8_embed(const int32_t* tokens, int rows, const int8_t* emb_q, const float* emb_s, int vocab, int dim,
               float* x, void* stream);

/* Read and clear the current device's error flags (bit 0: an out-of-range
 * token reached w8a8_embed; bit 1: a GEMV weight-tile wait gave up after its
 * bounded spin and the kernel stopped early; bit 2: an attention cache-tile
 * copy did not land within its bounded wait; bit 3: the same for an MoE weight
 * tile; bit 4: a tensor-core GEMM pipeline wait; bit 5: a tensor-parallel
 * exchange wait gave up; bit 6: w8a8_moe_ffn_rows found more pairs of one
 * expert than rows, routing that is not Top-k, and skipped the excess).
 * Synchronous with the device.
 * Plays the role of the overlay's sticky list status (llm/sa_funcsim.py:62-66,
 * firmware/rt/rt_fw.c:53-60). */
int w8a8_error_flags(uint32_t* flags);

/* Launch the kernels with programmatic dependent launch (1, the default) or
 * with plain stream ordering (0); returns the previous setting. Results are
 * identical either way; with it a kernel starts streaming its weights while
 * its predecessor finishes. Process-wide; not for concurrent callers. */
int w8a8_set_pdl(int enable);

/* Device timeline (trace builds only, -DW8A8_TRACE: libw8a8_b200_trace.so):
 * point the instrumented decode kernels at `records` (capacity records of 3
 * uint64: global timer ns, SM clock, kind << 56 | mark << 48 | smid << 32 |
 * CTA) and the device counter of records taken; null pointers stop recording.
 * W8A8_EINVAL in a normal build. The counterpart of the overlay's event
 * counters and profile dump (rtl/sysarray/sa_perf.v,
 * compiler/runtime/sa/sa_context.c:507-535). */
int w8a8_trace_bind(void* records, uint32_t* counter, uint32_t capacity);

/* W8A8 linear on int8 activations: acc = xq . W^T (int32), y = (f32(acc) * s_w) * s_x,
 * or y = resid + that when resid is not NULL (resid may equal y).
 * w: [n, k] int8 rows, s_w: [n]; xq: [rows, k], s_x: [rows]; y: [rows, n];
 * acc: [rows, n] int32 or NULL (only without resid). Replaces DeviceModel.linear
 * (llm/ref_model.py:198), compile_layer.linear (llm/compile_layer.py:93-182), the
 * GEMV command SaFuncSim.gemv (llm/sa_funcsim.py:138-162) and linear(w2) +
 * residual (llm/compile_model.py:343-344). */
int w8a8_linear(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w, const float* s_w, int n,
                const float* resid, float* y, int32_t* acc, void* stream);

/* Fused [rmsnorm ->] quant_act -> W8A8 linear [-> + residual] on fp32 rows x [rows, k].
 * norm_g: [k] RMSNorm gain, or NULL for quant_act(x) alone; resid: [rows, n] or
 * NULL (y = resid + linear; resid may equal y); s_x_out: [rows] or NULL.
 * Replaces the sequences rmsnorm + linear(wqkv / wcls) and linear(wo / w2) +
 * residual of ModelCompiler.layer / final (llm/compile_model.py:333-349). */
int w8a8_linear_fused(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w,
                      const float* s_w, int n, const float* resid, float* y, float* s_x_out, void* stream);

/* The decode chain's form of w8a8_linear_fused (the same results): x_amax
 * [rows] (quant_act without norm only) is max|x| per row already posted by the
 * kernel that wrote x (w8a8_attn's att_amax, w8a8_ffn_swiglu_chain's h_amax),
 * so the prologue skips its block-wide reduction; clear (clear_n words, or
 * NULL) is zeroed once this kernel has waited for its predecessors: a slot
 * whose readers have all finished, ready for the next step's atomics. */
int w8a8_linear_chain(const float* x, const float* norm_g, float eps, const uint32_t* x_amax, int rows, int k,
                      const int8_t* w, const float* s_w, int n, const float* resid, float* y, uint32_t* clear,
                      int clear_n, void* stream);

/* Decode SwiGLU dispatch: [rmsnorm ->] quant_act(x) -> gate and up W8A8 GEMVs ->
 * h = (g * RECIP(1 + EXP(-g))) * u -> amax -> h_q = i8(h * RECIP(amax * F(1/127))).
 * w_gate, w_up: [hidden, k]; h: [rows, hidden] fp32; h_q: [rows, hidden] int8,
 * s_h: [rows]. scratch: w8a8_ffn_scratch_bytes() bytes, zero before the first
 * call, left zero by every call. With h_q, s_h and scratch all NULL the call
 * stops at h (a following w8a8_linear_fused on h does the same quant_act in its
 * prologue: the decode chain uses that, it saves the grid-wide amax). Replaces ModelCompiler.ffn_up with fused SiLU
 * (llm/compile_model.py:295-328) and the FFN region of the IREE plugin
 * (FfnPlan, compiler/plugins/sa/transforms/SahlKernels.h:130-141). */
size_t w8a8_ffn_scratch_bytes(int rows);
int w8a8_ffn_swiglu(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                    const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                    int8_t* h_q, float* s_h, void* scratch, size_t scratch_bytes, void* stream);

/* The decode chain's SwiGLU: stops at h (no requantization) and posts max|h|
 * per row into h_amax (zero before the call) by atomic max for the down
 * projection's w8a8_linear_chain; clear as in w8a8_linear_chain. */
int w8a8_ffn_swiglu_chain(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                          const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                          uint32_t* h_amax, uint32_t* clear, int clear_n, void* stream);

/* Gated activations of the FFN dispatch: SiLU (Llama, Qwen3, Granite) or GELU's
 * tanh approximation (Gemma: hf_generic.SaGELUTanh, :840-856, with
 * A = F(-2 sqrt(2/pi)), B = F(-2 sqrt(2/pi) * 0.044715) as the reference's
 * host computes them). w8a8_ffn_gated / w8a8_gemm_gated are w8a8_ffn_swiglu /
 * w8a8_gemm_swiglu with h = act(g) * u. */
#define W8A8_ACT_SILU 0
#define W8A8_ACT_GELU_TANH 1
int w8a8_ffn_gated(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                   const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, int act, float* h,
                   int8_t* h_q, float* s_h, void* scratch, size_t scratch_bytes, void* stream);
int w8a8_gemm_gated(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w_gate, const float* s_gate,
                    const int8_t* w_up, const float* s_up, int hidden, int act, float* h, void* stream);

/* w8a8_ffn_swiglu with the requantization of h, for a caller that cannot hand
 * over a scratch buffer. This entry point has no counterpart in the reference:
 * the overlay's runtime owns one buffer for everything, so the question never
 * comes up there.
 *
 * Who needs it: a host that reserves all of its device memory once at start-up
 * (an arena or a memory pool with nothing left to give), or a plugin called
 * by a framework that hands it tensors but no allocator. cudaMalloc there is
 * either impossible or would synchronize the whole device in the middle of a
 * step. Here the grid-wide amax and the CTA counter live in a small static
 * device array inside the library (one per device, 320 bytes, enough for
 * W8A8_FFN_NOALLOC_MAX_ROWS rows), so nothing is allocated.
 *
 * - rows > W8A8_FFN_NOALLOC_MAX_ROWS returns W8A8_ESCRATCH (the static array
 *   is too small); h_q and s_h are required (without them use w8a8_ffn_swiglu,
 *   which then needs no scratch at all).
 * - The first call on each device looks up the array's device address with
 *   that device current; make that first call before any stream capture.
 * - Each call clears the array on `stream` before its launch.
 * - The array is shared by every call on the device: two calls that can run at
 *   the same time (other streams, other host threads) race. Order them.
 * Same arguments and results as w8a8_ffn_swiglu otherwise. */
#define W8A8_FFN_NOALLOC_MAX_ROWS 16
int w8a8_ffn_swiglu_noalloc(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w_gate,
                            const float* s_gate, const int8_t* w_up, const float* s_up, int hidden, float* h,
                            int8_t* h_q, float* s_h, void* stream);

/* Rows of x -> int8 rows for the tensor-core GEMM: xq = quant_act(x), or
 * quant_act(rmsnorm(x, norm_g)) when norm_g is not NULL; s_x [rows]. Any row
 * count. Replaces the quant_act (+ rmsnorm) steps that precede each linear of
 * a prefill chunk (compiler/frontend/qhf.py:376-405, llm/ref_model.py:191-207). */
int w8a8_quant_rows(const float* x, const float* norm_g, float eps, int rows, int k, int8_t* xq, float* s_x,
                    void* stream);

/* W8A8 linear for any number of rows on the tensor cores (tcgen05 kind::i8,
 * int32 accumulators in tensor memory): the same results as w8a8_linear, bit
 * for bit. xq [rows, k] int8 (w8a8_quant_rows), s_x [rows]; w [n, k], s_w [n];
 * y [rows, n] = (f32(acc) * s_w) * s_x [+ resid]; acc [rows, n] or NULL.
 * Replaces the prefill linear rows (SahlExpandKernels.cpp expandLinearRows,
 * compiler/frontend/qhf.py:376-405) and batched decode linears
 * (llm/runtime.py BatchLlamaDevice.step :193-208). */
int w8a8_gemm(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w, const float* s_w, int n,
              const float* resid, float* y, int32_t* acc, void* stream);

/* The SwiGLU pair on the tensor cores: h = (g * RECIP(1 + EXP(-g))) * u with
 * g, u the W8A8 linears of w_gate and w_up [hidden, k] (llm/ref_model.py:246-250;
 * the prefill FFN of compiler/frontend/qhf.py:396-400). h [rows, hidden]. */
int w8a8_gemm_swiglu(const int8_t* xq, const float* s_x, int rows, int k, const int8_t* w_gate, const float* s_gate,
                     const int8_t* w_up, const float* s_up, int hidden, float* h, void* stream);

/* Mixture-of-experts FFN for up to 16 rows, each with its own Top-k:
 * y = resid + sum_k w_k * expert_k(rmsnorm(x)), where the router's W8A8 logits
 * (router_q [experts, dim]) give the Top-k by value (ties: the lower id),
 * w = e * RECIP(sum e), e = EXP(v - v_0) (D = 16 ordered sum), and expert i is
 * the SwiGLU down(quant_act((g * RECIP(1 + EXP(-g))) * u)) with gate_q, up_q
 * [experts, expert_hidden, dim] and down_q [experts, dim, expert_hidden]; the
 * k results are folded in k order from 0. norm_g NULL: x is already the
 * normalized input (no RMSNorm). ids, w: [rows, top_k] outputs (the
 * routing). resid may equal y. scratch: w8a8_moe_scratch_bytes() bytes.
 * experts <= 64, top_k <= 16. Replaces hf_generic.QMixtralMoe.route / _row
 * (compiler/frontend/hf_generic.py:641-657) and the MoE lowering of the IREE
 * plugin (docs/moe_native_lowering_design.md). */
size_t w8a8_moe_scratch_bytes(int rows, int dim, int top_k, int expert_hidden);
int w8a8_moe_ffn(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                 const float* router_s, int experts, int top_k, const int8_t* gate_q, const float* gate_s,
                 const int8_t* up_q, const float* up_s, int expert_hidden, const int8_t* down_q, const float* down_s,
                 const float* resid, float* y, int32_t* ids, float* w, void* scratch, size_t scratch_bytes,
                 void* stream);

/* Expert parallelism (no counterpart in the reference, which runs on one
 * device): this rank holds experts [expert_lo, expert_lo + experts_local) of
 * the router's `experts` (gate_q .. down_s hold only those, indexed from 0);
 * the router runs whole. wy [rows, top_k, dim] receives w_j * y_j for the
 * slots of this rank's experts and +0 for the others (no combine, no
 * residual). An all-reduce SUM of wy over the ranks is exact (each element has
 * one nonzero contributor), and w8a8_moe_combine then folds it in k order:
 * y = resid + (((0 + t_0) + t_1) + ...) -- w8a8_moe_ffn's result bit for bit. */
int w8a8_moe_ffn_ep(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                    const float* router_s, int experts, int top_k, int expert_lo, int experts_local,
                    const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
                    int expert_hidden, const int8_t* down_q, const float* down_s, float* wy, int32_t* ids, float* w,
                    void* scratch, size_t scratch_bytes, void* stream);
int w8a8_moe_combine(const float* wy, int rows, int top_k, int dim, const float* resid, float* y, void* stream);

/* The MoE FFN of w8a8_moe_ffn (wy NULL: y = resid + the k-order fold, with
 * expert_lo 0 and experts_local = experts) or of w8a8_moe_ffn_ep (wy non-NULL:
 * the terms, resid and y unused) for up to W8A8_MOE_MAX_ROWS rows (batched
 * decode, prefill chunks), the same results bit for bit. The rows' (row, slot)
 * pairs are grouped by expert on the device, so each expert's weight tiles are
 * read once per call rather than once per pair (above 128 rows on the tensor
 * cores: grouped tcgen05 GEMMs over per-expert slabs of the rows). scratch:
 * w8a8_moe_rows_scratch_bytes() bytes: the w8a8_moe_ffn scratch plus
 * rows * top_k * dim fp32 terms, and above 128 rows each expert's slabs,
 * experts * ceil(rows / 128) * 128 * (dim + expert_hidden + 4) bytes, with two
 * rows * top_k per-pair arrays (about 200 MB at 4096 rows of a 32-expert,
 * dim 1024, hidden 512 layer); dim a multiple of 32. The reference runs the MoE per row
 * (compiler/frontend/hf_generic.py:641-657); this is that loop over a batch. */
#define W8A8_MOE_MAX_ROWS 4096
size_t w8a8_moe_rows_scratch_bytes(int rows, int dim, int experts, int top_k, int expert_hidden);
int w8a8_moe_ffn_rows(const float* x, const float* norm_g, float eps, int rows, int dim, const int8_t* router_q,
                      const float* router_s, int experts, int top_k, int expert_lo, int experts_local,
                      const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
                      int expert_hidden, const int8_t* down_q, const float* down_s, const float* resid, float* y,
                      float* wy, int32_t* ids, float* w, void* scratch, size_t scratch_bytes, void* stream);

/* Fused per-layer attention of one sequence over its int8 KV cache. */
typedef struct {
    int rows;                  /* query rows M (1: decode step, <= 16: prefill chunk) */
    int heads, kv_heads, head_dim, seq_len;
    int variant;               /* 0 NORM (llm/ref_model.py:233-243), 1 QSUM (hf_generic.py:264-292) */
    const int32_t* pos;        /* [rows] positions, device */
    const float* qkv;          /* [rows, (heads + 2 kv_heads) head_dim]: q | k | v */
    const float* q_norm;       /* [head_dim] QK-norm gains, or NULL (no QK-norm) */
    const float* k_norm;
    float eps;
    const float* rope_cos;     /* [seq_len, head_dim], pair-repeated */
    const float* rope_sin;
    float inv_sk, inv_sv;      /* F(1/s_k), F(1/s_v) */
    float a_k, a_v;            /* F(s_k/sqrt(head_dim)), F(s_v/127) */
    int8_t* k_cache;           /* [kv_heads, seq_len, head_dim] this layer's K, written at pos */
    int8_t* v_cache;           /* [kv_heads, head_dim, seq_len] this layer's V, transposed
                                  (seq_len a multiple of 16), written at pos */
    float* att;                /* [rows, heads head_dim] out */
    void* scratch;             /* unused (w8a8_attn_scratch_bytes() is 0); kept for the ABI layout */
    size_t scratch_bytes;
    uint32_t* att_amax;        /* [rows] or NULL: max|att| per row posted by atomic max (decode chain:
                                  the o-projection's w8a8_linear_chain reads it; zero before the call) */
    /* Per cache channel scales ([kv_heads * head_dim] fp32 each, or NULL for
     * the per-layer inv_sk / inv_sv / a_v), as hf_generic.SaCache
     * (compiler/frontend/hf_generic.py:153-187) computes them on the host from
     * calibrate_kv(channel=...) scales: K per channel -- k_scale = s_k (q * s_k
     * per head channel before q's quantization), inv_sk_ch = F(1) / s_k, and
     * a_k above = F(1 / sqrt(head_dim)); V per channel -- inv_sv_ch = F(1) /
     * s_v, a_v_ch = s_v * F(1/127). K and V are independent. */
    const float* k_scale;
    const float* inv_sk_ch;
    const float* inv_sv_ch;
    const float* a_v_ch;
} W8A8AttnArgs;

/* QK-norm, RoPE, the K/V rows appended at pos, per-head quant_act of q,
 * int32 scores, the softmax (global max first, no online rescaling), int8 p,
 * int32 p.V, dequantized head outputs. Row m attends positions <= pos[m]; all
 * rows' K/V are written before any row's attention. Replaces
 * ModelCompiler.rope + kv_append + attention (llm/compile_model.py:203-293),
 * DeviceModel.forward :225-243, hf_generic.sa_attention + SaCache.update
 * (:190-293) and the attention regions AttnLayerPlan / AttnChunkPlan
 * (SahlKernels.h:155-177). */
size_t w8a8_attn_scratch_bytes(int rows, int heads, int kv_heads, int head_dim, int seq_len);
int w8a8_attn(const W8A8AttnArgs* args, void* stream);

/* A prefill chunk of any number of rows of one sequence (rows at their own
 * positions, e.g. 256): w8a8_kv_append writes every row's K and V (QK-norm,
 * RoPE, int8, as w8a8_attn does) into the cache; then w8a8_attn_prefill runs
 * the attention of all rows in one launch, in groups of 16 (each row attends
 * t <= its position, all of them written). The same results as w8a8_attn over
 * consecutive 16-row chunks (hf_generic._attention_rows :306-363, each chunk's
 * K/V written before its attention), bit for bit. */
int w8a8_kv_append(const W8A8AttnArgs* args, void* stream);
int w8a8_attn_prefill(const W8A8AttnArgs* args, void* stream);
/* One launch: a thread-block cluster of up to 8 CTAs per KV head, each CTA
 * holding a chunk of up to 512 cache positions in shared memory; the chunks
 * meet at the hardware cluster barrier and exchange maxima and int32 partial
 * sums through distributed shared memory. w8a8_attn returns W8A8_EINVAL when
 * seq_len needs more than 8 x 512 positions or the chunk does not fit in
 * shared memory. */

/* The same attention for `slots` sequences of one row each (batched decode):
 * slot b uses pos[b], qkv row b and att row b, and the caches at
 * k_cache + b * slot_stride and v_cache + b * slot_stride bytes (args->rows
 * must be 1; slot_stride a multiple of head_dim and of seq_len). One CTA per
 * (KV head, slot) streams the slot's cache through TMA tiles. Each slot's row
 * is computed exactly as a one-row w8a8_attn call.
 * Replaces the attention of the batched list (llm/compile_batch.py via
 * BatchLlamaDevice.step, llm/runtime.py:193-208). */
int w8a8_attn_batch(const W8A8AttnArgs* args, int slots, size_t slot_stride, void* stream);

/* Greedy token per row (np.argmax: the first maximum). Replaces
 * Sampler.__call__ at temperature 0 (llm/runtime.py:55-57). */
int w8a8_argmax(const float* logits, int rows, int n, int32_t* out, void* stream);

/* Final RMSNorm -> quant_act -> classifier GEMV with the greedy argmax fused
 * into the epilogue: logits [rows, n] fp32; argmax_key [rows] (zero before the
 * call) receives the packed maximum (value, lowest index), which
 * w8a8_decode_advance turns into the next token. Replaces ModelCompiler.final
 * (llm/compile_model.py:347-349) and Sampler at temperature 0
 * (llm/runtime.py:55-57). */
int w8a8_classifier(const float* x, const float* norm_g, float eps, int rows, int k, const int8_t* w,
                    const float* s_w, int n, float* logits, uint64_t* argmax_key, void* stream);

/* One step of the on-device greedy decode loop, for m < rows (<= 32):
 * tokens[m] = the index in argmax_key[m], next_token[m] = the same (if not NULL),
 * argmax_key[m] = 0, pos[m] += 1; so that a captured decode step replays back to
 * back without the host. Replaces the host loop of LlamaDevice.generate
 * (llm/runtime.py:127-148) feeding greedy tokens back. */
int w8a8_decode_advance(int32_t* tokens, int32_t* pos, uint64_t* argmax_key, int32_t* next_token, int rows,
                        void* stream);

/* ------------------------------------------------------------------------
 * Tensor parallelism over the GPUs of one node (one process per GPU). The
 * reference runs on one device; these entry points have no counterpart there.
 * Its layer program is split as: q|k|v rows, gate and up rows and the
 * classifier's vocabulary rows by rank (column split), o and down by their
 * input columns (row split). The split stays exact: a row-split linear's int32
 * partials are summed exactly across ranks, and quant_act's max|x| of a
 * column-split activation is the maximum over ranks.
 *
 * Decode rows (at most W8A8_TP_ROWS) exchange over NVLink inside the kernels:
 * each rank owns an exchange region (w8a8_tp_alloc) mapped into every other
 * rank's process (w8a8_ipc_handle / w8a8_ipc_open). Values travel as 8-byte
 * words, the step epoch in the high half and the value in the low half; a
 * receiving kernel polls its own region until the words of this step arrived
 * (bounded: after ~0.2 s it gives up, reads zeros and sets error bit 5). The
 * region's first 4 bytes hold this rank's step epoch, advanced by
 * w8a8_tp_embed; exchange blocks start at W8A8_TP_HEADER bytes, 16-byte
 * aligned, and every rank lays them out identically. Every rank must run the
 * same sequence of calls, and each step must end with a dependency between
 * ranks (the greedy key exchange of w8a8_tp_advance, or a collective of the
 * caller's) before the next step's calls. Ranks must be on distinct GPUs. */
#define W8A8_TP_MAX_RANKS 8
#define W8A8_TP_ROWS 4
#define W8A8_TP_CTAS 512
#define W8A8_TP_HEADER 256
/* Exchange block sizes in 8-byte words for `ranks` ranks: the partials of a
 * row-split linear with n outputs; per-CTA row maxima; per-CTA greedy keys. */
#define W8A8_TP_PART_WORDS(ranks, n) ((size_t)(ranks) * W8A8_TP_ROWS * (size_t)(n))
#define W8A8_TP_AMAX_WORDS(ranks) ((size_t)(ranks) * (1 + W8A8_TP_CTAS) * W8A8_TP_ROWS)
#define W8A8_TP_KEY_WORDS(ranks) (2 * W8A8_TP_AMAX_WORDS(ranks))
/* ... and the expert-parallel MoE terms of decode rows: [ROWS][top_k][dim]
 * terms, then [ranks][ROWS] presence words. */
#define W8A8_TP_MOE_WORDS(ranks, top_k, dim) \
    ((size_t)W8A8_TP_ROWS * (top_k) * (size_t)(dim) + (size_t)(ranks) * W8A8_TP_ROWS)

typedef struct {
    int rank, ranks;                          /* 2 <= ranks <= W8A8_TP_MAX_RANKS */
    size_t bytes;                             /* region size (the same on every rank) */
    void* base[W8A8_TP_MAX_RANKS];            /* every rank's region as mapped in this process */
} W8A8TpComm;

/* The region: device memory of `bytes` (zeroed); its IPC handle (64 bytes);
 * another rank's region opened in this process (peer access over NVLink). */
int w8a8_tp_alloc(size_t bytes, void** region);
int w8a8_tp_free(void* region);
int w8a8_ipc_handle(const void* region, uint8_t handle[64]);
int w8a8_ipc_open(const uint8_t handle[64], void** region);
int w8a8_ipc_close(void* region);

/* w8a8_embed, and the step epoch advanced (the first call of a step). */
int w8a8_tp_embed(const W8A8TpComm* comm, const int32_t* tokens, int rows, const int8_t* emb_q, const float* emb_s,
                  int vocab, int dim, float* x, void* stream);

#define W8A8_TP_STORE 0   /* y = dequant (the classifier: + greedy keys to every rank) */
#define W8A8_TP_PARTIAL 1 /* the int32 accumulators to every rank (row-split o / down) */
#define W8A8_TP_SWIGLU 2  /* y = h of this rank's hidden rows; max|h| to every rank */

/* One decode GEMV of a rank's shard (rows <= W8A8_TP_ROWS). Prologue: when
 * part_in is set, x = resid + (f32(sum over ranks of part_in) * part_s_w) *
 * part_s_x, stored to x_out (the preceding row-split linear, finished here);
 * else x is read. Then [rmsnorm ->] quant_act, whose max|x| is amax_in's
 * maximum over every rank when set (a column-split activation). Blocks are
 * addresses in this rank's region. */
typedef struct {
    const W8A8TpComm* comm;
    int rows, k, n;
    const float* x;              /* [rows, k] (without part_in) */
    const uint64_t* part_in;     /* partials block of the preceding row-split linear, or NULL */
    const float* part_s_w;       /* [k] its weight scales */
    const float* part_s_x;       /* [rows] its activation scales (its s_x_out) */
    const float* resid;          /* [rows, k] the residual stream before it */
    float* x_out;                /* [rows, k] after it (may not alias resid) */
    const float* norm_g;         /* [k] RMSNorm gain, or NULL */
    float eps;
    const uint64_t* amax_in;     /* per-CTA max|x| block (quant_act without norm), or NULL */
    const int8_t* w;             /* [n, k] this rank's rows */
    const float* s_w;            /* [n] */
    const int8_t* w_up;          /* [n, k] SwiGLU up rows */
    const float* s_up;
    int epilogue;                /* W8A8_TP_STORE / _PARTIAL / _SWIGLU */
    float* y;                    /* STORE, SWIGLU: [rows, n] */
    uint64_t* part_out;          /* PARTIAL: partials block (n outputs) */
    uint64_t* amax_out;          /* SWIGLU: per-CTA max|h| block */
    uint64_t* key_out;           /* STORE: per-CTA key block, or NULL */
    int n_offset;                /* global index of output 0 (this rank's vocabulary slice) */
    float* s_x_out;              /* [rows] the prologue's scales, or NULL */
    int act;                     /* SWIGLU: W8A8_ACT_SILU or W8A8_ACT_GELU_TANH */
} W8A8TpLinearArgs;
int w8a8_tp_linear(const W8A8TpLinearArgs* a, void* stream);

/* w8a8_attn over this rank's heads (args: heads / kv_heads of the shard),
 * posting max|att| per row to every rank's amax_out block. */
int w8a8_tp_attn(const W8A8AttnArgs* a, const W8A8TpComm* comm, uint64_t* amax_out, void* stream);

/* w8a8_decode_advance over the key block: the greedy token of the last step
 * (the maximum key over every rank's classifier CTAs). */
int w8a8_tp_advance(const W8A8TpComm* comm, const uint64_t* keys, int32_t* tokens, int32_t* pos,
                    int32_t* next_token, int rows, void* stream);
/* Seed the key block (this rank's own) so that the next w8a8_tp_advance reads
 * `token`. */
int w8a8_tp_seed(const W8A8TpComm* comm, uint64_t* keys, int32_t token, void* stream);

/* Expert parallelism over the exchange (decode rows <= W8A8_TP_ROWS): as
 * w8a8_moe_ffn_ep, but each term w_j * y_j goes from its expert's rank into
 * every rank's `terms` block (W8A8_TP_MOE_WORDS words), with a presence word
 * per rank and row; w8a8_tp_moe_combine waits for the row's presence words
 * and the k terms of each output and folds them: y = resid + (((0 + t_0) +
 * t_1) + ...). No collective of the caller's is needed; the step is
 * capturable in a CUDA graph. */
int w8a8_tp_moe_ffn(const W8A8TpComm* comm, const float* x, const float* norm_g, float eps, int rows, int dim,
                    const int8_t* router_q, const float* router_s, int experts, int top_k, int expert_lo,
                    int experts_local, const int8_t* gate_q, const float* gate_s, const int8_t* up_q,
                    const float* up_s, int expert_hidden, const int8_t* down_q, const float* down_s, uint64_t* terms,
                    int32_t* ids, float* w, void* scratch, size_t scratch_bytes, void* stream);
int w8a8_tp_moe_combine(const W8A8TpComm* comm, const uint64_t* terms, int rows, int top_k, int dim,
                        const float* resid, float* y, void* stream);

/* Tensor-parallel rows beyond decode, with the caller's collectives between:
 * max|x| per row as float bits (all-reduce MAX as int32 across ranks), then
 * quant_act with that maximum; the linear epilogue on all-reduced int32
 * accumulators: y = [resid +] (f32(acc) * s_w) * s_x. */
int w8a8_row_amax(const float* x, int rows, int k, uint32_t* amax_bits, void* stream);
int w8a8_quant_rows_posted(const float* x, const uint32_t* amax_bits, int rows, int k, int8_t* xq, float* s_x,
                           void* stream);
int w8a8_dequant_resid(const int32_t* acc, const float* s_x, const float* s_w, int rows, int n, const float* resid,
                       float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* W8A8_B200_H */
