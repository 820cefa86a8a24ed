"""ctypes binding of libw8a8_b200.so (the C ABI of include/w8a8.h).

There is no fallback: if the library is missing or cannot be loaded, load()
raises. The prototypes below are the header's, one per entry point.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# W8A8_B200_LIB selects another build of the same ABI (the trace build,
# libw8a8_b200_trace.so); the default is the in-tree library
LIB_PATH = os.environ.get("W8A8_B200_LIB") or os.path.join(HERE, "libw8a8_b200.so")

W8A8_OK, W8A8_EINVAL, W8A8_EALIGN, W8A8_ECUDA, W8A8_ESCRATCH = 0, 1, 2, 3, 4
ABI_VERSION = 6
ACT_SILU, ACT_GELU_TANH = 0, 1
TP_MAX_RANKS, TP_ROWS, TP_CTAS, TP_HEADER = 8, 4, 512, 256
TP_STORE, TP_PARTIAL, TP_SWIGLU = 0, 1, 2


class W8A8AttnArgs(C.Structure):
    _fields_ = [("rows", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("seq_len", C.c_int), ("variant", C.c_int), ("pos", C.c_void_p), ("qkv", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("eps", C.c_float), ("rope_cos", C.c_void_p),
                ("rope_sin", C.c_void_p), ("inv_sk", C.c_float), ("inv_sv", C.c_float), ("a_k", C.c_float),
                ("a_v", C.c_float), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p), ("att", C.c_void_p),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("att_amax", C.c_void_p),
                ("k_scale", C.c_void_p), ("inv_sk_ch", C.c_void_p), ("inv_sv_ch", C.c_void_p),
                ("a_v_ch", C.c_void_p)]


class W8A8TpComm(C.Structure):
    _fields_ = [("rank", C.c_int), ("ranks", C.c_int), ("bytes", C.c_size_t),
                ("base", C.c_void_p * TP_MAX_RANKS)]


class W8A8TpLinearArgs(C.Structure):
    _fields_ = [("comm", C.POINTER(W8A8TpComm)), ("rows", C.c_int), ("k", C.c_int), ("n", C.c_int),
                ("x", C.c_void_p), ("part_in", C.c_void_p), ("part_s_w", C.c_void_p), ("part_s_x", C.c_void_p),
                ("resid", C.c_void_p), ("x_out", C.c_void_p), ("norm_g", C.c_void_p), ("eps", C.c_float),
                ("amax_in", C.c_void_p), ("w", C.c_void_p), ("s_w", C.c_void_p), ("w_up", C.c_void_p),
                ("s_up", C.c_void_p), ("epilogue", C.c_int), ("y", C.c_void_p), ("part_out", C.c_void_p),
                ("amax_out", C.c_void_p), ("key_out", C.c_void_p), ("n_offset", C.c_int), ("s_x_out", C.c_void_p),
                ("act", C.c_int)]


def tp_part_words(ranks, n):
    return ranks * TP_ROWS * n


def tp_amax_words(ranks):
    return ranks * (1 + TP_CTAS) * TP_ROWS


def tp_key_words(ranks):
    return 2 * tp_amax_words(ranks)


def tp_moe_words(ranks, top_k, dim):
    return TP_ROWS * top_k * dim + ranks * TP_ROWS


P, I, F, Z, L = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_int64
PROTOTYPES = {
    "w8a8_abi_version": (I, []),
    "w8a8_status_string": (C.c_char_p, [I]),
    "w8a8_sfu": (I, [I, P, P, L, P]),
    "w8a8_quant_act": (I, [P, I, I, P, P, P]),
    "w8a8_rmsnorm": (I, [P, P, I, I, F, P, P]),
    "w8a8_embed": (I, [P, I, P, P, I, I, P, P]),
    "w8a8_error_flags": (I, [C.POINTER(C.c_uint32)]),
    "w8a8_set_pdl": (I, [I]),
    "w8a8_trace_bind": (I, [P, P, C.c_uint32]),
    "w8a8_linear": (I, [P, P, I, I, P, P, I, P, P, P, P]),
    "w8a8_linear_fused": (I, [P, P, F, I, I, P, P, I, P, P, P, P]),
    "w8a8_linear_chain": (I, [P, P, F, P, I, I, P, P, I, P, P, P, I, P]),
    "w8a8_ffn_swiglu_chain": (I, [P, P, F, I, I, P, P, P, P, I, P, P, P, I, P]),
    "w8a8_ffn_scratch_bytes": (Z, [I]),
    "w8a8_ffn_swiglu": (I, [P, P, F, I, I, P, P, P, P, I, P, P, P, P, Z, P]),
    "w8a8_ffn_swiglu_noalloc": (I, [P, P, F, I, I, P, P, P, P, I, P, P, P, P]),
    "w8a8_ffn_gated": (I, [P, P, F, I, I, P, P, P, P, I, I, P, P, P, P, Z, P]),
    "w8a8_gemm_gated": (I, [P, P, I, I, P, P, P, P, I, I, P, P]),
    "w8a8_quant_rows": (I, [P, P, F, I, I, P, P, P]),
    "w8a8_gemm": (I, [P, P, I, I, P, P, I, P, P, P, P]),
    "w8a8_gemm_swiglu": (I, [P, P, I, I, P, P, P, P, I, P, P]),
    "w8a8_moe_scratch_bytes": (Z, [I, I, I, I]),
    "w8a8_moe_ffn": (I, [P, P, F, I, I, P, P, I, I, P, P, P, P, I, P, P, P, P, P, P, P, Z, P]),
    "w8a8_moe_ffn_ep": (I, [P, P, F, I, I, P, P, I, I, I, I, P, P, P, P, I, P, P, P, P, P, P, Z, P]),
    "w8a8_moe_combine": (I, [P, I, I, I, P, P, P]),
    "w8a8_moe_rows_scratch_bytes": (Z, [I, I, I, I, I]),
    "w8a8_moe_ffn_rows": (I, [P, P, F, I, I, P, P, I, I, I, I, P, P, P, P, I, P, P, P, P, P, P, P, P, Z, P]),
    "w8a8_attn_scratch_bytes": (Z, [I, I, I, I, I]),
    "w8a8_attn": (I, [C.POINTER(W8A8AttnArgs), P]),
    "w8a8_attn_batch": (I, [C.POINTER(W8A8AttnArgs), I, Z, P]),
    "w8a8_kv_append": (I, [C.POINTER(W8A8AttnArgs), P]),
    "w8a8_attn_prefill": (I, [C.POINTER(W8A8AttnArgs), P]),
    "w8a8_argmax": (I, [P, I, I, P, P]),
    "w8a8_classifier": (I, [P, P, F, I, I, P, P, I, P, P, P]),
    "w8a8_decode_advance": (I, [P, P, P, P, I, P]),
    "w8a8_tp_alloc": (I, [Z, C.POINTER(P)]),
    "w8a8_tp_free": (I, [P]),
    "w8a8_ipc_handle": (I, [P, C.POINTER(C.c_uint8)]),
    "w8a8_ipc_open": (I, [C.POINTER(C.c_uint8), C.POINTER(P)]),
    "w8a8_ipc_close": (I, [P]),
    "w8a8_tp_embed": (I, [C.POINTER(W8A8TpComm), P, I, P, P, I, I, P, P]),
    "w8a8_tp_linear": (I, [C.POINTER(W8A8TpLinearArgs), P]),
    "w8a8_tp_attn": (I, [C.POINTER(W8A8AttnArgs), C.POINTER(W8A8TpComm), P, P]),
    "w8a8_tp_advance": (I, [C.POINTER(W8A8TpComm), P, P, P, P, I, P]),
    "w8a8_tp_seed": (I, [C.POINTER(W8A8TpComm), P, C.c_int32, P]),
    "w8a8_tp_moe_ffn": (I, [C.POINTER(W8A8TpComm), P, P, F, I, I, P, P, I, I, I, I, P, P, P, P, I, P, P, P, P, P,
                            P, Z, P]),
    "w8a8_tp_moe_combine": (I, [C.POINTER(W8A8TpComm), P, I, I, I, P, P, P]),
    "w8a8_row_amax": (I, [P, I, I, P, P]),
    "w8a8_quant_rows_posted": (I, [P, P, I, I, P, P, P]),
    "w8a8_dequant_resid": (I, [P, P, P, I, I, P, P, P]),
}

_LIB = None


class W8A8Error(RuntimeError):
    def __init__(self, fn, status, msg):
        super().__init__(f"{fn}: status {status} ({msg})")
        self.fn, self.status = fn, status


def load(path=LIB_PATH):
    """Load the library once and bind the prototypes; raises if it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m torch2riscv_accelerator_b200.build` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    if lib.w8a8_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{path}: ABI version {lib.w8a8_abi_version()}, expected {ABI_VERSION}")
    _LIB = lib
    return lib


def check(fn_name, status):
    if status != W8A8_OK:
        raise W8A8Error(fn_name, status, load().w8a8_status_string(status).decode())
