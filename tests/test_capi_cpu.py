"""The C-ABI library on the CPU: it loads, exports every entry point that
include/w8a8.h declares, and rejects bad arguments before launching anything
(no GPU needed: validation runs before any CUDA call)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from torch2riscv_accelerator_b200 import _lib


def header_functions():
    text = open(os.path.join(ROOT, "include", "w8a8.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w8a8_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.PROTOTYPES, f"{n} has no ctypes prototype"


def test_abi_version_and_status_strings(lib):
    assert lib.w8a8_abi_version() == _lib.ABI_VERSION
    for s in range(5):
        assert lib.w8a8_status_string(s)


def test_argument_checks_return_status_without_launch(lib):
    assert lib.w8a8_linear(None, None, 1, 64, None, None, 64, None, None, None, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_linear(8, 8, 1, 64, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EALIGN     # misaligned w
    assert lib.w8a8_linear(16, 16, 1, 60, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EALIGN   # k % 16
    assert lib.w8a8_linear(16, 16, 17, 64, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EINVAL  # rows > 16
    assert lib.w8a8_linear(16, 16, 1, 64, 16, 16, 64, 16, 16, 16, None) == _lib.W8A8_EINVAL       # resid + acc
    assert lib.w8a8_linear_fused(16, 16, 0.0, 16, 16384, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_sfu(7, 16, 16, 10, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_sfu(0, None, None, 0, None) == _lib.W8A8_OK                                 # empty: no-op
    assert lib.w8a8_ffn_swiglu(16, 16, 0.0, 1, 64, 16, 16, 16, 16, 64, 16, 16, 16, 16, 0, None) == \
        _lib.W8A8_ESCRATCH
    assert lib.w8a8_argmax(None, 1, 1, None, None) == _lib.W8A8_EINVAL


def _attn_args(**kw):
    base = dict(rows=1, heads=4, kv_heads=2, head_dim=32, seq_len=64, variant=0, pos=16, qkv=16, q_norm=None,
                k_norm=None, eps=1e-5, rope_cos=16, rope_sin=16, inv_sk=1.0, inv_sv=1.0, a_k=1.0, a_v=1.0,
                k_cache=16, v_cache=16, att=16, scratch=16,
                scratch_bytes=_lib.load().w8a8_attn_scratch_bytes(1, 4, 2, 32, 64))
    base.update(kw)
    return _lib.W8A8AttnArgs(**base)


@pytest.mark.parametrize("kw,status", [
    (dict(rows=0), _lib.W8A8_EINVAL), (dict(rows=17), _lib.W8A8_EINVAL), (dict(heads=5), _lib.W8A8_EINVAL),
    (dict(heads=32, kv_heads=2), _lib.W8A8_EINVAL), (dict(variant=2), _lib.W8A8_EINVAL),
    (dict(head_dim=24), _lib.W8A8_EALIGN), (dict(k_cache=8), _lib.W8A8_EALIGN),
    (dict(q_norm=16), _lib.W8A8_EINVAL), (dict(seq_len=8192 + 128), _lib.W8A8_EINVAL),
    (dict(qkv=None), _lib.W8A8_EINVAL)])
def test_attn_argument_checks(lib, kw, status):
    a = _attn_args(**kw)
    assert lib.w8a8_attn(ctypes.byref(a), None) == status


def test_scratch_sizes(lib):
    """The cluster attention keeps everything in (distributed) shared memory;
    the SwiGLU dispatch needs a counter and a row-amax word per row."""
    assert lib.w8a8_attn_scratch_bytes(16, 16, 8, 128, 2048) == 0
    assert lib.w8a8_ffn_scratch_bytes(16) >= 256 + 64


def _moe(lib, rows=1, dim=64, experts=4, top_k=2, ih=128, scratch_bytes=None, x=16, norm_g=None):
    sb = lib.w8a8_moe_scratch_bytes(rows, dim, top_k, ih) if scratch_bytes is None else scratch_bytes
    return lib.w8a8_moe_ffn(x, norm_g, ctypes.c_float(1e-6), rows, dim, 16, 16, experts, top_k, 16, 16, 16, 16, ih,
                            16, 16, 16, 16, 16, 16, 16, sb, None)


def test_moe_argument_checks(lib):
    """Checked before anything is queued: row and expert limits, the 16-byte
    grid of dim / expert_hidden / pointers, and the scratch size."""
    assert _moe(lib, rows=17) == _lib.W8A8_EINVAL
    assert _moe(lib, experts=65) == _lib.W8A8_EINVAL
    assert _moe(lib, top_k=5, experts=4) == _lib.W8A8_EINVAL
    assert _moe(lib, top_k=17, experts=32) == _lib.W8A8_EINVAL
    assert _moe(lib, dim=72) == _lib.W8A8_EALIGN
    assert _moe(lib, ih=120) == _lib.W8A8_EALIGN
    assert _moe(lib, x=8) == _lib.W8A8_EALIGN
    assert _moe(lib, scratch_bytes=64) == _lib.W8A8_ESCRATCH
    assert _moe(lib, x=None) == _lib.W8A8_EINVAL
    # scratch: int8 row + scale + h of every slot + amax words, each 256-byte aligned
    assert lib.w8a8_moe_scratch_bytes(1, 1024, 8, 512) == 1024 + 256 + 8 * 512 * 4 + 256


def test_moe_rows_argument_checks(lib):
    """The grouped MoE entry: up to W8A8_MOE_MAX_ROWS rows, the one-GPU form
    (no wy) with all experts only, its own scratch size."""
    def call(rows=64, lo=0, local=4, wy=None, sb=None, x=16):
        sb = lib.w8a8_moe_rows_scratch_bytes(rows, 64, 4, 2, 128) if sb is None else sb
        return lib.w8a8_moe_ffn_rows(x, None, ctypes.c_float(1e-6), rows, 64, 16, 16, 4, 2, lo, local, 16, 16, 16,
                                     16, 128, 16, 16, 16, 16, wy, 16, 16, 16, sb, None)
    assert call(rows=4097) == _lib.W8A8_EINVAL
    assert call(lo=2, local=2) == _lib.W8A8_EINVAL                # one-GPU form: every expert
    assert call(lo=3, local=2, wy=16) == _lib.W8A8_EINVAL         # past the router's experts
    assert call(sb=lib.w8a8_moe_scratch_bytes(64, 64, 2, 128)) == _lib.W8A8_ESCRATCH
    assert call(x=8) == _lib.W8A8_EALIGN
    assert call(x=None) == _lib.W8A8_EINVAL
    # + the terms [rows, top_k, dim]; above 128 rows (the tensor-core path)
    # per expert a slab of int8 x and of int8 h (rows rounded up to 128), its
    # row count and pair list, and per pair its slab row and h scale (each
    # 256-byte aligned)
    assert (lib.w8a8_moe_rows_scratch_bytes(64, 64, 4, 2, 128) ==
            lib.w8a8_moe_scratch_bytes(64, 64, 2, 128) + 64 * 2 * 64 * 4)
    assert (lib.w8a8_moe_rows_scratch_bytes(200, 64, 4, 2, 128) ==
            lib.w8a8_moe_scratch_bytes(200, 64, 2, 128) + 200 * 2 * 64 * 4 + 4 * 256 * 64 + 4 * 256 * 128 + 256
            + 4 * 256 * 4 + 2 * 1792)


def test_gemm_and_batch_argument_checks(lib):
    """The tensor-core GEMM, the row quantizer and the batched attention check
    their arguments before anything is queued."""
    assert lib.w8a8_gemm(None, 16, 1, 64, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_gemm(16, 16, 1, 72, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EALIGN    # k % 16
    assert lib.w8a8_gemm(8, 16, 1, 64, 16, 16, 64, None, 16, None, None) == _lib.W8A8_EALIGN     # xq alignment
    assert lib.w8a8_gemm(16, 16, 1, 64, 16, 16, 64, 16, 16, 16, None) == _lib.W8A8_EINVAL       # resid + acc
    assert lib.w8a8_gemm_swiglu(16, 16, 1, 64, 16, 16, None, 16, 64, 16, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_quant_rows(16, None, ctypes.c_float(0.0), 0, 64, 16, 16, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_quant_rows(16, None, ctypes.c_float(0.0), 1, 40, 16, 16, None) == _lib.W8A8_EALIGN
    a = _attn_args(rows=2)
    assert lib.w8a8_attn_batch(ctypes.byref(a), 4, 1 << 20, None) == _lib.W8A8_EINVAL            # one row per slot
    a = _attn_args()
    assert lib.w8a8_attn_batch(ctypes.byref(a), 0, 1 << 20, None) == _lib.W8A8_EINVAL
    assert lib.w8a8_attn_batch(ctypes.byref(a), 4, 1000, None) == _lib.W8A8_EALIGN               # stride % 16
    assert lib.w8a8_attn_batch(ctypes.byref(a), 4, 1024, None) == _lib.W8A8_EINVAL               # < one cache
