"""Build the C-ABI library libw8a8_b200.so in-tree with nvcc for sm_100a.

    python -m torch2riscv_accelerator_b200.build [--force]

-fmad=false: no multiply-add contraction anywhere (the overlay rounds every
fp32 step once); -ftz=false, -prec-div / -prec-sqrt=true: IEEE behaviour.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libw8a8_b200.so")
SOURCES = ["capi.cu", "linear.cu", "gemv.cu", "attn.cu", "misc.cu", "moe.cu", "gemm.cu"]
HEADERS = ["w8a8_math.cuh", "w8a8_internal.h", "sfu_tables.h", "pdl.cuh", "tp.cuh", "linear_common.cuh", os.path.join("..", "..", "include", "w8a8.h")]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
              "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [__file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    srcs = [os.path.join(CSRC, f) for f in SOURCES]
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + NVCC_FLAGS + ["-o", tmp] + srcs
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
