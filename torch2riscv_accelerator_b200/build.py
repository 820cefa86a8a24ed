"""Build the C-ABI library libw8a8_b200.so in-tree with nvcc for sm_100a.

    python -m torch2riscv_accelerator_b200.build [--force] [--trace]

--trace builds libw8a8_b200_trace.so with the device timeline marks
(-DW8A8_TRACE, csrc/trace.cuh); the library the package loads is the plain one.

-fmad=false: no multiply-add contraction anywhere (the overlay rounds every
fp32 step once); -ftz=false, -prec-div / -prec-sqrt=true: IEEE behaviour.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libw8a8_b200.so")
TRACE_LIB = os.path.join(HERE, "libw8a8_b200_trace.so")
SOURCES = ["capi.cu", "linear.cu", "gemv.cu", "attn.cu", "misc.cu", "moe.cu", "gemm.cu"]
HEADERS = ["w8a8_math.cuh", "w8a8_internal.h", "sfu_tables.h", "pdl.cuh", "tp.cuh", "linear_common.cuh", "trace.cuh", "tc.cuh",
           os.path.join("..", "..", "include", "w8a8.h")]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
              "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def stale(lib=LIB):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [__file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, trace=False):
    """Compile every source to an object in parallel (one nvcc each), then link
    the shared library."""
    lib = TRACE_LIB if trace else LIB
    if not force and not stale(lib):
        return lib
    from concurrent.futures import ThreadPoolExecutor
    odir = os.path.join(HERE, "_build", "trace" if trace else "plain")
    os.makedirs(odir, exist_ok=True)
    flags = [f for f in NVCC_FLAGS if f != "-shared"] + (["-DW8A8_TRACE"] if trace else [])

    def one(f):
        obj = os.path.join(odir, f.replace(".cu", ".o"))
        cmd = [nvcc()] + flags + ["-c", "-o", obj, os.path.join(CSRC, f)]
        if verbose:
            print(" ".join(cmd))
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(len(SOURCES)) as ex:
        results = list(ex.map(one, SOURCES))
    for obj, r in results:
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {obj} ({r.returncode}):\n{r.stderr[-4000:]}")
    tmp = lib + ".tmp"
    r = subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp] +
                       [o for o, _ in results], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({r.returncode}):\n{r.stderr[-4000:]}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv))
