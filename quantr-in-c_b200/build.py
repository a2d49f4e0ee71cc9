"""Builds libquantr_cuda.so in-tree for sm_100a (B200).

    python quantr-in-c_b200/build.py [--force]

The library lands in quantr-in-c_b200/lib/ so it travels with the source tree
(no JIT cache).  Floating-point flags matter for parity: no fast-math, IEEE
division and square root, denormals preserved; the kernels additionally use
explicitly rounded intrinsics wherever the reference's operation order must be
reproduced.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libquantr_cuda.so")
SOURCES = ["gemv.cu", "engine.cu", "tc.cu", "moe.cu", "api.cu", "noalloc.cu", "decode.cu", "decode_persist.cu"]
HEADERS = ["formats.cuh", "kernels.cuh", "device_common.cuh", "quant_decode.cuh", "launch_util.cuh",
           "libm_ref.cuh", "engine_act.cuh", "decode_persist.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-v",
]


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    """Compiles the CUDA sources into LIB; returns its path."""
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [
        os.path.join(ROOT, "include", "quantr_cuda.h"), os.path.abspath(__file__)]
    if not force and not _stale(LIB, deps):
        return LIB
    objs = []
    for s in srcs:
        o = os.path.join(LIBDIR, os.path.basename(s) + ".o")
        cmd = [_nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-c", s, "-o", o]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        objs.append(o)
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB, *objs,
           "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
